"""Row-sharded decode: the row scan split into ranges, the lists assembled,
then the merge, must equal the one-call device decode bit for bit."""
import ctypes
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

FIELDS = ("parents", "tokens", "lengths", "from_logprob", "raw_scores", "scores", "final_raw_scores",
          "final_scores", "pool_parents", "pool_tokens", "pool_scores", "relaxed_weights", "weights")


def _make_x(B, T, K, V, seed, device):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    x = torch.randn((B, T, K, V), generator=g, device=device) * 2.0
    x -= 1.1 * torch.log(torch.arange(V, device=device, dtype=torch.float32) + 1.0)
    return torch.log_softmax(x, dim=-1).contiguous()


def _assert_same_trace(a, b):
    for f in FIELDS:
        ta, tb = getattr(a, f), getattr(b, f)
        if ta is None:
            assert tb is None
            continue
        assert torch.equal(ta, tb), f


@pytest.mark.parametrize("with_pool,K,V,pieces", [(False, 8, 32000, 3), (True, 4, 5003, 2), (True, 16, 2000, 5)])
def test_split_scan_then_merge_equals_decode(with_pool, K, V, pieces):
    import torch_dbs_extension as ext
    device = torch.device("cuda", 0)
    B, T = 3, 6
    opts = ext.DBSOptions(beam_size=K, eos_token=2, length_penalty_alpha=0.2, selected_temperature=0.7)
    x = _make_x(B, T, K, V, 5, device)
    want = ext.device_decode(x, opts, with_pool=with_pool, with_weights=True)
    lib = ext._library()
    h = ext._handle(opts)
    cap = ctypes.c_int()
    assert lib.dbs_device_row_list_capacity(h, int(with_pool), ctypes.byref(cap)) == 0
    rows = B * T * K
    lists = torch.empty((rows, cap.value), dtype=torch.int64, device=device)
    counts = torch.empty((rows,), dtype=torch.int32, device=device)
    bounds = torch.empty((rows,), dtype=torch.float32, device=device)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    per, ranges = ext.row_shards(rows, pieces)
    for begin, end in reversed(ranges):   # any order, any split
        rc = lib.dbs_device_scan_rows(h, ext._vp(x), B, T, V, int(with_pool), begin, end, ext._vp(lists),
                                      ext._vp(counts), ext._vp(bounds), stream)
        assert rc == 0, lib.dbs_last_error(h)
    P = max(K, K * opts.relaxed_pool_multiplier)
    got = ext.DeviceTrace(B, T, K, device, with_pool=with_pool, P=P, with_weights=True)
    outs = got.struct()
    rc = lib.dbs_device_merge_rows(h, ext._vp(x), B, T, V, ext._vp(lists), ext._vp(counts), ext._vp(bounds),
                                   ctypes.byref(outs), stream)
    assert rc == 0, lib.dbs_last_error(h)
    torch.cuda.synchronize()
    _assert_same_trace(got, want)


def test_scan_rows_rejects_bad_ranges():
    import torch_dbs_extension as ext
    device = torch.device("cuda", 0)
    opts = ext.DBSOptions(beam_size=2)
    x = _make_x(1, 2, 2, 50, 1, device)
    lib = ext._library()
    h = ext._handle(opts)
    buf = torch.empty(64, dtype=torch.int64, device=device)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for b, e in ((-1, 2), (3, 2), (0, 5)):
        rc = lib.dbs_device_scan_rows(h, ext._vp(x), 1, 2, 50, 0, b, e, ext._vp(buf), ext._vp(buf), ext._vp(buf), stream)
        assert rc == -2 and b"row range" in lib.dbs_last_error(h)


def _sharded_worker(rank, world, port, result_path):
    import torch.distributed as dist
    import torch_dbs_extension as ext
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    device = torch.device("cuda", rank)
    from datetime import timedelta
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=device)
    try:
        opts = ext.DBSOptions(beam_size=16, length_penalty_alpha=0.3)
        B, T, K, V = 1, 24, 16, 60000
        x = _make_x(B, T, K, V, 9, device)   # every rank holds the same log-probs
        got = ext.decode_row_sharded(x, opts, with_pool=True, with_weights=True)
        want = ext.device_decode(x, opts, with_pool=True, with_weights=True)
        torch.cuda.synchronize()
        ok = all(torch.equal(getattr(got, f), getattr(want, f)) for f in FIELDS)
        if rank == 0:
            with open(result_path, "w") as f:
                f.write("ok" if ok else "mismatch")
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_row_sharded_decode_on_two_gpus(tmp_path):
    import torch.multiprocessing as mp
    result = tmp_path / "result.txt"
    mp.start_processes(_sharded_worker, args=(2, 29611, str(result)), nprocs=2, start_method="spawn")
    assert result.read_text() == "ok"
