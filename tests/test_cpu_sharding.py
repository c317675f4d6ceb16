"""Host logic of the row-sharded decode on CPU: the row partition and the
all-gather assembly of per-rank list slices (gloo, world size 2)."""
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import torch_dbs_extension as ext


@pytest.mark.parametrize("rows,world", [(1, 1), (7, 2), (8, 2), (100, 3), (5, 8), (4096, 8)])
def test_row_shards_cover_every_row_once(rows, world):
    per, ranges = ext.row_shards(rows, world)
    assert len(ranges) == world
    seen = []
    for r, (b, e) in enumerate(ranges):
        assert b == min(rows, r * per) and b <= e <= b + per
        seen.extend(range(b, e))
    assert seen == list(range(rows))


def _gather_worker(rank, world, port, path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rows, C = 11, 3
        per, ranges = ext.row_shards(rows, world)
        lists = torch.full((world * per, C), -1, dtype=torch.int64)
        b, e = ranges[rank]
        for r in range(b, e):   # what this rank's scan writes: its own rows only
            lists[r] = torch.arange(C) + 100 * r
        out = [torch.empty((per, C), dtype=torch.int64) for _ in range(world)]
        dist.all_gather(out, lists[rank * per:(rank + 1) * per].clone())
        full = torch.cat(out)
        ok = all(torch.equal(full[r], torch.arange(C) + 100 * r) for r in range(rows))
        if rank == 0:
            with open(path, "w") as f:
                f.write("ok" if ok else "bad")
    finally:
        dist.destroy_process_group()


def test_list_slices_assemble_over_gloo(tmp_path):
    path = tmp_path / "r.txt"
    mp.start_processes(_gather_worker, args=(2, 29623, str(path)), nprocs=2, start_method="spawn")
    assert path.read_text() == "ok"


def _examples_worker(rank, world, port, path, counts):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        def share(r):
            n = counts[r]
            first = sum(counts[:r])
            ids = torch.arange(first, first + n)
            return {"scores": ids[:, None].float() * 0.5 + torch.arange(3).float(),
                    "tokens": (ids[:, None, None] * 100 + torch.arange(12).reshape(4, 3)).to(torch.int32),
                    "counts": ids * 7,
                    "flags": (ids % 2).to(torch.uint8)}
        got = ext.gather_examples(share(rank))
        want = {k: torch.cat([share(r)[k] for r in range(world)]) for k in share(0)}
        ok = all(torch.equal(got[k], want[k]) and got[k].dtype == want[k].dtype for k in want)
        if rank == 0:
            with open(path, "w") as f:
                f.write("ok" if ok else "bad")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("counts", [(3, 3), (4, 1), (2, 0, 5)])
def test_gather_examples_over_gloo(tmp_path, counts):
    """Per-example arrays of several dtypes and shapes come back in rank
    order on every rank, uneven shares (and an empty one) included."""
    path = tmp_path / "r.txt"
    port = 29631 + sum(counts) + len(counts)
    mp.start_processes(_examples_worker, args=(len(counts), port, str(path), counts), nprocs=len(counts),
                       start_method="spawn")
    assert path.read_text() == "ok"


class _FakeTrace:
    """Deterministic stand-in for a device decode of [B,T,K,V] log-probs on CPU."""
    def __init__(self, x):
        B, T, K, V = x.shape
        self.tokens = x.argmax(-1).to(torch.int32)
        self.parents = (self.tokens % K).to(torch.int32)
        self.final_scores = x[:, -1, :, :].max(-1).values.contiguous()


def _sharded_worker(rank, world, port, path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        T, K, V = 3, 2, 11
        counts = [3, 2][:world]

        def local(r):
            g = torch.Generator().manual_seed(100 + r)
            return torch.randn((counts[r], T, K, V), generator=g)

        def fake_backward(trace, grad_final, options, V_):
            B = trace.tokens.shape[0]
            idx = torch.arange(B * T * (K + 2 * K), dtype=torch.int64).reshape(B, -1)
            return {"counts": torch.full((B,), T * K, dtype=torch.int64), "indices": idx,
                    "values": idx.float() * grad_final.sum(), "grad_initial": grad_final * 2.0}

        ext.device_decode = lambda x, options, with_pool=False, with_weights=False: _FakeTrace(x)
        ext.device_backward_sparse = fake_backward
        opts = ext.DBSOptions(beam_size=K, relaxed_pool_multiplier=2)
        gf = torch.ones((counts[rank], K))
        got, trace = ext.decode_batch_sharded(local(rank), opts, grad_final=gf)
        ok = set(got) == {"final_scores", "tokens", "parents", "sparse_counts", "sparse_indices",
                          "sparse_values", "grad_initial"}
        for r in range(world):
            lo, hi = sum(counts[:r]), sum(counts[:r + 1])
            tr = _FakeTrace(local(r))
            bw = fake_backward(tr, torch.ones((counts[r], K)), opts, V)
            ok = ok and torch.equal(got["final_scores"][lo:hi], tr.final_scores)
            ok = ok and torch.equal(got["tokens"][lo:hi], tr.tokens) and torch.equal(got["parents"][lo:hi], tr.parents)
            ok = ok and torch.equal(got["sparse_counts"][lo:hi], bw["counts"])
            ok = ok and torch.equal(got["sparse_indices"][lo:hi], bw["indices"][:, :T * K])
            ok = ok and torch.equal(got["sparse_values"][lo:hi], bw["values"][:, :T * K])
            ok = ok and torch.equal(got["grad_initial"][lo:hi], bw["grad_initial"])
        ok = ok and got["tokens"].shape == (sum(counts), T, K) and trace.tokens.shape[0] == counts[rank]
        if rank == 0:
            with open(path, "w") as f:
                f.write("ok" if ok else "bad")
    finally:
        dist.destroy_process_group()


def test_decode_batch_sharded_assembles_every_rank_over_gloo(tmp_path):
    """The batch-sharded entry point's host logic (device calls replaced by
    deterministic CPU stand-ins): each rank's share decoded, its sparse
    gradient cut to T*K entries per example, and the whole batch's results
    on every rank in example order."""
    path = tmp_path / "r.txt"
    mp.start_processes(_sharded_worker, args=(2, 29647, str(path)), nprocs=2, start_method="spawn")
    assert path.read_text() == "ok"
