"""Fused decodes of uniform batches, and their neighbours.

A uniform batch of 2 to 64 examples (every example with the same steps and
beams) without sequence constraints whose merge is the selection merge (more
than 256 candidates per step) is decoded by one cooperative launch: scan
warps list the rows step by step across the examples and count each listed
row per (example, step); merge CTAs run each example's steps as soon as the
step's rows are listed, so the merge follows the scan instead of waiting for
it. Row lists hold at most 64 entries and step 0's one live row is completed
by the merge (a radix-selected floor over the row). These cases check every
example against the oracle, bit-exact: step counts that do not divide, EOS
and length penalty, pools of 512 from 8 beams (and of 1024, which take the
separate launches), a rejected input (the launch
writes no output) followed by good decodes, a workspace that holds an
earlier call's lists, and the sparse backward from the fused trace; plus the
paths beside it (sequence constraints and 16-bit rows, which keep separate
launches).
"""
import ctypes

import numpy as np
import pytest
import torch

import dbs_ctypes as dc
from parity import assert_decode_equal, log_softmax_np

pytestmark = pytest.mark.gpu


def _check_host_batch(lib, orc, opts, x, backward_examples=()):
    B, T, K, V = x.shape
    dec = dc.Decoder(lib, dc.Options(**opts))
    br = dec.decode_batch(np.ascontiguousarray(x), B, T, V)
    for b in range(B):
        r = lib.dbs_batch_result_at(br, b)
        want = orc.decode(orc.options(**opts), np.ascontiguousarray(x[b]), T, V)
        assert_decode_equal(dc.read_result(lib, r), want, f"example {b}")
        if b in backward_examples:
            gf = np.random.default_rng(b).standard_normal(K).astype(np.float32)
            bw = dec.backward(r, None, None, gf)
            got = dc.read_backward(lib, bw, K=K)
            lib.dbs_free_backward(bw)
            wb = orc.backward_sparse(want, None, None, gf)
            assert np.array_equal(got["indices"], wb["indices"]), f"example {b} sparse indices"
            assert np.array_equal(got["values"], wb["values"]), f"example {b} sparse values"
    lib.dbs_free_batch_result(br)
    dec.close()


@pytest.mark.parametrize("B,T,K,V,mult,alpha,eos", [
    (4, 17, 32, 300, 8, 0.0, -1),    # 3-step segments, the last one 2 steps
    (6, 40, 16, 257, 8, 0.4, 3),     # 5-step segments, EOS carries and length penalty
    (3, 16, 8, 500, 64, 0.0, 2),     # pool 512 from 8 beams: 4096 candidates per step
    (2, 9, 16, 700, 64, 0.2, 3),     # pool 1024 from 16 beams: above the compact merge's 512
])
def test_pipelined_uniform_batch(libdbs, oracle_lib, B, T, K, V, mult, alpha, eos):
    rng = np.random.default_rng(B * 1000 + T)
    x = log_softmax_np(1.3 * rng.standard_normal((B, T, K, V)).astype(np.float32))
    opts = dict(beam_size=K, relaxed_pool_multiplier=mult, length_penalty_alpha=alpha, eos_token=eos)
    _check_host_batch(libdbs, oracle_lib, opts, x, backward_examples=(0, B - 1))


def test_pipelined_batch_rejects_nan_then_decodes(libdbs, oracle_lib):
    B, T, K, V = 3, 20, 32, 200
    rng = np.random.default_rng(11)
    x = log_softmax_np(rng.standard_normal((B, T, K, V)).astype(np.float32))
    opts = dict(beam_size=K)
    bad = x.copy()
    bad[1, 0, 0, 0] = np.inf   # index 0 of example 1 is always sampled
    dec = dc.Decoder(libdbs, dc.Options(**opts))
    with pytest.raises(dc.DBSError, match="NaN or \\+Inf"):
        dec.decode_batch(np.ascontiguousarray(bad), B, T, V)
    dec.close()
    for _ in range(2):
        _check_host_batch(libdbs, oracle_lib, opts, x)


def test_pipelined_batch_with_sequence_constraints(libdbs, oracle_lib):
    # equal steps and beams through the variable entry point: banned tokens,
    # a forced first token, a minimum length before EOS, repetition penalty
    # and no repeated 2-gram (the merge keeps the beams' prefixes across its
    # segment launches)
    import torch_dbs_extension as ext
    rng = np.random.default_rng(21)
    B, T, K, V = 4, 23, 8, 300
    steps = np.full(B, T, np.int32)
    beams = np.full(B, K, np.int32)
    eos = np.full(B, 2, np.int32)
    minl = np.full(B, 5, np.int32)
    banned = np.zeros((B, V), np.uint8)
    banned[:, rng.choice(V, 20, replace=False)] = 1
    banned[:, 2] = 0
    forced = np.full((B, T), -1, np.int32)
    forced[:, 0] = 7
    x = log_softmax_np(1.5 * rng.standard_normal((B, T, K, V)).astype(np.float32))
    opts = ext.DBSOptions(beam_size=K, eos_token=2, min_length=5, relaxed_pool_multiplier=4)
    h = ext._handle(opts)
    dev = torch.device("cuda")
    P = 4 * K
    sel, pool, fin = B * T * K, B * T * P, B * K
    mk = lambda n, dt: torch.empty(n, dtype=dt, device=dev)
    out = dict(parents=mk(sel, torch.int32), tokens=mk(sel, torch.int32), lengths=mk(sel, torch.int32),
               from_logprob=mk(sel, torch.uint8), raw_scores=mk(sel, torch.float32), scores=mk(sel, torch.float32),
               weights=mk(sel, torch.float32), pool_parents=mk(pool, torch.int32), pool_tokens=mk(pool, torch.int32),
               pool_lengths=mk(pool, torch.int32), pool_from_logprob=mk(pool, torch.uint8),
               pool_raw_scores=mk(pool, torch.float32), pool_scores=mk(pool, torch.float32),
               relaxed_weights=mk(pool, torch.float32), final_raw_scores=mk(fin, torch.float32),
               final_scores=mk(fin, torch.float32))
    s = dc.DBSDeviceDecodeOutputs()
    for name, _ in dc.DBSDeviceDecodeOutputs._fields_:
        setattr(s, name, out[name].data_ptr())
    xd = torch.tensor(x, device=dev)
    bd = torch.tensor(banned, device=dev)
    fd = torch.tensor(forced, device=dev)
    lib = ext._library()
    rc = lib.dbs_device_decode_batch_variable_ex(
        h, ext._vp(xd), B, T, K, V, steps.ctypes.data_as(ctypes.c_void_p), beams.ctypes.data_as(ctypes.c_void_p),
        eos.ctypes.data_as(ctypes.c_void_p), minl.ctypes.data_as(ctypes.c_void_p), ext._vp(bd), ext._vp(fd),
        ctypes.c_float(1.3), 2, ctypes.byref(s), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, lib.dbs_last_error(h)
    torch.cuda.synchronize()
    for b in range(B):
        o = oracle_lib.options(beam_size=K, eos_token=2, min_length=5, relaxed_pool_multiplier=4)
        want = oracle_lib.decode(o, x[b], T, V, banned=banned[b], forced=forced[b].copy(), min_length=5,
                                 repetition_penalty=1.3, no_repeat_ngram_size=2)
        got = {f: out[f].view(B, -1)[b].cpu().numpy() for f in out}
        assert_decode_equal(got, want, f"constrained example {b}")


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_pipelined_typed_batch(libdbs, oracle_lib, dtype):
    rng = np.random.default_rng(31)
    B, T, K, V = 3, 18, 16, 260
    x = log_softmax_np(rng.standard_normal((B, T, K, V)).astype(np.float32))
    if dtype == "f16":
        h16 = x.astype(np.float16)
        bits, wide, code = h16.view(np.uint16), h16.astype(np.float32), dc.DBS_DTYPE_F16
    else:
        bits = (x.view(np.uint32) >> 16).astype(np.uint16)
        wide = (bits.astype(np.uint32) << 16).view(np.float32)
        code = dc.DBS_DTYPE_BF16
    opts = dict(beam_size=K)
    dec = dc.Decoder(libdbs, dc.Options(**opts))
    br = ctypes.c_void_p()
    rc = libdbs.dbs_decode_batch_typed(dec.h, np.ascontiguousarray(bits).ctypes.data_as(ctypes.c_void_p), code, B, T,
                                       V, 0, ctypes.byref(br))
    assert rc == 0, libdbs.dbs_last_error(dec.h)
    for b in range(B):
        want = oracle_lib.decode(oracle_lib.options(**opts), np.ascontiguousarray(wide[b]), T, V)
        assert_decode_equal(dc.read_result(libdbs, libdbs.dbs_batch_result_at(br, b)), want, f"{dtype} example {b}")
    libdbs.dbs_free_batch_result(br)
    dec.close()


def test_pipelined_batch_after_other_inputs(oracle_lib):
    # The workspace keeps the row lists of earlier calls. A scan segment that
    # starts while the previous one still holds the SMs must still list every
    # one of its rows (else the merge would read an earlier call's lists):
    # 32 examples of 2048 rows per step segment, after two decodes of other
    # log-probs of the same shape, every example against the oracle.
    import torch_dbs_extension as ext
    B, T, K, V = 32, 64, 32, 2000
    dev = torch.device("cuda")
    gen = torch.Generator(device=dev).manual_seed(77)
    opts = ext.DBSOptions(beam_size=K)
    noise = torch.log_softmax(3.0 * torch.randn((B, T, K, V), device=dev, generator=gen), dim=-1)
    for _ in range(2):
        ext.device_decode(noise, opts, with_pool=True, with_weights=True)
    del noise
    x = torch.log_softmax(torch.randn((B, T, K, V), device=dev, generator=gen), dim=-1)
    tr = ext.device_decode(x, opts, with_pool=True, with_weights=True)
    torch.cuda.synchronize()
    xh = x.cpu().numpy()
    fields = ("parents", "tokens", "lengths", "raw_scores", "scores", "weights", "pool_parents", "pool_tokens",
              "pool_lengths", "pool_raw_scores", "pool_scores", "relaxed_weights", "final_scores", "final_raw_scores")
    host = {f: getattr(tr, f).cpu().numpy().reshape(B, -1) for f in fields}
    for b in range(B):
        want = oracle_lib.decode(oracle_lib.options(beam_size=K), xh[b], T, V)
        assert_decode_equal({f: host[f][b] for f in fields}, want, f"example {b}")
