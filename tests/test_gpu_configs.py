"""The benchmark configurations' shapes on the device against the oracle.

Each case keeps the configuration's vocabulary, beam and pool sizes and
option set, with fewer examples / steps so the scalar oracle finishes in
seconds; inputs follow the configurations' recipes (seeded, generated on the
device). Checked bit-exact: parents, tokens, lengths, pool tokens, final
scores and the sparse backward of grad_final = e_0.
"""
import ctypes

import numpy as np
import pytest
import torch

import dbs_ctypes as dc

pytestmark = pytest.mark.gpu


def _gen(B, T, K, V, seed, sigma=1.0, spike=False):
    dev = torch.device("cuda", 0)
    x = torch.empty((B, T, K, V), dtype=torch.float32, device=dev)
    g = torch.Generator(device=dev)
    for b in range(B):
        g.manual_seed(seed * 1_000_003 + b)
        x[b].normal_(generator=g)
        x[b].mul_(sigma)
        if spike:   # per step 64 seeded ids get +8 in every row of the step
            for t in range(T):
                ids = torch.randint(0, V, (64,), generator=g, device=dev)
                x[b, t, :, ids] += 8.0
        x[b] = torch.log_softmax(x[b], dim=-1)
    return x


def _decode_and_backward(opts, x):
    import torch_dbs_extension as ext
    B, T, K, V = x.shape
    P = max(K, K * opts.relaxed_pool_multiplier)
    tr = ext.device_decode(x, opts, with_pool=True, with_weights=True)
    gf = torch.zeros((B, K), device=x.device)
    gf[:, 0] = 1.0
    cap = T * (K + P)
    si = torch.empty((B, cap), dtype=torch.int64, device=x.device)
    sv = torch.empty((B, cap), dtype=torch.float32, device=x.device)
    sc = torch.empty((B,), dtype=torch.int64, device=x.device)
    lib = ext._library()
    h = ext._handle(opts)
    s = tr.struct()
    rc = lib.dbs_device_backward_batch_ex(h, B, T, V, ctypes.byref(s), None, None, ext._vp(gf), None, ext._vp(si),
                                          ext._vp(sv), ext._vp(sc), None, 0,
                                          ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, lib.dbs_last_error(h)
    torch.cuda.synchronize()
    return tr, si, sv, sc


def _check_example(oracle_lib, opts_kw, x, b, tr, si, sv, sc):
    T, K, V = x.shape[1:]
    o = oracle_lib.options(**opts_kw)
    want = oracle_lib.decode(o, x[b].cpu().numpy(), T, V)
    for f in ("parents", "tokens", "lengths", "pool_tokens", "pool_parents"):
        assert np.array_equal(getattr(tr, f)[b].cpu().numpy().ravel(), want[f]), f
    assert np.array_equal(tr.final_scores[b].cpu().numpy(), want["final_scores"])
    gf = np.zeros(K, dtype=np.float32)
    gf[0] = 1.0
    wb = oracle_lib.backward_sparse(want, None, None, gf)
    n = int(sc[b].item())
    assert n == len(wb["indices"])
    assert np.array_equal(si[b, :n].cpu().numpy(), wb["indices"])
    assert np.array_equal(sv[b, :n].cpu().numpy(), wb["values"])


@pytest.mark.parametrize("K", [32, 64, 128])
def test_third_config_shapes(oracle_lib, K):
    # V = 50257, defaults (P = 8K), log_softmax(N(0,1)); B and T reduced
    import torch_dbs_extension as ext
    x = _gen(2, 12, K, 50257, seed=3)
    opts = ext.DBSOptions(beam_size=K)
    tr, si, sv, sc = _decode_and_backward(opts, x)
    _check_example(oracle_lib, dict(beam_size=K), x, 1, tr, si, sv, sc)


def test_fifth_config_shape(oracle_lib):
    # B = 1, K = 16, V = 256000, spiked log-probs, P = 128; T reduced
    import torch_dbs_extension as ext
    x = _gen(1, 24, 16, 256000, seed=5, spike=True)
    opts = ext.DBSOptions(beam_size=16)
    tr, si, sv, sc = _decode_and_backward(opts, x)
    _check_example(oracle_lib, dict(beam_size=16), x, 0, tr, si, sv, sc)


def test_fourth_config_shape(libdbs, oracle_lib):
    # variable batch with every constraint: V = 128256, K_b in {1,2,4,8,16},
    # 256 banned ids, forced first token, min length 8 with eos 2,
    # repetition penalty 1.2, no-repeat 3-grams; T_b reduced to 8..20
    import torch_dbs_extension as ext
    rng = np.random.default_rng(4)
    B, maxT, maxK, V = 5, 20, 16, 128256
    steps = rng.integers(8, maxT + 1, B).astype(np.int32)
    beams = np.array([1, 2, 4, 8, 16], np.int32)
    eos = np.full(B, 2, np.int32)
    minl = np.full(B, 8, np.int32)
    banned = np.zeros((B, V), np.uint8)
    banned[:, rng.choice(V, 256, replace=False)] = 1
    forced = np.full((B, maxT), -1, np.int32)
    forced[:, 0] = 1
    x = _gen(B, maxT, maxK, V, seed=4, sigma=1.5)
    opts = ext.DBSOptions(beam_size=16, eos_token=2, min_length=8)
    h = ext._handle(opts)
    dev = x.device
    sel = int((steps * beams).sum())
    pool = int((steps * beams * 8).sum())
    fin = int(beams.sum())
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
    bd = torch.tensor(banned, device=dev)
    fd = torch.tensor(forced, device=dev)
    lib = ext._library()
    rc = lib.dbs_device_decode_batch_variable_ex(
        h, ext._vp(x), B, maxT, maxK, V, steps.ctypes.data_as(ctypes.c_void_p), beams.ctypes.data_as(ctypes.c_void_p),
        eos.ctypes.data_as(ctypes.c_void_p), minl.ctypes.data_as(ctypes.c_void_p), ext._vp(bd), ext._vp(fd),
        ctypes.c_float(1.2), 3, ctypes.byref(s), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, lib.dbs_last_error(h)
    torch.cuda.synchronize()
    sel_off = np.concatenate([[0], np.cumsum(steps * beams)])
    pool_off = np.concatenate([[0], np.cumsum(steps * beams * 8)])
    fin_off = np.concatenate([[0], np.cumsum(beams)])
    for b in range(B):
        T, K = int(steps[b]), int(beams[b])
        o = oracle_lib.options(beam_size=K, eos_token=2, min_length=8)
        want = oracle_lib.decode(o, x[b, :T, :K].cpu().numpy(), T, V, banned=banned[b], forced=forced[b, :T].copy(),
                                 min_length=8, repetition_penalty=1.2, no_repeat_ngram_size=3)
        a, c = sel_off[b], sel_off[b + 1]
        for f in ("parents", "tokens", "lengths"):
            assert np.array_equal(out[f][a:c].cpu().numpy(), want[f]), (b, f)
        pa, pc = pool_off[b], pool_off[b + 1]
        assert np.array_equal(out["pool_tokens"][pa:pc].cpu().numpy(), want["pool_tokens"]), b
        assert np.array_equal(out["final_scores"][fin_off[b]:fin_off[b + 1]].cpu().numpy(), want["final_scores"]), b
