"""Relaxed-pool decodes of 32 or more examples and 64K or more rows, with
pools above 64 entries, keep row lists of 64 entries (step 0's one live row
keeps a list of up to min(P, 64*K, 1024) entries): the step merge proves, per step, that
no row holds more of the pool than its list, and rescans the rows it cannot
prove from HBM. Every path of that (run merge and selection merge, 16-bit
rows, static constraints, exact ties at the list cut, a dominant beam whose
row holds the whole pool, log-probs that round to one score) is compared
with the oracle, example by example. Vocabularies are small so that the
oracle decodes the 64K rows in seconds."""
import ctypes

import numpy as np
import pytest

import dbs_ctypes as dc
from parity import assert_decode_equal, log_softmax_np

pytestmark = pytest.mark.gpu



def _merge_rescans(lib, h):
    row = ctypes.c_int64()
    merge = ctypes.c_int64()
    assert lib.dbs_device_last_rescan_counts(h, ctypes.byref(row), ctypes.byref(merge)) == 0
    return int(merge.value)


def _check_batch(lib, orc, opts, x, T, V, label, backward_examples=(0,)):
    dec = dc.Decoder(lib, dc.Options(**opts))
    br = dec.decode_batch(np.ascontiguousarray(x), x.shape[0], T, V)
    rescans = _merge_rescans(lib, dec.h)
    K = opts["beam_size"]
    for b in range(x.shape[0]):
        r = lib.dbs_batch_result_at(br, b)
        want = orc.decode(orc.options(**opts), np.ascontiguousarray(x[b]), T, V)
        assert_decode_equal(dc.read_result(lib, r), want, f"{label} example {b}")
        if b in backward_examples:
            gf = np.zeros(K, dtype=np.float32)
            gf[0] = 1.0
            bw = dec.backward(r, None, None, gf)
            got = dc.read_backward(lib, bw, K=K)
            lib.dbs_free_backward(bw)
            wb = orc.backward_sparse(want, None, None, gf)
            assert np.array_equal(got["indices"], wb["indices"]), f"{label} example {b} sparse indices"
            assert np.array_equal(got["values"], wb["values"]), f"{label} example {b} sparse values"
    lib.dbs_free_batch_result(br)
    dec.close()
    return rescans


@pytest.mark.parametrize("B,K,T,V,alpha,eos", [
    (64, 16, 64, 400, 0.3, 2),      # pool 128: run merge of 16 x 64 candidates
    (32, 32, 64, 300, 0.0, -1),     # pool 256: selection merge of 32 x 64 candidates
    (32, 64, 32, 600, 0.0, 5),      # pool 512: selection merge of 64 x 64 candidates
])
def test_short_lists_normal_rows(libdbs, oracle_lib, B, K, T, V, alpha, eos):
    rng = np.random.default_rng(K * 31 + V)
    x = log_softmax_np(rng.standard_normal((B, T, K, V)).astype(np.float32))
    opts = dict(beam_size=K, length_penalty_alpha=alpha, eos_token=eos)
    _check_batch(libdbs, oracle_lib, opts, x, T, V, f"K={K}", backward_examples=(0, B - 1))


def test_short_lists_dominant_beam_is_rescanned(libdbs, oracle_lib):
    # one token of every step-0 row is nearly certain, so at step 1 the beam
    # that took it outscores the others by ~13 nats and its row (beam 0's)
    # holds the whole pool of 256: more than its list of 64 + 128 entries,
    # so the merge rescans it
    rng = np.random.default_rng(8)
    B, K, T, V = 64, 16, 64, 400
    z = rng.standard_normal((B, T, K, V)).astype(np.float32)
    z[:, 0, :, 5] += 16.0
    x = log_softmax_np(z)
    rescans = _check_batch(libdbs, oracle_lib, dict(beam_size=K, relaxed_pool_multiplier=16), x, T, V, "dominant")
    assert rescans >= B


def test_short_lists_spiked_rows(libdbs, oracle_lib):
    # 64 shared token ids get +8 in every row of a step: each row's best 64
    # are the same ids, so the cut of every list lies at the end of the spikes
    rng = np.random.default_rng(5)
    B, K, T, V = 64, 16, 64, 700
    z = rng.standard_normal((B, T, K, V)).astype(np.float32)
    for b in range(B):
        for t in range(T):
            z[b, t, :, rng.choice(V, 64, replace=False)] += 8.0
    _check_batch(libdbs, oracle_lib, dict(beam_size=K), log_softmax_np(z), T, V, "spiked")


def test_short_lists_exact_ties_at_the_cut(libdbs, oracle_lib):
    # few distinct values per row: the 64th and 65th entries of a list tie
    # exactly, so the token order decides and the merge must prove it
    rng = np.random.default_rng(9)
    B, K, T, V = 64, 16, 64, 300
    x = rng.choice(np.array([-2.0, -3.0, -4.0, -6.5], np.float32), size=(B, T, K, V), p=[0.03, 0.07, 0.2, 0.7])
    _check_batch(libdbs, oracle_lib, dict(beam_size=K, eos_token=3), x.astype(np.float32), T, V, "ties")


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_short_lists_16bit_rows(libdbs, oracle_lib, dtype):
    rng = np.random.default_rng(77)
    B, K, T, V = 32, 32, 64, 259   # odd rows: unaligned 16-bit heads and tails
    x = log_softmax_np(1.5 * rng.standard_normal((B, T, K, V)).astype(np.float32))
    if dtype == "f16":
        h = x.astype(np.float16)
        bits, wide, code = h.view(np.uint16), h.astype(np.float32), dc.DBS_DTYPE_F16
    else:
        bits = (x.view(np.uint32) >> 16).astype(np.uint16)
        wide = (bits.astype(np.uint32) << 16).view(np.float32)
        code = dc.DBS_DTYPE_BF16
    opts = dict(beam_size=K, eos_token=2, length_penalty_alpha=0.2)
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


def test_short_lists_variable_batch_with_static_constraints(libdbs, oracle_lib):
    # banned tokens, forced steps, minimum EOS lengths and mixed beam sizes
    # (only the examples with pools above 64 get short lists); the rescans
    # apply the same per-row filters as the scan
    rng = np.random.default_rng(21)
    Bv, maxT, maxK, V = 40, 64, 32, 300
    x = log_softmax_np(1.5 * rng.standard_normal((Bv, maxT, maxK, V)).astype(np.float32))
    steps = rng.integers(56, maxT + 1, Bv).astype(np.int32)
    beams = np.full(Bv, 32, np.int32)
    beams[-4:] = (1, 2, 4, 8)
    eos = np.full(Bv, 2, np.int32)
    minlen = rng.integers(0, 5, Bv).astype(np.int32)
    banned = np.zeros((Bv, V), np.uint8)
    banned[:, rng.choice(V, 40, replace=False)] = 1
    forced = np.full((Bv, maxT), -1, np.int32)
    forced[:, 0] = 1
    forced[rng.random(Bv) < 0.3, 2] = 5
    base = dict(beam_size=4)
    dec = dc.Decoder(libdbs, dc.Options(**base))
    br = dec.decode_batch_variable(np.ascontiguousarray(x), Bv, maxT, maxK, V, steps, beams, eos, minlen, banned,
                                   forced)
    for b in range(Bv):
        T, K = int(steps[b]), int(beams[b])
        opts = dict(base, beam_size=K, eos_token=2, min_length=int(minlen[b]))
        cons = dict(banned=banned[b], forced=forced[b, :T].copy(), min_length=int(minlen[b]))
        want = oracle_lib.decode(oracle_lib.options(**opts), np.ascontiguousarray(x[b, :T, :K]), T, V, **cons)
        assert_decode_equal(dc.read_result(libdbs, libdbs.dbs_batch_result_at(br, b)), want, f"example {b}")
    libdbs.dbs_free_batch_result(br)
    dec.close()


def test_short_lists_pool_longer_than_the_step0_list(libdbs, oracle_lib):
    # a pool of 1280 entries without weights (device API): step 0's one live
    # row lists 1024 entries, fewer than the pool, so the merge completes
    # step 0 from a rescan of that row
    import torch
    import torch_dbs_extension as ext
    rng = np.random.default_rng(41)
    B, T, K, V = 32, 64, 32, 300
    x = log_softmax_np(rng.standard_normal((B, T, K, V)).astype(np.float32))
    opts = ext.DBSOptions(beam_size=K, relaxed_pool_multiplier=40)
    xd = torch.tensor(x, device="cuda")
    tr = ext.DeviceTrace(B, T, K, xd.device, with_pool=True, P=40 * K)
    s = tr.struct()
    s.relaxed_weights = None   # weights are limited to pools of 1024; the decode itself is not
    lib = ext._library()
    h = ext._handle(opts)
    rc = lib.dbs_device_decode_batch_ex(h, ext._vp(xd), B, T, V, ctypes.byref(s), None, 0,
                                        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, lib.dbs_last_error(h)
    torch.cuda.synchronize()
    for b in (0, 17, B - 1):
        want = oracle_lib.decode(oracle_lib.options(beam_size=K, relaxed_pool_multiplier=40),
                                 np.ascontiguousarray(x[b]), T, V)
        for f in ("parents", "tokens", "lengths", "raw_scores", "pool_parents", "pool_tokens", "pool_raw_scores",
                  "final_scores"):
            assert np.array_equal(getattr(tr, f)[b].cpu().numpy().ravel(), want[f]), (b, f)
