"""Parity of the device decoder, called through the drop-in C ABI of
lib/libdbs.so, against the oracle (plain-C restatement of the reference)."""
import ctypes

import numpy as np
import pytest

import dbs_ctypes as dc
from parity import (assert_close_rel, assert_decode_equal, assert_sparse_equal, degenerate_cases,
                    log_softmax_np, random_case)

pytestmark = pytest.mark.gpu


def _oracle_decode(orc, opts, x, T, V, cons):
    o = orc.options(**opts)
    return orc.decode(o, x, T, V, **cons)


def _product_decode(lib, opts, x, T, V, cons):
    return dc.decode_and_read(lib, dc.Options(**opts), np.ascontiguousarray(x), T, V, **cons)


@pytest.mark.parametrize("seed", range(8))
def test_random_small_cases_bit_exact(libdbs, oracle_lib, seed):
    rng = np.random.default_rng(1000 + seed)
    for case in range(40):
        opts, x, T, V, cons = random_case(rng)
        want = _oracle_decode(oracle_lib, opts, x, T, V, cons)
        got = _product_decode(libdbs, opts, x, T, V, cons)
        assert_decode_equal(got, want, f"seed={seed} case={case} opts={opts} cons={list(cons)}")


@pytest.mark.parametrize("seed", range(4))
def test_sparse_backward_matches_oracle(libdbs, oracle_lib, seed):
    rng = np.random.default_rng(2000 + seed)
    for case in range(30):
        opts, x, T, V, cons = random_case(rng, allow_constraints=False)
        fwd = _oracle_decode(oracle_lib, opts, x, T, V, {})
        K, P = fwd["K"], fwd["P"]
        gf = rng.standard_normal(K).astype(np.float32)
        use_sel = rng.random() < 0.5
        use_rel = rng.random() < 0.5
        gs = rng.standard_normal(T * K).astype(np.float32) if use_sel else None
        gr = rng.standard_normal(T * P).astype(np.float32) if use_rel else None
        want = oracle_lib.backward_sparse(fwd, gs, gr, gf)
        dec = dc.Decoder(libdbs, dc.Options(**opts))
        r = dec.decode(x, T, V)
        b = dec.backward(r, gs, gr, gf, mode="sparse")
        got = dc.read_backward(libdbs, b, K=K)
        libdbs.dbs_free_backward(b)
        # grad_final-only gradients use the same float ops as the reference;
        # weight-dependent terms inherit the weights' tolerance.
        rtol = 1e-5 if not (use_sel or use_rel) else 8e-3
        assert_sparse_equal(got, want, rtol, f"seed={seed} case={case}")
        # dense backward carries the same values
        if T * K * V <= 200000:
            bd = dec.backward(r, gs, gr, gf, mode="dense")
            dense = dc.read_backward(libdbs, bd, dense_count=T * K * V, K=K)
            libdbs.dbs_free_backward(bd)
            wd = oracle_lib.backward_dense(fwd, gs, gr, gf)
            assert_close_rel(dense["grad_log_probs"], wd["grad_log_probs"], rtol, "dense")
        libdbs.dbs_free_result(r)
        dec.close()


def test_grad_final_backward_is_bit_exact(libdbs, oracle_lib):
    rng = np.random.default_rng(7)
    for case in range(40):
        opts, x, T, V, _ = random_case(rng, allow_constraints=False)
        fwd = _oracle_decode(oracle_lib, opts, x, T, V, {})
        gf = rng.standard_normal(fwd["K"]).astype(np.float32)
        want = oracle_lib.backward_sparse(fwd, None, None, gf)
        out = dc.decode_and_read(libdbs, dc.Options(**opts), x, T, V, grad_final=gf)
        b = out["backward"]
        assert np.array_equal(b["indices"], want["indices"])
        assert np.array_equal(b["values"], want["values"]), f"case {case}"
        assert np.array_equal(b["grad_initial"], want["grad_initial"])


def test_uniform_batch_matches_per_example(libdbs, oracle_lib):
    rng = np.random.default_rng(11)
    B, T, K, V = 5, 6, 4, 301
    x = log_softmax_np(rng.standard_normal((B, T, K, V)).astype(np.float32) * 2)
    opts = dict(beam_size=K, eos_token=3, length_penalty_alpha=0.2, selected_temperature=0.7)
    dec = dc.Decoder(libdbs, dc.Options(**opts))
    br = dec.decode_batch(np.ascontiguousarray(x), B, T, V, 4)
    assert libdbs.dbs_batch_result_size(br) == B
    for b in range(B):
        r = libdbs.dbs_batch_result_at(br, b)
        got = dc.read_result(libdbs, r)
        want = _oracle_decode(oracle_lib, opts, x[b], T, V, {})
        assert_decode_equal(got, want, f"example {b}")
    libdbs.dbs_free_batch_result(br)
    dec.close()


def test_variable_batch_matches_per_example(libdbs, oracle_lib):
    rng = np.random.default_rng(12)
    B, maxT, maxK, V = 6, 7, 5, 97
    x = log_softmax_np(rng.standard_normal((B, maxT, maxK, V)).astype(np.float32) * 1.5)
    steps = rng.integers(1, maxT + 1, B).astype(np.int32)
    beams = rng.integers(1, maxK + 1, B).astype(np.int32)
    eos = rng.integers(-1, 6, B).astype(np.int32)
    minlen = rng.integers(-1, 4, B).astype(np.int32)
    banned = (rng.random((B, V)) < 0.1).astype(np.uint8)
    forced = np.where(rng.random((B, maxT)) < 0.2, rng.integers(0, V, (B, maxT)), -1).astype(np.int32)
    base = dict(beam_size=3, relaxed_pool_multiplier=4, length_penalty_alpha=0.35)
    dec = dc.Decoder(libdbs, dc.Options(**base))
    br = dec.decode_batch_variable(np.ascontiguousarray(x), B, maxT, maxK, V, steps, beams, eos, minlen, banned,
                                   forced)
    for b in range(B):
        T, K = int(steps[b]), int(beams[b])
        opts = dict(base, beam_size=K, eos_token=int(eos[b]), min_length=max(0, int(minlen[b])))
        cons = dict(banned=banned[b], forced=forced[b, :T].copy(), min_length=int(minlen[b]))
        want = _oracle_decode(oracle_lib, opts, np.ascontiguousarray(x[b, :T, :K]), T, V, cons)
        got = dc.read_result(libdbs, libdbs.dbs_batch_result_at(br, b))
        assert_decode_equal(got, want, f"example {b}")
    libdbs.dbs_free_batch_result(br)
    dec.close()


@pytest.mark.parametrize("V", [31999, 32000, 32003, 50257])
def test_vocab_sized_rows_and_alignment(libdbs, oracle_lib, V):
    rng = np.random.default_rng(V)
    T, K = 4, 8
    bias = -1.1 * np.log(np.arange(V, dtype=np.float32) + 1.0)
    x = log_softmax_np(2.0 * rng.standard_normal((T, K, V)).astype(np.float32) + bias)
    opts = dict(beam_size=K, eos_token=2, length_penalty_alpha=0.2, selected_temperature=0.7)
    want = _oracle_decode(oracle_lib, opts, x, T, V, {})
    got = _product_decode(libdbs, opts, x, T, V, {})
    assert_decode_equal(got, want, f"V={V}")


def test_large_pool(libdbs, oracle_lib):
    rng = np.random.default_rng(5)
    T, K, V = 3, 32, 5000   # P = 256
    x = log_softmax_np(rng.standard_normal((T, K, V)).astype(np.float32))
    opts = dict(beam_size=K)
    want = _oracle_decode(oracle_lib, opts, x, T, V, {})
    got = _product_decode(libdbs, opts, x, T, V, {})
    assert_decode_equal(got, want, "K=32")


@pytest.mark.parametrize("K,T,V,mult,alpha", [
    (64, 4, 3000, 8, 0.0),      # P = 512: row lists cut to 128 entries
    (128, 3, 2000, 8, 0.3),     # P = 1024: row lists cut to 64 entries
    (96, 3, 1500, 2, 0.0),      # P = 192, K*P above the per-step capacity
])
def test_beam_times_pool_above_merge_capacity(libdbs, oracle_lib, K, T, V, mult, alpha):
    # K * P exceeds the merge's per-step candidate capacity, so the row lists
    # are shorter than P and the merge must prove (or rescan) every step;
    # at t = 0 the single live parent always needs its row rescanned.
    rng = np.random.default_rng(K * 7 + V)
    bias = -1.1 * np.log(np.arange(V, dtype=np.float32) + 1.0)
    x = log_softmax_np(1.5 * rng.standard_normal((T, K, V)).astype(np.float32) + bias)
    opts = dict(beam_size=K, relaxed_pool_multiplier=mult, length_penalty_alpha=alpha, eos_token=2)
    want = _oracle_decode(oracle_lib, opts, x, T, V, {})
    got = _product_decode(libdbs, opts, x, T, V, {})
    assert_decode_equal(got, want, f"K={K} P={want['P']}")


@pytest.mark.parametrize("mult", [8, 16])
def test_rows_of_very_different_sharpness(libdbs, oracle_lib, mult):
    # Long row lists start from a threshold taken from an earlier row; rows
    # that alternate between sharp and flat distributions make that guess
    # far too high (the row is scanned again) or far too low (slow but exact).
    rng = np.random.default_rng(mult)
    T, K, V = 4, 8, 6000
    scale = np.where(np.arange(K) % 2 == 0, 12.0, 0.3).astype(np.float32)
    x = log_softmax_np(rng.standard_normal((T, K, V)).astype(np.float32) * scale[None, :, None])
    opts = dict(beam_size=K, relaxed_pool_multiplier=mult, eos_token=2)
    want = _oracle_decode(oracle_lib, opts, x, T, V, {})
    got = _product_decode(libdbs, opts, x, T, V, {})
    assert_decode_equal(got, want, f"mult={mult}")
    # a batch with enough rows (9600) that every warp scans several and the
    # speculative threshold is used, failing on every sharp-after-flat row
    B, T, V = 40, 30, 2000
    xb = log_softmax_np(rng.standard_normal((B, T, K, V)).astype(np.float32) * scale[None, None, :, None])
    dec = dc.Decoder(libdbs, dc.Options(**opts))
    br = dec.decode_batch(np.ascontiguousarray(xb), B, T, V, 4)
    for b in range(0, B, 3):
        w = _oracle_decode(oracle_lib, opts, xb[b], T, V, {})
        assert_decode_equal(dc.read_result(libdbs, libdbs.dbs_batch_result_at(br, b)), w, f"batch example {b}")
    libdbs.dbs_free_batch_result(br)
    dec.close()



@pytest.mark.parametrize("K,mult,flat,cons", [
    (8, 8, 0.75, False), (8, 16, 0.65, False), (8, 8, 0.75, True), (32, 8, 0.8, False),
])
def test_speculative_threshold_small_misses(libdbs, oracle_lib, K, mult, flat, cons):
    # Rows alternate between scale 1 and a slightly flatter scale, so a row
    # that follows a scale-1 row usually misses its speculative threshold by
    # a few entries (fewer than 32): the second pass then starts from the
    # lane maxima of what the first pass rejected. With bans and a minimum
    # length on the example the second pass starts from scratch instead.
    rng = np.random.default_rng(100 + mult + K)
    # 9600 rows: every warp scans several (lists of 256 entries at K = 32)
    B, T, V = (40, 30, 2000) if K == 8 else (10, 30, 4000)
    scale = np.where(np.arange(K) % 2 == 0, 1.0, flat).astype(np.float32)
    xb = log_softmax_np(rng.standard_normal((B, T, K, V)).astype(np.float32) * scale[None, None, :, None])
    # a few rows with most values -inf: some lanes reject nothing finite
    xb[3, 4, 1, 40:] = -np.inf
    xb[7, 9, :, :V - 500] = -np.inf
    opts = dict(beam_size=K, relaxed_pool_multiplier=mult, eos_token=2)
    kw = {}
    if cons:
        opts["min_length"] = 6
        banned = (rng.random(V) < 0.02).astype(np.uint8)
        kw = dict(banned=banned, min_length=6)
    dec = dc.Decoder(libdbs, dc.Options(**opts))
    if cons:
        br = dec.decode_batch_variable(np.ascontiguousarray(xb), B, T, K, V, steps=np.full(B, T, np.int32),
                                       beams=np.full(B, K, np.int32), eos=np.full(B, 2, np.int32),
                                       min_lengths=np.full(B, 6, np.int32),
                                       banned=np.ascontiguousarray(np.tile(kw["banned"], (B, 1))), threads=4)
    else:
        br = dec.decode_batch(np.ascontiguousarray(xb), B, T, V, 4)
    for b in sorted(set(range(0, B, 4)) | {3, 7}):
        w = _oracle_decode(oracle_lib, opts, xb[b], T, V, kw)
        assert_decode_equal(dc.read_result(libdbs, libdbs.dbs_batch_result_at(br, b)), w, f"example {b}")
    libdbs.dbs_free_batch_result(br)
    dec.close()


def test_rounding_collisions_in_merged_rows(libdbs, oracle_lib):
    # Parent scores near -1000 (float spacing 6e-5) make log-probs 1e-5
    # apart round to one raw score; with their tokens in reverse order a
    # row's candidates are not in key order, so the step merge must not
    # merge the rows as sorted runs (64-entry lists, 8 beams).
    T, K, V = 3, 8, 120
    x = np.full((T, K, V), -50.0, dtype=np.float32)
    x[0] = -1000.0 - 0.001 * np.arange(V, dtype=np.float32)
    for t in (1, 2):
        x[t, :, 10] = -1.00001
        x[t, :, 5] = -1.00002
        for i in range(20):
            x[t, :, 60 - i] = np.float32(-2.0 - 1e-6 * i)
    opts = dict(beam_size=K, relaxed_pool_multiplier=8)
    want = _oracle_decode(oracle_lib, opts, x, T, V, {})
    got = _product_decode(libdbs, opts, x, T, V, {})
    assert_decode_equal(got, want, "rounding collisions")

def test_massive_ties_with_large_beam(libdbs, oracle_lib):
    # constant rows: thousands of candidates share one key prefix, so the
    # merge's radix selection cannot narrow them and sorts them all
    T, K, V = 3, 64, 400
    x = np.full((T, K, V), -2.0, dtype=np.float32)
    x[:, :, 5] = -1.0
    x[1, 7, 100:180] = -1.5
    opts = dict(beam_size=K, relaxed_pool_multiplier=8)
    want = _oracle_decode(oracle_lib, opts, x, T, V, {})
    got = _product_decode(libdbs, opts, x, T, V, {})
    assert_decode_equal(got, want, "ties K=64")


def test_large_beam_with_constraints(libdbs, oracle_lib):
    rng = np.random.default_rng(77)
    T, K, V = 4, 64, 1200
    x = log_softmax_np(1.5 * rng.standard_normal((T, K, V)).astype(np.float32))
    banned = (rng.random(V) < 0.05).astype(np.uint8)
    opts = dict(beam_size=K, relaxed_pool_multiplier=4, eos_token=2, min_length=2)
    cons = dict(banned=banned, repetition_penalty=1.3, no_repeat_ngram_size=2)
    want = _oracle_decode(oracle_lib, opts, x, T, V, cons)
    got = _product_decode(libdbs, opts, x, T, V, cons)
    assert_decode_equal(got, want, "K=64 constrained")


def test_dense_ties_force_the_rescan_path(libdbs, oracle_lib):
    # every row is constant: every list boundary is an exact tie, so the step
    # merge has to rescan rows to prove the token order
    T, K, V = 3, 4, 300
    x = np.full((T, K, V), -1.0, dtype=np.float32)
    x[:, :, 7] = -0.5
    x[1, 2, 200:260] = -0.25
    opts = dict(beam_size=K, relaxed_pool_multiplier=3)
    want = _oracle_decode(oracle_lib, opts, x, T, V, {})
    got = _product_decode(libdbs, opts, x, T, V, {})
    assert_decode_equal(got, want, "ties")


def test_nan_and_pos_inf_rejected_negative_inf_accepted(libdbs):
    T, K, V = 2, 2, 16
    x = log_softmax_np(np.random.default_rng(0).standard_normal((T, K, V)).astype(np.float32))
    for bad in (np.nan, np.inf):
        y = x.copy()
        y[0, 0, 0] = bad
        dec = dc.Decoder(libdbs, dc.Options(beam_size=K))
        with pytest.raises(dc.DBSError, match="NaN or \\+Inf") as ei:
            dec.decode(y, T, V)
        assert ei.value.rc == -2
        st = dec.stats()
        assert st.last_error_category == 1
        dec.close()
    y = x.copy()
    y[0, 0, 0] = -np.inf
    out = dc.decode_and_read(libdbs, dc.Options(beam_size=K), y, T, V)
    assert np.isfinite(out["final_scores"]).all()


def test_validation_disabled_skips_pos_inf(libdbs, oracle_lib):
    T, K, V = 2, 3, 8
    x = np.full((T, K, V), -4.0, dtype=np.float32)
    x[:, :, 1] = -0.05
    x[0, 0, 2] = np.inf
    x[1, 1, 5] = np.inf
    opts = dict(beam_size=K, validate_inputs=0, relaxed_pool_multiplier=3)
    want = _oracle_decode(oracle_lib, opts, x, T, V, {})
    got = _product_decode(libdbs, opts, x, T, V, {})
    assert_decode_equal(got, want, "+inf")


@pytest.mark.parametrize("seed", range(3))
def test_token_filter_matches_oracle(libdbs, oracle_lib, seed):
    """Host token filter: same results as the oracle and the same sequence of
    filter calls (which the CPU tests pin to the reference library)."""
    from oracle import TOKEN_FILTER_FN
    from parity import logging_filter
    rng = np.random.default_rng(500 + seed)
    T, K, V = 5, 3 + seed, 300
    x = log_softmax_np(rng.standard_normal((T, K, V)).astype(np.float32) * 2)
    opts = dict(beam_size=K, eos_token=4, relaxed_pool_multiplier=3, length_penalty_alpha=0.2)
    cons = dict(banned=(rng.random(V) < 0.05).astype(np.uint8), forced=np.array([-1, 7, -1, -1, -1], np.int32),
                min_length=2, repetition_penalty=1.3, no_repeat_ngram_size=2 if seed else 0)
    log_got, log_want = [], []
    f_got = dc.TOKEN_FILTER_FN(logging_filter(log_got))
    f_want = TOKEN_FILTER_FN(logging_filter(log_want))
    want = oracle_lib.decode(oracle_lib.options(**opts), x, T, V, token_filter=f_want, batch_index=seed, **cons)
    dec = dc.Decoder(libdbs, dc.Options(**opts))
    r = dec.decode_constrained_ex(np.ascontiguousarray(x), T, V, token_filter=f_got, batch_index=seed, **cons)
    got = dc.read_result(libdbs, r)
    libdbs.dbs_free_result(r)
    dec.close()
    assert_decode_equal(got, want, f"filter seed {seed}")
    assert log_got == log_want


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_typed_decode_widening(libdbs, oracle_lib, dtype):
    rng = np.random.default_rng(3)
    T, K, V = 3, 4, 200
    x = log_softmax_np(rng.standard_normal((T, K, V)).astype(np.float32))
    if dtype == "f16":
        h = x.astype(np.float16)
        bits = h.view(np.uint16)
        wide = h.astype(np.float32)
        code = dc.DBS_DTYPE_F16
    else:
        bits = (x.view(np.uint32) >> 16).astype(np.uint16)
        wide = (bits.astype(np.uint32) << 16).view(np.float32)
        code = dc.DBS_DTYPE_BF16
    opts = dict(beam_size=K)
    want = _oracle_decode(oracle_lib, opts, wide, T, V, {})
    dec = dc.Decoder(libdbs, dc.Options(**opts))
    r = ctypes.c_void_p()
    rc = libdbs.dbs_decode_typed(dec.h, bits.ctypes.data_as(ctypes.c_void_p), code, T, V, ctypes.byref(r))
    assert rc == 0, libdbs.dbs_last_error(dec.h)
    got = dc.read_result(libdbs, r)
    libdbs.dbs_free_result(r)
    dec.close()
    assert_decode_equal(got, want, dtype)



@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_typed_long_lists_with_ties_at_the_cut(libdbs, oracle_lib, dtype):
    # 16-bit rows, 64-entry lists: the first 256 values hold 150 copies of
    # one value, so the compaction after them keeps more than 2C entries
    # tied at the C-th value and must cut exactly before the next 256-value
    # group (all above the cut) is appended.
    T, K, V = 2, 8, 4096
    x = np.full((T, K, V), -10.0, dtype=np.float32)
    first = np.where(np.arange(256) % 256 < 150, -6.0, -9.0).astype(np.float32)
    np.random.default_rng(4).shuffle(first)
    x[:, :, :256] = first
    x[:, :, 256:512] = -5.0 + 0.03125 * (np.arange(256) % 32)
    x[1, 3, 700] = -1.0
    if dtype == "f16":
        bits = x.astype(np.float16).view(np.uint16)
        wide = bits.view(np.float16).astype(np.float32)
        code = dc.DBS_DTYPE_F16
    else:
        bits = (x.view(np.uint32) >> 16).astype(np.uint16)
        wide = (bits.astype(np.uint32) << 16).view(np.float32)
        code = dc.DBS_DTYPE_BF16
    assert np.array_equal(wide, x)   # every value is exact in both formats
    opts = dict(beam_size=K, relaxed_pool_multiplier=8)
    want = _oracle_decode(oracle_lib, opts, wide, T, V, {})
    dec = dc.Decoder(libdbs, dc.Options(**opts))
    r = ctypes.c_void_p()
    rc = libdbs.dbs_decode_typed(dec.h, np.ascontiguousarray(bits).ctypes.data_as(ctypes.c_void_p), code, T, V,
                                 ctypes.byref(r))
    assert rc == 0, libdbs.dbs_last_error(dec.h)
    got = dc.read_result(libdbs, r)
    libdbs.dbs_free_result(r)
    dec.close()
    assert_decode_equal(got, want, dtype)

def _to16(x, dtype):
    if dtype == "f16":
        h = x.astype(np.float16)
        return h.view(np.uint16), h.astype(np.float32), dc.DBS_DTYPE_F16
    bits = (x.view(np.uint32) >> 16).astype(np.uint16)
    return bits, (bits.astype(np.uint32) << 16).view(np.float32), dc.DBS_DTYPE_BF16


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
@pytest.mark.parametrize("K,V,mult,B", [(8, 32003, 1, 5), (8, 32000, 8, 3), (4, 50257, 8, 2), (16, 4099, 4, 40)])
def test_typed_batch_reads_16bit_natively(libdbs, oracle_lib, dtype, K, V, mult, B):
    # vocab-sized rows with odd lengths (unaligned 16-bit heads and tails),
    # short (C = K) and long (C = P > 32) row lists, and a batch large enough
    # for the long-list speculation; compared with the oracle on the widened
    # values, which are exact
    rng = np.random.default_rng(V + K)
    T = 6
    bias = -1.1 * np.log(np.arange(V, dtype=np.float32) + 1.0)
    x = log_softmax_np(2.0 * rng.standard_normal((B, T, K, V)).astype(np.float32) + bias)
    bits, wide, code = _to16(x, dtype)
    opts = dict(beam_size=K, relaxed_pool_multiplier=mult, eos_token=2, length_penalty_alpha=0.2)
    dec = dc.Decoder(libdbs, dc.Options(**opts))
    br = ctypes.c_void_p()
    rc = libdbs.dbs_decode_batch_typed(dec.h, np.ascontiguousarray(bits).ctypes.data_as(ctypes.c_void_p), code, B, T,
                                       V, 0, ctypes.byref(br))
    assert rc == 0, libdbs.dbs_last_error(dec.h)
    for b in range(0, B, max(1, B // 4)):
        want = _oracle_decode(oracle_lib, opts, np.ascontiguousarray(wide[b]), T, V, {})
        got = dc.read_result(libdbs, libdbs.dbs_batch_result_at(br, b))
        assert_decode_equal(got, want, f"{dtype} example {b}")
    libdbs.dbs_free_batch_result(br)
    dec.close()


@pytest.mark.parametrize("K,V,T,alpha", [(4, 300, 7, 0.0), (8, 2000, 12, 0.6)])
def test_model_step_decode_matches_prefix_decodes(libdbs, oracle_lib, K, V, T, alpha):
    # The reference fills step t from the tokens of step t-1 and the final
    # scores of a decode of steps 0..t-1 (src/differentiable_beam.cpp:
    # 3506-3586); the oracle side below does exactly that, the product decodes
    # incrementally. Both the callbacks' arguments and the results must match.
    rng = np.random.default_rng(K * V + T)
    base = rng.standard_normal((T, K, V)).astype(np.float32)

    def make_step(log):
        @dc.MODEL_STEP_FN
        def step(user, batch, t, prev_tokens, prev_scores, k_, v_, out):
            toks = [prev_tokens[k] for k in range(K)]
            scs = [prev_scores[k] for k in range(K)]
            log.append((t, tuple(toks), tuple(np.float32(v) for v in scs)))
            row = base[t].copy()
            for k in range(K):
                if toks[k] >= 0:
                    row[k, (toks[k] * 7 + 3) % V] += 3.0
                row[k] += np.float32(0.01) * np.float32(scs[k])
            row = log_softmax_np(row)
            ctypes.memmove(out, row.ctypes.data, row.nbytes)
            return 0
        return step

    opts = dict(beam_size=K, eos_token=2, length_penalty_alpha=alpha, relaxed_pool_multiplier=2)
    log_got = []
    cb = make_step(log_got)
    dec = dc.Decoder(libdbs, dc.Options(**opts))
    r = ctypes.c_void_p()
    assert libdbs.dbs_decode_model_steps(dec.h, cb, None, 0, T, V, ctypes.byref(r)) == 0, libdbs.dbs_last_error(dec.h)
    got = dc.read_result(libdbs, r)
    libdbs.dbs_free_result(r)
    dec.close()

    # oracle: the reference's procedure, one prefix decode per step
    log_want = []
    fill = make_step(log_want)
    x = np.zeros((T, K, V), dtype=np.float32)
    toks = np.full(K, -1, np.int32)
    scs = np.zeros(K, np.float32)
    o = oracle_lib.options(**opts)
    for t in range(T):
        buf = (ctypes.c_float * (K * V))()
        fill(None, 0, t, toks.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
             scs.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), K, V, buf)
        x[t] = np.frombuffer(buf, dtype=np.float32).reshape(K, V)
        if t + 1 < T:
            part = oracle_lib.decode(o, np.ascontiguousarray(x[:t + 1]), t + 1, V)
            toks = part["tokens"][t * K:(t + 1) * K].astype(np.int32).copy()
            scs = part["final_scores"].astype(np.float32).copy()
    want = oracle_lib.decode(o, x, T, V)
    assert log_got == log_want
    assert_decode_equal(got, want, "model steps")


def test_model_step_decode(libdbs):
    # the reference's own model-step case (tests/dbs_tests.cpp:158-209)
    @dc.MODEL_STEP_FN
    def step(user, batch, t, prev_tokens, prev_scores, K, V, out):
        for k in range(K):
            for v in range(V):
                out[k * V + v] = -10.0
            preferred = k if t == 0 else (prev_tokens[k] + 1) % V
            out[k * V + preferred] = 0.0
        return 0

    dec = dc.Decoder(libdbs, dc.Options(beam_size=2, relaxed_pool_multiplier=4, vocab_block=64))
    r = ctypes.c_void_p()
    assert libdbs.dbs_decode_model_steps(dec.h, step, None, 0, 3, 6, ctypes.byref(r)) == 0
    assert libdbs.dbs_result_steps(r) == 3
    tok = dc.read_result(libdbs, r)["tokens"]
    assert tok[0] == 0
    assert dec.stats().used_model_step_callback == 1
    libdbs.dbs_free_result(r)
    dec.close()


def test_concurrent_calls_on_one_handle(libdbs, oracle_lib):
    """The reference's decoder is safe to share between threads; several host
    threads decoding (and running the backward) on one handle at once must get
    the results they get one at a time."""
    import threading
    rng = np.random.default_rng(8)
    T, K, V = 5, 4, 3000
    xs = [log_softmax_np(rng.standard_normal((T, K, V)).astype(np.float32) * 2) for _ in range(8)]
    opts = dict(beam_size=K, eos_token=2, length_penalty_alpha=0.2, relaxed_pool_multiplier=4)
    gf = np.ones(K, dtype=np.float32)
    want = [dc.decode_and_read(libdbs, dc.Options(**opts), x, T, V, grad_final=gf) for x in xs]
    dec = dc.Decoder(libdbs, dc.Options(**opts))
    got = [None] * (3 * len(xs))
    errors = []

    def work(tid):
        try:
            for rep in range(3):
                i = (tid + rep * 4) % len(xs)
                r = dec.decode(np.ascontiguousarray(xs[i]), T, V)
                out = dc.read_result(libdbs, r)
                b = dec.backward(r, None, None, gf, mode="sparse")
                out["backward"] = dc.read_backward(libdbs, b, K=K)
                libdbs.dbs_free_backward(b)
                libdbs.dbs_free_result(r)
                got[tid * 3 + rep] = (i, out)
        except Exception as exc:   # surfaced by the main thread
            errors.append(exc)

    threads = [threading.Thread(target=work, args=(t,)) for t in range(8)]
    for th in threads:
        th.start()
    for th in threads:
        th.join()
    dec.close()
    assert not errors, errors
    for entry in got:
        i, out = entry
        assert_decode_equal(out, want[i], f"thread result {i}")
        assert np.array_equal(out["backward"]["indices"], want[i]["backward"]["indices"])
        assert np.array_equal(out["backward"]["values"], want[i]["backward"]["values"])


@pytest.mark.parametrize("idx", range(len(degenerate_cases())))
def test_degenerate_shapes_and_values(libdbs, oracle_lib, idx):
    opts, x, cons = degenerate_cases()[idx]
    T, K, V = x.shape
    want = _oracle_decode(oracle_lib, opts, x, T, V, cons)
    got = _product_decode(libdbs, opts, np.ascontiguousarray(x), T, V, cons)
    assert_decode_equal(got, want, f"degenerate case {idx}")


def test_more_examples_than_sms_with_sequence_constraints(libdbs, oracle_lib):
    # 200 examples (more than the GPU's SMs, so the step merge runs two
    # 256-thread CTAs per SM) with repetition penalty, 2-gram blocking,
    # banned and forced tokens, mixed steps and beams: every example against
    # the oracle
    rng = np.random.default_rng(31)
    B, maxT, maxK, V = 200, 7, 6, 90
    x = log_softmax_np(1.5 * rng.standard_normal((B, maxT, maxK, V)).astype(np.float32))
    x[:, :, :, :5] += 1.0   # a few favoured tokens, so that repeats and blocked 2-grams occur
    x = log_softmax_np(x)
    steps = rng.integers(2, maxT + 1, B).astype(np.int32)
    beams = rng.integers(1, maxK + 1, B).astype(np.int32)
    banned = (rng.random((B, V)) < 0.05).astype(np.uint8)
    forced = np.where(rng.random((B, maxT)) < 0.1, rng.integers(0, V, (B, maxT)), -1).astype(np.int32)
    base = dict(beam_size=3, eos_token=4, relaxed_pool_multiplier=3)
    results = []
    for b in range(B):
        T, K = int(steps[b]), int(beams[b])
        cons = dict(banned=banned[b], forced=forced[b, :T].copy(), repetition_penalty=1.3, no_repeat_ngram_size=2)
        results.append((T, K, cons))
    # the variable-batch C ABI has no sequence constraints; the device
    # variable batch does (dbs_device_decode_batch_variable_ex)
    import torch
    import torch_dbs_extension as ext
    dev = torch.device("cuda", 0)
    xd = torch.tensor(x, device=dev)
    eos = np.full(B, 4, np.int32)
    minl = np.zeros(B, np.int32)
    sel = int((steps.astype(np.int64) * beams).sum())
    pool = int((steps.astype(np.int64) * beams * 3).sum())
    fin = int(beams.sum())
    sel_names = ("parents", "tokens", "lengths", "from_logprob", "raw_scores", "scores", "weights")
    out = {}
    for name, _ in dc.DBSDeviceDecodeOutputs._fields_:
        n = sel if name in sel_names else (fin if name.startswith("final") else pool)
        dt = torch.uint8 if "from_logprob" in name else (
            torch.int32 if name.split("_")[-1] in ("parents", "tokens", "lengths") else torch.float32)
        out[name] = torch.empty(max(n, 1), dtype=dt, device=dev)
    s = dc.DBSDeviceDecodeOutputs()
    for name, _ in dc.DBSDeviceDecodeOutputs._fields_:
        setattr(s, name, out[name].data_ptr())
    bd = torch.tensor(banned, device=dev)
    fd = torch.tensor(forced, device=dev)
    h = ext._handle(ext.DBSOptions(**base))
    lib = ext._library()
    rc = lib.dbs_device_decode_batch_variable_ex(
        h, ext._vp(xd), B, maxT, maxK, V, steps.ctypes.data_as(ctypes.c_void_p), beams.ctypes.data_as(ctypes.c_void_p),
        eos.ctypes.data_as(ctypes.c_void_p), minl.ctypes.data_as(ctypes.c_void_p), ext._vp(bd), ext._vp(fd),
        ctypes.c_float(1.3), 2, ctypes.byref(s), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, lib.dbs_last_error(h)
    torch.cuda.synchronize()
    sel_off = np.concatenate([[0], np.cumsum(steps.astype(np.int64) * beams)])
    pool_off = np.concatenate([[0], np.cumsum(steps.astype(np.int64) * beams * 3)])
    fin_off = np.concatenate([[0], np.cumsum(beams)])
    host = {f: out[f].cpu().numpy() for f in ("parents", "tokens", "lengths", "raw_scores", "pool_tokens",
                                               "pool_parents", "final_scores")}
    for b, (T, K, cons) in enumerate(results):
        opts = dict(base, beam_size=K)
        want = oracle_lib.decode(oracle_lib.options(**opts), np.ascontiguousarray(x[b, :T, :K]), T, V, **cons)
        a, c = sel_off[b], sel_off[b + 1]
        for f in ("parents", "tokens", "lengths", "raw_scores"):
            assert np.array_equal(host[f][a:c], want[f]), (b, f)
        for f in ("pool_tokens", "pool_parents"):
            assert np.array_equal(host[f][pool_off[b]:pool_off[b + 1]], want[f]), (b, f)
        assert np.array_equal(host["final_scores"][fin_off[b]:fin_off[b + 1]], want["final_scores"]), b
