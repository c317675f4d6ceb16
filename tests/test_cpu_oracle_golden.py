"""The oracle (plain-C restatement) against the reference's own outputs.

Pins the oracle before it is trusted as the checker: every golden case (the
reference's handcrafted parity cases, its C ABI test inputs, seeded random
cases and the first-config workload) must match bit-exactly on ints and
scores, within the reference's tolerances on weights and weight-dependent
gradients, and bit-exactly on grad_final-only gradients.
"""
import numpy as np
import pytest

from parity import (assert_decode_equal, assert_sparse_close, config1_input, golden_config1, load_golden)

CASES = load_golden()


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_oracle_matches_reference_golden(oracle_lib, case):
    o = oracle_lib.options(**case["opts"])
    fwd = oracle_lib.decode(o, case["x"], case["T"], case["V"], **case["cons"])
    assert_decode_equal(fwd, case["want"], case["name"])
    K, P = fwd["K"], fwd["P"]
    T = case["T"]
    gsel = ((np.arange(T * K) % 7) - 3).astype(np.float32) * 0.125
    grel = ((np.arange(T * P) % 11) - 5).astype(np.float32) * 0.03125
    gfin = (np.arange(K) + 1).astype(np.float32) * 0.2
    bw = oracle_lib.backward_sparse(fwd, gsel, grel, gfin)
    assert_sparse_close(bw, case["bw_all"], 8e-3, case["name"])
    bf = oracle_lib.backward_sparse(fwd, None, None, gfin)
    for k in ("indices", "values", "grad_initial"):
        assert np.array_equal(bf[k], case["bw_final"][k]), f"{case['name']} grad_final-only {k}"


def test_oracle_matches_reference_first_config(oracle_lib):
    sha, want = golden_config1()
    x, got_sha = config1_input()
    assert got_sha == sha, "regenerated first-config input drifted from the fixture"
    for b in range(4):
        o = oracle_lib.options(beam_size=4)
        fwd = oracle_lib.decode(o, x[b], 4, 32000)
        assert_decode_equal(fwd, want[b][0], f"config1[{b}]")
        bw = oracle_lib.backward_sparse(fwd, None, None, np.array([1, 0, 0, 0], np.float32))
        for k in ("indices", "values", "grad_initial"):
            assert np.array_equal(bw[k], want[b][1][k])


def test_reference_debug_unit_tests_pass():
    """The reference's own C ABI unit tests, built in Debug (asserts live)."""
    import os
    import subprocess
    exe = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref",
                       "dbs_tests_debug")
    if not os.path.exists(exe):
        pytest.skip("reference tests not built here (no reference tree)")
    out = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0 and "dbs_tests passed" in out.stdout


def test_reference_scalar_and_simd_paths_agree():
    """The reference's own scalar-vs-SIMD harness (tests/simd_internal_tests.cpp):
    the scalar path the oracle restates agrees with the SIMD kernels the
    reference library dispatches to (the CPU baseline's kernel)."""
    import os
    import subprocess
    exe = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref",
                       "dbs_simd_parity")
    if not os.path.exists(exe):
        pytest.skip("reference harness not built here (no reference tree)")
    out = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0 and "dbs_simd_internal_tests passed" in out.stdout, out.stdout[-2000:]


def test_oracle_live_against_reference_random(oracle_lib):
    """Seeded random cases beyond the fixtures, against oracle/_ref directly."""
    import dbs_ctypes as dc
    from oracle import reference_library_path
    from parity import random_case
    path = reference_library_path()
    if path is None:
        pytest.skip("oracle/_ref not built")
    ref = dc.load_library(path, device_api=False)
    rng = np.random.default_rng(99)
    for i in range(150):
        opts, x, T, V, cons = random_case(rng)
        o = oracle_lib.options(**opts)
        want = dc.decode_and_read(ref, dc.Options(**opts), np.ascontiguousarray(x), T, V, **cons)
        got = oracle_lib.decode(o, x, T, V, **cons)
        assert_decode_equal(got, want, f"random {i}")


def test_oracle_backward_live_against_reference_random(oracle_lib):
    """The surrogate backward on seeded random cases beyond the fixtures,
    against oracle/_ref directly: with grad_final alone bit-exact (indices,
    values, grad_initial, and the dense form); with selected and relaxed
    weight gradients too, within the reference's weight tolerance (its
    weights use a SIMD exp)."""
    import dbs_ctypes as dc
    from oracle import reference_library_path
    from parity import random_case
    path = reference_library_path()
    if path is None:
        pytest.skip("oracle/_ref not built")
    ref = dc.load_library(path, device_api=False)
    rng = np.random.default_rng(123)
    for i in range(80):
        opts, x, T, V, cons = random_case(rng)
        x = np.ascontiguousarray(x)
        dec = dc.Decoder(ref, dc.Options(**opts))
        r = dec.decode_constrained_ex(x, T, V, **cons) if cons else dec.decode(x, T, V)
        try:
            fwd = oracle_lib.decode(oracle_lib.options(**opts), x, T, V, **cons)
            K, P = fwd["K"], fwd["P"]
            gfin = rng.standard_normal(K).astype(np.float32)
            gsel = rng.standard_normal(T * K).astype(np.float32)
            grel = rng.standard_normal(T * P).astype(np.float32)
            b = dec.backward(r, None, None, gfin, mode="sparse")
            want = dc.read_backward(ref, b, K=K)
            ref.dbs_free_backward(b)
            got = oracle_lib.backward_sparse(fwd, None, None, gfin)
            for k in ("indices", "values", "grad_initial"):
                assert np.array_equal(got[k], want[k]), f"random {i}: grad_final-only {k}"
            b = dec.backward(r, gsel, grel, gfin, mode="sparse")
            want = dc.read_backward(ref, b, K=K)
            ref.dbs_free_backward(b)
            got = oracle_lib.backward_sparse(fwd, gsel, grel, gfin)
            assert_sparse_close(got, want, 8e-3, f"random {i}")
            # the dense form (dbs_backward_dense), grad_final alone
            b = dec.backward(r, None, None, gfin, mode="dense")
            want = dc.read_backward(ref, b, dense_count=T * K * V, K=K)
            ref.dbs_free_backward(b)
            got = oracle_lib.backward_dense(fwd, None, None, gfin)
            assert not want["sparse"]
            for k in ("grad_log_probs", "grad_initial"):
                assert np.array_equal(got[k], want[k]), f"random {i}: dense {k}"
        finally:
            ref.dbs_free_result(r)
            dec.close()


@pytest.mark.parametrize("seed", range(4))
def test_variable_batch_restatement_matches_reference(oracle_lib, seed):
    """dbs_decode_batch_variable restated per example as the GPU tests check
    it (the example's beam size, steps, EOS and minimum length as its
    options, its banned row and forced prefix as constraints, its [T_b,K_b]
    corner of the padded input), against the reference library's own
    variable batch on the same padded input."""
    import dbs_ctypes as dc
    from oracle import reference_library_path
    from parity import log_softmax_np
    path = reference_library_path()
    if path is None:
        pytest.skip("oracle/_ref not built")
    ref = dc.load_library(path, device_api=False)
    rng = np.random.default_rng(700 + seed)
    B, maxT, maxK, V = 6, 7, 5, 97
    x = log_softmax_np(rng.standard_normal((B, maxT, maxK, V)).astype(np.float32) * 1.5)
    steps = rng.integers(1, maxT + 1, B).astype(np.int32)
    beams = rng.integers(1, maxK + 1, B).astype(np.int32)
    eos = rng.integers(-1, 6, B).astype(np.int32)
    minlen = rng.integers(-1, 4, B).astype(np.int32)
    banned = (rng.random((B, V)) < 0.1).astype(np.uint8)
    forced = np.where(rng.random((B, maxT)) < 0.2, rng.integers(0, V, (B, maxT)), -1).astype(np.int32)
    base = dict(beam_size=3, relaxed_pool_multiplier=4, length_penalty_alpha=0.35)
    dec = dc.Decoder(ref, dc.Options(**base))
    br = dec.decode_batch_variable(np.ascontiguousarray(x), B, maxT, maxK, V, steps, beams, eos, minlen, banned,
                                   forced, threads=1)
    try:
        for b in range(B):
            T, K = int(steps[b]), int(beams[b])
            opts = dict(base, beam_size=K, eos_token=int(eos[b]), min_length=max(0, int(minlen[b])))
            cons = dict(banned=banned[b], forced=forced[b, :T].copy(), min_length=int(minlen[b]))
            got = oracle_lib.decode(oracle_lib.options(**opts), np.ascontiguousarray(x[b, :T, :K]), T, V, **cons)
            want = dc.read_result(ref, ref.dbs_batch_result_at(br, b))
            assert_decode_equal(got, want, f"seed {seed} example {b}")
    finally:
        ref.dbs_free_batch_result(br)
        dec.close()


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_typed_widening_matches_reference(oracle_lib, dtype):
    """dbs_decode_typed restated as the oracle's fp32 decode of the exactly
    widened values (as the GPU tests check it), against the reference
    library's own typed decode of the same 16-bit words: near-zero log-probs
    that are subnormal in fp16, -inf entries and signed zeros included."""
    import ctypes
    import dbs_ctypes as dc
    from oracle import reference_library_path
    from parity import log_softmax_np
    path = reference_library_path()
    if path is None:
        pytest.skip("oracle/_ref not built")
    ref = dc.load_library(path, device_api=False)
    rng = np.random.default_rng(17)
    for i in range(12):
        T, K, V = int(rng.integers(1, 6)), int(rng.integers(1, 6)), int(rng.integers(2, 300))
        x = log_softmax_np(rng.standard_normal((T, K, V)).astype(np.float32) * float(rng.choice([0.5, 3.0])))
        x[rng.random(x.shape) < 0.05] = -np.inf
        x[rng.random(x.shape) < 0.02] = -1e-6
        x[rng.random(x.shape) < 0.02] = -0.0
        if dtype == "f16":
            h = x.astype(np.float16)
            bits = np.ascontiguousarray(h.view(np.uint16))
            wide = h.astype(np.float32)
            code = dc.DBS_DTYPE_F16
        else:
            bits = np.ascontiguousarray((x.view(np.uint32) >> 16).astype(np.uint16))
            wide = (bits.astype(np.uint32) << 16).view(np.float32)
            code = dc.DBS_DTYPE_BF16
        opts = dict(beam_size=K, eos_token=int(rng.integers(-1, V)), length_penalty_alpha=0.4)
        got = oracle_lib.decode(oracle_lib.options(**opts), np.ascontiguousarray(wide), T, V)
        dec = dc.Decoder(ref, dc.Options(**opts))
        r = ctypes.c_void_p()
        rc = ref.dbs_decode_typed(dec.h, bits.ctypes.data_as(ctypes.c_void_p), code, T, V, ctypes.byref(r))
        assert rc == 0, ref.dbs_last_error(dec.h)
        want = dc.read_result(ref, r)
        ref.dbs_free_result(r)
        dec.close()
        assert_decode_equal(got, want, f"{dtype} case {i}")


@pytest.mark.parametrize("K,V,T,alpha", [(4, 300, 7, 0.0), (8, 2000, 12, 0.6), (3, 50, 9, 0.3)])
def test_model_step_restatement_matches_reference(oracle_lib, K, V, T, alpha):
    """dbs_decode_model_steps restated as the GPU tests check it: step t is
    filled from the tokens of step t-1 and the final scores of an oracle
    decode of steps 0..t-1, then the whole trace decoded. Against the
    reference library's own model-step decode with the same callback: the
    callbacks' arguments and the results must match."""
    import ctypes
    import dbs_ctypes as dc
    from oracle import reference_library_path
    from parity import log_softmax_np
    path = reference_library_path()
    if path is None:
        pytest.skip("oracle/_ref not built")
    ref = dc.load_library(path, device_api=False)
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
    log_ref = []
    cb = make_step(log_ref)
    dec = dc.Decoder(ref, dc.Options(**opts))
    r = ctypes.c_void_p()
    assert ref.dbs_decode_model_steps(dec.h, cb, None, 0, T, V, ctypes.byref(r)) == 0, ref.dbs_last_error(dec.h)
    want = dc.read_result(ref, r)
    ref.dbs_free_result(r)
    dec.close()

    log_orc = []
    fill = make_step(log_orc)
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
    got = oracle_lib.decode(o, x, T, V)
    assert log_orc == log_ref
    assert_decode_equal(got, want, "model steps")


def _reference_scalar_lib():
    """oracle/_ref/libdbs_ref_scalar.so (the reference library with a switch
    to its scalar kernels, oracle/ref_scalar.cpp), pinned to the scalar path
    for this thread."""
    import ctypes
    import os
    import dbs_ctypes as dc
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref",
                        "libdbs_ref_scalar.so")
    if not os.path.exists(path):
        pytest.skip("oracle/_ref/libdbs_ref_scalar.so not built (needs the reference source tree)")
    lib = dc.load_library(path, device_api=False)
    lib.dbs_ref_force_scalar.argtypes = [ctypes.c_int]
    lib.dbs_ref_force_scalar.restype = None
    lib.dbs_ref_force_scalar(1)
    assert lib.dbs_selected_kernel_name() == b"scalar"
    return lib


def _assert_all_equal(got, want, label):
    for k, v in want.items():
        if isinstance(v, np.ndarray) and k in got:
            assert np.array_equal(np.asarray(got[k]), v, equal_nan=v.dtype.kind == "f"), f"{label}: {k}"


def test_oracle_bit_exact_against_the_reference_scalar_path(oracle_lib):
    """With the reference pinned to its scalar kernels (the path the oracle
    restates), every output is bit-exact, the selected and relaxed weights
    included, and so is the sparse and dense backward with selected,
    relaxed and final gradients: seeded random cases and the degenerate
    cases. (Against the SIMD kernels the reference picks by default, weights
    differ in the last bits; see the tolerance-based checks above.)"""
    import dbs_ctypes as dc
    from parity import degenerate_cases, random_case
    ref = _reference_scalar_lib()
    rng = np.random.default_rng(5)
    cases = [random_case(rng) for _ in range(120)]
    cases += [(o, x, x.shape[0], x.shape[2], c) for o, x, c in degenerate_cases()]
    for i, (opts, x, T, V, cons) in enumerate(cases):
        x = np.ascontiguousarray(x)
        dec = dc.Decoder(ref, dc.Options(**opts))
        r = dec.decode_constrained_ex(x, T, V, **cons) if cons else dec.decode(x, T, V)
        try:
            want = dc.read_result(ref, r)
            fwd = oracle_lib.decode(oracle_lib.options(**opts), x, T, V, **cons)
            _assert_all_equal(fwd, want, f"case {i}")
            K, P = fwd["K"], fwd["P"]
            gf = rng.standard_normal(K).astype(np.float32)
            gs = rng.standard_normal(T * K).astype(np.float32)
            gr = rng.standard_normal(T * P).astype(np.float32)
            b = dec.backward(r, gs, gr, gf, mode="sparse")
            wb = dc.read_backward(ref, b, K=K)
            ref.dbs_free_backward(b)
            _assert_all_equal(oracle_lib.backward_sparse(fwd, gs, gr, gf), wb, f"case {i} sparse backward")
            b = dec.backward(r, gs, gr, gf, mode="dense")
            wd = dc.read_backward(ref, b, dense_count=T * K * V, K=K)
            ref.dbs_free_backward(b)
            _assert_all_equal(oracle_lib.backward_dense(fwd, gs, gr, gf), wd, f"case {i} dense backward")
        finally:
            ref.dbs_free_result(r)
            dec.close()


def test_oracle_token_filter_matches_reference(oracle_lib):
    """The token filter: same results and the same sequence of filter calls
    (batch index, step, parent, prefix, token) as the reference library."""
    import dbs_ctypes as dc
    from oracle import TOKEN_FILTER_FN, reference_library_path
    from parity import logging_filter
    path = reference_library_path()
    if path is None:
        pytest.skip("oracle/_ref not built")
    ref = dc.load_library(path, device_api=False)
    rng = np.random.default_rng(31)
    for i in range(12):
        T, K, V = int(rng.integers(1, 6)), int(rng.integers(1, 5)), int(rng.integers(5, 40))
        x = (rng.standard_normal((T, K, V)) * 2).astype(np.float32)
        x = x - np.log(np.exp(x).sum(-1, keepdims=True))
        opts = dict(beam_size=K, eos_token=int(rng.integers(-1, V)), relaxed_pool_multiplier=2,
                    length_penalty_alpha=0.3)
        cons = dict(banned=(rng.random(V) < 0.1).astype(np.uint8), no_repeat_ngram_size=int(rng.integers(0, 3)),
                    repetition_penalty=float(rng.choice([1.0, 1.4])), min_length=int(rng.integers(-1, 3)))
        log_ref, log_orc = [], []
        f_ref = dc.TOKEN_FILTER_FN(logging_filter(log_ref))
        f_orc = TOKEN_FILTER_FN(logging_filter(log_orc))
        dec = dc.Decoder(ref, dc.Options(**opts))
        r = dec.decode_constrained_ex(np.ascontiguousarray(x), T, V, token_filter=f_ref, batch_index=3, **cons)
        want = dc.read_result(ref, r)
        ref.dbs_free_result(r)
        dec.close()
        got = oracle_lib.decode(oracle_lib.options(**opts), x, T, V, token_filter=f_orc, batch_index=3, **cons)
        assert_decode_equal(got, want, f"filter case {i}")
        assert log_orc == log_ref, f"filter case {i}: call sequence differs"



def test_oracle_degenerate_cases_match_reference(oracle_lib):
    """Edge shapes and values (V=1, -inf rows, overflow near -FLT_MAX, K > V,
    signed zeros) against oracle/_ref directly."""
    import dbs_ctypes as dc
    from oracle import reference_library_path
    from parity import degenerate_cases
    path = reference_library_path()
    if path is None:
        pytest.skip("oracle/_ref not built")
    ref = dc.load_library(path, device_api=False)
    for i, (opts, x, cons) in enumerate(degenerate_cases()):
        T, K, V = x.shape
        want = dc.decode_and_read(ref, dc.Options(**opts), np.ascontiguousarray(x), T, V, **cons)
        got = oracle_lib.decode(oracle_lib.options(**opts), x, T, V, **cons)
        assert_decode_equal(got, want, f"degenerate {i}")
