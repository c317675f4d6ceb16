"""Shared parity gates and seeded case generators for the tests.

Gates (the reference's contract for this path):
  * tokens, parents, lengths, pool ints, sparse indices: bit-exact;
  * raw / ranking / final scores: bit-exact (same IEEE float operations);
  * selected weights within 3e-3 and relaxed weights within 5e-3 (the
    reference's own scalar-vs-SIMD tolerances, src/differentiable_beam.cpp:
    2545-2548), gradient values within 1e-5 relative (the required gate) when
    they depend only on grad_final, 8e-3 otherwise (:2551-2560).
"""
from __future__ import annotations

import numpy as np

INT_FIELDS = ("parents", "tokens", "lengths", "pool_parents", "pool_tokens", "pool_lengths")
SCORE_FIELDS = ("raw_scores", "scores", "pool_raw_scores", "pool_scores", "final_scores", "final_raw_scores")
WEIGHT_TOL = {"weights": 3e-3, "relaxed_weights": 5e-3}


def assert_decode_equal(got: dict, want: dict, label: str = "", weights: bool = True) -> None:
    for f in INT_FIELDS:
        g, w = np.asarray(got[f]), np.asarray(want[f])
        assert g.shape == w.shape, f"{label} {f} shape {g.shape} != {w.shape}"
        if not np.array_equal(g, w):
            i = int(np.flatnonzero(g != w)[0])
            raise AssertionError(f"{label} {f}[{i}]: got {g[i]} want {w[i]}")
    for f in SCORE_FIELDS:
        g, w = np.asarray(got[f], dtype=np.float32), np.asarray(want[f], dtype=np.float32)
        same = (g == w) | (np.isnan(g) & np.isnan(w))
        if not same.all():
            i = int(np.flatnonzero(~same)[0])
            raise AssertionError(f"{label} {f}[{i}]: got {g[i]!r} want {w[i]!r}")
    if weights:
        for f, tol in WEIGHT_TOL.items():
            g, w = np.asarray(got[f]), np.asarray(want[f])
            if g.size:
                d = float(np.max(np.abs(g - w)))
                assert d <= tol, f"{label} {f} max diff {d} > {tol}"


def assert_close_rel(got, want, rtol, label=""):
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    assert got.shape == want.shape, f"{label} shape {got.shape} != {want.shape}"
    err = np.abs(got - want)
    lim = rtol * np.maximum(np.abs(want), 1.0)
    if not (err <= lim).all():
        i = int(np.flatnonzero(err > lim)[0])
        raise AssertionError(f"{label}[{i}]: got {got[i]!r} want {want[i]!r} (rtol {rtol})")


def assert_sparse_close(got: dict, want: dict, tol: float, label: str = "") -> None:
    """Weight-dependent sparse gradients: compared as dense maps within `tol`.

    Entries whose value is below the tolerance may exist on one side only:
    the reference's SIMD sigmoid floors at FLT_MIN where the scalar one returns
    a subnormal, so a relaxed weight of ~1e-38 can make a ~1e-40 draw appear
    or vanish."""
    keys = np.union1d(np.asarray(got["indices"]), np.asarray(want["indices"]))
    g = dict(zip(np.asarray(got["indices"]).tolist(), np.asarray(got["values"]).tolist()))
    w = dict(zip(np.asarray(want["indices"]).tolist(), np.asarray(want["values"]).tolist()))
    gv = np.array([g.get(k, 0.0) for k in keys.tolist()])
    wv = np.array([w.get(k, 0.0) for k in keys.tolist()])
    assert_close_rel(gv, wv, tol, label + " sparse values")
    assert_close_rel(got["grad_initial"], want["grad_initial"], tol, label + " grad_initial")


def assert_sparse_equal(got: dict, want: dict, rtol: float, label: str = "") -> None:
    gi, wi = np.asarray(got["indices"]), np.asarray(want["indices"])
    assert gi.shape == wi.shape and np.array_equal(gi, wi), f"{label} sparse indices differ ({gi.size} vs {wi.size})"
    assert_close_rel(got["values"], want["values"], rtol, label + " sparse values")
    assert_close_rel(got["grad_initial"], want["grad_initial"], rtol, label + " grad_initial")


def log_softmax_np(logits: np.ndarray) -> np.ndarray:
    m = logits.max(axis=-1, keepdims=True)
    z = logits - m
    return (z - np.log(np.exp(z).sum(axis=-1, keepdims=True))).astype(np.float32)


def random_case(rng: np.random.Generator, max_T=6, max_K=6, max_V=64, allow_constraints=True):
    """A small seeded case covering EOS, length penalty, ties and constraints."""
    T = int(rng.integers(1, max_T + 1))
    K = int(rng.integers(1, max_K + 1))
    V = int(rng.integers(2, max_V + 1))
    eos = int(rng.integers(0, V)) if rng.random() < 0.5 else -1
    opts = dict(
        beam_size=K,
        eos_token=eos,
        relaxed_pool_multiplier=int(rng.integers(1, 6)),
        length_penalty_alpha=float(rng.choice([0.0, 0.0, 0.2, 0.75])),
        min_length=int(rng.integers(0, 4)),
        selected_temperature=float(rng.choice([1.0, 0.7])),
        soft_topk_temperature=float(rng.choice([0.25, 0.4])),
        validate_inputs=1,
    )
    x = log_softmax_np(rng.standard_normal((T, K, V)).astype(np.float32) * float(rng.choice([0.5, 1.5, 4.0])))
    if rng.random() < 0.3:
        x = (np.round(x * 2) / 2).astype(np.float32)  # exact ties
    if rng.random() < 0.1:
        x[rng.random(x.shape) < 0.3] = -np.inf
    cons = {}
    if allow_constraints and rng.random() < 0.5:
        if rng.random() < 0.5:
            cons["banned"] = (rng.random(V) < 0.2).astype(np.uint8)
        if rng.random() < 0.4:
            cons["forced"] = np.where(rng.random(T) < 0.3, rng.integers(0, V, T), -1).astype(np.int32)
        if rng.random() < 0.5:
            cons["repetition_penalty"] = 1.2
        if rng.random() < 0.5:
            cons["no_repeat_ngram_size"] = int(rng.integers(1, 4))
        cons["min_length"] = int(rng.integers(-1, 4))
    return opts, x, T, V, cons


# ---------------------------------------------------------------------------
# Golden fixtures (tests/golden/golden.npz, generated from the reference by
# tests/golden/make_golden.py)
# ---------------------------------------------------------------------------
import json as _json
import os as _os

GOLDEN = _os.path.join(_os.path.dirname(_os.path.abspath(__file__)), "golden", "golden.npz")


def load_golden():
    z = np.load(GOLDEN, allow_pickle=False)
    cases = []
    for name in z["names"]:
        name = str(name)
        meta = _json.loads(str(z[f"{name}/meta"]))
        cons = {}
        for k, v in meta["cons"].items():
            if k == "banned":
                cons[k] = np.asarray(v, dtype=np.uint8)
            elif k == "forced":
                cons[k] = np.asarray(v, dtype=np.int32)
            else:
                cons[k] = v
        want = {k.split("/", 1)[1]: z[k] for k in z.files if k.startswith(name + "/") and "/bw_" not in k}
        bw_all = {k: z[f"{name}/bw_all/{k}"] for k in ("indices", "values", "grad_initial")}
        bw_final = {k: z[f"{name}/bw_final/{k}"] for k in ("indices", "values", "grad_initial")}
        cases.append(dict(name=name, opts=meta["opts"], T=meta["T"], V=meta["V"], cons=cons, x=z[f"{name}/x"],
                          want=want, bw_all=bw_all, bw_final=bw_final))
    return cases


def golden_config1():
    z = np.load(GOLDEN, allow_pickle=False)
    out = []
    for b in range(4):
        want = {k.split("/", 2)[2]: z[k] for k in z.files if k.startswith(f"config1/{b}/") and "/bw/" not in k}
        bw = {k: z[f"config1/{b}/bw/{k}"] for k in ("indices", "values", "grad_initial")}
        out.append((want, bw))
    return str(z["config1/x_sha"]), out


def config1_input():
    import hashlib
    import torch
    torch.manual_seed(0)
    x = torch.log_softmax(1.5 * torch.randn(4, 4, 4, 32000, dtype=torch.float32), dim=-1).numpy()
    return x, hashlib.sha256(x.tobytes()).hexdigest()


def logging_filter(log):
    """A deterministic token filter that depends on the beam's prefix and
    appends every call (batch index, step, parent, prefix, token) to `log`;
    returns the raw callable (wrap it in the binding's CFUNCTYPE)."""
    def fn(user, batch_index, step, parent, prefix, prefix_len, token):
        pre = tuple(prefix[i] for i in range(prefix_len)) if prefix_len else ()
        log.append((batch_index, step, parent, pre, token))
        last = pre[-1] if pre else 0
        return int((token * 7 + step * 3 + parent + last) % 5 != 0)
    return fn


def degenerate_cases():
    """Edge shapes and values: V=1, a single step and beam, rows entirely -inf,
    log-probs near -FLT_MAX (parent + lp overflows), more beams than tokens with
    all tokens but one banned, and a -0.0 / +0.0 tie."""
    rng = np.random.default_rng(42)
    cases = []
    # one-token vocabulary, with and without EOS / min length
    cases.append((dict(beam_size=3), np.zeros((4, 3, 1), np.float32), {}))
    cases.append((dict(beam_size=2, eos_token=0, min_length=2), np.zeros((3, 2, 1), np.float32), {}))
    # single step, single beam
    cases.append((dict(beam_size=1), log_softmax_np(rng.standard_normal((1, 1, 50)).astype(np.float32)), {}))
    # every log-prob -inf except one row
    x = np.full((3, 4, 30), -np.inf, np.float32)
    x[1, 0, 7] = -0.5
    cases.append((dict(beam_size=4, relaxed_pool_multiplier=2), x, {}))
    # values near -FLT_MAX: parent + lp overflows to -inf
    x = np.full((4, 2, 20), -3.0e38, np.float32)
    x[:, :, 3] = -1.0
    x[2, 1, 5] = -2.0e38
    cases.append((dict(beam_size=2, length_penalty_alpha=0.5), x, {}))
    # more beams than tokens, all banned but one, forced steps
    x = log_softmax_np(rng.standard_normal((3, 6, 4)).astype(np.float32))
    banned = np.array([1, 1, 0, 1], np.uint8)
    cases.append((dict(beam_size=6), x, dict(banned=banned, forced=np.array([-1, 2, -1], np.int32))))
    # -0.0 and +0.0 log-probs tie
    x = np.full((2, 2, 8), -5.0, np.float32)
    x[:, :, 1] = -0.0
    x[:, :, 6] = 0.0
    cases.append((dict(beam_size=2, eos_token=6), x, {}))
    return cases

