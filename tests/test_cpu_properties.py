"""The full-size GPU tests judge the device decoder through size-independent
properties (tests/properties.py). Here those checks run on the oracle's own
traces, so a property that the reference's algorithm does not satisfy, or a
replay that misreads a constraint, fails on the CPU first; and a planted
mistake in an oracle trace must be caught."""
import math
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from parity import log_softmax_np
from properties import check_uniform_properties, replay_constrained


def _uniform_trace(orc, x, K):
    B, T, _, V = x.shape
    P = 8 * K
    outs = [orc.decode(orc.options(beam_size=K), np.ascontiguousarray(x[b]), T, V) for b in range(B)]
    tr = SimpleNamespace()
    shapes = dict(parents=(T, K), tokens=(T, K), lengths=(T, K), from_logprob=(T, K), raw_scores=(T, K),
                  scores=(T, K), weights=(T, K), pool_parents=(T, P), pool_tokens=(T, P), pool_lengths=(T, P),
                  pool_from_logprob=(T, P), pool_raw_scores=(T, P), pool_scores=(T, P), relaxed_weights=(T, P),
                  final_raw_scores=(K,), final_scores=(K,))
    for f, shp in shapes.items():
        setattr(tr, f, torch.tensor(np.stack([o[f].reshape(shp) for o in outs])))
    gf = np.zeros(K, np.float32)
    gf[0] = 1.0
    bws = [orc.backward_sparse(o, None, None, gf) for o in outs]
    cap = T * (K + P)
    si = torch.zeros((B, cap), dtype=torch.int64)
    sv = torch.zeros((B, cap), dtype=torch.float32)
    sc = torch.tensor([len(bw["indices"]) for bw in bws], dtype=torch.int64)
    for b, bw in enumerate(bws):
        si[b, :len(bw["indices"])] = torch.tensor(bw["indices"])
        sv[b, :len(bw["values"])] = torch.tensor(bw["values"])
    return tr, si, sv, sc, P


def test_uniform_properties_hold_for_the_oracle(oracle_lib):
    rng = np.random.default_rng(3)
    B, T, K, V = 3, 6, 4, 700
    x = log_softmax_np(rng.standard_normal((B, T, K, V)).astype(np.float32))
    tr, si, sv, sc, P = _uniform_trace(oracle_lib, x, K)
    check_uniform_properties(torch.tensor(x), tr, si, sv, sc, K, P, "oracle")


def test_uniform_properties_catch_a_dropped_pool_entry(oracle_lib):
    rng = np.random.default_rng(4)
    B, T, K, V = 2, 5, 4, 500
    x = log_softmax_np(rng.standard_normal((B, T, K, V)).astype(np.float32))
    tr, si, sv, sc, P = _uniform_trace(oracle_lib, x, K)
    # plant a mistake: the best log-prob of the last pool entry's row is
    # lowered below every other value, as if the decoder had skipped it
    b, t = 1, 3
    p = int(tr.pool_parents[b, t, P - 1])
    v = int(tr.pool_tokens[b, t, P - 1])
    y = torch.tensor(x)
    y[b, t, p, v] = -1e30
    with pytest.raises(AssertionError):
        check_uniform_properties(y, tr, si, sv, sc, K, P, "planted")


def _constrained_trace(orc, rng, T, K, V):
    x = log_softmax_np(1.5 * rng.standard_normal((T, K, V)).astype(np.float32))
    banned = np.zeros(V, np.uint8)
    banned[rng.choice(V, 20, replace=False)] = 1
    banned[1] = 0
    forced = np.full(T, -1, np.int32)
    forced[0] = 1
    # a row favours a few tokens so that repeats, EOS and blocked 3-grams occur
    x[:, :, :6] += 3.0
    x = log_softmax_np(x)
    r = orc.decode(orc.options(beam_size=K, eos_token=2, min_length=4), x, T, V, banned=banned, forced=forced,
                   min_length=4, repetition_penalty=1.2, no_repeat_ngram_size=3)
    ex = {f: r[f].reshape(T, K) for f in ("parents", "tokens", "from_logprob", "raw_scores")}
    par = np.maximum(ex["parents"], 0)
    tok = np.maximum(ex["tokens"], 0)
    ex["lp"] = x[np.arange(T)[:, None], par, tok]
    return ex, set(np.flatnonzero(banned).tolist())


@pytest.mark.parametrize("seed", range(4))
def test_constraint_replay_accepts_the_oracle(oracle_lib, seed):
    rng = np.random.default_rng(10 + seed)
    ex, banned = _constrained_trace(oracle_lib, rng, 14, 4, 40)
    replay_constrained(ex, banned, 2, 4, np.float32(math.log(1.2)), 3, f"seed {seed}")


def test_constraint_replay_catches_a_banned_token(oracle_lib):
    rng = np.random.default_rng(20)
    ex, banned = _constrained_trace(oracle_lib, rng, 14, 4, 40)
    # plant a mistake: a beam extended at a late step takes a banned token
    t, j = (int(v[-1]) for v in np.nonzero(ex["from_logprob"]))
    assert t > 0
    bad = dict(ex)
    bad["tokens"] = ex["tokens"].copy()
    bad["tokens"][t, j] = min(banned)
    with pytest.raises(AssertionError, match="banned"):
        replay_constrained(bad, banned, 2, 4, np.float32(math.log(1.2)), 3, "planted")


def test_constraint_replay_catches_a_repeated_ngram():
    # a hand-made trace: one beam writes 1 6 7 1 6 and then 7 again
    toks = [1, 6, 7, 1, 6, 7]
    T = len(toks)
    ex = {"parents": np.zeros((T, 1), np.int32), "tokens": np.array(toks, np.int32)[:, None],
          "from_logprob": np.ones((T, 1), np.uint8), "lp": np.full((T, 1), -1.0, np.float32)}
    raw = []
    acc, seen = np.float32(0.0), []
    for v in toks:
        lp = np.float32(-1.0) - np.float32(math.log(1.2)) if v in seen else np.float32(-1.0)
        acc = np.float32(acc + np.float32(lp))
        raw.append(acc)
        seen.append(v)
    ex["raw_scores"] = np.array(raw, np.float32)[:, None]
    with pytest.raises(AssertionError, match="3-gram"):
        replay_constrained(ex, set(), 2, 4, np.float32(math.log(1.2)), 3, "planted")
