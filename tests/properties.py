"""Size-independent properties of decode traces, used by the full-size GPU
tests (and checked against the oracle's own traces on the CPU).

check_uniform_properties: a default-option decode (length penalty 0, no EOS)
of a uniform batch: ranges, the selection as the head of the pool, pool
order, score recurrence, pool completeness against a top-k of every row,
final scores, weights, and the sparse backward of grad_final = e_0.

replay_constrained: one example's selected trace replayed on the host under
forced / banned / minimum-length EOS / repetition-penalty / no-repeat-n-gram
constraints (the filter order of src/differentiable_beam.cpp:327-357 and
:512-549 of the reference).
"""
import math

import numpy as np
import torch


def check_uniform_properties(x, tr, si, sv, sc, K, P, label):
    """Size-independent properties of a default-option decode (alpha 0, no
    EOS) of a uniform batch, checked on the device."""
    B, T, _, V = x.shape
    dev = x.device
    bi = torch.arange(B, device=dev)[:, None]
    pp, pt, praw = tr.pool_parents.long(), tr.pool_tokens.long(), tr.pool_raw_scores
    assert bool(((pp >= 0) & (pp < K)).all()) and bool(((pt >= 0) & (pt < V)).all()), f"{label} pool range"
    steps = torch.arange(1, T + 1, device=dev, dtype=torch.int32)[None, :, None]
    assert bool((tr.pool_lengths == steps).all()) and bool((tr.lengths == steps).all()), f"{label} lengths"
    assert bool((pp[:, 0] == 0).all()), f"{label} step 0 has one live parent"
    assert bool((tr.pool_from_logprob == 1).all()) and bool((tr.from_logprob == 1).all())
    # the selection is the head of the pool; ranking scores equal raw scores
    assert torch.equal(tr.parents, tr.pool_parents[..., :K]) and torch.equal(tr.tokens, tr.pool_tokens[..., :K])
    assert torch.equal(tr.raw_scores, praw[..., :K]) and torch.equal(tr.scores, tr.raw_scores), label
    assert torch.equal(tr.pool_scores, praw), label
    # pool order: score desc, then (parent, token) asc
    key = pp * V + pt
    a, b = praw[..., :-1], praw[..., 1:]
    assert bool(((a > b) | ((a == b) & (key[..., :-1] < key[..., 1:]))).all()), f"{label} pool order"
    kk = min(P + 1, V)
    prev = torch.full((B, K), -math.inf, device=dev)
    prev[:, 0] = 0.0
    for t in range(T):
        xt = x[:, t]
        ppt = pp[:, t]
        lp = xt[bi, ppt, pt[:, t]]
        assert torch.equal(praw[:, t], prev.gather(1, ppt) + lp), f"{label} t={t}: score != parent + log-prob"
        vals = torch.topk(xt.reshape(B * K, V), kk, dim=1).values.view(B, K, kk)
        oh = torch.nn.functional.one_hot(ppt, K)
        rank_in_row = oh.cumsum(1).gather(2, ppt[..., None]).squeeze(2) - 1
        # the pool's entries from each parent are that row's best log-probs:
        # compared after the (monotone) rounding of parent + log-prob, since
        # two log-probs that round to one score tie and go by token order
        best = prev.gather(1, ppt) + vals[bi, ppt, rank_in_row]
        assert torch.equal(praw[:, t], best), f"{label} t={t}: a row's pool entries are not its best"
        cnt = oh.sum(1)
        nxt = vals.gather(2, cnt.clamp(max=kk - 1)[..., None]).squeeze(2)
        beaten = (prev + nxt) > praw[:, t, P - 1:P]
        assert not bool((beaten & torch.isfinite(prev) & (cnt < kk)).any()), f"{label} t={t}: pool incomplete"
        prev = tr.raw_scores[:, t]
    assert torch.equal(tr.final_raw_scores, tr.raw_scores[:, T - 1]) and torch.equal(tr.final_scores,
                                                                                      tr.final_raw_scores)
    ws = tr.weights.double().sum(-1)
    assert bool(((ws - 1.0).abs() <= 1e-5).all()), f"{label} selected weights do not sum to 1"
    # relaxed weights: sigmoids of the pool scores around one threshold per
    # step, so within [0, 1] and non-increasing along the pool order (their
    # sum only approaches K: the reference's bisection stops on its interval)
    rw = tr.relaxed_weights
    assert bool(((rw >= 0) & (rw <= 1)).all()), f"{label} relaxed weights outside [0, 1]"
    assert bool((rw[..., 1:] <= rw[..., :-1] + 1e-6).all()), f"{label} relaxed weights not monotone"
    # sparse backward of grad_final = e_0: 1.0 on each step of beam 0's backtrace
    par = tr.parents.cpu().numpy()
    tok = tr.tokens.cpu().numpy()
    k = np.zeros(B, np.int64)
    want = np.empty((B, T), np.int64)
    rows = np.arange(B)
    for t in range(T - 1, -1, -1):
        p_ = par[rows, t, k].astype(np.int64)
        want[:, t] = (t * K + p_) * V + tok[rows, t, k]
        k = p_
    assert bool((sc == T).all()), f"{label} sparse counts"
    assert np.array_equal(si[:, :T].cpu().numpy(), want), f"{label} sparse indices"
    assert bool((sv[:, :T] == 1.0).all()), f"{label} sparse values"


def replay_constrained(ex, banned_set, eos, min_len, logpen, ngram, label):
    """Replays one example's selected trace on the host and checks every
    constraint and score recurrence. `ex` holds [T,K] arrays and the log-prob
    of every selected (t, parent, token)."""
    T, K = ex["parents"].shape
    prev_raw = np.full(K, -np.inf, np.float32)
    prev_raw[0] = 0.0
    prefixes = [[] for _ in range(K)]
    ended = np.zeros(K, bool)
    for t in range(T):
        new_prefixes = []
        new_ended = np.zeros(K, bool)
        for j in range(K):
            p, v = int(ex["parents"][t, j]), int(ex["tokens"][t, j])
            raw = ex["raw_scores"][t, j]
            if p < 0:
                assert v == -1 and raw == -np.inf, f"{label} t={t} j={j} empty slot"
                new_prefixes.append([])
                continue
            assert 0 <= p < K and np.isfinite(prev_raw[p]), f"{label} t={t} j={j} parent {p}"
            pre = prefixes[p]
            if not ex["from_logprob"][t, j]:
                # an ended beam carried forward with its score
                assert ended[p] and v == eos and raw == prev_raw[p], f"{label} t={t} j={j} carry"
                new_prefixes.append(pre)
                new_ended[j] = True
                continue
            assert not ended[p], f"{label} t={t} j={j} extends an ended beam"
            assert v not in banned_set, f"{label} t={t} j={j} banned token {v}"
            if t == 0:
                assert v == 1, f"{label} step 0 token {v} is not the forced one"
            if v == eos:
                assert t + 1 >= min_len, f"{label} t={t} EOS before the minimum length"
            seq = pre + [v]
            if len(seq) >= ngram:
                tail = tuple(seq[-ngram:])
                earlier = {tuple(seq[i:i + ngram]) for i in range(len(seq) - ngram)}
                assert tail not in earlier, f"{label} t={t} j={j} repeats the {ngram}-gram {tail}"
            lp = ex["lp"][t, j]
            if v in pre:
                want = np.float32(prev_raw[p]) + np.float32(np.float32(lp) - logpen)
                assert abs(float(raw) - float(want)) <= 1e-5 * abs(float(want)) + 1e-6, f"{label} t={t} j={j}"
            else:
                assert raw == np.float32(prev_raw[p]) + np.float32(lp), f"{label} t={t} j={j} score"
            new_prefixes.append(seq)
            new_ended[j] = v == eos
        prefixes = new_prefixes
        ended = new_ended
        prev_raw = ex["raw_scores"][t].copy()
