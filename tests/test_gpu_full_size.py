"""The large configurations at their full sizes, checked through properties
that hold at any size, plus oracle spot checks of single examples.

* 256 examples, 64 steps, V = 50257, K = 32 / 64 / 128 (pool 8K), rows
  log_softmax(N(0,1)): 105 / 211 / 421 GB of log-probs, decoded in batches
  of at most 105 GB (examples are independent, so a batch split changes
  nothing). For every example and step: backpointers and tokens in range,
  the selection equal to the head of the pool, the pool ordered by
  (score desc, parent asc, token asc), every pool score equal to its
  parent's score plus its log-prob (fp32 add), and the pool complete: the
  entries from each parent are that row's best log-probs, and the parent's
  next-best candidate does not beat the last pool entry (checked with a
  device top-k of every row). Final scores, weight sums, and the sparse
  backward of grad_final = e_0 (exactly 1.0 on beam 0's backtrace). Three
  examples per beam size are compared with the oracle bit for bit.
* 512 examples, up to 128 steps, V = 128256, K_b in {1,2,4,8,16}, with 256
  banned ids, forced token 1 at step 0, minimum length 8 before EOS 2,
  repetition penalty 1.2 and no repeated 3-gram: decoded in batches of 64
  examples (67 GB of padded log-probs each). Every selected entry of every
  example is replayed on the host: forced / banned / EOS rules, no repeated
  3-gram in any beam's prefix, scores equal to parent score plus the
  (penalised) log-prob. Two examples per batch against the oracle, one of
  them also through the host C ABI with the sparse backward.
* 1 example, 256 steps, K = 16, V = 256000 with 64 spiked ids per step:
  the whole decode and sparse backward against the oracle.

Inputs are generated on the device with one seeded generator per example.
"""
import ctypes
import math
import traceback

import numpy as np
import pytest
import torch

import dbs_ctypes as dc
from parity import assert_decode_equal
from properties import check_uniform_properties, replay_constrained

pytestmark = pytest.mark.gpu

_BATCH_BYTES = 106 * 10 ** 9   # largest slice of log-probs decoded at once


def _free():
    torch.cuda.synchronize()
    torch.cuda.empty_cache()


def _run_freeing(fn, *args):
    """Runs fn(*args). A failure is reported only after the device memory
    that fn's frames held has been released: the traceback of a failed check
    would otherwise keep ~100 GB alive for the tests that follow."""
    failure = None
    try:
        fn(*args)
    except Exception:
        failure = traceback.format_exc()
    _free()
    if failure:
        pytest.fail(failure, pytrace=False)


def _gen_rows(x, b_global, sigma=1.0, spike=False, T=None, K=None, seed=7):
    """Fill x[:T, :K] (one example's [T,K,V] slab) from the example's seeded
    generator: log_softmax(sigma * N(0,1) [+ 8 on 64 ids per step])."""
    V = x.shape[-1]
    T = x.shape[0] if T is None else T
    K = x.shape[1] if K is None else K
    g = torch.Generator(device=x.device)
    g.manual_seed(seed * 1_000_003 + b_global)
    z = torch.empty((T, K, V), device=x.device)
    z.normal_(generator=g)
    if sigma != 1.0:
        z.mul_(sigma)
    if spike:
        for t in range(T):
            ids = torch.randint(0, V, (64,), generator=g, device=x.device)
            z[t, :, ids] += 8.0
    x[:T, :K] = torch.log_softmax(z, dim=-1)


def _device_decode_backward(x, opts):
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


def _oracle_example(oracle_lib, x, tr, si, sv, sc, b, opts_kw, label):
    T, K, V = x.shape[1:]
    want = oracle_lib.decode(oracle_lib.options(**opts_kw), x[b].cpu().numpy(), T, V)
    got = {f: getattr(tr, f)[b].cpu().numpy().ravel() for f in
           ("parents", "tokens", "lengths", "raw_scores", "scores", "weights", "pool_parents", "pool_tokens",
            "pool_lengths", "pool_raw_scores", "pool_scores", "relaxed_weights", "final_scores", "final_raw_scores")}
    assert_decode_equal(got, want, f"{label} example {b}")
    gf = np.zeros(K, dtype=np.float32)
    gf[0] = 1.0
    wb = oracle_lib.backward_sparse(want, None, None, gf)
    n = int(sc[b].item())
    assert n == len(wb["indices"])
    assert np.array_equal(si[b, :n].cpu().numpy(), wb["indices"])
    assert np.array_equal(sv[b, :n].cpu().numpy(), wb["values"])


@pytest.mark.parametrize("K", [32, 64, 128])
def test_large_beam_batch_full_size(oracle_lib, K):
    import torch_dbs_extension as ext
    B, T, V = 256, 64, 50257
    per = max(1, min(B, _BATCH_BYTES // (4 * T * K * V)))
    opts = ext.DBSOptions(beam_size=K)
    P = 8 * K
    dev = torch.device("cuda", 0)

    def batch(b0):
        nb = min(per, B - b0)
        x = torch.empty((nb, T, K, V), dtype=torch.float32, device=dev)
        for b in range(nb):
            _gen_rows(x[b], b0 + b, seed=3)
        tr, si, sv, sc = _device_decode_backward(x, opts)
        label = f"K={K} examples {b0}..{b0 + nb - 1}"
        check_uniform_properties(x, tr, si, sv, sc, K, P, label)
        if b0 == 0:
            for b in sorted({0, nb // 2, nb - 1}):
                _oracle_example(oracle_lib, x, tr, si, sv, sc, b, dict(beam_size=K), label)

    for b0 in range(0, B, per):
        _run_freeing(batch, b0)


def test_huge_vocab_single_sequence_full_size(oracle_lib):
    import torch_dbs_extension as ext
    T, K, V = 256, 16, 256000

    def run():
        x = torch.empty((1, T, K, V), dtype=torch.float32, device=torch.device("cuda", 0))
        _gen_rows(x[0], 0, spike=True, seed=5)
        tr, si, sv, sc = _device_decode_backward(x, ext.DBSOptions(beam_size=K))
        _oracle_example(oracle_lib, x, tr, si, sv, sc, 0, dict(beam_size=K), "B=1 T=256 K=16 V=256000")

    _run_freeing(run)


def test_variable_constrained_batch_full_size(libdbs, oracle_lib):
    import torch_dbs_extension as ext
    rng = np.random.default_rng(4)
    B, maxT, maxK, V = 512, 128, 16, 128256
    eos_tok, min_len, pen, ngram = 2, 8, 1.2, 3
    steps_all = rng.integers(8, maxT + 1, B).astype(np.int32)
    beams_all = rng.choice(np.array([1, 2, 4, 8, 16], np.int32), B).astype(np.int32)
    banned_ids = rng.choice(V, 256, replace=False)
    banned_row = np.zeros(V, np.uint8)
    banned_row[banned_ids] = 1
    banned_set = set(int(v) for v in banned_ids)
    logpen = np.float32(math.log(pen))
    opts = ext.DBSOptions(beam_size=maxK, eos_token=eos_tok, min_length=min_len)
    h = ext._handle(opts)
    lib = ext._library()
    dev = torch.device("cuda", 0)
    per = 64

    def batch(b0):
        nb = min(per, B - b0)
        steps = np.ascontiguousarray(steps_all[b0:b0 + nb])
        beams = np.ascontiguousarray(beams_all[b0:b0 + nb])
        x = torch.zeros((nb, maxT, maxK, V), dtype=torch.float32, device=dev)
        for b in range(nb):
            _gen_rows(x[b], b0 + b, sigma=1.5, T=int(steps[b]), K=int(beams[b]), seed=4)
        eos = np.full(nb, eos_tok, np.int32)
        minl = np.full(nb, min_len, np.int32)
        banned = torch.tensor(np.tile(banned_row, (nb, 1)), device=dev)
        forced_np = np.full((nb, maxT), -1, np.int32)
        forced_np[:, 0] = 1
        forced = torch.tensor(forced_np, device=dev)
        sel = int((steps.astype(np.int64) * beams).sum())
        pool = int((steps.astype(np.int64) * beams * 8).sum())
        fin = int(beams.sum())
        mk = lambda n, dt: torch.empty(n, dtype=dt, device=dev)
        out = dict(parents=mk(sel, torch.int32), tokens=mk(sel, torch.int32), lengths=mk(sel, torch.int32),
                   from_logprob=mk(sel, torch.uint8), raw_scores=mk(sel, torch.float32),
                   scores=mk(sel, torch.float32), weights=mk(sel, torch.float32),
                   pool_parents=mk(pool, torch.int32), pool_tokens=mk(pool, torch.int32),
                   pool_lengths=mk(pool, torch.int32), pool_from_logprob=mk(pool, torch.uint8),
                   pool_raw_scores=mk(pool, torch.float32), pool_scores=mk(pool, torch.float32),
                   relaxed_weights=mk(pool, torch.float32), final_raw_scores=mk(fin, torch.float32),
                   final_scores=mk(fin, torch.float32))
        s = dc.DBSDeviceDecodeOutputs()
        for name, _ in dc.DBSDeviceDecodeOutputs._fields_:
            setattr(s, name, out[name].data_ptr())
        rc = lib.dbs_device_decode_batch_variable_ex(
            h, ext._vp(x), nb, maxT, maxK, V, steps.ctypes.data_as(ctypes.c_void_p),
            beams.ctypes.data_as(ctypes.c_void_p), eos.ctypes.data_as(ctypes.c_void_p),
            minl.ctypes.data_as(ctypes.c_void_p), ext._vp(banned), ext._vp(forced), ctypes.c_float(pen), ngram,
            ctypes.byref(s), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        assert rc == 0, lib.dbs_last_error(h)
        torch.cuda.synchronize()
        sel_off = np.concatenate([[0], np.cumsum(steps.astype(np.int64) * beams)])
        # log-prob of every selected (t, parent, token), gathered on the device
        par = out["parents"].cpu().numpy().astype(np.int64)
        tok = out["tokens"].cpu().numpy().astype(np.int64)
        ex_of = np.repeat(np.arange(nb), steps.astype(np.int64) * beams)
        t_of = np.concatenate([np.repeat(np.arange(int(steps[b])), int(beams[b])) for b in range(nb)])
        flat = (((ex_of * maxT + t_of) * maxK + np.maximum(par, 0)) * V + np.maximum(tok, 0))
        lp = x.view(-1)[torch.tensor(flat, device=dev)].cpu().numpy()
        host = {f: out[f].cpu().numpy() for f in ("parents", "tokens", "from_logprob", "raw_scores")}
        for b in range(nb):
            T, K = int(steps[b]), int(beams[b])
            a, c = sel_off[b], sel_off[b + 1]
            ex = {f: host[f][a:c].reshape(T, K) for f in host}
            ex["lp"] = lp[a:c].reshape(T, K)
            replay_constrained(ex, banned_set, eos_tok, min_len, logpen, ngram, f"example {b0 + b}")
        # oracle spot checks: the cheapest example with K_b >= 8, and the cheapest overall
        cost = steps.astype(np.int64) * beams
        big = [b for b in np.argsort(cost) if beams[b] >= 8][:1]
        picks = sorted(set(big + [int(np.argmin(cost))]))
        pool_off = np.concatenate([[0], np.cumsum(steps.astype(np.int64) * beams * 8)])
        fin_off = np.concatenate([[0], np.cumsum(beams)])
        for b in picks:
            T, K = int(steps[b]), int(beams[b])
            xb = np.ascontiguousarray(x[b, :T, :K].cpu().numpy())
            cons = dict(banned=banned_row, forced=forced_np[b, :T].copy(), min_length=min_len,
                        repetition_penalty=pen, no_repeat_ngram_size=ngram)
            o = oracle_lib.options(beam_size=K, eos_token=eos_tok, min_length=min_len)
            want = oracle_lib.decode(o, xb, T, V, **cons)
            a, c = sel_off[b], sel_off[b + 1]
            for f in ("parents", "tokens", "lengths"):
                assert np.array_equal(out[f][a:c].cpu().numpy(), want[f]), (b0 + b, f)
            assert np.array_equal(out["pool_tokens"][pool_off[b]:pool_off[b + 1]].cpu().numpy(), want["pool_tokens"])
            assert np.array_equal(out["final_scores"][fin_off[b]:fin_off[b + 1]].cpu().numpy(), want["final_scores"])
            if b == picks[-1]:
                # the same example through the reference's host C ABI, with its sparse backward
                got = dc.decode_and_read(libdbs, dc.Options(beam_size=K, eos_token=eos_tok, min_length=min_len), xb,
                                         T, V, grad_final=np.eye(K, dtype=np.float32)[0], **cons)
                assert_decode_equal(got, want, f"host ABI example {b0 + b}")
                wb = oracle_lib.backward_sparse(want, None, None, np.eye(K, dtype=np.float32)[0])
                assert np.array_equal(got["backward"]["indices"], wb["indices"])
                assert np.array_equal(got["backward"]["values"], wb["values"])

    for b0 in range(0, B, per):
        _run_freeing(batch, b0)
