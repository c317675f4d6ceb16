"""The benchmark's own workloads, at their own shapes, against the oracle.

* The torch final_scores batch (bench.py --config 2): all 64 examples of
  B=64, T=32, K=8, V=32000 with the Zipf-biased logits bench.py generates,
  eos 2, length penalty 0.2, selected temperature 0.7; y = final_scores(x),
  y.sum().backward(). Final scores bit-exact, the dense gradient within 1e-5
  relative of the oracle's sparse backward scattered into zeros.
* The large-beam batch (bench.py's default line): the first 16 of its 256
  examples (T=64, K=32, V=50257, log_softmax(N(0,1)), default options, pool
  of 256), decoded as one 16-example call (the fused decode) and, for the
  same examples, inside a 32-example call; every trace array against the
  oracle, and the sparse backward of grad_final = e_0.
"""
import ctypes
import os
import sys

import numpy as np
import pytest
import torch

from parity import assert_close_rel, assert_decode_equal

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def test_config2_batch_all_examples(oracle_lib):
    import bench
    import torch_dbs_extension as ext
    B, T, K, V = (bench.WORKLOAD[k] for k in "BTKV")
    dev = torch.device("cuda", 0)
    x = bench.make_inputs(torch, B, T, K, V, 0, dev)
    x.requires_grad_(True)
    opts = ext.DBSOptions(**bench.OPTIONS)
    y = ext.final_scores(x, opts)
    y.sum().backward()
    torch.cuda.synchronize()
    xh = x.detach().cpu().numpy()
    yh = y.detach().cpu().numpy()
    gh = x.grad.cpu().numpy()
    o = oracle_lib.options(**bench.OPTIONS)
    ones = np.ones(K, dtype=np.float32)
    for b in range(B):
        fwd = oracle_lib.decode(o, xh[b], T, V)
        assert np.array_equal(yh[b], fwd["final_scores"]), f"example {b} final scores"
        sp = oracle_lib.backward_sparse(fwd, None, None, ones)
        want = np.zeros(T * K * V, dtype=np.float32)
        np.add.at(want, sp["indices"], sp["values"])
        assert_close_rel(gh[b].ravel(), want, 1e-5, f"example {b} gradient")


def _decode_with_backward(lib, ext, x, opts):
    B, T, K, V = (int(s) for s in x.shape)
    P = 8 * K
    tr = ext.device_decode(x, opts, with_pool=True, with_weights=True)
    gf = torch.zeros((B, K), device=x.device)
    gf[:, 0] = 1.0
    cap = T * (K + P)
    si = torch.empty((B, cap), dtype=torch.int64, device=x.device)
    sv = torch.empty((B, cap), dtype=torch.float32, device=x.device)
    sc = torch.empty((B,), dtype=torch.int64, device=x.device)
    gi = torch.empty((B, K), device=x.device)
    h = ext._handle(opts)
    s = tr.struct()
    rc = lib.dbs_device_backward_batch(h, B, T, V, ctypes.byref(s), None, None, ext._vp(gf), None, ext._vp(si),
                                       ext._vp(sv), ext._vp(sc), ext._vp(gi),
                                       ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, lib.dbs_last_error(h)
    torch.cuda.synchronize()
    return tr, si, sv, sc, gi


def test_config3_first_examples(oracle_lib):
    import bench
    import torch_dbs_extension as ext
    T, K, V = (bench.WORKLOAD3[k] for k in "TKV")
    dev = torch.device("cuda", 0)
    x = bench.make_inputs3(torch, 32, T, K, V, 0, dev)
    opts = ext.DBSOptions(**bench.OPTIONS3)
    lib = ext._library()
    fields = ("parents", "tokens", "lengths", "raw_scores", "scores", "weights", "pool_parents", "pool_tokens",
              "pool_lengths", "pool_raw_scores", "pool_scores", "relaxed_weights", "final_scores", "final_raw_scores")
    runs = [_decode_with_backward(lib, ext, x[:16].contiguous(), opts), _decode_with_backward(lib, ext, x, opts)]
    xh = x[:16].cpu().numpy()
    o = oracle_lib.options(**bench.OPTIONS3)
    gf = np.zeros(K, dtype=np.float32)
    gf[0] = 1.0
    for b in range(16):
        want = oracle_lib.decode(o, xh[b], T, V)
        wb = oracle_lib.backward_sparse(want, None, None, gf)
        for label, (tr, si, sv, sc, gi) in zip(("16-example call", "32-example call"), runs):
            got = {f: getattr(tr, f)[b].cpu().numpy().ravel() for f in fields}
            assert_decode_equal(got, want, f"{label} example {b}")
            n = int(sc[b].item())
            assert n == len(wb["indices"]), f"{label} example {b} sparse count"
            assert np.array_equal(si[b, :n].cpu().numpy(), wb["indices"])
            assert_close_rel(sv[b, :n].cpu().numpy(), wb["values"], 1e-5, f"{label} example {b} values")
            assert_close_rel(gi[b].cpu().numpy(), wb["grad_initial"], 1e-5, f"{label} example {b} grad_initial")
