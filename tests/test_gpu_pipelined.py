"""Single-example decodes long enough for the pipelined schedule.

With one example and the selection merge, the decode scans segments of steps
on a helper stream while `stream` merges the segments already scanned, the
beam state passing between merge launches. These cases check the results
against the oracle (bit-exact), including segment boundaries at odd steps
with repetition penalty and n-gram blocking (prefix buffers swap once per
step), a rejected input followed by a good decode on the same workspace, and
the torch path, whose dense-gradient zero fill runs after the scans.
"""
import numpy as np
import pytest
import torch

import dbs_ctypes as dc
from parity import assert_close_rel, assert_decode_equal, log_softmax_np

pytestmark = pytest.mark.gpu


def _oracle_decode(orc, opts, x, T, V, cons):
    return orc.decode(orc.options(**opts), x, T, V, **cons)


@pytest.mark.parametrize("K,T,V,mult,cons", [
    (64, 96, 400, 8, {}),                                       # 16-step segments
    (24, 110, 300, 2, dict(repetition_penalty=1.3, no_repeat_ngram_size=2)),   # 21-step segments
    (16, 260, 700, 8, {}),                                      # 32-step segments, as for V = 256000
])
def test_pipelined_single_example_decode(libdbs, oracle_lib, K, T, V, mult, cons):
    rng = np.random.default_rng(K + T)
    x = log_softmax_np(1.5 * rng.standard_normal((T, K, V)).astype(np.float32))
    opts = dict(beam_size=K, relaxed_pool_multiplier=mult, eos_token=3, length_penalty_alpha=0.2)
    want = _oracle_decode(oracle_lib, opts, x, T, V, cons)
    got = dc.decode_and_read(libdbs, dc.Options(**opts), np.ascontiguousarray(x), T, V, **cons)
    assert_decode_equal(got, want, f"K={K} T={T}")


def test_pipelined_rejects_nan_then_decodes(libdbs, oracle_lib):
    T, K, V = 96, 64, 300
    rng = np.random.default_rng(5)
    x = log_softmax_np(rng.standard_normal((T, K, V)).astype(np.float32))
    opts = dict(beam_size=K, relaxed_pool_multiplier=8)
    bad = x.copy()
    bad[0, 0, 0] = np.nan   # index 0 is always among the validation samples
    dec = dc.Decoder(libdbs, dc.Options(**opts))
    with pytest.raises(dc.DBSError, match="NaN or \\+Inf"):
        dec.decode(np.ascontiguousarray(bad), T, V)
    dec.close()
    want = _oracle_decode(oracle_lib, opts, x, T, V, {})
    for _ in range(2):
        got = dc.decode_and_read(libdbs, dc.Options(**opts), np.ascontiguousarray(x), T, V)
        assert_decode_equal(got, want, "after a rejected call")


def test_pipelined_final_scores_and_gradient(oracle_lib):
    import torch_dbs_extension as ext
    T, K, V = 100, 32, 257   # K*K = 1024 candidates per step: selection merge, 16-step segments
    rng = np.random.default_rng(9)
    x = log_softmax_np(2 * rng.standard_normal((1, T, K, V)).astype(np.float32))
    opts = dict(beam_size=K, eos_token=2, length_penalty_alpha=0.2, selected_temperature=0.7)
    gout = rng.standard_normal((1, K)).astype(np.float32)
    o = oracle_lib.options(**opts)
    fwd = oracle_lib.decode(o, np.ascontiguousarray(x[0]), T, V)
    sp = oracle_lib.backward_sparse(fwd, None, None, gout[0])
    want_g = np.zeros(T * K * V, dtype=np.float32)
    want_g[sp["indices"]] += sp["values"]
    xt = torch.tensor(x, device="cuda", requires_grad=True)
    y = ext.final_scores(xt, ext.DBSOptions(**opts))
    assert np.array_equal(y.detach().cpu().numpy()[0], fwd["final_scores"])
    y.backward(torch.tensor(gout, device="cuda"))
    assert_close_rel(xt.grad.cpu().numpy().ravel(), want_g, 1e-5, "grad")
