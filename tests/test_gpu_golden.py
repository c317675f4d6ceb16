"""The device decoder (through the C ABI of lib/libdbs.so) against the golden
fixtures generated from the reference itself."""
import numpy as np
import pytest

import dbs_ctypes as dc
from parity import (assert_decode_equal, assert_sparse_close, config1_input, golden_config1, load_golden)

pytestmark = pytest.mark.gpu
CASES = load_golden()


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_product_matches_reference_golden(libdbs, case):
    T, V = case["T"], case["V"]
    dec = dc.Decoder(libdbs, dc.Options(**case["opts"]))
    x = np.ascontiguousarray(case["x"])
    r = dec.decode_constrained_ex(x, T, V, **case["cons"]) if case["cons"] else dec.decode(x, T, V)
    got = dc.read_result(libdbs, r)
    assert_decode_equal(got, case["want"], case["name"])
    K, P = got["K"], got["P"]
    gsel = ((np.arange(T * K) % 7) - 3).astype(np.float32) * 0.125
    grel = ((np.arange(T * P) % 11) - 5).astype(np.float32) * 0.03125
    gfin = (np.arange(K) + 1).astype(np.float32) * 0.2
    b = dec.backward(r, gsel, grel, gfin)
    assert_sparse_close(dc.read_backward(libdbs, b, K=K), case["bw_all"], 8e-3, case["name"])
    libdbs.dbs_free_backward(b)
    b = dec.backward(r, None, None, gfin)
    bf = dc.read_backward(libdbs, b, K=K)
    libdbs.dbs_free_backward(b)
    for k in ("indices", "values", "grad_initial"):
        assert np.array_equal(bf[k], case["bw_final"][k]), f"{case['name']} grad_final-only {k}"
    libdbs.dbs_free_result(r)
    dec.close()


def test_product_matches_reference_first_config(libdbs):
    """B=4,T=4,K=4,V=32000 through dbs_decode_batch + dbs_backward(e_0)."""
    sha, want = golden_config1()
    x, got_sha = config1_input()
    assert got_sha == sha
    dec = dc.Decoder(libdbs, dc.Options(beam_size=4))
    br = dec.decode_batch(np.ascontiguousarray(x), 4, 4, 32000, 0)
    e0 = np.array([1, 0, 0, 0], np.float32)
    for b in range(4):
        r = libdbs.dbs_batch_result_at(br, b)
        assert_decode_equal(dc.read_result(libdbs, r), want[b][0], f"config1[{b}]")
        bw = dec.backward(r, None, None, e0)
        out = dc.read_backward(libdbs, bw, K=4)
        libdbs.dbs_free_backward(bw)
        for k in ("indices", "values", "grad_initial"):
            assert np.array_equal(out[k], want[b][1][k])
    libdbs.dbs_free_batch_result(br)
    dec.close()
