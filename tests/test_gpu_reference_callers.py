"""The reference's own callers, run against this library as a drop-in.

oracle/Makefile compiles three of the reference's callers, from the
reference's own sources, against this repository's include/dbs.h and
lib/libdbs.so (nothing of the reference's library is linked in):

* its C ABI unit tests (tests/dbs_tests.cpp, built in Debug so every assert
  runs), which must print "dbs_tests passed";
* its microbenchmark (benchmarks/dbs_bench.cpp), which must exit 0 and print
  its CSV row;
* its ctypes torch binding (python/torch_dbs.py, byte-compiled), loaded with
  DBS_LIBRARY pointing at lib/libdbs.so, whose forward and backward must
  match the oracle;
* its JAX binding (python/jax_dbs.py, byte-compiled): host callbacks that
  call dbs_create / dbs_decode / dbs_backward and the sparse accessors
  through ctypes, wrapped in jax.custom_vjp and jax.pure_callback. jax is
  not installed, so an eager stand-in for those two (and for the
  ShapeDtypeStruct / float32 names the module reads) lets the module load;
  its forward and backward callbacks then run on lib/libdbs.so and must
  match the oracle.

They are built on a host with the reference's source tree and carried to the
GPU host prebuilt; each test skips when its artefact is absent.
"""
import importlib.machinery
import importlib.util
import os
import subprocess
import sys
import types

import numpy as np
import pytest
import torch

from parity import assert_close_rel, log_softmax_np

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "oracle", "_ref")
LIBDBS = os.path.join(ROOT, "differentiable-beam-search-cuda_b200", "lib", "libdbs.so")


def _need(name):
    path = os.path.join(REF, name)
    if not os.path.exists(path):
        pytest.skip(f"{name} not built (oracle/Makefile, needs the reference source tree)")
    return path


def test_reference_unit_tests_pass_on_the_dropin():
    exe = _need("dbs_tests_dropin")
    out = subprocess.run([exe], capture_output=True, text=True, timeout=900)
    assert out.returncode == 0, (out.stdout[-3000:], out.stderr[-3000:])
    assert "dbs_tests passed" in out.stdout


def test_reference_microbenchmark_runs_on_the_dropin():
    exe = _need("dbs_bench_dropin")
    out = subprocess.run([exe, "8", "4", "32000", "2", "3"], capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-3000:]
    lines = [l for l in out.stdout.splitlines() if l.strip()]
    assert lines[0].startswith("T,K,V,B,repeats,forward_us")
    row = lines[1].split(",")
    assert row[:5] == ["8", "4", "32000", "2", "3"]
    assert row[10] == "cuda"          # dbs_selected_kernel_name of the drop-in
    assert int(row[9]) > 0            # sparse gradient entries


def test_reference_torch_binding_on_the_dropin(oracle_lib, monkeypatch):
    pyc = _need("torch_dbs.bytecode")
    monkeypatch.setenv("DBS_LIBRARY", LIBDBS)
    loader = importlib.machinery.SourcelessFileLoader("reference_torch_dbs", pyc)
    spec = importlib.util.spec_from_loader("reference_torch_dbs", loader)
    mod = importlib.util.module_from_spec(spec)
    monkeypatch.setitem(sys.modules, spec.name, mod)   # its dataclasses look their module up
    loader.exec_module(mod)
    rng = np.random.default_rng(12)
    T, K, V = 6, 4, 700
    x = log_softmax_np(1.5 * rng.standard_normal((T, K, V)).astype(np.float32))
    gout = rng.standard_normal(K).astype(np.float32)
    kw = dict(beam_size=K, eos_token=3, length_penalty_alpha=0.3, selected_temperature=0.8)
    xt = torch.tensor(x, requires_grad=True)
    y = mod.final_scores(xt, mod.DBSOptions(**kw))
    y.backward(torch.tensor(gout))
    want = oracle_lib.decode(oracle_lib.options(**kw), x, T, V)
    assert np.array_equal(y.detach().numpy(), want["final_scores"])
    sp = oracle_lib.backward_sparse(want, None, None, gout)
    g = np.zeros(T * K * V, dtype=np.float32)
    np.add.at(g, sp["indices"], sp["values"])
    assert_close_rel(xt.grad.numpy().ravel(), g, 1e-5, "reference binding gradient")


def _eager_jax():
    """The few names python/jax_dbs.py uses from jax, run eagerly: a
    custom_vjp whose forward is the wrapped function and whose registered
    (fwd, bwd) pair is kept for the test, and a pure_callback that calls the
    host function on numpy arrays."""
    jax = types.ModuleType("jax")
    jnp = types.ModuleType("jax.numpy")
    jnp.float32 = np.float32
    jax.numpy = jnp
    jax.rules = []

    class _CustomVJP:
        def __init__(self, fn):
            self.fn = fn

        def defvjp(self, fwd, bwd):
            jax.rules.append((fwd, bwd))

        def __call__(self, *args):
            return self.fn(*args)

    def pure_callback(callback, result_shape_dtype, *args):
        out = np.asarray(callback(*(np.asarray(a) for a in args)))
        assert out.shape == tuple(result_shape_dtype.shape) and out.dtype == result_shape_dtype.dtype
        return out

    jax.custom_vjp = _CustomVJP
    jax.pure_callback = pure_callback
    jax.ShapeDtypeStruct = lambda shape, dtype: types.SimpleNamespace(shape=shape, dtype=np.dtype(dtype))
    return jax, jnp


@pytest.mark.parametrize("kw", [
    dict(beam_size=4),
    dict(beam_size=5, eos_token=7, length_penalty_alpha=0.6, selected_temperature=0.7, min_length=2),
])
def test_reference_jax_binding_on_the_dropin(oracle_lib, monkeypatch, kw):
    pyc = _need("jax_dbs.bytecode")
    jax, jnp = _eager_jax()
    monkeypatch.setitem(sys.modules, "jax", jax)
    monkeypatch.setitem(sys.modules, "jax.numpy", jnp)
    loader = importlib.machinery.SourcelessFileLoader("reference_jax_dbs", pyc)
    spec = importlib.util.spec_from_loader("reference_jax_dbs", loader)
    mod = importlib.util.module_from_spec(spec)
    monkeypatch.setitem(sys.modules, spec.name, mod)   # its dataclasses look their module up
    loader.exec_module(mod)
    rng = np.random.default_rng(31 + kw["beam_size"])
    T, K, V = 7, kw["beam_size"], 900
    x = log_softmax_np(1.3 * rng.standard_normal((T, K, V)).astype(np.float32))
    gout = rng.standard_normal(K).astype(np.float32)
    opts = mod.DBSOptions(**kw)

    y = mod.final_scores(x, opts, LIBDBS)            # forward: pure_callback -> dbs_decode
    fwd, bwd = jax.rules[-1]
    y2, saved = fwd(x)
    (grad,) = bwd(saved, gout)                       # backward: pure_callback -> dbs_backward

    want = oracle_lib.decode(oracle_lib.options(**kw), x, T, V)
    assert np.array_equal(y, want["final_scores"])
    assert np.array_equal(y2, want["final_scores"])
    sp = oracle_lib.backward_sparse(want, None, None, gout)
    g = np.zeros(T * K * V, dtype=np.float32)
    np.add.at(g, sp["indices"], sp["values"])
    assert grad.shape == (T, K, V)
    assert_close_rel(grad.ravel(), g, 1e-5, "reference JAX binding gradient")
