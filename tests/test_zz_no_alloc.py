"""dbs_device_backward_sparse_noalloc against dbs_device_backward_batch_ex.

The allocation-free sparse backward keeps its only scratch in a static device
array; on the same trace and gradients it must produce what the allocating
entry point produces, on two calls in a row (the second reuses the scratch
the first left behind). This file is collected last so it also runs after
every other test has used the library.
"""
import ctypes

import numpy as np
import pytest
import torch

import dbs_ctypes
import torch_dbs_extension as ext

pytestmark = pytest.mark.gpu


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _vp(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _sparse_outputs(B, T, K, P, device):
    cap = T * (K + P)
    return (torch.full((B, cap), -7, dtype=torch.int64, device=device),
            torch.full((B, cap), float("nan"), dtype=torch.float32, device=device),
            torch.full((B,), -7, dtype=torch.int64, device=device),
            torch.full((B, K), float("nan"), dtype=torch.float32, device=device))


@pytest.mark.parametrize("opts_kw,shape", [
    (dict(beam_size=4, eos_token=2, length_penalty_alpha=0.3, relaxed_pool_multiplier=3), (3, 6, 97)),
    (dict(beam_size=8, eos_token=2, length_penalty_alpha=0.2, selected_temperature=0.7), (5, 9, 1000)),
])
def test_noalloc_sparse_backward_matches_allocating_entry(opts_kw, shape):
    B, T, V = shape
    torch.manual_seed(11)
    device = torch.device("cuda", 0)
    opts = ext.DBSOptions(**opts_kw)
    K = opts.beam_size
    P = max(K, K * opts.relaxed_pool_multiplier)
    x = torch.log_softmax(1.5 * torch.randn(B, T, K, V, device=device), dim=-1).contiguous()
    trace = ext.device_decode(x, opts, with_pool=True, with_weights=True)
    gs = torch.randn(B, T, K, device=device)
    gr = torch.randn(B, T, P, device=device)
    gf = torch.randn(B, K, device=device)

    lib = ext._library()
    h = ext._handle(opts)
    tr = trace.struct()

    ref = _sparse_outputs(B, T, K, P, device)
    rc = lib.dbs_device_backward_batch_ex(h, B, T, V, ctypes.byref(tr), _vp(gs), _vp(gr), _vp(gf), None,
                                          _vp(ref[0]), _vp(ref[1]), _vp(ref[2]), _vp(ref[3]), 0, _stream())
    assert rc == 0, lib.dbs_last_error(h)
    torch.cuda.synchronize()
    counts = ref[2].cpu().numpy()
    assert (counts > 0).all()

    for _ in range(2):   # two calls in a row on the same scratch
        out = _sparse_outputs(B, T, K, P, device)
        rc = lib.dbs_device_backward_sparse_noalloc(h, B, T, V, ctypes.byref(tr), _vp(gs), _vp(gr), _vp(gf),
                                                    _vp(out[0]), _vp(out[1]), _vp(out[2]), _vp(out[3]), _stream())
        assert rc == 0, lib.dbs_last_error(h)
        torch.cuda.synchronize()
        assert np.array_equal(out[2].cpu().numpy(), counts)
        idx_ref, idx = ref[0].cpu().numpy(), out[0].cpu().numpy()
        val_ref, val = ref[1].cpu().numpy(), out[1].cpu().numpy()
        for b in range(B):
            n = int(counts[b])
            assert np.array_equal(idx[b, :n], idx_ref[b, :n])
            # same kernel body and arithmetic: equal within the 1e-5 relative gate
            np.testing.assert_allclose(val[b, :n], val_ref[b, :n], rtol=1e-5, atol=0)
        np.testing.assert_allclose(out[3].cpu().numpy(), ref[3].cpu().numpy(), rtol=1e-5, atol=0)


def test_noalloc_rejects_sizes_beyond_its_scratch():
    opts = ext.DBSOptions(beam_size=4)
    lib = ext._library()
    h = ext._handle(opts)
    tr = dbs_ctypes.DBSDeviceDecodeOutputs()
    dummy = ctypes.c_void_p(16)   # never dereferenced: the sizes are rejected first
    rc = lib.dbs_device_backward_sparse_noalloc(h, 1, 511, 100, ctypes.byref(tr), None, None, None,
                                                dummy, dummy, dummy, None, _stream())
    assert rc == -2
    assert b"at most 510 steps" in lib.dbs_last_error(h)
    rc = lib.dbs_device_backward_sparse_noalloc(h, 1024, 300, 100, ctypes.byref(tr), None, None, None,
                                                dummy, dummy, dummy, None, _stream())
    assert rc == -2
    assert b"262144" in lib.dbs_last_error(h)


def _synthetic_trace(B, T, K, P, V, device, seed):
    """A trace with the layout a decode writes (parents < K, tokens < V,
    lengths t + 1, weights in (0, 1)); the backward reads nothing else."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    t1 = torch.arange(1, T + 1, dtype=torch.int32)
    arrays = dict(
        parents=torch.randint(0, K, (B, T, K), generator=g, dtype=torch.int32),
        tokens=torch.randint(0, V, (B, T, K), generator=g, dtype=torch.int32),
        lengths=t1.view(1, T, 1).expand(B, T, K).contiguous(),
        from_logprob=torch.randint(0, 2, (B, T, K), generator=g, dtype=torch.uint8),
        weights=torch.rand((B, T, K), generator=g),
        pool_parents=torch.randint(0, K, (B, T, P), generator=g, dtype=torch.int32),
        pool_tokens=torch.randint(0, V, (B, T, P), generator=g, dtype=torch.int32),
        pool_lengths=t1.view(1, T, 1).expand(B, T, P).contiguous(),
        pool_from_logprob=torch.randint(0, 2, (B, T, P), generator=g, dtype=torch.uint8),
        relaxed_weights=torch.rand((B, T, P), generator=g),
    )
    arrays = {k: v.to(device) for k, v in arrays.items()}
    s = dbs_ctypes.DBSDeviceDecodeOutputs()
    for name, _ in dbs_ctypes.DBSDeviceDecodeOutputs._fields_:
        setattr(s, name, arrays[name].data_ptr() if name in arrays else None)
    return s, arrays


@pytest.mark.parametrize("B,T,K,mult,V", [
    (2, 510, 4, 3, 100),       # the longest trace the scratch allows
    (1024, 256, 2, 2, 50),     # batch_size * steps = 262144, the scratch's whole step-count table
    (2, 5, 64, 63, 5000),      # beam + pool = 4096 entries per step
])
def test_noalloc_at_its_limits(B, T, K, mult, V):
    device = torch.device("cuda", 0)
    opts = ext.DBSOptions(beam_size=K, relaxed_pool_multiplier=mult, length_penalty_alpha=0.4,
                          selected_temperature=0.8)
    P = K * mult
    tr, arrays = _synthetic_trace(B, T, K, P, V, device, seed=B + T + K)
    gen = torch.Generator(device=device).manual_seed(5)
    gs = torch.randn((B, T, K), device=device, generator=gen)
    gr = torch.randn((B, T, P), device=device, generator=gen)
    gf = torch.randn((B, K), device=device, generator=gen)
    lib = ext._library()
    h = ext._handle(opts)
    ref = _sparse_outputs(B, T, K, P, device)
    rc = lib.dbs_device_backward_batch_ex(h, B, T, V, ctypes.byref(tr), _vp(gs), _vp(gr), _vp(gf), None,
                                          _vp(ref[0]), _vp(ref[1]), _vp(ref[2]), _vp(ref[3]), 0, _stream())
    assert rc == 0, lib.dbs_last_error(h)
    torch.cuda.synchronize()
    counts = ref[2].cpu().numpy()
    for _ in range(2):
        out = _sparse_outputs(B, T, K, P, device)
        rc = lib.dbs_device_backward_sparse_noalloc(h, B, T, V, ctypes.byref(tr), _vp(gs), _vp(gr), _vp(gf),
                                                    _vp(out[0]), _vp(out[1]), _vp(out[2]), _vp(out[3]), _stream())
        assert rc == 0, lib.dbs_last_error(h)
        torch.cuda.synchronize()
        assert np.array_equal(out[2].cpu().numpy(), counts)
        n_max = int(counts.max())
        idx_ref, idx = ref[0][:, :n_max].cpu().numpy(), out[0][:, :n_max].cpu().numpy()
        val_ref, val = ref[1][:, :n_max].cpu().numpy(), out[1][:, :n_max].cpu().numpy()
        for b in range(B):
            n = int(counts[b])
            assert np.array_equal(idx[b, :n], idx_ref[b, :n]), f"example {b} indices"
            np.testing.assert_allclose(val[b, :n], val_ref[b, :n], rtol=1e-5, atol=1e-30)
        np.testing.assert_allclose(out[3].cpu().numpy(), ref[3].cpu().numpy(), rtol=1e-5, atol=1e-30)
