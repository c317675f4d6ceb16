"""The PyTorch final_scores / decode mirror on the device against the oracle."""
import numpy as np
import pytest
import torch

from parity import assert_close_rel, log_softmax_np

pytestmark = pytest.mark.gpu


def _dense_from_sparse(sp, T, K, V):
    g = np.zeros(T * K * V, dtype=np.float32)
    g[sp["indices"]] += sp["values"]
    return g.reshape(T, K, V)


def _oracle_scores_and_grad(orc, opts_dict, x, gout):
    """Per-example oracle decode + sparse backward, as the reference op does."""
    B, T, K, V = x.shape
    scores = np.zeros((B, K), dtype=np.float32)
    grad = np.zeros_like(x)
    for b in range(B):
        o = orc.options(**opts_dict)
        fwd = orc.decode(o, np.ascontiguousarray(x[b]), T, V)
        scores[b] = fwd["final_scores"]
        if gout is not None:
            sp = orc.backward_sparse(fwd, None, None, gout[b])
            grad[b] = _dense_from_sparse(sp, T, K, V)
    return scores, grad


OPTION_SETS = [
    dict(beam_size=2),
    dict(beam_size=4, eos_token=2),
    dict(beam_size=3, eos_token=5, selected_temperature=0.7, soft_topk_temperature=0.4, relaxed_pool_multiplier=3,
         vocab_block=7, length_penalty_alpha=0.35, soft_topk_tolerance=1e-5, soft_topk_max_iters=64, min_length=2),
    dict(beam_size=8, eos_token=2, length_penalty_alpha=0.2, selected_temperature=0.7),
    dict(beam_size=33),
    # K*K above the merge's per-step capacity: row lists are cut to 64
    dict(beam_size=128, eos_token=2, length_penalty_alpha=0.3),
]


@pytest.mark.parametrize("opts", OPTION_SETS)
def test_final_scores_forward_backward(oracle_lib, opts):
    import torch_dbs_extension as ext
    rng = np.random.default_rng(opts["beam_size"])
    B, T, V = 3, 5, 257
    K = opts["beam_size"]
    x = log_softmax_np(rng.standard_normal((B, T, K, V)).astype(np.float32) * 2)
    gout = rng.standard_normal((B, K)).astype(np.float32)
    want_s, want_g = _oracle_scores_and_grad(oracle_lib, opts, x, gout)
    xt = torch.tensor(x, device="cuda", requires_grad=True)
    y = ext.final_scores(xt, ext.DBSOptions(**opts))
    assert y.shape == (B, K) and y.is_cuda
    assert np.array_equal(y.detach().cpu().numpy(), want_s)
    y.backward(torch.tensor(gout, device="cuda"))
    assert xt.grad is not None and xt.grad.is_cuda
    assert_close_rel(xt.grad.cpu().numpy().ravel(), want_g.ravel(), 1e-5, "grad")


def test_unbatched_and_cpu_tensor(oracle_lib):
    import torch_dbs_extension as ext
    rng = np.random.default_rng(2)
    T, K, V = 4, 3, 129
    x = log_softmax_np(rng.standard_normal((T, K, V)).astype(np.float32))
    want_s, want_g = _oracle_scores_and_grad(oracle_lib, dict(beam_size=K), x[None], np.ones((1, K), np.float32))
    xc = torch.tensor(x, requires_grad=True)
    y = ext.final_scores(xc, ext.DBSOptions(beam_size=K))
    assert y.shape == (K,) and not y.is_cuda
    assert np.array_equal(y.detach().numpy(), want_s[0])
    y.sum().backward()
    assert not xc.grad.is_cuda
    assert_close_rel(xc.grad.numpy().ravel(), want_g[0].ravel(), 1e-5, "grad")


def test_batched_equals_per_example():
    import torch_dbs_extension as ext
    torch.manual_seed(1)
    x = torch.log_softmax(torch.randn(4, 3, 2, 64, device="cuda"), dim=-1)
    opts = ext.DBSOptions(beam_size=2, eos_token=1)
    batched = ext.final_scores(x, opts)
    manual = torch.stack([ext.final_scores(x[b], opts) for b in range(4)])
    assert torch.equal(batched, manual)


def test_non_contiguous_and_half_inputs():
    import torch_dbs_extension as ext
    torch.manual_seed(314)
    base = torch.log_softmax(torch.randn(3, 5, 2, 257), dim=-1)
    x = base.transpose(0, 1)
    opts = ext.DBSOptions(beam_size=2)
    want = torch.stack([ext.final_scores(x[b].contiguous(), opts) for b in range(x.size(0))])
    got = ext.final_scores(x.cuda(), opts).cpu()
    assert torch.equal(got, want)
    half = ext.final_scores(x.cuda().half(), opts)
    assert half.shape == want.shape and torch.isfinite(half).all()


def test_uses_current_stream():
    import torch_dbs_extension as ext
    torch.manual_seed(2026)
    x = torch.log_softmax(torch.randn(2, 5, 3, 257, device="cuda"), dim=-1)
    opts = ext.DBSOptions(beam_size=3, eos_token=7)
    ref = ext.final_scores(x, opts)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        y = ext.final_scores(x, opts)
        marker = torch.empty((), device="cuda").fill_(1.0)
    s.synchronize()
    assert torch.equal(y, ref)
    assert marker.item() == 1.0


def test_nan_and_pos_inf_raise():
    import torch_dbs_extension as ext
    x = torch.log_softmax(torch.randn(4, 2, 16, device="cuda"), dim=-1)
    opts = ext.DBSOptions(beam_size=2)
    for bad in (float("nan"), float("inf")):
        y = x.clone()
        y[0, 0, 0] = bad
        with pytest.raises(RuntimeError, match="NaN or \\+Inf"):
            ext.final_scores(y, opts)
    y = x.clone()
    y[0, 0, 0] = -float("inf")
    assert torch.isfinite(ext.final_scores(y, opts)).all()


def test_decode_returns_tokens_and_scores(oracle_lib):
    import torch_dbs_extension as ext
    x = torch.full((2, 3, 2, 8), -4.0)
    x[:, :, :, 0] = -0.1
    x[:, :, :, 1] = -0.2
    opts = ext.DBSOptions(beam_size=2)
    tokens, scores = ext.decode(x.cuda(), opts)
    assert tokens.shape == (2, 3, 2) and tokens.dtype == torch.int32
    assert torch.equal(scores, ext.final_scores(x.cuda(), opts))
    o = oracle_lib.options(beam_size=2)
    fwd = oracle_lib.decode(o, x[0].numpy(), 3, 8)
    assert np.array_equal(tokens[0].cpu().numpy().ravel(), fwd["tokens"])


def test_torch_ops_schemas(oracle_lib):
    import torch_dbs_extension as ext
    rng = np.random.default_rng(9)
    T, K, V = 3, 2, 40
    x = log_softmax_np(rng.standard_normal((T, K, V)).astype(np.float32))
    opts = ext.DBSOptions(beam_size=K, eos_token=3, length_penalty_alpha=0.2)
    g = torch.tensor([1.0, -0.5])
    y = torch.ops.dbs.final_scores_forward(torch.tensor(x).cuda(), *opts.args())
    grad = torch.ops.dbs.final_scores_backward(torch.tensor(x).cuda(), g.cuda(), *opts.args())
    want_s, want_g = _oracle_scores_and_grad(oracle_lib, dict(beam_size=K, eos_token=3, length_penalty_alpha=0.2),
                                             x[None], g.numpy()[None])
    assert np.array_equal(y.cpu().numpy(), want_s[0])
    assert_close_rel(grad.cpu().numpy().ravel(), want_g[0].ravel(), 1e-5, "op grad")
