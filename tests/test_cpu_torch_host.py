"""Host-side logic of the PyTorch mirror: option and shape validation with the
reference's messages (python/torch_dbs_extension.py:73-140), op registration,
and the loud failure when no CUDA device is present."""
import pytest
import torch

import torch_dbs_extension as ext
from torch_dbs_extension import DBSOptions, final_scores


def test_options_args_order_matches_reference():
    o = DBSOptions(beam_size=3)
    assert o.args() == (3, -1, 1.0, 0.25, 8, 4096, 0.0, 1.0e-4, 48, 0, 1, 100_000_000)


@pytest.mark.parametrize("kwargs,message", [
    ({"selected_temperature": 0.0}, "selected_temperature must be positive"),
    ({"soft_topk_temperature": 0.0}, "soft_topk_temperature must be positive"),
    ({"relaxed_pool_multiplier": 0}, "relaxed_pool_multiplier must be positive"),
    ({"vocab_block": 0}, "vocab_block must be positive"),
    ({"length_penalty_alpha": -0.1}, "length_penalty_alpha cannot be negative"),
    ({"soft_topk_tolerance": 0.0}, "soft_topk_tolerance must be positive"),
    ({"soft_topk_max_iters": 0}, "soft_topk_max_iters must be positive"),
    ({"max_dense_gradient_elements": 0}, "max_dense_gradient_elements must be positive"),
    ({"selected_temperature": float("nan")}, "selected_temperature must be finite"),
    ({"validate_inputs": 2}, "validate_inputs must be 0 or 1"),
    ({"min_length": -1}, "min_length cannot be negative"),
])
def test_invalid_options_raise_value_error(kwargs, message):
    with pytest.raises(ValueError, match=message):
        final_scores(torch.randn(4, 2, 16), DBSOptions(beam_size=2, **kwargs))


def test_bad_shapes_raise_value_error():
    opts = DBSOptions(beam_size=2)
    with pytest.raises(ValueError):
        final_scores(torch.randn(2, 3), opts)
    with pytest.raises(ValueError):
        final_scores(torch.randn(4, 3, 16), opts)
    with pytest.raises(ValueError):
        final_scores(torch.empty(0, 2, 8), opts)
    with pytest.raises(ValueError):
        final_scores(torch.empty(1, 4, 3, 8), opts)


def test_eos_outside_vocab():
    x = torch.randn(3, 2, 8)
    with pytest.raises(ValueError, match="eos_token"):
        final_scores(x, DBSOptions(beam_size=2, eos_token=8))
    with pytest.raises(ValueError, match="eos_token"):
        final_scores(x, DBSOptions(beam_size=2, eos_token=-2))


def test_ops_registered_with_reference_schemas():
    fwd = torch.ops.dbs.final_scores_forward.default._schema
    bwd = torch.ops.dbs.final_scores_backward.default._schema
    assert len(fwd.arguments) == 13 and len(bwd.arguments) == 14
    assert [a.name for a in fwd.arguments][1:] == [f.name for f in ext.fields(DBSOptions)]


@pytest.mark.skipif(torch.cuda.is_available(), reason="only meaningful without a CUDA device")
def test_no_cuda_device_fails_loudly():
    x = torch.log_softmax(torch.randn(2, 2, 8), dim=-1)
    with pytest.raises(RuntimeError, match="CUDA"):
        final_scores(x, DBSOptions(beam_size=2))
