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


def _reference_module(monkeypatch):
    """The reference's torch module, byte-compiled by oracle/Makefile, loaded
    with an empty stand-in for its compiled op library: its options,
    validation and error messages are pure Python and run before any op."""
    import importlib.machinery
    import importlib.util
    import os
    import sys
    import types
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    pyc = os.path.join(root, "oracle", "_ref", "torch_dbs_extension.bytecode")
    if not os.path.exists(pyc):
        pytest.skip("oracle/_ref/torch_dbs_extension.bytecode not built (needs the reference source tree)")
    monkeypatch.setitem(sys.modules, "dbs_torch_ext", types.ModuleType("dbs_torch_ext"))
    monkeypatch.setitem(sys.modules, "dbs_torch_cuda_ext", None)   # "not built": the import raises
    loader = importlib.machinery.SourcelessFileLoader("reference_torch_dbs_extension", pyc)
    spec = importlib.util.spec_from_loader("reference_torch_dbs_extension", loader)
    mod = importlib.util.module_from_spec(spec)
    monkeypatch.setitem(sys.modules, spec.name, mod)   # its dataclasses look their module up
    loader.exec_module(mod)
    return mod


def _outcome(fn):
    try:
        fn()
    except (ValueError, TypeError) as e:
        return type(e).__name__, str(e)
    return "accepted", ""


_BAD_OPTIONS = [dict(beam_size=0), dict(beam_size=-1), dict(beam_size=2 ** 31), dict(eos_token=-2),
                dict(selected_temperature=0.0), dict(selected_temperature=-1.0),
                dict(selected_temperature=float("inf")), dict(soft_topk_temperature=float("nan")),
                dict(relaxed_pool_multiplier=0), dict(vocab_block=-4),
                dict(length_penalty_alpha=-0.5), dict(length_penalty_alpha=float("nan")),
                dict(soft_topk_tolerance=0.0), dict(soft_topk_max_iters=-1), dict(min_length=-2),
                dict(validate_inputs=-1), dict(validate_inputs=3), dict(max_dense_gradient_elements=-5)]
_BAD_SHAPES = [(2, 3), (5,), (1, 2, 3, 4, 5), (4, 3, 16), (0, 2, 8), (3, 2, 0), (1, 4, 3, 8), (0, 3, 2, 8),
               (2, 0, 2, 8)]


@pytest.mark.parametrize("kw", _BAD_OPTIONS)
def test_option_errors_match_the_reference_module(monkeypatch, kw):
    """final_scores and decode reject bad options with the reference
    module's exception type and message."""
    ref = _reference_module(monkeypatch)
    x = torch.randn(3, 2, 16)
    opts = dict(dict(beam_size=2), **kw)
    for fn in ("final_scores", "decode"):
        ours = _outcome(lambda: getattr(ext, fn)(x, ext.DBSOptions(**opts)))
        theirs = _outcome(lambda: getattr(ref, fn)(x, ref.DBSOptions(**opts)))
        assert ours == theirs and ours[0] != "accepted", (fn, kw)


@pytest.mark.parametrize("shape", _BAD_SHAPES)
def test_shape_errors_match_the_reference_module(monkeypatch, shape):
    ref = _reference_module(monkeypatch)
    x = torch.randn(*shape) if 0 not in shape else torch.empty(*shape)
    for fn in ("final_scores", "decode"):
        ours = _outcome(lambda: getattr(ext, fn)(x, ext.DBSOptions(beam_size=2)))
        theirs = _outcome(lambda: getattr(ref, fn)(x, ref.DBSOptions(beam_size=2)))
        assert ours == theirs and ours[0] != "accepted", (fn, shape)


@pytest.mark.parametrize("eos", [16, 17, -2, 1000])
def test_eos_errors_match_the_reference_module(monkeypatch, eos):
    ref = _reference_module(monkeypatch)
    x = torch.randn(3, 2, 16)
    ours = _outcome(lambda: ext.final_scores(x, ext.DBSOptions(beam_size=2, eos_token=eos)))
    theirs = _outcome(lambda: ref.final_scores(x, ref.DBSOptions(beam_size=2, eos_token=eos)))
    assert ours == theirs and ours[0] != "accepted"


def test_options_match_the_reference_module(monkeypatch):
    """The same dataclass fields, defaults and args() order."""
    ref = _reference_module(monkeypatch)
    assert [(f.name, f.default) for f in ext.fields(ext.DBSOptions)] == \
        [(f.name, f.default) for f in ref.fields(ref.DBSOptions)]
    o = dict(beam_size=5, eos_token=3, selected_temperature=0.7, relaxed_pool_multiplier=3, min_length=2)
    assert ext.DBSOptions(**o).args() == ref.DBSOptions(**o).args()


def test_op_schemas_equal_the_reference_text():
    """torch.ops.dbs schemas, as registered here, against the reference's
    TORCH_LIBRARY(dbs, m) strings (tests/golden/op_schemas.json, extracted
    by tests/golden/make_op_schemas.py)."""
    import json
    import os
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "op_schemas.json")
    want = json.load(open(path))["schemas"]
    got = [str(torch.ops.dbs.final_scores_forward.default._schema),
           str(torch.ops.dbs.final_scores_backward.default._schema)]
    assert got == ["dbs::" + s for s in want]
