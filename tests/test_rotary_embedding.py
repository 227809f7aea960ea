"""``RotaryEmbedding`` (nn/position.py:61-232) on CPU: field and input checks, the cached / uncached
tables, and ``apply_rotary_pos_emb``'s argument checks (raised before any device work), case by case as
the reference's ``tests/test_rope.py:44-210`` states them."""
import numpy as np
import pytest
import torch

from jaxml_b200.nn import RotaryEmbedding

X = torch.ones(1, 2, 1, 4)


@pytest.mark.parametrize("kwargs,exc,match", [
    ({"dim": True, "max_length": 8}, TypeError, "dim must be an integer"),
    ({"dim": np.bool_(True), "max_length": 8}, TypeError, "dim must be an integer"),
    ({"dim": 1.5, "max_length": 8}, TypeError, "dim must be an integer"),
    ({"dim": 0, "max_length": 8}, ValueError, "dim must be positive"),
    ({"dim": 4, "max_length": True}, TypeError, "max_length must be an integer"),
    ({"dim": 4, "max_length": 1.5}, TypeError, "max_length must be an integer"),
    ({"dim": 4, "max_length": 0}, ValueError, "max_length must be positive"),
    ({"dim": 4, "max_length": 8, "base": True}, TypeError, "base must be a real number"),
    ({"dim": 4, "max_length": 8, "base": float("nan")}, ValueError, "base must be finite"),
    ({"dim": 4, "max_length": 8, "base": 0.0}, ValueError, "base must be positive"),
    ({"dim": 4, "max_length": 8, "rope_scale": "1.0"}, TypeError, "rope_scale must be a real number"),
    ({"dim": 4, "max_length": 8, "rope_scale": float("inf")}, ValueError, "rope_scale must be finite"),
    ({"dim": 4, "max_length": 8, "rope_scale": 0.5}, ValueError, "rope scale"),
    ({"dim": 4, "max_length": 8, "rotary_pct": np.bool_(True)}, TypeError, "rotary_pct must be a real number"),
    ({"dim": 4, "max_length": 8, "rotary_pct": float("nan")}, ValueError, "rotary_pct must be finite"),
    ({"dim": 4, "max_length": 8, "rotary_pct": 0.0}, ValueError, "rotary_pct must be in"),
    ({"dim": 4, "max_length": 8, "rotary_pct": 1.5}, ValueError, "rotary_pct must be in"),
    ({"dim": 4, "max_length": 8, "dtype": None}, TypeError, "dtype must be a valid"),
    ({"dim": 4, "max_length": 8, "dtype": "not-a-dtype"}, TypeError, "dtype must be a valid"),
    ({"dim": 4, "max_length": 8, "disable_cache": 1}, TypeError, "disable_cache must be a boolean"),
])
def test_field_checks(kwargs, exc, match):
    with pytest.raises(exc, match=match):
        RotaryEmbedding(**kwargs).init(0, X)


@pytest.mark.parametrize("disable_cache", [False, True])
def test_numpy_scalar_fields(disable_cache):
    rope = RotaryEmbedding(dim=np.int64(4), max_length=np.int64(8), base=np.float64(10000.0), dtype=np.float32,
                           disable_cache=np.bool_(disable_cache), rotary_pct=np.float64(1.0),
                           rope_scale=np.float64(1.0))
    v = rope.init(0, X, seq_len=np.int64(2))
    cos, sin = rope.apply(v, X, seq_len=np.int64(2))
    assert cos.dtype == torch.float32 and sin.dtype == torch.float32
    assert tuple(cos.shape) == ((2, 4) if disable_cache else (8, 4))


def test_seq_len_checks_and_uncached_tables():
    rope = RotaryEmbedding(dim=4, max_length=8)
    for bad in (True, np.bool_(True), 1.5):
        with pytest.raises(TypeError, match="seq_len must be an integer"):
            rope.init(0, X, seq_len=bad)
    rope = RotaryEmbedding(dim=4, max_length=4)
    v = rope.init(0, X, seq_len=2)
    with pytest.raises(ValueError, match="max_length=4"):
        rope.apply(v, X, seq_len=5)
    with pytest.raises(ValueError, match="max_length=4"):
        rope.init(0, X, seq_len=5)
    rope = RotaryEmbedding(dim=4, max_length=4, disable_cache=True)
    v = rope.init(0, X, seq_len=2)
    cos, sin = rope.apply(v, X, seq_len=5)
    assert tuple(cos.shape) == (5, 4) and tuple(sin.shape) == (5, 4)
    full = RotaryEmbedding(dim=4, max_length=8)
    c8, _ = full.apply(full.init(0, X), X)
    torch.testing.assert_close(cos, c8[:5])


@pytest.mark.parametrize("x,exc,match", [(torch.ones(2), ValueError, "batch and sequence axes"),
                                         (torch.ones(0, 2, 1, 4), ValueError, "empty axes"),
                                         (torch.ones(1, 0, 1, 4), ValueError, "empty axes"),
                                         (torch.ones(1, 2, 0, 4), ValueError, "empty axes"),
                                         (torch.ones(1, 2, 1, 4, dtype=torch.int32), TypeError,
                                          "x must contain floating point")])
def test_input_checks(x, exc, match):
    with pytest.raises(exc, match=match):
        RotaryEmbedding(dim=4, max_length=8).init(0, x)


@pytest.mark.parametrize("value", [float("nan"), float("inf"), -float("inf")])
def test_non_finite_input(value):
    x = X.clone()
    x[0, 0, 0, 0] = value
    with pytest.raises(ValueError, match="x must contain only finite values"):
        RotaryEmbedding(dim=4, max_length=8).init(0, x)


def _defaults():
    return {"q": torch.ones(1, 2, 2, 4), "k": torch.ones(1, 2, 1, 4), "cos": torch.ones(4, 4),
            "sin": torch.zeros(4, 4), "position_ids": torch.arange(2, dtype=torch.int32)[None]}


@pytest.mark.parametrize("kwargs,exc,match", [
    ({"q": torch.ones(1, 2, 4), "k": torch.ones(1, 2, 1, 4)}, ValueError, "q must be a 4D array"),
    ({"k": torch.ones(1, 2, 4)}, ValueError, "k must be a 4D array"),
    ({"q": torch.ones(0, 2, 2, 4)}, ValueError, "q must not contain empty axes"),
    ({"q": torch.ones(1, 2, 2, 0)}, ValueError, "q must not contain empty axes"),
    ({"k": torch.ones(1, 2, 0, 4)}, ValueError, "k must not contain empty axes"),
    ({"q": torch.ones(1, 2, 2, 4, dtype=torch.int32)}, TypeError, "q must contain floating point"),
    ({"k": torch.ones(1, 2, 1, 4, dtype=torch.int32)}, TypeError, "k must contain floating point"),
    ({"cos": torch.ones(4, 4, dtype=torch.int32)}, TypeError, "cos must contain floating point"),
    ({"sin": torch.ones(4, 4, dtype=torch.int32)}, TypeError, "sin must contain floating point"),
    ({"q": torch.ones(1, 3, 1, 4)}, ValueError, "matching batch, sequence"),
    ({"cos": torch.ones(4), "sin": torch.ones(4, 4)}, ValueError, "cos and sin must be 2D"),
    ({"cos": torch.ones(4, 4), "sin": torch.ones(5, 4)}, ValueError, "same shape"),
    ({"cos": torch.ones(0, 4), "sin": torch.ones(0, 4)}, ValueError, "at least one position"),
    ({"cos": torch.ones(4, 3), "sin": torch.ones(4, 3)}, ValueError, "positive and even"),
    ({"cos": torch.ones(4, 6), "sin": torch.ones(4, 6)}, ValueError, "cannot exceed"),
    ({"position_ids": torch.arange(2)}, ValueError, "position_ids must be a 2D array"),
    ({"position_ids": torch.arange(3, dtype=torch.int32)[None]}, ValueError, "position_ids shape must be broadcastable"),
    ({"position_ids": torch.arange(2, dtype=torch.float32)[None]}, TypeError, "integer positions"),
    ({"position_ids": torch.tensor([[-1, 0]], dtype=torch.int32)}, ValueError, "non-negative positions"),
    ({"position_ids": torch.tensor([[0, 4]], dtype=torch.int32)}, ValueError, "within rotary table length"),
])
def test_apply_rotary_pos_emb_checks(kwargs, exc, match):
    args = _defaults()
    args.update(kwargs)
    with pytest.raises(exc, match=match):
        RotaryEmbedding.apply_rotary_pos_emb(**args)


@pytest.mark.parametrize("value", [float("nan"), float("inf"), -float("inf")])
@pytest.mark.parametrize("field", ["q", "k", "cos", "sin"])
def test_apply_rotary_pos_emb_non_finite(field, value):
    args = _defaults()
    args[field][(0,) * args[field].ndim] = value
    with pytest.raises(ValueError, match=f"{field} must contain only finite values"):
        RotaryEmbedding.apply_rotary_pos_emb(**args)
