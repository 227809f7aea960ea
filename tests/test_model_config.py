"""ModelConfig validation and normalisation: the reference's ``tests/test_config.py`` cases against
``jaxml_b200.config.ModelConfig`` (CPU only)."""
import numpy as np
import pytest

from jaxml_b200.config import ModelConfig


def _kw(**overrides):
    return {"hidden_size": 48, "head_dim": 8, "num_heads": 6, "num_layers": 2, "max_position_embeddings": 256,
            "vocab_size": 1024, "use_rope": False} | overrides


def test_defaults_and_numpy_normalisation():
    assert ModelConfig(**_kw()).attn_scale == 8 ** -0.5
    c = ModelConfig(**_kw(hidden_size=np.int64(48), intermediate_ratio=(np.int64(3), np.int64(1)),
                          num_kv_heads=np.int64(3), sliding_window=np.int64(32), sliding_window_pattern=np.int64(2)))
    assert (c.hidden_size, c.intermediate_ratio, c.num_kv_heads, c.sliding_window, c.sliding_window_pattern) == \
        (48, (3, 1), 3, 32, 2)
    c = ModelConfig(**_kw(use_bias=np.bool_(True), use_alibi=np.bool_(False), use_rope=np.bool_(True),
                          upcast_alibi=np.bool_(False), use_parallel_residual=np.bool_(False)))
    assert (c.use_bias, c.use_alibi, c.use_rope, c.upcast_alibi, c.use_parallel_residual) == \
        (True, False, True, False, False)
    c = ModelConfig(**_kw(norm_eps=np.float32(1e-5), attn_scale=np.float64(0.25), rope_theta=np.float64(5000.0),
                          rope_scale=np.float32(2.0), rotary_pct=np.float64(0.5)))
    assert c.norm_eps == pytest.approx(1e-5) and (c.attn_scale, c.rope_theta, c.rope_scale, c.rotary_pct) == \
        (0.25, 5000.0, 2.0, 0.5)
    assert ModelConfig(**_kw(head_dim=3, hidden_size=18, num_heads=6, use_rope=True)).head_dim == 3


@pytest.mark.parametrize("overrides,match", [
    ({"hidden_size": 48.0}, "hidden_size must be an integer"),
    ({"head_dim": True}, "head_dim must be an integer"),
    ({"head_dim": np.bool_(True)}, "head_dim must be an integer"),
    ({"intermediate_ratio": (8.0, 3)}, "intermediate_ratio numerator must be an integer"),
    ({"intermediate_ratio": (8, False)}, "intermediate_ratio denominator must be an integer"),
    ({"num_kv_heads": 3.0}, "num_kv_heads must be an integer"),
    ({"num_kv_heads": np.bool_(True)}, "num_kv_heads must be an integer"),
    ({"sliding_window": 32.0}, "sliding_window must be an integer"),
    ({"sliding_window_pattern": np.bool_(True)}, "sliding_window_pattern must be an integer"),
])
def test_non_integer_counts(overrides, match):
    with pytest.raises(TypeError, match=match):
        ModelConfig(**_kw(**overrides))


@pytest.mark.parametrize("overrides,exc,match", [
    ({"norm_eps": True}, TypeError, "norm_eps must be a real number"),
    ({"attn_scale": "0.5"}, TypeError, "attn_scale must be a real number"),
    ({"rope_theta": np.bool_(True)}, TypeError, "rope_theta must be a real number"),
    ({"rope_scale": float("nan")}, ValueError, "rope_scale must be finite"),
    ({"rotary_pct": float("inf")}, ValueError, "rotary_pct must be finite"),
    ({"attn_scale": -float("inf")}, ValueError, "attn_scale must be finite"),
])
def test_invalid_float_fields(overrides, exc, match):
    with pytest.raises(exc, match=match):
        ModelConfig(**_kw(**overrides))


@pytest.mark.parametrize("field", ["use_bias", "use_alibi", "use_rope", "upcast_alibi", "use_parallel_residual"])
def test_non_boolean_flags(field):
    with pytest.raises(TypeError, match=f"{field} must be a boolean"):
        ModelConfig(**_kw(**{field: 1}))


@pytest.mark.parametrize("overrides,match", [
    ({"hidden_size": 0}, "hidden_size"), ({"head_dim": 0}, "head_dim"), ({"num_heads": 0}, "num_heads"),
    ({"num_layers": 0}, "num_layers"), ({"max_position_embeddings": 0}, "max_position_embeddings"),
    ({"vocab_size": 0}, "vocab_size"), ({"intermediate_ratio": (8, 0)}, "intermediate_ratio"),
    ({"intermediate_ratio": (8, 3, 1)}, "intermediate_ratio"),
    ({"intermediate_ratio": (1, 100)}, "positive intermediate_size"), ({"norm_eps": 0.0}, "norm_eps"),
    ({"num_kv_heads": 0}, "num_key_value_heads"), ({"num_kv_heads": 4}, "divisible"),
    ({"sliding_window": 0}, "sliding_window"), ({"sliding_window_pattern": 0}, "sliding_window_pattern"),
    ({"sliding_window": 32}, "sliding_window and sliding_window_pattern"),
    ({"sliding_window_pattern": 2}, "sliding_window and sliding_window_pattern"),
    ({"attn_scale": 0.0}, "attn_scale"), ({"use_alibi": True, "use_rope": True}, "AliBi and RoPE"),
    ({"rope_theta": 0.0}, "rope_theta"), ({"rope_scale": 0.5}, "rope_scale"),
    ({"rotary_pct": 0.0}, "rotary_pct"), ({"rotary_pct": 1.5}, "rotary_pct"),
])
def test_invalid_invariants(overrides, match):
    with pytest.raises(ValueError, match=match):
        ModelConfig(**_kw(**overrides))


# ---- ModelConfig.from_hf (the reference's from_hf cases; transformers configs only, no weights) ----
def _llama_hf(**kw):
    from transformers import LlamaConfig

    return LlamaConfig(**({"hidden_size": 48, "intermediate_size": 144, "num_hidden_layers": 2,
                           "max_position_embeddings": 256, "vocab_size": 1024, "num_attention_heads": 6,
                           "num_key_value_heads": 3} | kw))


def test_from_hf_llama_subclass_and_fields():
    from transformers import LlamaConfig

    class CustomLlamaConfig(LlamaConfig):
        pass

    hf = CustomLlamaConfig(hidden_size=48, intermediate_size=144, num_hidden_layers=2, max_position_embeddings=256,
                           vocab_size=1024, num_attention_heads=6, num_key_value_heads=3, rope_theta=5000.0,
                           rms_norm_eps=1e-5)
    c = ModelConfig.from_hf(hf)
    assert (c.hidden_size, c.head_dim, c.num_heads, c.num_key_value_heads, c.intermediate_size) == (48, 8, 6, 3, 144)
    assert c.rope_theta == 5000.0 and c.norm_eps == 1e-5
    hf = _llama_hf()
    object.__setattr__(hf, "head_dim", np.int64(8))
    assert ModelConfig.from_hf(hf).head_dim == 8


@pytest.mark.parametrize("head_dim,exc,match", [(0, ValueError, "head_dim must be positive"),
                                                (-1, ValueError, "head_dim must be positive"),
                                                (True, TypeError, "head_dim must be an integer"),
                                                (1.5, TypeError, "head_dim must be an integer")])
def test_from_hf_invalid_head_dim(head_dim, exc, match):
    hf = _llama_hf()
    object.__setattr__(hf, "head_dim", head_dim)
    with pytest.raises(exc, match=match):
        ModelConfig.from_hf(hf)


def test_from_hf_non_divisible_head_dim_fallback():
    hf = _llama_hf()
    object.__setattr__(hf, "hidden_size", 50)
    object.__setattr__(hf, "intermediate_size", 150)
    object.__setattr__(hf, "head_dim", None)
    with pytest.raises(ValueError, match="hidden_size must be divisible"):
        ModelConfig.from_hf(hf)


@pytest.mark.parametrize("field,value,exc,match", [
    ("hidden_size", True, TypeError, "hidden_size must be an integer"),
    ("hidden_size", 0, ValueError, "hidden_size must be positive"),
    ("intermediate_size", np.bool_(True), TypeError, "intermediate_size must be an integer"),
    ("intermediate_size", 0, ValueError, "intermediate_size must be positive"),
    ("num_attention_heads", True, TypeError, "num_attention_heads must be an integer"),
    ("num_attention_heads", 0, ValueError, "num_attention_heads must be positive"),
    ("num_hidden_layers", np.bool_(True), TypeError, "num_hidden_layers must be an integer"),
    ("num_hidden_layers", 0, ValueError, "num_hidden_layers must be positive"),
    ("max_position_embeddings", 1.5, TypeError, "max_position_embeddings must be an integer"),
    ("max_position_embeddings", 0, ValueError, "max_position_embeddings must be positive"),
    ("vocab_size", "1024", TypeError, "vocab_size must be an integer"),
    ("vocab_size", 0, ValueError, "vocab_size must be positive"),
    ("num_key_value_heads", True, TypeError, "num_key_value_heads must be an integer"),
    ("num_key_value_heads", 0, ValueError, "num_key_value_heads must be positive"),
])
def test_from_hf_invalid_fields(field, value, exc, match):
    hf = _llama_hf()
    object.__setattr__(hf, "head_dim", 8)
    object.__setattr__(hf, field, value)
    with pytest.raises(exc, match=match):
        ModelConfig.from_hf(hf)


def test_from_hf_unsupported_config():
    with pytest.raises(ValueError, match="Unsupported config class"):
        ModelConfig.from_hf(object())
