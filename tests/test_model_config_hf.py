"""``ModelConfig.from_hf`` (config.py:252-354 of the reference) on the architecture-specific fields: the
rope scaling factor, GPT-NeoX's rotary settings, Gemma3's sliding window and query scaling (the
reference's ``tests/test_config.py:337-581`` cases)."""
import numpy as np
import pytest

from jaxml_b200 import ModelConfig

transformers = pytest.importorskip("transformers")


def _llama(**kw):
    c = transformers.LlamaConfig(hidden_size=48, intermediate_size=144, num_hidden_layers=2,
                                 max_position_embeddings=256, vocab_size=1024, num_attention_heads=6,
                                 num_key_value_heads=3)
    for k, v in kw.items():
        object.__setattr__(c, k, v)
    return c


def _gemma(**kw):
    c = transformers.Gemma3TextConfig(hidden_size=48, head_dim=8, intermediate_size=144, num_hidden_layers=4,
                                      max_position_embeddings=256, vocab_size=1024, num_attention_heads=6,
                                      num_key_value_heads=3, sliding_window=32, sliding_window_pattern=2,
                                      rope_scaling={"factor": 8.0, "rope_type": "linear"})
    for k, v in kw.items():
        object.__setattr__(c, k, v)
    return c


@pytest.mark.parametrize("family,value,exc,match", [
    ("llama", True, TypeError, "num_key_value_heads must be an integer"),
    ("llama", 0, ValueError, "num_key_value_heads must be positive"),
    ("gemma", np.bool_(True), TypeError, "num_key_value_heads must be an integer"),
    ("gemma", 0, ValueError, "num_key_value_heads must be positive"),
])
def test_invalid_key_value_head_count(family, value, exc, match):
    c = _llama(head_dim=8) if family == "llama" else _gemma()
    object.__setattr__(c, "num_key_value_heads", value)
    with pytest.raises(exc, match=match):
        ModelConfig.from_hf(c)


def test_integer_like_rope_scaling_factor():
    c = _llama()
    c.__dict__["rope_parameters"] = {"factor": np.float64(2.0), "rope_theta": 10000.0, "rope_type": "linear"}
    assert ModelConfig.from_hf(c).rope_scale == 2.0


@pytest.mark.parametrize("rope,exc,match", [
    ({"rope_type": "linear"}, ValueError, "rope_scaling must include a factor"),
    ("linear", TypeError, "rope_parameters must be a mapping"),
    ({"factor": True}, TypeError, "rope_scaling factor must be a real number"),
    ({"factor": float("nan")}, ValueError, "rope_scaling factor must be finite"),
    ({"factor": 0.5}, ValueError, "rope_scale must be greater than or equal to 1.0"),
])
def test_invalid_rope_scaling_factor(rope, exc, match):
    c = _llama()
    c.__dict__["rope_parameters"] = ({"rope_theta": 10000.0} | rope) if isinstance(rope, dict) else rope
    with pytest.raises(exc, match=match):
        ModelConfig.from_hf(c)


def test_neox_fields():
    c = transformers.GPTNeoXConfig(hidden_size=48, intermediate_size=144, num_hidden_layers=2,
                                   max_position_embeddings=256, vocab_size=1024, num_attention_heads=6,
                                   rotary_emb_base=12345.0, rotary_pct=0.5, use_parallel_residual=False,
                                   attention_bias=True)
    cfg = ModelConfig.from_hf(c)
    assert cfg.num_key_value_heads == 6 and cfg.rope_theta == 12345.0 and cfg.rotary_pct == 0.5
    assert cfg.use_parallel_residual is False and cfg.use_bias is True


@pytest.mark.parametrize("hidden,pct,match", [(6, 0.5, "positive rotary dimension"), (18, 1.0, "even rotary dimension")])
def test_neox_invalid_rotary_dimension(hidden, pct, match):
    c = transformers.GPTNeoXConfig(hidden_size=hidden, intermediate_size=hidden * 3, num_hidden_layers=2,
                                   max_position_embeddings=256, vocab_size=1024, num_attention_heads=6,
                                   rotary_emb_base=12345.0, rotary_pct=pct)
    with pytest.raises(ValueError, match=match):
        ModelConfig.from_hf(c)


def test_gemma_fields():
    c = _gemma()
    cfg = ModelConfig.from_hf(c)
    assert (cfg.hidden_size, cfg.head_dim, cfg.num_key_value_heads) == (48, 8, 3)
    assert cfg.rope_scale == 8.0 and cfg.sliding_window == 32 and cfg.sliding_window_pattern == 2
    assert cfg.attn_scale == c.query_pre_attn_scalar ** -0.5


def test_gemma_sliding_window_pair():
    with pytest.raises(TypeError, match="sliding_window_pattern must be an integer"):
        ModelConfig.from_hf(_gemma(sliding_window_pattern=True))
    with pytest.raises(ValueError, match="sliding_window and sliding_window_pattern"):
        ModelConfig.from_hf(_gemma(sliding_window_pattern=None))


@pytest.mark.parametrize("value,exc,match", [(True, TypeError, "query_pre_attn_scalar must be a real number"),
                                             (float("nan"), ValueError, "query_pre_attn_scalar must be finite"),
                                             (0.0, ValueError, "query_pre_attn_scalar must be positive"),
                                             (-1.0, ValueError, "query_pre_attn_scalar must be positive")])
def test_gemma_invalid_query_pre_attn_scalar(value, exc, match):
    with pytest.raises(exc, match=match):
        ModelConfig.from_hf(_gemma(query_pre_attn_scalar=value))
