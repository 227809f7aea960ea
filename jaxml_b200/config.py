"""``ModelConfig``: the model shape description, same fields, defaults and checks as the reference.

Mirrors ``config.py:125-250`` (dataclass + ``__post_init__`` validation, ``num_key_value_heads`` and
``intermediate_size`` properties) and ``config.py:252-354`` (``from_hf`` for Llama / GPT-NeoX / Gemma3).
"""
from __future__ import annotations

import dataclasses
import math
from collections.abc import Mapping
from dataclasses import dataclass, fields
from typing import Optional

from ._checks import normalize_bool, normalize_count, normalize_float


@dataclass(frozen=True)
class ModelConfig:
    head_dim: int
    hidden_size: int
    num_heads: int
    num_layers: int
    max_position_embeddings: int
    vocab_size: int
    intermediate_ratio: tuple = (8, 3)
    norm_eps: float = 1e-6
    num_kv_heads: Optional[int] = None
    sliding_window: Optional[int] = None
    sliding_window_pattern: Optional[int] = None
    attn_scale: Optional[float] = None
    use_bias: bool = False
    use_alibi: bool = False
    use_rope: bool = True
    upcast_alibi: bool = True
    rope_theta: float = 10_000.0
    rope_scale: float = 1.0
    rotary_pct: float = 1.0
    use_parallel_residual: bool = True

    def __post_init__(self):
        def put(name, value):
            object.__setattr__(self, name, value)

        for name in ("use_bias", "use_alibi", "use_rope", "upcast_alibi", "use_parallel_residual"):
            put(name, normalize_bool(name, getattr(self, name)))
        for name in ("head_dim", "hidden_size", "num_heads", "num_layers", "max_position_embeddings", "vocab_size"):
            value = normalize_count(name, getattr(self, name))
            put(name, value)
            if value <= 0:
                raise ValueError(f"{name} must be positive, got {value}.")
        ratio = self.intermediate_ratio
        if not hasattr(ratio, "__len__") or len(ratio) != 2:
            raise ValueError(f"intermediate_ratio must contain numerator and denominator, got {ratio}.")
        ratio = (normalize_count("intermediate_ratio numerator", ratio[0]),
                 normalize_count("intermediate_ratio denominator", ratio[1]))
        put("intermediate_ratio", ratio)
        if ratio[0] <= 0 or ratio[1] <= 0:
            raise ValueError(f"intermediate_ratio values must be positive, got {ratio}.")
        if self.hidden_size * ratio[0] // ratio[1] <= 0:
            raise ValueError(f"intermediate_ratio must produce a positive intermediate_size, got {ratio}.")
        for name in ("norm_eps", "rope_theta", "rope_scale", "rotary_pct"):
            put(name, normalize_float(name, getattr(self, name)))
        if self.norm_eps <= 0:
            raise ValueError(f"norm_eps must be positive, got {self.norm_eps}.")
        if self.num_kv_heads is not None:
            put("num_kv_heads", normalize_count("num_kv_heads", self.num_kv_heads))
        if self.num_key_value_heads <= 0:
            raise ValueError(f"num_key_value_heads must be positive, got {self.num_key_value_heads}.")
        if self.num_heads % self.num_key_value_heads != 0:
            raise ValueError(
                "num_heads must be divisible by num_key_value_heads, "
                f"got {self.num_heads} and {self.num_key_value_heads}."
            )
        if self.sliding_window is not None:
            put("sliding_window", normalize_count("sliding_window", self.sliding_window))
            if self.sliding_window <= 0:
                raise ValueError(f"sliding_window must be positive when set, got {self.sliding_window}.")
        if self.sliding_window_pattern is not None:
            put("sliding_window_pattern", normalize_count("sliding_window_pattern", self.sliding_window_pattern))
        if (self.sliding_window is None) != (self.sliding_window_pattern is None):
            raise ValueError("sliding_window and sliding_window_pattern must both be set or both be None.")
        if self.sliding_window_pattern is not None and self.sliding_window_pattern <= 0:
            raise ValueError(f"sliding_window_pattern must be positive when set, got {self.sliding_window_pattern}.")
        if self.attn_scale is None:
            put("attn_scale", self.head_dim ** -0.5)
        else:
            put("attn_scale", normalize_float("attn_scale", self.attn_scale))
            if self.attn_scale <= 0:
                raise ValueError(f"attn_scale must be positive, got {self.attn_scale}.")
        if self.use_alibi and self.use_rope:
            raise ValueError("AliBi and RoPE cannot both be used.")
        if self.rope_theta <= 0:
            raise ValueError(f"rope_theta must be positive, got {self.rope_theta}.")
        if self.rope_scale < 1.0:
            raise ValueError(f"rope_scale must be greater than or equal to 1.0, got {self.rope_scale}.")
        if not 0 < self.rotary_pct <= 1:
            raise ValueError(f"rotary_pct must be in (0, 1], got {self.rotary_pct}.")

    def replace(self, **kwargs):
        args = {f.name: getattr(self, f.name) for f in fields(self)} | kwargs
        return self.__class__(**args)

    @property
    def num_key_value_heads(self) -> int:
        return self.num_heads if self.num_kv_heads is None else self.num_kv_heads

    @property
    def intermediate_size(self) -> int:
        return self.hidden_size * self.intermediate_ratio[0] // self.intermediate_ratio[1]

    @property
    def rotary_dim(self) -> int:
        return self.head_dim if self.rotary_pct >= 1.0 else int(self.head_dim * self.rotary_pct)

    @classmethod
    def from_hf(cls, config) -> "ModelConfig":
        """Llama / GPT-NeoX / Gemma3 HF configs (``config.py:252-354``)."""
        from transformers import Gemma3TextConfig, GPTNeoXConfig, LlamaConfig

        if isinstance(config, LlamaConfig):
            kind = "llama"
        elif isinstance(config, GPTNeoXConfig):
            kind = "gpt_neox"
        elif isinstance(config, Gemma3TextConfig):
            kind = "gemma3"
        else:
            raise ValueError(f"Unsupported config class {config.__class__}")
        # shared fields, validated under their HF names before anything is derived from them
        hidden = _hf_count("hidden_size", config.hidden_size)
        inter = _hf_count("intermediate_size", config.intermediate_size)
        factor = math.gcd(inter, hidden)
        head_dim = getattr(config, "head_dim", None)
        if head_dim is not None:
            head_dim = _hf_count("head_dim", head_dim)
        else:
            heads = _hf_count("num_attention_heads", config.num_attention_heads)
            if hidden % heads:
                raise ValueError("hidden_size must be divisible by num_attention_heads when head_dim is not set.")
            head_dim = hidden // heads
        num_heads = _hf_count("num_attention_heads", config.num_attention_heads)
        num_layers = _hf_count("num_hidden_layers", config.num_hidden_layers)
        max_pos = _hf_count("max_position_embeddings", config.max_position_embeddings)
        vocab = _hf_count("vocab_size", config.vocab_size)
        attn_scale = head_dim ** -0.5
        kw = dict(use_parallel_residual=True, rotary_pct=1.0, use_bias=False, sliding_window=None,
                  sliding_window_pattern=None)
        if kind == "llama":
            norm_eps = config.rms_norm_eps
            num_kv = _hf_count("num_key_value_heads", config.num_key_value_heads)
            rope_theta = _hf_rope_theta(config)
            rope_scale = _hf_rope_scale(config)
        elif kind == "gpt_neox":
            norm_eps = config.layer_norm_eps
            num_kv = num_heads
            rope_theta = _hf_rope_theta(config, fallback="rotary_emb_base")
            rope_scale = 1.0     # GPT-NeoX configs carry no position scaling
            kw.update(use_parallel_residual=config.use_parallel_residual, rotary_pct=_hf_rotary_pct(config),
                      use_bias=True)
        else:
            qpas = normalize_float("query_pre_attn_scalar", config.query_pre_attn_scalar)
            if qpas <= 0:
                raise ValueError(f"query_pre_attn_scalar must be positive, got {qpas}.")
            attn_scale = qpas ** -0.5
            norm_eps = config.rms_norm_eps
            num_kv = _hf_count("num_key_value_heads", config.num_key_value_heads)
            rope_theta = _hf_rope_theta(config, kind="full_attention")
            rope_scale = _hf_rope_scale(config, kind="full_attention")
            kw.update(sliding_window=config.sliding_window, sliding_window_pattern=_gemma_pattern(config))
        pct = kw["rotary_pct"]
        rd = head_dim if pct >= 1.0 else int(head_dim * pct)
        if rd <= 0:
            raise ValueError(f"rotary_pct must produce a positive rotary dimension, got rotary_pct={pct} and "
                             f"head_dim={head_dim}.")
        if rd % 2:
            raise ValueError(f"rotary_pct must produce an even rotary dimension, got rotary_dim={rd}, "
                             f"rotary_pct={pct}, and head_dim={head_dim}.")
        return cls(hidden_size=hidden, head_dim=head_dim, num_heads=num_heads,
                   num_layers=num_layers, max_position_embeddings=max_pos,
                   vocab_size=vocab, intermediate_ratio=(inter // factor, hidden // factor),
                   norm_eps=norm_eps, num_kv_heads=num_kv, use_rope=True, rope_theta=rope_theta,
                   rope_scale=rope_scale, attn_scale=attn_scale, **kw)


def _hf_count(name: str, value) -> int:
    value = normalize_count(name, value)
    if value <= 0:
        raise ValueError(f"{name} must be positive, got {value}.")
    return value


def _hf_rope_parameters(config, kind=None):
    """The config's ``rope_parameters`` (for Gemma3, the entry of one attention kind), or {}."""
    rp = getattr(config, "rope_parameters", None)
    if rp is None:
        return {}
    if not isinstance(rp, Mapping):
        raise TypeError(f"rope_parameters must be a mapping when set, got {type(rp)}.")
    if kind is None:
        return rp
    sub = rp.get(kind, {})
    if not isinstance(sub, Mapping):
        raise TypeError(f"rope_parameters[{kind!r}] must be a mapping when set, got {type(sub)}.")
    return sub


def _hf_rope_theta(config, fallback: str = "rope_theta", kind=None) -> float:
    rp = _hf_rope_parameters(config, kind)
    if "rope_theta" in rp:
        return normalize_float("rope_theta", rp["rope_theta"])
    if not hasattr(config, fallback):
        raise ValueError(f"{config.__class__.__name__} must expose rope_theta.")
    return normalize_float("rope_theta", getattr(config, fallback))


def _hf_rope_scale(config, kind=None) -> float:
    """The position divisor: the ``factor`` of ``rope_scaling`` (or of ``rope_parameters``), else 1."""
    rs = getattr(config, "rope_scaling", None)
    if rs is not None and not isinstance(rs, Mapping):
        raise TypeError(f"rope_scaling must be a mapping when set, got {type(rs)}.")
    if isinstance(rs, Mapping):
        sub = rs
        if kind is not None and kind in rs:
            sub = rs[kind]
            if not isinstance(sub, Mapping):
                raise TypeError(f"rope_scaling[{kind!r}] must be a mapping when set, got {type(sub)}.")
        if "factor" in sub:
            return normalize_float("rope_scaling factor", sub["factor"])
        if sub.get("rope_type") not in (None, "default"):
            raise ValueError("rope_scaling must include a factor when set.")
    rp = _hf_rope_parameters(config, kind)
    if "factor" in rp:
        return normalize_float("rope_parameters factor", rp["factor"])
    return 1.0


def _hf_rotary_pct(config) -> float:
    v = getattr(config, "rotary_pct", None)
    if v is not None:
        return normalize_float("rotary_pct", v)
    rp = _hf_rope_parameters(config)
    if "partial_rotary_factor" in rp:
        return normalize_float("rotary_pct", rp["partial_rotary_factor"])
    return 1.0


def _gemma_pattern(config):
    """``sliding_window_pattern`` as the config states it; configs without the attribute give it through
    ``layer_types`` (the first full-attention layer's index + 1)."""
    if hasattr(config, "sliding_window_pattern"):
        return config.sliding_window_pattern
    types = getattr(config, "layer_types", None)
    if types:
        for i, t in enumerate(types):
            if t == "full_attention":
                return i + 1
    return None


__all__ = ["ModelConfig", "dataclasses"]
