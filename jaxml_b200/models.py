"""Model classes with the reference's names: ``LlamaModelWithHead``, ``GPTNeoXModelWithHead``,
``GemmaModelWithHead`` (models/llama.py:228-273, models/gpt_neox.py:225-272, models/gemma3.py:286-331).

They describe the architecture (``config`` + compute ``dtype``) the way a Flax module does before it is
bound to parameters; ``Engine`` packs the parameter tree for the GPU kernels.  ``init`` returns a
random parameter tree in the reference's Flax layout.
"""
from __future__ import annotations

import torch

from ._checks import normalize_dtype
from .config import ModelConfig


class _DecoderWithHead:
    family = ""

    def __init__(self, config: ModelConfig, dtype=torch.float32):
        if not isinstance(config, ModelConfig):
            raise TypeError(f"config must be a ModelConfig, got {type(config)}.")
        if self.family != "gemma3" and config.hidden_size != config.num_heads * config.head_dim:
            name = {"llama": "Llama", "neox": "GPT-NeoX"}[self.family]
            raise ValueError(
                f"{name} hidden_size must equal num_heads * head_dim; got hidden_size={config.hidden_size}, "
                f"num_heads={config.num_heads}, head_dim={config.head_dim}."
            )
        if self.family == "neox" and config.num_heads != config.num_key_value_heads:
            raise ValueError(
                "fused_qkv requires num_heads to equal num_key_value_heads, "
                f"got {config.num_heads} and {config.num_key_value_heads}."
            )
        self.config = config
        self.dtype = normalize_dtype("dtype", dtype)

    # Block properties of the reference (nn/module.py:55-91)
    @property
    def num_layers(self) -> int:
        return self.config.num_layers

    @property
    def head_dim(self) -> int:
        return self.config.head_dim

    @property
    def hidden_size(self) -> int:
        return self.config.hidden_size

    @property
    def num_heads(self) -> int:
        return self.config.num_heads

    def init(self, seed: int = 0, *_, std: float = 0.02) -> dict:
        """Random N(0, std) kernels, unit norm weights, in the reference's parameter layout."""
        return random_params(self.family, self.config, seed=seed, std=std)

    def __repr__(self) -> str:
        return f"{type(self).__name__}(config={self.config!r}, dtype={self.dtype})"


class LlamaModelWithHead(_DecoderWithHead):
    family = "llama"


class GPTNeoXModelWithHead(_DecoderWithHead):
    family = "neox"


class GemmaModelWithHead(_DecoderWithHead):
    family = "gemma3"


def random_params(family: str, cfg: ModelConfig, seed: int = 0, std: float = 0.02, dtype=torch.float32,
                  device="cpu") -> dict:
    """Parameter tree with N(0, std) kernels (Appendix-B names of the reference's Flax modules)."""
    g = torch.Generator(device=device).manual_seed(seed)
    d, H, Hkv, hd, V, F = (cfg.hidden_size, cfg.num_heads, cfg.num_key_value_heads, cfg.head_dim, cfg.vocab_size,
                           cfg.intermediate_size)

    def rnd(*shape):
        return (torch.randn(*shape, generator=g, device=device, dtype=torch.float32) * std).to(dtype)

    def norm(bias=False, gemma=False):
        p = {"weight": rnd(d) if gemma else torch.ones(d, dtype=dtype, device=device)}
        if bias:
            p["bias"] = rnd(d)
        return p

    layers = {}
    for i in range(cfg.num_layers):
        if family == "neox":
            lp = {"self_attn": {"qkv_proj": {"kernel": rnd(d, 3, H, hd), "bias": rnd(3, H, hd)},
                                "o_proj": {"kernel": rnd(H * hd, d), "bias": rnd(d)}},
                  "mlp": {"up_proj": {"kernel": rnd(d, F), "bias": rnd(F)},
                          "down_proj": {"kernel": rnd(F, d), "bias": rnd(d)}},
                  "input_layernorm": norm(True), "post_attention_layernorm": norm(True)}
        else:
            gm = family == "gemma3"
            sa = {"q_proj": {"kernel": rnd(d, H, hd)}, "k_proj": {"kernel": rnd(d, Hkv, hd)},
                  "v_proj": {"kernel": rnd(d, Hkv, hd)}, "o_proj": {"kernel": rnd(H * hd, d)}}
            if gm:
                sa["q_norm"] = {"weight": rnd(hd)}
                sa["k_norm"] = {"weight": rnd(hd)}
            lp = {"self_attn": sa,
                  "mlp": {"gate_proj": {"kernel": rnd(d, F)}, "up_proj": {"kernel": rnd(d, F)},
                          "down_proj": {"kernel": rnd(F, d)}},
                  "input_layernorm": norm(gemma=gm), "post_attention_layernorm": norm(gemma=gm)}
            if gm:
                lp["pre_feedforward_layernorm"] = norm(gemma=True)
                lp["post_feedforward_layernorm"] = norm(gemma=True)
        layers[f"layers_{i}"] = lp
    body = {"embed_tokens": {"embedding": rnd(V, d)}, "norm": norm(family == "neox", family == "gemma3"), **layers}
    return {"params": {"gpt_neox" if family == "neox" else "model": body, "lm_head": {"kernel": rnd(d, V)}}}
