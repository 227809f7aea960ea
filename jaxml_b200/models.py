"""Model classes with the reference's names: ``LlamaModelWithHead``, ``GPTNeoXModelWithHead``,
``GemmaModelWithHead`` (models/llama.py:228-273, models/gpt_neox.py:225-272, models/gemma3.py:286-331).

They describe the architecture (``config`` + compute ``dtype``) the way a Flax module does before it is
bound to parameters; ``Engine`` packs the parameter tree for the GPU kernels.  ``init`` returns a
random parameter tree in the reference's Flax layout.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

from ._checks import normalize_dtype
from .config import ModelConfig
from .nn import GemmaRMSNorm  # noqa: F401  (models/gemma3.py:89-106 lives in jaxml.models)


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

    def apply(self, params, input_ids, attention_mask=None, position_ids=None, kv_caches=None, use_cache=False,
              output_attentions=False, output_hidden_states=False, keep_last_n_logits: int = 0):
        """``*ModelWithHead.__call__`` (models/llama.py:247-273, gpt_neox.py:245-272, gemma3.py:304-331)
        on the GPU kernels for a cache-free forward: logits ``[B, S]`` (or the last ``keep_last_n_logits``
        positions) in the model dtype, in a ``CausalLMOutputWithCache``.  Right-padded masks; token ids
        below 0 read row 0 like the reference.  Cached decoding, position ids, per-layer hidden states
        and attention weights are the Engine's business here and raise ``NotImplementedError``."""
        import numpy as np

        from ._checks import normalize_bool, normalize_count

        use_cache = normalize_bool("use_cache", use_cache)
        output_attentions = normalize_bool("output_attentions", output_attentions)
        output_hidden_states = normalize_bool("output_hidden_states", output_hidden_states)
        keep = normalize_count("keep_last_n_logits", keep_last_n_logits)
        if keep < 0:
            raise ValueError(f"keep_last_n_logits must be non-negative, got {keep}.")
        if kv_caches is not None or use_cache or position_ids is not None:
            raise NotImplementedError("apply with KV caches or position ids: use Engine.generate for cached decoding.")
        if output_attentions or output_hidden_states:
            raise NotImplementedError("apply does not return attention weights or per-layer hidden states.")
        ids, mask = _check_model_inputs(self.config, input_ids, attention_mask)
        B, S = ids.shape
        rt = self._runtime(params, B, S)
        dev = rt.w.device
        logits = rt.forward_logits(ids.to(dev), mask.to(dev), keep)
        return CausalLMOutputWithCache(logits=logits)

    def _full_tree(self, params):
        """The parameter tree the runtime packs (the with-head layout)."""
        return params

    def _runtime(self, params, B: int, S: int):
        """Packed weights (cached per parameter tree) and a runtime sized for B rows of S tokens."""
        from .runtime import DecoderRuntime, ModelWeights

        dev = torch.device("cuda", torch.cuda.current_device())
        cache = self.__dict__.setdefault("_apply_cache", {})
        key = (id(params), dev.index)
        if cache.get("key") != key:
            cache.clear()
            cache["key"] = key
            cache["params"] = params   # keeps the tree alive while its id is the cache key
            cache["weights"] = ModelWeights(self.family, self.config, self._full_tree(params), self.dtype, dev)
        T = ((S + 255) // 256) * 256
        rt = cache.get("rt")
        if rt is None or rt.B != B or rt.T < T:
            cache["rt"] = rt = DecoderRuntime(cache["weights"], B, T)
        return rt

    def __repr__(self) -> str:
        return f"{type(self).__name__}(config={self.config!r}, dtype={self.dtype})"


def _check_model_inputs(config, input_ids, attention_mask):
    """input_ids / attention_mask checks of models/_utils.py:78-177 (same messages); returns int32 ids with
    negative placeholders mapped to row 0 and the boolean mask.  Raised before any device work."""
    import numpy as np

    ids = input_ids if isinstance(input_ids, torch.Tensor) else torch.as_tensor(np.asarray(input_ids))
    if ids.ndim != 2:
        raise ValueError(f"input_ids must be a 2D array, got shape {tuple(ids.shape)}.")
    if ids.is_floating_point() or ids.is_complex() or ids.dtype == torch.bool:
        raise TypeError(f"input_ids must contain integer token ids, got dtype {ids.dtype}.")
    if ids.shape[0] == 0:
        raise ValueError("input_ids must contain at least one batch row.")
    if ids.shape[1] == 0:
        raise ValueError("input_ids must contain at least one token.")
    if bool((ids >= config.vocab_size).any()):
        raise ValueError(f"input_ids token ids must be less than vocab_size={config.vocab_size}.")
    B, S = ids.shape
    if attention_mask is None:
        # negative ids are placeholders: masked out by default
        mask = ids >= 0
        if not bool(mask.any(dim=1).all()):
            raise ValueError("input_ids must contain at least one non-negative token per batch row when "
                             "attention_mask is None.")
    else:
        mask = attention_mask if isinstance(attention_mask, torch.Tensor) else torch.as_tensor(
            np.asarray(attention_mask))
        if mask.ndim != 2:
            raise ValueError(f"attention_mask must be a 2D array, got shape {tuple(mask.shape)}.")
        if tuple(mask.shape) != (B, S):
            raise ValueError(f"attention_mask shape must match input_ids, got {tuple(mask.shape)} and {(B, S)}.")
        if mask.is_floating_point() or mask.is_complex():
            raise TypeError(f"attention_mask must be boolean or integer, got dtype {mask.dtype}.")
        if mask.dtype != torch.bool and bool(((mask != 0) & (mask != 1)).any()):
            raise ValueError("attention_mask integer values must be 0 or 1.")
        mask = mask.to(torch.bool)
        if not bool(mask.any(dim=1).all()):
            raise ValueError("attention_mask must contain at least one valid token per batch row.")
        if bool((mask & (ids < 0)).any()):
            raise ValueError("attention_mask must not mark negative placeholder token ids as valid.")
    ids = torch.where(ids < 0, torch.zeros_like(ids), ids).to(torch.int32)
    if S > 1 and bool((mask[:, :-1].to(torch.int8) < mask[:, 1:].to(torch.int8)).any()):
        raise NotImplementedError("apply takes right-padded attention masks (the kernels attend to key prefixes).")
    return ids, mask


@dataclass
class CausalLMOutputWithCache:
    """``outputs.py``: logits, and (not produced by ``apply`` here) caches, hidden states, weights."""

    logits: torch.Tensor
    kv_caches: Optional[tuple] = None
    hidden_states: Optional[tuple] = None
    attention_weights: Optional[tuple] = None


@dataclass
class BaseModelOutputWithCache:
    """``outputs.py``: the decoder stack's final hidden states (and, not produced here, caches etc.)."""

    last_hidden_state: torch.Tensor
    kv_caches: Optional[tuple] = None
    hidden_states: Optional[tuple] = None
    attention_weights: Optional[tuple] = None


class LlamaModelWithHead(_DecoderWithHead):
    family = "llama"


class GPTNeoXModelWithHead(_DecoderWithHead):
    family = "neox"


class GemmaModelWithHead(_DecoderWithHead):
    family = "gemma3"


class _DecoderStack(_DecoderWithHead):
    """``*Model`` (the stack without the LM head): parameters are the body subtree
    (``{"params": {"embed_tokens": ..., "layers_0": ..., "norm": ...}}``)."""

    @property
    def _body(self) -> str:
        return "gpt_neox" if self.family == "neox" else "model"

    def init(self, seed: int = 0, *_, std: float = 0.02) -> dict:
        return {"params": random_params(self.family, self.config, seed=seed, std=std)["params"][self._body]}

    def _full_tree(self, params):
        if not isinstance(params, dict) or "params" not in params:
            raise ValueError("params must be a mapping with a 'params' entry.")
        body = params["params"]
        emb = body["embed_tokens"]["embedding"]
        emb = emb if isinstance(emb, torch.Tensor) else torch.as_tensor(emb)
        # the stack's output does not depend on the head; the tied embedding stands in for it
        return {"params": {self._body: body, "lm_head": {"kernel": emb.T}}}

    def apply(self, params, input_ids, attention_mask=None, position_ids=None, kv_caches=None,
              output_attentions=False, output_hidden_states=False, use_cache=False):
        """``*Model.__call__`` (models/llama.py:161-225, gpt_neox.py:158-222, gemma3.py:215-283) on the GPU
        kernels for a cache-free forward: ``last_hidden_state`` [B, S, d] after the final norm, in a
        ``BaseModelOutputWithCache``.  Same inputs, checks and limits as ``*ModelWithHead.apply``."""
        from ._checks import normalize_bool

        use_cache = normalize_bool("use_cache", use_cache)
        output_attentions = normalize_bool("output_attentions", output_attentions)
        output_hidden_states = normalize_bool("output_hidden_states", output_hidden_states)
        if kv_caches is not None or use_cache or position_ids is not None:
            raise NotImplementedError("apply with KV caches or position ids: use Engine.generate for cached decoding.")
        if output_attentions or output_hidden_states:
            raise NotImplementedError("apply does not return attention weights or per-layer hidden states.")
        ids, mask = _check_model_inputs(self.config, input_ids, attention_mask)
        B, S = ids.shape
        rt = self._runtime(params, B, S)
        dev = rt.w.device
        return BaseModelOutputWithCache(last_hidden_state=rt.forward_hidden(ids.to(dev), mask.to(dev)))


class LlamaModel(_DecoderStack):
    family = "llama"


class GPTNeoXModel(_DecoderStack):
    family = "neox"


class GemmaModel(_DecoderStack):
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
