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
from .decoders import (GemmaDecoder, GemmaMLP, GPTNeoXDecoder, GPTNeoXMLP, LlamaDecoder,  # noqa: F401
                       LlamaMLP)
from .nn import GemmaRMSNorm  # noqa: F401  (models/gemma3.py:89-106 lives in jaxml.models)

# models/__init__.py of the reference: the architecture entry points, in its order
__all__ = ["GPTNeoXDecoder", "GPTNeoXMLP", "GPTNeoXModel", "GPTNeoXModelWithHead", "GemmaDecoder", "GemmaMLP",
           "GemmaModel", "GemmaModelWithHead", "GemmaRMSNorm", "LlamaDecoder", "LlamaMLP", "LlamaModel",
           "LlamaModelWithHead"]


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

    intermediate_size = property(lambda self: self.config.intermediate_size)
    norm_eps = property(lambda self: self.config.norm_eps)
    use_bias = property(lambda self: self.config.use_bias)
    attn_scale = property(lambda self: self.config.attn_scale)

    def init(self, key=0, input_ids=None, *_, std: float = 0.02, **__) -> dict:
        """Random N(0, std) kernels, unit norm weights, in the reference's parameter layout.  ``key`` is an
        int seed or a PRNG key (two uint32 words); example ``input_ids``, when given, are checked as
        ``apply`` checks them (the reference's ``init`` runs the model on them)."""
        if input_ids is not None:
            _prepare_model_inputs(self.config, input_ids, None)
        tree = random_params(self.family, self.config, seed=_seed_of(key), std=std)
        tree["cache"] = {self._body_key: self._rope_cache()}
        return tree

    @property
    def _body_key(self) -> str:
        return "gpt_neox" if self.family == "neox" else "model"

    def _rope_cache(self) -> dict:
        """The rotary tables in the model dtype, as the stack's ``cache`` collection holds them
        (``rotary_emb``, and ``rotary_emb_local`` for Gemma3).  ``apply`` does not read them: the kernels
        take their own copy of the same tables."""
        from .nn import RotaryEmbedding

        cfg = self.config
        specs = {"rotary_emb": (cfg.rope_theta, cfg.rope_scale)}
        if self.family == "gemma3":
            specs["rotary_emb_local"] = (10000.0, 1.0)
        out = {}
        for name, (base, scale) in specs.items():
            rope = RotaryEmbedding(dim=cfg.head_dim, max_length=cfg.max_position_embeddings, base=base,
                                   dtype=self.dtype, rotary_pct=cfg.rotary_pct, rope_scale=scale)
            out[name] = rope.init(0, torch.zeros(1, 1, 1))["cache"]
        return out

    def apply(self, params, input_ids, attention_mask=None, position_ids=None, kv_caches=None, use_cache=False,
              output_attentions=False, output_hidden_states=False, keep_last_n_logits: int = 0):
        """``*ModelWithHead.__call__`` (models/llama.py:247-273, gpt_neox.py:245-272, gemma3.py:304-331) on
        the GPU kernels: logits ``[B, S]`` (or the last ``keep_last_n_logits`` positions) in the model dtype,
        in a ``CausalLMOutputWithCache``.  A cache-free call without position ids or hidden states runs on
        the fused prefill runtime; calls with KV caches (a prompt into empty caches, or one token per row
        into populated ones), position ids, ``output_hidden_states`` or ``output_attentions`` run layer by
        layer through the decoder blocks.  Masks must be right-padded."""
        from ._checks import normalize_count

        keep = normalize_count("keep_last_n_logits", keep_last_n_logits)
        if keep < 0:
            raise ValueError(f"keep_last_n_logits must be non-negative, got {keep}.")
        hidden, caches, states, weights, is_logits = self._stack(params, input_ids, attention_mask, position_ids,
                                                                 kv_caches, use_cache, output_attentions,
                                                                 output_hidden_states, keep)
        if is_logits:
            return CausalLMOutputWithCache(logits=hidden, kv_caches=caches)
        h = hidden if keep == 0 else hidden[:, -keep:]
        head = self._head_kernel(params)
        B, n, d = h.shape
        from . import nn as _nn

        logits = _nn._dense(h.reshape(B * n, d), head, None, self.dtype).reshape(B, n, -1)
        _nn._check_status(h.device, "lm_head")
        return CausalLMOutputWithCache(logits=logits, kv_caches=caches, hidden_states=states,
                                       attention_weights=weights)

    def _head_kernel(self, params) -> torch.Tensor:
        """The LM head kernel [d, V] on the device in the model dtype (cached with the converted tree)."""
        return self._device_params(params)["lm_head"]["kernel"]

    def _body(self, params) -> dict:
        return self._device_params(params)["gpt_neox" if self.family == "neox" else "model"]

    def _device_params(self, params) -> dict:
        """The whole parameter tree on the device in the model dtype, cached per tree."""
        from .decoders import device_tree

        dev = torch.device("cuda", torch.cuda.current_device())
        cache = self.__dict__.setdefault("_layered_cache", {})
        key = (id(params), dev.index, self.dtype)
        if cache.get("key") != key:
            cache.clear()
            if not isinstance(params, dict) or "params" not in params:
                raise ValueError("params must be a mapping with a 'params' entry.")
            cache["key"] = key
            cache["params"] = params   # keeps the tree alive while its id is the cache key
            cache["tree"] = device_tree(self._full_tree(params)["params"], self.dtype, dev)
            cache["rope"] = {}
        return cache["tree"]

    def _stack(self, params, input_ids, attention_mask, position_ids, kv_caches, use_cache, output_attentions,
               output_hidden_states, keep):
        """The stack below the head.  Returns ``(last_hidden_state, kv_caches, hidden_states,
        attention_weights, False)``; on the fused runtime path of a model with a head, ``(logits, kv_caches,
        None, None, True)``."""
        from ._checks import normalize_bool

        use_cache = normalize_bool("use_cache", use_cache)
        output_attentions = normalize_bool("output_attentions", output_attentions)
        output_hidden_states = normalize_bool("output_hidden_states", output_hidden_states)
        ids, mask, kv_caches, pos = _prepare_model_inputs(self.config, input_ids, attention_mask, kv_caches,
                                                          position_ids)
        L = self.config.num_layers
        if mask is not None and not _right_padded(mask):
            raise NotImplementedError("apply takes right-padded attention masks (the kernels attend to key prefixes).")
        if kv_caches is None and pos is None and not output_hidden_states and not output_attentions:
            B, S = ids.shape
            rt = self._runtime(params, B, S)
            dev = rt.w.device
            caches = (None,) * L if use_cache else None
            if self._has_head:
                return rt.forward_logits(ids.to(dev), mask.to(dev), keep), caches, None, None, True
            return rt.forward_hidden(ids.to(dev), mask.to(dev)), caches, None, None, False
        from .decoders import layered_forward, _cached_sequence_length

        body = self._body(params)
        dev = body["embed_tokens"]["embedding"].device
        cached_len = _cached_sequence_length(kv_caches)
        h, caches, states, weights = layered_forward(
            self.family, self.config, self.dtype, body, ids.to(dev), None if mask is None else mask.to(dev),
            None if pos is None else pos.to(dev), kv_caches, cached_len, self.__dict__["_layered_cache"]["rope"],
            output_attentions)
        return (h, caches if use_cache else None, states if output_hidden_states else None,
                weights if output_attentions else None, False)

    _has_head = True

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


def _seed_of(key) -> int:
    """An int seed, or the seed a PRNG key stands for: ``PRNGKey(s)`` is the words ``(s >> 32, s & mask)``,
    so the key's words read back as ``(hi << 32) | lo`` (``init(PRNGKey(7))`` draws as ``init(7)``)."""
    import numpy as np

    if key is None:
        return 0
    if isinstance(key, (int, np.integer)) and not isinstance(key, (bool, np.bool_)):
        return int(key) & ((1 << 63) - 1)
    words = np.asarray(key.cpu() if isinstance(key, torch.Tensor) else key).reshape(-1).astype(np.int64)
    seed = 0
    for w in words.tolist():
        seed = (seed << 32) | (int(w) & 0xFFFFFFFF)
    return seed & ((1 << 63) - 1)


def _right_padded(mask: torch.Tensor) -> bool:
    return mask.shape[1] <= 1 or not bool((mask[:, :-1].to(torch.int8) < mask[:, 1:].to(torch.int8)).any())


def _as_t(x) -> torch.Tensor:
    import numpy as np

    return x if isinstance(x, torch.Tensor) else torch.as_tensor(np.asarray(x))


def _prepare_model_inputs(config, input_ids, attention_mask, kv_caches=None, position_ids=None):
    """models/_utils.py:78-217 (``prepare_model_inputs``, ``prepare_position_ids``,
    ``prepare_default_attention_mask``) with the same messages, raised before any device work.  Returns
    ``(ids, mask, kv_caches, position_ids)``: int32 ids with negative placeholders mapped to 0, the
    boolean mask (the default ``ids >= 0`` unless populated caches carry the mask, then None or the
    caller's), the caches as a tuple (or None) and the position ids (or None)."""
    from .cache import KVCache

    ids = _as_t(input_ids)
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
    L = config.num_layers
    if kv_caches is not None:
        try:
            kv_caches = tuple(kv_caches)
        except TypeError as e:
            raise TypeError("kv_caches must be a sequence containing one cache per layer.") from e
        if len(kv_caches) != L:
            raise ValueError(f"kv_caches must contain one cache per layer, got {len(kv_caches)} and expected {L}.")
        for idx, c in enumerate(kv_caches):
            if c is not None and not isinstance(c, KVCache):
                raise TypeError(f"kv_caches entries must be KVCache instances or None, got {type(c)} at index {idx}.")
            if c is not None:
                c.validate_state()
    expected = tuple(ids.shape)
    populated = () if kv_caches is None else tuple(
        tuple(c.mask.shape) for c in kv_caches if c is not None and c.mask is not None)
    if populated:
        expected = populated[0]
        if any(s != expected for s in populated):
            raise ValueError("kv_caches populated entries must share attention mask shape.")
        if expected[0] != ids.shape[0]:
            raise ValueError("kv_caches populated entries must share input_ids batch size; "
                             f"got {expected[0]} and {ids.shape[0]}.")
    mask = None
    if attention_mask is not None:
        mask = _as_t(attention_mask)
        if mask.ndim != 2:
            raise ValueError(f"attention_mask must be a 2D array, got shape {tuple(mask.shape)}.")
        if mask.is_floating_point() or mask.is_complex():
            raise TypeError(f"attention_mask must be boolean or integer, got dtype {mask.dtype}.")
        if tuple(mask.shape) != expected:
            raise ValueError("attention_mask shape must match input_ids shape or populated KV cache mask shape; "
                             f"got {tuple(mask.shape)} and expected {expected}.")
        if mask.dtype != torch.bool and bool(((mask != 0) & (mask != 1)).any()):
            raise ValueError("attention_mask integer values must be 0 or 1.")
        mask = mask.to(torch.bool)
        if not bool(mask.any(dim=1).all()):
            raise ValueError("attention_mask must contain at least one valid token per batch row.")
        if tuple(mask.shape) == tuple(ids.shape) and bool((mask & (ids.to(mask.device) < 0)).any()):
            raise ValueError("attention_mask must not mark negative placeholder input_ids as valid.")
    negative = bool((ids < 0).any())
    if negative and mask is not None and tuple(mask.shape) != tuple(ids.shape):
        raise ValueError("input_ids must not contain negative placeholder ids when attention_mask is not token-shaped.")
    if negative and mask is None and populated:
        raise ValueError("input_ids must not contain negative placeholder ids when using populated KV caches.")
    pos = None
    if position_ids is not None:
        pos = _as_t(position_ids)
        if pos.ndim != 2:
            raise ValueError(f"position_ids must be a 2D array, got shape {tuple(pos.shape)}.")
        if pos.is_floating_point() or pos.is_complex() or pos.dtype == torch.bool:
            raise TypeError(f"position_ids must contain integer positions, got dtype {pos.dtype}.")
        if pos.shape[1] != ids.shape[1] or pos.shape[0] not in (1, ids.shape[0]):
            raise ValueError("position_ids shape must be broadcastable to input_ids batch and sequence axes, "
                             f"got {tuple(pos.shape)} and {tuple(ids.shape)}.")
        if bool((pos < 0).any()):
            raise ValueError("position_ids must contain non-negative positions.")
        if bool((pos >= config.max_position_embeddings).any()):
            raise ValueError(
                f"position_ids must be less than max_position_embeddings={config.max_position_embeddings}.")
    if mask is None and not populated:
        mask = ids >= 0
        if not bool(mask.any(dim=1).all()):
            raise ValueError("input_ids must contain at least one non-negative token per batch row when "
                             "attention_mask is omitted.")
    ids = torch.where(ids < 0, torch.zeros_like(ids), ids).to(torch.int32)
    return ids, mask, kv_caches, pos


@dataclass
class CausalLMOutputWithCache:
    """``outputs.py``: logits, and the updated caches, per-layer hidden states and attention weights when
    asked for."""

    logits: torch.Tensor
    kv_caches: Optional[tuple] = None
    hidden_states: Optional[tuple] = None
    attention_weights: Optional[tuple] = None


@dataclass
class BaseModelOutputWithCache:
    """``outputs.py``: the decoder stack's final hidden states, and the updated caches, per-layer hidden
    states and attention weights when asked for."""

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

    _has_head = False

    def init(self, key=0, input_ids=None, *_, std: float = 0.02, **__) -> dict:
        if input_ids is not None:
            _prepare_model_inputs(self.config, input_ids, None)
        return {"params": random_params(self.family, self.config, seed=_seed_of(key),
                                        std=std)["params"][self._body_key],
                "cache": self._rope_cache()}

    def _full_tree(self, params):
        if not isinstance(params, dict) or "params" not in params:
            raise ValueError("params must be a mapping with a 'params' entry.")
        body = params["params"]
        emb = body["embed_tokens"]["embedding"]
        emb = emb if isinstance(emb, torch.Tensor) else torch.as_tensor(emb)
        # the stack's output does not depend on the head; the tied embedding stands in for it
        return {"params": {self._body_key: body, "lm_head": {"kernel": emb.T}}}

    def apply(self, params, input_ids, attention_mask=None, position_ids=None, kv_caches=None,
              output_attentions=False, output_hidden_states=False, use_cache=False):
        """``*Model.__call__`` (models/llama.py:161-225, gpt_neox.py:158-222, gemma3.py:215-283):
        ``last_hidden_state`` [B, S, d] after the final norm, the updated caches (``use_cache``), the
        per-layer hidden states (``output_hidden_states``) and attention weights (``output_attentions``) in
        a ``BaseModelOutputWithCache``.  Same inputs, paths and limits as ``*ModelWithHead.apply``."""
        h, caches, states, weights, _ = self._stack(params, input_ids, attention_mask, position_ids, kv_caches,
                                                    use_cache, output_attentions, output_hidden_states, 0)
        return BaseModelOutputWithCache(last_hidden_state=h, kv_caches=caches, hidden_states=states,
                                        attention_weights=weights)


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
