"""Torch state dict -> parameter tree in the reference's Flax layout.

Mirrors ``utils.py:197-371`` (``torch_to_jax_states``: ``layers.N`` -> ``layers_N``, dense weights
transposed to ``[in, out]``, q/k/v reshaped to ``[d, heads, head_dim]``, fused NeoX QKV to
``[d, 3, heads, head_dim]``, norm weights kept as they are) and ``hf_utils.py:57-93`` (the Llama / Gemma /
NeoX wrappers, including the NeoX key renames).  Leaves are torch tensors (CPU) rather than numpy arrays.
"""
from __future__ import annotations

import re
from collections.abc import Mapping

import torch

from ._checks import normalize_dtype

_NORM_KEYS = {"post_attention_layernorm", "pre_feedforward_layernorm", "post_feedforward_layernorm",
              "input_layernorm", "norm", "q_norm", "k_norm"}


def _normalize_state_key(key: str) -> list[str]:
    out: list[str] = []
    for seg in key.split("."):
        if not seg:
            raise ValueError(f"State key {key!r} must not contain empty path segments.")
        if seg.isdigit() and out:
            out[-1] += "_" + seg
        else:
            out.append(seg)
    return out


def torch_to_jax_states(states, dtype=torch.float32, head_dim: int | None = None) -> dict:
    dtype = normalize_dtype("dtype", dtype)
    if isinstance(states, torch.nn.Module):
        states = states.state_dict()
    if not isinstance(states, Mapping) or not states:
        raise ValueError("PyTorch state dict must contain at least one tensor.")
    tree: dict = {"params": {}}
    for key, value in states.items():
        path = _normalize_state_key(key)
        t = value.detach().cpu().to(torch.float32)
        leaf = path[-1]
        if len(path) >= 2 and path[-2] in _NORM_KEYS:
            pass
        elif "embed_tokens" in path:
            if leaf == "weight":
                path[-1] = "embedding"
        elif any(p in path for p in ("q_proj", "k_proj", "v_proj")):
            if leaf == "weight":
                path[-1] = "kernel"
                t = t.T if head_dim is None else t.T.reshape(t.shape[1], -1, head_dim)
            elif leaf == "bias" and head_dim is not None:
                t = t.reshape(-1, head_dim)
        elif "qkv_proj" in path:
            if leaf == "weight":
                path[-1] = "kernel"
                if head_dim is None:
                    t = t.T.reshape(t.shape[1], 3, -1)
                else:
                    t = t.T.reshape(t.shape[1], -1, 3, head_dim).permute(0, 2, 1, 3)
            elif leaf == "bias":
                t = t.reshape(3, -1) if head_dim is None else t.reshape(-1, 3, head_dim).permute(1, 0, 2)
        else:
            if leaf == "weight":
                path[-1] = "kernel"
                t = t.T
        cursor = tree["params"]
        for seg in path[:-1]:
            cursor = cursor.setdefault(seg, {})
        cursor[path[-1]] = t.contiguous().to(dtype)
    return tree


def _head_dim(config) -> int:
    hd = getattr(config, "head_dim", None)
    return hd if hd else config.hidden_size // config.num_attention_heads


def to_llama_jax_params(model, dtype=torch.float32) -> dict:
    return torch_to_jax_states(model.state_dict(), dtype=dtype, head_dim=_head_dim(model.config))


def to_gemma_jax_params(model, dtype=torch.float32) -> dict:
    return torch_to_jax_states(model.state_dict(), dtype=dtype, head_dim=_head_dim(model.config))


_NEOX_SUB = (
    (r"embed_in(.*)", r"embed_tokens\1"),
    (r"final_layer_norm(.*)", r"norm\1"),
    (r"embed_out(.*)", r"lm_head\1"),
    (r"attention\.(.*)", r"self_attn.\1"),
    (r"query_key_value(.*)", r"qkv_proj\1"),
    (r"dense\.(.*)", r"o_proj.\1"),
    (r"dense_h_to_4h(.*)", r"up_proj\1"),
    (r"dense_4h_to_h(.*)", r"down_proj\1"),
)


def to_neox_jax_params(model, dtype=torch.float32) -> dict:
    renamed = {}
    for key, value in model.state_dict().items():
        name = key
        for pat, rep in _NEOX_SUB:
            name = re.sub(pat, rep, name)
        renamed[name] = value
    return torch_to_jax_states(renamed, dtype=dtype, head_dim=_head_dim(model.config))
