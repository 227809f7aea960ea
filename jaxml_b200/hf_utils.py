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

from ._checks import normalize_count, normalize_dtype

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


def _positive(name: str, value) -> int:
    value = normalize_count(name, value)
    if value <= 0:
        raise ValueError(f"{name} must be positive, got {value}.")
    return value


def _head_dim(config) -> int:
    """The config's head_dim, else hidden_size / num_attention_heads (validated like the reference)."""
    hd = getattr(config, "head_dim", None)
    if hd is not None:
        return _positive("head_dim", hd)
    hidden = _positive("hidden_size", config.hidden_size)
    heads = _positive("num_attention_heads", config.num_attention_heads)
    if hidden % heads:
        raise ValueError("hidden_size must be divisible by num_attention_heads when head_dim is not set.")
    return hidden // heads


def _model_states(model, what: str):
    """(config, state dict) of an HF-like model, checked before any conversion."""
    config = getattr(model, "config", None)
    if config is None:
        raise ValueError(f"Expected the {what} model to expose a config.")
    sd = getattr(model, "state_dict", None)
    if not callable(sd):
        raise TypeError(f"Expected the {what} model to provide a callable state_dict.")
    states = sd()
    if not isinstance(states, Mapping):
        raise TypeError(f"The {what} model's state_dict must be a mapping, got {type(states)}.")
    if not states:
        raise ValueError("PyTorch state dict must contain at least one tensor.")
    return config, states


def to_llama_jax_params(model, dtype=torch.float32) -> dict:
    config, states = _model_states(model, "Llama")
    return torch_to_jax_states(states, dtype=dtype, head_dim=_head_dim(config))


def to_gemma_jax_params(model, dtype=torch.float32) -> dict:
    config, states = _model_states(model, "Gemma")
    return torch_to_jax_states(states, dtype=dtype, head_dim=_head_dim(config))


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
    config, states = _model_states(model, "GPT-NeoX")
    renamed, origin = {}, {}
    for key, value in states.items():
        name = key
        for pat, rep in _NEOX_SUB:
            name = re.sub(pat, rep, name)
        if name in renamed:
            raise ValueError(f"State keys {origin[name]!r} and {key!r} map to the same jaxml destination {name!r}.")
        renamed[name], origin[name] = value, key
    return torch_to_jax_states(renamed, dtype=dtype, head_dim=_head_dim(config))


# ------------------------------------------------------------------------------------------------
# Loading a Hugging Face causal LM (local path or hub id) into a model class + parameter tree
# (hf_utils.py:96-250 of the reference: architecture names, dtype strings, model_type checks).
# ------------------------------------------------------------------------------------------------
_HF_DTYPES = {"float32": torch.float32, "fp32": torch.float32, "float16": torch.float16, "fp16": torch.float16,
              "bfloat16": torch.bfloat16, "bf16": torch.bfloat16}


def _normalize_hf_architecture(architecture) -> str:
    if not isinstance(architecture, str):
        raise TypeError(f"architecture must be a string, got {type(architecture)}.")
    a = architecture.lower().replace("-", "_")
    aliases = {"auto": "auto", "llama": "llama", "neox": "neox", "gpt_neox": "neox", "gemma": "gemma",
               "gemma3": "gemma", "gemma_3": "gemma"}
    if a not in aliases:
        raise ValueError(f"Unsupported Hugging Face architecture {architecture!r}.")
    return aliases[a]


def _normalize_hf_model_name(name) -> str:
    import os

    try:
        path = os.fspath(name)
    except TypeError as e:
        raise TypeError(f"name must be a string or path-like object, got {type(name)}.") from e
    if not isinstance(path, str):
        raise TypeError(f"name must resolve to a string path, got {type(path)}.")
    if not path.strip():
        raise ValueError("name must be non-empty.")
    return path


def _validate_hf_dtype(dtype):
    if isinstance(dtype, torch.dtype):
        name = str(dtype).replace("torch.", "")
        if name not in _HF_DTYPES:
            raise ValueError(f"Unsupported dtype {dtype!r}; expected one of {sorted(_HF_DTYPES)}.")
        return name
    if not isinstance(dtype, str):
        raise TypeError(f"Expected dtype to be a string such as 'float32' or 'bfloat16', got {dtype!r}.")
    if dtype.lower() not in _HF_DTYPES:
        raise ValueError(f"Unsupported dtype {dtype!r}; expected one of {sorted(_HF_DTYPES)}.")
    return dtype


def _check_model_type(config, expected: tuple, what: str):
    mt = getattr(config, "model_type", None)
    if mt not in expected:
        raise ValueError(f"Expected Hugging Face {what} model_type to be one of {expected}, got {mt!r}.")


def load_model_from_hf(name, architecture: str = "auto", dtype: str = "float32", **from_pretrained_kwargs):
    """(model class instance, reference parameter tree) from a supported HF causal LM.  The model class
    computes in `dtype`; leaves are CPU torch tensors in that dtype."""
    from .config import ModelConfig
    from .models import GemmaModelWithHead, GPTNeoXModelWithHead, LlamaModelWithHead

    name = _normalize_hf_model_name(name)
    dtype = _validate_hf_dtype(dtype)
    arch = _normalize_hf_architecture(architecture)
    try:
        from transformers import AutoConfig, AutoModelForCausalLM
    except ImportError as e:
        raise ImportError("Please install transformers library.") from e
    if arch == "auto":
        mt = getattr(AutoConfig.from_pretrained(name, **from_pretrained_kwargs), "model_type", None)
        arch = {"llama": "llama", "gpt_neox": "neox", "gemma3": "gemma", "gemma3_text": "gemma"}.get(mt)
        if arch is None:
            raise ValueError(f"Unsupported Hugging Face model type {mt!r}.")
    tdt = _HF_DTYPES[dtype.lower()]
    hf = AutoModelForCausalLM.from_pretrained(name, **from_pretrained_kwargs)
    if arch == "llama":
        _check_model_type(hf.config, ("llama",), "Llama")
        return LlamaModelWithHead(ModelConfig.from_hf(hf.config), dtype=tdt), to_llama_jax_params(hf, dtype=tdt)
    if arch == "neox":
        _check_model_type(hf.config, ("gpt_neox",), "GPT-NeoX")
        return GPTNeoXModelWithHead(ModelConfig.from_hf(hf.config), dtype=tdt), to_neox_jax_params(hf, dtype=tdt)
    lm = getattr(hf, "language_model", hf)
    _check_model_type(lm.config, ("gemma3_text", "gemma3"), "Gemma")
    return GemmaModelWithHead(ModelConfig.from_hf(lm.config), dtype=tdt), to_gemma_jax_params(lm, dtype=tdt)
