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

from ._checks import normalize_count

_NORM_KEYS = {"post_attention_layernorm", "pre_feedforward_layernorm", "post_feedforward_layernorm",
              "input_layernorm", "norm", "q_norm", "k_norm"}


_STATE_DTYPES = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32,
                 "float64": torch.float64}


def _state_dtype(dtype) -> torch.dtype:
    """utils.py:57-69: a dtype name or a torch floating dtype among float16 / bfloat16 / float32 / float64."""
    if isinstance(dtype, torch.dtype):
        name = str(dtype).replace("torch.", "")
    elif isinstance(dtype, str):
        name = dtype
    else:
        raise TypeError(f"Expected dtype to be a string or torch.dtype, got {type(dtype)}.")
    if name not in _STATE_DTYPES:
        raise ValueError(f"Unsupported dtype {dtype!r}. Supported dtypes are: {', '.join(_STATE_DTYPES)}.")
    return _STATE_DTYPES[name]


def _normalize_state_key(key) -> list[str]:
    """``layers.3.mlp`` -> ``["layers_3", "mlp"]`` (a numeric segment joins the one before it)."""
    if not isinstance(key, str):
        raise TypeError(f"State key must be a string, got {type(key)}.")
    if not key:
        raise ValueError("State key must be non-empty.")
    out: list[str] = []
    for seg in key.split("."):
        if not seg:
            raise ValueError(f"State key {key!r} must not contain empty path segments.")
        if seg.isdigit() and out:
            out[-1] += "_" + seg
        else:
            out.append(seg)
    return out


def _state_tensor(value, key: str) -> torch.Tensor:
    if not isinstance(value, torch.Tensor):
        raise TypeError(f"State value for key {key!r} must be a torch.Tensor, got {type(value)}.")
    t = value.detach().cpu()
    if t.numel() == 0:
        raise ValueError(f"State value for key {key!r} must not be empty.")
    if not t.is_floating_point():
        raise TypeError(f"State value for key {key!r} must contain floating point values, got dtype {t.dtype}.")
    if not bool(torch.isfinite(t).all()):
        raise ValueError(f"State value for key {key!r} must contain only finite values.")
    return t.to(torch.float32) if t.dtype in (torch.bfloat16, torch.float16) else t


def _insert_leaf(tree: dict, path: list[str], value, key: str):
    cursor = tree
    for seg in path[:-1]:
        nxt = cursor.setdefault(seg, {})
        if not isinstance(nxt, dict):
            raise ValueError(f"State key {key!r} conflicts with existing leaf at destination {'.'.join(path)!r}.")
        cursor = nxt
    if path[-1] in cursor:
        raise ValueError(f"Multiple state keys map to destination {'.'.join(path)!r}.")
    cursor[path[-1]] = value


def _divisible(n: int, by: int, what: str, by_name: str):
    if n % by:
        raise ValueError(f"{what} {n} must be divisible by {by_name}.")


def torch_to_jax_states(states, dtype=torch.float32, head_dim: int | None = None) -> dict:
    """utils.py:258-371: a torch module or state dict as the reference's parameter tree.  Dense weights
    become ``kernel`` ``[in, out]``; with ``head_dim`` the q / k / v projections become ``[d, heads,
    head_dim]`` and a fused ``qkv_proj`` ``[d, 3, heads, head_dim]`` (without it, ``[d, 3, -1]``);
    embeddings become ``embedding``; norm weights stay as they are.  Leaves are CPU tensors in ``dtype``."""
    dtype = _state_dtype(dtype)
    if head_dim is not None:
        if isinstance(head_dim, bool) or type(head_dim).__name__ == "bool_":
            raise TypeError(f"head_dim must be an integer when set, got {type(head_dim)}.")
        try:
            head_dim = normalize_count("head_dim", head_dim)
        except TypeError as e:
            raise TypeError(f"head_dim must be an integer when set, got {type(head_dim)}.") from e
        if head_dim <= 0:
            raise ValueError(f"head_dim must be positive when set, got {head_dim}.")
    if isinstance(states, torch.nn.Module):
        states = states.state_dict()
    elif not isinstance(states, Mapping):
        raise TypeError(f"Expected input to be either a PyTorch module or a mapping, got {type(states)}.")
    if not states:
        raise ValueError("PyTorch state dict must contain at least one tensor.")
    tree: dict = {"params": {}}
    hd = head_dim
    for key, value in states.items():
        path = _normalize_state_key(key)
        leaf = path[-1]
        if len(path) >= 2 and path[-2] in _NORM_KEYS:
            _insert_leaf(tree["params"], path, _state_tensor(value, key).contiguous().to(dtype), key)
            continue
        t = _state_tensor(value, key)
        if "embed_tokens" in path:
            if leaf == "weight":
                path[-1] = "embedding"
        elif any(p in path for p in ("q_proj", "k_proj", "v_proj")):
            if leaf == "weight":
                path[-1] = "kernel"
                if hd is not None:
                    _divisible(t.shape[0], hd, "Q/K/V projection output dimension", f"head_dim {hd}")
                t = t.T if hd is None else t.T.reshape(t.shape[1], -1, hd)
            elif leaf == "bias" and hd is not None:
                _divisible(t.shape[0], hd, "Q/K/V projection bias length", f"head_dim {hd}")
                t = t.reshape(-1, hd)
        elif "qkv_proj" in path:
            if leaf == "weight":
                path[-1] = "kernel"
                if hd is None:
                    _divisible(t.shape[0], 3, "Fused QKV projection output dimension", "3")
                    t = t.T.reshape(t.shape[1], 3, -1)
                else:
                    _divisible(t.shape[0], 3 * hd, "Fused QKV projection output dimension", f"3 * head_dim {3 * hd}")
                    t = t.T.reshape(t.shape[1], -1, 3, hd).permute(0, 2, 1, 3)
            elif leaf == "bias":
                if hd is None:
                    _divisible(t.shape[0], 3, "Fused QKV projection bias length", "3")
                    t = t.reshape(3, -1)
                else:
                    _divisible(t.shape[0], 3 * hd, "Fused QKV projection bias length", f"3 * head_dim {3 * hd}")
                    t = t.reshape(-1, 3, hd).permute(1, 0, 2)
        elif leaf == "weight":
            path[-1] = "kernel"
            t = t.T
        _insert_leaf(tree["params"], path, t.contiguous().to(dtype), key)
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


def _model_config(model, what: str):
    config = getattr(model, "config", None)
    if config is None:
        raise ValueError(f"Expected the {what} model to expose a config.")
    return config


def _model_states(model, what: str):
    """(config, state dict) of an HF-like model, checked before any conversion."""
    config = _model_config(model, what)
    sd = getattr(model, "state_dict", None)
    if not callable(sd):
        raise TypeError(f"Expected the {what} model to provide a callable state_dict.")
    states = sd()
    if not isinstance(states, Mapping):
        raise TypeError(f"The {what} model's state_dict must be a mapping, got {type(states)}.")
    if not states:
        raise ValueError("PyTorch state dict must contain at least one tensor.")
    return config, states


def to_llama_jax_params(model, dtype="float16") -> dict:
    config, states = _model_states(model, "Llama")
    return torch_to_jax_states(states, dtype=dtype, head_dim=_head_dim(config))


def to_gemma_jax_params(model, dtype="bfloat16") -> dict:
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


def to_neox_jax_params(model, dtype="float16") -> dict:
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


def _infer_hf_architecture(name: str, **config_kwargs) -> str:
    """The architecture of a checkpoint from its config's ``model_type`` (hf_utils.py:139-157)."""
    try:
        from transformers import AutoConfig
    except ImportError as e:
        raise ImportError("Please install transformers library.") from e
    mt = getattr(AutoConfig.from_pretrained(name, **config_kwargs), "model_type", None)
    arch = {"llama": "llama", "gpt_neox": "neox", "gemma3": "gemma", "gemma3_text": "gemma"}.get(mt)
    if arch is None:
        raise ValueError(f"Unsupported Hugging Face model type {mt!r}.")
    return arch


def load_model_from_hf(name, architecture: str = "auto", dtype: str = "float32", **from_pretrained_kwargs):
    """(model class instance, reference parameter tree) from a supported HF causal LM (hf_utils.py:160-181):
    the name, dtype and architecture are checked before anything is loaded, ``auto`` reads the
    checkpoint's config, and the per-architecture loader does the rest."""
    name = _normalize_hf_model_name(name)
    dtype = _validate_hf_dtype(dtype)
    arch = _normalize_hf_architecture(architecture)
    if arch == "auto":
        arch = _infer_hf_architecture(name, **from_pretrained_kwargs)
    loader = {"llama": load_llama_from_hf, "neox": load_neox_from_hf, "gemma": load_gemma_from_hf}[arch]
    return loader(name, dtype=dtype, **from_pretrained_kwargs)


def _auto_model(name: str, **kw):
    try:
        from transformers import AutoModelForCausalLM
    except ImportError as e:
        raise ImportError("Please install transformers library.") from e
    return AutoModelForCausalLM.from_pretrained(name, **kw)


def load_llama_from_hf(name, dtype: str = "float32", **from_pretrained_kwargs):
    """A Llama checkpoint (local path or hub id) as ``(LlamaModelWithHead, params)`` with parameters in
    ``dtype``; the model class keeps the default compute dtype, as in the reference (hf_utils.py:184-202)."""
    from .config import ModelConfig
    from .models import LlamaModelWithHead

    name = _normalize_hf_model_name(name)
    tdt = _HF_DTYPES[_validate_hf_dtype(dtype).lower()]
    hf = _auto_model(name, **from_pretrained_kwargs)
    cfg = _model_config(hf, "Llama")
    _check_model_type(cfg, ("llama",), "Llama")
    params = to_llama_jax_params(hf, dtype=tdt)
    return LlamaModelWithHead(ModelConfig.from_hf(cfg)), params


def load_neox_from_hf(name, dtype: str = "float32", **from_pretrained_kwargs):
    """A GPT-NeoX checkpoint as ``(GPTNeoXModelWithHead, params)`` (hf_utils.py:205-223)."""
    from .config import ModelConfig
    from .models import GPTNeoXModelWithHead

    name = _normalize_hf_model_name(name)
    tdt = _HF_DTYPES[_validate_hf_dtype(dtype).lower()]
    hf = _auto_model(name, **from_pretrained_kwargs)
    cfg = _model_config(hf, "GPT-NeoX")
    _check_model_type(cfg, ("gpt_neox",), "GPT-NeoX")
    params = to_neox_jax_params(hf, dtype=tdt)
    return GPTNeoXModelWithHead(ModelConfig.from_hf(cfg)), params


def load_gemma_from_hf(name, dtype: str = "float32", **from_pretrained_kwargs):
    """A Gemma3 checkpoint as ``(GemmaModelWithHead, params)`` (hf_utils.py:226-250): the multimodal
    wrapper (``model_type`` gemma3) is checked, then its ``language_model`` (gemma3_text) is converted.
    A text-only checkpoint, whose causal LM is the text model itself, is taken as it is."""
    from .config import ModelConfig
    from .models import GemmaModelWithHead

    name = _normalize_hf_model_name(name)
    tdt = _HF_DTYPES[_validate_hf_dtype(dtype).lower()]
    hf = _auto_model(name, **from_pretrained_kwargs)
    wrapper_cfg = _model_config(hf, "Gemma")
    if getattr(wrapper_cfg, "model_type", None) == "gemma3_text":
        lm = hf
    else:
        _check_model_type(wrapper_cfg, ("gemma3",), "Gemma")
        try:
            lm = hf.language_model
        except AttributeError as e:
            raise ValueError("Expected Hugging Face Gemma model to expose a language_model module.") from e
    cfg = _model_config(lm, "Gemma text")
    _check_model_type(cfg, ("gemma3_text",), "Gemma text")
    params = to_gemma_jax_params(lm, dtype=tdt)
    return GemmaModelWithHead(ModelConfig.from_hf(cfg)), params
