"""``GenerationConfig`` and ``TextGenerationPipeline``: prompts in, text out, over ``Engine.generate``.

Same names, arguments, defaults and validation messages as the reference's ``text_generation.py``
(``GenerationConfig`` :63-90, ``TextGenerationPipeline`` :194-355): the tokenizer (any callable with
``batch_decode``, e.g. an HF tokenizer) turns prompts into ``input_ids`` / ``attention_mask`` arrays, the
engine generates int32 tokens on the GPU, and ``batch_decode`` turns them back into strings.
``from_hf`` loads a supported HF causal LM (local path or hub id) and its tokenizer.
"""
from __future__ import annotations

from collections.abc import Mapping
from collections.abc import Sequence as SequenceABC
from dataclasses import dataclass, field
from typing import Any, Optional

import numpy as np
import torch

from ._checks import normalize_bool as _flag
from ._checks import normalize_count as _count
from ._checks import normalize_dtype
from ._checks import normalize_float as _real
from .engine import Engine, InferenceConfig
from .hf_utils import _normalize_hf_architecture, _normalize_hf_model_name, _validate_hf_dtype, load_model_from_hf


def _kwargs(name: str, value) -> dict:
    if value is None:
        return {}
    if not isinstance(value, Mapping):
        raise TypeError(f"{name} must be a mapping when set, got {type(value)}.")
    return dict(value)


def _check_tokenizer(tokenizer):
    if not callable(tokenizer):
        raise TypeError(f"tokenizer must be callable, got {type(tokenizer)}.")
    if not callable(getattr(tokenizer, "batch_decode", None)):
        raise TypeError("tokenizer must provide a callable batch_decode method.")
    return tokenizer


@dataclass(frozen=True)
class GenerationConfig:
    """Sampling options of one generation call (the keyword arguments of ``Engine.generate``)."""

    seed: int = 0
    max_new_tokens: int = 100
    top_k: int = 0
    top_p: float = 1.0
    min_p: float = 0.0
    temperature: float = 1.0
    fuse_decoding: bool = False
    include_prompt: bool = True

    def __post_init__(self):
        seed = _count("seed", self.seed)
        n = _count("max_new_tokens", self.max_new_tokens)
        k = _count("top_k", self.top_k)
        if n < 0:
            raise ValueError(f"max_new_tokens must be non-negative, got {n}.")
        if k < 0:
            raise ValueError(f"top_k must be non-negative, got {k}.")
        for name, value in (("seed", seed), ("max_new_tokens", n), ("top_k", k),
                            ("top_p", _real("top_p", self.top_p)), ("min_p", _real("min_p", self.min_p)),
                            ("temperature", _real("temperature", self.temperature)),
                            ("fuse_decoding", _flag("fuse_decoding", self.fuse_decoding)),
                            ("include_prompt", _flag("include_prompt", self.include_prompt))):
            object.__setattr__(self, name, value)

    def as_kwargs(self) -> dict:
        return {"seed": self.seed, "max_new_tokens": self.max_new_tokens, "top_k": self.top_k, "top_p": self.top_p,
                "min_p": self.min_p, "temperature": self.temperature, "fuse_decoding": self.fuse_decoding,
                "include_prompt": self.include_prompt}


def _generation_options(config: Optional[GenerationConfig], overrides: dict) -> dict:
    """The config's values updated by keyword overrides, re-validated as one GenerationConfig."""
    if config is None:
        config = GenerationConfig()
    elif not isinstance(config, GenerationConfig):
        raise TypeError(f"generation_config must be a GenerationConfig when set, got {type(config)}.")
    return GenerationConfig(**(config.as_kwargs() | overrides)).as_kwargs()


def _check_token_arrays(input_ids, attention_mask):
    ids = np.asarray(input_ids.cpu() if isinstance(input_ids, torch.Tensor) else input_ids)
    if ids.ndim != 2:
        raise ValueError(f"tokenizer input_ids must be a 2D array, got shape {ids.shape}.")
    if not np.issubdtype(ids.dtype, np.integer):
        raise TypeError(f"tokenizer input_ids must contain integer token ids, got dtype {ids.dtype}.")
    if ids.shape[0] == 0:
        raise ValueError("tokenizer input_ids must contain at least one batch row.")
    if ids.shape[1] == 0:
        raise ValueError("tokenizer input_ids must contain at least one token.")
    if bool((ids < 0).any()):
        raise ValueError("tokenizer input_ids token ids must be non-negative.")
    if attention_mask is None:
        return ids, None
    mask = np.asarray(attention_mask.cpu() if isinstance(attention_mask, torch.Tensor) else attention_mask)
    if mask.ndim != 2:
        raise ValueError(f"tokenizer attention_mask must be a 2D array, got shape {mask.shape}.")
    if not (mask.dtype == np.bool_ or np.issubdtype(mask.dtype, np.integer)):
        raise TypeError(f"tokenizer attention_mask must be boolean or integer, got dtype {mask.dtype}.")
    if mask.shape != ids.shape:
        raise ValueError(
            f"tokenizer attention_mask shape must match input_ids shape; got {mask.shape} and {ids.shape}.")
    if mask.dtype != np.bool_ and bool(((mask != 0) & (mask != 1)).any()):
        raise ValueError("tokenizer attention_mask integer values must be 0 or 1.")
    mask = mask.astype(bool)
    if not bool(mask.any(axis=1).all()):
        raise ValueError("tokenizer attention_mask must contain at least one valid token per batch row.")
    return ids, mask


def _check_generated(tokens) -> np.ndarray:
    t = np.asarray(tokens.cpu() if isinstance(tokens, torch.Tensor) else tokens)
    if t.ndim != 2:
        raise ValueError(f"engine.generate must return a 2D token array, got shape {t.shape}.")
    if not np.issubdtype(t.dtype, np.integer):
        raise TypeError(f"engine.generate must return integer token ids, got dtype {t.dtype}.")
    if bool((t < 0).any()):
        raise ValueError("engine.generate token ids must be non-negative.")
    return t


def _check_decoded(decoded, batch: int) -> list:
    if isinstance(decoded, (str, bytes)) or not isinstance(decoded, SequenceABC):
        raise TypeError(f"tokenizer.batch_decode must return a sequence of strings, got {type(decoded)}.")
    decoded = list(decoded)
    if len(decoded) != batch:
        raise ValueError("tokenizer.batch_decode output batch size must match token batch size; "
                         f"got {len(decoded)} and {batch}.")
    if not all(isinstance(x, str) for x in decoded):
        raise TypeError("tokenizer.batch_decode must return a sequence of strings.")
    return decoded


@dataclass
class TextGenerationPipeline:
    """Tokenize -> ``engine.generate`` -> decode."""

    engine: Any
    tokenizer: Any
    default_tokenize_kwargs: dict = field(default_factory=lambda: {"padding": True})
    default_decode_kwargs: dict = field(default_factory=lambda: {"skip_special_tokens": True})

    def __post_init__(self):
        if not callable(getattr(self.engine, "generate", None)):
            raise TypeError("engine must provide a callable generate method.")
        self.tokenizer = _check_tokenizer(self.tokenizer)
        self.default_tokenize_kwargs = _kwargs("default_tokenize_kwargs", self.default_tokenize_kwargs)
        self.default_decode_kwargs = _kwargs("default_decode_kwargs", self.default_decode_kwargs)

    @classmethod
    def from_hf(cls, name, architecture: str = "auto", model_dtype: str = "float32", engine_dtype: Any = torch.float32,
                inference_config=None, use_tpu: bool = False, cache_stride: int = 256, tokenizer: Any = None,
                tokenizer_kwargs: Optional[dict] = None, model_kwargs: Optional[dict] = None):
        """Pipeline over a supported HF checkpoint (local path or hub id): the model is converted to the
        reference's parameter tree in ``model_dtype`` and packed for this GPU; the tokenizer defaults to
        AutoTokenizer.  The kernels compute in the model's dtype; ``engine_dtype`` is the engine's dtype
        (the caches ``Engine.init_cache`` makes), as in the reference."""
        name = _normalize_hf_model_name(name)
        architecture = _normalize_hf_architecture(architecture)
        model_dtype = _validate_hf_dtype(model_dtype)
        engine_dtype = normalize_dtype("engine_dtype", engine_dtype)
        if inference_config is None:
            inference_config = InferenceConfig()
        elif not isinstance(inference_config, InferenceConfig):
            raise TypeError(f"inference_config must be an InferenceConfig, got {type(inference_config)}.")
        use_tpu = _flag("use_tpu", use_tpu)
        cache_stride = _count("cache_stride", cache_stride)
        if cache_stride <= 0:
            raise ValueError(f"cache_stride must be positive, got {cache_stride}.")
        tokenizer_kwargs = _kwargs("tokenizer_kwargs", tokenizer_kwargs)
        model_kwargs = _kwargs("model_kwargs", model_kwargs)
        if tokenizer is None:
            try:
                from transformers import AutoTokenizer
            except ImportError as e:
                raise ImportError("Please install transformers library.") from e
            tokenizer = AutoTokenizer.from_pretrained(name, **tokenizer_kwargs)
        tokenizer = _check_tokenizer(tokenizer)
        model, params = load_model_from_hf(name, architecture=architecture, dtype=model_dtype, **model_kwargs)
        engine = Engine(model, inference_config, params, dtype=engine_dtype, cache_stride=cache_stride)
        engine.init_params(use_tpu=use_tpu)
        return cls(engine=engine, tokenizer=tokenizer)

    def _encode(self, prompts, tokenize_kwargs=None):
        single = isinstance(prompts, str)
        if single:
            batch = [prompts]
        else:
            if not isinstance(prompts, SequenceABC):
                raise TypeError(f"prompts must be a string or a sequence of strings, got {type(prompts)}.")
            batch = list(prompts)
        if not batch:
            raise ValueError("prompts must contain at least one prompt.")
        if not all(isinstance(p, str) for p in batch):
            raise TypeError("prompts must be a string or a sequence of strings.")
        enc = self.tokenizer(batch, return_tensors="np",
                             **(self.default_tokenize_kwargs | _kwargs("tokenize_kwargs", tokenize_kwargs)))
        ids = self._field(enc, "input_ids")
        mask = self._field(enc, "attention_mask", default=None)
        ids, mask = _check_token_arrays(ids, mask)
        return single, ids, mask

    @staticmethod
    def _field(encoded, name: str, default: Any = ...):
        if isinstance(encoded, Mapping):
            if name in encoded:
                return encoded[name]
        elif hasattr(encoded, name):
            return getattr(encoded, name)
        if default is ...:
            raise ValueError(f"tokenizer output must contain {name!r}.")
        return default

    def generate_tokens(self, prompts, generation_config: Optional[GenerationConfig] = None, tokenize_kwargs=None,
                        **generation_kwargs) -> np.ndarray:
        kwargs = _generation_options(generation_config, generation_kwargs)
        _, ids, mask = self._encode(prompts, tokenize_kwargs=tokenize_kwargs)
        return self._generate_tokens_from_arrays(ids, mask, **kwargs)

    def _generate_tokens_from_arrays(self, input_ids, attention_mask, generation_config=None,
                                     **generation_kwargs) -> np.ndarray:
        kwargs = _generation_options(generation_config, generation_kwargs)
        ids, mask = _check_token_arrays(input_ids, attention_mask)
        tokens = _check_generated(self.engine.generate(ids, attention_mask=mask, **kwargs))
        if tokens.shape[0] != ids.shape[0]:
            raise ValueError("engine.generate token batch size must match input batch size; "
                             f"got {tokens.shape[0]} and {ids.shape[0]}.")
        expected = (ids.shape[1] if kwargs["include_prompt"] else 0) + kwargs["max_new_tokens"]
        if tokens.shape[1] != expected:
            raise ValueError("engine.generate token length must match requested generation length; "
                             f"got {tokens.shape[1]} and expected {expected}.")
        return tokens

    def generate_text(self, prompts, generation_config: Optional[GenerationConfig] = None, tokenize_kwargs=None,
                      decode_kwargs=None, **generation_kwargs):
        kwargs = _generation_options(generation_config, generation_kwargs)
        decode_kwargs = _kwargs("decode_kwargs", decode_kwargs)
        single, ids, mask = self._encode(prompts, tokenize_kwargs=tokenize_kwargs)
        tokens = self._generate_tokens_from_arrays(ids, mask, **kwargs)
        decoded = _check_decoded(self.tokenizer.batch_decode(tokens, **(self.default_decode_kwargs | decode_kwargs)),
                                 batch=tokens.shape[0])
        return decoded[0] if single else decoded
