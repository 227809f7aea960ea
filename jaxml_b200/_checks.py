"""Argument normalisation shared by the API classes.

The messages follow the reference's helpers word for word so callers that match them with regexes keep
working (``_normalize_count`` / ``_normalize_bool`` / ``_normalize_float`` in ``config.py``,
``cache.py``, ``inference_engine/engine.py`` and ``nn/*.py`` of the reference).
"""
from __future__ import annotations

import math
import operator
from numbers import Real
from typing import Any

import numpy as np
import torch

_DTYPES = {
    "float32": torch.float32, "fp32": torch.float32, "f32": torch.float32,
    "bfloat16": torch.bfloat16, "bf16": torch.bfloat16,
    "float16": torch.float16, "fp16": torch.float16,
}


def normalize_count(name: str, value: Any) -> int:
    if isinstance(value, (bool, np.bool_)):
        raise TypeError(f"{name} must be an integer, got {type(value)}.")
    try:
        return operator.index(value)
    except TypeError as e:
        raise TypeError(f"{name} must be an integer, got {type(value)}.") from e


def normalize_bool(name: str, value: Any) -> bool:
    if isinstance(value, (bool, np.bool_)):
        return bool(value)
    raise TypeError(f"{name} must be a boolean, got {type(value)}.")


def normalize_float(name: str, value: Any) -> float:
    if isinstance(value, (bool, np.bool_)) or not isinstance(value, Real):
        raise TypeError(f"{name} must be a real number, got {type(value)}.")
    value = float(value)
    if not math.isfinite(value):
        raise ValueError(f"{name} must be finite, got {value}.")
    return value


def normalize_dtype(name: str, value: Any) -> torch.dtype:
    """Accepts torch dtypes, numpy dtypes and dtype names (``"bfloat16"``, ``jnp.bfloat16``-style names)."""
    if value is None:
        raise TypeError(f"{name} must be a valid dtype, got {value!r}.")
    if isinstance(value, torch.dtype):
        return value
    key = getattr(value, "__name__", None) or getattr(value, "name", None) or str(value)
    key = str(key).replace("torch.", "").replace("jnp.", "").lower()
    if key in _DTYPES:
        return _DTYPES[key]
    try:
        npd = np.dtype(value)
    except TypeError as e:
        raise TypeError(f"{name} must be a valid dtype, got {value!r}.") from e
    if npd.name in _DTYPES:
        return _DTYPES[npd.name]
    raise TypeError(f"{name} must be a valid dtype, got {value!r}.")


def dtype_name(dtype: torch.dtype) -> str:
    return {torch.float32: "float32", torch.bfloat16: "bfloat16", torch.float16: "float16"}[dtype]
