"""Sampling-method selection, as ``inference_engine/sampling.py:90-188`` of the reference.

The selection logic (``normalize_sampling_params`` clipping and warnings, ``SamplingMethod.from_values``)
runs on the host; the selected method runs on the GPU (``csrc/sample.cu``): greedy argmax and plain
temperature sampling.  The min-p / top-k / top-p filters are not implemented on the device yet and
raise ``NotImplementedError`` when selected.
"""
from __future__ import annotations

import logging
import math
import numbers
import operator
from dataclasses import dataclass

import numpy as np

from ._checks import normalize_bool

logger = logging.getLogger(__name__)


def _clip_value(name: str, value, lo, hi):
    if value < lo:
        logger.warning("Parameter %s is lower than %f (%f), setting it to be %f", name, lo, value, lo)
        return lo
    if value > hi:
        logger.warning("Parameter %s is higher than %f (%f), setting it to be %f", name, hi, value, hi)
        return hi
    return value


def _normalize_top_k(top_k) -> int:
    if isinstance(top_k, (bool, np.bool_)):
        raise TypeError(f"top_k must be an integer, got {type(top_k)}.")
    try:
        top_k = operator.index(top_k)
    except TypeError as e:
        raise TypeError(f"top_k must be an integer, got {type(top_k)}.") from e
    return _clip_value("top_k", top_k, 0, float("inf"))


def _normalize_real(name: str, value) -> float:
    if isinstance(value, (bool, np.bool_)) or not isinstance(value, numbers.Real):
        raise TypeError(f"{name} must be a real number, got {type(value)}.")
    value = float(value)
    if not math.isfinite(value):
        raise ValueError(f"{name} must be finite, got {value}.")
    return value


@dataclass(frozen=True)
class SamplingParams:
    top_k: int
    top_p: float
    min_p: float
    temp: float


def normalize_sampling_params(top_k, top_p, min_p, temp) -> SamplingParams:
    return SamplingParams(
        top_k=_normalize_top_k(top_k),
        top_p=_clip_value("top_p", _normalize_real("top_p", top_p), 0.0, 1.0),
        min_p=_clip_value("min_p", _normalize_real("min_p", min_p), 0.0, 1.0),
        temp=_clip_value("temp", _normalize_real("temp", temp), 0.0, float("inf")),
    )


@dataclass(frozen=True)
class SamplingMethod:
    use_top_k: bool
    use_top_p: bool
    use_min_p: bool
    use_greedy: bool

    def __post_init__(self):
        for name in ("use_top_k", "use_top_p", "use_min_p", "use_greedy"):
            object.__setattr__(self, name, normalize_bool(name, getattr(self, name)))

    @classmethod
    def from_values(cls, top_k, top_p, min_p, temp) -> "SamplingMethod":
        p = normalize_sampling_params(top_k=top_k, top_p=top_p, min_p=min_p, temp=temp)
        greedy = p.temp <= 0.0 or p.top_p <= 0.0 or p.top_k == 1
        return cls(use_top_k=p.top_k > 0 and not greedy, use_top_p=p.top_p < 1.0 and not greedy,
                   use_min_p=p.min_p > 0.0 and not greedy, use_greedy=greedy)

    @property
    def device_supported(self) -> bool:
        return self.use_greedy or not (self.use_top_k or self.use_top_p or self.use_min_p)

    def require_device_support(self):
        if not self.device_supported:
            raise NotImplementedError(
                "min-p / top-k / top-p filtering is not implemented on the GPU path; use greedy decoding "
                "(temperature <= 0) or plain temperature sampling."
            )
