"""Sampling-method selection, as ``inference_engine/sampling.py:90-188`` of the reference.

The selection logic (``normalize_sampling_params`` clipping and warnings, ``SamplingMethod.from_values``)
runs on the host; the selected method runs on the GPU: greedy argmax and temperature sampling in
``csrc/sample.cu``, preceded for min-p / top-k / top-p by ``filter_logits_`` (``sampling.py:34-72``,
applied in the reference's order min-p, top-k, top-p) on the device logits.
"""
from __future__ import annotations

import logging
import math
import numbers
import operator
from dataclasses import dataclass

import numpy as np

import torch

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
    def uses_filters(self) -> bool:
        return not self.use_greedy and (self.use_top_k or self.use_top_p or self.use_min_p)


def _probs(logits: torch.Tensor) -> torch.Tensor:
    """Vocabulary softmax in float32, rounded to the logits' dtype (the reference applies jax.nn.softmax
    to model-dtype logits), returned as float32."""
    x = logits.float()
    e = torch.exp(x - x.amax(dim=-1, keepdim=True))
    return (e / e.sum(dim=-1, keepdim=True)).to(logits.dtype).float()


def filter_logits_(logits: torch.Tensor, out: torch.Tensor, top_k: int, top_p: float, min_p: float) -> torch.Tensor:
    """min-p, then top-k, then top-p filtering of device logits ``[B, V]`` into ``out`` (filtered entries
    -inf), inference_engine/sampling.py:34-72.  The reference's own comparisons are kept: min-p keeps
    probabilities >= min_p (unless that keeps nothing in a row), top-k keeps logits >= the k-th largest
    (ties included), top-p keeps logits >= the sorted logit at the count of cumulative probabilities
    below top_p.  Where the reference's JAX arithmetic is not visible from its source: probabilities in
    float32 rounded to the logits' dtype, the cumulative sum in float32, a cutoff index past the end
    clamped to the last entry.  Device tensor ops only (capturable in a CUDA graph)."""
    neg = float("-inf")   # a scalar: no host-to-device copy while a CUDA graph is being captured
    x = logits
    if min_p > 0.0:
        keep = _probs(x) >= min_p
        x = x.masked_fill(keep.any(dim=-1, keepdim=True) & ~keep, neg)
    if top_k > 0:
        k = min(int(top_k), x.shape[-1])
        cutoff = torch.topk(x.float(), k, dim=-1).values[..., -1:]
        x = x.masked_fill(x.float() < cutoff, neg)
    if top_p < 1.0:
        srt = torch.sort(x.float(), dim=-1, descending=True).values
        cum = torch.cumsum(_probs(srt.to(x.dtype)), dim=-1)
        idx = (cum < top_p).sum(dim=-1, keepdim=True).clamp(max=x.shape[-1] - 1)
        x = x.masked_fill(x.float() < torch.gather(srt, -1, idx), neg)
    out.copy_(x)
    return out
