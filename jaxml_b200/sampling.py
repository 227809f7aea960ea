"""Sampling, as ``inference_engine/sampling.py`` of the reference.

The selection logic (``normalize_sampling_params`` clipping and warnings, ``SamplingMethod.from_values``)
runs on the host; the selected method runs on the GPU: greedy argmax and temperature sampling in
``csrc/sample.cu``, preceded for min-p / top-k / top-p by ``filter_logits_`` (``sampling.py:34-75``,
applied in the reference's order min-p, top-k, top-p), which runs CUDA float32 / bfloat16 logits through
the filter kernel (``csrc/filter.cu``, ``jx_filter_logits``).  The reference's public functions
(``top_k_filtering``, ``top_p_filtering``, ``min_p_filtering``, ``greedy_fn``,
``SamplingMethod.get_sampling_fn``) are here too, with its checks, on torch tensors: CUDA float32 /
bfloat16 logits through the same kernel, host tensors through torch ops; their categorical draw is the
sampling kernel.
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

    def get_sampling_fn(self):
        """sampling.py:169-188: ``greedy_fn``, or ``fn(rng, logits, top_k, top_p, min_p, temp)`` that applies
        the selected filters (min-p, top-k, top-p) and draws ``jax.random.categorical(rng, logits / temp)``
        on the sampling kernel (CUDA logits)."""
        if self.use_greedy:
            return greedy_fn
        pipeline = [fn for use, fn in ((self.use_min_p, min_p_filtering), (self.use_top_k, top_k_filtering),
                                       (self.use_top_p, top_p_filtering)) if use]

        def _sampling_fn(rng, logits, top_k, top_p, min_p, temp):
            x = _validate_logits(logits)
            temp = _normalize_real("temp", temp)
            if temp <= 0.0:
                raise ValueError(f"temp must be positive for non-greedy sampling, got {temp}.")
            for fn in pipeline:
                x = fn(rng, x, top_k, top_p, min_p, temp)
            return categorical(rng, x, temp)

        return _sampling_fn


# ------------------------------------------------------------------------------------------------
# the reference's sampling functions (sampling.py:18-77) on torch tensors
# ------------------------------------------------------------------------------------------------
def _validate_logits(logits) -> torch.Tensor:
    x = logits if isinstance(logits, torch.Tensor) else torch.as_tensor(np.asarray(logits))
    if x.ndim == 0:
        raise ValueError("logits must have at least one dimension for the vocabulary axis.")
    if x.shape[-1] <= 0:
        raise ValueError(f"logits must have a non-empty vocabulary axis, got shape {tuple(x.shape)}.")
    if not x.is_floating_point():
        raise TypeError(f"logits must contain floating point values, got dtype {x.dtype}.")
    if bool((torch.isnan(x) | torch.isposinf(x)).any()):
        raise ValueError("logits must not contain NaN or positive infinity.")
    if x.numel() and not bool(torch.isfinite(x).any(dim=-1).all()):
        raise ValueError("logits must contain at least one finite value per vocabulary row.")
    return x


def _probability(name: str, value) -> float:
    return _clip_value(name, _normalize_real(name, value), 0.0, 1.0)


def _keep_min_p(x: torch.Tensor, min_p: float) -> torch.Tensor:
    keep = _probs(x) >= min_p
    return x.masked_fill(keep.any(dim=-1, keepdim=True) & ~keep, float("-inf"))


def _keep_top_k(x: torch.Tensor, k: int) -> torch.Tensor:
    cutoff = torch.topk(x.float(), min(int(k), x.shape[-1]), dim=-1).values[..., -1:]
    return x.masked_fill(x.float() < cutoff, float("-inf"))


def _keep_top_p(x: torch.Tensor, top_p: float) -> torch.Tensor:
    srt = torch.sort(x.float(), dim=-1, descending=True).values
    cum = torch.cumsum(_probs(srt.to(x.dtype)), dim=-1)
    idx = (cum < top_p).sum(dim=-1, keepdim=True).clamp(max=x.shape[-1] - 1)
    return x.masked_fill(x.float() < torch.gather(srt, -1, idx), float("-inf"))


def _on_kernel(x: torch.Tensor) -> bool:
    return x.device.type == "cuda" and x.dtype in (torch.float32, torch.bfloat16)


def _filter_kernel(x: torch.Tensor, out: torch.Tensor | None, top_k: int, top_p: float,
                   min_p: float) -> torch.Tensor:
    """``jx_filter_logits`` over the rows of CUDA ``x`` [..., V] into ``out`` (a new tensor when None)."""
    from . import _native as N

    V = x.shape[-1]
    rows = x.numel() // V
    xc = x.reshape(rows, V)
    if xc.stride(-1) != 1 or (rows > 1 and xc.stride(0) < V):
        xc = xc.contiguous()
    o = torch.empty_like(xc) if out is None else out.reshape(rows, V)
    if o.stride(-1) != 1 or (rows > 1 and o.stride(0) < V):
        raise ValueError("filter output rows must be contiguous.")
    a = N.JxFilterArgs()
    a.B, a.V = rows, V
    a.logits, a.ld_in = xc.data_ptr(), xc.stride(0) if rows > 1 else V
    a.out, a.ld_out = o.data_ptr(), o.stride(0) if rows > 1 else V
    a.dtype = N.JX_BF16 if x.dtype == torch.bfloat16 else N.JX_F32
    a.top_k = int(min(top_k, 2 ** 31 - 1))
    a.top_p, a.min_p = float(top_p), float(min_p)
    N.check(N.load().jx_filter_logits(a, torch.cuda.current_stream(x.device).cuda_stream), "jx_filter_logits")
    return o.reshape(x.shape) if out is None else out


def top_k_filtering(rng, logits, top_k, *args) -> torch.Tensor:
    """Logits below the k-th largest of their row set to -inf (ties kept); ``top_k <= 0`` keeps all."""
    x = _validate_logits(logits)
    k = _normalize_top_k(top_k)
    if k <= 0:
        return x
    return _filter_kernel(x, None, k, 1.0, 0.0) if _on_kernel(x) else _keep_top_k(x, k)


def top_p_filtering(rng, logits, top_k, top_p, min_p, *args) -> torch.Tensor:
    """Logits below the sorted logit where the cumulative probability reaches ``top_p`` set to -inf;
    ``top_p >= 1`` keeps all, ``top_p <= 0`` keeps the row maximum."""
    x = _validate_logits(logits)
    p = _probability("top_p", top_p)
    if p >= 1.0:
        return x
    if _on_kernel(x):
        return _filter_kernel(x, None, 0, p, 0.0)
    if p <= 0.0:
        return x.masked_fill(x < x.amax(dim=-1, keepdim=True), float("-inf"))
    return _keep_top_p(x, p)


def min_p_filtering(rng, logits, top_k, top_p, min_p, *args) -> torch.Tensor:
    """Tokens whose probability is below ``min_p`` set to -inf, unless no token of the row qualifies."""
    x = _validate_logits(logits)
    p = _probability("min_p", min_p)
    if _on_kernel(x):
        return x if p <= 0.0 else _filter_kernel(x, None, 0, 1.0, p)
    return _keep_min_p(x, p)


def greedy_fn(rng, logits, *args) -> torch.Tensor:
    """The first index of each row's maximum."""
    return _validate_logits(logits).argmax(-1)


_GUMBEL: dict = {}


def categorical(rng, logits: torch.Tensor, temp: float) -> torch.Tensor:
    """``jax.random.categorical(rng, logits / temp)`` over the last axis of CUDA float32 / bfloat16 logits
    on ``jx_sample`` (Gumbel-max, threefry draws by flat element index); int32 of the leading shape."""
    from . import _native as N

    x = _validate_logits(logits)
    if x.device.type != "cuda":
        raise RuntimeError("categorical runs on CUDA logits only (the sampling kernel).")
    if x.dtype not in (torch.float32, torch.bfloat16):
        raise NotImplementedError(f"the sampling kernel takes float32 or bfloat16 logits, got {x.dtype}.")
    key = np.asarray(rng.cpu() if isinstance(rng, torch.Tensor) else rng).astype(np.uint64).reshape(-1)
    if key.shape != (2,):
        raise ValueError(f"rng must be a PRNG key of two uint32 words, got shape {key.shape}.")
    dev = x.device
    V = x.shape[-1]
    rows = x.numel() // V
    if rows > 65535:
        raise NotImplementedError(f"the sampling kernel takes at most 65535 rows, got {rows}.")
    chunk = 4096
    nchunks = (V + chunk - 1) // chunk
    xc = x.reshape(rows, V).contiguous()
    words = np.array([0, 0, key[0] & 0xFFFFFFFF, key[1] & 0xFFFFFFFF], dtype=np.uint32).view(np.int32)
    state = torch.from_numpy(words.copy()).to(dev)
    if dev.index not in _GUMBEL:
        from .runtime import gumbel_table_bf16

        _GUMBEL[dev.index] = gumbel_table_bf16().to(dev)
    ws = torch.empty(rows * nchunks, dtype=torch.int64, device=dev)
    counters = torch.zeros(rows + 1, dtype=torch.int32, device=dev)
    tokens = torch.empty(rows, dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    s = N.JxSampleArgs()
    s.B, s.V, s.logits, s.ld = rows, V, xc.data_ptr(), V
    s.dtype = N.JX_BF16 if x.dtype == torch.bfloat16 else N.JX_F32
    s.greedy, s.temp, s.chunk = 0, float(temp), chunk
    s.vocab_offset, s.vocab_total = 0, V
    s.rng, s.gumbel_tab = state.data_ptr(), _GUMBEL[dev.index].data_ptr()
    s.ws, s.counters, s.finalize = ws.data_ptr(), counters.data_ptr(), 1
    s.ld_tok, s.tokens_out = 1, tokens.data_ptr()
    s.update_pos, s.advance_rng = 0, 0
    s.status = status.data_ptr()
    N.check(N.load().jx_sample(s, 0, torch.cuda.current_stream(dev).cuda_stream), "jx_sample")
    return tokens.reshape(x.shape[:-1])


def _probs(logits: torch.Tensor) -> torch.Tensor:
    """Vocabulary softmax in float32, rounded to the logits' dtype (the reference applies jax.nn.softmax
    to model-dtype logits), returned as float32."""
    x = logits.float()
    e = torch.exp(x - x.amax(dim=-1, keepdim=True))
    return (e / e.sum(dim=-1, keepdim=True)).to(logits.dtype).float()


def filter_logits_(logits: torch.Tensor, out: torch.Tensor, top_k: int, top_p: float, min_p: float) -> torch.Tensor:
    """min-p, then top-k, then top-p filtering of logits ``[B, V]`` into ``out`` (filtered entries -inf),
    inference_engine/sampling.py:34-75.  The reference's own comparisons are kept: min-p keeps
    probabilities >= min_p (unless that keeps nothing in a row), top-k keeps logits >= the k-th largest
    (ties included), top-p keeps logits >= the sorted logit at the count of cumulative probabilities
    below top_p.  Where the reference's JAX arithmetic is not visible from its source: probabilities in
    float32 rounded to the logits' dtype, a cutoff index past the end clamped to the last entry.  CUDA
    float32 / bfloat16 logits run through the filter kernel (one launch, capturable in a CUDA graph; its
    top-p cumulative masses are exact); other tensors through torch ops with a float32 cumulative sum."""
    if _on_kernel(logits):
        return _filter_kernel(logits, out, top_k, top_p, min_p)
    x = logits
    if min_p > 0.0:
        x = _keep_min_p(x, min_p)
    if top_k > 0:
        x = _keep_top_k(x, top_k)
    if top_p < 1.0:
        x = _keep_top_p(x, top_p)
    out.copy_(x)
    return out
