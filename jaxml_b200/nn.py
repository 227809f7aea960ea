"""``jaxml_b200.nn``: the reference's building blocks (``nn/__init__.py``) on CUDA tensors.

``Module``, ``Block``, ``Embed``, ``DenseGeneral``, ``RMSNorm``, ``LayerNorm``, ``RotaryEmbedding``,
``Attention`` and ``AttentionWithRoPE`` take the reference's constructor fields (validated as in its
``setup``) and are used the Flax way:

    m = RMSNorm(hidden_size=4096, eps=1e-5, dtype=torch.bfloat16)
    variables = m.init(key, x)          # {"params": {"weight": ...}}, the reference's names and shapes
    y = m.apply(variables, x)

``apply`` runs on the library's kernels (``jx_norm`` for norms and embedding gathers, ``jx_linear_decode``
/ ``jx_linear_prefill`` / ``jx_linear_f32`` for projections, ``jx_rope_apply``, ``jx_attention``) with the
reference's rounding points, and raises when its inputs are not CUDA tensors: there is no CPU path.
Each ``apply`` reads the library's status word back (one device synchronisation), so device-side range
errors surface as exceptions.  ``init`` validates the inputs like the reference's ``init`` (which runs
``__call__``) but launches nothing; initial values come from torch's generator seeded by the key and
follow the reference's initialisers in distribution only.

Supported combinations are those the kernels implement: float32 or bfloat16 data with parameters of
the same dtype for norms; right-padded (prefix) attention masks; a KV cache that is empty before a
multi-token call.  Anything else raises ``NotImplementedError`` naming the missing case.
"""
from __future__ import annotations

import math
import operator
from collections import OrderedDict
from dataclasses import dataclass
from typing import Optional

import numpy as np
import torch

from . import _native as N
from ._checks import normalize_bool, normalize_count, normalize_dtype, normalize_float
from .cache import KVCache
from .config import ModelConfig

# nn/__init__.py of the reference, in its order (AttentionOutput, GemmaRMSNorm and initializers are here
# too, outside the star-import list as there)
__all__ = ["Attention", "AttentionWithRoPE", "Block", "DenseGeneral", "Embed", "LayerNorm", "Module", "RMSNorm",
           "RotaryEmbedding"]

_REQ = object()


# ------------------------------------------------------------------------------------------------
# initialisers (flax.linen.initializers semantics: variance_scaling, xavier_uniform, zeros, ones)
# ------------------------------------------------------------------------------------------------
class initializers:
    """Factories with the signatures of ``flax.linen.initializers``; each returns
    ``fn(generator, shape, dtype, in_axis, out_axis) -> tensor``."""

    @staticmethod
    def variance_scaling(scale: float = 1.0, mode: str = "fan_in", distribution: str = "truncated_normal",
                         in_axis=-2, out_axis=-1):
        def fn(gen, shape, dtype, in_axis=in_axis, out_axis=out_axis):
            shape = tuple(shape)
            ins = _axes(in_axis, len(shape))
            outs = _axes(out_axis, len(shape))
            recept = int(np.prod([s for i, s in enumerate(shape) if i not in ins and i not in outs])) or 1
            fan_in = int(np.prod([shape[i] for i in ins])) * recept
            fan_out = int(np.prod([shape[i] for i in outs])) * recept
            denom = {"fan_in": fan_in, "fan_out": fan_out, "fan_avg": (fan_in + fan_out) / 2}[mode]
            var = scale / max(denom, 1)
            t = torch.empty(shape, dtype=torch.float32)
            if distribution == "truncated_normal":
                std = math.sqrt(var) / 0.87962566103423978
                torch.nn.init.trunc_normal_(t, std=std, a=-2 * std, b=2 * std, generator=gen)
            elif distribution == "normal":
                t.normal_(0.0, math.sqrt(var), generator=gen)
            elif distribution == "uniform":
                a = math.sqrt(3 * var)
                t.uniform_(-a, a, generator=gen)
            else:
                raise ValueError(f"invalid distribution {distribution!r}")
            return t.to(dtype)
        return fn

    @staticmethod
    def xavier_uniform(in_axis=-2, out_axis=-1):
        return initializers.variance_scaling(1.0, "fan_avg", "uniform", in_axis, out_axis)

    @staticmethod
    def zeros(gen=None, shape=(), dtype=torch.float32, *args, **kwargs):
        return torch.zeros(tuple(shape), dtype=dtype)

    @staticmethod
    def ones(gen=None, shape=(), dtype=torch.float32, *args, **kwargs):
        return torch.ones(tuple(shape), dtype=dtype)


def _axes(a, ndim):
    a = (a,) if isinstance(a, (int, np.integer)) else tuple(a)
    return tuple(int(x) % ndim for x in a)


def _generator(key) -> torch.Generator:
    """torch generator seeded by an int seed or a uint32[2] PRNG key (``prng.prng_key``)."""
    g = torch.Generator()
    if key is None:
        seed = 0
    elif isinstance(key, (int, np.integer)) and not isinstance(key, (bool, np.bool_)):
        seed = int(key)
    else:
        # PRNGKey(s) holds the words (s >> 32, s & 0xFFFFFFFF): read them back as that seed, so that
        # keys made from different small seeds draw differently
        seed = 0
        for v in (torch.as_tensor(key).reshape(-1).to("cpu", torch.int64) & 0xFFFFFFFF).tolist():
            seed = (seed << 32) | int(v)
    g.manual_seed(seed & ((1 << 63) - 1))
    return g


def _device():
    return torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else torch.device("cpu")


# ------------------------------------------------------------------------------------------------
# kernel plumbing
# ------------------------------------------------------------------------------------------------
def _jdt(dtype: torch.dtype) -> int:
    if dtype == torch.bfloat16:
        return N.JX_BF16
    if dtype == torch.float32:
        return N.JX_F32
    raise NotImplementedError(f"the CUDA kernels take float32 or bfloat16 data, got {dtype}.")


def _need_cuda(name: str, *ts):
    for t in ts:
        if t is not None and (not isinstance(t, torch.Tensor) or t.device.type != "cuda"):
            raise RuntimeError(f"{name}: jaxml_b200.nn runs on CUDA tensors only (got {getattr(t, 'device', type(t))}).")


class _DevState:
    """Per-device scratch of the module-level calls: status word, projection workspace and counters."""

    def __init__(self, dev):
        lib = N.load()
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        ws = N.LL()
        N.check(lib.jx_linear_decode_workspace(148, 64, ws), "jx_linear_decode_workspace")
        self.ws = torch.zeros(ws.value, dtype=torch.float32, device=dev)
        self.counters = torch.zeros(1024, dtype=torch.int32, device=dev)

    def counters_for(self, np_rows: int) -> torch.Tensor:
        need = np_rows // 64 + 1
        if self.counters.numel() < need:
            self.counters = torch.zeros(need, dtype=torch.int32, device=self.counters.device)
        return self.counters


_STATE: dict = {}
_PACKED: "OrderedDict" = OrderedDict()   # packed bf16 weights, keyed by the source tensor's identity


def _state(dev) -> _DevState:
    key = (dev.type, dev.index)
    if key not in _STATE:
        _STATE[key] = _DevState(dev)
    return _STATE[key]


def _stream(dev) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _check_status(dev, where: str):
    st = _state(dev).status
    code = int(st.item())
    if code != 0:
        st.zero_()
        raise RuntimeError(f"{where}: device status {code} ({'index out of range' if code == N.JX_ERR_RANGE else 'error'}).")


def _rup(x: int, m: int) -> int:
    return (x + m - 1) // m * m


def _pack(src: torch.Tensor, rows: int, cols: int, ld: int, transposed: int, rp: int, cp: int) -> torch.Tensor:
    out = torch.zeros(rp * cp, dtype=torch.bfloat16, device=src.device)
    sdt = N.JX_BF16 if src.dtype == torch.bfloat16 else N.JX_F32
    N.check(N.load().jx_pack_k128(src.data_ptr(), sdt, rows, cols, ld, transposed, out.data_ptr(), rp, cp,
                                  _stream(src.device)), "jx_pack_k128")
    return out


def _packed_weight(w_kn: torch.Tensor, Np: int, Kp: int) -> torch.Tensor:
    """The [K, N] kernel in the K128 operand layout (bf16), cached per source tensor version."""
    key = (w_kn.data_ptr(), w_kn._version, tuple(w_kn.shape), w_kn.dtype, Np, Kp)
    hit = _PACKED.get(key)
    if hit is not None:
        _PACKED.move_to_end(key)
        return hit[1]
    K, Nn = w_kn.shape
    packed = _pack(w_kn, Nn, K, Nn, 1, Np, Kp)
    _PACKED[key] = (w_kn, packed)        # holds the source so its address is not reused while cached
    # least recently used first out, beyond 64 entries or 2 GiB of packed weights
    while len(_PACKED) > 1 and (len(_PACKED) > 64 or
                                sum(v[1].numel() * 2 for v in _PACKED.values()) > (2 << 30)):
        _PACKED.popitem(last=False)
    return packed


def _dense(x2: torch.Tensor, w_kn: torch.Tensor, bias: Optional[torch.Tensor], dtype: torch.dtype) -> torch.Tensor:
    """[M, K] x [K, N] (+ bias [N]) -> [M, N] in `dtype` on the projection kernels (one rounding of
    acc + bias to the dtype)."""
    lib = N.load()
    dev = x2.device
    M, K = x2.shape
    Nn = w_kn.shape[1]
    st = _state(dev)
    out = torch.empty(M, Nn, dtype=dtype, device=dev)
    e = N.JxEpilogue()
    e.kind, e.M, e.N = N.JX_EPI_STORE, M, Nn
    e.out, e.ldo = out.data_ptr(), Nn
    b = None if bias is None else bias.to(dtype).contiguous()
    e.bias = None if b is None else b.data_ptr()
    if dtype == torch.float32:
        xx = x2.to(torch.float32).contiguous()
        ww = w_kn.to(torch.float32).contiguous()
        N.check(lib.jx_linear_f32(xx.data_ptr(), K, ww.data_ptr(), M, Nn, K, e, 0, _stream(dev)), "jx_linear_f32")
        return out
    if dtype != torch.bfloat16:
        raise NotImplementedError(f"DenseGeneral on the CUDA kernels computes in float32 or bfloat16, got {dtype}.")
    Kp, Np = _rup(K, 128), _rup(Nn, 128)
    wp = _packed_weight(w_kn.contiguous(), Np, Kp)
    xx = x2.to(torch.bfloat16).contiguous()
    if M <= 64:
        Mp = 16 if M <= 16 else (32 if M <= 32 else 64)
        xp = _pack(xx, M, K, K, 0, Mp, Kp)
        cnt = st.counters_for(Np)
        N.check(lib.jx_linear_decode(wp.data_ptr(), xp.data_ptr(), Np, Kp, M, e, st.ws.data_ptr(), st.ws.numel(),
                                     cnt.data_ptr(), st.status.data_ptr(), 148, 0, _stream(dev)), "jx_linear_decode")
    else:
        Mp = _rup(M, 128)
        xp = _pack(xx, M, K, K, 0, Mp, Kp)
        N.check(lib.jx_linear_prefill(xp.data_ptr(), wp.data_ptr(), Mp, Np, Kp, e, st.status.data_ptr(), 0,
                                      _stream(dev)), "jx_linear_prefill")
    return out


def _norm_rows(x2: torch.Tensor, kind: int, eps: float, w: torch.Tensor, b: Optional[torch.Tensor]) -> torch.Tensor:
    dev = x2.device
    M, d = x2.shape
    out = torch.empty_like(x2)
    a = N.JxNormArgs()
    a.M, a.d, a.eps, a.kind, a.kind_pre = M, d, eps, kind, N.JX_NORM_NONE
    a.h, a.ldh = x2.data_ptr(), d
    a.w, a.b = w.data_ptr(), None if b is None else b.data_ptr()
    a.out, a.ldo = out.data_ptr(), d
    a.status = _state(dev).status.data_ptr()
    N.check(N.load().jx_norm(a, _jdt(x2.dtype), 0, _stream(dev)), "jx_norm")
    return out


def _finite(name: str, x: torch.Tensor):
    if x.is_floating_point() and not bool(torch.isfinite(x).all()):
        raise ValueError(f"{name} must contain only finite values.")


def _as_float_input(name: str, x) -> torch.Tensor:
    x = x if isinstance(x, torch.Tensor) else torch.as_tensor(np.asarray(x))
    if not x.is_floating_point():
        raise TypeError(f"{name} must contain floating point values, got dtype {x.dtype}.")
    return x


# ------------------------------------------------------------------------------------------------
# module machinery
# ------------------------------------------------------------------------------------------------
class _Base:
    """Constructor with the reference's dataclass fields (positional in declaration order, or by name)."""

    _fields: tuple = ()

    def __init__(self, *args, **kwargs):
        names = [n for n, _ in self._fields]
        if len(args) > len(names):
            raise TypeError(f"{type(self).__name__} takes at most {len(names)} positional fields.")
        vals = dict(zip(names, args))
        for k, v in kwargs.items():
            if k not in names:
                raise TypeError(f"{type(self).__name__} got an unexpected field {k!r}.")
            if k in vals:
                raise TypeError(f"{type(self).__name__} got multiple values for field {k!r}.")
            vals[k] = v
        for n, default in self._fields:
            if n not in vals:
                if default is _REQ:
                    raise TypeError(f"{type(self).__name__} is missing the required field {n!r}.")
                vals[n] = default
            object.__setattr__(self, n, vals[n])

    def __repr__(self):
        inner = ", ".join(f"{n}={getattr(self, n)!r}" for n, _ in self._fields)
        return f"{type(self).__name__}({inner})"

    # subclasses implement these three
    def _setup(self):
        pass

    def _init_vars(self, gen, *args, **kwargs) -> dict:
        return {"params": {}}

    def _call(self, variables: dict, *args, **kwargs):
        raise NotImplementedError

    def _check_inputs(self, variables: dict, *args, **kwargs):
        pass

    def init(self, key, *args, **kwargs) -> dict:
        """Validates the fields and the example inputs; returns the variables (``{"params": ...}``)."""
        self._setup()
        variables = self._init_vars(_generator(key), *args, **kwargs)
        self._check_inputs(variables, *args, **kwargs)
        return variables

    def apply(self, variables, *args, method=None, **kwargs):
        """Runs the module (or, with ``method``, one of its methods: a function of the class such as
        ``Attention.mha``, or its name) on ``variables``, the Flax way."""
        self._setup()
        if not isinstance(variables, dict):
            raise TypeError(f"variables must be a mapping, got {type(variables)}.")
        if method is None:
            return self._call(variables, *args, **kwargs)
        name = method if isinstance(method, str) else getattr(method, "__name__", None)
        fn = getattr(type(self), name, None) if name else None
        if name is None or name.startswith("_") or not callable(fn):
            raise ValueError(f"{type(self).__name__} has no method {method!r} to apply.")
        return fn(self, variables, *args, **kwargs)


def _params(variables: dict) -> dict:
    if "params" not in variables:
        raise ValueError(f"The key 'params' was not found in variables. Got keys: {list(variables)}.")
    return variables["params"]


class Module(_Base):
    """``nn/module.py:31-52``: kernel initialiser fields shared by the parameterised layers."""

    _fields = (("kernel_init", initializers.variance_scaling), ("kernel_init_args", (1.0, "fan_in", "truncated_normal")),
               ("kernel_axes", ()), ("with_logical_partitioning", True))

    def _setup(self):
        wlp = normalize_bool("with_logical_partitioning", self.with_logical_partitioning)
        if wlp and self.kernel_axes is not None:
            if isinstance(self.kernel_axes, str):
                raise TypeError("kernel_axes must be a tuple of axis names, not a string.")
            for a in tuple(self.kernel_axes):
                if a is not None and not isinstance(a, str):
                    raise TypeError(f"kernel_axes entries must be strings or None, got {type(a)}.")

    def _kernel(self, gen, shape, dtype, in_axis, out_axis):
        if normalize_bool("with_logical_partitioning", self.with_logical_partitioning):
            if not self.kernel_axes:
                raise ValueError("with_logical_partitioning is True. Kernel axes must be specified.")
            if len(tuple(self.kernel_axes)) != len(shape):
                raise ValueError(f"kernel_axes must contain one axis name per kernel dimension, got "
                                 f"{tuple(self.kernel_axes)} for shape {tuple(shape)}.")
        fn = self.kernel_init(*self.kernel_init_args)
        return fn(gen, shape, dtype, in_axis, out_axis).to(_device())


class Block(_Base):
    """``nn/module.py:55-92``: a model building block over a ``ModelConfig``."""

    _fields = (("config", _REQ), ("dtype", torch.float32))

    def _setup(self):
        if not isinstance(self.config, ModelConfig):
            raise TypeError(f"config must be a ModelConfig, got {type(self.config)}.")
        object.__setattr__(self, "dtype", normalize_dtype("dtype", self.dtype))

    num_heads = property(lambda self: self.config.num_heads)
    num_layers = property(lambda self: self.config.num_layers)
    head_dim = property(lambda self: self.config.head_dim)
    hidden_size = property(lambda self: self.config.hidden_size)
    intermediate_size = property(lambda self: self.config.intermediate_size)
    norm_eps = property(lambda self: self.config.norm_eps)
    use_bias = property(lambda self: self.config.use_bias)
    attn_scale = property(lambda self: self.config.attn_scale)


# ------------------------------------------------------------------------------------------------
# norms (nn/norms.py:83-168)
# ------------------------------------------------------------------------------------------------
def _check_hidden(module: str, x, hidden_size: int) -> torch.Tensor:
    x = x if isinstance(x, torch.Tensor) else torch.as_tensor(np.asarray(x))
    if x.ndim == 0:
        raise ValueError(f"{module} input must have at least one dimension.")
    if not x.is_floating_point():
        raise TypeError(f"{module} input must contain floating point values, got dtype {x.dtype}.")
    if x.numel() == 0:
        raise ValueError(f"{module} input must not contain empty axes, got shape {tuple(x.shape)}.")
    if x.shape[-1] != hidden_size:
        raise ValueError(f"{module} hidden dimension mismatch: got {x.shape[-1]} and expected {hidden_size}.")
    _finite(f"{module} input", x)
    return x


class _NormBase(_Base):
    _name = ""
    _kind = N.JX_NORM_RMS

    def _setup(self):
        hs = normalize_count("hidden_size", self.hidden_size)
        eps = normalize_float("eps", self.eps)
        normalize_bool("upcast", self.upcast)
        dt = normalize_dtype("dtype", self.dtype)
        if hs <= 0:
            raise ValueError(f"hidden_size must be positive, got {hs}.")
        if eps <= 0:
            raise ValueError(f"eps must be positive, got {eps}.")
        object.__setattr__(self, "hidden_size", hs)
        object.__setattr__(self, "eps", eps)
        object.__setattr__(self, "dtype", dt)

    def _init_vars(self, gen, *args, **kwargs):
        p = {"weight": torch.ones(self.hidden_size, dtype=self.dtype, device=_device())}
        if getattr(self, "use_bias", False):
            p["bias"] = torch.zeros(self.hidden_size, dtype=self.dtype, device=_device())
        return {"params": p}

    def _check_inputs(self, variables, hidden_states=None, *args, **kwargs):
        _check_hidden(self._name, hidden_states, self.hidden_size)

    def _call(self, variables, hidden_states):
        p = _params(variables)
        x = _check_hidden(self._name, hidden_states, self.hidden_size)
        w = p["weight"]
        b = p.get("bias") if getattr(self, "use_bias", False) else None
        _need_cuda(self._name, x, w, b)
        if not normalize_bool("upcast", self.upcast):
            raise NotImplementedError(f"{self._name}(upcast=False): the CUDA norm kernels compute in float32.")
        if w.dtype != x.dtype or (b is not None and b.dtype != x.dtype):
            raise NotImplementedError(f"{self._name}: parameters ({w.dtype}) must have the input's dtype ({x.dtype}).")
        y = _norm_rows(x.reshape(-1, x.shape[-1]).contiguous(), self._kind, self.eps, w.contiguous(),
                       None if b is None else b.contiguous())
        _check_status(x.device, self._name)
        return y.reshape(x.shape)


class RMSNorm(_NormBase):
    """``nn/norms.py:83-117``: ``weight * (x32 / sqrt(mean(x32^2) + eps)).astype(x.dtype)``."""

    _fields = (("hidden_size", _REQ), ("eps", 1e-6), ("axis_name", "embed"), ("upcast", True), ("dtype", torch.float32))
    _name = "RMSNorm"
    _kind = N.JX_NORM_RMS


class LayerNorm(_NormBase):
    """``nn/norms.py:120-168``: float32 mean / population variance, weight and bias, cast at the end."""

    _fields = (("hidden_size", _REQ), ("eps", 1e-6), ("axis_name", "embed"), ("upcast", True), ("use_bias", True),
               ("dtype", torch.float32))
    _name = "LayerNorm"
    _kind = N.JX_NORM_LAYER

    def _setup(self):
        super()._setup()
        object.__setattr__(self, "use_bias", normalize_bool("use_bias", self.use_bias))


class GemmaRMSNorm(_NormBase):
    """``models/gemma3.py:89-106``: ``((1 + w32) * x32 * rsqrt(mean(x32^2) + eps)).astype(x.dtype)``; the
    weight starts at zero."""

    _fields = (("hidden_size", _REQ), ("eps", 1e-6), ("axis_name", "embed"), ("upcast", True), ("dtype", torch.float32))
    _name = "GemmaRMSNorm"
    _kind = N.JX_NORM_GEMMA

    def _setup(self):
        super()._setup()
        if not normalize_bool("upcast", self.upcast):
            raise ValueError("GemmaRMSNorm requires upcast=True.")

    def _init_vars(self, gen, *args, **kwargs):
        return {"params": {"weight": torch.zeros(self.hidden_size, dtype=self.dtype, device=_device())}}


# ------------------------------------------------------------------------------------------------
# Embed (nn/embedding.py:38-111)
# ------------------------------------------------------------------------------------------------
class Embed(Module):
    """Row gather ``embedding[ids]`` in ``dtype`` (``one_hot`` gives the same values)."""

    _fields = (("num_embeddings", _REQ), ("features", _REQ), ("dtype", torch.float32),
               ("kernel_axes", ("vocab", "embed")), ("one_hot", False)) + tuple(
        f for f in Module._fields if f[0] != "kernel_axes")

    def _setup(self):
        super()._setup()
        V = normalize_count("num_embeddings", self.num_embeddings)
        d = normalize_count("features", self.features)
        normalize_bool("one_hot", self.one_hot)
        object.__setattr__(self, "dtype", normalize_dtype("dtype", self.dtype))
        if V <= 0:
            raise ValueError(f"num_embeddings must be positive, got {V}.")
        if d <= 0:
            raise ValueError(f"features must be positive, got {d}.")
        object.__setattr__(self, "num_embeddings", V)
        object.__setattr__(self, "features", d)

    def _ids(self, inputs) -> torch.Tensor:
        ids = inputs if isinstance(inputs, torch.Tensor) else torch.as_tensor(np.asarray(inputs))
        if ids.numel() == 0:
            raise ValueError("Embed inputs must contain at least one token id.")
        if ids.is_floating_point() or ids.is_complex() or ids.dtype == torch.bool:
            raise ValueError("Input type must be an integer or unsigned integer.")
        if bool((ids < 0).any()):
            raise ValueError("Input token ids must be non-negative.")
        if bool((ids >= self.num_embeddings).any()):
            raise ValueError(f"Input token ids must be less than num_embeddings={self.num_embeddings}.")
        return ids

    def _init_vars(self, gen, inputs=None, *args, **kwargs):
        if inputs is not None:
            ids = inputs if isinstance(inputs, torch.Tensor) else torch.as_tensor(np.asarray(inputs))
            if ids.numel() == 0:
                raise ValueError("Embed inputs must contain at least one token id.")
        return {"params": {"embedding": self._kernel(gen, (self.num_embeddings, self.features), self.dtype, 0, 1)}}

    def _check_inputs(self, variables, inputs=None, *args, **kwargs):
        self._ids(inputs)

    def _call(self, variables, inputs):
        table = _params(variables)["embedding"]
        ids = self._ids(inputs)
        _need_cuda("Embed", table)
        table = table.to(self.dtype).contiguous()
        dev = table.device
        flat = ids.reshape(-1).to(device=dev, dtype=torch.int32).contiguous()
        out = torch.empty(flat.numel(), self.features, dtype=self.dtype, device=dev)
        a = N.JxNormArgs()
        a.M, a.d, a.kind, a.kind_pre = flat.numel(), self.features, N.JX_NORM_NONE, N.JX_NORM_NONE
        a.vocab, a.ids, a.table = self.num_embeddings, flat.data_ptr(), table.data_ptr()
        a.h, a.ldh = out.data_ptr(), self.features
        a.status = _state(dev).status.data_ptr()
        N.check(N.load().jx_norm(a, _jdt(self.dtype), 0, _stream(dev)), "jx_norm (embedding gather)")
        _check_status(dev, "Embed")
        return out.reshape(tuple(ids.shape) + (self.features,))


# ------------------------------------------------------------------------------------------------
# DenseGeneral (nn/linear.py:91-182)
# ------------------------------------------------------------------------------------------------
def _tuple(x):
    return tuple(x) if isinstance(x, (tuple, list)) else (x,)


def _int_value(name: str, v) -> int:
    if isinstance(v, (bool, np.bool_)):
        raise TypeError(f"{name} values must be integers, got {type(v)}.")
    try:
        return operator.index(v)
    except TypeError as e:
        raise TypeError(f"{name} values must be integers, got {type(v)}.") from e


def _shape_dims(name: str, values) -> tuple:
    out = []
    for v in values:
        v = _int_value(name, v)
        if v <= 0:
            raise ValueError(f"{name} values must be positive, got {v}.")
        out.append(v)
    return tuple(out)


def _norm_axes(axes, ndim: int) -> tuple:
    out = []
    for ax in axes:
        ax = _int_value("axis", ax)
        ax = ax if ax >= 0 else ndim + ax
        if ax < 0 or ax >= ndim:
            raise ValueError(f"axis {ax} is out of bounds for input rank {ndim}.")
        out.append(ax)
    if len(set(out)) != len(out):
        raise ValueError(f"axis values must be unique, got {tuple(out)}.")
    return tuple(out)


class DenseGeneral(Module):
    """``dot_general(x.astype(dtype), kernel.astype(dtype))`` over ``axis`` (+ bias in dtype): output
    axes are the non-contracted input axes, then ``features``."""

    _fields = (("features", _REQ), ("axis", -1), ("weight_dtype", torch.float32), ("dtype", torch.float32)) + tuple(
        Module._fields) + (("use_bias", False), ("bias_init", initializers.zeros), ("precision", "default"))

    def _setup(self):
        super()._setup()
        object.__setattr__(self, "features", _shape_dims("features", _tuple(self.features)))
        object.__setattr__(self, "dtype", normalize_dtype("dtype", self.dtype))
        object.__setattr__(self, "weight_dtype", normalize_dtype("weight_dtype", self.weight_dtype))
        object.__setattr__(self, "use_bias", normalize_bool("use_bias", self.use_bias))

    def _prep(self, inputs):
        x = _as_float_input("DenseGeneral inputs", inputs)
        if x.numel() == 0:
            raise ValueError(f"DenseGeneral inputs must not contain empty axes, got shape {tuple(x.shape)}.")
        _finite("DenseGeneral inputs", x)
        axis = _norm_axes(_tuple(self.axis), x.ndim)
        return x, axis

    def _init_vars(self, gen, inputs=None, *args, **kwargs):
        x, axis = self._prep(inputs)
        kshape = tuple(x.shape[a] for a in axis) + self.features
        n_in = len(axis)
        p = {"kernel": self._kernel(gen, kshape, self.weight_dtype, tuple(range(n_in)),
                                    tuple(range(n_in, len(kshape))))}
        if self.use_bias:
            p["bias"] = self.bias_init(gen, self.features, self.weight_dtype).to(_device())
        return {"params": p}

    def _call(self, variables, inputs):
        p = _params(variables)
        x, axis = self._prep(inputs)
        kernel = p["kernel"]
        kshape = tuple(x.shape[a] for a in axis) + self.features
        if tuple(kernel.shape) != kshape:
            raise ValueError(f"kernel shape {tuple(kernel.shape)} does not match the expected {kshape}.")
        bias = p.get("bias") if self.use_bias else None
        _need_cuda("DenseGeneral", x, kernel, bias)
        batch = [i for i in range(x.ndim) if i not in axis]
        xt = x.permute(*batch, *axis)
        bshape = tuple(x.shape[i] for i in batch)
        K = int(np.prod([x.shape[a] for a in axis]))
        Nf = int(np.prod(self.features))
        x2 = xt.reshape(-1, K)
        y = _dense(x2, kernel.reshape(K, Nf), None if bias is None else bias.reshape(Nf), self.dtype)
        _check_status(x.device, "DenseGeneral")
        return y.reshape(bshape + self.features)


# ------------------------------------------------------------------------------------------------
# RotaryEmbedding (nn/position.py:61-232)
# ------------------------------------------------------------------------------------------------
class RotaryEmbedding(_Base):
    """cos / sin tables (float32 angles, cast to the dtype) in the ``cache`` collection, and
    ``apply_rotary_pos_emb`` on the library's RoPE kernel."""

    _fields = (("dim", _REQ), ("max_length", 2048), ("base", 10000.0), ("dtype", torch.float32),
               ("disable_cache", False), ("rotary_pct", 1.0), ("rope_scale", 1.0))

    @staticmethod
    def rotate_half(x: torch.Tensor) -> torch.Tensor:
        h = x.shape[-1] // 2
        return torch.cat([-x[..., h:], x[..., :h]], dim=-1)

    @staticmethod
    def apply_rotary_pos_emb(q, k, cos, sin, position_ids):
        """``nn/position.py:78-141``: q, k ``[B, S, H, hd]``, cos / sin ``[n_pos, rd]``, position_ids
        ``[B or 1, S]``."""
        q, k = _as_float_input("q", q), _as_float_input("k", k)
        cos, sin = _as_float_input("cos", cos), _as_float_input("sin", sin)
        pos = position_ids if isinstance(position_ids, torch.Tensor) else torch.as_tensor(np.asarray(position_ids))
        if q.ndim != 4:
            raise ValueError(f"q must be a 4D array, got shape {tuple(q.shape)}.")
        if k.ndim != 4:
            raise ValueError(f"k must be a 4D array, got shape {tuple(k.shape)}.")
        for name, v in (("q", q), ("k", k)):
            if any(s <= 0 for s in v.shape):
                raise ValueError(f"{name} must not contain empty axes, got shape {tuple(v.shape)}.")
        for name, v in (("q", q), ("k", k), ("cos", cos), ("sin", sin)):
            _finite(name, v)
        if q.shape[:2] != k.shape[:2] or q.shape[-1] != k.shape[-1]:
            raise ValueError(f"q and k must have matching batch, sequence, and head dimensions, got {tuple(q.shape)} "
                             f"and {tuple(k.shape)}.")
        if cos.ndim != 2 or sin.ndim != 2:
            raise ValueError(f"cos and sin must be 2D arrays, got shapes {tuple(cos.shape)} and {tuple(sin.shape)}.")
        if cos.shape != sin.shape:
            raise ValueError(f"cos and sin must have the same shape, got {tuple(cos.shape)} and {tuple(sin.shape)}.")
        if cos.shape[0] <= 0:
            raise ValueError("cos and sin must contain at least one position.")
        rd = cos.shape[-1]
        if rd <= 0 or rd % 2:
            raise ValueError(f"rotary dimension must be positive and even, got {rd}.")
        if rd > q.shape[-1]:
            raise ValueError(f"rotary dimension cannot exceed q/k head dimension, got {rd} and {q.shape[-1]}.")
        if pos.ndim != 2:
            raise ValueError(f"position_ids must be a 2D array, got shape {tuple(pos.shape)}.")
        if pos.shape[1] != q.shape[1] or pos.shape[0] not in (1, q.shape[0]):
            raise ValueError("position_ids shape must be broadcastable to q/k batch and sequence axes, "
                             f"got {tuple(pos.shape)} and {tuple(q.shape[:2])}.")
        if pos.is_floating_point() or pos.dtype == torch.bool:
            raise TypeError(f"position_ids must contain integer positions, got dtype {pos.dtype}.")
        if bool((pos < 0).any()):
            raise ValueError("position_ids must contain non-negative positions.")
        if bool((pos >= cos.shape[0]).any()):
            raise ValueError(f"position_ids must be within rotary table length {cos.shape[0]}.")
        _need_cuda("apply_rotary_pos_emb", q, k, cos, sin)
        if not (q.dtype == k.dtype == cos.dtype == sin.dtype):
            raise NotImplementedError("apply_rotary_pos_emb on the CUDA kernel needs q, k, cos and sin of one dtype, "
                                      f"got {q.dtype}, {k.dtype}, {cos.dtype}, {sin.dtype}.")
        if q.shape[-1] > 256:
            raise NotImplementedError(f"apply_rotary_pos_emb on the CUDA kernel supports head dims up to 256, got {q.shape[-1]}.")
        dev = q.device
        B, S, Hq, hd = q.shape
        Hk = k.shape[2]
        pos = pos.to(device=dev, dtype=torch.int32).expand(B, S).contiguous().reshape(-1)
        qc, kc = q.contiguous(), k.contiguous()
        q_out, k_out = torch.empty_like(qc), torch.empty_like(kc)
        a = N.JxRopeArgs()
        a.M, a.Hq, a.Hk, a.hd, a.rd, a.n_pos = B * S, Hq, Hk, hd, rd, cos.shape[0]
        a.q, a.k, a.q_out, a.k_out = qc.data_ptr(), kc.data_ptr(), q_out.data_ptr(), k_out.data_ptr()
        cc, ss = cos.contiguous(), sin.contiguous()
        a.cos, a.sin, a.pos = cc.data_ptr(), ss.data_ptr(), pos.data_ptr()
        a.status = _state(dev).status.data_ptr()
        N.check(N.load().jx_rope_apply(a, _jdt(q.dtype), 0, _stream(dev)), "jx_rope_apply")
        _check_status(dev, "apply_rotary_pos_emb")
        return q_out, k_out

    @property
    def full_rotate(self):
        return self.rotary_pct >= 1.0

    def _setup(self):
        dim = normalize_count("dim", self.dim)
        ml = normalize_count("max_length", self.max_length)
        base = normalize_float("base", self.base)
        scale = normalize_float("rope_scale", self.rope_scale)
        pct = normalize_float("rotary_pct", self.rotary_pct)
        dt = normalize_dtype("dtype", self.dtype)
        normalize_bool("disable_cache", self.disable_cache)
        if dim <= 0:
            raise ValueError(f"dim must be positive, got {dim}.")
        if ml <= 0:
            raise ValueError(f"max_length must be positive, got {ml}.")
        if base <= 0:
            raise ValueError(f"base must be positive, got {base}.")
        if scale < 1.0:
            raise ValueError(f"a rope scale below 1.0 is most likely a mix-up of dividing and multiplying the "
                             f"positions (they are divided by it), got {scale}.")
        if not 0 < pct <= 1:
            raise ValueError(f"rotary_pct must be in (0, 1], got {pct}.")
        rd = dim if pct >= 1.0 else int(dim * pct)
        if rd <= 0:
            raise ValueError(f"Rotary dimension cannot be less than or equal to 0. The `rotary_pct`({pct}) might be "
                             f"too small relative to the head dim ({dim}).")
        if rd % 2 == 1:
            raise ValueError(f"Rotary dimension cannot be an odd number. Please adjust the `rotary_pct`({pct}) "
                             f"according to the head dim ({dim}).")
        for n, v in (("dim", dim), ("max_length", ml), ("base", base), ("rope_scale", scale), ("rotary_pct", pct),
                     ("dtype", dt)):
            object.__setattr__(self, n, v)
        object.__setattr__(self, "rotary_dim", rd)

    def _inv_freq(self) -> torch.Tensor:
        rd = self.rotary_dim
        return 1.0 / (torch.tensor(self.base, dtype=torch.float32) ** (torch.arange(0, rd, 2, dtype=torch.float32) / rd))

    def get_emb(self, seq_len: int, inv_freq: Optional[torch.Tensor] = None) -> torch.Tensor:
        inv = self._inv_freq() if inv_freq is None else inv_freq.to("cpu", torch.float32)
        t = torch.arange(seq_len, dtype=torch.float32) / torch.tensor(self.rope_scale, dtype=torch.float32)
        freqs = t[:, None] * inv[None, :]
        return torch.cat([freqs, freqs], dim=-1)

    def _init_vars(self, gen, *args, **kwargs):
        cache = {"inv_freq": self._inv_freq().to(_device())}
        if not normalize_bool("disable_cache", self.disable_cache):
            emb = self.get_emb(self.max_length)
            cache["cos_cached"] = torch.cos(emb).to(self.dtype).to(_device())
            cache["sin_cached"] = torch.sin(emb).to(self.dtype).to(_device())
        return {"cache": cache}

    def _x(self, x):
        x = x if isinstance(x, torch.Tensor) else torch.as_tensor(np.asarray(x))
        if x.ndim < 2:
            raise ValueError(f"x must have batch and sequence axes, got shape {tuple(x.shape)}.")
        if any(s <= 0 for s in x.shape):
            raise ValueError(f"x must not contain empty axes, got shape {tuple(x.shape)}.")
        if not x.is_floating_point():
            raise TypeError(f"x must contain floating point values, got dtype {x.dtype}.")
        _finite("x", x)
        return x

    def _seq_len(self, x: torch.Tensor, seq_len, cached_rows: Optional[int]) -> int:
        seq_len = normalize_count("seq_len", x.shape[1] if seq_len is None else seq_len)
        if seq_len <= 0:
            raise ValueError(f"seq_len must be positive, got {seq_len}.")
        if cached_rows is not None and seq_len > cached_rows:
            raise ValueError(f"Cached rotary embeddings only cover max_length={cached_rows}, got seq_len={seq_len}. "
                             "Set disable_cache=True to compute longer embeddings dynamically.")
        return seq_len

    def _check_inputs(self, variables, x=None, seq_len=None, **kwargs):
        x = self._x(x)
        cached = None if normalize_bool("disable_cache", self.disable_cache) else self.max_length
        self._seq_len(x, seq_len, cached)

    def _call(self, variables, x, seq_len=None):
        x = self._x(x)
        cache = variables.get("cache", {})
        if normalize_bool("disable_cache", self.disable_cache):
            seq_len = self._seq_len(x, seq_len, None)
            emb = self.get_emb(seq_len, cache.get("inv_freq"))
            return torch.cos(emb).to(x.dtype).to(x.device), torch.sin(emb).to(x.dtype).to(x.device)
        if "cos_cached" not in cache:
            raise ValueError("RotaryEmbedding variables have no 'cache' collection: pass the variables init returned.")
        cos, sin = cache["cos_cached"], cache["sin_cached"]
        self._seq_len(x, seq_len, cos.shape[0])
        return cos.to(device=x.device, dtype=x.dtype), sin.to(device=x.device, dtype=x.dtype)


# ------------------------------------------------------------------------------------------------
# Attention (nn/attention.py:178-557)
# ------------------------------------------------------------------------------------------------
@dataclass
class AttentionOutput:
    """``outputs.py``: the attention block's output, optional weights and the updated cache."""

    attention_output: torch.Tensor
    attention_weight: Optional[torch.Tensor] = None
    kv_cache: Optional[KVCache] = None


def _check_hidden_states(x) -> torch.Tensor:
    x = x if isinstance(x, torch.Tensor) else torch.as_tensor(np.asarray(x))
    if x.ndim != 3:
        raise ValueError(f"hidden_states must be a 3D array, got shape {tuple(x.shape)}.")
    if any(s <= 0 for s in x.shape):
        raise ValueError(f"hidden_states must not contain empty axes, got shape {tuple(x.shape)}.")
    if not x.is_floating_point():
        raise TypeError(f"hidden_states must contain floating point values, got dtype {x.dtype}.")
    _finite("hidden_states", x)
    return x


def _prefix_lengths(mask: torch.Tensor) -> torch.Tensor:
    """Valid-prefix length per row of a right-padded boolean mask [B, T]."""
    m = mask.to(torch.bool)
    if m.shape[1] > 1 and bool((m[:, :-1].to(torch.int8) < m[:, 1:].to(torch.int8)).any()):
        raise NotImplementedError("attention on the CUDA kernels takes right-padded (prefix) masks only.")
    return m.sum(dim=1).to(torch.int32)


def _mha(q, k, v, lengths, len_add: int, causal: bool, window: int, scale: float, dtype, weights: bool = False):
    """q [B, S, Hq, hd], k / v [B, T, Hkv, hd], keys j < lengths[b] + len_add visible -> [B, S, Hq*hd], and
    with ``weights`` also the softmax probabilities [B, Hq, S, T] (else None)."""
    dev = q.device
    B, S, Hq, hd = q.shape
    T, Hkv = k.shape[1], k.shape[2]
    qc, kc, vc = q.to(dtype).contiguous(), k.to(dtype).contiguous(), v.to(dtype).contiguous()
    out = torch.empty(B * S, Hq * hd, dtype=dtype, device=dev)
    w = torch.empty(B, Hq, S, T, dtype=dtype, device=dev) if weights else None
    ln = lengths.to(device=dev, dtype=torch.int32).contiguous()
    a = N.JxAttnArgs()
    a.B, a.S, a.Hq, a.Hkv, a.hd, a.T = B, S, Hq, Hkv, hd, T
    a.q, a.k, a.v = qc.data_ptr(), kc.data_ptr(), vc.data_ptr()
    a.len_ptr, a.len_add = ln.data_ptr(), len_add
    a.causal, a.window, a.scale = 1 if (causal and S > 1) else 0, window, scale
    a.out, a.ldo, a.out_rp = out.data_ptr(), Hq * hd, 0
    a.status = _state(dev).status.data_ptr()
    a.weights = None if w is None else w.data_ptr()
    N.check(N.load().jx_attention(a, _jdt(dtype), 0, _stream(dev)), "jx_attention")
    return out.reshape(B, S, Hq * hd), w


def _as_states(x) -> torch.Tensor:
    return x if isinstance(x, torch.Tensor) else torch.as_tensor(np.asarray(x))


def _check_states(name: str, x: torch.Tensor):
    """A finite float [batch, sequence, head, head_dim] array (nn/attention.py:48-64)."""
    if x.ndim != 4:
        raise ValueError(f"{name} must be a 4D array, got shape {tuple(x.shape)}.")
    for axis, size in zip(("batch", "sequence", "head", "head_dim"), x.shape):
        if size <= 0:
            raise ValueError(f"{name} {axis} axis must be non-empty, got shape {tuple(x.shape)}.")
    if not x.is_floating_point():
        raise TypeError(f"{name} must contain floating point values, got dtype {x.dtype}.")
    _finite(name, x)


def _optional_positive(name: str, value) -> Optional[int]:
    if value is None:
        return None
    if isinstance(value, (bool, np.bool_)):
        raise TypeError(f"{name} must be an integer when set, got {type(value)}.")
    try:
        value = normalize_count(name, value)
    except TypeError as e:
        raise TypeError(f"{name} must be an integer when set, got {type(value)}.") from e
    if value <= 0:
        raise ValueError(f"{name} must be positive when set, got {value}.")
    return value


class Attention(Block):
    """Projections, optional QK norm, KV-cache update, masked softmax attention (``mha``) and o_proj,
    without positional encoding (``nn/attention.py:449-491``)."""

    _fields = Block._fields + (("kernel_init", initializers.xavier_uniform), ("kernel_init_args", ()),
                               ("with_logical_partitioning", True), ("weight_dtype", torch.float32),
                               ("fused_qkv", False), ("use_alibi", False), ("qk_norm_cls_and_args", None),
                               ("mm_precision", "high"))

    def _setup(self):
        super()._setup()
        object.__setattr__(self, "weight_dtype", normalize_dtype("weight_dtype", self.weight_dtype))
        normalize_bool("with_logical_partitioning", self.with_logical_partitioning)
        normalize_bool("fused_qkv", self.fused_qkv)
        self.num_key_value_heads = self.config.num_key_value_heads
        if self.fused_qkv and self.num_heads != self.num_key_value_heads:
            raise ValueError("fused_qkv requires num_heads to equal num_key_value_heads, "
                             f"got {self.num_heads} and {self.num_key_value_heads}.")

    def _dense(self, features, axes):
        return DenseGeneral(features=features, axis=-1, kernel_init=self.kernel_init,
                            kernel_init_args=self.kernel_init_args,
                            with_logical_partitioning=self.with_logical_partitioning, kernel_axes=axes,
                            dtype=self.dtype, weight_dtype=self.weight_dtype, use_bias=self.use_bias,
                            precision=self.mm_precision)

    def _projections(self):
        H, Hkv, hd = self.num_heads, self.num_key_value_heads, self.head_dim
        if self.fused_qkv:
            mods = {"qkv_proj": self._dense((3, H, hd), ("embed", "qkv", "heads", "head_states"))}
        else:
            mods = {"q_proj": self._dense((H, hd), ("embed", "heads", "head_states")),
                    "k_proj": self._dense((Hkv, hd), ("embed", "heads", "head_states")),
                    "v_proj": self._dense((Hkv, hd), ("embed", "heads", "head_states"))}
        mods["o_proj"] = DenseGeneral(features=self.hidden_size, dtype=self.dtype, weight_dtype=self.weight_dtype,
                                      kernel_init=self.kernel_init, kernel_init_args=(),
                                      with_logical_partitioning=self.with_logical_partitioning,
                                      kernel_axes=("heads_merged", "embed"), use_bias=self.use_bias,
                                      precision=self.mm_precision)
        return mods

    def _qk_norms(self):
        if self.qk_norm_cls_and_args is None:
            return None
        cls, args = self.qk_norm_cls_and_args
        return cls(**args), cls(**args)

    def _init_vars(self, gen, hidden_states=None, *args, **kwargs):
        x = _check_hidden_states(hidden_states)
        mods = self._projections()
        p = {}
        for name, m in mods.items():
            if name == "o_proj":
                ex = torch.zeros(x.shape[:2] + (self.num_heads * self.head_dim,), dtype=x.dtype)
            else:
                ex = x
            m._setup()
            p[name] = m._init_vars(gen, ex)["params"]
        norms = self._qk_norms()
        if norms is not None:
            for name, m in zip(("q_norm", "k_norm"), norms):
                m._setup()
                p[name] = m._init_vars(gen)["params"]
        return {"params": p}

    def _check_inputs(self, variables, hidden_states=None, *args, **kwargs):
        _check_hidden_states(hidden_states)

    def qkv(self, variables, hidden: torch.Tensor):
        p = _params(variables)
        mods = self._projections()
        if self.fused_qkv:
            out = mods["qkv_proj"].apply({"params": p["qkv_proj"]}, hidden)
            q, k, v = out[:, :, 0], out[:, :, 1], out[:, :, 2]
        else:
            q, k, v = (mods[n].apply({"params": p[n]}, hidden) for n in ("q_proj", "k_proj", "v_proj"))
        norms = self._qk_norms()
        if norms is not None:
            q = norms[0].apply({"params": p["q_norm"]}, q)
            k = norms[1].apply({"params": p["k_norm"]}, k)
        return q, k, v

    def repeat_kv(self, variables, key_states, value_states):
        """nn/attention.py:294-319: key / value states [B, T, Hkv, hd] broadcast to the query heads
        [B, T, Hkv * n_rep, hd] (head h reads KV head h // n_rep).  The kernels index the shared head
        instead; this method is for callers that want the repeated arrays."""
        k, v = _as_states(key_states), _as_states(value_states)
        for name, x in (("key_states", k), ("value_states", v)):
            _check_states(name, x)
        if k.shape != v.shape:
            raise ValueError(f"key_states and value_states must have the same shape, got {tuple(k.shape)} and "
                             f"{tuple(v.shape)}.")
        Hkv, hd = self.config.num_key_value_heads, self.config.head_dim
        if k.shape[2] != Hkv:
            raise ValueError(f"key_states and value_states must match config.num_key_value_heads, got {k.shape[2]} "
                             f"and expected {Hkv}.")
        if k.shape[-1] != hd:
            raise ValueError(f"key_states and value_states must match config.head_dim, got {k.shape[-1]} and "
                             f"expected {hd}.")
        n_rep = self.config.num_heads // Hkv
        if n_rep == 1:
            return k, v
        B, T = k.shape[:2]
        return tuple(x[:, :, :, None, :].expand(B, T, Hkv, n_rep, hd).reshape(B, T, Hkv * n_rep, hd) for x in (k, v))

    def mha(self, variables, query_states, key_states, value_states, attention_mask=None, causal=True,
            sliding_window=None, alibi_slope=None, softmax_fp32=True, output_attentions=False):
        """nn/attention.py:321-400 on ``jx_attention``: ``(attn_output [B, S, H, hd], weights [B, H, S, T] or
        None)`` for q [B, S, H, hd] and k / v [B, T, H, hd] (already repeated).  Same checks and
        messages; the kernel takes prefix (right-padded) masks, a float32 softmax and no ALiBi slope,
        and anything else raises ``NotImplementedError``."""
        q, k, v = _as_states(query_states), _as_states(key_states), _as_states(value_states)
        for name, x in (("query_states", q), ("key_states", k), ("value_states", v)):
            _check_states(name, x)
        if k.shape != v.shape:
            raise ValueError(f"key_states and value_states must have the same shape, got {tuple(k.shape)} and "
                             f"{tuple(v.shape)}.")
        if q.shape[0] != k.shape[0] or q.shape[2:] != k.shape[2:]:
            raise ValueError("query_states and key_states must have matching batch, head count, and head dimension, "
                             f"got {tuple(q.shape)} and {tuple(k.shape)}.")
        window = _optional_positive("sliding_window", sliding_window)
        causal = normalize_bool("causal", causal)
        softmax_fp32 = normalize_bool("softmax_fp32", softmax_fp32)
        output_attentions = normalize_bool("output_attentions", output_attentions)
        if alibi_slope is not None:
            slope = _as_states(alibi_slope)
            if slope.ndim != 1:
                raise ValueError("alibi_slope must be a 1D array with one value per attention head, got shape "
                                 f"{tuple(slope.shape)}.")
            if slope.shape[0] != q.shape[2]:
                raise ValueError(f"alibi_slope must contain {q.shape[2]} values, got {slope.shape[0]}.")
            if not slope.is_floating_point():
                raise TypeError(f"alibi_slope must contain floating point values, got dtype {slope.dtype}.")
            _finite("alibi_slope", slope)
        B, S, T = q.shape[0], q.shape[1], k.shape[1]
        lengths = None
        if attention_mask is not None:
            m = _as_states(attention_mask)
            if tuple(m.shape) != (B, T):
                raise ValueError("attention_mask shape must match attention batch and key length, "
                                 f"got {tuple(m.shape)} and {(B, T)}.")
            if m.is_floating_point() or m.is_complex():
                raise TypeError(f"attention_mask must be boolean or integer, got dtype {m.dtype}.")
            if m.dtype != torch.bool and bool(((m != 0) & (m != 1)).any()):
                raise ValueError("attention_mask integer values must be 0 or 1.")
            lengths = _prefix_lengths(m.to(torch.bool))
        if alibi_slope is not None:
            raise NotImplementedError("ALiBi attention is not implemented by the CUDA attention kernels.")
        if not softmax_fp32:
            raise NotImplementedError("softmax_fp32=False: the CUDA attention kernels compute the softmax in float32.")
        if window is not None and S > 1 and not causal:
            raise NotImplementedError("a sliding window on a non-causal multi-query call is not implemented by the "
                                      "CUDA attention kernels.")
        _need_cuda("Attention.mha", q, k, v)
        if lengths is None:
            lengths = torch.full((B,), T, dtype=torch.int32)
        out, w = _mha(q, k, v, lengths, 0, causal, window or 0, float(self.attn_scale), q.dtype,
                      weights=output_attentions)
        _check_status(q.device, "Attention.mha")
        return out.reshape(B, S, q.shape[2], q.shape[3]), w

    def apply_kv_cache(self, variables, key_states, value_states, attention_mask, kv_cache):
        """nn/attention.py:280-292: ``(keys, values, mask, cache)`` after writing this call's key / value
        states into ``kv_cache`` (or the states themselves and None without a cache)."""
        if kv_cache is not None and not isinstance(kv_cache, KVCache):
            raise TypeError(f"kv_cache must be a KVCache instance or None, got {type(kv_cache)}.")
        if kv_cache is None:
            return key_states, value_states, attention_mask, None
        kv_cache = kv_cache.update(key_states, value_states, attention_mask)
        return kv_cache.k, kv_cache.v, kv_cache.mask, kv_cache

    def post_mha(self, variables, attn_output: torch.Tensor) -> torch.Tensor:
        o = self._projections()["o_proj"]
        return o.apply({"params": _params(variables)["o_proj"]}, attn_output.reshape(attn_output.shape[:2] + (-1,)))

    @staticmethod
    def _preflight(output_attentions, use_flash, kv_cache) -> bool:
        """The call's flags and cache type, checked before any projection (nn/attention.py:139-144, 448-517)."""
        output_attentions = normalize_bool("output_attentions", output_attentions)
        if normalize_bool("use_flash", use_flash):
            raise NotImplementedError("JAX flash attention is not enabled in jaxml yet.")
        if kv_cache is not None and not isinstance(kv_cache, KVCache):
            raise TypeError(f"kv_cache must be a KVCache instance or None, got {type(kv_cache)}.")
        return output_attentions

    def _attend(self, variables, hidden, q, k, v, attention_mask, kv_cache, sliding_window, output_attentions,
                use_flash):
        output_attentions = self._preflight(output_attentions, use_flash, kv_cache)
        window = 0 if sliding_window is None else normalize_count("sliding_window", sliding_window)
        if window < 0:
            raise ValueError(f"sliding_window must be positive when set, got {window}.")
        B, S = hidden.shape[:2]
        if kv_cache is not None:
            if kv_cache.k is not None and S > 1:
                raise NotImplementedError("a multi-token call on a populated KV cache (chunked prefill) is not "
                                          "implemented by the CUDA attention kernels.")
            kv_cache = kv_cache.update(k, v, attention_mask)
            keys, values = kv_cache.k, kv_cache.v
            lengths, len_add = kv_cache.pos_id[:, 0], 1
            if S > 1:
                _prefix_lengths(kv_cache.mask)
        else:
            keys, values = k, v
            mask = torch.ones(B, S, dtype=torch.bool, device=hidden.device) if attention_mask is None else (
                attention_mask if isinstance(attention_mask, torch.Tensor) else torch.as_tensor(attention_mask))
            lengths, len_add = _prefix_lengths(mask.to(hidden.device)), 0
        _need_cuda("Attention", q, keys, values)
        out, w = _mha(q, keys, values, lengths, len_add, True, window, float(self.attn_scale), self.dtype,
                      weights=output_attentions)
        _check_status(q.device, "Attention")
        return AttentionOutput(attention_output=self.post_mha(variables, out), attention_weight=w, kv_cache=kv_cache)

    def _call(self, variables, hidden_states, attention_mask=None, position_ids=None, kv_cache=None,
              output_attentions=False, use_flash=False, sliding_window=None, **kwargs):
        x = _check_hidden_states(hidden_states)
        self._preflight(output_attentions, use_flash, kv_cache)
        if self.config.use_alibi:
            raise NotImplementedError("ALiBi attention is not implemented by the CUDA attention kernels.")
        if position_ids is not None:
            raise NotImplementedError("MHA with given position_ids is not implemented.")
        q, k, v = self.qkv(variables, x)
        return self._attend(variables, x, q, k, v, attention_mask, kv_cache, sliding_window, output_attentions,
                            use_flash)


def _cos_sin_pair(cos_sin):
    """nn/attention.py:164-175: a (cos, sin) pair of arrays."""
    if cos_sin is None:
        raise ValueError("AttentionWithRoPE requires cos_sin.")
    if isinstance(cos_sin, (torch.Tensor, np.ndarray)):
        raise TypeError("cos_sin must be a pair of cosine and sine arrays, not a single array.")
    try:
        cos, sin = cos_sin
    except TypeError as e:
        raise TypeError(f"cos_sin must be a pair of cosine and sine arrays, got {type(cos_sin)}.") from e
    except ValueError as e:
        raise ValueError("cos_sin must contain exactly two arrays: cosine and sine.") from e
    return cos, sin


class AttentionWithRoPE(Attention):
    """``nn/attention.py:494-557``: RoPE on q and k (``cos_sin`` from ``RotaryEmbedding``) before the cache
    update."""

    def _setup(self):
        super()._setup()
        if self.config.use_alibi:
            raise NotImplementedError("Having ALiBi and RoPE together is not intended (though the math works).")

    def _call(self, variables, hidden_states, cos_sin=None, attention_mask=None, position_ids=None, kv_cache=None,
              output_attentions=False, use_flash=False, sliding_window=None):
        x = _check_hidden_states(hidden_states)
        self._preflight(output_attentions, use_flash, kv_cache)
        cos, sin = _cos_sin_pair(cos_sin)
        q, k, v = self.qkv(variables, x)
        if attention_mask is None and kv_cache is not None and kv_cache.mask is not None:
            attention_mask = kv_cache.next_mask
        if position_ids is None:
            if kv_cache is not None and kv_cache.pos_id is not None:
                position_ids = kv_cache.next_pos_id
            else:
                position_ids = torch.arange(k.shape[1], device=x.device)[None].expand(k.shape[0], -1)
        q, k = RotaryEmbedding.apply_rotary_pos_emb(q, k, cos, sin, position_ids)
        return self._attend(variables, x, q, k, v, attention_mask, kv_cache, sliding_window, output_attentions,
                            use_flash)
