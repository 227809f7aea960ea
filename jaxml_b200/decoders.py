"""The reference's decoder building blocks on the library's kernels, and the layer-by-layer model call.

``LlamaMLP`` / ``LlamaDecoder`` (models/llama.py:43-143), ``GPTNeoXMLP`` / ``GPTNeoXDecoder``
(models/gpt_neox.py:44-140) and ``GemmaMLP`` / ``GemmaDecoder`` (models/gemma3.py:41-179) are
``jaxml_b200.nn`` blocks: the reference's fields, parameter names (``self_attn``, ``mlp``,
``input_layernorm`` ...) and ``init`` / ``apply`` use.  Their projections and attention are the ``nn``
modules (``DenseGeneral``, ``Attention`` / ``AttentionWithRoPE``); the residual adds and the norms after
them are one ``jx_norm`` launch each (``h + a`` rounded to the dtype, then the norm of the sum), and the
MLP activation is ``jx_mlp_act``.  The hidden states are cast to the block's dtype on entry.

``layered_forward`` is the model call of models/llama.py:161-225 (gpt_neox.py:158-222,
gemma3.py:215-283) through these blocks.  The model classes use it for the calls the fused decode /
prefill runtime does not take: KV caches, explicit position ids and per-layer hidden states.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import numpy as np
import torch

from . import _native as N
from . import nn
from ._checks import normalize_bool
from .cache import KVCache

__all__ = ["DecoderOutput", "LlamaMLP", "LlamaDecoder", "GPTNeoXMLP", "GPTNeoXDecoder", "GemmaMLP", "GemmaDecoder",
           "layered_forward"]


@dataclass
class DecoderOutput:
    """``outputs.py``: one decoder layer's output hidden states, updated cache and attention weights."""

    hidden_states: torch.Tensor
    kv_cache: Optional[KVCache] = None
    attention_weight: Optional[torch.Tensor] = None


# ------------------------------------------------------------------------------------------------
# kernels
# ------------------------------------------------------------------------------------------------
def _mlp_act(gate: torch.Tensor, up: Optional[torch.Tensor], kind: int) -> torch.Tensor:
    """``jx_mlp_act``: dtype(dtype(act(gate)) * up) for the GLU kinds, dtype(gelu_erf(gate)) otherwise."""
    dev = gate.device
    F = gate.shape[-1]
    g = gate.contiguous()
    u = None if up is None else up.to(g.dtype).contiguous()
    out = torch.empty_like(g)
    M = g.numel() // F
    N.check(N.load().jx_mlp_act(g.data_ptr(), F, None if u is None else u.data_ptr(), F, out.data_ptr(), F, M, F, kind,
                                nn._jdt(g.dtype), 0, nn._stream(dev)), "jx_mlp_act")
    return out


def _add_norm(h: torch.Tensor, a: Optional[torch.Tensor] = None, *, kind: int = N.JX_NORM_NONE, w=None, b=None,
              eps: float = 1e-6, kind_pre: int = N.JX_NORM_NONE, w_pre=None, b_pre=None):
    """One ``jx_norm`` launch over the rows of ``h`` [..., d]: ``h' = dtype(h + pre(a))`` when ``a`` is given
    (``pre`` = the ``kind_pre`` norm with ``w_pre`` / ``b_pre``, or nothing), then ``out = norm(h')`` when
    ``kind`` is a norm.  Returns ``(h', out)`` as new tensors (``out`` None without a norm)."""
    dev = h.device
    d = h.shape[-1]
    hh = h.reshape(-1, d).contiguous()
    if a is not None:
        hh = hh.clone()          # the kernel writes the sum back into h
    M = hh.shape[0]
    out = torch.empty_like(hh) if kind != N.JX_NORM_NONE else None
    aa = None if a is None else a.to(hh.dtype).reshape(-1, d).contiguous()
    args = N.JxNormArgs()
    args.M, args.d, args.eps, args.kind, args.kind_pre = M, d, float(eps), kind, kind_pre
    args.h, args.ldh = hh.data_ptr(), d
    if aa is not None:
        args.a, args.lda = aa.data_ptr(), d
    args.w_pre, args.b_pre = _ptr(w_pre), _ptr(b_pre)
    args.w, args.b = _ptr(w), _ptr(b)
    if out is not None:
        args.out, args.ldo = out.data_ptr(), d
    args.status = nn._state(dev).status.data_ptr()
    N.check(N.load().jx_norm(args, nn._jdt(hh.dtype), 0, nn._stream(dev)), "jx_norm")
    nn._check_status(dev, "decoder residual / norm")
    return hh.reshape(h.shape), None if out is None else out.reshape(h.shape)


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


def _embed(table: torch.Tensor, ids: torch.Tensor, dtype: torch.dtype, scale: float) -> torch.Tensor:
    """Row gather ``table[ids]`` in ``dtype`` times ``scale`` (rounded once; 0 = no scale) on ``jx_norm``."""
    dev = table.device
    V, d = table.shape
    t = table.to(dtype).contiguous()
    flat = ids.reshape(-1).to(device=dev, dtype=torch.int32).contiguous()
    out = torch.empty(flat.numel(), d, dtype=dtype, device=dev)
    a = N.JxNormArgs()
    a.M, a.d, a.kind, a.kind_pre = flat.numel(), d, N.JX_NORM_NONE, N.JX_NORM_NONE
    a.vocab, a.ids, a.table, a.embed_scale = V, flat.data_ptr(), t.data_ptr(), float(scale)
    a.h, a.ldh = out.data_ptr(), d
    a.status = nn._state(dev).status.data_ptr()
    N.check(N.load().jx_norm(a, nn._jdt(dtype), 0, nn._stream(dev)), "jx_norm (embedding gather)")
    nn._check_status(dev, "embedding")
    return out.reshape(tuple(ids.shape) + (d,))


def _weight(p: dict, name: str, dtype) -> Optional[torch.Tensor]:
    w = p.get(name)
    if w is None:
        return None
    w = w if isinstance(w, torch.Tensor) else torch.as_tensor(np.asarray(w))
    return w.to(device=nn._device(), dtype=dtype).contiguous()


def _hidden(module: str, x, hidden_size: int, dtype) -> torch.Tensor:
    """models/_utils.py:37-49 (``validate_mlp_input``): a finite float [B, S, d] array, cast to ``dtype``."""
    x = x if isinstance(x, torch.Tensor) else torch.as_tensor(np.asarray(x))
    if x.ndim != 3:
        raise ValueError(f"{module} input must be a 3D array, got shape {tuple(x.shape)}.")
    if not x.is_floating_point():
        raise TypeError(f"{module} input must contain floating point values, got dtype {x.dtype}.")
    if any(s <= 0 for s in x.shape):
        raise ValueError(f"{module} input must not contain empty axes, got shape {tuple(x.shape)}.")
    if x.shape[-1] != hidden_size:
        raise ValueError(f"{module} hidden dimension mismatch: got {x.shape[-1]} and expected {hidden_size}.")
    nn._finite(f"{module} input", x)
    return x.to(dtype)


# ------------------------------------------------------------------------------------------------
# MLPs (models/llama.py:43-95, gpt_neox.py:44-88, gemma3.py:41-95)
# ------------------------------------------------------------------------------------------------
class _MLP(nn.Block):
    _fields = nn.Block._fields + (("kernel_init", nn.initializers.xavier_uniform), ("act_fn", None))
    _name = ""
    _kind = N.JX_EPI_GLU_SILU
    _glu = True
    _precision = "default"

    def _setup(self):
        super()._setup()
        if self.act_fn is not None:
            raise NotImplementedError(f"{self._name}: act_fn other than the default; the activation kernel computes "
                                      "silu (Llama), tanh-approximate gelu (Gemma) and exact gelu (GPT-NeoX).")

    def _mods(self) -> dict:
        def dense(features, axes):
            return nn.DenseGeneral(features=features, dtype=self.dtype, kernel_init=self.kernel_init,
                                   kernel_init_args=(), with_logical_partitioning=True, kernel_axes=axes,
                                   use_bias=self.use_bias, precision=self._precision)

        F, d = self.intermediate_size, self.hidden_size
        mods = {"gate_proj": dense(F, ("embed", "intermediate"))} if self._glu else {}
        mods["up_proj"] = dense(F, ("embed", "intermediate"))
        mods["down_proj"] = dense(d, ("intermediate", "embed"))
        return mods

    def _init_vars(self, gen, x=None, *args, **kwargs):
        x = _hidden(self._name, x, self.hidden_size, self.dtype)
        p = {}
        for name, m in self._mods().items():
            m._setup()
            ex = torch.zeros(tuple(x.shape[:-1]) + (self.intermediate_size,), dtype=x.dtype) if name == "down_proj" else x
            p[name] = m._init_vars(gen, ex)["params"]
        return {"params": p}

    def _check_inputs(self, variables, x=None, *args, **kwargs):
        _hidden(self._name, x, self.hidden_size, self.dtype)

    def _call(self, variables, x, **kwargs):
        x = _hidden(self._name, x, self.hidden_size, self.dtype)
        p = nn._params(variables)
        mods = self._mods()
        up = mods["up_proj"].apply({"params": p["up_proj"]}, x)
        if self._glu:
            gate = mods["gate_proj"].apply({"params": p["gate_proj"]}, x)
            act = _mlp_act(gate, up, self._kind)
        else:
            act = _mlp_act(up, None, self._kind)
        return mods["down_proj"].apply({"params": p["down_proj"]}, act)


class LlamaMLP(_MLP):
    """``down_proj(silu(gate_proj(x)) * up_proj(x))`` (models/llama.py:43-95)."""

    _name = "LlamaMLP"
    _kind = N.JX_EPI_GLU_SILU


class GemmaMLP(_MLP):
    """``down_proj(gelu_tanh(gate_proj(x)) * up_proj(x))`` (models/gemma3.py:41-95)."""

    _name = "GemmaMLP"
    _kind = N.JX_EPI_GLU_GELU_TANH


class GPTNeoXMLP(_MLP):
    """``down_proj(gelu_erf(up_proj(x)))`` with ``precision="high"`` (models/gpt_neox.py:44-88)."""

    _name = "GPTNeoXMLP"
    _kind = N.JX_EPI_ACT_GELU_ERF
    _glu = False
    _precision = "high"


# ------------------------------------------------------------------------------------------------
# decoder layers (models/llama.py:98-143, gpt_neox.py:91-140, gemma3.py:109-179)
# ------------------------------------------------------------------------------------------------
class _Decoder(nn.Block):
    _arch = ""
    _mlp_cls = LlamaMLP
    _norm_cls = nn.RMSNorm
    _norm_kind = N.JX_NORM_RMS
    _norm_names = ("input_layernorm", "post_attention_layernorm")

    def _setup(self):
        super()._setup()
        cfg = self.config
        if self._arch and cfg.hidden_size != cfg.num_heads * cfg.head_dim:
            raise ValueError(f"{self._arch} hidden_size must equal num_heads * head_dim; got hidden_size="
                             f"{cfg.hidden_size}, num_heads={cfg.num_heads}, head_dim={cfg.head_dim}.")

    def _attn(self):
        cls = nn.AttentionWithRoPE if self.config.use_rope else nn.Attention
        return cls(self.config, dtype=self.dtype)

    def _norm(self):
        return self._norm_cls(hidden_size=self.hidden_size, eps=self.norm_eps, dtype=self.dtype, upcast=True)

    def _init_vars(self, gen, hidden_states=None, *args, **kwargs):
        x = _hidden(type(self).__name__, hidden_states, self.hidden_size, self.dtype)
        attn, mlp = self._attn(), self._mlp_cls(self.config, dtype=self.dtype)
        attn._setup()
        mlp._setup()
        p = {"self_attn": attn._init_vars(gen, x)["params"], "mlp": mlp._init_vars(gen, x)["params"]}
        for name in self._norm_names:
            m = self._norm()
            m._setup()
            p[name] = m._init_vars(gen)["params"]
        return {"params": p}

    def _check_inputs(self, variables, hidden_states=None, *args, **kwargs):
        _hidden(type(self).__name__, hidden_states, self.hidden_size, self.dtype)

    def _nw(self, p, name):
        return _weight(p[name], "weight", self.dtype), _weight(p[name], "bias", self.dtype)

    def _attention(self, p, x, cos_sin, attention_mask, position_ids, kv_cache, output_attentions, sliding_window=None):
        attn = self._attn()
        kw = dict(attention_mask=attention_mask, position_ids=position_ids, kv_cache=kv_cache,
                  output_attentions=output_attentions, sliding_window=sliding_window)
        if self.config.use_rope:
            kw["cos_sin"] = cos_sin
        return attn.apply({"params": p["self_attn"]}, x, **kw)

    def _call(self, variables, hidden_states, cos_sin=None, attention_mask=None, position_ids=None, kv_cache=None,
              output_attentions=False, training=False):
        p = nn._params(variables)
        normalize_bool("output_attentions", output_attentions)
        h = _hidden(type(self).__name__, hidden_states, self.hidden_size, self.dtype)
        return self._layer(p, h, cos_sin, attention_mask, position_ids, kv_cache, output_attentions)

    def _layer(self, p, h, cos_sin, attention_mask, position_ids, kv_cache, output_attentions) -> DecoderOutput:
        eps, kind = self.norm_eps, self._norm_kind
        w_in, b_in = self._nw(p, "input_layernorm")
        w_post, b_post = self._nw(p, "post_attention_layernorm")
        _, x = _add_norm(h, kind=kind, w=w_in, b=b_in, eps=eps)
        out = self._attention(p, x, cos_sin, attention_mask, position_ids, kv_cache, output_attentions)
        # h = h + attn, then the post-attention norm of the sum, in one launch
        h, x = _add_norm(h, out.attention_output, kind=kind, w=w_post, b=b_post, eps=eps)
        m = self._mlp_cls(self.config, dtype=self.dtype).apply({"params": p["mlp"]}, x)
        h, _ = _add_norm(h, m)
        return DecoderOutput(hidden_states=h, kv_cache=out.kv_cache, attention_weight=out.attention_weight)


class LlamaDecoder(_Decoder):
    """``h += attn(rmsnorm(h)); h += mlp(rmsnorm(h))`` (models/llama.py:98-143)."""

    _arch = "Llama"


class GPTNeoXDecoder(_Decoder):
    """LayerNorm decoder with the fused ``qkv_proj`` and the parallel residual
    ``mlp(ln2(h)) + attn(ln1(h)) + h`` when ``use_parallel_residual`` (models/gpt_neox.py:91-140)."""

    _arch = "GPT-NeoX"
    _mlp_cls = GPTNeoXMLP
    _norm_cls = nn.LayerNorm
    _norm_kind = N.JX_NORM_LAYER

    def _attn(self):
        cls = nn.AttentionWithRoPE if self.config.use_rope else nn.Attention
        return cls(self.config, fused_qkv=True, dtype=self.dtype, mm_precision="high")

    def _norm(self):
        return nn.LayerNorm(hidden_size=self.hidden_size, eps=self.norm_eps, dtype=self.dtype, upcast=True,
                            use_bias=True)

    def _layer(self, p, h, cos_sin, attention_mask, position_ids, kv_cache, output_attentions) -> DecoderOutput:
        if not self.config.use_parallel_residual:
            return super()._layer(p, h, cos_sin, attention_mask, position_ids, kv_cache, output_attentions)
        eps, kind = self.norm_eps, self._norm_kind
        w_in, b_in = self._nw(p, "input_layernorm")
        w_post, b_post = self._nw(p, "post_attention_layernorm")
        _, x = _add_norm(h, kind=kind, w=w_in, b=b_in, eps=eps)
        out = self._attention(p, x, cos_sin, attention_mask, position_ids, kv_cache, output_attentions)
        _, x2 = _add_norm(h, kind=kind, w=w_post, b=b_post, eps=eps)
        m = self._mlp_cls(self.config, dtype=self.dtype).apply({"params": p["mlp"]}, x2)
        s, _ = _add_norm(m, out.attention_output)      # dtype(mlp + attn)
        h, _ = _add_norm(h, s)                         # dtype((mlp + attn) + h)
        return DecoderOutput(hidden_states=h, kv_cache=out.kv_cache, attention_weight=out.attention_weight)


class GemmaDecoder(_Decoder):
    """Gemma3 layer: QK norm, sliding-window attention on local layers (``use_sliding``), and the post-
    attention / pre- and post-feed-forward Gemma RMS norms (models/gemma3.py:109-179)."""

    _fields = _Decoder._fields + (("use_sliding", False),)
    _mlp_cls = GemmaMLP
    _norm_cls = nn.GemmaRMSNorm
    _norm_kind = N.JX_NORM_GEMMA
    _norm_names = ("input_layernorm", "post_attention_layernorm", "pre_feedforward_layernorm",
                   "post_feedforward_layernorm")

    def _setup(self):
        super()._setup()
        normalize_bool("use_sliding", self.use_sliding)
        if not self.config.use_rope:
            raise ValueError("Gemma3 decoder requires use_rope=True.")

    def _attn(self):
        args = dict(hidden_size=self.head_dim, eps=self.norm_eps, dtype=self.dtype)
        return nn.AttentionWithRoPE(self.config, dtype=self.dtype, qk_norm_cls_and_args=(nn.GemmaRMSNorm, args))

    def _norm(self):
        return nn.GemmaRMSNorm(hidden_size=self.hidden_size, eps=self.norm_eps, dtype=self.dtype)

    def _attention(self, p, x, cos_sin, attention_mask, position_ids, kv_cache, output_attentions, sliding_window=None):
        # QK-norm weights in the compute dtype (the norm kernels take parameters of the input's dtype)
        sa = dict(p["self_attn"])
        for name in ("q_norm", "k_norm"):
            if name in sa:
                sa[name] = {"weight": _weight(sa[name], "weight", self.dtype)}
        sw = self.config.sliding_window if normalize_bool("use_sliding", self.use_sliding) else None
        return super()._attention({"self_attn": sa}, x, cos_sin, attention_mask, position_ids, kv_cache,
                                  output_attentions, sliding_window=sw)

    def _layer(self, p, h, cos_sin, attention_mask, position_ids, kv_cache, output_attentions) -> DecoderOutput:
        eps, G = self.norm_eps, N.JX_NORM_GEMMA
        w_in, _ = self._nw(p, "input_layernorm")
        w_pa, _ = self._nw(p, "post_attention_layernorm")
        w_pf, _ = self._nw(p, "pre_feedforward_layernorm")
        w_po, _ = self._nw(p, "post_feedforward_layernorm")
        _, x = _add_norm(h, kind=G, w=w_in, eps=eps)
        out = self._attention(p, x, cos_sin, attention_mask, position_ids, kv_cache, output_attentions)
        # h = h + post_attention_norm(attn); x = pre_feedforward_norm(h)
        h, x = _add_norm(h, out.attention_output, kind=G, w=w_pf, eps=eps, kind_pre=G, w_pre=w_pa)
        m = self._mlp_cls(self.config, dtype=self.dtype).apply({"params": p["mlp"]}, x)
        # h = h + post_feedforward_norm(mlp)
        h, _ = _add_norm(h, m, kind_pre=G, w_pre=w_po, eps=eps)
        return DecoderOutput(hidden_states=h, kv_cache=out.kv_cache, attention_weight=out.attention_weight)


DECODERS = {"llama": LlamaDecoder, "neox": GPTNeoXDecoder, "gemma3": GemmaDecoder}


# ------------------------------------------------------------------------------------------------
# the model call, layer by layer (models/llama.py:161-225, gpt_neox.py:158-222, gemma3.py:215-283)
# ------------------------------------------------------------------------------------------------
def _cached_sequence_length(kv_caches) -> Optional[int]:
    """models/_utils.py:190-203: the populated caches' common sequence length (None without caches)."""
    if kv_caches is None:
        return None
    n = None
    for idx, c in enumerate(kv_caches):
        if c is None or c.k is None:
            continue
        if n is None:
            n = c.k.shape[1]
        elif c.k.shape[1] != n:
            raise ValueError("kv_caches populated entries must share cached sequence length; "
                             f"got {n} and {c.k.shape[1]} at index {idx}.")
    return n


def _rope_vars(cfg, dtype, base: float, scale: float):
    rope = nn.RotaryEmbedding(dim=cfg.head_dim, max_length=cfg.max_position_embeddings, base=base, dtype=dtype,
                              rotary_pct=cfg.rotary_pct, rope_scale=scale)
    return rope, rope.init(0, torch.zeros(1, 1, 1))


def layered_forward(family: str, cfg, dtype, body: dict, ids: torch.Tensor, attention_mask: Optional[torch.Tensor],
                    position_ids: Optional[torch.Tensor], kv_caches: Optional[tuple], cached_len: Optional[int],
                    rope_cache: dict, output_attentions: bool = False):
    """Embedding, the decoder layers and the final norm over ``body`` (the stack's parameters, leaves on
    the device in ``dtype``).  ``ids`` [B, S] with placeholders already mapped to 0; ``attention_mask``
    the prepared boolean mask or None (populated caches); ``cached_len`` the caches' sequence length (the
    rotary table length the reference checks).  Returns ``(last_hidden_state, next_caches, hidden_states,
    attention_weights)``: hidden_states the input of every layer followed by the final-norm output, the
    weights [B, H, S, T] of every layer when ``output_attentions`` (else Nones)."""
    d = cfg.hidden_size
    scale = 0.0
    if family == "gemma3":
        # inputs_embeds *= hidden_size ** 0.5 in the dtype (the scalar rounded to the dtype first)
        scale = float(torch.tensor(d ** 0.5, dtype=torch.float32).to(dtype).float())
    h = _embed(body["embed_tokens"]["embedding"], ids, dtype, scale)
    key = (dtype, cfg.head_dim, cfg.max_position_embeddings, cfg.rope_theta, cfg.rope_scale, cfg.rotary_pct)
    if rope_cache.get("key") != key:
        rope_cache.clear()
        rope_cache["key"] = key
        rope_cache["global"] = _rope_vars(cfg, dtype, cfg.rope_theta, cfg.rope_scale)
        if family == "gemma3":
            rope_cache["local"] = _rope_vars(cfg, dtype, 10000.0, 1.0)
    rope, rv = rope_cache["global"]
    cos_sin = rope.apply(rv, h, seq_len=cached_len)
    cos_sin_local = None
    stride = 1
    if family == "gemma3":
        lrope, lrv = rope_cache["local"]
        cos_sin_local = lrope.apply(lrv, h, seq_len=cached_len)
        stride = cfg.sliding_window_pattern or 1
    hidden, caches, weights = [], [], []
    for idx in range(cfg.num_layers):
        hidden.append(h)
        if family == "gemma3":
            dec = GemmaDecoder(cfg, dtype=dtype, use_sliding=((idx + 1) % stride) > 0)
            cs = cos_sin_local if (idx + 1) % stride else cos_sin
        else:
            dec = DECODERS[family](cfg, dtype=dtype)
            cs = cos_sin
        cache = None if kv_caches is None else kv_caches[idx]
        out = dec.apply({"params": body[f"layers_{idx}"]}, h, cos_sin=cs, attention_mask=attention_mask,
                        position_ids=position_ids, kv_cache=cache, output_attentions=output_attentions)
        h = out.hidden_states
        caches.append(out.kv_cache)
        weights.append(out.attention_weight)
    fw = _weight(body["norm"], "weight", dtype)
    fb = _weight(body["norm"], "bias", dtype)
    kind = {"llama": N.JX_NORM_RMS, "neox": N.JX_NORM_LAYER, "gemma3": N.JX_NORM_GEMMA}[family]
    _, h = _add_norm(h, kind=kind, w=fw, b=fb, eps=cfg.norm_eps)
    hidden.append(h)
    return h, tuple(caches), tuple(hidden), tuple(weights)


def device_tree(tree, dtype: torch.dtype, dev: torch.device):
    """The parameter tree with every floating leaf as a ``dtype`` tensor on ``dev`` (the reference casts
    parameters to the compute dtype where it uses them)."""
    if isinstance(tree, dict):
        return {k: device_tree(v, dtype, dev) for k, v in tree.items()}
    t = tree if isinstance(tree, torch.Tensor) else torch.as_tensor(np.asarray(tree))
    if t.is_floating_point():
        return t.to(device=dev, dtype=dtype).contiguous()
    return t.to(dev)

