"""Oracle (test infrastructure only): jaxml's decoder math restated on torch CPU tensors.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` import this
module, and only to compare against; the product path never calls it.

Every function follows the reference's JAX/Flax code op by op, including where it rounds to the
model dtype (bfloat16 configs round after every op; float32 configs are plain float32):

* dense projections          -- ``nn/linear.py:119-182`` (inputs and kernel cast to dtype, f32-accumulated
                                dot, result in dtype, bias added in dtype)
* RMSNorm / LayerNorm         -- ``nn/norms.py:83-117`` / ``nn/norms.py:120-168``
* Gemma RMSNorm               -- ``models/gemma3.py:89-106``
* rotary tables / rotation    -- ``nn/position.py:147-232`` / ``nn/position.py:71-141``
* attention (mask semantics)  -- ``nn/attention.py:321-400``, GQA ``:294-319``, RoPE path ``:501-557``
* KV cache update             -- ``cache.py:183-243``; positions ``utils.py:183-194``; rollback/resize ``cache.py:245-282``
* Llama / NeoX / Gemma3 stacks -- ``models/llama.py:82-273``, ``models/gpt_neox.py:44-272``, ``models/gemma3.py:41-331``
* input preparation           -- ``models/_utils.py:61-217``
* generation loop             -- ``inference_engine/engine.py:488-610``, ``_generate.py:185-405``
* sampling                    -- ``inference_engine/sampling.py:75-188`` (see ``oracle/threefry.py``)

Pinning: the float32 path is checked against HF transformers' eager torch models at the reference's
own tolerance (``atol=1e-5``) and greedy-token identity, exactly as the reference's tests do
(``tests/test_llama.py``, ``tests/test_neox.py``, ``tests/test_gemma.py``), plus the reference's
known-answer tests for masks, caches and sampling filters (``tests/test_oracle_*.py``).  The bfloat16
rounding points follow the reference source; they are not pinned against a running JAX (JAX is not
installed on either machine).
"""
from __future__ import annotations

import contextlib
import math
from dataclasses import dataclass
from typing import Optional

import numpy as np
import torch

from . import threefry

F32 = torch.float32


def _f32(x: torch.Tensor) -> torch.Tensor:
    return x.to(F32)


def _scalar(value: float, dtype) -> torch.Tensor:
    """A weak-typed Python scalar meeting an array of ``dtype``: converted to ``dtype`` first."""
    return torch.tensor(value, dtype=F32).to(dtype).to(F32)


# ----------------------------------------------------------------------------------------------
# Layers
# ----------------------------------------------------------------------------------------------
_ACC = [F32]


@contextlib.contextmanager
def accumulation(acc_dtype):
    """Runs every float32 step (projection and attention sums, softmax, norm statistics) in ``acc_dtype``
    (float64) instead: a variant of the restatement, not the restatement, used by tests to measure how far
    the bfloat16 results of the same math move when only the precision / order of those sums changes.
    The model-dtype rounding points are the same."""
    old = _ACC[0]
    _ACC[0] = acc_dtype
    try:
        yield
    finally:
        _ACC[0] = old


def dense(x: torch.Tensor, kernel: torch.Tensor, bias: Optional[torch.Tensor], dtype, n_in: int = 1) -> torch.Tensor:
    """``DenseGeneral`` contracting the last ``n_in`` axes of ``x`` with the first ``n_in`` of ``kernel``."""
    acc = _ACC[0]
    xin = x.to(dtype).to(acc)
    w = kernel.to(dtype).to(acc)
    kdim = int(np.prod(kernel.shape[:n_in]))
    out_shape = tuple(x.shape[: x.ndim - n_in]) + tuple(kernel.shape[n_in:])
    y = (xin.reshape(-1, kdim) @ w.reshape(kdim, -1)).reshape(out_shape).to(dtype)
    if bias is not None:
        y = (_f32(y) + _f32(bias.to(dtype))).to(dtype)
    return y


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    in_dtype = x.dtype
    x32 = x.to(_ACC[0])
    ms = (x32 * x32).mean(-1, keepdim=True)
    y = (x32 / torch.sqrt(ms + torch.tensor(eps, dtype=_ACC[0]))).to(in_dtype)
    out_dtype = torch.promote_types(weight.dtype, in_dtype)
    return (_f32(weight) * _f32(y)).to(out_dtype)


def gemma_rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    in_dtype = x.dtype
    x32 = x.to(_ACC[0])
    ms = (x32 * x32).mean(-1, keepdim=True)
    y = x32 * (1.0 / torch.sqrt(ms + torch.tensor(eps, dtype=_ACC[0])))
    return ((weight.to(_ACC[0]) + 1.0) * y).to(in_dtype)


def layernorm(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor], eps: float) -> torch.Tensor:
    in_dtype = x.dtype
    acc = _ACC[0]
    x32 = x.to(acc)
    mean = x32.mean(-1, keepdim=True)
    var = ((x32 - mean) ** 2).mean(-1, keepdim=True)
    out = (x32 - mean) / torch.sqrt(var + torch.tensor(eps, dtype=acc)) * weight.to(acc)
    if bias is not None:
        out = out + bias.to(acc)
    return out.to(in_dtype)


def rotary_dim(head_dim: int, rotary_pct: float) -> int:
    return head_dim if rotary_pct >= 1.0 else int(head_dim * rotary_pct)


def rope_tables(head_dim: int, rotary_pct: float, base: float, rope_scale: float, max_len: int, dtype):
    """``RotaryEmbedding.setup``: float32 angles, cos/sin rounded to the model dtype."""
    rd = rotary_dim(head_dim, rotary_pct)
    inv_freq = 1.0 / (torch.tensor(base, dtype=F32) ** (torch.arange(0, rd, 2, dtype=F32) / rd))
    t = torch.arange(max_len, dtype=F32) / torch.tensor(rope_scale, dtype=F32)
    freqs = t[:, None] * inv_freq[None, :]
    emb = torch.cat([freqs, freqs], dim=-1)
    return torch.cos(emb).to(dtype), torch.sin(emb).to(dtype)


def _rotate_half(x: torch.Tensor) -> torch.Tensor:
    h = x.shape[-1] // 2
    return torch.cat([-x[..., h:], x[..., :h]], dim=-1)


def apply_rope(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, position_ids: torch.Tensor):
    rd = cos.shape[-1]
    c = cos[position_ids][:, :, None, :]
    s = sin[position_ids][:, :, None, :]

    def rot(x):
        xr = x[..., :rd]
        a = (_f32(xr) * _f32(c)).to(x.dtype)
        b = (_f32(_rotate_half(xr)) * _f32(s)).to(x.dtype)
        e = (_f32(a) + _f32(b)).to(x.dtype)
        if rd < x.shape[-1]:
            e = torch.cat([e, x[..., rd:]], dim=-1)
        return e

    return rot(q), rot(k)


def repeat_kv(x: torch.Tensor, n_rep: int) -> torch.Tensor:
    if n_rep == 1:
        return x
    b, t, h, d = x.shape
    return x[:, :, :, None, :].expand(b, t, h, n_rep, d).reshape(b, t, h * n_rep, d)


def mha(q, k, v, attention_mask, causal: bool, sliding_window: Optional[int], attn_scale: float, return_weights=False):
    """``Attention.mha``: q ``[B,S,H,hd]``, k/v ``[B,T,H,hd]`` (already repeated), mask ``[B,T]`` bool."""
    dtype = q.dtype
    acc = _ACC[0]
    x = torch.einsum("bshn,bthn->bhst", q.to(acc), k.to(acc)).to(dtype)
    x = _f32((_f32(x) * _scalar(attn_scale, dtype)).to(dtype))
    _, _, q_len, k_len = x.shape
    neg = torch.zeros_like(x, dtype=torch.bool)
    if causal and q_len != 1:
        neg |= torch.triu(torch.ones(q_len, k_len, dtype=torch.bool), diagonal=1)[None, None]
    if sliding_window is not None:
        if q_len != 1:
            neg |= torch.tril(torch.ones(q_len, k_len, dtype=torch.bool), diagonal=-sliding_window)[None, None]
        elif attention_mask is not None:
            positions = torch.arange(k_len)[None, :]
            current = torch.where(attention_mask, positions, torch.full_like(positions, -1)).max(-1, keepdim=True).values
            window = positions >= current - sliding_window + 1
            neg |= ~window[:, None, None, :]
        else:
            neg[..., : k_len - sliding_window] = True
    if attention_mask is not None:
        neg |= ~attention_mask[:, None, None, :]
    x = x.masked_fill(neg, float("-inf"))
    all_masked = torch.isneginf(x).all(-1, keepdim=True)
    x = torch.where(all_masked, torch.zeros_like(x), x)
    # jax.nn.softmax: exp(x - max) / sum(exp(x - max)) with a true division (torch's CPU softmax
    # multiplies by the reciprocal, which rounds differently)
    x = x.to(acc)
    e = torch.exp(x - x.max(-1, keepdim=True).values)
    p = (e / e.sum(-1, keepdim=True)).to(dtype)
    out = torch.einsum("bhst,bthn->bshn", p.to(acc), v.to(acc)).to(dtype)
    return (out, p) if return_weights else out


# ----------------------------------------------------------------------------------------------
# KV cache (functional, as ``cache.py``)
# ----------------------------------------------------------------------------------------------
def default_pos_ids(mask: torch.Tensor) -> torch.Tensor:
    """``utils.get_default_pos_ids``: last True index per row (argmax of mask * arange)."""
    t = mask.shape[1]
    return torch.argmax(mask.to(torch.int64) * torch.arange(t)[None, :], dim=1).to(torch.int32)[:, None]


@dataclass
class OracleKVCache:
    max_seq_len: int
    dtype: torch.dtype
    k: Optional[torch.Tensor] = None
    v: Optional[torch.Tensor] = None
    mask: Optional[torch.Tensor] = None
    pos_id: Optional[torch.Tensor] = None

    def update(self, k, v, mask):
        k = k.to(self.dtype)
        v = v.to(self.dtype)
        if self.k is None:
            if mask is None:
                mask = torch.ones(k.shape[:2], dtype=torch.bool)
            mask = mask.to(torch.bool)
            pos = default_pos_ids(mask)
            pad = self.max_seq_len - k.shape[1]
            kp = torch.cat([k, torch.zeros((k.shape[0], pad) + tuple(k.shape[2:]), dtype=k.dtype)], dim=1)
            vp = torch.cat([v, torch.zeros((v.shape[0], pad) + tuple(v.shape[2:]), dtype=v.dtype)], dim=1)
            mp = torch.cat([mask, torch.zeros((mask.shape[0], pad), dtype=torch.bool)], dim=1)
            return OracleKVCache(self.max_seq_len, self.dtype, kp, vp, mp, pos)
        assert k.shape[1] == 1
        nxt = self.pos_id + 1
        if bool((nxt >= self.max_seq_len).any()):
            raise ValueError(f"Cannot decode past max_seq_len={self.max_seq_len}.")
        b = torch.arange(k.shape[0])
        nk, nv, nm = self.k.clone(), self.v.clone(), self.mask.clone()
        nk[b, nxt[:, 0]] = k[:, 0]
        nv[b, nxt[:, 0]] = v[:, 0]
        nm[b, nxt[:, 0]] = True
        return OracleKVCache(self.max_seq_len, self.dtype, nk, nv, nm, nxt)

    def rollback(self, n: int):
        prev = self.pos_id - n
        keep = torch.arange(self.k.shape[1])[None, :] <= prev
        nk = torch.where(keep[..., None, None], self.k, torch.zeros_like(self.k))
        nv = torch.where(keep[..., None, None], self.v, torch.zeros_like(self.v))
        return OracleKVCache(self.max_seq_len, self.dtype, nk, nv, keep, prev)

    def resize(self, new_size: int):
        if self.k is None:
            return OracleKVCache(new_size, self.dtype)
        if new_size > self.max_seq_len:
            pad = new_size - self.max_seq_len
            b = self.k.shape[0]
            nk = torch.cat([self.k, torch.zeros((b, pad) + tuple(self.k.shape[2:]), dtype=self.k.dtype)], 1)
            nv = torch.cat([self.v, torch.zeros((b, pad) + tuple(self.v.shape[2:]), dtype=self.v.dtype)], 1)
            nm = torch.cat([self.mask, torch.zeros((b, pad), dtype=torch.bool)], 1)
            return OracleKVCache(new_size, self.dtype, nk, nv, nm, self.pos_id)
        return OracleKVCache(new_size, self.dtype, self.k[:, :new_size], self.v[:, :new_size],
                             self.mask[:, :new_size], self.pos_id)


# ----------------------------------------------------------------------------------------------
# Decoder stacks
# ----------------------------------------------------------------------------------------------
def _t(x) -> torch.Tensor:
    if isinstance(x, torch.Tensor):
        return x.detach().cpu()
    return torch.from_numpy(np.asarray(x))


def _root(params, family: str):
    p = params["params"] if "params" in params else params
    return p, p["gpt_neox" if family == "neox" else "model"]


def _attention_block(family, cfg, lp, h, cos, sin, attention_mask, position_ids, cache, sliding_window, dtype):
    """``AttentionWithRoPE.__call__`` (``nn/attention.py:501-557``). Returns (out, new_cache)."""
    sa = lp["self_attn"]
    H, Hkv, hd = cfg.num_heads, cfg.num_key_value_heads, cfg.head_dim
    if family == "neox":
        qkv = dense(h, _t(sa["qkv_proj"]["kernel"]), _t(sa["qkv_proj"]["bias"]) if "bias" in sa["qkv_proj"] else None, dtype)
        q, k, v = qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2]
    else:
        def proj(name):
            b = sa[name].get("bias")
            return dense(h, _t(sa[name]["kernel"]), None if b is None else _t(b), dtype)
        q, k, v = proj("q_proj"), proj("k_proj"), proj("v_proj")
    if family == "gemma3":
        q = gemma_rmsnorm(q, _t(sa["q_norm"]["weight"]).to(dtype), cfg.norm_eps)
        k = gemma_rmsnorm(k, _t(sa["k_norm"]["weight"]).to(dtype), cfg.norm_eps)
    if attention_mask is None:
        attention_mask = cache.mask if (cache is not None and cache.mask is not None) else torch.ones(h.shape[:2], dtype=torch.bool)
    if position_ids is None:
        if cache is not None and cache.pos_id is not None:
            position_ids = (cache.pos_id + 1).to(torch.int64)
        else:
            position_ids = torch.arange(k.shape[1])[None].repeat(k.shape[0], 1)
    q, k = apply_rope(q, k, cos, sin, position_ids.to(torch.int64))
    if cache is not None:
        cache = cache.update(k, v, attention_mask)
        k, v, attention_mask = cache.k, cache.v, cache.mask
    n_rep = H // Hkv
    k, v = repeat_kv(k, n_rep), repeat_kv(v, n_rep)
    out = mha(q, k, v, attention_mask, True, sliding_window, cfg.attn_scale)
    o_b = sa["o_proj"].get("bias")
    out = dense(out.reshape(out.shape[0], out.shape[1], -1), _t(sa["o_proj"]["kernel"]), None if o_b is None else _t(o_b), dtype)
    return out, cache


def _gelu_tanh(x32: torch.Tensor) -> torch.Tensor:
    return 0.5 * x32 * (1.0 + torch.tanh(math.sqrt(2.0 / math.pi) * (x32 + 0.044715 * x32 * x32 * x32)))


def _gelu_erf(x32: torch.Tensor) -> torch.Tensor:
    return x32 * (torch.erf(x32 * math.sqrt(0.5)) + 1.0) / 2.0


def _mlp(family, lp, x, dtype):
    m = lp["mlp"]

    def proj(name, inp):
        b = m[name].get("bias")
        return dense(inp, _t(m[name]["kernel"]), None if b is None else _t(b), dtype)

    if family == "neox":
        up = proj("up_proj", x)
        act = _gelu_erf(_f32(up)).to(dtype)
        return proj("down_proj", act)
    gate = proj("gate_proj", x)
    up = proj("up_proj", x)
    g32 = _f32(gate)
    if family == "llama":
        act = (g32 * torch.sigmoid(g32)).to(dtype)
    else:
        act = _gelu_tanh(g32).to(dtype)
    prod = (_f32(act) * _f32(up)).to(dtype)
    return proj("down_proj", prod)


def _add(a, b):
    return (_f32(a) + _f32(b)).to(a.dtype)


def _norm(family, p, x, eps):
    if family == "neox":
        return layernorm(x, _t(p["weight"]).to(x.dtype), _t(p["bias"]).to(x.dtype) if "bias" in p else None, eps)
    if family == "gemma3":
        return gemma_rmsnorm(x, _t(p["weight"]).to(x.dtype), eps)
    return rmsnorm(x, _t(p["weight"]).to(x.dtype), eps)


def _uses_sliding(family, cfg, idx: int) -> bool:
    if family != "gemma3" or cfg.sliding_window is None:
        return False
    stride = cfg.sliding_window_pattern or 1
    return ((idx + 1) % stride) > 0


@dataclass
class OracleOutput:
    logits: Optional[torch.Tensor]
    last_hidden_state: torch.Tensor
    kv_caches: Optional[tuple]
    hidden_states: tuple


def forward(family: str, cfg, params, input_ids, dtype, attention_mask=None, kv_caches=None,
            keep_last_n_logits: int = 0, with_head: bool = True, position_ids=None) -> OracleOutput:
    """``*ModelWithHead.__call__`` (``models/llama.py:245-273`` and siblings)."""
    root, mp = _root(params, family)
    input_ids = _t(input_ids).to(torch.int64)
    if attention_mask is not None:
        attention_mask = _t(attention_mask).to(torch.bool)
    populated = kv_caches is not None and any(c is not None and c.mask is not None for c in kv_caches)
    if attention_mask is None and not populated:
        attention_mask = input_ids >= 0
    ids = torch.where(input_ids < 0, torch.zeros_like(input_ids), input_ids)
    table = _t(mp["embed_tokens"]["embedding"]).to(dtype)
    h = table[ids].to(dtype)
    if family == "gemma3":
        h = (_f32(h) * _scalar(cfg.hidden_size ** 0.5, dtype)).to(dtype)
    cos, sin = rope_tables(cfg.head_dim, cfg.rotary_pct, cfg.rope_theta, cfg.rope_scale, cfg.max_position_embeddings, dtype)
    if family == "gemma3":
        cos_l, sin_l = rope_tables(cfg.head_dim, cfg.rotary_pct, 10000.0, 1.0, cfg.max_position_embeddings, dtype)
    hidden = []
    new_caches = []
    for idx in range(cfg.num_layers):
        hidden.append(h)
        lp = mp[f"layers_{idx}"]
        cache = None if kv_caches is None else kv_caches[idx]
        sw = cfg.sliding_window if _uses_sliding(family, cfg, idx) else None
        if family == "gemma3" and (idx + 1) % (cfg.sliding_window_pattern or 1):
            c_, s_ = cos_l, sin_l
        else:
            c_, s_ = cos, sin
        if family == "llama":
            a, cache = _attention_block(family, cfg, lp, _norm(family, lp["input_layernorm"], h, cfg.norm_eps), c_, s_,
                                        attention_mask, position_ids, cache, sw, dtype)
            h = _add(h, a)
            h = _add(_mlp(family, lp, _norm(family, lp["post_attention_layernorm"], h, cfg.norm_eps), dtype), h)
        elif family == "neox":
            a, cache = _attention_block(family, cfg, lp, _norm(family, lp["input_layernorm"], h, cfg.norm_eps), c_, s_,
                                        attention_mask, position_ids, cache, sw, dtype)
            if cfg.use_parallel_residual:
                m = _mlp(family, lp, _norm(family, lp["post_attention_layernorm"], h, cfg.norm_eps), dtype)
                h = _add(_add(m, a), h)
            else:
                ar = _add(a, h)
                m = _mlp(family, lp, _norm(family, lp["post_attention_layernorm"], ar, cfg.norm_eps), dtype)
                h = _add(m, ar)
        else:
            a, cache = _attention_block(family, cfg, lp, _norm(family, lp["input_layernorm"], h, cfg.norm_eps), c_, s_,
                                        attention_mask, position_ids, cache, sw, dtype)
            h = _add(h, _norm(family, lp["post_attention_layernorm"], a, cfg.norm_eps))
            m = _mlp(family, lp, _norm(family, lp["pre_feedforward_layernorm"], h, cfg.norm_eps), dtype)
            h = _add(h, _norm(family, lp["post_feedforward_layernorm"], m, cfg.norm_eps))
        new_caches.append(cache)
    h = _norm(family, mp["norm"], h, cfg.norm_eps)
    hidden.append(h)
    logits = None
    if with_head:
        hs = h if keep_last_n_logits == 0 else h[:, -keep_last_n_logits:]
        logits = dense(hs, _t(root["lm_head"]["kernel"]), None, dtype)
    return OracleOutput(logits, h, tuple(new_caches) if kv_caches is not None else None, tuple(hidden))


# ----------------------------------------------------------------------------------------------
# Generation (Engine.generate with greedy / temperature sampling)
# ----------------------------------------------------------------------------------------------
def _probs(logits: torch.Tensor) -> torch.Tensor:
    """softmax over the vocabulary: float32 arithmetic, result rounded to the logits' dtype (the
    reference applies jax.nn.softmax to model-dtype logits)."""
    x = logits.to(torch.float32)
    e = torch.exp(x - x.max(dim=-1, keepdim=True).values)
    return (e / e.sum(dim=-1, keepdim=True)).to(logits.dtype).to(torch.float32)


def filter_logits(logits: torch.Tensor, top_k: int = 0, top_p: float = 1.0, min_p: float = 0.0) -> torch.Tensor:
    """min-p, then top-k, then top-p filtering of ``[..., V]`` logits, filtered entries set to -inf
    (inference_engine/sampling.py:34-72 and :169-188 for the order).  Restated choices where the
    reference's JAX arithmetic is not visible from its source: probabilities are computed in float32 and
    rounded to the logits' dtype; the top-p cumulative sum runs in float32 over those rounded
    probabilities; a cutoff index past the end is clamped to the last sorted entry."""
    neg = torch.tensor(float("-inf"), dtype=logits.dtype)
    if min_p > 0.0:
        keep = _probs(logits) >= min_p
        any_kept = keep.any(dim=-1, keepdim=True)
        logits = torch.where(any_kept, torch.where(keep, logits, neg), logits)
    if top_k > 0:
        k = min(top_k, logits.shape[-1])
        cutoff = torch.topk(logits.to(torch.float32), k, dim=-1).values[..., -1:]
        logits = torch.where(logits.to(torch.float32) >= cutoff, logits, neg)
    if top_p < 1.0:
        srt = torch.sort(logits.to(torch.float32), dim=-1, descending=True).values
        cum = torch.cumsum(_probs(srt.to(logits.dtype)), dim=-1)
        idx = (cum < top_p).sum(dim=-1, keepdim=True).clamp(max=logits.shape[-1] - 1)
        cutoff = torch.gather(srt, -1, idx)
        logits = torch.where(logits.to(torch.float32) < cutoff, neg, logits)
    return logits


def sample(logits: torch.Tensor, key, temperature: float, greedy: bool, top_k: int = 0, top_p: float = 1.0,
           min_p: float = 0.0) -> torch.Tensor:
    """``greedy_fn`` / ``categorical(subkey, filtered logits / temp)`` on ``[B,1,V]`` logits; returns
    ``[B,1]`` int32."""
    if greedy:
        return torch.argmax(_f32(logits), dim=-1).to(torch.int32)
    if top_k > 0 or top_p < 1.0 or min_p > 0.0:
        logits = filter_logits(logits, top_k, top_p, min_p)
    arr = _f32(logits).numpy()
    if logits.dtype == torch.bfloat16:
        out = threefry.categorical_bf16(key, arr, temperature)
    else:
        out = threefry.categorical_f32(key, arr, temperature)
    return torch.from_numpy(out)


def generate(family: str, cfg, params, prompt_tokens, dtype, max_new_tokens: int = 10, temperature: float = 1.0,
             seed: int = 0, cache_stride: int = 256, attention_mask=None, include_prompt: bool = True,
             top_k: int = 0, top_p: float = 1.0, min_p: float = 0.0):
    """``Engine.generate`` (greedy, temperature, min-p / top-k / top-p), including the chunk/resize loop."""
    prompt = _t(prompt_tokens).to(torch.int32)
    if prompt.ndim == 1:
        prompt = prompt[None]
    greedy = temperature <= 0.0 or top_p <= 0.0 or top_k == 1
    B, P = prompt.shape
    if max_new_tokens == 0:
        return prompt if include_prompt else prompt[:, :0]
    key = threefry.prng_key(seed)
    cache_len = (P // cache_stride + 1) * cache_stride
    caches = tuple(OracleKVCache(cache_len, dtype) for _ in range(cfg.num_layers))
    out_tokens = []
    generated = 0
    next_input = prompt
    while generated < max_new_tokens:
        capacity = cache_len - (P + generated)
        count = min(max_new_tokens - generated, capacity)
        if count <= 0:
            cache_len += cache_stride
            caches = tuple(c.resize(cache_len) for c in caches)
            continue
        chunk = []
        if generated == 0:
            out = forward(family, cfg, params, next_input, dtype, attention_mask=attention_mask, kv_caches=caches,
                          keep_last_n_logits=1)
            caches = out.kv_caches
            ks = threefry.split(key)
            key, sub = ks[0], ks[1]
            tok = sample(out.logits[:, -1:], sub, temperature, greedy, top_k, top_p, min_p)
            chunk.append(tok)
            steps = count - 1
        else:
            tok = next_input[:, -1:]
            steps = count
        for _ in range(steps):
            ks = threefry.split(key)
            key, sub = ks[0], ks[1]
            out = forward(family, cfg, params, tok, dtype, kv_caches=caches, keep_last_n_logits=1)
            caches = out.kv_caches
            tok = sample(out.logits, sub, temperature, greedy, top_k, top_p, min_p)
            chunk.append(tok)
        chunk = torch.cat(chunk, dim=1)
        out_tokens.append(chunk)
        generated += chunk.shape[1]
        next_input = chunk[:, -1:]
    res = torch.cat(out_tokens, dim=1)
    if include_prompt:
        res = torch.cat([prompt, res], dim=1)
    return res


# ----------------------------------------------------------------------------------------------
# Random-init weights (N(0, 0.02)) in the reference's Flax parameter layout
# ----------------------------------------------------------------------------------------------
def init_params(family: str, cfg, seed: int = 0, std: float = 0.02, dtype=torch.float32, num_layers=None):
    """Parameter tree in the Flax layout of the reference (kernel ``[in..., out...]``)."""
    g = torch.Generator().manual_seed(seed)
    d, H, Hkv, hd, V = cfg.hidden_size, cfg.num_heads, cfg.num_key_value_heads, cfg.head_dim, cfg.vocab_size
    F = cfg.intermediate_size
    L = cfg.num_layers if num_layers is None else num_layers

    def rnd(*shape):
        return (torch.randn(*shape, generator=g, dtype=F32) * std).to(dtype)

    def ones(n):
        return torch.ones(n, dtype=dtype)

    def norm_p(n, bias=False):
        p = {"weight": ones(n) if family != "gemma3" else rnd(n)}
        if bias:
            p["bias"] = rnd(n)
        return p

    layers = {}
    for i in range(L):
        lp = {}
        if family == "neox":
            lp["self_attn"] = {"qkv_proj": {"kernel": rnd(d, 3, H, hd), "bias": rnd(3, H, hd)},
                               "o_proj": {"kernel": rnd(H * hd, d), "bias": rnd(d)}}
            lp["mlp"] = {"up_proj": {"kernel": rnd(d, F), "bias": rnd(F)},
                         "down_proj": {"kernel": rnd(F, d), "bias": rnd(d)}}
            lp["input_layernorm"] = norm_p(d, True)
            lp["post_attention_layernorm"] = norm_p(d, True)
        else:
            sa = {"q_proj": {"kernel": rnd(d, H, hd)}, "k_proj": {"kernel": rnd(d, Hkv, hd)},
                  "v_proj": {"kernel": rnd(d, Hkv, hd)}, "o_proj": {"kernel": rnd(H * hd, d)}}
            if family == "gemma3":
                sa["q_norm"] = {"weight": rnd(hd)}
                sa["k_norm"] = {"weight": rnd(hd)}
            lp["self_attn"] = sa
            lp["mlp"] = {"gate_proj": {"kernel": rnd(d, F)}, "up_proj": {"kernel": rnd(d, F)},
                         "down_proj": {"kernel": rnd(F, d)}}
            lp["input_layernorm"] = norm_p(d)
            lp["post_attention_layernorm"] = norm_p(d)
            if family == "gemma3":
                lp["pre_feedforward_layernorm"] = norm_p(d)
                lp["post_feedforward_layernorm"] = norm_p(d)
        layers[f"layers_{i}"] = lp
    body = {"embed_tokens": {"embedding": rnd(V, d)}, "norm": norm_p(d, family == "neox"), **layers}
    root = {"gpt_neox" if family == "neox" else "model": body, "lm_head": {"kernel": rnd(d, V)}}
    return {"params": root}
