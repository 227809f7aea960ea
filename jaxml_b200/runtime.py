"""Device runtime of one decoder model on one GPU (one tensor-parallel rank).

It owns the packed weights, the KV cache, the activation buffers and the kernel workspaces, and runs
the prefill and decode passes of jaxml's Llama / GPT-NeoX / Gemma3 stacks (models/llama.py:91-273,
models/gpt_neox.py:83-272, models/gemma3.py:109-331) as a fixed sequence of libjxb200 calls on the
current CUDA stream.  A decode step needs no host work (positions, step index and PRNG key live on the
device), so it is captured once in a CUDA graph and replayed per token.

HBM layout (bfloat16 models): every projection weight is packed once into the K128 tiled layout
(``include/jxb200.h``): QKV as one [(Hq+2Hkv)*hd, d] matrix per layer, gate/up interleaved in 32-row
groups so the SiLU/GELU product is formed in the projection epilogue, o_proj / down / lm_head as
[out, in].  float32 models keep the reference's [in, out] kernel layout for the CUDA-core GEMM.  The KV
cache is the reference's [B, T, Hkv, hd] per layer (here [L, B, T, Hkv_local, hd]); the padding mask
and positions are shared by all layers.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

import numpy as np
import torch

from . import _native as N
from ._native import ptr

FAMILIES = ("llama", "neox", "gemma3")


def _rup(x: int, m: int) -> int:
    return (x + m - 1) // m * m


def _jx_dtype(dtype: torch.dtype) -> int:
    if dtype == torch.bfloat16:
        return N.JX_BF16
    if dtype == torch.float32:
        return N.JX_F32
    raise TypeError(f"unsupported compute dtype {dtype}; use bfloat16 or float32")


def rope_tables(head_dim: int, rotary_pct: float, base: float, rope_scale: float, max_len: int, dtype):
    """Rotary cos/sin tables as RotaryEmbedding.setup builds them (nn/position.py:177-200): float32
    angles t * inv_freq, inv_freq = 1 / base^(arange(0, rd, 2) / rd), then cos/sin rounded to dtype."""
    rd = head_dim if rotary_pct >= 1.0 else int(head_dim * rotary_pct)
    inv = 1.0 / (torch.tensor(base, dtype=torch.float32) ** (torch.arange(0, rd, 2, dtype=torch.float32) / rd))
    t = torch.arange(max_len, dtype=torch.float32) / torch.tensor(rope_scale, dtype=torch.float32)
    freqs = t[:, None] * inv[None, :]
    emb = torch.cat([freqs, freqs], dim=-1)
    return torch.cos(emb).to(dtype), torch.sin(emb).to(dtype)


def _bf16_round64(x: np.ndarray) -> np.ndarray:
    """float64 -> nearest bfloat16 (ties to even), returned as float32."""
    f = x.astype(np.float32)
    u = f.view(np.uint32).astype(np.uint64)
    r = (((u + (((u >> np.uint64(16)) & np.uint64(1)) + np.uint64(0x7FFF))) >> np.uint64(16)) << np.uint64(16))
    out = r.astype(np.uint32).view(np.float32)
    mid = (f.view(np.uint32) & np.uint32(0xFFFF)) == np.uint32(0x8000)
    if np.any(mid):
        resid = x - f.astype(np.float64)
        base = (f.view(np.uint32) & np.uint32(0xFFFF0000))
        away = (base + np.uint32(0x10000)).view(np.float32)
        toward = base.view(np.float32)
        up = np.where(f >= 0, resid > 0, resid < 0)
        down = np.where(f >= 0, resid < 0, resid > 0)
        out = np.where(mid & up, away, np.where(mid & down, toward, out))
    return out.astype(np.float32)


def gumbel_table_bf16() -> torch.Tensor:
    """The 256 Gumbel values a bfloat16 jax.random.gumbel can produce: draw b -> u = (b >> 1) / 128
    (u = 2^-126 when that is 0), g = -log(-log(u)) with each op rounded to bfloat16."""
    b = np.arange(256, dtype=np.uint32)
    u = ((b >> 1).astype(np.float64)) / 128.0
    u = np.where(u == 0.0, 2.0 ** -126, u)
    l1 = _bf16_round64(np.log(u))
    l2 = _bf16_round64(np.log(-l1.astype(np.float64)))
    return torch.from_numpy((-l2).astype(np.float32))


# ------------------------------------------------------------------------------------------------
# Weights
# ------------------------------------------------------------------------------------------------
@dataclass
class LayerWeights:
    wqkv: torch.Tensor
    bqkv: Optional[torch.Tensor]
    wo: torch.Tensor
    bo: Optional[torch.Tensor]
    wgu: torch.Tensor           # gate/up interleaved (GLU) or up (NeoX)
    bgu: Optional[torch.Tensor]
    wd: torch.Tensor
    bd: Optional[torch.Tensor]
    norms: dict = field(default_factory=dict)   # name -> (weight, bias)
    qn: Optional[torch.Tensor] = None
    kn: Optional[torch.Tensor] = None
    sliding: bool = False
    local_rope: bool = False


def _tt(x, device, dtype=None):
    if not isinstance(x, torch.Tensor):
        x = torch.as_tensor(np.asarray(x))
    x = x.to(device=device)
    return x if dtype is None else x.to(dtype)


class ModelWeights:
    """Packs a parameter tree in the reference's Flax layout (Appendix-B names) for one TP rank."""

    def __init__(self, family: str, cfg, params, dtype: torch.dtype, device, tp_rank: int = 0, tp_size: int = 1):
        if family not in FAMILIES:
            raise ValueError(f"unknown model family {family!r}")
        self.family, self.cfg, self.dtype, self.device = family, cfg, dtype, torch.device(device)
        self.tp_rank, self.tp_size = tp_rank, tp_size
        self.jdt = _jx_dtype(dtype)
        self.bf16 = dtype == torch.bfloat16
        H, Hkv, hd, d = cfg.num_heads, cfg.num_key_value_heads, cfg.head_dim, cfg.hidden_size
        F, V = cfg.intermediate_size, cfg.vocab_size
        t = tp_size
        if H % t or Hkv % t:
            raise ValueError(f"tp_size={t} must divide num_heads={H} and num_key_value_heads={Hkv}.")
        if F % t or V % t:
            raise ValueError(f"tp_size={t} must divide intermediate_size={F} and vocab_size={V}.")
        self.Hq, self.Hkv, self.hd, self.d = H // t, Hkv // t, hd, d
        self.F, self.V, self.V_total = F // t, V // t, V
        self.vocab_offset = tp_rank * self.V
        self.rd = cfg.rotary_dim
        self.nqkv = (self.Hq + 2 * self.Hkv) * hd
        self.glu = family != "neox"
        self.F32 = _rup(self.F, 32)
        self.Kp_d = _rup(d, 128)
        self.Kp_o = _rup(self.Hq * hd, 128)
        self.Kp_f = _rup(self.F, 128)
        self.Np_qkv = _rup(self.nqkv, 128)
        self.Np_d = _rup(d, 128)
        self.Np_gu = _rup(2 * self.F32 if self.glu else self.F, 128)
        self.Np_v = _rup(self.V, 128)
        p = params["params"] if "params" in params else params
        body = p["gpt_neox" if family == "neox" else "model"]
        dev = self.device
        self.embed = _tt(body["embed_tokens"]["embedding"], dev, dtype).contiguous()
        if self.embed.shape != (V, d):
            raise ValueError(f"embedding must have shape {(V, d)}, got {tuple(self.embed.shape)}.")
        fn = body["norm"]
        self.final_norm = (_tt(fn["weight"], dev, dtype), _tt(fn["bias"], dev, dtype) if "bias" in fn else None)
        head = _tt(p["lm_head"]["kernel"], dev)                               # [d, V]
        head = head[:, self.vocab_offset:self.vocab_offset + self.V]
        self.lm_head = self._pack_kn(head, self.Np_v, self.Kp_d)
        self.layers = [self._layer(body[f"layers_{i}"], i) for i in range(cfg.num_layers)]
        mp = cfg.max_position_embeddings
        self.cos, self.sin = (x.to(dev) for x in rope_tables(hd, cfg.rotary_pct, cfg.rope_theta, cfg.rope_scale, mp, dtype))
        if family == "gemma3":
            self.cos_l, self.sin_l = (x.to(dev) for x in rope_tables(hd, cfg.rotary_pct, 10000.0, 1.0, mp, dtype))
        self.embed_scale = 0.0
        if family == "gemma3":
            self.embed_scale = float(torch.tensor(d ** 0.5, dtype=torch.float32).to(dtype).float())
        self.gumbel = gumbel_table_bf16().to(dev)
        if dev.type == "cuda":
            torch.cuda.synchronize(dev)

    # -- packing helpers -------------------------------------------------------------------------
    def _pack_kn(self, w_kn: torch.Tensor, Np: int, Kp: int) -> torch.Tensor:
        """Kernel in [K, N] layout -> K128 bfloat16 [Np, Kp] (bf16 models) or contiguous [K, N] float32."""
        if not self.bf16:
            return w_kn.to(torch.float32).contiguous()
        src = w_kn.contiguous()
        if src.dtype not in (torch.float32, torch.bfloat16):
            src = src.to(torch.float32)
        K, Nn = src.shape
        out = torch.empty(Np * Kp, dtype=torch.bfloat16, device=self.device)
        sdt = N.JX_BF16 if src.dtype == torch.bfloat16 else N.JX_F32
        N.call("jx_pack_k128", ptr(src), sdt, Nn, K, Nn, 1, ptr(out), Np, Kp, torch.cuda.current_stream(self.device).cuda_stream)
        return out

    def _bias(self, parts, n_pad: int) -> Optional[torch.Tensor]:
        if parts is None:
            return None
        b = torch.cat([x.reshape(-1) for x in parts]).to(self.dtype)
        out = torch.zeros(n_pad, dtype=self.dtype, device=self.device)
        out[: b.numel()] = b
        return out

    def _glu_interleave(self, g: torch.Tensor, u: torch.Tensor) -> torch.Tensor:
        """[K, F] gate and up -> [K, 2*F32] columns in groups of 64: 32 gate, then the same 32 up."""
        K = g.shape[0]
        pad = self.F32 - g.shape[1]
        if pad:
            z = torch.zeros(K, pad, dtype=g.dtype, device=g.device)
            g, u = torch.cat([g, z], 1), torch.cat([u, z], 1)
        return torch.stack([g.reshape(K, -1, 32), u.reshape(K, -1, 32)], dim=2).reshape(K, 2 * self.F32)

    def _layer(self, lp, idx: int) -> LayerWeights:
        cfg, dev, hd = self.cfg, self.device, self.hd
        r, t = self.tp_rank, self.tp_size
        sa, mlp = lp["self_attn"], lp["mlp"]
        qs = slice(r * self.Hq, (r + 1) * self.Hq)
        ks = slice(r * self.Hkv, (r + 1) * self.Hkv)
        d = self.d
        if self.family == "neox":
            k = _tt(sa["qkv_proj"]["kernel"], dev)                              # [d, 3, H, hd]
            q_w, k_w, v_w = (k[:, i, qs].reshape(d, -1) for i in range(3))
            b = sa["qkv_proj"].get("bias")
            bq = None if b is None else [(_tt(b, dev)[i, qs]) for i in range(3)]
        else:
            q_w = _tt(sa["q_proj"]["kernel"], dev)[:, qs].reshape(d, -1)
            k_w = _tt(sa["k_proj"]["kernel"], dev)[:, ks].reshape(d, -1)
            v_w = _tt(sa["v_proj"]["kernel"], dev)[:, ks].reshape(d, -1)
            bq = None
            if "bias" in sa["q_proj"]:
                bq = [_tt(sa["q_proj"]["bias"], dev)[qs], _tt(sa["k_proj"]["bias"], dev)[ks],
                      _tt(sa["v_proj"]["bias"], dev)[ks]]
        wqkv = self._pack_kn(torch.cat([q_w, k_w, v_w], dim=1), self.Np_qkv, self.Kp_d)
        bqkv = self._bias(bq, self.Np_qkv) if bq is not None else None
        o_k = _tt(sa["o_proj"]["kernel"], dev)[r * self.Hq * hd:(r + 1) * self.Hq * hd]   # [Hq*hd, d]
        wo = self._pack_kn(o_k, self.Np_d, self.Kp_o)
        bo = None
        if "bias" in sa["o_proj"] and r == 0:
            bo = self._bias([_tt(sa["o_proj"]["bias"], dev)], self.Np_d)
        fs = slice(r * self.F, (r + 1) * self.F)
        if self.glu:
            g = _tt(mlp["gate_proj"]["kernel"], dev)[:, fs]
            u = _tt(mlp["up_proj"]["kernel"], dev)[:, fs]
            wgu = self._pack_kn(self._glu_interleave(g, u), self.Np_gu, self.Kp_d)
            bgu = None
            if "bias" in mlp["gate_proj"]:
                bg = _tt(mlp["gate_proj"]["bias"], dev)[fs].reshape(1, -1)
                bu = _tt(mlp["up_proj"]["bias"], dev)[fs].reshape(1, -1)
                bgu = self._bias([self._glu_interleave(bg, bu)], self.Np_gu)
        else:
            wgu = self._pack_kn(_tt(mlp["up_proj"]["kernel"], dev)[:, fs], self.Np_gu, self.Kp_d)
            bgu = None
            if "bias" in mlp["up_proj"]:
                bgu = self._bias([_tt(mlp["up_proj"]["bias"], dev)[fs]], self.Np_gu)
        down = _tt(mlp["down_proj"]["kernel"], dev)[fs]
        if self.glu and not self.bf16 and self.F32 > self.F:
            # float32 GLU activations are [M, F32] with zero padding columns: pad the down rows to match.
            down = torch.cat([down, torch.zeros(self.F32 - self.F, d, dtype=down.dtype, device=dev)], 0)
        wd = self._pack_kn(down, self.Np_d, self.Kp_f)
        bd = None
        if "bias" in mlp["down_proj"] and r == 0:
            bd = self._bias([_tt(mlp["down_proj"]["bias"], dev)], self.Np_d)
        norms = {}
        for name in ("input_layernorm", "post_attention_layernorm", "pre_feedforward_layernorm",
                     "post_feedforward_layernorm"):
            if name in lp:
                norms[name] = (_tt(lp[name]["weight"], dev, self.dtype),
                               _tt(lp[name]["bias"], dev, self.dtype) if "bias" in lp[name] else None)
        lw = LayerWeights(wqkv, bqkv, wo, bo, wgu, bgu, wd, bd, norms)
        if self.family == "gemma3":
            lw.qn = _tt(sa["q_norm"]["weight"], dev, self.dtype)
            lw.kn = _tt(sa["k_norm"]["weight"], dev, self.dtype)
            pat = cfg.sliding_window_pattern or 1
            lw.local_rope = bool((idx + 1) % pat)
            lw.sliding = lw.local_rope and cfg.sliding_window is not None
        return lw

    @property
    def norm_kind(self) -> int:
        return {"llama": N.JX_NORM_RMS, "neox": N.JX_NORM_LAYER, "gemma3": N.JX_NORM_GEMMA}[self.family]


# ------------------------------------------------------------------------------------------------
# Persistent decode step
# ------------------------------------------------------------------------------------------------
class PersistentDecode:
    """Arguments of the persistent decode-step kernel (``jx_decode_step``) for one runtime: every layer,
    the final norm and the LM head of a Llama-family bf16 decode step in one cooperative launch, on the
    runtime's own buffers.  ``eligible`` says when the kernel covers the runtime's model and batch."""

    @staticmethod
    def eligible(rt) -> bool:
        w, cfg = rt.w, rt.w.cfg
        biases = any(x is not None for lw in w.layers for x in (lw.bqkv, lw.bo, lw.bgu, lw.bd))
        norm_bias = any(v[1] is not None for lw in w.layers for v in lw.norms.values()) or w.final_norm[1] is not None
        return (w.bf16 and w.family == "llama" and rt.comm is None and w.hd == 128 and rt.dec["Mp"] == 16
                and rt.fast_attn and (w.Hq // w.Hkv) <= 16 and w.rd % 16 == 0 and w.rd <= 128
                and cfg.sliding_window is None and not biases and not norm_bias and w.d % 8 == 0 and w.d <= 8192
                and w.Np_gu >= 2 * w.F32)

    def __init__(self, rt):
        w, cfg, dev = rt.w, rt.w.cfg, rt.w.device
        ptrs = []
        for lw in w.layers:
            ptrs += [lw.wqkv.data_ptr(), lw.wo.data_ptr(), lw.wgu.data_ptr(), lw.wd.data_ptr(),
                     lw.norms["input_layernorm"][0].data_ptr(), lw.norms["post_attention_layernorm"][0].data_ptr()]
        self.layer_ptrs = torch.tensor(ptrs, dtype=torch.int64, device=dev)
        self.sync = torch.zeros(6, dtype=torch.int32, device=dev)
        a = N.JxStepArgs()
        a.M, a.L, a.d, a.Hq, a.Hkv, a.hd = rt.B, cfg.num_layers, w.d, w.Hq, w.Hkv, w.hd
        a.F, a.V, a.vocab = w.F, w.V, cfg.vocab_size
        a.T, a.rd, a.max_pos = rt.T, w.rd, cfg.max_position_embeddings
        a.Np_qkv, a.Np_d, a.Np_gu, a.Np_v = w.Np_qkv, w.Np_d, w.Np_gu, w.Np_v
        a.Kp_d, a.Kp_o, a.Kp_f = w.Kp_d, w.Kp_o, w.Kp_f
        a.eps, a.scale = cfg.norm_eps, cfg.attn_scale
        a.layers, a.embed, a.ids = ptr(self.layer_ptrs), ptr(w.embed), ptr(rt.next_ids)
        a.final_norm, a.lm_head = ptr(w.final_norm[0]), ptr(w.lm_head)
        d = rt.dec
        a.h, a.xn, a.qkv, a.attn, a.act = ptr(d["h"]), ptr(d["xn"]), ptr(d["qkv"]), ptr(d["attn"]), ptr(d["act"])
        a.logits = ptr(rt.logits_buf())
        a.k_cache, a.v_cache, a.cos, a.sin = ptr(rt.k_cache), ptr(rt.v_cache), ptr(w.cos), ptr(w.sin)
        a.pos_id = ptr(rt.pos_id)
        a.ws, a.ws_floats, a.counters = ptr(rt.gemv_ws), rt.gemv_ws.numel(), ptr(rt.gemv_counters)
        a.attn_ws, a.attn_ws_bytes, a.attn_counters = ptr(rt.attn_ws), rt.attn_ws.numel() * 4, ptr(rt.attn_counters)
        a.sync, a.status, a.grid = ptr(self.sync), ptr(rt.status), rt.grid
        self.args = a

    def launch(self, stream):
        N.check(N.load().jx_decode_step(self.args, stream), "jx_decode_step")


# ------------------------------------------------------------------------------------------------
# Runtime
# ------------------------------------------------------------------------------------------------
class DecoderRuntime:
    """Buffers + the prefill / decode call sequences for a batch of ``B`` rows and ``T`` cache slots."""

    # True: decode steps of the models it covers run as one persistent kernel (PersistentDecode) plus the
    # sampling kernel.  Off by default: on the Llama-3-8B shape (batch 16) it measures 4.9-5.3 ms per step
    # against 4.14 ms for the one-launch-per-op path (8 kernels per layer), which stays the default.
    persistent_decode = False

    def __init__(self, weights: ModelWeights, B: int, T: int, comm=None):
        self.w = weights
        self.B, self.T = B, T
        self.comm = comm
        if comm is not None:
            comm.prepare_peer(weights.device)   # collective: outside any graph capture
        w = weights
        dev, dt = w.device, w.dtype
        cfg = w.cfg
        L = cfg.num_layers
        self.stream_ptr = lambda: torch.cuda.current_stream(dev).cuda_stream
        self.k_cache = torch.zeros(L, B, T, w.Hkv, w.hd, dtype=dt, device=dev)
        self.v_cache = torch.zeros_like(self.k_cache)
        self.mask = torch.zeros(B, T, dtype=torch.uint8, device=dev)
        self.pos_id = torch.zeros(B, dtype=torch.int32, device=dev)
        self.status = torch.zeros(4, dtype=torch.int32, device=dev)
        self.rng = torch.zeros(4, dtype=torch.int32, device=dev)
        self.step = torch.zeros(1, dtype=torch.int32, device=dev)
        self.next_ids = torch.zeros(B, dtype=torch.int32, device=dev)
        self.tokens_out = None
        n_sms = torch.cuda.get_device_properties(dev).multi_processor_count
        self.grid = n_sms
        self.Mp_dec = 16 * ((B + 15) // 16) if B <= 32 else 64
        if B > 64:
            self.Mp_dec = 0   # decode runs through the prefill GEMM
        self.dec = self._alloc_acts(B, self.Mp_dec if self.Mp_dec else _rup(B, 128))
        self.pre = None
        self.pre_shape = None
        ws_floats = N.LL()
        N.check(N.load().jx_linear_decode_workspace(self.grid, 64, ws_floats), "workspace query")
        self.gemv_ws = torch.zeros(ws_floats.value, dtype=torch.float32, device=dev)
        max_blocks = max(w.Np_qkv, w.Np_d, w.Np_gu, w.Np_v) // 64 + 1
        self.gemv_counters = torch.zeros(max_blocks, dtype=torch.int32, device=dev)
        self.sample_chunk = 4096
        nchunks = (w.V + self.sample_chunk - 1) // self.sample_chunk
        self.sample_ws = torch.zeros(B * nchunks, dtype=torch.int64, device=dev)
        # min-p / top-k / top-p: (top_k, top_p, min_p) of the current generation, or None
        self.filters = None
        self._flog = None
        self.sample_counters = torch.zeros(B + 1, dtype=torch.int32, device=dev)
        self.row_best = torch.zeros(B, dtype=torch.int64, device=dev)
        self.row_map = (torch.arange(B, dtype=torch.int32, device=dev))
        # tensor-core decode attention: bf16, head_dim 64/128/256, up to 16 query heads per KV head
        self.fast_attn = w.bf16 and w.hd in (64, 128, 256) and (w.Hq // w.Hkv) <= 16
        if self.fast_attn:
            nb = N.LL()
            N.check(N.load().jx_decode_attention_workspace(B, w.Hq, w.hd, T, 0, nb), "attention workspace")
            self.attn_ws = torch.zeros((nb.value + 3) // 4, dtype=torch.float32, device=dev)
            self.attn_counters = torch.zeros(B * w.Hkv, dtype=torch.int32, device=dev)
        self.graph = None
        # fuse_decoding: a graph of several consecutive decode steps, keyed like self.graph plus the count
        self.graph_multi = None
        # slots that a prompt row with no visible key attends over (0 = the whole buffer): the reference's
        # cache length when the prompt ran, before its chunk loop grows the cache (engine.py:543-557)
        self.uniform_T = 0
        # the persistent decode-step kernel's plan when it runs this runtime's layers (else None)
        self.fused_step = None
        self._launches = 0
        self.launches_last_step = 0
        self._push_pending = False
        # normalisation prologue of the decode projections (jx_epilogue.pn_*): epoch, arrivals, row flags
        self.pn_sync = torch.zeros(2 + 16, dtype=torch.int32, device=dev)
        # the normalisation tail's arrival counter (self-resetting)
        self.tn_sync = torch.zeros(1, dtype=torch.int32, device=dev)
        self._pending_norm = None
        if self.persistent_decode and PersistentDecode.eligible(self):
            self.fused_step = PersistentDecode(self)

    # -- buffers ------------------------------------------------------------------------------------
    def _alloc_acts(self, M: int, Mp: int) -> dict:
        w, dev, dt = self.w, self.w.device, self.w.dtype
        a = {"M": M, "Mp": Mp}
        a["h"] = torch.zeros(Mp, w.d, dtype=dt, device=dev)
        # Under tensor parallelism `tmp` holds float32 partial sums of the row-parallel projections, so
        # the all-reduce adds unrounded values and the result is rounded once, as on one GPU.
        a["tmp"] = torch.zeros(Mp, w.d, dtype=torch.float32 if self.comm is not None else dt, device=dev)
        a["qkv"] = torch.zeros(Mp, w.nqkv, dtype=dt, device=dev)
        a["q"] = torch.zeros(Mp, w.Hq * w.hd, dtype=dt, device=dev)
        if w.bf16:
            a["xn"] = torch.zeros(Mp * w.Kp_d, dtype=dt, device=dev)
            a["xn2"] = torch.zeros(Mp * w.Kp_d, dtype=dt, device=dev)
            a["attn"] = torch.zeros(Mp * w.Kp_o, dtype=dt, device=dev)
            a["act"] = torch.zeros(Mp * w.Kp_f, dtype=dt, device=dev)
        else:
            a["xn"] = torch.zeros(Mp, w.d, dtype=dt, device=dev)
            a["xn2"] = torch.zeros(Mp, w.d, dtype=dt, device=dev)
            a["attn"] = torch.zeros(Mp, w.Hq * w.hd, dtype=dt, device=dev)
            a["act"] = torch.zeros(Mp, w.F32 if w.glu else w.F, dtype=dt, device=dev)
        return a

    def _prefill_acts(self, M: int) -> dict:
        Mp = _rup(M, 128) if self.w.bf16 else M
        if self.pre is None or self.pre["Mp"] < Mp:
            self.pre = None
            torch.cuda.empty_cache()
            self.pre = self._alloc_acts(M, Mp)
        self.pre["M"] = M
        return self.pre

    # -- single ops ----------------------------------------------------------------------------------
    def _norm(self, acts, *, out_key="xn", kind=None, w=None, b=None, a=None, kind_pre=N.JX_NORM_NONE, w_pre=None,
              b_pre=None, ids=None, out2_key=None, w2=None, b2=None, row_map=None, M=None, out_acts=None):
        self._flush_norm()   # a recorded prologue norm comes first
        W = self.w
        M = acts["M"] if M is None else M
        oa = acts if out_acts is None else out_acts
        args = N.JxNormArgs()
        args.M, args.d, args.eps = M, W.d, W.cfg.norm_eps
        args.kind = W.norm_kind if kind is None else kind
        args.kind_pre = kind_pre
        args.vocab = W.cfg.vocab_size
        args.ids = ptr(ids)
        args.table = ptr(W.embed)
        args.embed_scale = W.embed_scale if ids is not None else 0.0
        args.row_map = ptr(row_map)
        args.a = ptr(a)
        args.a_f32 = 1 if (a is not None and a.dtype == torch.float32 and W.dtype != torch.float32) else 0
        args.lda = W.d
        args.h = ptr(acts["h"])
        args.ldh = W.d
        args.w_pre, args.b_pre = ptr(w_pre), ptr(b_pre)
        args.w, args.b = ptr(w), ptr(b)
        if out_key is not None:
            args.out = ptr(oa[out_key])
            args.ldo = W.d
            args.out_rp = oa["Mp"] if W.bf16 else 0
        if out2_key is not None:
            args.w2, args.b2 = ptr(w2), ptr(b2)
            args.out2 = ptr(oa[out2_key])
            args.ldo2 = W.d
            args.out2_rp = oa["Mp"] if W.bf16 else 0
        if self._push_pending and a is not None and a.data_ptr() == acts["tmp"].data_ptr():
            # `a` is the sum of the partials the last projection pushed into the receive slots
            self.comm.peer.push_norm(args, W.d, W.d)
            self._push_pending = False
        args.status = ptr(self.status)
        self._launches += 1
        N.check(N.load().jx_norm(args, W.jdt, 1, self.stream_ptr()), "jx_norm")

    # L2 prefetch of the next decode projection's weights (jx_epilogue.pf_*) is off: on the Llama-8B
    # decode step every budget tried made the step slower (4.39 ms off, 4.46-4.99 ms on).
    l2_prefetch = False

    def _pf(self, w_t, Np, Kp, budget=40e6):
        """L2 prefetch request for the next decode projection (jx_epilogue.pf_*): its weights, and how many
        128-wide K chunks per CTA fit `budget` bytes over the grid (the library clamps it to what each
        CTA of that call reads).  None while `l2_prefetch` is off."""
        if not self.l2_prefetch:
            return None
        rows = 128 if (Np % 128 == 0 and Np // 128 >= self.grid) else 64
        return (w_t, Np, Kp, max(1, int(budget // (self.grid * rows * 256))))

    # Single-GPU decode: run the RMSNorm / LayerNorm that feeds a projection (no residual input, no second
    # output) in that projection's prologue instead of a separate jx_norm launch.  Off: on the Llama-8B
    # decode step it measured 4.668 ms against 4.297 ms with the separate kernel (the 16 CTAs that
    # normalise a row each start their share of the projection that much later, and every CTA waits for
    # them before loading the activations).
    norm_prologue = False

    def _defer_norm(self, acts, w, b) -> bool:
        """Records the norm of h into xn for the next decode projection's prologue; False when the
        prologue does not apply (then the caller launches jx_norm)."""
        W = self.w
        if not (self.norm_prologue and self.comm is None and W.bf16 and acts["Mp"] == 16 and W.d % 8 == 0
                and W.norm_kind in (N.JX_NORM_RMS, N.JX_NORM_GEMMA, N.JX_NORM_LAYER)):
            return False
        self._pending_norm = (acts, w, b)
        return True

    def _flush_norm(self):
        """Launches a recorded prologue norm as jx_norm (the next call could not take it)."""
        if self._pending_norm is not None:
            acts, w, b = self._pending_norm
            self._pending_norm = None
            self._norm(acts, w=w, b=b)

    # The norm that follows a decode projection's residual add can run in that projection's last CTA
    # (jx_epilogue.tn_*: the row-split kernel's normalisation tail, bit-identical to jx_norm) instead of a
    # separate launch.  Off: one SM normalising 16 rows x 4096 took 35-50 us per call, and the decode
    # step went from 3.89-3.94 to 6.48-7.70 ms; the norm kernel spreads the same work over 16 CTAs.
    tail_norm = False

    def _tail_ok(self, acts, Np) -> bool:
        """The decode projection of Np packed rows takes the row-split kernel with a normalisation tail."""
        W = self.w
        if not (self.tail_norm and self.comm is None and W.bf16 and acts["Mp"] == 16 and W.d % 256 == 0
                and W.d <= 8192 and W.norm_kind in (N.JX_NORM_RMS, N.JX_NORM_GEMMA, N.JX_NORM_LAYER)):
            return False
        g = self.grid if self.grid > 0 else 148
        if Np // 128 >= g:
            return False   # the tcgen05 kernel
        return any(Np % (16 * rg) == 0 and Np // (16 * rg) <= g for rg in (2, 3))

    def _linear(self, acts, w_t, Np, Kp, x_key, kind, *, N_valid, bias=None, out=None, ldo=0, out_rp=0, res=None,
                ldr=0, res2=None, ldr2=0, K_logical=None, N_cols=None, pf=None, tail=None):
        """One projection.  `tail` = (w, b): the norm of this call's output (the residual stream h) into
        acts["xn"], in the projection's last CTA (the caller checked _tail_ok)."""
        W = self.w
        pending = self._pending_norm
        # the prologue needs one CTA per token row: at least M work items whichever decode kernel runs
        if pending is not None and not (x_key == "xn" and pending[0] is acts and W.bf16 and acts["Mp"] <= 64
                                        and min(self.grid, (Np // 128) * (Kp // 128)) >= acts["M"]):
            self._flush_norm()
            pending = None
        e = N.JxEpilogue()
        e.kind, e.M, e.N = kind, acts["M"], N_valid
        e.bias, e.out, e.ldo, e.out_rp = ptr(bias), ptr(out), ldo, out_rp
        e.res, e.ldr, e.res2, e.ldr2 = ptr(res), ldr, ptr(res2), ldr2
        if pf is not None and W.bf16 and acts["Mp"] <= 64:
            e.pf_w, e.pf_np, e.pf_kp, e.pf_iters = ptr(pf[0]), pf[1], pf[2], pf[3]
        if kind == N.JX_EPI_PUSH_F32:
            self.comm.peer.push_epilogue(e, ldo)
            self._push_pending = True
        if pending is not None:
            _, w, b = pending
            self._pending_norm = None
            e.pn_h, e.pn_ldh, e.pn_w, e.pn_b = ptr(acts["h"]), W.d, ptr(w), ptr(b)
            e.pn_sync, e.pn_kind, e.pn_d, e.pn_eps = ptr(self.pn_sync), W.norm_kind, W.d, W.cfg.norm_eps
        lib = N.load()
        self._launches += 1
        if not W.bf16:
            rc = lib.jx_linear_f32(ptr(acts[x_key]), K_logical, ptr(w_t), acts["M"], N_cols, K_logical, e, 1,
                                   self.stream_ptr())
            N.check(rc, "jx_linear_f32")
        elif acts["Mp"] <= 64:
            if tail is not None:
                e.tn_x, e.tn_rp, e.tn_w, e.tn_b = ptr(acts["xn"]), acts["Mp"], ptr(tail[0]), ptr(tail[1])
                e.tn_sync, e.tn_kind, e.tn_eps = ptr(self.tn_sync), W.norm_kind, W.cfg.norm_eps
            rc = lib.jx_linear_decode(ptr(w_t), ptr(acts[x_key]), Np, Kp, acts["M"], e, ptr(self.gemv_ws),
                                      self.gemv_ws.numel(), ptr(self.gemv_counters), ptr(self.status), self.grid, 1,
                                      self.stream_ptr())
            if rc == N.JX_ERR_UNSUPPORTED and tail is not None:
                # another decode kernel was selected (jx_set_decode_linear_impl): a separate norm then
                e.tn_x = None
                rc = lib.jx_linear_decode(ptr(w_t), ptr(acts[x_key]), Np, Kp, acts["M"], e, ptr(self.gemv_ws),
                                          self.gemv_ws.numel(), ptr(self.gemv_counters), ptr(self.status), self.grid,
                                          1, self.stream_ptr())
                N.check(rc, "jx_linear_decode")
                self._norm(acts, w=tail[0], b=tail[1])
                return
            N.check(rc, "jx_linear_decode")
        else:
            rc = lib.jx_linear_prefill(ptr(acts[x_key]), ptr(w_t), acts["Mp"], Np, Kp, e, ptr(self.status), 1,
                                       self.stream_ptr())
            N.check(rc, "jx_linear_prefill")

    # Tensor-parallel decode of the sequential-residual families: each row-parallel projection pushes its
    # float32 partial into every rank's receive slot (JX_EPI_PUSH_F32) and the norm that follows sums
    # them, with no all-reduce kernel in between.  Off: the pull all-reduce (jx_allreduce_f32).
    peer_push = True

    def _push_ok(self, acts) -> bool:
        W = self.w
        return (self.peer_push and self.comm is not None and self.comm.peer is not None and W.bf16
                and acts["Mp"] <= 64 and W.d % 256 == 0 and W.d <= 8192
                and acts["Mp"] * W.d <= self.comm.PEER_MAX_FLOATS)

    def _tp_dst(self, acts) -> torch.Tensor:
        """Where a row-parallel projection writes its float32 partial sum: the peer partials buffer of the
        next all-reduce for decode-sized activations, else acts["tmp"] (all-reduced in place by NCCL)."""
        buf = self.comm.partial_buffer(acts["Mp"] * self.w.d) if acts["Mp"] <= 128 else None
        return acts["tmp"] if buf is None else buf.view(acts["Mp"], self.w.d)

    def _allreduce(self, src: torch.Tensor, rows: int, acts):
        """All-reduce of the partial sums in `src` (from _tp_dst) into acts["tmp"]."""
        if self.comm is None:
            return
        if src.data_ptr() == acts["tmp"].data_ptr():
            self.comm.all_reduce(src[:rows])
        else:
            self._launches += 1
            self.comm.all_reduce_partial(src[:rows].reshape(-1), acts["tmp"][:rows].reshape(-1), self.status)

    # -- one pass over the stack -----------------------------------------------------------------------
    def _layers(self, acts, S: int, decode: bool):
        W = self.w
        for li, lw in enumerate(W.layers):
            nx = W.layers[li + 1] if li + 1 < len(W.layers) else None
            # o_proj's weights are prefetched into L2 whole, during RoPE and attention
            self._linear(acts, lw.wqkv, W.Np_qkv, W.Kp_d, "xn", N.JX_EPI_STORE, N_valid=W.nqkv, bias=lw.bqkv,
                         out=acts["qkv"], ldo=W.nqkv, K_logical=W.d, N_cols=W.nqkv,
                         pf=self._pf(lw.wo, W.Np_d, W.Kp_o, budget=64e6))
            fuse_rope = decode and self.fast_attn and self.fused_rope and lw.qn is None
            if not fuse_rope:
                self._qkv_rope_append(acts, li, lw, S, decode)
            if decode and self.fast_attn:
                self._decode_attention(acts, li, lw, fuse_rope)
            elif not decode and self.fast_attn and S > 1:
                self._prefill_attention(acts, li, lw, S)
            else:
                self._generic_attention(acts, li, lw, S, decode)
            self._o_and_mlp(acts, lw, nx)
        self._flush_norm()
        if self.comm is not None and self.comm.align(self.status):
            self._launches += 1

    def _qkv_rope_append(self, acts, li, lw, S, decode):
        W, cfg = self.w, self.w.cfg
        qa = N.JxQkvArgs()
        qa.M, qa.S, qa.Hq, qa.Hkv, qa.hd, qa.rd = acts["M"], S, W.Hq, W.Hkv, W.hd, W.rd
        qa.qkv, qa.ld_qkv = ptr(acts["qkv"]), W.nqkv
        qa.qn_w, qa.kn_w, qa.eps = ptr(lw.qn), ptr(lw.kn), cfg.norm_eps
        cos, sin = (W.cos_l, W.sin_l) if lw.local_rope else (W.cos, W.sin)
        qa.max_pos, qa.cos, qa.sin = cfg.max_position_embeddings, ptr(cos), ptr(sin)
        qa.pos_id, qa.decode, qa.T = ptr(self.pos_id), 1 if decode else 0, self.T
        qa.q_out, qa.k_cache, qa.v_cache = ptr(acts["q"]), ptr(self.k_cache[li]), ptr(self.v_cache[li])
        qa.status = ptr(self.status)
        self._launches += 1
        N.check(N.load().jx_qkv_rope_append(qa, W.jdt, 1, self.stream_ptr()), "jx_qkv_rope_append")

    def _generic_attention(self, acts, li, lw, S, decode):
        W, cfg = self.w, self.w.cfg
        at = N.JxAttnArgs()
        at.B, at.S, at.Hq, at.Hkv, at.hd, at.T = self.B, S, W.Hq, W.Hkv, W.hd, self.T
        at.q, at.k, at.v = ptr(acts["q"]), ptr(self.k_cache[li]), ptr(self.v_cache[li])
        at.len_ptr, at.len_add = ptr(self.pos_id), 2 if decode else 1
        at.causal = 0 if (decode or S == 1) else 1
        at.window = cfg.sliding_window if lw.sliding else 0
        at.scale = cfg.attn_scale
        at.out = ptr(acts["attn"])
        at.ldo = W.Hq * W.hd
        at.out_rp = acts["Mp"] if W.bf16 else 0
        at.status = ptr(self.status)
        at.uniform_T = self.uniform_T
        self._launches += 1
        N.check(N.load().jx_attention(at, W.jdt, 1, self.stream_ptr()), "jx_attention")

    # Decode attention reads q, k and v straight from the fused projection output and does the RoPE and
    # the cache append itself (no separate RoPE kernel) for the families without QK norm.
    fused_rope = True

    def _decode_attention(self, acts, li, lw, fuse_rope=False):
        W, cfg = self.w, self.w.cfg
        a = N.JxDAttnArgs()
        if fuse_rope:
            cos, sin = (W.cos_l, W.sin_l) if lw.local_rope else (W.cos, W.sin)
            a.qkv, a.ld_qkv, a.cos, a.sin = ptr(acts["qkv"]), W.nqkv, ptr(cos), ptr(sin)
            a.rd, a.max_pos = W.rd, cfg.max_position_embeddings
        a.B, a.Hq, a.Hkv, a.hd, a.T = self.B, W.Hq, W.Hkv, W.hd, self.T
        a.window = cfg.sliding_window if lw.sliding else 0
        a.cache_rows = self.k_cache.shape[0] * self.B * self.T
        a.layer_row0 = li * self.B * self.T
        a.q, a.k_base, a.v_base = ptr(acts["q"]), ptr(self.k_cache), ptr(self.v_cache)
        a.len_ptr, a.len_add = ptr(self.pos_id), 2
        a.scale = cfg.attn_scale
        a.out, a.out_rp = ptr(acts["attn"]), acts["Mp"]
        a.ws, a.ws_bytes = ptr(self.attn_ws), self.attn_ws.numel() * 4
        a.counters, a.status = ptr(self.attn_counters), ptr(self.status)
        self._launches += 2
        N.check(N.load().jx_decode_attention(a, 1, self.stream_ptr()), "jx_decode_attention")

    def _prefill_attention(self, acts, li, lw, S):
        W, cfg = self.w, self.w.cfg
        a = N.JxPAttnArgs()
        a.B, a.S, a.Hq, a.Hkv, a.hd, a.T = self.B, S, W.Hq, W.Hkv, W.hd, self.T
        a.window = cfg.sliding_window if lw.sliding else 0
        a.cache_rows = self.k_cache.shape[0] * self.B * self.T
        a.layer_row0 = li * self.B * self.T
        a.q, a.k_base, a.v_base = ptr(acts["q"]), ptr(self.k_cache), ptr(self.v_cache)
        a.len_ptr, a.len_add = ptr(self.pos_id), 1
        a.scale = cfg.attn_scale
        a.out, a.out_rp = ptr(acts["attn"]), acts["Mp"]
        a.status = ptr(self.status)
        a.uniform_T = self.uniform_T
        self._launches += 1
        N.check(N.load().jx_prefill_attention(a, 1, self.stream_ptr()), "jx_prefill_attention")

    def _o_and_mlp(self, acts, lw, nx):
        """o_proj, residual / post-attention norm, MLP, residual and the next layer's input norm."""
        W, cfg, fam = self.w, self.w.cfg, self.w.family
        M, Mp, d, hd = acts["M"], acts["Mp"], W.d, W.hd
        tp = self.comm is not None
        parallel = fam == "neox" and cfg.use_parallel_residual
        store = N.JX_EPI_STORE_F32 if tp else N.JX_EPI_STORE
        tail = None   # the post-attention norm in o_proj's tail
        # each decode projection warms L2 with the first weights of the one after it
        pf_gu = self._pf(lw.wgu, W.Np_gu, W.Kp_d)
        pf_d = self._pf(lw.wd, W.Np_d, W.Kp_f)
        pf_next = self._pf(nx.wqkv, W.Np_qkv, W.Kp_d) if nx is not None else self._pf(W.lm_head, W.Np_v, W.Kp_d)
        push = tp and not parallel and self._push_ok(acts)
        if push:
            self._linear(acts, lw.wo, W.Np_d, W.Kp_o, "attn", N.JX_EPI_PUSH_F32, N_valid=d, bias=lw.bo,
                         ldo=d, K_logical=W.Hq * hd, N_cols=d)
        elif fam == "gemma3" or parallel or tp:
            # o_proj result kept apart: Gemma normalises it, NeoX's parallel residual adds it with the
            # MLP output, and under tensor parallelism it is a partial sum to all-reduce first.
            dst = self._tp_dst(acts) if tp else acts["tmp"]
            self._linear(acts, lw.wo, W.Np_d, W.Kp_o, "attn", store, N_valid=d, bias=lw.bo,
                         out=dst, ldo=d, K_logical=W.Hq * hd, N_cols=d, pf=pf_gu)
            if not parallel:
                self._allreduce(dst, M, acts)
        else:
            pn = lw.norms["post_attention_layernorm"]
            tail = (pn[0], pn[1]) if self._tail_ok(acts, W.Np_d) else None
            self._linear(acts, lw.wo, W.Np_d, W.Kp_o, "attn", N.JX_EPI_RESID, N_valid=d, bias=lw.bo,
                         out=acts["h"], ldo=d, res=acts["h"], ldr=d, K_logical=W.Hq * hd, N_cols=d, pf=pf_gu,
                         tail=tail)
        # ---- MLP input ----
        if fam == "gemma3":
            pa = lw.norms["post_attention_layernorm"]
            pf = lw.norms["pre_feedforward_layernorm"]
            self._norm(acts, a=acts["tmp"], kind_pre=N.JX_NORM_GEMMA, w_pre=pa[0], b_pre=pa[1], w=pf[0], b=pf[1])
            mlp_in = "xn"
        elif parallel:
            mlp_in = "xn2"      # ln2(h) was produced together with ln1(h)
        else:
            pn = lw.norms["post_attention_layernorm"]
            if tp:
                self._norm(acts, a=acts["tmp"], w=pn[0], b=pn[1])
            elif tail is not None:
                pass   # normalised in o_proj's tail
            elif not self._defer_norm(acts, pn[0], pn[1]):
                self._norm(acts, w=pn[0], b=pn[1])
            mlp_in = "xn"
        # ---- MLP ----
        if W.glu:
            kind = N.JX_EPI_GLU_SILU if fam == "llama" else N.JX_EPI_GLU_GELU_TANH
            self._linear(acts, lw.wgu, W.Np_gu, W.Kp_d, mlp_in, kind, N_valid=W.F, bias=lw.bgu,
                         out=acts["act"], ldo=W.F32, out_rp=Mp if W.bf16 else 0, K_logical=d, N_cols=2 * W.F32,
                         pf=pf_d)
        else:
            self._linear(acts, lw.wgu, W.Np_gu, W.Kp_d, mlp_in, N.JX_EPI_ACT_GELU_ERF, N_valid=W.F, bias=lw.bgu,
                         out=acts["act"], ldo=W.F, out_rp=Mp if W.bf16 else 0, K_logical=d, N_cols=W.F, pf=pf_d)
        Fk = W.F32 if (W.glu and not W.bf16) else W.F
        down_kw = dict(N_valid=d, bias=lw.bd, K_logical=Fk, N_cols=d, pf=pf_next)
        if parallel and tp:
            # attn_partial + mlp_partial accumulate in dst, all-reduced once into tmp; h += tmp in the next norm.
            self._linear(acts, lw.wd, W.Np_d, W.Kp_f, "act", N.JX_EPI_ACC_F32, out=dst, ldo=d, **down_kw)
            self._allreduce(dst, M, acts)
        elif push:
            self._linear(acts, lw.wd, W.Np_d, W.Kp_f, "act", N.JX_EPI_PUSH_F32, ldo=d,
                         **dict(down_kw, pf=None))
        elif fam == "gemma3" or tp:
            dst = self._tp_dst(acts) if tp else acts["tmp"]
            self._linear(acts, lw.wd, W.Np_d, W.Kp_f, "act", store, out=dst, ldo=d, **down_kw)
            self._allreduce(dst, M, acts)
        elif parallel:
            self._linear(acts, lw.wd, W.Np_d, W.Kp_f, "act", N.JX_EPI_RESID2, out=acts["h"], ldo=d,
                         res=acts["h"], ldr=d, res2=acts["tmp"], ldr2=d, **down_kw)
        else:
            down_tail = None
            if nx is not None and not (fam == "neox" and cfg.use_parallel_residual) and self._tail_ok(acts, W.Np_d):
                inw = nx.norms["input_layernorm"]
                down_tail = (inw[0], inw[1])
            self._linear(acts, lw.wd, W.Np_d, W.Kp_f, "act", N.JX_EPI_RESID, out=acts["h"], ldo=d,
                         res=acts["h"], ldr=d, tail=down_tail, **down_kw)
            if down_tail is not None:
                return   # the next layer's input norm ran in down's tail
        # ---- next layer's input norm (the final norm is done by the caller) ----
        if nx is None:
            if fam == "gemma3":
                pf = lw.norms["post_feedforward_layernorm"]
                self._norm(acts, out_key=None, a=acts["tmp"], kind_pre=N.JX_NORM_GEMMA, w_pre=pf[0], b_pre=pf[1])
            elif tp:
                self._norm(acts, out_key=None, a=acts["tmp"], kind=N.JX_NORM_NONE)
            return
        self._input_norm(acts, nx, after=lw)

    def _input_norm(self, acts, lw: LayerWeights, after: Optional[LayerWeights] = None, ids=None):
        W, fam, cfg = self.w, self.w.family, self.w.cfg
        tp = self.comm is not None
        inw = lw.norms["input_layernorm"]
        kw = {}
        if after is not None:
            if fam == "gemma3":
                pf = after.norms["post_feedforward_layernorm"]
                kw = dict(a=acts["tmp"], kind_pre=N.JX_NORM_GEMMA, w_pre=pf[0], b_pre=pf[1])
            elif tp:
                kw = dict(a=acts["tmp"])
        if fam == "neox" and cfg.use_parallel_residual:
            pn = lw.norms["post_attention_layernorm"]
            self._norm(acts, w=inw[0], b=inw[1], out2_key="xn2", w2=pn[0], b2=pn[1], ids=ids, **kw)
        elif kw or ids is not None or not self._defer_norm(acts, inw[0], inw[1]):
            self._norm(acts, w=inw[0], b=inw[1], ids=ids, **kw)

    def _head(self, acts_src, row_map):
        """Final norm of the selected rows into the decode buffers, LM head projection into logits."""
        W = self.w
        dec = self.dec
        fw, fb = W.final_norm
        self._norm(acts_src, w=fw, b=fb, row_map=row_map, M=self.B, out_acts=dec)
        l0 = W.layers[0]   # the next decode step starts with layer 0's qkv projection
        self._linear(dec, W.lm_head, W.Np_v, W.Kp_d, "xn", N.JX_EPI_STORE, N_valid=W.V, out=self.logits_buf(),
                     ldo=W.V, K_logical=W.d, N_cols=W.V, pf=self._pf(l0.wqkv, W.Np_qkv, W.Kp_d))

    def logits_buf(self):
        if getattr(self, "_logits", None) is None:
            self._logits = torch.zeros(self.dec["Mp"], self.w.V, dtype=self.w.dtype, device=self.w.device)
        return self._logits

    def _filtered_logits(self):
        """Full-vocabulary logits [B, V] after the min-p / top-k / top-p filters (tensor parallelism: the
        vocabulary shards are all-gathered first, so every rank filters and samples the same values)."""
        W = self.w
        lg = self.logits_buf()[:self.B]
        if self.comm is not None:
            lg = self.comm.all_gather_vocab(lg)
        if self._flog is None or tuple(self._flog.shape) != (self.B, W.V_total):
            self._flog = torch.empty(self.B, W.V_total, dtype=W.dtype, device=W.device)
            nchunks = (W.V_total + self.sample_chunk - 1) // self.sample_chunk
            self._flog_ws = torch.zeros(self.B * nchunks, dtype=torch.int64, device=W.device)
        from .sampling import filter_logits_

        top_k, top_p, min_p = self.filters
        return filter_logits_(lg, self._flog, top_k, top_p, min_p)

    def _sample(self, greedy: bool, temp: float, update_pos: bool):
        W = self.w
        s = N.JxSampleArgs()
        s.B, s.V = self.B, W.V
        s.logits, s.ld = ptr(self.logits_buf()), W.V
        s.dtype = W.jdt
        s.greedy = 1 if greedy else 0
        s.temp = float(temp) if not greedy else 1.0
        s.chunk = self.sample_chunk
        s.vocab_offset, s.vocab_total = W.vocab_offset, W.V_total
        s.rng, s.gumbel_tab = ptr(self.rng), ptr(W.gumbel)
        s.ws, s.row_best, s.counters = ptr(self.sample_ws), ptr(self.row_best), ptr(self.sample_counters)
        tp = self.comm is not None
        if self.filters is not None and not greedy:
            # filtered full-vocabulary logits, sampled as one shard on every rank
            flog = self._filtered_logits()
            s.V, s.logits, s.ld = W.V_total, ptr(flog), W.V_total
            s.vocab_offset, s.vocab_total = 0, W.V_total
            s.ws = ptr(self._flog_ws)
            tp = False
        s.finalize = 0 if tp else 1
        s.ld_tok = self.tokens_out.shape[1]
        s.tokens_out, s.step, s.next_ids = ptr(self.tokens_out), ptr(self.step), ptr(self.next_ids)
        s.pos_id, s.mask, s.T_mask = ptr(self.pos_id), ptr(self.mask), self.T
        s.update_pos = 1 if update_pos else 0
        s.advance_rng = 1
        s.status = ptr(self.status)
        self._launches += 1
        N.check(N.load().jx_sample(s, 1, self.stream_ptr()), "jx_sample")
        if tp:
            self._launches += 1
            gathered = self.comm.all_gather_keys(self.row_best)
            N.check(N.load().jx_sample_finalize(s, ptr(gathered), self.comm.size, self.stream_ptr()), "jx_sample_finalize")

    # -- public passes --------------------------------------------------------------------------------
    def reset(self, prompt_mask: torch.Tensor, seed_key, sub_key, n_tokens: int):
        """Clear the cache state for a new prompt. ``prompt_mask`` is [B, P] bool (right padded)."""
        B, P = prompt_mask.shape
        self.mask.zero_()
        self.mask[:, :P] = prompt_mask.to(torch.uint8)
        ar = torch.arange(P, device=prompt_mask.device)
        last = torch.argmax(prompt_mask.to(torch.int64) * ar[None, :], dim=1)
        self.pos_id.copy_(last.to(torch.int32))
        words = np.array([seed_key[0], seed_key[1], sub_key[0], sub_key[1]], dtype=np.uint32).view(np.int32)
        self.rng.copy_(torch.from_numpy(words.copy()).to(self.w.device))
        self.step.zero_()
        if self.tokens_out is None or self.tokens_out.shape[1] < n_tokens:
            self.tokens_out = torch.zeros(self.B, max(n_tokens, 1), dtype=torch.int32, device=self.w.device)
            self.graph = None
            self.graph_multi = None
        self.status.zero_()

    def prefill(self, ids: torch.Tensor, greedy: bool, temp: float):
        """Embeds and runs the prompt [B, P] (device int32) through the stack, samples the first token."""
        B, P = ids.shape
        acts = self._prefill_acts(B * P)
        self.k_cache.zero_()
        self.v_cache.zero_()
        flat = ids.reshape(-1).contiguous()
        self._input_norm(acts, self.w.layers[0], ids=flat)
        self._layers(acts, P, decode=False)
        rm = (torch.arange(B, dtype=torch.int32, device=ids.device) * P + (P - 1)).contiguous()
        self._prefill_rowmap = rm
        self._head(acts, rm)
        self._sample(greedy, temp, update_pos=False)

    def _forward_normed(self, ids: torch.Tensor, prompt_mask: torch.Tensor, keep: int) -> tuple:
        """Rows [B, P] (device int32, right-padded ``prompt_mask``) through the stack, then the final norm
        of the last ``keep`` positions of every row (all P when 0) into fresh activation buffers."""
        if self.comm is not None:
            raise NotImplementedError("a cache-free forward under tensor parallelism (the Engine path covers it).")
        W = self.w
        B, P = ids.shape
        self.reset(prompt_mask, np.zeros(2, np.uint32), np.zeros(2, np.uint32), 1)
        acts = self._prefill_acts(B * P)
        self.k_cache.zero_()
        self.v_cache.zero_()
        self._input_norm(acts, W.layers[0], ids=ids.reshape(-1).contiguous())
        self._layers(acts, P, decode=False)
        n = P if keep <= 0 else min(keep, P)
        dev = ids.device
        rows = (torch.arange(B, device=dev)[:, None] * P + torch.arange(P - n, P, device=dev)[None]).reshape(-1)
        M2 = B * n
        out_acts = self._alloc_acts(M2, _rup(M2, 128) if W.bf16 else M2)
        fw, fb = W.final_norm
        self._norm(acts, w=fw, b=fb, row_map=rows.to(torch.int32).contiguous(), M=M2, out_acts=out_acts)
        return out_acts, n

    def forward_logits(self, ids: torch.Tensor, prompt_mask: torch.Tensor, keep: int = 0) -> torch.Tensor:
        """The reference's ``*ModelWithHead.__call__`` without a cache (models/llama.py:247-273): final norm
        and LM head over the last ``keep`` positions of every row (all when 0).  Returns logits
        [B, kept, V] in the model dtype.  Single GPU only."""
        W = self.w
        B = ids.shape[0]
        out_acts, n = self._forward_normed(ids, prompt_mask, keep)
        logits = torch.empty(B * n, W.V, dtype=W.dtype, device=ids.device)
        self._linear(out_acts, W.lm_head, W.Np_v, W.Kp_d, "xn", N.JX_EPI_STORE, N_valid=W.V, out=logits, ldo=W.V,
                     K_logical=W.d, N_cols=W.V)
        return logits.view(B, n, W.V)

    def forward_hidden(self, ids: torch.Tensor, prompt_mask: torch.Tensor) -> torch.Tensor:
        """The reference's ``*Model.__call__`` without a cache (models/llama.py:161-225): the final-normed
        hidden states [B, P, d] in the model dtype.  Single GPU only."""
        W = self.w
        B, P = ids.shape
        out_acts, _ = self._forward_normed(ids, prompt_mask, 0)
        if not W.bf16:
            return out_acts["xn"][:B * P].reshape(B, P, W.d).clone()
        out = torch.empty(B * P, W.d, dtype=W.dtype, device=ids.device)
        N.check(N.load().jx_unpack_k128(ptr(out_acts["xn"]), B * P, W.d, out_acts["Mp"], ptr(out), N.JX_BF16, W.d,
                                        self.stream_ptr()), "jx_unpack_k128")
        return out.view(B, P, W.d)

    def decode_step(self, greedy: bool, temp: float):
        self._launches = 0
        if self.fused_step is not None:
            self._launches += 1
            self.fused_step.launch(self.stream_ptr())
        else:
            acts = self.dec
            self._input_norm(acts, self.w.layers[0], ids=self.next_ids)
            self._layers(acts, 1, decode=True)
            self._head(acts, self.row_map)
        self._sample(greedy, temp, update_pos=True)
        self.launches_last_step = self._launches

    def decode_path_name(self) -> str:
        if self.fused_step is not None:
            return "persistent decode-step kernel"
        return "one launch per op (norm, qkv, attention scores and pv, o_proj, norm, gate/up, down per layer)"

    def count_launches_per_decode_step(self) -> int:
        """libjxb200 kernel launches in one decode step (counted while the step was issued)."""
        return self.launches_last_step

    # decode steps per graph under fuse_decoding (one replay per 16 tokens)
    fused_steps = 16

    def capture_decode(self, greedy: bool, temp: float, steps: int = 1):
        """Captures `steps` consecutive decode steps in one CUDA graph (run one eager step first to warm
        up).  Every step reads its position, step index and key from device memory, so one graph of n
        steps replays n steps of the sequence."""
        key = (greedy, float(temp), self.filters, steps)
        slot = self.graph if steps == 1 else self.graph_multi
        if slot is not None and slot[0] == key:
            return slot[1]
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream(self.w.device)
        s.wait_stream(torch.cuda.current_stream(self.w.device))
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                for _ in range(steps):
                    self.decode_step(greedy, temp)
        torch.cuda.current_stream(self.w.device).wait_stream(s)
        if steps == 1:
            self.graph = (key, g)
        else:
            self.graph_multi = (key, g)
        return g

    def generate(self, prompt: torch.Tensor, mask: torch.Tensor, n_new: int, greedy: bool, temp: float, seed: int,
                 fuse: bool = False, first_len: int = 0):
        """Prefill + (n_new - 1) decode steps on the device; returns device tokens [B, n_new].

        The first decode step runs eagerly (it also warms every kernel up); the rest replay a captured
        CUDA graph of one step, or with `fuse` (the reference's fuse_decoding: the decode loop compiled
        as one scan, _generate.py:365-380) a graph of `fused_steps` steps, the remainder on the one-step
        graph.  Key flow as _generate.py: key = PRNGKey(seed); key, sub = split(key) before the first
        sample, and one split per decode step on the device.  `first_len` is the cache length the
        reference's chunk loop starts with (engine.py:543-557); the buffer here is allocated at its final
        length, which changes nothing but the uniform attention of a prompt row with no visible key, so
        that attention is confined to the first `first_len` slots.
        """
        from . import prng

        key, sub = prng.split(prng.prng_key(seed))
        self.reset(mask, key, sub, n_new)
        self.uniform_T = first_len
        try:
            self.prefill(prompt, greedy, temp)
        finally:
            self.uniform_T = 0
        if n_new > 1:
            self.decode_step(greedy, temp)
        rest = max(n_new - 2, 0)
        if fuse and rest >= 2:
            k = min(self.fused_steps, rest)
            g = self.capture_decode(greedy, temp, k)
            for _ in range(rest // k):
                g.replay()
            rest %= k
        if rest:
            g = self.capture_decode(greedy, temp)
            for _ in range(rest):
                g.replay()
        return self.tokens_out[:, :n_new]

    def rng_key(self) -> np.ndarray:
        return self.rng[:2].cpu().numpy().view(np.uint32).copy()

    def check_status(self):
        st = int(self.status[0].item())
        if st != 0:
            self.status.zero_()
            self.gemv_counters.zero_()
            self.sample_counters.zero_()
            self.tn_sync.zero_()
            if self.fast_attn:
                self.attn_counters.zero_()
                self.attn_ws.zero_()   # (the queue form's claim counters live in its tail)
            raise N.NativeError(f"device status {st} ({N.STATUS_NAMES.get(st, st)}) during generation")
