"""ctypes binding of ``libjxb200.so`` (declared in ``include/jxb200.h``).

The library is the only compute path: if it cannot be loaded, every op raises instead of falling back.
"""
from __future__ import annotations

import ctypes
import os
import re

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libjxb200.so")
HEADER = os.path.join(os.path.dirname(PKG), "include", "jxb200.h")

JX_OK, JX_ERR_ARG, JX_ERR_SHAPE, JX_ERR_DTYPE, JX_ERR_RANGE, JX_ERR_TIMEOUT, JX_ERR_CUDA, JX_ERR_UNSUPPORTED = range(8)
JX_F32, JX_BF16 = 0, 1
JX_NORM_NONE, JX_NORM_RMS, JX_NORM_GEMMA, JX_NORM_LAYER = 0, 1, 2, 3
(JX_EPI_STORE, JX_EPI_RESID, JX_EPI_GLU_SILU, JX_EPI_GLU_GELU_TANH, JX_EPI_ACT_GELU_ERF, JX_EPI_RESID2,
 JX_EPI_STORE_F32, JX_EPI_ACC_F32, JX_EPI_PUSH_F32) = range(9)

STATUS_NAMES = {
    JX_OK: "ok", JX_ERR_ARG: "bad argument", JX_ERR_SHAPE: "bad shape", JX_ERR_DTYPE: "bad dtype",
    JX_ERR_RANGE: "index out of range", JX_ERR_TIMEOUT: "device wait timed out", JX_ERR_CUDA: "CUDA error",
    JX_ERR_UNSUPPORTED: "unsupported",
}

P = ctypes.c_void_p
LL = ctypes.c_longlong
I = ctypes.c_int
F = ctypes.c_float


class JxEpilogue(ctypes.Structure):
    _fields_ = [("kind", I), ("M", I), ("N", I), ("pf_iters", I), ("bias", P), ("out", P), ("ldo", LL),
                ("out_rp", LL), ("res", P), ("ldr", LL), ("res2", P), ("ldr2", LL), ("pf_w", P), ("pf_np", LL),
                ("pf_kp", LL), ("pf_rows", I), ("pf_grid", I), ("peer_bases", P), ("peer_recv_off", LL),
                ("peer_slot_bytes", LL), ("peer_flag_off", LL), ("peer_seq_off", LL), ("peer_rank", I), ("peer_world", I),
                ("pn_h", P), ("pn_ldh", LL), ("pn_w", P), ("pn_b", P), ("pn_sync", P), ("pn_kind", I), ("pn_d", I),
                ("pn_eps", F), ("_pad1", I), ("tn_x", P), ("tn_rp", LL), ("tn_w", P), ("tn_b", P), ("tn_sync", P),
                ("tn_kind", I), ("tn_eps", F)]


class JxNormArgs(ctypes.Structure):
    _fields_ = [("M", I), ("d", I), ("eps", F), ("kind", I), ("kind_pre", I), ("vocab", I), ("ids", P),
                ("table", P), ("embed_scale", F), ("a_f32", I), ("row_map", P), ("a", P), ("lda", LL), ("h", P),
                ("ldh", LL), ("w_pre", P), ("b_pre", P), ("w", P), ("b", P), ("out", P), ("ldo", LL),
                ("out_rp", LL), ("w2", P), ("b2", P), ("out2", P), ("ldo2", LL), ("out2_rp", LL), ("status", P),
                ("peer_recv", P), ("peer_stride", LL), ("peer_flags", P), ("peer_seq", P), ("peer_world", I),
                ("peer_units", I)]


class JxQkvArgs(ctypes.Structure):
    _fields_ = [("M", I), ("S", I), ("Hq", I), ("Hkv", I), ("hd", I), ("rd", I), ("qkv", P), ("ld_qkv", LL),
                ("qn_w", P), ("kn_w", P), ("eps", F), ("max_pos", I), ("cos", P), ("sin", P), ("pos_id", P),
                ("decode", I), ("T", I), ("q_out", P), ("k_cache", P), ("v_cache", P), ("status", P)]


class JxAttnArgs(ctypes.Structure):
    _fields_ = [("B", I), ("S", I), ("Hq", I), ("Hkv", I), ("hd", I), ("T", I), ("q", P), ("k", P), ("v", P),
                ("len_ptr", P), ("len_add", I), ("causal", I), ("window", I), ("scale", F), ("out", P),
                ("ldo", LL), ("out_rp", LL), ("status", P), ("weights", P), ("uniform_T", I), ("_pad1", I)]


class JxRopeArgs(ctypes.Structure):
    _fields_ = [("M", I), ("Hq", I), ("Hk", I), ("hd", I), ("rd", I), ("n_pos", I), ("q", P), ("k", P), ("q_out", P),
                ("k_out", P), ("cos", P), ("sin", P), ("pos", P), ("status", P)]


class JxDAttnArgs(ctypes.Structure):
    _fields_ = [("B", I), ("Hq", I), ("Hkv", I), ("hd", I), ("T", I), ("window", I), ("cache_rows", LL),
                ("layer_row0", LL), ("q", P), ("k_base", P), ("v_base", P), ("len_ptr", P), ("len_add", I),
                ("scale", F), ("out", P), ("out_rp", LL), ("ws", P), ("ws_bytes", LL), ("counters", P),
                ("status", P), ("qkv", P), ("ld_qkv", LL), ("cos", P), ("sin", P), ("rd", I), ("max_pos", I)]


class JxPAttnArgs(ctypes.Structure):
    _fields_ = [("B", I), ("S", I), ("Hq", I), ("Hkv", I), ("hd", I), ("T", I), ("window", I), ("uniform_T", I),
                ("cache_rows", LL), ("layer_row0", LL), ("q", P), ("k_base", P), ("v_base", P), ("len_ptr", P),
                ("len_add", I), ("scale", F), ("out", P), ("out_rp", LL), ("status", P)]


class JxSampleArgs(ctypes.Structure):
    _fields_ = [("B", I), ("V", I), ("logits", P), ("ld", LL), ("dtype", I), ("greedy", I), ("temp", F),
                ("chunk", I), ("vocab_offset", LL), ("vocab_total", LL), ("rng", P), ("gumbel_tab", P), ("ws", P),
                ("row_best", P), ("counters", P), ("finalize", I), ("ld_tok", I), ("tokens_out", P), ("step", P),
                ("next_ids", P), ("pos_id", P), ("mask", P), ("T_mask", I), ("update_pos", I),
                ("advance_rng", I), ("_pad0", I), ("status", P)]


class JxFilterArgs(ctypes.Structure):
    _fields_ = [("B", I), ("V", I), ("logits", P), ("ld_in", LL), ("out", P), ("ld_out", LL), ("dtype", I),
                ("top_k", I), ("top_p", F), ("min_p", F)]


class JxStepArgs(ctypes.Structure):
    _fields_ = [("M", I), ("L", I), ("d", I), ("Hq", I), ("Hkv", I), ("hd", I), ("F", I), ("V", I), ("vocab", I),
                ("T", I), ("rd", I), ("max_pos", I), ("Np_qkv", LL), ("Np_d", LL), ("Np_gu", LL), ("Np_v", LL),
                ("Kp_d", LL), ("Kp_o", LL), ("Kp_f", LL), ("eps", F), ("scale", F), ("layers", P), ("embed", P),
                ("ids", P), ("final_norm", P), ("lm_head", P), ("h", P), ("xn", P), ("qkv", P), ("attn", P),
                ("act", P), ("logits", P), ("k_cache", P), ("v_cache", P), ("cos", P), ("sin", P), ("pos_id", P),
                ("ws", P), ("ws_floats", LL), ("counters", P), ("attn_ws", P), ("attn_ws_bytes", LL),
                ("attn_counters", P), ("sync", P), ("status", P), ("grid", I)]


_PROTOS = {
    "jx_version": (ctypes.c_char_p, []),
    "jx_last_error": (ctypes.c_char_p, []),
    "jx_device_sm_count": (I, [ctypes.POINTER(I)]),
    "jx_memset_async": (I, [P, I, LL, P]),
    "jx_pack_k128": (I, [P, I, LL, LL, LL, I, P, LL, LL, P]),
    "jx_unpack_k128": (I, [P, LL, LL, LL, P, I, LL, P]),
    "jx_norm": (I, [ctypes.POINTER(JxNormArgs), I, I, P]),
    "jx_linear_decode_workspace": (I, [I, I, ctypes.POINTER(LL)]),
    "jx_set_decode_linear_impl": (I, [I]),
    "jx_set_prefill_tile_group": (I, [I]),
    "jx_set_prefill_linear_impl": (I, [I]),
    "jx_set_prefill_attention_impl": (I, [I]),
    "jx_linear_decode": (I, [P, P, LL, LL, I, ctypes.POINTER(JxEpilogue), P, LL, P, P, I, I, P]),
    "jx_linear_decode_noalloc": (I, [P, P, LL, LL, I, ctypes.POINTER(JxEpilogue), P, I, I, P]),
    "jx_linear_prefill": (I, [P, P, LL, LL, LL, ctypes.POINTER(JxEpilogue), P, I, P]),
    "jx_linear_f32": (I, [P, LL, P, I, I, I, ctypes.POINTER(JxEpilogue), I, P]),
    "jx_qkv_rope_append": (I, [ctypes.POINTER(JxQkvArgs), I, I, P]),
    "jx_rope_apply": (I, [ctypes.POINTER(JxRopeArgs), I, I, P]),
    "jx_mlp_act": (I, [P, LL, P, LL, P, LL, LL, LL, I, I, I, P]),
    "jx_attention": (I, [ctypes.POINTER(JxAttnArgs), I, I, P]),
    "jx_decode_attention_workspace": (I, [I, I, I, I, I, ctypes.POINTER(LL)]),
    "jx_decode_attention": (I, [ctypes.POINTER(JxDAttnArgs), I, P]),
    "jx_set_decode_attention_impl": (I, [I]),
    "jx_prefill_attention": (I, [ctypes.POINTER(JxPAttnArgs), I, P]),
    "jx_sample": (I, [ctypes.POINTER(JxSampleArgs), I, P]),
    "jx_filter_logits": (I, [ctypes.POINTER(JxFilterArgs), P]),
    "jx_decode_step": (I, [ctypes.POINTER(JxStepArgs), P]),
    "jx_set_decode_step_lookahead": (I, [I]),
    "jx_sample_finalize": (I, [ctypes.POINTER(JxSampleArgs), P, I, P]),
    "jx_comm_alloc": (I, [LL, ctypes.POINTER(P)]),
    "jx_comm_free": (I, [P]),
    "jx_ipc_get_handle": (I, [P, ctypes.c_char_p]),
    "jx_ipc_open_handle": (I, [ctypes.c_char_p, ctypes.POINTER(P)]),
    "jx_ipc_close_handle": (I, [P]),
    "jx_comm_layout": (I, [LL, I, ctypes.POINTER(LL)]),
    "jx_allreduce_f32": (I, [ctypes.POINTER(P), I, I, LL, I, LL, P, P, I, P]),
}

_lib = None


class NativeError(RuntimeError):
    pass


def header_symbols() -> list[str]:
    """Function names declared in include/jxb200.h."""
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\**\s+\**(jx_\w+)\s*\(", text, flags=re.M)))


def load(path: str = LIB_PATH):
    """Loads the library (it must have been built with ``jaxml_b200.build``)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise NativeError(f"libjxb200.so not found at {path}; build it with `python -m jaxml_b200.build`.")
    lib = ctypes.CDLL(path)
    for name, (res, args) in _PROTOS.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(rc: int, what: str):
    if rc != JX_OK:
        msg = load().jx_last_error().decode(errors="replace")
        raise NativeError(f"{what} failed ({STATUS_NAMES.get(rc, rc)}): {msg}")


def call(name: str, *args):
    rc = getattr(load(), name)(*args)
    check(rc, name)
    return rc


def ptr(t) -> int | None:
    """Device pointer of a torch tensor (None for None)."""
    return None if t is None else t.data_ptr()
