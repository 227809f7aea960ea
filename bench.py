#!/usr/bin/env python
"""Decode throughput of a Llama-3-8B-shaped bfloat16 model (jaxml's Engine.generate path on B200).

Workload (the headline configuration): 32 layers, d 4096, 32 query / 8 KV heads x 128, SwiGLU FFN
14336, vocab 128256, RoPE theta 5e5, RMSNorm eps 1e-5, random N(0, 0.02) weights (seed 0), batch 16,
512 uniform-random prompt ids per row (seed 0), greedy decoding.  One step = one decode step of the
whole batch (16 tokens).  The device-timed steps are steps warmup+1 .. warmup+steps of a generation
(the line states the contexts they ran at); the e2e leg always generates the workload's 256 new tokens
through Engine.generate.  Weights (15 GB) are far larger than L2, so no flush is needed between steps.

--gpus N > 1 (launched with torchrun) runs tensor parallelism over N GPUs (NCCL): heads, FFN columns and
the vocabulary are split N ways; the batch and total work stay fixed (strong scaling).

--impl reference times the CPU restatement of jaxml's math (the oracle; JAX itself is not installed) on
the host cores for the same metric.  Each of its steps is a bounded sample of one decode step: one
decoder layer of the batch at context 512 plus 1/32 of the LM head; the metric scales the sample time
by 32 (the line says so in "extrapolated").
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)


# DRAM bytes (read 235079424 + write 4493056) of one launch of the tcgen05 decode projection on the
# gate/up shape (M=16, N=28672, K=4096), from an ncu --set full capture of
# `python bench.py --micro gemv --shape 28672,4096`.
GEMV_TC_GATEUP_TRAFFIC = 239572480


def l8_config(num_layers=32):
    from jaxml_b200.config import ModelConfig

    return ModelConfig(hidden_size=4096, head_dim=128, num_heads=32, num_kv_heads=8, num_layers=num_layers,
                       intermediate_ratio=(7, 2), max_position_embeddings=131072, vocab_size=128256,
                       norm_eps=1e-5, rope_theta=500000.0)


def nx_config():
    from jaxml_b200.config import ModelConfig

    return ModelConfig(hidden_size=512, head_dim=64, num_heads=8, num_layers=6, max_position_embeddings=2048,
                       vocab_size=50304, intermediate_ratio=(4, 1), norm_eps=1e-5, rotary_pct=0.25,
                       use_parallel_residual=True, use_bias=True)


def g12_config(num_layers=48):
    from jaxml_b200.config import ModelConfig

    return ModelConfig(hidden_size=3840, head_dim=256, num_heads=16, num_kv_heads=8, num_layers=num_layers,
                       intermediate_ratio=(4, 1), max_position_embeddings=8704, vocab_size=262144, norm_eps=1e-6,
                       sliding_window=1024, sliding_window_pattern=6, rope_theta=1000000.0, attn_scale=256 ** -0.5)


def l70_config(num_layers=80):
    from jaxml_b200.config import ModelConfig

    return ModelConfig(hidden_size=8192, head_dim=128, num_heads=64, num_kv_heads=8, num_layers=num_layers,
                       intermediate_ratio=(7, 2), max_position_embeddings=131072, vocab_size=128256,
                       norm_eps=1e-5, rope_theta=500000.0)


# The configurations (model shape, batch, prompt, new tokens, compute dtype).  l8 is the headline.
CONFIGS = {
    "l8": dict(family="llama", make=l8_config, B=16, P=512, new=256, dtype="bf16",
               name="Llama-3-8B-shape bf16"),
    "nx": dict(family="neox", make=nx_config, B=1, P=32, new=64, dtype="f32",
               name="GPT-NeoX pythia-70m-shape fp32"),
    "g12": dict(family="gemma3", make=g12_config, B=8, P=8192, new=128, dtype="bf16",
                name="Gemma3-12B-shape bf16"),
    "l70": dict(family="llama", make=l70_config, B=64, P=2048, new=128, dtype="bf16",
                name="Llama-3-70B-shape bf16"),
}


class LazyLayers(dict):
    """The per-layer parameter subtrees of a random-init model, made when first read and not kept: packing
    a rank's shard of a 70B-shaped model then never holds more than one full layer on the device."""

    def __init__(self, family, cfg, seed, dtype, device, body):
        super().__init__(body)
        self.family, self.cfg, self.seed, self.dtype, self.device = family, cfg, seed, dtype, device

    def __getitem__(self, key):
        if isinstance(key, str) and key.startswith("layers_") and not dict.__contains__(self, key):
            from jaxml_b200.models import random_params

            i = int(key.split("_")[1])
            one = random_params(self.family, self.cfg.replace(num_layers=1), seed=self.seed * 100003 + i + 1,
                                dtype=self.dtype, device=self.device)
            body = one["params"]["gpt_neox" if self.family == "neox" else "model"]
            return body["layers_0"]
        return dict.__getitem__(self, key)

    def __contains__(self, key):
        if isinstance(key, str) and key.startswith("layers_"):
            return int(key.split("_")[1]) < self.cfg.num_layers
        return dict.__contains__(self, key)


def lazy_random_params(family, cfg, seed, dtype, device):
    """random_params' tree (N(0, 0.02) kernels) with layers made on demand (LazyLayers)."""
    from jaxml_b200.models import random_params

    top = random_params(family, cfg.replace(num_layers=1), seed=seed, dtype=dtype, device=device)
    root = "gpt_neox" if family == "neox" else "model"
    body = {k: v for k, v in top["params"][root].items() if not k.startswith("layers_")}
    top["params"][root] = LazyLayers(family, cfg, seed, dtype, device, body)
    return top


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--config", choices=sorted(CONFIGS), default="l8",
                    help="model / workload: l8 Llama-3-8B shape (headline), nx pythia-70m shape fp32, g12 Gemma3-12B "
                         "shape, l70 Llama-3-70B shape (tensor parallel only)")
    ap.add_argument("--steps", type=int, default=252)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=None, help="batch rows (default: the config's)")
    ap.add_argument("--prompt", type=int, default=None, help="prompt length (default: the config's)")
    ap.add_argument("--layers", type=int, default=None, help="decoder layers (default: the config's)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-temp", action="store_true", help="skip the temperature-0.8 decode timing")
    ap.add_argument("--tail-norms", action="store_true",
                    help="decode step: the norms after o_proj / down in those projections' last CTA")
    ap.add_argument("--per-op", action="store_true",
                    help="decode with one kernel launch per op instead of the persistent decode-step kernel")
    ap.add_argument("--e2e-tokens", type=int, default=None,
                    help="new tokens per row of the e2e generation (default: the config's, 256 for l8)")
    ap.add_argument("--tp-pull", action="store_true",
                    help="tensor-parallel decode: separate pull all-reduce kernels instead of the push-fused projections")
    ap.add_argument("--micro", choices=["gemv", "attn", "gemm", "allreduce", "tpx", "filter", "sweep"], default=None,
                    help="single-kernel microbenchmark on Llama-3-8B layer shapes instead of the decode step")
    ap.add_argument("--ctx", type=int, default=4096, help="context length of --micro attn")
    ap.add_argument("--shape", default="28672,4096", help="N,K of --micro gemv (default: fused gate/up)")
    ap.add_argument("--gemv-impl", type=int, default=0, help="--micro gemv kernel: 0 by shape, 1 mma.sync, 2 tcgen05")
    ap.add_argument("--grids", default="148", help="--micro gemv: comma-separated CTA counts to time (one line each)")
    ap.add_argument("--tile-groups", default="", help="--micro gemm: comma-separated tile-group sizes to time")
    ap.add_argument("--attn-impl", type=int, default=0, help="decode attention form: 0 by shape, 1 split, 2 cluster, 3 column pv, 4 cluster-split, 5 queue")
    ap.add_argument("--tokens", type=int, default=8192, help="token rows of --micro gemm (prefill B x P)")
    ap.add_argument("--gemm-impl", type=int, default=0, help="--micro gemm kernel: 0 by shape, 1 mma.sync, 2 tcgen05")
    return ap.parse_args()


# ------------------------------------------------------------------------------------------------
# clocks sampled during the timed region
# ------------------------------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------------------------------------
# algorithmic bytes
# ------------------------------------------------------------------------------------------------
def step_bytes(cfg, B, ctx_mean, tp=1, family="llama", elem=2):
    """Weight + KV bytes one decode step must move per GPU: every layer's projection weights (and norms),
    the final norm, the LM head (vocabulary-parallel under tensor parallelism), the B embedding rows, and
    the K / V of the keys each layer attends to (Gemma3's sliding-window layers only their window)."""
    d, H, Hkv, hd, F, V = (cfg.hidden_size, cfg.num_heads, cfg.num_key_value_heads, cfg.head_dim,
                           cfg.intermediate_size, cfg.vocab_size)
    mlp = 2 * d * F if family == "neox" else 3 * d * F
    per_layer = (d * (H + 2 * Hkv) * hd + H * hd * d + mlp) / tp + 2 * d
    weights = elem * (cfg.num_layers * per_layer + d + d * V / tp + B * d)
    kv = 0.0
    for i in range(cfg.num_layers):
        local = family == "gemma3" and cfg.sliding_window and (i + 1) % (cfg.sliding_window_pattern or 1)
        keys = min(ctx_mean, cfg.sliding_window) if local else ctx_mean
        kv += B * keys * 2 * (Hkv / tp) * hd * elem
    return weights + kv, weights, kv


# DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum) from single-kernel ncu captures
# of the bench's micro shapes, where one was taken (profiles/ names the capture); None otherwise.
NCU_TRAFFIC = {
    "gate/up projection": (GEMV_TC_GATEUP_TRAFFIC, "ncu --set full of `bench.py --micro gemv --shape 28672,4096` "
                           "(profiles/gemv_tc_gateup_ncu.md)"),
    "o_proj projection": (33720000, "ncu --set full of `bench.py --micro gemv --shape 4096,4096 --gemv-impl 1` "
                          "(profiles/gemv_k128_o_proj_ncu.md)"),
}


def kernel_table(rt, cfg, ctx, step_ms, n_layers=8):
    """Per-kernel device time of the decode step's kernels, each launched back to back over `n_layers`
    distinct layers (weights larger than L2 in total) from a CUDA graph and timed with CUDA events on the
    replay stream.  bytes = algorithmic bytes per launch (weights as stored, activations in and out, K/V
    of `ctx` keys); share = time per launch x launches per step / the measured step time."""
    import torch

    from jaxml_b200 import _native as N

    w, acts = rt.w, rt.dec
    B, d = rt.B, w.d
    layers = w.layers[:n_layers]
    L = cfg.num_layers
    rows = []

    def add(kernel, per_step, fns, nbytes):
        us = _graph_ms(lambda _s: [f() for f in fns], len(fns)) * 1e3
        tr = NCU_TRAFFIC.get(kernel)
        rows.append({"kernel": kernel, "launches_per_step": per_step, "us": us, "bytes": nbytes,
                     "gbs": nbytes / us / 1e3, "share": us * per_step / (step_ms * 1e3),
                     "traffic": tr[0] if tr else None, "traffic_note": tr[1] if tr else "no ncu capture"})

    if rt.fused_step is not None:
        # the persistent decode-step kernel: one launch runs every layer, the final norm and the LM head
        nbytes, _, _ = step_bytes(cfg, B, ctx)
        add("decode_step_kernel (persistent: %d layers + final norm + LM head)" % L, 1,
            [lambda: rt.fused_step.launch(torch.cuda.current_stream().cuda_stream)] * 4, nbytes)
        return rows
    else:
        x_b = 2 * B * d
        add("qkv projection", L, [lambda lw=lw: rt._linear(acts, lw.wqkv, w.Np_qkv, w.Kp_d, "xn", N.JX_EPI_STORE,
                                                          N_valid=w.nqkv, out=acts["qkv"], ldo=w.nqkv)
                                  for lw in layers], 2 * w.nqkv * d + x_b + 2 * B * w.nqkv)
        add("attention (scores + pv)", L, [lambda li=li, lw=lw: rt._decode_attention(acts, li, lw, True)
                                           for li, lw in enumerate(layers)],
            B * ctx * 2 * w.Hkv * w.hd * 2 + 2 * B * w.nqkv + 2 * B * w.Hq * w.hd)
        add("o_proj projection", L, [lambda lw=lw: rt._linear(acts, lw.wo, w.Np_d, w.Kp_o, "attn", N.JX_EPI_RESID,
                                                             N_valid=d, out=acts["h"], ldo=d, res=acts["h"], ldr=d)
                                     for lw in layers], 2 * d * w.Hq * w.hd + 2 * B * w.Hq * w.hd + 2 * x_b)
        add("norm", 2 * L + 1, [lambda lw=lw: rt._norm(acts, w=lw.norms["post_attention_layernorm"][0])
                                for lw in layers], 2 * x_b)
        add("gate/up projection", L, [lambda lw=lw: rt._linear(acts, lw.wgu, w.Np_gu, w.Kp_d, "xn", N.JX_EPI_GLU_SILU,
                                                              N_valid=w.F, out=acts["act"], ldo=w.F32,
                                                              out_rp=acts["Mp"]) for lw in layers],
            2 * 2 * w.F * d + x_b + 2 * B * w.F)
        add("down projection", L, [lambda lw=lw: rt._linear(acts, lw.wd, w.Np_d, w.Kp_f, "act", N.JX_EPI_RESID,
                                                           N_valid=d, out=acts["h"], ldo=d, res=acts["h"], ldr=d)
                                   for lw in layers], 2 * d * w.F + 2 * B * w.F + 2 * x_b)
    add("LM head projection", 1, [lambda: rt._linear(acts, w.lm_head, w.Np_v, w.Kp_d, "xn", N.JX_EPI_STORE,
                                                     N_valid=w.V, out=rt.logits_buf(), ldo=w.V)] * 4,
        2 * w.V * d + 2 * B * d + 2 * B * w.V)
    return rows


def prefill_table(rt, cfg, prefill_ms, n_layers=8):
    """Per-op device time of the prefill's kernels (sequential-residual Llama layers), each launched back
    to back over `n_layers` distinct layers from a CUDA graph and timed with CUDA events on the replay
    stream, on the prefill's own buffers (the timing does not depend on their values).  flop / bytes =
    algorithmic work per launch (causal attention: the visible half of the score matrix); share = time
    per launch x launches per prefill / the measured prefill time.  The RoPE + append rows rewrite the
    K/V cache of the first layers: run it after everything that reads the runtime's cache."""
    from jaxml_b200 import _native as N

    w, acts = rt.w, rt.pre
    M, Mp, d = acts["M"], acts["Mp"], w.d
    S = M // rt.B
    layers = w.layers[:n_layers]
    L = cfg.num_layers
    Fk = w.F32 if (w.glu and not w.bf16) else w.F
    rows = []

    def add(op, per, fns, flop=None, nbytes=None):
        us = _graph_ms(lambda _s: [f() for f in fns], len(fns)) * 1e3
        r = {"op": op, "launches_per_prefill": per, "us": us, "share": us * per / (prefill_ms * 1e3)}
        if flop is not None:
            r.update(flop=flop, tflops=flop / us / 1e6)
        if nbytes is not None:
            r.update(bytes=nbytes, gbs=nbytes / us / 1e3)
        rows.append(r)

    add("qkv projection (tcgen05 GEMM)", L,
        [lambda lw=lw: rt._linear(acts, lw.wqkv, w.Np_qkv, w.Kp_d, "xn", N.JX_EPI_STORE, N_valid=w.nqkv, bias=lw.bqkv,
                                  out=acts["qkv"], ldo=w.nqkv, K_logical=d, N_cols=w.nqkv) for lw in layers],
        flop=2.0 * M * w.nqkv * d)
    add("RoPE + KV append", L, [lambda li=li, lw=lw: rt._qkv_rope_append(acts, li, lw, S, False)
                                for li, lw in enumerate(layers)], nbytes=4.0 * M * w.nqkv)
    add("attention (causal)", L, [lambda li=li, lw=lw: rt._prefill_attention(acts, li, lw, S)
                                  for li, lw in enumerate(layers)], flop=2.0 * rt.B * w.Hq * w.hd * S * S)
    add("o_proj projection (tcgen05 GEMM, residual add)", L,
        [lambda lw=lw: rt._linear(acts, lw.wo, w.Np_d, w.Kp_o, "attn", N.JX_EPI_RESID, N_valid=d, bias=lw.bo,
                                  out=acts["h"], ldo=d, res=acts["h"], ldr=d, K_logical=w.Hq * w.hd, N_cols=d)
         for lw in layers], flop=2.0 * M * d * w.Hq * w.hd)
    add("norm", 2 * L - 1, [lambda lw=lw: rt._norm(acts, w=lw.norms["post_attention_layernorm"][0],
                                                   b=lw.norms["post_attention_layernorm"][1]) for lw in layers],
        nbytes=4.0 * M * d)
    add("gate/up projection (tcgen05 GEMM, SwiGLU)", L,
        [lambda lw=lw: rt._linear(acts, lw.wgu, w.Np_gu, w.Kp_d, "xn", N.JX_EPI_GLU_SILU, N_valid=w.F, bias=lw.bgu,
                                  out=acts["act"], ldo=w.F32, out_rp=Mp, K_logical=d, N_cols=2 * w.F32)
         for lw in layers], flop=2.0 * M * 2 * w.F * d)
    add("down projection (tcgen05 GEMM, residual add)", L,
        [lambda lw=lw: rt._linear(acts, lw.wd, w.Np_d, w.Kp_f, "act", N.JX_EPI_RESID, out=acts["h"], ldo=d,
                                  res=acts["h"], ldr=d, N_valid=d, bias=lw.bd, K_logical=Fk, N_cols=d)
         for lw in layers], flop=2.0 * M * d * w.F)
    rt.check_status()
    return rows


# ------------------------------------------------------------------------------------------------
# CPU baseline: the oracle restatement on the host cores (bounded sample)
# ------------------------------------------------------------------------------------------------
def cpu_decode_samples(conf, B, ctx, n_warm=1, n_timed=3, budget_s=60.0, seed=0):
    """Seconds per sample of one decode step of configuration `conf` on the host cores (the oracle): one
    decoder layer of the batch at context `ctx` plus 1/L of the LM head's columns, so L samples (L = the
    model's layers) are one full step's work.  Times up to `n_timed` samples after `n_warm` untimed ones,
    stopping early once `budget_s` seconds of timed work have run.  Returns (sample seconds, threads, L)."""
    import torch

    from oracle import jaxml_oracle as O

    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    full = conf["make"]()
    L = full.num_layers
    cfg = full.replace(num_layers=1)
    dt = torch.bfloat16 if conf["dtype"] == "bf16" else torch.float32
    family = conf["family"]
    params = O.init_params(family, cfg, seed=seed, dtype=dt)
    head = params["params"]["lm_head"]["kernel"][:, : max(1, cfg.vocab_size // L)].contiguous()
    T = (ctx // 256 + 1) * 256
    g = torch.Generator().manual_seed(seed)
    c = O.OracleKVCache(T, dt)
    k = (torch.randn(B, ctx, cfg.num_key_value_heads, cfg.head_dim, generator=g)).to(dt)
    caches = (c.update(k, k.clone(), None),)
    tok = torch.randint(0, cfg.vocab_size, (B, 1), generator=g, dtype=torch.int32)

    def one():
        out = O.forward(family, cfg, params, tok, dt, kv_caches=caches, with_head=False)
        O.dense(out.last_hidden_state, head, None, dt)
    for _ in range(n_warm):
        one()
    times = []
    for _ in range(n_timed):
        t0 = time.perf_counter()
        one()
        times.append(time.perf_counter() - t0)
        if sum(times) > budget_s:
            break
    return times, threads, L


def cpu_sample_note(B, ctx, L):
    return ("torch-CPU restatement of jaxml's math (JAX is not installed): each sample is one decoder layer of a "
            "batch-%d decode step at context %d plus 1/%d of the LM head; tok/s = %d / (%d x sample time)"
            % (B, ctx, L, B, L))


def metric_of(conf):
    return "decode tok/s (box) & p50 step latency, %s, TP=1/2/4/8" % conf["name"]


def reference_arm(args):
    """--impl reference: the oracle timed on the host cores, the same metric and config.  Rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    conf = CONFIGS[args.config]
    times, threads, L = cpu_decode_samples(conf, B=args.batch, ctx=args.prompt, n_warm=max(1, min(args.warmup, 2)),
                                           n_timed=max(1, args.steps), budget_s=60.0)
    sample_s = sum(times) / len(times)
    value = args.batch / (L * sample_s)
    line = {
        "metric": metric_of(conf), "value": value, "unit": "tok/s", "n_gpus": args.gpus, "steps": len(times),
        "warmup": max(1, min(args.warmup, 2)), "ms_per_step": sample_s * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": conf["dtype"],
        "data": "synthetic (uniform-random ids, N(0,0.02) weights, seed 0)",
        "config": {"workload": "%s decode, batch %d, context %d (one layer + 1/%d LM head per step, scaled by %d)"
                               % (conf["name"], args.batch, args.prompt, L, L),
                   "global_batch": args.batch, "seq_len": args.prompt, "parallelism": "cpu"},
        "extrapolated": {"timed": "one decoder layer + 1/%d of the LM head per step (a 1/%d sample of a decode step)"
                                  % (L, L), "scale": L, "full_step_ms": L * sample_s * 1e3},
        "impl": "reference",
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": cpu_sample_note(args.batch, args.prompt, L)},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------------
# GPU arm
# ------------------------------------------------------------------------------------------------
def gpu_arm(args):
    import numpy as np
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    from jaxml_b200 import Engine, GemmaModelWithHead, GPTNeoXModelWithHead, InferenceConfig, LlamaModelWithHead

    tp = world
    if args.attn_impl:
        from jaxml_b200 import _native as N

        N.call("jx_set_decode_attention_impl", args.attn_impl)
    if args.tp_pull or args.per_op or args.tail_norms:
        from jaxml_b200.runtime import DecoderRuntime

        if args.tail_norms:
            DecoderRuntime.tail_norm = True

        if args.tp_pull:
            DecoderRuntime.peer_push = False
        if args.per_op:
            DecoderRuntime.persistent_decode = False
    conf = CONFIGS[args.config]
    family = conf["family"]
    cfg = conf["make"]().replace(num_layers=args.layers)
    dt = torch.bfloat16 if conf["dtype"] == "bf16" else torch.float32
    elem = 2 if conf["dtype"] == "bf16" else 4
    B, P = args.batch, args.prompt
    n_new = 1 + args.warmup + args.steps
    dev = torch.device("cuda", local)
    params = lazy_random_params(family, cfg, seed=0, dtype=dt, device=dev)
    cls = {"llama": LlamaModelWithHead, "neox": GPTNeoXModelWithHead, "gemma3": GemmaModelWithHead}[family]
    model = cls(cfg, dtype=dt)
    engine = Engine(model, InferenceConfig(tp_size=tp), params, dtype=dt)
    engine.init_params(params)
    del params
    torch.cuda.empty_cache()
    g = torch.Generator().manual_seed(0)
    prompt = torch.randint(0, cfg.vocab_size, (B, P), generator=g, dtype=torch.int32)

    # ---- device-resident decode steps (inputs already in HBM) ----
    rt = engine._runtime_for(B, engine.buffer_length(P, n_new))
    from jaxml_b200 import prng

    key, sub = prng.split(prng.prng_key(0))
    ids_d = prompt.to(dev)
    rt.reset(torch.ones(B, P, dtype=torch.bool, device=dev), key, sub, n_new)
    rt.prefill(ids_d, True, 1.0)                     # warm (first use allocates prefill buffers)
    rt.reset(torch.ones(B, P, dtype=torch.bool, device=dev), key, sub, n_new)
    torch.cuda.synchronize()
    pf0, pf1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    pf0.record()
    rt.prefill(ids_d, True, 1.0)
    pf1.record()
    torch.cuda.synchronize()
    prefill_ms = pf0.elapsed_time(pf1)
    rt.decode_step(True, 1.0)          # eager step: warms every kernel
    graph = rt.capture_decode(True, 1.0)
    for _ in range(args.warmup - 1):
        graph.replay()
    torch.cuda.synchronize()
    launches_per_step = rt.count_launches_per_decode_step()
    events = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        events[0].record()
        for i in range(args.steps):
            graph.replay()
            events[i + 1].record()
        torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    step_ms = [events[i].elapsed_time(events[i + 1]) for i in range(args.steps)]
    total_ms = events[0].elapsed_time(events[-1])
    if dist is not None:
        t = torch.tensor([total_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
    rt.check_status()
    ctx_first = P + args.warmup + 1          # valid keys (after the append) at the first timed step
    ctx_last = ctx_first + args.steps - 1
    ctx_mean = (ctx_first + ctx_last) / 2.0
    value = B * args.steps / (total_ms / 1e3)
    sbytes, wbytes, kvbytes = step_bytes(cfg, B, ctx_mean, tp, family, elem)
    step_ms_mean = total_ms / args.steps

    # ---- tensor parallelism: the ranks' greedy tokens, a TP=1 run of the same prompt, the exchange cost ----
    parity, exchange = None, None
    if dist is not None:
        toks = rt.tokens_out[:, :n_new].contiguous()
        gathered = [torch.empty_like(toks) for _ in range(world)]
        dist.all_gather(gathered, toks)
        ranks_identical = all(torch.equal(gathered[0], t) for t in gathered)
        # the prompt's logits at TP=N, gathered over the vocabulary shards (every rank takes part)
        rt.reset(torch.ones(B, P, dtype=torch.bool, device=dev), key, sub, n_new)
        rt.prefill(ids_d, True, 1.0)
        lgN = rt.comm.all_gather_vocab(rt.logits_buf()[:B]).float().cpu()
        rt.check_status()
        vs1 = None
        if rank == 0:
            k = min(n_new, 16)
            full_w = step_bytes(cfg, B, ctx_first, 1, family, elem)[1]
            if full_w <= 40e9:
                params1 = lazy_random_params(family, cfg, seed=0, dtype=dt, device=dev)
                eng1 = Engine(model, InferenceConfig(tp_size=1), params1, dtype=dt)
                eng1.init_params(params1)
                del params1
                rt1 = eng1._runtime_for(B, engine.buffer_length(P, n_new))
                rt1.reset(torch.ones(B, P, dtype=torch.bool, device=dev), key, sub, k)
                rt1.prefill(ids_d, True, 1.0)
                lg1 = rt1.logits_buf()[:B].float().cpu()
                t1 = rt1.generate(ids_d, torch.ones(B, P, dtype=torch.bool, device=dev), k, True, 1.0, 0)[:, :k].cpu()
                rt1.check_status()
                eq = t1 == gathered[0][:, :k].cpu()
                first = next((j for j in range(k) if not bool(eq[:, j].all())), None)
                vs1 = {"tokens": k, "token_match_frac": float(eq.float().mean().item()), "first_divergence_step": first,
                       "note": "greedy tokens of a TP=1 engine on rank 0's GPU, same weights and prompt; bf16 "
                               "float32-partial sums in another order can flip a near-tie, after which the "
                               "sequences differ"}
                if lgN.shape == lg1.shape:
                    dlt = (lgN - lg1).abs()
                    top2 = lg1.topk(2, dim=-1).values
                    gap = top2[:, 0] - top2[:, 1]
                    differ = lgN.argmax(-1) != lg1.argmax(-1)
                    vs1["prompt_logits"] = {
                        "max_abs_diff": float(dlt.max().item()), "mean_abs_diff": float(dlt.mean().item()),
                        "max_abs_logit": float(lg1.abs().max().item()),
                        "rows_argmax_differ": int(differ.sum().item()),
                        "rows_argmax_differ_with_top2_gap_above_max_diff":
                            int((differ & (gap > dlt.max(dim=-1).values * 2)).sum().item()),
                        "min_top2_gap": float(gap.min().item())}
                else:
                    vs1["prompt_logits"] = {"skipped": "gathered %s vs %s" % (tuple(lgN.shape), tuple(lg1.shape))}
                del rt1, eng1
                torch.cuda.empty_cache()
            else:
                vs1 = {"skipped": "the full weights (%.0f GB) are not built beside the shard" % (full_w / 1e9)}
        dist.barrier()
        parity = {"ranks_identical": ranks_identical, "tokens": n_new, "vs_tp1": vs1}
        if family != "neox":
            # two row-parallel exchanges per layer (o_proj, down), each against its no-exchange floor
            mode = "pull" if args.tp_pull else "push"
            costs = tp_exchange_costs(B, cfg.hidden_size, (("o_proj", cfg.num_heads * cfg.head_dim // tp),
                                                           ("down", cfg.intermediate_size // tp)), world, rank, dev)
            per_layer = sum(c[mode + "_us"] - c["local_us"] for c in costs.values())
            exchange = {"mode": mode, "exchange_us_per_step": per_layer * cfg.num_layers,
                        "share_of_step": per_layer * cfg.num_layers / (step_ms_mean * 1e3), "per_layer": costs,
                        "how": "tp_exchange_costs: each row-parallel projection + its norm, 32 launches per CUDA "
                               "graph, with and without the exchange (max over ranks)"}

    # ---- temperature 0.8 with a fixed seed (the workload's sampled variant), same steps ----
    temp_line = None
    if not args.no_temp:
        rt.reset(torch.ones(B, P, dtype=torch.bool, device=dev), key, sub, n_new)
        rt.prefill(ids_d, False, 0.8)
        rt.decode_step(False, 0.8)
        graph_t = rt.capture_decode(False, 0.8)
        for _ in range(args.warmup - 1):
            graph_t.replay()
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()
        t0e, t1e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0e.record()
        for _ in range(args.steps):
            graph_t.replay()
        t1e.record()
        torch.cuda.synchronize()
        tms = t0e.elapsed_time(t1e)
        if dist is not None:
            t = torch.tensor([tms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            tms = float(t.item())
        rt.check_status()
        temp_line = {"value": B * args.steps / (tms / 1e3), "unit": "tok/s", "ms_per_step": tms / args.steps,
                     "seed": 0, "temperature": 0.8}
        del graph_t

    # ---- per-kernel durations (graph replays, CUDA events) and the dominant kernel ----
    table = kernel_table(rt, cfg, ctx_last, step_ms_mean) if tp == 1 and args.config == "l8" else None
    ptable = None
    if tp == 1 and args.config == "l8":
        try:
            ptable = prefill_table(rt, cfg, prefill_ms)
        except Exception as exc:   # a measurement aid: report, do not lose the bench line
            ptable = {"error": str(exc)[:300]}

    # ---- end to end through Engine.generate with host buffers: the workload's 256 new tokens ----
    e2e = None
    if not args.no_e2e:
        n_e2e = args.e2e_tokens
        engine.generate(prompt, max_new_tokens=n_e2e, temperature=0.0)   # warm (graph capture)
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        t0 = time.perf_counter()
        out = engine.generate(prompt, max_new_tokens=n_e2e, temperature=0.0, include_prompt=False)
        el = time.perf_counter() - t0
        if dist is not None:
            t = torch.tensor([el], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            el = float(t.item())
        e2e = {"value": B * n_e2e / el, "unit": "tok/s", "h2d_bytes_per_step": round(prompt.numel() * 4 / n_e2e, 1),
               "d2h_bytes_per_step": int(out.numel() * 4 // n_e2e),
               "note": "Engine.generate(host prompt [%d, %d]) incl. H2D copy, prefill, %d decode steps, D2H of "
                       "the [%d, %d] tokens; %d new tokens per row" % (B, P, n_e2e - 1, B, n_e2e, n_e2e)}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        times, threads, L = cpu_decode_samples(conf, B=B, ctx=P, n_warm=1, n_timed=3, budget_s=30.0)
        sample_s = sum(times) / len(times)
        cpu = {"value": B / (L * sample_s), "unit": "tok/s", "cores": threads, "kind": "port",
               "sample": cpu_sample_note(B, P, L) + "; %d samples timed" % len(times)}

    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except OSError:
        pass
    hbm_peak = peaks.get("hbm_gbs", 6650.0)
    peak_src = "MEASURED_PEAKS.json hbm_gbs (burst copy)" if "hbm_gbs" in peaks else "fallback 6650 GB/s"
    roofline = None
    if table is not None:
        dom = max(table, key=lambda r: r["share"])
        roofline = {"bound": "hbm", "achieved": dom["gbs"], "peak": hbm_peak, "unit": "GB/s",
                    "frac": dom["gbs"] / hbm_peak, "traffic": dom["traffic"],
                    "traffic_note": dom["traffic_note"], "kernel": dom["kernel"], "share_of_step": dom["share"],
                    "algorithmic_bytes_per_launch": dom["bytes"], "us_per_launch": dom["us"],
                    "peak_source": peak_src}
        for r in table:
            r["frac"] = r["gbs"] / hbm_peak
    if rank == 0:
        line = {
            "metric": metric_of(conf), "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": step_ms_mean,
            "p50_step_ms": statistics.median(step_ms), "prefill_ms": prefill_ms,
            "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": conf["dtype"],
            "data": "synthetic (uniform-random prompt ids, N(0,0.02) random-init weights, seed 0)",
            "config": {"workload": "%s greedy decode, batch %d, prompt %d: %d timed decode steps "
                                   "at contexts %d..%d (e2e: %s new tokens)"
                                   % (conf["name"], B, P, args.steps, ctx_first, ctx_last,
                                      args.e2e_tokens if e2e else "no"),
                       "config": args.config, "layers": cfg.num_layers,
                       "global_batch": B, "seq_len": P, "parallelism": f"tp{tp}",
                       "tp_exchange": None if tp == 1 else ("pull all-reduce" if args.tp_pull else "push-fused"),
                       "decode_path": rt.decode_path_name(),
                       "decode_attention": ["by shape", "split", "cluster", "column pv", "cluster-split", "queue"][args.attn_impl],
                       "l2": "inputs larger than L2 (%.2f GB of weights per step)" % (wbytes / 1e9)},
            "roofline": roofline,
            "kernels": table,
            "prefill_kernels": ptable,
            "step_roofline": {"bytes_per_step": sbytes, "weight_bytes": wbytes, "kv_bytes": kvbytes,
                              "achieved_gbs": sbytes / (step_ms_mean * 1e-3) / 1e9,
                              "frac": sbytes / (step_ms_mean * 1e-3) / 1e9 / hbm_peak, "peak_source": peak_src},
            "temperature_0.8": temp_line,
            "parity": parity,
            "tp_exchange": exchange,
            "clocks": clocks.summary(),
            "gpu_launches": launches_per_step * args.steps,
            "e2e": e2e,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    # every graph that captured an NCCL all-reduce goes before the process group does
    del graph, rt
    engine.close()
    import gc

    gc.collect()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def _graph_ms(launch_all, n, reps=5):
    """Device milliseconds per launch of `n` back-to-back launches issued by `launch_all(stream)`, captured
    once in a CUDA graph and replayed `reps` times (CUDA events on the replay stream), so host-side
    launch cost is not measured."""
    import torch

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        launch_all(side.cuda_stream)          # warm: lazy module loading, one-time attribute setup
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=side):
        launch_all(side.cuda_stream)
    g.replay()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    cur = torch.cuda.current_stream()
    start.record(cur)
    for _ in range(reps):
        g.replay()
    end.record(cur)
    torch.cuda.synchronize()
    return start.elapsed_time(end) / (reps * n)


def micro_allreduce(args):
    """Latency of one decode-step all-reduce of the row-parallel partial sums (batch x 4096 float32) at
    TP = WORLD_SIZE (launch under torchrun): NCCL vs the NVLink peer kernel, each captured 64 times in a
    CUDA graph and replayed; max over ranks.  Prints one JSON line from rank 0."""
    import datetime

    import torch
    import torch.distributed as dist

    from jaxml_b200.engine import TPComm

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world < 2:
        print(json.dumps({"micro": "allreduce", "skipped": "needs WORLD_SIZE >= 2 (torchrun)"}))
        return
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    comm = TPComm()
    n = args.batch * 4096
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    comm.prepare_peer(dev)
    plain = torch.randn(n, device=dev)
    res = torch.empty(n, device=dev)
    for b in comm.peer.data:
        b[:n].copy_(torch.randn(n, device=dev))

    def peer_call():
        comm.all_reduce_partial(comm.partial_buffer(n), res, status)
    out = {}
    for name, fn in (("nccl", lambda: dist.all_reduce(plain)), ("peer", peer_call)):
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(3):
                fn()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for _ in range(64):
                fn()
        g.replay()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(5):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / (5 * 64) * 1e3], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        out[name] = float(t.item())
        del g
    st = int(status.item())
    comm.close()
    if rank == 0:
        print(json.dumps({"micro": "allreduce", "world": world, "floats": n, "bytes": 4 * n,
                          "nccl_us": out["nccl"], "peer_us": out["peer"], "status": st}), flush=True)
    dist.barrier()
    dist.destroy_process_group()


def tp_exchange_costs(M, d, shapes, world, rank, dev):
    """Row-parallel decode projections and their exchange at TP = world (process group already up): for
    each (name, K) in `shapes` the projection ([M, K] x [d, K]^T) followed by the norm that consumes the
    sum, three ways, each captured 32 times in a CUDA graph and replayed (max over ranks): `local` = no
    exchange (the projection's float32 partial fed to the norm as is: the compute-only floor), `pull` =
    projection, jx_allreduce_f32, norm, `push` = projection with JX_EPI_PUSH_F32 and the push-mode norm.
    Returns {name: {"K", "local_us", "pull_us", "push_us", "status"}}."""
    import torch
    import torch.distributed as dist

    from jaxml_b200 import _native as N
    from jaxml_b200.engine import TPComm

    lib = N.load()
    comm = TPComm()
    peer = comm.prepare_peer(dev)
    Mp = 16 if M <= 16 else 64
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    ws_n = N.LL()
    N.check(lib.jx_linear_decode_workspace(148, 64, ws_n), "ws")
    ws = torch.zeros(ws_n.value, dtype=torch.float32, device=dev)
    cnt = torch.zeros(d // 64 + 1, dtype=torch.int32, device=dev)
    nw = torch.ones(d, dtype=torch.bfloat16, device=dev)
    h = torch.zeros(M, d, dtype=torch.bfloat16, device=dev)
    xn = torch.zeros(M, d, dtype=torch.bfloat16, device=dev)
    part = torch.zeros(M, d, dtype=torch.float32, device=dev)
    tmp = torch.zeros(M, d, dtype=torch.float32, device=dev)
    res = {}
    for name, K in shapes:
        copies = 4   # distinct weight copies (4 x 2 x d x K bytes, above L2 for the down shape)
        ws_list = [(0.02 * torch.randn(d * K, device=dev)).to(torch.bfloat16) for _ in range(copies)]
        xp = torch.randn(Mp * K, device=dev).to(torch.bfloat16)

        def one(stream, mode, i):
            e = N.JxEpilogue()
            e.M, e.N, e.ldo = M, d, d
            if mode == "push":
                peer.push_epilogue(e, d)
            else:
                e.kind = N.JX_EPI_STORE_F32
                e.out = (part if mode == "local" else comm.partial_buffer(M * d)).data_ptr()
            src = comm.partial_buffer(M * d) if mode == "pull" else None
            N.check(lib.jx_linear_decode(ws_list[i % copies].data_ptr(), xp.data_ptr(), d, K, M, e, ws.data_ptr(),
                                         ws.numel(), cnt.data_ptr(), status.data_ptr(), 148, 1, stream), "linear")
            if mode == "pull":
                comm.all_reduce_partial(src, tmp.view(-1), status)
            a = N.JxNormArgs()
            a.M, a.d, a.eps, a.kind = M, d, 1e-5, N.JX_NORM_RMS
            a.h, a.ldh, a.w, a.out, a.ldo, a.status = h.data_ptr(), d, nw.data_ptr(), xn.data_ptr(), d, status.data_ptr()
            if mode == "push":
                peer.push_norm(a, d, d)
            else:
                a.a, a.a_f32, a.lda = (part if mode == "local" else tmp).data_ptr(), 1, d
            N.check(lib.jx_norm(a, N.JX_BF16, 1, stream), "norm")

        out = {"K": K}
        for mode in ("local", "pull", "push"):
            def launch_all(stream, mode=mode):
                for i in range(32):   # the current stream is `stream` here (warm-up and capture)
                    one(stream, mode, i)
            dist.barrier()
            ms = _graph_ms(launch_all, 32, reps=5)
            t = torch.tensor([ms * 1e3], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            out[mode + "_us"] = float(t.item())
        out["status"] = int(status.item())
        res[name] = out
        del ws_list
    torch.cuda.synchronize()
    comm.close()
    dist.barrier()
    return res


def micro_tp_exchange(args):
    """The Llama-3-8B row-parallel shapes of tp_exchange_costs (o_proj: K = 4096 / TP, down: K = 14336 / TP;
    N = 4096, batch rows) at TP = WORLD_SIZE (launch under torchrun).  Prints one JSON line per shape from
    rank 0."""
    import datetime

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world < 2:
        print(json.dumps({"micro": "tpx", "skipped": "needs WORLD_SIZE >= 2 (torchrun)"}))
        return
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    res = tp_exchange_costs(args.batch, 4096, (("o_proj", 4096 // world), ("down", 14336 // world)), world, rank, dev)
    if rank == 0:
        for name, r in res.items():
            print(json.dumps({"micro": "tpx", "world": world, "shape": name, "M": args.batch, "N": 4096, **r}),
                  flush=True)
    dist.destroy_process_group()


def micro(args):
    """Single-kernel microbenchmarks on Llama-3-8B layer shapes (bf16, N(0,1) activations, N(0,0.02)
    weights): `gemv` = the decode projection on the gate/up weights of 8 distinct layers (1.9 GB, larger
    than L2); `attn` = decode attention over a [B, ctx] cache.  Prints one JSON line."""
    import torch

    from jaxml_b200 import _native as N

    N.load()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    B = args.batch
    rup = lambda x, m: (x + m - 1) // m * m
    if args.micro == "filter":
        # min-p / top-k / top-p over [B, 128256] bf16 logits (Llama-3's vocabulary): the filter kernel,
        # and the same filters as torch device ops (sort / top-k) for comparison
        from jaxml_b200.sampling import _keep_min_p, _keep_top_k, _keep_top_p, filter_logits_

        V, (top_k, top_p, min_p) = 128256, (50, 0.9, 0.02)
        xs = [(torch.randn(B, V, device=dev) * 2.5).to(torch.bfloat16) for _ in range(8)]
        outs = [torch.empty_like(x) for x in xs]

        def run_kernel(stream):
            with torch.cuda.stream(torch.cuda.ExternalStream(stream)):
                for x, o in zip(xs, outs):
                    filter_logits_(x, o, top_k, top_p, min_p)
        ms = _graph_ms(run_kernel, len(xs))

        def torch_ops(x):
            return _keep_top_p(_keep_top_k(_keep_min_p(x, min_p), top_k), top_p)
        for x in xs:
            torch_ops(x)
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(3):
            for x in xs:
                torch_ops(x)
        end.record()
        torch.cuda.synchronize()
        # rows whose kept set differs from the torch ops' (their top-p cumulative sum runs in float32,
        # the kernel's is exact)
        differ = sum(int((torch.isfinite(o) != torch.isfinite(torch_ops(x))).any(dim=-1).sum().item())
                     for x, o in zip(xs, outs))
        print(json.dumps({"micro": "filter", "shape": f"B={B} V={V} bf16", "top_k": top_k, "top_p": top_p,
                          "min_p": min_p, "us": ms * 1e3, "torch_ops_us": start.elapsed_time(end) / (3 * len(xs)) * 1e3,
                          "rows_differing_from_torch_ops": differ, "rows": B * len(xs)}), flush=True)
        return
    if args.micro == "gemm":
        # prefill projection: [tokens, K] x [N, K]^T, bf16 K128 operands, plain store epilogue
        Nn, K = (int(v) for v in args.shape.split(","))
        M = args.tokens
        N.call("jx_set_prefill_linear_impl", args.gemm_impl)
        Mp, Np, Kp = rup(M, 128), rup(Nn, 128), rup(K, 128)
        copies = max(2, min(8, int(1.2e9 // (Nn * K * 2))))       # distinct weight copies
        ws = [torch.empty(Np * Kp, dtype=torch.bfloat16, device=dev).normal_(0, 0.02) for _ in range(copies)]
        x = torch.randn(Mp * Kp, device=dev).to(torch.bfloat16)
        out = torch.empty(M, Nn, dtype=torch.bfloat16, device=dev)
        st = torch.zeros(1, dtype=torch.int32, device=dev)
        e = N.JxEpilogue()
        e.kind, e.M, e.N, e.out, e.ldo = N.JX_EPI_STORE, M, Nn, out.data_ptr(), Nn

        def run(w, stream):
            N.call("jx_linear_prefill", x.data_ptr(), w.data_ptr(), Mp, Np, Kp, e, st.data_ptr(), 1, stream)
        flops = 2.0 * M * Nn * K
        peaks = {}
        try:
            peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
        except OSError:
            pass
        peak = peaks.get("bf16_tflops", 1590.0)
        groups = [int(g) for g in args.tile_groups.split(",")] if args.tile_groups else [None]
        for gi, gm in enumerate(groups):
            if gm is not None:
                N.call("jx_set_prefill_tile_group", gm)
            ms = _graph_ms(lambda stream: [run(w, stream) for w in ws], copies)
            line = {"micro": "gemm", "impl": ["by-shape", "mma.sync", "tcgen05"][args.gemm_impl],
                    "shape": f"M={M} N={Nn} K={K}", "tile_group": gm, "us": ms * 1e3, "tflops": flops / ms / 1e9,
                    "frac_of_measured_bf16": flops / ms / 1e9 / peak, "status": int(st.item())}
            if gi < len(groups) - 1:
                print(json.dumps(line), flush=True)
    elif args.micro == "gemv":
        Nn, K = (int(v) for v in args.shape.split(","))
        glu = Nn == 2 * 14336 and K == 4096
        copies = max(2, min(64, int(2e9 // (Nn * K * 2))))       # distinct weight copies: > L2 in total
        N.call("jx_set_decode_linear_impl", args.gemv_impl)
        Mp = 16 if B <= 16 else (32 if B <= 32 else 64)
        Np, Kp = rup(Nn, 128), rup(K, 128)
        ws = [torch.empty(Np * Kp, dtype=torch.bfloat16, device=dev).normal_(0, 0.02) for _ in range(copies)]
        x = torch.randn(Mp * Kp, device=dev).to(torch.bfloat16)
        out = torch.zeros(Mp * rup(Nn, 128), dtype=torch.bfloat16, device=dev)
        nws = N.LL()
        N.check(N.load().jx_linear_decode_workspace(148, B, nws), "ws")
        wsp = torch.zeros(nws.value, dtype=torch.float32, device=dev)
        cnt = torch.zeros(Np // 64 + 1, dtype=torch.int32, device=dev)
        e = N.JxEpilogue()
        if glu:
            e.kind, e.M, e.N, e.out, e.out_rp = N.JX_EPI_GLU_SILU, B, Nn // 2, out.data_ptr(), Mp
        else:
            e.kind, e.M, e.N, e.out, e.ldo = N.JX_EPI_STORE, B, Nn, out.data_ptr(), Nn

        def run(w, st, grid):
            N.call("jx_linear_decode", w.data_ptr(), x.data_ptr(), Np, Kp, B, e, wsp.data_ptr(), wsp.numel(),
                   cnt.data_ptr(), None, grid, 1, st)
        nbytes = 2 * Nn * K + 2 * B * K + 2 * B * (Nn // 2 if glu else Nn)
        grids = [int(g) for g in args.grids.split(",")]
        for grid in grids[:-1]:
            ms = _graph_ms(lambda st: [run(w, st, grid) for w in ws], copies)
            print(json.dumps({"micro": "gemv", "impl": ["by-shape", "mma.sync", "tcgen05", "row-split"][args.gemv_impl],
                              "shape": f"M={B} N={Nn} K={K}", "grid": grid, "us": ms * 1e3,
                              "gbs": nbytes / ms / 1e6}), flush=True)
        ms = _graph_ms(lambda st: [run(w, st, grids[-1]) for w in ws], copies)
        line = {"micro": "gemv", "impl": ["by-shape", "mma.sync", "tcgen05", "row-split"][args.gemv_impl], "shape": f"M={B} N={Nn} K={K}",
                "grid": grids[-1], "us": ms * 1e3, "gbs": nbytes / ms / 1e6}
    else:
        ctx, L = args.ctx, 8
        Hq, Hkv, hd = 32, 8, 128
        T = rup(ctx + 1, 256)
        kc = torch.randn(L, B, T, Hkv, hd, device=dev).to(torch.bfloat16)
        vc = torch.randn_like(kc)
        q = torch.randn(16 * ((B + 15) // 16), Hq * hd, device=dev).to(torch.bfloat16)
        pos = torch.full((B,), ctx - 2, dtype=torch.int32, device=dev)
        Mp = 16 * ((B + 15) // 16) if B <= 32 else 64
        out = torch.zeros(max(Mp, rup(B, 16)) * Hq * hd, dtype=torch.bfloat16, device=dev)
        nb = N.LL()
        N.check(N.load().jx_decode_attention_workspace(B, Hq, hd, T, 0, nb), "ws")
        wsp = torch.zeros(nb.value // 4 + 1, dtype=torch.float32, device=dev)
        cnt = torch.zeros(B * Hkv, dtype=torch.int32, device=dev)
        a = N.JxDAttnArgs()
        a.B, a.Hq, a.Hkv, a.hd, a.T, a.window, a.cache_rows = B, Hq, Hkv, hd, T, 0, L * B * T
        a.q, a.k_base, a.v_base, a.len_ptr, a.len_add, a.scale = (q.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                                                                  pos.data_ptr(), 2, hd ** -0.5)
        a.out, a.out_rp, a.ws, a.ws_bytes, a.counters = out.data_ptr(), max(Mp, rup(B, 16)), wsp.data_ptr(), wsp.numel() * 4, cnt.data_ptr()

        N.call("jx_set_decode_attention_impl", args.attn_impl)

        def run(layer, st):
            a.layer_row0 = layer * B * T
            N.call("jx_decode_attention", a, 1, st)
        ms = _graph_ms(lambda st: [run(l, st) for l in range(L)], L)
        nbytes = B * ctx * 2 * Hkv * hd * 2
        line = {"micro": "attn", "impl": ["by-shape", "split", "cluster", "column", "cluster-split", "queue"][args.attn_impl], "shape": f"B={B} ctx={ctx} Hq={Hq} Hkv={Hkv} hd={hd}", "us": ms * 1e3,
                "gbs": nbytes / ms / 1e6}
    print(json.dumps(line), flush=True)


def micro_sweep(args):
    """The single-layer decode microbenchmark sweep on one GPU (Llama-3-8B layer shapes, bf16), one JSON line
    per point, each timed as back-to-back launches replayed from a CUDA graph:
      attn  decode attention (the default form) for B in {1, 4, 16, 64, 256} x context in {1k, 4k, 16k,
            32k}: K/V bytes read per launch and GB/s (as many distinct layers of cache as fit in ~24 GB);
      proj  the decode projections of one tensor-parallel rank for TP in {1, 2, 4, 8} (qkv and gate/up
            split by output rows, o_proj and down by K) at M in {1, 16, 64} token rows (distinct weight
            copies, more than L2 in total);
      norm  the vectorised RMSNorm with the residual add over [M, 4096] rows, M in {1, 16, 64, 256}.
    The exchange of the row-parallel projections needs several GPUs: `--micro tpx` under torchrun."""
    import torch

    from jaxml_b200 import _native as N

    lib = N.load()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    rup = lambda x, m: (x + m - 1) // m * m
    Hq, Hkv, hd, d, F = 32, 8, 128, 4096, 14336
    hbm = 6550.0
    try:
        hbm = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))["hbm_gbs"]
    except (OSError, KeyError):
        pass

    def emit(kind, **kw):
        print(json.dumps({"sweep": kind, **kw}), flush=True)

    # ---- decode attention ----
    for B in (1, 4, 16, 64, 256):
        for ctx in (1024, 4096, 16384, 32768):
            T = rup(ctx + 1, 256)
            per_layer = 2 * B * T * Hkv * hd * 2
            L = max(1, min(8, int(24e9 // per_layer)))
            kc = torch.empty(L, B, T, Hkv, hd, dtype=torch.bfloat16, device=dev).normal_()
            vc = torch.empty_like(kc).normal_()
            q = torch.randn(rup(B, 16), Hq * hd, device=dev).to(torch.bfloat16)
            pos = torch.full((B,), ctx - 2, dtype=torch.int32, device=dev)
            orp = rup(B, 16)
            out = torch.zeros(orp * Hq * hd, dtype=torch.bfloat16, device=dev)
            nb = N.LL()
            N.check(lib.jx_decode_attention_workspace(B, Hq, hd, T, 0, nb), "ws")
            wsp = torch.zeros(nb.value // 4 + 1, dtype=torch.float32, device=dev)
            cnt = torch.zeros(B * Hkv, dtype=torch.int32, device=dev)
            st = torch.zeros(1, dtype=torch.int32, device=dev)
            a = N.JxDAttnArgs()
            a.B, a.Hq, a.Hkv, a.hd, a.T, a.window, a.cache_rows = B, Hq, Hkv, hd, T, 0, L * B * T
            a.q, a.k_base, a.v_base, a.len_ptr, a.len_add, a.scale = (q.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                                                                      pos.data_ptr(), 2, hd ** -0.5)
            a.out, a.out_rp, a.ws, a.ws_bytes = out.data_ptr(), orp, wsp.data_ptr(), wsp.numel() * 4
            a.counters, a.status = cnt.data_ptr(), st.data_ptr()

            def run(layer, stream):
                a.layer_row0 = layer * B * T
                N.check(lib.jx_decode_attention(a, 1, stream), "attention")
            ms = _graph_ms(lambda stream: [run(l, stream) for l in range(L)], L)
            nbytes = B * ctx * 2 * Hkv * hd * 2
            emit("attn", B=B, ctx=ctx, layers=L, us=ms * 1e3, bytes=nbytes, gbs=nbytes / ms / 1e6,
                 frac=nbytes / ms / 1e6 / hbm, status=int(st.item()))
            del kc, vc, wsp
            torch.cuda.empty_cache()

    # ---- decode projections of one TP rank ----
    for tp in (1, 2, 4, 8):
        shapes = (("qkv", (Hq + 2 * Hkv) * hd // tp, d, False), ("o_proj", d, Hq * hd // tp, False),
                  ("gate/up", 2 * F // tp, d, True), ("down", d, F // tp, False))
        for name, Nn, K, glu in shapes:
            Np, Kp = rup(Nn, 128), rup(K, 128)
            copies = max(2, min(64, int(2e9 // (Np * Kp * 2))))
            ws = [torch.empty(Np * Kp, dtype=torch.bfloat16, device=dev).normal_(0, 0.02) for _ in range(copies)]
            for M in (1, 16, 64):
                Mp = 16 if M <= 16 else (32 if M <= 32 else 64)
                x = torch.randn(Mp * Kp, device=dev).to(torch.bfloat16)
                out = torch.zeros(Mp * Np, dtype=torch.bfloat16, device=dev)
                nws = N.LL()
                N.check(lib.jx_linear_decode_workspace(148, M, nws), "ws")
                wsp = torch.zeros(nws.value, dtype=torch.float32, device=dev)
                cnt = torch.zeros(Np // 64 + 1, dtype=torch.int32, device=dev)
                st = torch.zeros(1, dtype=torch.int32, device=dev)
                e = N.JxEpilogue()
                if glu:
                    e.kind, e.M, e.N, e.out, e.out_rp = N.JX_EPI_GLU_SILU, M, Nn // 2, out.data_ptr(), Mp
                else:
                    e.kind, e.M, e.N, e.out, e.ldo = N.JX_EPI_STORE, M, Nn, out.data_ptr(), Nn

                def run(w, stream):
                    N.check(lib.jx_linear_decode(w.data_ptr(), x.data_ptr(), Np, Kp, M, e, wsp.data_ptr(), wsp.numel(),
                                                 cnt.data_ptr(), st.data_ptr(), 148, 1, stream), "linear")
                ms = _graph_ms(lambda stream: [run(w, stream) for w in ws], copies)
                nbytes = 2 * Nn * K + 2 * M * K + 2 * M * (Nn // 2 if glu else Nn)
                emit("proj", tp=tp, name=name, M=M, N=Nn, K=K, us=ms * 1e3, bytes=nbytes, gbs=nbytes / ms / 1e6,
                     frac=nbytes / ms / 1e6 / hbm, status=int(st.item()))
            del ws
            torch.cuda.empty_cache()

    # ---- norm (residual add + RMSNorm) ----
    for M in (1, 16, 64, 256):
        hs = [torch.randn(M, d, device=dev).to(torch.bfloat16) for _ in range(8)]
        res = torch.randn(M, d, device=dev).to(torch.bfloat16)
        w = torch.ones(d, dtype=torch.bfloat16, device=dev)
        xn = torch.zeros(M, d, dtype=torch.bfloat16, device=dev)
        st = torch.zeros(1, dtype=torch.int32, device=dev)

        def run(h, stream):
            a = N.JxNormArgs()
            a.M, a.d, a.eps, a.kind = M, d, 1e-5, N.JX_NORM_RMS
            a.h, a.ldh, a.w, a.out, a.ldo, a.status = h.data_ptr(), d, w.data_ptr(), xn.data_ptr(), d, st.data_ptr()
            a.a, a.a_f32, a.lda = res.data_ptr(), 0, d
            N.check(lib.jx_norm(a, N.JX_BF16, 1, stream), "norm")
        ms = _graph_ms(lambda stream: [run(h, stream) for h in hs], len(hs))
        nbytes = 2 * M * d * 4 + 2 * d   # residual in, added input in, sum out, normalised out; weights
        emit("norm", M=M, d=d, us=ms * 1e3, bytes=nbytes, gbs=nbytes / ms / 1e6, status=int(st.item()))


def main():
    args = parse()
    conf = CONFIGS[args.config]
    if args.batch is None:
        args.batch = conf["B"]
    if args.prompt is None:
        args.prompt = conf["P"]
    if args.layers is None:
        args.layers = conf["make"]().num_layers
    if args.e2e_tokens is None:
        args.e2e_tokens = conf["new"]
    if args.micro == "allreduce":
        micro_allreduce(args)
        return
    if args.micro == "tpx":
        micro_tp_exchange(args)
        return
    if args.micro == "sweep":
        micro_sweep(args)
        return
    if args.micro:
        micro(args)
        return
    if args.impl == "reference":
        reference_arm(args)
        return
    gpu_arm(args)


if __name__ == "__main__":
    main()
