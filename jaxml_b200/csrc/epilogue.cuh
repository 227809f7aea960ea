// Fused GEMM epilogues shared by the decode GEMV, the prefill GEMM and the float32 GEMM.
//
// A finished output tile arrives as float32 accumulators indexed by (row m, packed weight row n).
// Each epilogue reproduces the reference's rounding points: the projection result is rounded to the
// model dtype before the bias / residual / activation ops, each of which rounds again
// (nn/linear.py:161-182 for the bias, models/llama.py:133-137 for the residual adds,
// models/llama.py:82-88 / gemma3.py:80-86 / gpt_neox.py:75-80 for the activations).
#pragma once
#include <type_traits>

#include "common.cuh"

namespace jxb {

typedef jx_epilogue EpiParams;

// L2 prefetch of the next decode projection's first weight chunks for CTA c (jx_epilogue.pf_w): the
// same stream-K split as the next call (pf_grid CTAs over pf_np / pf_rows blocks x pf_kp / 128 chunks).
__device__ __forceinline__ void prefetch_next_weights(const EpiParams& e, int c) {
  if (!e.pf_w || e.pf_iters <= 0 || c >= e.pf_grid) return;
  const long long R = e.pf_rows, kc = e.pf_kp >> 7;
  const long long total = (e.pf_np / R) * kc;
  const long long it0 = total * c / e.pf_grid, it1 = total * (c + 1) / e.pf_grid;
  const long long n = it1 - it0 < e.pf_iters ? it1 - it0 : e.pf_iters;
  const uint64_t pol = l2_policy_evict_last();
  const bf16* w = reinterpret_cast<const bf16*>(e.pf_w);
  for (long long i = 0; i < n; ++i) {
    const long long it = it0 + i, nb = it / kc, kk = it - nb * kc;
    bulk_prefetch_l2(w + ((kk * (e.pf_np >> 3) + nb * (R >> 3)) << 10), (uint32_t)(R * 256), pol);
  }
}

// After a JX_EPI_PUSH_F32 epilogue of output columns [n0, n0 + cols) (called by one thread once every
// thread of the block has stored): flag its 64-column units at every rank with this call's epoch
// (the receiving rank's push counter + 1, which is ours too: all ranks make the same calls).
__device__ __forceinline__ unsigned push_epoch(const EpiParams& e) {
  const unsigned char* const* bases = reinterpret_cast<const unsigned char* const*>(e.peer_bases);
  return *reinterpret_cast<const volatile unsigned*>(bases[e.peer_rank] + e.peer_seq_off);
}

__device__ __forceinline__ void push_signal(const EpiParams& e, long long n0, int cols) {
  const unsigned char* const* bases = reinterpret_cast<const unsigned char* const*>(e.peer_bases);
  const unsigned ep = push_epoch(e), v = ep + 1;
  // Release pattern: the CTA barrier before this call orders every thread's slot stores before this
  // thread's fence (cumulativity), and the fence orders them before the flag stores below.
  fence_acq_rel_sys();
  const long long set_off = e.peer_flag_off + (long long)(ep & 1) * kPushMaxUnits * 8 * 4;
  const int u0 = (int)(n0 >> 6), nu = cols >> 6;
  for (int r = 0; r < e.peer_world; ++r)
    for (int u = 0; u < nu; ++u) {
      unsigned* f = reinterpret_cast<unsigned*>(const_cast<unsigned char*>(bases[r]) + set_off) + (u0 + u) * 8 +
                    e.peer_rank;
      st_relaxed_sys(f, v);
    }
}

// ---- normalisation prologue (jx_epilogue.pn_*) ----
__device__ __forceinline__ void pn_load8(const bf16* p, float* v) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

// Sum over the nt threads of a named barrier group (tid in [0, nt), nt a multiple of 32, red >= nt / 32).
__device__ __forceinline__ float pn_group_sum(float v, float* red, int tid, int nt, int bar) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((tid & 31) == 0) red[tid >> 5] = v;
  named_bar_sync(bar, nt);
  float t = 0.f;
  for (int w = 0; w < nt / 32; ++w) t += red[w];
  named_bar_sync(bar, nt);
  return t;
}

// Row m of h normalised (jx_norm's arithmetic: float32 statistics, the reference's bf16 roundings) into
// row m of the K128 activation operand X with Mp row padding, by the nt threads of barrier group `bar`.
__device__ __forceinline__ void prologue_norm_row(const EpiParams& e, bf16* X, long long Mp, int m, int tid, int nt,
                                                  int bar, float* red) {
  const bf16* h = reinterpret_cast<const bf16*>(e.pn_h) + (long long)m * e.pn_ldh;
  const bf16* w = reinterpret_cast<const bf16*>(e.pn_w);
  const bf16* b = reinterpret_cast<const bf16*>(e.pn_b);
  const int d = e.pn_d;
  float s = 0.f, s2 = 0.f;
  for (int j = tid * 8; j < d; j += nt * 8) {
    float x[8];
    pn_load8(h + j, x);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      s += x[i];
      s2 += x[i] * x[i];
    }
  }
  float mean = 0.f, den;
  if (e.pn_kind == JX_NORM_LAYER) {
    mean = pn_group_sum(s, red, tid, nt, bar) / (float)d;
    float v = 0.f;
    for (int j = tid * 8; j < d; j += nt * 8) {
      float x[8];
      pn_load8(h + j, x);
#pragma unroll
      for (int i = 0; i < 8; ++i) v += (x[i] - mean) * (x[i] - mean);
    }
    den = sqrtf(pn_group_sum(v, red, tid, nt, bar) / (float)d + e.pn_eps);
  } else {
    den = sqrtf(pn_group_sum(s2, red, tid, nt, bar) / (float)d + e.pn_eps);
  }
  const float inv = 1.0f / den;
  for (int j = tid * 8; j < d; j += nt * 8) {
    float x[8], wv[8], bv[8], y[8];
    pn_load8(h + j, x);
    pn_load8(w + j, wv);
    if (b) pn_load8(b + j, bv);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (e.pn_kind == JX_NORM_LAYER)
        y[i] = rnd<bf16>((x[i] - mean) / den * wv[i] + (b ? bv[i] : 0.f));
      else if (e.pn_kind == JX_NORM_RMS)
        y[i] = rnd<bf16>(wv[i] * rnd<bf16>(x[i] / den));
      else
        y[i] = rnd<bf16>((wv[i] + 1.0f) * (x[i] * inv));
    }
    uint4 u;
    u.x = pack_bf16x2(y[0], y[1]);
    u.y = pack_bf16x2(y[2], y[3]);
    u.z = pack_bf16x2(y[4], y[5]);
    u.w = pack_bf16x2(y[6], y[7]);
    *reinterpret_cast<uint4*>(X + k128_offset(m, j, Mp)) = u;
  }
}

// The prologue's part of a CTA: CTA c < M normalises row c and flags it with epoch ep + 1 (after every
// thread of the group has stored).  Called by the nt threads of barrier group `bar` after their wait on
// the previous kernel.
__device__ __forceinline__ void prologue_rows(const EpiParams& e, bf16* X, long long Mp, int c, int ep, int tid, int nt,
                                              int bar, float* red) {
  if (c >= e.M) return;
  prologue_norm_row(e, X, Mp, c, tid, nt, bar, red);
  named_bar_sync(bar, nt);
  if (tid == 0) {
    __threadfence();
    st_release_gpu(e.pn_sync + 2 + c, ep + 1);
  }
}

// Wait (bounded) until the M rows of this call's X are written; then async-proxy loads may read them.
// The row flags are read together (independent relaxed loads, one round trip per poll), then one
// acquire fence orders the rows' contents before the loads that follow.
__device__ __forceinline__ bool prologue_wait(const EpiParams& e, int ep) {
  const volatile int* f = e.pn_sync + 2;
  uint64_t t0 = 0;
  for (bool first = true;; first = false) {
    int v[16];
#pragma unroll
    for (int m = 0; m < 16; ++m) v[m] = m < e.M ? f[m] : ep + 1;
    bool all = true;
#pragma unroll
    for (int m = 0; m < 16; ++m) all &= v[m] == ep + 1;
    if (all) break;
    if (first) {
      t0 = globaltimer_ns();
    } else if (globaltimer_ns() - t0 > kWaitLimitNs) {
      return false;
    }
  }
  asm volatile("fence.acq_rel.gpu;" ::: "memory");
  fence_proxy_async_global();
  return true;
}

// End of a CTA of a prologue call (one thread, after every thread of the CTA has read the epoch): the
// last CTA to arrive advances the epoch for the next call.
__device__ __forceinline__ void prologue_arrive(const EpiParams& e, int ep) {
  __threadfence();
  if (atomicAdd(e.pn_sync + 1, 1) == (int)(gridDim.x * gridDim.y * gridDim.z) - 1) {
    e.pn_sync[1] = 0;
    e.pn_sync[0] = ep + 1;
    __threadfence();
  }
}

template <typename T>
__device__ __forceinline__ float bias_at(const EpiParams& e, long long n) {
  return e.bias ? to_f(reinterpret_cast<const T*>(e.bias)[n]) : 0.0f;
}

// tile(m, j) for m in [0, rows), j in [0, cols); n0 = packed weight row of column 0 (a multiple of 64).
template <typename T, typename TileFn>
__device__ __forceinline__ void run_epilogue(const EpiParams& e, long long m0, int rows, long long n0, int cols,
                                             TileFn tile, int tid, int nthreads) {
  if (e.kind == JX_EPI_GLU_SILU || e.kind == JX_EPI_GLU_GELU_TANH) {
    // Packed weight rows come in groups of 64: 32 gate rows, then the 32 up rows of the same columns.
    const int half = cols >> 1;
    for (int idx = tid; idx < rows * half; idx += nthreads) {
      const int m = idx / half, jj = idx - m * half;
      const int grp = jj >> 5, j = jj & 31;
      const long long row = m0 + m;
      const long long ng = n0 + grp * 64 + j;
      const long long col = ((n0 >> 6) + grp) * 32 + j;
      if (row >= e.M || col >= e.N) continue;
      const float g = rnd<T>(rnd<T>(tile(m, grp * 64 + j)) + bias_at<T>(e, ng));
      const float u = rnd<T>(rnd<T>(tile(m, grp * 64 + 32 + j)) + bias_at<T>(e, ng + 32));
      const float a = rnd<T>(e.kind == JX_EPI_GLU_SILU ? silu_f(g) : gelu_tanh_f(g));
      const long long o = e.out_rp > 0 ? k128_offset(row, col, e.out_rp) : row * e.ldo + col;
      reinterpret_cast<T*>(e.out)[o] = from_f<T>(a * u);
    }
    return;
  }
  if (e.kind == JX_EPI_PUSH_F32) {
    // row-parallel partial sums stored over NVLink into this rank's receive slot of every rank's region
    // (the flags follow in push_signal, once every thread of the CTA has stored its part)
    const unsigned char* const* bases = reinterpret_cast<const unsigned char* const*>(e.peer_bases);
    const long long slot =
        e.peer_recv_off + ((long long)(push_epoch(e) & 1) * e.peer_world + e.peer_rank) * e.peer_slot_bytes;
    const int q4 = cols >> 2;
    for (int idx = tid; idx < rows * q4; idx += nthreads) {
      const int m = idx / q4, j = (idx - m * q4) * 4;
      const long long row = m0 + m, n = n0 + j;
      if (row >= e.M || n >= e.N) continue;
      float4 v;
      v.x = tile(m, j) + bias_at<T>(e, n);
      v.y = tile(m, j + 1) + bias_at<T>(e, n + 1);
      v.z = tile(m, j + 2) + bias_at<T>(e, n + 2);
      v.w = tile(m, j + 3) + bias_at<T>(e, n + 3);
      const long long off = slot + (row * e.ldo + n) * 4;
      for (int r = 0; r < e.peer_world; ++r)
        *reinterpret_cast<float4*>(const_cast<unsigned char*>(bases[r]) + off) = v;
    }
    return;
  }
  if (e.kind == JX_EPI_STORE_F32 || e.kind == JX_EPI_ACC_F32) {
    // float32 partial sums of a row-parallel projection: no rounding until they are all-reduced
    float* out = reinterpret_cast<float*>(e.out);
    for (int idx = tid; idx < rows * cols; idx += nthreads) {
      const int m = idx / cols, j = idx - m * cols;
      const long long row = m0 + m, n = n0 + j;
      if (row >= e.M || n >= e.N) continue;
      const float v = tile(m, j) + bias_at<T>(e, n);
      if (e.kind == JX_EPI_STORE_F32)
        out[row * e.ldo + n] = v;
      else
        out[row * e.ldo + n] += v;
    }
    return;
  }
  if constexpr (std::is_same<T, bf16>::value) {
    // bfloat16 STORE / RESID / RESID2 in chunks of 8 columns: every residual load of a thread's (up to 4)
    // chunks is issued before any store.  The output may alias the residual, so a per-element loop would
    // wait for one L2 round trip per element.
    const bool al = !((reinterpret_cast<uintptr_t>(e.out) | reinterpret_cast<uintptr_t>(e.res) |
                       reinterpret_cast<uintptr_t>(e.res2)) & 15);
    const bool kind_ok = e.kind == JX_EPI_STORE || e.kind == JX_EPI_RESID || e.kind == JX_EPI_RESID2;
    if (kind_ok && al && cols % 8 == 0 && n0 % 8 == 0 && e.ldo % 8 == 0 && e.ldr % 8 == 0 && e.ldr2 % 8 == 0) {
      const T* res = reinterpret_cast<const T*>(e.res);
      const T* res2 = reinterpret_cast<const T*>(e.res2);
      T* out = reinterpret_cast<T*>(e.out);
      const int cpr = cols >> 3, nchunks = rows * cpr;
      for (int base = tid; base < nchunks; base += 4 * nthreads) {
        uint4 r[4], r2[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int idx = base + u * nthreads;
          r[u] = r2[u] = make_uint4(0, 0, 0, 0);
          if (idx >= nchunks) continue;
          const int m = idx / cpr, j = (idx - m * cpr) * 8;
          const long long row = m0 + m, n = n0 + j;
          if (row >= e.M || n + 8 > e.N) continue;
          if (e.kind != JX_EPI_STORE) r[u] = *reinterpret_cast<const uint4*>(res + row * e.ldr + n);
          if (e.kind == JX_EPI_RESID2) r2[u] = *reinterpret_cast<const uint4*>(res2 + row * e.ldr2 + n);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int idx = base + u * nthreads;
          if (idx >= nchunks) continue;
          const int m = idx / cpr, j = (idx - m * cpr) * 8;
          const long long row = m0 + m, n = n0 + j;
          if (row >= e.M || n >= e.N) continue;
          if (n + 8 > e.N) {   // ragged edge of the output: element by element
            for (int i = 0; i < 8 && n + i < e.N; ++i) {
              float v = rnd<T>(tile(m, j + i));
              if (e.bias) v = rnd<T>(v + bias_at<T>(e, n + i));
              if (e.kind == JX_EPI_RESID) v = v + to_f(res[row * e.ldr + n + i]);
              if (e.kind == JX_EPI_RESID2) v = rnd<T>(v + to_f(res2[row * e.ldr2 + n + i])) + to_f(res[row * e.ldr + n + i]);
              out[row * e.ldo + n + i] = from_f<T>(v);
            }
            continue;
          }
          const __nv_bfloat162* rh = reinterpret_cast<const __nv_bfloat162*>(&r[u]);
          const __nv_bfloat162* rh2 = reinterpret_cast<const __nv_bfloat162*>(&r2[u]);
          float y[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            float v = rnd<T>(tile(m, j + i));
            if (e.bias) v = rnd<T>(v + bias_at<T>(e, n + i));
            const float2 rr = __bfloat1622float2(rh[i >> 1]);
            const float rv = (i & 1) ? rr.y : rr.x;
            if (e.kind == JX_EPI_RESID) {
              v = v + rv;
            } else if (e.kind == JX_EPI_RESID2) {
              const float2 qq = __bfloat1622float2(rh2[i >> 1]);
              v = rnd<T>(v + ((i & 1) ? qq.y : qq.x)) + rv;
            }
            y[i] = v;
          }
          uint4 o;
          o.x = pack_bf16x2(y[0], y[1]);
          o.y = pack_bf16x2(y[2], y[3]);
          o.z = pack_bf16x2(y[4], y[5]);
          o.w = pack_bf16x2(y[6], y[7]);
          *reinterpret_cast<uint4*>(out + row * e.ldo + n) = o;
        }
      }
      return;
    }
  }
  for (int idx = tid; idx < rows * cols; idx += nthreads) {
    const int m = idx / cols, j = idx - m * cols;
    const long long row = m0 + m, n = n0 + j;
    if (row >= e.M || n >= e.N) continue;
    float v = rnd<T>(tile(m, j));
    if (e.bias) v = rnd<T>(v + bias_at<T>(e, n));
    switch (e.kind) {
      case JX_EPI_STORE:
        reinterpret_cast<T*>(e.out)[row * e.ldo + n] = from_f<T>(v);
        break;
      case JX_EPI_RESID: {
        const float r = to_f(reinterpret_cast<const T*>(e.res)[row * e.ldr + n]);
        reinterpret_cast<T*>(e.out)[row * e.ldo + n] = from_f<T>(v + r);
        break;
      }
      case JX_EPI_RESID2: {
        const float r2 = to_f(reinterpret_cast<const T*>(e.res2)[row * e.ldr2 + n]);
        const float r = to_f(reinterpret_cast<const T*>(e.res)[row * e.ldr + n]);
        reinterpret_cast<T*>(e.out)[row * e.ldo + n] = from_f<T>(rnd<T>(v + r2) + r);
        break;
      }
      case JX_EPI_ACT_GELU_ERF:
        if (e.out_rp > 0)
          reinterpret_cast<T*>(e.out)[k128_offset(row, n, e.out_rp)] = from_f<T>(gelu_erf_f(v));
        else
          reinterpret_cast<T*>(e.out)[row * e.ldo + n] = from_f<T>(gelu_erf_f(v));
        break;
      default:
        break;
    }
  }
}

}  // namespace jxb
