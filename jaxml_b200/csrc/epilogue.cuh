// Fused GEMM epilogues shared by the decode GEMV, the prefill GEMM and the float32 GEMM.
//
// A finished output tile arrives as float32 accumulators indexed by (row m, packed weight row n).
// Each epilogue reproduces the reference's rounding points: the projection result is rounded to the
// model dtype before the bias / residual / activation ops, each of which rounds again
// (nn/linear.py:161-182 for the bias, models/llama.py:133-137 for the residual adds,
// models/llama.py:82-88 / gemma3.py:80-86 / gpt_neox.py:75-80 for the activations).
#pragma once
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
