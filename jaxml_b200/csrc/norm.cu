// Fused embedding / residual-add / normalisation kernels (one CTA per token row; prefill-sized calls
// that only normalise take one warp per row, norm_rows_kernel).
//
// Per row m it can, in order:
//   1. gather the embedding row of ids[m] (ids < 0 read row 0, models/llama.py:188) and scale it by the
//      bfloat16-rounded sqrt(d) for Gemma3 (gemma3.py:245);
//   2. add a second input into the residual stream h, optionally normalising that input first
//      (Gemma3's post-attention / post-feedforward norms, gemma3.py:166-173) and store h back;
//   3. normalise h with RMSNorm (norms.py:110-117), Gemma RMSNorm (gemma3.py:94-106) or LayerNorm
//      (norms.py:157-168) into one or two outputs (two for GPT-NeoX's parallel residual, which feeds
//      ln1(h) to attention and ln2(h) to the MLP).  bfloat16 outputs can be written in the K128 tiled
//      layout that the projection kernels read.
#include "common.cuh"

namespace jxb {

typedef jx_norm_args NormArgs;

template <int NT>
__device__ __forceinline__ float block_sum(float v, float* red) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
  if (threadIdx.x < 32) {
    t = threadIdx.x < NT / 32 ? red[threadIdx.x] : 0.f;
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) red[NT / 32] = t;
  }
  __syncthreads();
  return red[NT / 32];
}

// Normalise x (float32 copy of a row of model-dtype values, in shared memory) in place into y (float
// values already rounded to T).
template <typename T, int NT>
__device__ void normalize_row(const float* x, float* y, int d, int kind, float eps, const T* w, const T* b,
                              float* red) {
  if (kind == JX_NORM_LAYER) {
    float s = 0.f;
    for (int j = threadIdx.x; j < d; j += NT) s += x[j];
    const float mean = block_sum<NT>(s, red) / (float)d;
    float v = 0.f;
    for (int j = threadIdx.x; j < d; j += NT) {
      const float t = x[j] - mean;
      v += t * t;
    }
    const float var = block_sum<NT>(v, red) / (float)d;
    const float den = sqrtf(var + eps);
    for (int j = threadIdx.x; j < d; j += NT) {
      float o = (x[j] - mean) / den * to_f(w[j]);
      if (b) o += to_f(b[j]);
      y[j] = rnd<T>(o);
    }
    return;
  }
  float s = 0.f;
  for (int j = threadIdx.x; j < d; j += NT) s += x[j] * x[j];
  const float ms = block_sum<NT>(s, red) / (float)d;
  const float den = sqrtf(ms + eps);
  if (kind == JX_NORM_RMS) {
    for (int j = threadIdx.x; j < d; j += NT) y[j] = rnd<T>(to_f(w[j]) * rnd<T>(x[j] / den));
  } else {  // JX_NORM_GEMMA
    const float inv = 1.0f / den;
    for (int j = threadIdx.x; j < d; j += NT) y[j] = rnd<T>((to_f(w[j]) + 1.0f) * (x[j] * inv));
  }
}

template <typename T>
__device__ __forceinline__ void store_row(const float* y, int d, long long m, void* out, long long ldo,
                                          long long out_rp, int NT) {
  T* o = reinterpret_cast<T*>(out);
  for (int j = threadIdx.x; j < d; j += NT) {
    const long long off = out_rp > 0 ? k128_offset(m, j, out_rp) : m * ldo + j;
    o[off] = from_f<T>(y[j]);
  }
}

template <typename T, int NT>
__global__ void __launch_bounds__(NT) norm_kernel(NormArgs p) {
  extern __shared__ float sm[];
  float* x = sm;            // [d]
  float* y = sm + p.d;      // [d]
  float* red = sm + 2 * p.d;  // [NT/32 + 1]
  const long long m = blockIdx.x;
  const int d = p.d;
  pdl_trigger();
  pdl_wait();
  T* h = reinterpret_cast<T*>(p.h);

  if (p.ids) {
    int id = p.ids[m];
    if (id < 0) id = 0;
    if (id >= p.vocab) {
      set_status(p.status, JX_ERR_RANGE);
      id = 0;
    }
    const T* row = reinterpret_cast<const T*>(p.table) + (long long)id * d;
    const float sc = p.embed_scale;
    for (int j = threadIdx.x; j < d; j += NT) {
      float v = to_f(row[j]);
      if (sc != 0.f) v = rnd<T>(v * sc);
      x[j] = v;
      h[m * p.ldh + j] = from_f<T>(v);
    }
    __syncthreads();
  } else {
    const long long src = p.row_map ? (long long)p.row_map[m] : m;
    for (int j = threadIdx.x; j < d; j += NT) x[j] = to_f(h[src * p.ldh + j]);
    __syncthreads();
  }

  if (p.a) {
    const T* a = reinterpret_cast<const T*>(p.a);
    const float* af = reinterpret_cast<const float*>(p.a);
    // a float32 input (an all-reduced partial sum) is rounded to the model dtype first
    auto a_at = [&](int j) { return p.a_f32 ? rnd<T>(af[m * p.lda + j]) : to_f(a[m * p.lda + j]); };
    if (p.kind_pre != JX_NORM_NONE) {
      for (int j = threadIdx.x; j < d; j += NT) y[j] = a_at(j);
      __syncthreads();
      // normalise y in place: copy to a temp in the output half first
      float* t = y;
      normalize_row<T, NT>(t, t, d, p.kind_pre, p.eps, reinterpret_cast<const T*>(p.w_pre),
                           reinterpret_cast<const T*>(p.b_pre), red);
      __syncthreads();
      for (int j = threadIdx.x; j < d; j += NT) x[j] = rnd<T>(x[j] + t[j]);
    } else {
      for (int j = threadIdx.x; j < d; j += NT) x[j] = rnd<T>(x[j] + a_at(j));
    }
    __syncthreads();
    for (int j = threadIdx.x; j < d; j += NT) h[m * p.ldh + j] = from_f<T>(x[j]);
    __syncthreads();
  }

  if (p.out) {
    normalize_row<T, NT>(x, y, d, p.kind, p.eps, reinterpret_cast<const T*>(p.w), reinterpret_cast<const T*>(p.b),
                         red);
    __syncthreads();
    store_row<T>(y, d, m, p.out, p.ldo, p.out_rp, NT);
    __syncthreads();
  }
  if (p.out2) {
    normalize_row<T, NT>(x, y, d, p.kind, p.eps, reinterpret_cast<const T*>(p.w2),
                         reinterpret_cast<const T*>(p.b2), red);
    __syncthreads();
    store_row<T>(y, d, m, p.out2, p.ldo2, p.out2_rp, NT);
  }
}

// ------------------------------------------------------------------------------------------------
// bfloat16 rows with d % 8 == 0 and d <= 8192: one thread per 8 consecutive elements (a 16-byte vector),
// the whole row in registers, one pass, 16-byte loads and stores (a K128 output keeps 8 consecutive K
// elements of a row contiguous).  Same semantics as norm_kernel.
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ float vblock_sum(float v, float* red) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = (blockDim.x + 31) >> 5;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : 0.f;
  for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  return t;
}

__device__ __forceinline__ void vload8(const bf16* p, float* v) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

__device__ __forceinline__ void vstore8(bf16* p, const float* v) {
  uint4 u;
  u.x = pack_bf16x2(v[0], v[1]);
  u.y = pack_bf16x2(v[2], v[3]);
  u.z = pack_bf16x2(v[4], v[5]);
  u.w = pack_bf16x2(v[6], v[7]);
  *reinterpret_cast<uint4*>(p) = u;
}

// Normalise the 8 values of this thread (the row is spread over the block); wv / bv: this thread's 8
// weights and biases (bv unused without a bias).
__device__ __forceinline__ void vnormalize_wb(const float* x, float* y, int d, int kind, float eps, const float* wv,
                                              const float* bv, bool has_b, int j0, float* red) {
  const bool b = has_b;
  if (kind == JX_NORM_LAYER) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) s += x[i];
    const float mean = vblock_sum(s, red) / (float)d;
    float v = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) v += (x[i] - mean) * (x[i] - mean);
    const float den = sqrtf(vblock_sum(v, red) / (float)d + eps);
#pragma unroll
    for (int i = 0; i < 8; ++i) y[i] = rnd<bf16>((x[i] - mean) / den * wv[i] + (b ? bv[i] : 0.f));
    return;
  }
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) s += x[i] * x[i];
  const float den = sqrtf(vblock_sum(s, red) / (float)d + eps);
  if (kind == JX_NORM_RMS) {
#pragma unroll
    for (int i = 0; i < 8; ++i) y[i] = rnd<bf16>(wv[i] * rnd<bf16>(x[i] / den));
  } else {
    const float inv = 1.0f / den;
#pragma unroll
    for (int i = 0; i < 8; ++i) y[i] = rnd<bf16>((wv[i] + 1.0f) * (x[i] * inv));
  }
}

__device__ __forceinline__ void vnormalize(const float* x, float* y, int d, int kind, float eps, const bf16* w,
                                           const bf16* b, int j0, float* red) {
  float wv[8], bv[8];
  vload8(w + j0, wv);
  if (b) vload8(b + j0, bv);
  vnormalize_wb(x, y, d, kind, eps, wv, bv, b != nullptr, j0, red);
}

// Push mode: wait, bounded, until every 64-column unit carries epoch v from every rank (thread t polls
// unit t / world, source t % world).  False on timeout.
__device__ __forceinline__ bool peer_wait(const NormArgs& p, unsigned v) {
  bool ok = true;
  const int t = threadIdx.x;
  if (t < p.peer_units * p.peer_world) {
    const unsigned* f = p.peer_flags + ((v - 1) & 1) * kPushMaxUnits * 8 + (t / p.peer_world) * 8 + (t % p.peer_world);
    if (ld_acquire_sys(f) != v) {
      const uint64_t t0 = globaltimer_ns();
      while (ld_acquire_sys(f) != v) {
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          ok = false;
          break;
        }
      }
    }
  }
  return __syncthreads_and(ok) != 0;
}

// Rank-order float32 sum of the 8 partials at (m, j0) in this rank's receive slots of set `set`.
__device__ __forceinline__ void peer_sum8(const NormArgs& p, unsigned set, long long m, int j0, float4& s0,
                                          float4& s1) {
  const float* base =
      reinterpret_cast<const float*>(p.peer_recv) + (long long)set * p.peer_world * p.peer_stride + m * p.lda + j0;
  s0 = __ldcv(reinterpret_cast<const float4*>(base));
  s1 = __ldcv(reinterpret_cast<const float4*>(base) + 1);
  for (int r = 1; r < p.peer_world; ++r) {
    const float4* q = reinterpret_cast<const float4*>(base + r * p.peer_stride);
    const float4 u0 = __ldcv(q), u1 = __ldcv(q + 1);
    s0.x += u0.x, s0.y += u0.y, s0.z += u0.z, s0.w += u0.w;
    s1.x += u1.x, s1.y += u1.y, s1.z += u1.z, s1.w += u1.w;
  }
}

__global__ void __launch_bounds__(1024) norm_vec_kernel(NormArgs p) {
  __shared__ float red[32];
  __shared__ unsigned s_epoch;
  const long long m = blockIdx.x;
  const int j0 = threadIdx.x * 8;
  // the norm weights do not depend on the previous kernel: load them before waiting on it
  float wv[8], bv[8];
  if (p.out) {
    vload8(reinterpret_cast<const bf16*>(p.w) + j0, wv);
    if (p.b) vload8(reinterpret_cast<const bf16*>(p.b) + j0, bv);
  }
  pdl_trigger();
  pdl_wait();
  const bool push = p.peer_world > 0;
  if (push) {
    if (threadIdx.x == 0) s_epoch = *reinterpret_cast<volatile unsigned*>(p.peer_seq);
    __syncthreads();
    if (!peer_wait(p, s_epoch + 1) && threadIdx.x == 0) set_status(p.status, JX_ERR_TIMEOUT);
  }
  bf16* h = reinterpret_cast<bf16*>(p.h);
  float x[8], y[8];
  if (p.ids) {
    int id = p.ids[m];
    if (id < 0) id = 0;
    if (id >= p.vocab) {
      set_status(p.status, JX_ERR_RANGE);
      id = 0;
    }
    vload8(reinterpret_cast<const bf16*>(p.table) + (long long)id * p.d + j0, x);
    if (p.embed_scale != 0.f) {
#pragma unroll
      for (int i = 0; i < 8; ++i) x[i] = rnd<bf16>(x[i] * p.embed_scale);
    }
    vstore8(h + m * p.ldh + j0, x);
  } else {
    const long long src = p.row_map ? (long long)p.row_map[m] : m;
    vload8(h + src * p.ldh + j0, x);
  }
  if (p.a || push) {
    float a[8];
    if (push) {
      float4 u0, u1;
      peer_sum8(p, s_epoch & 1, m, j0, u0, u1);
      a[0] = rnd<bf16>(u0.x), a[1] = rnd<bf16>(u0.y), a[2] = rnd<bf16>(u0.z), a[3] = rnd<bf16>(u0.w);
      a[4] = rnd<bf16>(u1.x), a[5] = rnd<bf16>(u1.y), a[6] = rnd<bf16>(u1.z), a[7] = rnd<bf16>(u1.w);
    } else if (p.a_f32) {
      // a float32 input (an all-reduced partial sum) is rounded to bf16 first
      const float4* af = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p.a) + m * p.lda + j0);
      const float4 u0 = af[0], u1 = af[1];
      a[0] = rnd<bf16>(u0.x), a[1] = rnd<bf16>(u0.y), a[2] = rnd<bf16>(u0.z), a[3] = rnd<bf16>(u0.w);
      a[4] = rnd<bf16>(u1.x), a[5] = rnd<bf16>(u1.y), a[6] = rnd<bf16>(u1.z), a[7] = rnd<bf16>(u1.w);
    } else {
      vload8(reinterpret_cast<const bf16*>(p.a) + m * p.lda + j0, a);
    }
    if (p.kind_pre != JX_NORM_NONE) {
      float t[8];
      vnormalize(a, t, p.d, p.kind_pre, p.eps, reinterpret_cast<const bf16*>(p.w_pre),
                 reinterpret_cast<const bf16*>(p.b_pre), j0, red);
#pragma unroll
      for (int i = 0; i < 8; ++i) x[i] = rnd<bf16>(x[i] + t[i]);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) x[i] = rnd<bf16>(x[i] + a[i]);
    }
    vstore8(h + m * p.ldh + j0, x);
  }
  if (p.out) {
    vnormalize_wb(x, y, p.d, p.kind, p.eps, wv, bv, p.b != nullptr, j0, red);
    bf16* o = reinterpret_cast<bf16*>(p.out);
    vstore8(o + (p.out_rp > 0 ? k128_offset(m, j0, p.out_rp) : m * p.ldo + j0), y);
  }
  if (p.out2) {
    vnormalize(x, y, p.d, p.kind, p.eps, reinterpret_cast<const bf16*>(p.w2), reinterpret_cast<const bf16*>(p.b2),
               j0, red);
    bf16* o = reinterpret_cast<bf16*>(p.out2);
    vstore8(o + (p.out2_rp > 0 ? k128_offset(m, j0, p.out2_rp) : m * p.ldo2 + j0), y);
  }
  if (push) {
    // every CTA read the epoch before arriving, so the last to arrive may advance it
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      if (atomicAdd(p.peer_seq + 1, 1u) == gridDim.x - 1) {
        p.peer_seq[1] = 0;
        p.peer_seq[0] = s_epoch + 1;
        __threadfence();
      }
    }
  }
}

// ------------------------------------------------------------------------------------------------
// Prefill-sized calls (M >= kNormRowsMin rows) that only normalise h into one output: one warp per row.
// One CTA per row (norm_vec_kernel) keeps a single 16-byte load per thread in flight and left most of
// the HBM bandwidth unused at 8192 rows; here a warp copies its whole row into shared memory with
// 16-byte cp.async copies, all in flight at once, then works from there.  Lane l takes vectors l, l + 32,
// l + 64, ... (16-byte vector v = elements 8v .. 8v + 7), the vectors that threads l, l + 32, ... of
// norm_vec_kernel hold, and forms the same per-vector partial sums, the same xor-shuffle tree over each
// group of 32 vectors (a warp there) and the same tree over the group totals as vblock_sum: the outputs
// are bit-identical to norm_vec_kernel's.
// ------------------------------------------------------------------------------------------------
constexpr int kNormRowsMin = 256;
constexpr int kNormRowsWarps = 4;          // rows per CTA
constexpr int kNormRowsMaxGroups = 16;     // d / 256 (groups of 32 vectors) <= 16

__device__ __forceinline__ float warp_tree_sum(float v) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n cp.async.wait_group 0;" ::: "memory");
}

__global__ void __launch_bounds__(32 * kNormRowsWarps) norm_rows_kernel(NormArgs p) {
  extern __shared__ uint4 rows_sm[];   // [kNormRowsWarps][d / 8] vectors
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long m = (long long)blockIdx.x * kNormRowsWarps + warp;
  pdl_trigger();
  pdl_wait();
  if (m >= p.M) return;
  const int ng = p.d >> 8;
  uint4* row = rows_sm + warp * (p.d >> 3);
  const uint4* hr = reinterpret_cast<const uint4*>(reinterpret_cast<const bf16*>(p.h) + m * p.ldh);
  for (int g = 0; g < ng; ++g) cp_async16(row + g * 32 + lane, hr + g * 32 + lane);
  cp_async_wait_all();
  __syncwarp();
  // Each group's xor-tree total is the same in every lane; lane g keeps group g's, and the xor tree over
  // the lanes (zero above the group count) is vblock_sum's second stage.
  float t = 0.f, mean = 0.f, den;
  if (p.kind == JX_NORM_LAYER) {
    for (int g = 0; g < ng; ++g) {
      float x[8];
      unpack8(row[g * 32 + lane], x);
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) s += x[i];
      const float sg = warp_tree_sum(s);
      if (g == lane) t = sg;
    }
    mean = warp_tree_sum(t) / (float)p.d;
    t = 0.f;
    for (int g = 0; g < ng; ++g) {
      float x[8];
      unpack8(row[g * 32 + lane], x);
      float v = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) v += (x[i] - mean) * (x[i] - mean);
      const float sg = warp_tree_sum(v);
      if (g == lane) t = sg;
    }
    den = sqrtf(warp_tree_sum(t) / (float)p.d + p.eps);
  } else {
    for (int g = 0; g < ng; ++g) {
      float x[8];
      unpack8(row[g * 32 + lane], x);
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) s += x[i] * x[i];
      const float sg = warp_tree_sum(s);
      if (g == lane) t = sg;
    }
    den = sqrtf(warp_tree_sum(t) / (float)p.d + p.eps);
  }
  const bf16* w = reinterpret_cast<const bf16*>(p.w);
  const bf16* bias = reinterpret_cast<const bf16*>(p.b);
  bf16* o = reinterpret_cast<bf16*>(p.out);
  for (int g = 0; g < ng; ++g) {
    const int j0 = g * 256 + lane * 8;
    float x[8], wv[8], bv[8], y[8];
    unpack8(row[g * 32 + lane], x);
    vload8(w + j0, wv);
    if (p.kind == JX_NORM_LAYER) {
      const bool b = bias != nullptr;
      if (b) vload8(bias + j0, bv);
#pragma unroll
      for (int i = 0; i < 8; ++i) y[i] = rnd<bf16>((x[i] - mean) / den * wv[i] + (b ? bv[i] : 0.f));
    } else if (p.kind == JX_NORM_RMS) {
#pragma unroll
      for (int i = 0; i < 8; ++i) y[i] = rnd<bf16>(wv[i] * rnd<bf16>(x[i] / den));
    } else {
      const float inv = 1.0f / den;
#pragma unroll
      for (int i = 0; i < 8; ++i) y[i] = rnd<bf16>((wv[i] + 1.0f) * (x[i] * inv));
    }
    vstore8(o + (p.out_rp > 0 ? k128_offset(m, j0, p.out_rp) : m * p.ldo + j0), y);
  }
}

static bool norm_rows_ok(const NormArgs& p) {
  const uintptr_t ptrs = reinterpret_cast<uintptr_t>(p.h) | reinterpret_cast<uintptr_t>(p.out) |
                         reinterpret_cast<uintptr_t>(p.w) | reinterpret_cast<uintptr_t>(p.b);
  return p.M >= kNormRowsMin && p.peer_world == 0 && !p.ids && !p.row_map && !p.a && !p.out2 && p.out && p.w &&
         p.kind_pre == JX_NORM_NONE &&
         (p.kind == JX_NORM_RMS || p.kind == JX_NORM_GEMMA || p.kind == JX_NORM_LAYER) && p.d % 256 == 0 &&
         p.d <= 256 * kNormRowsMaxGroups && (ptrs & 15) == 0 && p.ldh % 8 == 0 && (p.out_rp > 0 || p.ldo % 8 == 0);
}

int run_norm(int dtype, const NormArgs& p, bool pdl, cudaStream_t stream) {
  if (p.M <= 0 || p.d <= 0) return JX_ERR_SHAPE;
  const bool aligned = ((p.ldh | p.lda | p.ldo | p.ldo2) & 7) == 0;
  const bool vec = dtype == JX_BF16 && p.d % 8 == 0 && p.d / 8 <= 1024 && (p.d / 8) % 32 == 0 && aligned;
  if (p.peer_world != 0) {
    // push mode: the vectorised kernel only; the partials are float32 rows of lda floats
    if (!vec || p.peer_world < 1 || p.peer_world > 8 || p.d % 64 || p.peer_units != p.d / 64) return JX_ERR_SHAPE;
    if (!p.peer_recv || !p.peer_flags || !p.peer_seq || p.a) return JX_ERR_ARG;
    if ((p.lda & 3) || (p.peer_stride & 3) || ((uintptr_t)p.peer_recv & 15) || ((uintptr_t)p.peer_seq & 7) ||
        (long long)p.M * p.lda > p.peer_stride)
      return JX_ERR_ARG;
  }
  if (vec && norm_rows_ok(p)) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((p.M + kNormRowsWarps - 1) / kNormRowsWarps));
    cfg.blockDim = dim3(32 * kNormRowsWarps);
    cfg.dynamicSmemBytes = (size_t)kNormRowsWarps * p.d * 2;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return launch_ex(&cfg, norm_rows_kernel, p) == cudaSuccess ? JX_OK : JX_ERR_CUDA;
  }
  if (vec) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.M);
    cfg.blockDim = dim3(p.d / 8);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return launch_ex(&cfg, norm_vec_kernel, p) == cudaSuccess ? JX_OK : JX_ERR_CUDA;
  }
  constexpr int NT = 256;
  const size_t smem = (size_t)(2 * p.d + NT / 32 + 1) * sizeof(float);
  if (smem > 200 * 1024) return JX_ERR_SHAPE;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.M);
  cfg.blockDim = dim3(NT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t err;
  if (dtype == JX_BF16) {
    if (smem > 48 * 1024)
      cudaFuncSetAttribute(norm_kernel<bf16, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    err = launch_ex(&cfg, norm_kernel<bf16, NT>, p);
  } else if (dtype == JX_F32) {
    if (smem > 48 * 1024)
      cudaFuncSetAttribute(norm_kernel<float, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    err = launch_ex(&cfg, norm_kernel<float, NT>, p);
  } else {
    return JX_ERR_DTYPE;
  }
  return err == cudaSuccess ? JX_OK : JX_ERR_CUDA;
}

}  // namespace jxb
