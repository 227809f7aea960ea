// min-p, top-k and top-p filtering of vocabulary logits (inference_engine/sampling.py:34-75 for the three
// filters, :169-188 for their order: min-p, then top-k, then top-p), filtered entries set to -inf.
//
// One thread-block cluster of CS CTAs per logits row; CTA r holds columns [r * slice, (r + 1) * slice) of
// the row in shared memory as float32 (read from HBM once), so every later pass runs out of shared memory
// and the cluster combines its CTAs' partial results through distributed shared memory, in rank order.
//
//   max       row maximum (exact in any order)
//   min-p     probabilities p_i = dtype(exp(x_i - max) / sum), the sum in float32 in a fixed order
//             (per-thread strips, the warp butterfly, the warps, the ranks); entries with p_i < min_p
//             set to -inf unless no entry of the row has p_i >= min_p
//   top-k     the k-th largest value (with multiplicity) by a most-significant-digit radix select over
//             order-preserving 32-bit keys, 8 bits a pass (2 passes for bfloat16 rows, whose keys differ
//             only in their upper 16 bits): integer histograms, exact; entries below it set to -inf
//   top-p     the reference keeps x >= sorted[idx], idx = #{i : cumsum(sorted probabilities)_i < top_p}
//             (clamped to the last entry).  Since the cumulative sum only grows, sorted[idx] is the
//             largest value t whose mass G(t) = sum of p_i over x_i >= t reaches top_p (every value when
//             the whole row's mass stays below it).  The same radix descent finds t from per-digit masses;
//             the masses are summed as 2^-56 fixed-point integers, so they are exact and independent of
//             the summation order (the reference's float32 cumulative sum differs from the exact one by
//             its rounding; only a row whose cumulative sum passes within that rounding of top_p at the
//             cutoff can keep a different set)
//
// The kernel only reads and writes its own row slice, so out may alias logits.  Cluster barriers are
// hardware barriers (no spin loops).
#include "common.cuh"

namespace jxb {

constexpr int kFlThreads = 512;
constexpr int kFlWarps = kFlThreads / 32;
constexpr int kFlMaxCS = 8;             // portable cluster size
constexpr int kFlMaxSlice = 49152;      // float32 columns per CTA (192 KB of shared memory)
constexpr double kFlFix = 72057594037927936.0;   // 2^56

struct FilterArgs {
  int B, V;
  const void* logits;
  long long ld_in;
  void* out;
  long long ld_out;
  int top_k;
  float min_p;
  unsigned long long top_p_fix;   // float32(top_p) * 2^56; ~0 = top-p off
};

// Order-preserving key: a larger float has a larger unsigned key (-inf lowest; NaN is excluded upstream).
// -0.0 takes the key of +0.0 (the reference compares values, and -0.0 >= 0.0).
__device__ __forceinline__ uint32_t fl_key(float v) {
  const uint32_t u = __float_as_uint(v == 0.f ? 0.f : v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ uint32_t dsmem_ld_u32(uint32_t cluster_addr) {
  uint32_t v;
  asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(cluster_addr) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long dsmem_ld_u64(uint32_t cluster_addr) {
  unsigned long long v;
  asm volatile("ld.shared::cluster.u64 %0, [%1];" : "=l"(v) : "r"(cluster_addr) : "memory");
  return v;
}

struct FlShared {
  float wred[kFlWarps];
  float bc;                          // block broadcast
  float pub[4];                      // this CTA's partials: max, min-p sum, min-p kept count, top-p sum
  unsigned cnt[2][256];              // top-k digit counts (double-buffered across passes)
  unsigned long long mass[2][256];   // top-p digit masses
  unsigned tot_cnt[256];
  unsigned long long tot_mass[256];
  uint32_t sel_digit;
  unsigned long long sel_rest;
};

// Fixed-order block sum / max (every thread gets the result).
__device__ __forceinline__ float fl_block_sum(float v, FlShared& s) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) s.wred[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = s.wred[0];
    for (int w = 1; w < kFlWarps; ++w) t += s.wred[w];
    s.bc = t;
  }
  __syncthreads();
  return s.bc;
}
__device__ __forceinline__ float fl_block_max(float v, FlShared& s) {
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if ((threadIdx.x & 31) == 0) s.wred[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = s.wred[0];
    for (int w = 1; w < kFlWarps; ++w) t = fmaxf(t, s.wred[w]);
    s.bc = t;
  }
  __syncthreads();
  return s.bc;
}

// Cluster-wide combination of pub[slot] (written by thread 0 of every CTA before the call) in rank order.
__device__ __forceinline__ float fl_cluster_sum(FlShared& s, int slot, int CS) {
  cluster_sync_all();
  const uint32_t a = smem_u32(&s.pub[slot]);
  float t = 0.f;
  for (int r = 0; r < CS; ++r) t += dsmem_ld_f32(dsmem_map(a, (uint32_t)r));
  return t;
}
__device__ __forceinline__ float fl_cluster_max(FlShared& s, int slot, int CS) {
  cluster_sync_all();
  const uint32_t a = smem_u32(&s.pub[slot]);
  float t = -INFINITY;
  for (int r = 0; r < CS; ++r) t = fmaxf(t, dsmem_ld_f32(dsmem_map(a, (uint32_t)r)));
  return t;
}

template <typename T>
__global__ void __launch_bounds__(kFlThreads, 1) filter_kernel(FilterArgs a, int slice) {
  extern __shared__ __align__(16) float vals[];
  __shared__ FlShared s;
  const int CS = (int)cluster_nctarank(), rank = (int)cluster_ctarank();
  const int row = blockIdx.x / CS, tid = threadIdx.x;
  const long long c0 = (long long)rank * slice;
  const int n = (int)(a.V - c0 < slice ? (a.V - c0 > 0 ? a.V - c0 : 0) : slice);
  const T* src = reinterpret_cast<const T*>(a.logits) + row * a.ld_in + c0;
  T* dst = reinterpret_cast<T*>(a.out) + row * a.ld_out + c0;
  const bool is_bf16 = sizeof(T) == 2;

  float lmax = -INFINITY;
  for (int i = tid; i < n; i += kFlThreads) {
    const float v = to_f(src[i]);
    vals[i] = v;
    lmax = fmaxf(lmax, v);
  }
  lmax = fl_block_max(lmax, s);
  if (tid == 0) s.pub[0] = lmax;
  const float M = fl_cluster_max(s, 0, CS);
  // (a row without a finite value is rejected before the call; such a row passes through unchanged)
  const bool live = M > -INFINITY;

  // ---------------- min-p ----------------
  if (a.min_p > 0.f && live) {
    float ls = 0.f;
    for (int i = tid; i < n; i += kFlThreads) ls += expf(vals[i] - M);
    ls = fl_block_sum(ls, s);
    if (tid == 0) s.pub[1] = ls;
    const float S = fl_cluster_sum(s, 1, CS);
    float lk = 0.f;
    for (int i = tid; i < n; i += kFlThreads) lk += rnd<T>(expf(vals[i] - M) / S) >= a.min_p ? 1.f : 0.f;
    lk = fl_block_sum(lk, s);
    if (tid == 0) s.pub[2] = lk;
    const float kept = fl_cluster_sum(s, 2, CS);
    if (kept > 0.f)
      for (int i = tid; i < n; i += kFlThreads)
        if (rnd<T>(expf(vals[i] - M) / S) < a.min_p) vals[i] = -INFINITY;
    __syncthreads();
  }

  const int passes = is_bf16 ? 2 : 4;
  int buf = 0;   // histogram buffer of the next pass (top-k then top-p, alternating)

  // ---------------- top-k ----------------
  if (a.top_k > 0 && a.top_k < a.V && live) {
    uint32_t prefix = 0, pmask = 0;
    unsigned kk = (unsigned)a.top_k;   // rank of the wanted value among the entries matching the prefix
    for (int p = 0; p < passes; ++p, buf ^= 1) {
      const int shift = 24 - 8 * p;
      if (tid < 256) s.cnt[buf][tid] = 0;
      __syncthreads();
      for (int i = tid; i < n; i += kFlThreads) {
        const uint32_t key = fl_key(vals[i]);
        if ((key & pmask) == prefix) atomicAdd(&s.cnt[buf][(key >> shift) & 255u], 1u);
      }
      cluster_sync_all();
      if (tid < 256) {
        const uint32_t ad = smem_u32(&s.cnt[buf][tid]);
        unsigned t = 0;
        for (int r = 0; r < CS; ++r) t += dsmem_ld_u32(dsmem_map(ad, (uint32_t)r));
        s.tot_cnt[tid] = t;
      }
      __syncthreads();
      if (tid == 0) {
        unsigned above = 0;
        int d = 255;
        for (; d > 0; --d) {
          if (above + s.tot_cnt[d] >= kk) break;
          above += s.tot_cnt[d];
        }
        s.sel_digit = (uint32_t)d;
        s.sel_rest = above;
      }
      __syncthreads();
      prefix |= s.sel_digit << shift;
      pmask |= 255u << shift;
      kk -= (unsigned)s.sel_rest;
    }
    for (int i = tid; i < n; i += kFlThreads)
      if (fl_key(vals[i]) < prefix) vals[i] = -INFINITY;
    __syncthreads();
  }

  // ---------------- top-p ----------------
  if (a.top_p_fix != ~0ull && live) {
    const unsigned long long P = a.top_p_fix;
    uint32_t cut = 0;
    if (P == 0) {
      cut = fl_key(M);   // top_p <= 0: the cutoff is the first sorted entry
    } else {
      float ls = 0.f;
      for (int i = tid; i < n; i += kFlThreads) ls += expf(vals[i] - M);
      ls = fl_block_sum(ls, s);
      if (tid == 0) s.pub[3] = ls;
      const float S = fl_cluster_sum(s, 3, CS);
      uint32_t prefix = 0, pmask = 0;
      unsigned long long above = 0;   // mass of the entries above the prefix's range
      bool all = false;                // the whole row's mass stays below top_p: keep everything
      for (int p = 0; p < passes; ++p, buf ^= 1) {
        const int shift = 24 - 8 * p;
        if (tid < 256) s.mass[buf][tid] = 0;
        __syncthreads();
        for (int i = tid; i < n; i += kFlThreads) {
          const float v = vals[i];
          const uint32_t key = fl_key(v);
          if ((key & pmask) != prefix) continue;
          const float q = rnd<T>(expf(v - M) / S);
          const unsigned long long f = __double2ull_rz((double)q * kFlFix);
          if (f) atomicAdd(&s.mass[buf][(key >> shift) & 255u], f);
        }
        cluster_sync_all();
        if (tid < 256) {
          const uint32_t ad = smem_u32(&s.mass[buf][tid]);
          unsigned long long t = 0;
          for (int r = 0; r < CS; ++r) t += dsmem_ld_u64(dsmem_map(ad, (uint32_t)r));
          s.tot_mass[tid] = t;
        }
        __syncthreads();
        if (tid == 0) {
          unsigned long long acc = above;
          int d = 255;
          for (; d >= 0; --d) {
            if (acc + s.tot_mass[d] >= P) break;
            acc += s.tot_mass[d];
          }
          s.sel_digit = d < 0 ? 0xffffffffu : (uint32_t)d;
          s.sel_rest = acc;
        }
        __syncthreads();
        if (s.sel_digit == 0xffffffffu) {   // only possible in the first pass
          all = true;
          break;
        }
        prefix |= s.sel_digit << shift;
        pmask |= 255u << shift;
        above = s.sel_rest;
      }
      cut = all ? 0u : prefix;
    }
    for (int i = tid; i < n; i += kFlThreads)
      if (fl_key(vals[i]) < cut) vals[i] = -INFINITY;
    __syncthreads();
  }

  for (int i = tid; i < n; i += kFlThreads) dst[i] = from_f<T>(vals[i]);
  cluster_sync_all();   // no CTA leaves while another may still read its shared memory
}

template <typename T>
static int launch_filter(const FilterArgs& a, int cs, int slice, cudaStream_t stream) {
  static bool configured = false;
  const int smem = slice * 4;
  if (!configured) {
    if (cudaFuncSetAttribute(filter_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, kFlMaxSlice * 4) !=
        cudaSuccess)
      return JX_ERR_CUDA;
    configured = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(a.B * cs));
  cfg.blockDim = dim3(kFlThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cs;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return launch_ex(&cfg, filter_kernel<T>, a, slice) == cudaSuccess ? JX_OK : JX_ERR_CUDA;
}

int run_filter_logits(const jx_filter_args& p, cudaStream_t stream) {
  if (p.B < 0 || p.V <= 0 || p.ld_in < p.V || p.ld_out < p.V) return JX_ERR_SHAPE;
  if (p.B == 0) return JX_OK;
  if (p.B > 65535 / kFlMaxCS || (long long)p.V > (long long)kFlMaxCS * kFlMaxSlice) return JX_ERR_SHAPE;
  if (p.dtype != JX_F32 && p.dtype != JX_BF16) return JX_ERR_DTYPE;
  // about 16K columns a CTA, at most 8 CTAs a row
  int cs = (p.V + 16383) / 16384;
  cs = cs > kFlMaxCS ? kFlMaxCS : cs;
  int slice = (p.V + cs - 1) / cs;
  slice = (slice + 7) & ~7;
  FilterArgs a;
  a.B = p.B;
  a.V = p.V;
  a.logits = p.logits;
  a.ld_in = p.ld_in;
  a.out = p.out;
  a.ld_out = p.ld_out;
  a.top_k = p.top_k;
  a.min_p = p.min_p > 0.f ? p.min_p : 0.f;
  if (!(p.top_p < 1.0f))
    a.top_p_fix = ~0ull;
  else if (!(p.top_p > 0.0f))
    a.top_p_fix = 0;
  else
    a.top_p_fix = (unsigned long long)((double)p.top_p * kFlFix);
  return p.dtype == JX_BF16 ? launch_filter<bf16>(a, cs, slice, stream) : launch_filter<float>(a, cs, slice, stream);
}

}  // namespace jxb
