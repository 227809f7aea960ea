// Attention prologue after the fused QKV projection: optional per-head QK RMSNorm (Gemma3,
// nn/attention.py:274-276 with gemma3.py:89-106), rotary embedding on the first rotary_dim dims
// (nn/position.py:78-141, half-split "rotate_half" form, applied in the model dtype), and the KV-cache
// append (cache.py:183-243): k and v of token row m are written into the cache slot of that token.
//
// Positions: in prefill (decode == 0) row m = b*S + s sits at position s and cache slot s; in decode
// (S == 1) row b sits at pos_id[b] + 1, the slot after the last valid one.
#include "common.cuh"

namespace jxb {

typedef jx_qkv_args QkvArgs;

template <typename T>
__global__ void __launch_bounds__(256) qkv_rope_append_kernel(QkvArgs p) {
  extern __shared__ float buf[];  // [8 warps][hd]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* v = buf + warp * p.hd;
  const long long m = blockIdx.x;
  // Dependents are released only after this grid's own wait: when the decode attention that follows
  // starts, every kernel before this one has completed, so it may load the keys and values of earlier
  // steps before its own wait.
  pdl_wait();
  pdl_trigger();
  const int b = (int)(m / p.S), s = (int)(m % p.S);
  int pos = s;
  if (p.decode) pos = p.pos_id[b] + 1;
  if (pos < 0 || pos >= p.max_pos || pos >= p.T) {
    set_status(p.status, JX_ERR_RANGE);
    return;
  }
  const T* row = reinterpret_cast<const T*>(p.qkv) + m * p.ld_qkv;
  const T* cos = reinterpret_cast<const T*>(p.cos) + (long long)pos * p.rd;
  const T* sin = reinterpret_cast<const T*>(p.sin) + (long long)pos * p.rd;
  const int n_heads = p.Hq + 2 * p.Hkv;
  const int half = p.rd >> 1;
  // grid.y spreads the heads of a row over CTAs of 8 warps, one head per warp
  for (int head = blockIdx.y * 8 + warp; head < n_heads; head += 8 * gridDim.y) {
    const bool is_q = head < p.Hq, is_k = !is_q && head < p.Hq + p.Hkv;
    const T* src = row + (long long)head * p.hd;
    for (int j = lane; j < p.hd; j += 32) v[j] = to_f(src[j]);
    __syncwarp();
    const T* nw = is_q ? reinterpret_cast<const T*>(p.qn_w) : (is_k ? reinterpret_cast<const T*>(p.kn_w) : nullptr);
    if (nw) {
      float ss = 0.f;
      for (int j = lane; j < p.hd; j += 32) ss += v[j] * v[j];
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      const float inv = 1.0f / sqrtf(ss / (float)p.hd + p.eps);
      __syncwarp();
      for (int j = lane; j < p.hd; j += 32) v[j] = rnd<T>((to_f(nw[j]) + 1.0f) * (v[j] * inv));
      __syncwarp();
    }
    float outv[8];
    int cnt = 0;
    for (int j = lane; j < p.hd; j += 32, ++cnt) {
      float o = v[j];
      if ((is_q || is_k) && j < p.rd) {
        const float rot = j < half ? -v[j + half] : v[j - half];
        const float a = rnd<T>(v[j] * to_f(cos[j]));
        const float c = rnd<T>(rot * to_f(sin[j]));
        o = rnd<T>(a + c);
      }
      outv[cnt] = o;
    }
    __syncwarp();
    cnt = 0;
    for (int j = lane; j < p.hd; j += 32, ++cnt) {
      if (is_q) {
        reinterpret_cast<T*>(p.q_out)[(m * p.Hq + head) * p.hd + j] = from_f<T>(outv[cnt]);
      } else {
        const int kvh = is_k ? head - p.Hq : head - p.Hq - p.Hkv;
        T* cache = reinterpret_cast<T*>(is_k ? p.k_cache : p.v_cache);
        cache[(((long long)b * p.T + pos) * p.Hkv + kvh) * p.hd + j] = from_f<T>(outv[cnt]);
      }
    }
    __syncwarp();
  }
}

// Prefill-sized calls (M >= kRopeRowsMin token rows, decode == 0) of bfloat16 models without QK norm,
// hd % 8 == 0 and rd % 16 == 0: one CTA per token row in 16-byte vectors.  The kernel above keeps one
// head (256 bytes) per warp in flight and left most of the HBM bandwidth unused at 8192 rows.  Here the
// CTA first loads every vector of the row into shared memory (the rotate-half partner of a vector is
// the vector rd / 16 places away in the same head), then each thread rotates and stores its vectors.
// The per-element arithmetic is the kernel's above, so q, k and v are bit-identical to it.
constexpr int kRopeRowsMin = 256;
constexpr int kRopeRowsMaxBytes = 48 * 1024;   // one token row of q, k and v in shared memory

__global__ void __launch_bounds__(256) qkv_rope_rows_kernel(QkvArgs p) {
  extern __shared__ uint4 rowv[];   // [(Hq + 2 Hkv) * hd / 8] vectors of 8 bf16
  const long long m = blockIdx.x;
  pdl_wait();
  pdl_trigger();
  const int b = (int)(m / p.S), pos = (int)(m % p.S);
  if (pos >= p.max_pos || pos >= p.T) {
    if (threadIdx.x == 0) set_status(p.status, JX_ERR_RANGE);
    return;
  }
  const int vph = p.hd >> 3;                    // vectors per head
  const int nv = (p.Hq + 2 * p.Hkv) * vph;
  const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const bf16*>(p.qkv) + m * p.ld_qkv);
  for (int v = threadIdx.x; v < nv; v += blockDim.x) rowv[v] = src[v];
  __syncthreads();
  const int rv = p.rd >> 3, hv = p.rd >> 4;     // rotated vectors of a head, half of them
  const bf16* cos = reinterpret_cast<const bf16*>(p.cos) + (long long)pos * p.rd;
  const bf16* sin = reinterpret_cast<const bf16*>(p.sin) + (long long)pos * p.rd;
  for (int v = threadIdx.x; v < nv; v += blockDim.x) {
    const int head = v / vph, jv = v - head * vph;
    const bool is_q = head < p.Hq, is_k = !is_q && head < p.Hq + p.Hkv;
    uint4 o = rowv[v];
    if ((is_q || is_k) && jv < rv) {
      const bool lo = jv < hv;
      float x[8], r[8], c[8], sn[8], y[8];
      unpack8(o, x);
      unpack8(rowv[lo ? v + hv : v - hv], r);
      unpack8(*reinterpret_cast<const uint4*>(cos + jv * 8), c);
      unpack8(*reinterpret_cast<const uint4*>(sin + jv * 8), sn);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float rot = lo ? -r[i] : r[i];
        const float a = rnd<bf16>(x[i] * c[i]);
        const float cc = rnd<bf16>(rot * sn[i]);
        y[i] = rnd<bf16>(a + cc);
      }
      o.x = pack_bf16x2(y[0], y[1]);
      o.y = pack_bf16x2(y[2], y[3]);
      o.z = pack_bf16x2(y[4], y[5]);
      o.w = pack_bf16x2(y[6], y[7]);
    }
    bf16* dst;
    if (is_q) {
      dst = reinterpret_cast<bf16*>(p.q_out) + (m * p.Hq + head) * p.hd;
    } else {
      const int kvh = is_k ? head - p.Hq : head - p.Hq - p.Hkv;
      dst = reinterpret_cast<bf16*>(is_k ? p.k_cache : p.v_cache) + (((long long)b * p.T + pos) * p.Hkv + kvh) * p.hd;
    }
    *reinterpret_cast<uint4*>(dst + jv * 8) = o;
  }
}

static bool qkv_rope_rows_ok(int dtype, const QkvArgs& p) {
  const uintptr_t ptrs = reinterpret_cast<uintptr_t>(p.qkv) | reinterpret_cast<uintptr_t>(p.cos) |
                         reinterpret_cast<uintptr_t>(p.sin) | reinterpret_cast<uintptr_t>(p.q_out) |
                         reinterpret_cast<uintptr_t>(p.k_cache) | reinterpret_cast<uintptr_t>(p.v_cache);
  return dtype == JX_BF16 && !p.decode && p.M >= kRopeRowsMin && !p.qn_w && !p.kn_w && p.hd % 8 == 0 &&
         p.rd % 16 == 0 && p.ld_qkv % 8 == 0 && (ptrs & 15) == 0 &&
         (long long)(p.Hq + 2 * p.Hkv) * p.hd * 2 <= kRopeRowsMaxBytes;
}

int run_qkv_rope_append(int dtype, const QkvArgs& p, bool pdl, cudaStream_t stream) {
  if (p.M <= 0 || p.S <= 0 || p.hd <= 0 || p.hd > 256 || p.rd < 0 || p.rd > p.hd || (p.rd & 1)) return JX_ERR_SHAPE;
  if (p.decode && p.S != 1) return JX_ERR_SHAPE;
  if (qkv_rope_rows_ok(dtype, p)) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.M);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = (size_t)(p.Hq + 2 * p.Hkv) * p.hd * 2;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return launch_ex(&cfg, qkv_rope_rows_kernel, p) == cudaSuccess ? JX_OK : JX_ERR_CUDA;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.M, (p.Hq + 2 * p.Hkv + 7) / 8);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = 8 * p.hd * sizeof(float);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t err;
  if (dtype == JX_BF16)
    err = launch_ex(&cfg, qkv_rope_append_kernel<bf16>, p);
  else if (dtype == JX_F32)
    err = launch_ex(&cfg, qkv_rope_append_kernel<float>, p);
  else
    return JX_ERR_DTYPE;
  return err == cudaSuccess ? JX_OK : JX_ERR_CUDA;
}

// ------------------------------------------------------------------------------------------------
// Standalone rotary embedding (RotaryEmbedding.apply_rotary_pos_emb, nn/position.py:78-141): q and k
// rows at arbitrary positions, cos / sin tables in the same dtype, the first rd dims rotated with
// rotate_half in the model dtype (q*cos and rotate_half(q)*sin each rounded, then their sum), the rest
// passed through.  One warp per head, grid (rows, ceil((Hq + Hk) / 8)).
// ------------------------------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(256) rope_apply_kernel(jx_rope_args p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long m = blockIdx.x;
  pdl_trigger();
  pdl_wait();
  const int pos = p.pos[m];
  const bool bad = pos < 0 || pos >= p.n_pos;
  if (bad && threadIdx.x == 0) set_status(p.status, JX_ERR_RANGE);
  const int half = p.rd >> 1;
  for (int head = blockIdx.y * 8 + warp; head < p.Hq + p.Hk; head += 8 * gridDim.y) {
    const bool is_q = head < p.Hq;
    const T* src = reinterpret_cast<const T*>(is_q ? p.q : p.k) +
                   (m * (is_q ? p.Hq : p.Hk) + (is_q ? head : head - p.Hq)) * (long long)p.hd;
    T* dst = reinterpret_cast<T*>(is_q ? p.q_out : p.k_out) +
             (m * (is_q ? p.Hq : p.Hk) + (is_q ? head : head - p.Hq)) * (long long)p.hd;
    const T* cos = reinterpret_cast<const T*>(p.cos) + (long long)(bad ? 0 : pos) * p.rd;
    const T* sin = reinterpret_cast<const T*>(p.sin) + (long long)(bad ? 0 : pos) * p.rd;
    // every lane reads its inputs before any lane writes (dst may alias src)
    float o[8];
    int cnt = 0;
    for (int j = lane; j < p.hd; j += 32, ++cnt) {
      const float x = to_f(src[j]);
      if (bad) {
        o[cnt] = 0.f;
      } else if (j < p.rd) {
        const float rot = j < half ? -to_f(src[j + half]) : to_f(src[j - half]);
        // separate roundings of both products (no fused multiply-add), as two dtype multiplies then an add
        o[cnt] = rnd<T>(__fadd_rn(rnd<T>(__fmul_rn(x, to_f(cos[j]))), rnd<T>(__fmul_rn(rot, to_f(sin[j])))));
      } else {
        o[cnt] = x;
      }
    }
    __syncwarp();
    cnt = 0;
    for (int j = lane; j < p.hd; j += 32, ++cnt) dst[j] = from_f<T>(o[cnt]);
    __syncwarp();
  }
}

int run_rope_apply(int dtype, const jx_rope_args& p, bool pdl, cudaStream_t stream) {
  if (p.M <= 0 || p.Hq < 0 || p.Hk < 0 || p.Hq + p.Hk <= 0 || p.hd <= 0 || p.hd > 256 || p.rd <= 0 ||
      p.rd > p.hd || (p.rd & 1) || p.n_pos <= 0 || p.M > 2147483647)
    return JX_ERR_SHAPE;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.M, (p.Hq + p.Hk + 7) / 8);
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t err;
  if (dtype == JX_BF16)
    err = launch_ex(&cfg, rope_apply_kernel<bf16>, p);
  else if (dtype == JX_F32)
    err = launch_ex(&cfg, rope_apply_kernel<float>, p);
  else
    return JX_ERR_DTYPE;
  return err == cudaSuccess ? JX_OK : JX_ERR_CUDA;
}

}  // namespace jxb
