// Attention for any head size and dtype on CUDA cores (one CTA per query row and head).  It serves the
// float32 path and shapes the tensor-core kernels do not cover, and reproduces Attention.mha
// (nn/attention.py:321-400) exactly: scores = dtype(dtype(q.k) * dtype(attn_scale)); causal, sliding
// window and prefix-padding masks; a row with no visible key attends uniformly to the first uniform_T
// slots (all T by default: the reference's cache length);
// float32 softmax rounded to dtype (optionally stored: the attention weights); dtype(sum p*v) with
// float32 accumulation.  KV heads are shared by n_rep = Hq / Hkv query heads (repeat_kv, :294-319) by
// indexing, not copying.
#include "common.cuh"

namespace jxb {

typedef jx_attn_args AttnArgs;

template <typename T>
__global__ void __launch_bounds__(128) attention_generic_kernel(AttnArgs p) {
  extern __shared__ float sc[];  // [T] scores, then [4] reduction scratch
  const int s = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x;
  const int kvh = h / (p.Hq / p.Hkv);
  const long long row = (long long)b * p.S + s;
  pdl_trigger();
  pdl_wait();
  int valid = p.len_ptr ? p.len_ptr[b] + p.len_add : p.T;
  if (valid > p.T) {
    set_status(p.status, JX_ERR_RANGE);
    valid = p.T;
  }
  // Anchor of the causal / window masks: the query's own position in prefill, the newest token in decode.
  const int anchor = p.causal ? s : valid - 1;
  const T* q = reinterpret_cast<const T*>(p.q) + (row * p.Hq + h) * p.hd;
  const T* K = reinterpret_cast<const T*>(p.k);
  const T* V = reinterpret_cast<const T*>(p.v);
  const float scale_t = rnd<T>(p.scale);
  float* red = sc + p.T;
  // Keys that can be visible: [j_lo, j_hi).  Every key outside is masked, so the loops below stay on this
  // range unless the whole row is masked (then every one of the T slots gets the same probability).
  int j_hi = valid, j_lo = 0;
  if (p.causal && anchor + 1 < j_hi) j_hi = anchor + 1;
  if (p.window > 0 && anchor - p.window + 1 > j_lo) j_lo = anchor - p.window + 1;
  if (j_hi < j_lo) j_hi = j_lo;
  const int warp = tid >> 5, lane = tid & 31;

  // scores: a warp per key, lanes over the head dimension
  float mx = -INFINITY;
  for (int j = j_lo + warp; j < j_hi; j += 4) {
    const T* kr = K + (((long long)b * p.T + j) * p.Hkv + kvh) * p.hd;
    float dot = 0.f;
    for (int d = lane; d < p.hd; d += 32) dot += to_f(q[d]) * to_f(kr[d]);
    for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
    const float x = rnd<T>(rnd<T>(dot) * scale_t);
    mx = fmaxf(mx, x);
    if (lane == 0) sc[j] = x;
  }
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) red[warp] = mx;
  __syncthreads();
  mx = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  const bool all_masked = (mx == -INFINITY);
  if (all_masked) {
    j_lo = 0;
    j_hi = p.uniform_T > 0 && p.uniform_T < p.T ? p.uniform_T : p.T;
  }
  __syncthreads();
  float l = 0.f;
  for (int j = j_lo + tid; j < j_hi; j += 128) {
    const float e = all_masked ? 1.0f : expf(sc[j] - mx);
    sc[j] = e;
    l += e;
  }
  for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
  if (lane == 0) red[warp] = l;
  __syncthreads();
  l = (red[0] + red[1]) + (red[2] + red[3]);
  for (int j = j_lo + tid; j < j_hi; j += 128) sc[j] = rnd<T>(sc[j] / l);
  __syncthreads();
  if (p.weights) {
    // the probabilities themselves (Attention.mha with output_attentions): [B, Hq, S, T], zero where masked
    T* w = reinterpret_cast<T*>(p.weights) + (((long long)b * p.Hq + h) * p.S + s) * p.T;
    for (int j = tid; j < p.T; j += 128) w[j] = from_f<T>(j >= j_lo && j < j_hi ? sc[j] : 0.f);
  }
  for (int d = tid; d < p.hd; d += 128) {
    float acc = 0.f;
    for (int j = j_lo; j < j_hi; ++j) {
      const float pj = sc[j];
      if (pj != 0.f) acc += pj * to_f(V[(((long long)b * p.T + j) * p.Hkv + kvh) * p.hd + d]);
    }
    const long long col = (long long)h * p.hd + d;
    const long long off = p.out_rp > 0 ? k128_offset(row, col, p.out_rp) : row * p.ldo + col;
    reinterpret_cast<T*>(p.out)[off] = from_f<T>(acc);
  }
}

int run_attention_generic(int dtype, const AttnArgs& p, bool pdl, cudaStream_t stream) {
  if (p.B <= 0 || p.S <= 0 || p.Hq <= 0 || p.Hkv <= 0 || p.hd <= 0 || p.T <= 0) return JX_ERR_SHAPE;
  if (p.Hq % p.Hkv) return JX_ERR_SHAPE;
  const size_t smem = (size_t)(p.T + 4) * sizeof(float);
  if (smem > 200 * 1024) return JX_ERR_SHAPE;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.S, p.Hq, p.B);
  cfg.blockDim = dim3(128);
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
      cudaFuncSetAttribute(attention_generic_kernel<bf16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    err = launch_ex(&cfg, attention_generic_kernel<bf16>, p);
  } else if (dtype == JX_F32) {
    if (smem > 48 * 1024)
      cudaFuncSetAttribute(attention_generic_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    err = launch_ex(&cfg, attention_generic_kernel<float>, p);
  } else {
    return JX_ERR_DTYPE;
  }
  return err == cudaSuccess ? JX_OK : JX_ERR_CUDA;
}

}  // namespace jxb
