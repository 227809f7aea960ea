// On-device token selection and end-of-step bookkeeping.
//
// Greedy (sampling.py:75-77): first index of the maximum of the model-dtype logits.
// Temperature (sampling.py:181-186): jax.random.categorical(subkey, logits / temp) =
// argmax(gumbel + dtype(logits / dtype(temp))), the Gumbel draw of flat element b*V + v coming from
// threefry2x32(subkey, (hi, lo) of that index) (JAX's partitionable threefry: 32-bit draw x0 ^ x1;
// a bfloat16 uniform keeps its low 8 bits, whose top 7 become the mantissa).  The 256 possible
// bfloat16 Gumbel values are a table computed on the host.
//
// The row finisher writes the token, the next decode input and (decode) advances pos_id / mask by one
// (cache.py:237-243); the last row finisher advances the step counter and splits the key for the next
// step (jax.random.split, _generate.py:205), so a captured step graph needs no host work.
#include "common.cuh"

namespace jxb {

__device__ __forceinline__ uint32_t rotl32(uint32_t x, int r) { return (x << r) | (x >> (32 - r)); }

// Threefry-2x32, 20 rounds (Salmon et al., SC'11).
__device__ __forceinline__ void threefry2x32(uint32_t k0, uint32_t k1, uint32_t& x0, uint32_t& x1) {
  const uint32_t ks[3] = {k0, k1, k0 ^ k1 ^ 0x1BD11BDAu};
  const int rot[2][4] = {{13, 15, 26, 6}, {17, 29, 16, 24}};
  x0 += ks[0];
  x1 += ks[1];
#pragma unroll
  for (int g = 0; g < 5; ++g) {
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      x0 += x1;
      x1 = rotl32(x1, rot[g & 1][r]);
      x1 ^= x0;
    }
    x0 += ks[(g + 1) % 3];
    x1 += ks[(g + 2) % 3] + (uint32_t)(g + 1);
  }
}

__device__ __forceinline__ unsigned long long order_key(float v, long long idx) {
  uint32_t b = __float_as_uint(v);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((unsigned long long)b << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)idx);
}

typedef jx_sample_args SampleArgs;

__device__ void finish_row(const SampleArgs& p, int b, unsigned long long best) {
  const int token = (int)(0xFFFFFFFFu - (uint32_t)(best & 0xFFFFFFFFull));
  const int col = p.step ? *p.step : 0;
  if (p.tokens_out) {
    if (col >= 0 && col < p.ld_tok)
      p.tokens_out[(long long)b * p.ld_tok + col] = token;
    else
      set_status(p.status, JX_ERR_RANGE);
  }
  if (p.next_ids) p.next_ids[b] = token;
  if (p.update_pos && p.pos_id) {
    const int np = p.pos_id[b] + 1;
    p.pos_id[b] = np;
    if (p.mask && np < p.T_mask) p.mask[(long long)b * p.T_mask + np] = 1;
  }
}

__device__ void finish_step(const SampleArgs& p) {
  if (p.step) *p.step += 1;
  if (p.advance_rng && p.rng) {
    uint32_t a0 = 0, a1 = 0, b0 = 0, b1 = 1;
    threefry2x32(p.rng[0], p.rng[1], a0, a1);
    threefry2x32(p.rng[0], p.rng[1], b0, b1);
    p.rng[0] = a0;
    p.rng[1] = a1;
    p.rng[2] = b0;
    p.rng[3] = b1;
  }
}

template <typename T>
__global__ void __launch_bounds__(256) sample_kernel(SampleArgs p) {
  __shared__ unsigned long long red[8];
  __shared__ int last_flag;
  const int b = blockIdx.y, cidx = blockIdx.x;
  const int nchunks = gridDim.x;
  pdl_trigger();
  pdl_wait();
  const T* row = reinterpret_cast<const T*>(p.logits) + (long long)b * p.ld;
  const int v0 = cidx * p.chunk, v1 = min(p.V, v0 + p.chunk);
  const uint32_t s0 = p.rng ? p.rng[2] : 0u, s1 = p.rng ? p.rng[3] : 0u;
  const bool is_bf16 = p.dtype == JX_BF16;
  const float temp_t = is_bf16 ? rnd<bf16>(p.temp) : p.temp;
  unsigned long long best = 0ull;
  for (int v = v0 + threadIdx.x; v < v1; v += 256) {
    const float l = to_f(row[v]);
    const long long gidx = p.vocab_offset + v;
    float t;
    if (p.greedy) {
      t = l;
    } else {
      const unsigned long long flat = (unsigned long long)b * (unsigned long long)p.vocab_total + gidx;
      uint32_t x0 = (uint32_t)(flat >> 32), x1 = (uint32_t)(flat & 0xFFFFFFFFull);
      threefry2x32(s0, s1, x0, x1);
      const uint32_t bits = x0 ^ x1;
      if (is_bf16) {
        const float scaled = rnd<bf16>(l / temp_t);
        t = rnd<bf16>(p.gumbel_tab[bits & 0xFFu] + scaled);
      } else {
        float u = __uint_as_float((bits >> 9) | 0x3F800000u) - 1.0f;
        const float tiny = 1.17549435e-38f;
        u = fmaxf(u + tiny, tiny);
        const float l1 = (float)log((double)u);
        const float g = -(float)log((double)(-l1));
        t = g + l / p.temp;
      }
    }
    const unsigned long long k = order_key(t, gidx);
    best = k > best ? k : best;
  }
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
    best = other > best ? other : best;
  }
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < 8; ++w) best = red[w] > best ? red[w] : best;
    p.ws[(long long)b * nchunks + cidx] = best;
    __threadfence();
    const int prev = atomicAdd(&p.counters[b], 1);
    last_flag = (prev == nchunks - 1);
  }
  __syncthreads();
  if (!last_flag || threadIdx.x != 0) return;
  __threadfence();
  unsigned long long rb = 0ull;
  for (int c = 0; c < nchunks; ++c) {
    const unsigned long long k = __ldcg(&p.ws[(long long)b * nchunks + c]);
    rb = k > rb ? k : rb;
  }
  p.counters[b] = 0;
  if (!p.finalize) {
    p.row_best[b] = rb;
    return;
  }
  finish_row(p, b, rb);
  __threadfence();
  const int done = atomicAdd(&p.counters[p.B], 1);
  if (done == p.B - 1) {
    p.counters[p.B] = 0;
    finish_step(p);
  }
}

// Combine per-shard (value, index) keys gathered from the tensor-parallel ranks: [n_shards, B].
__global__ void sample_finalize_kernel(SampleArgs p, const unsigned long long* gathered, int n_shards) {
  pdl_wait();
  const int b = threadIdx.x;
  if (b < p.B) {
    unsigned long long rb = 0ull;
    for (int r = 0; r < n_shards; ++r) {
      const unsigned long long k = gathered[(long long)r * p.B + b];
      rb = k > rb ? k : rb;
    }
    finish_row(p, b, rb);
  }
  __syncthreads();
  if (threadIdx.x == 0) finish_step(p);
}

int run_sample(const SampleArgs& p, bool pdl, cudaStream_t stream) {
  if (p.B <= 0 || p.V <= 0 || p.chunk <= 0) return JX_ERR_SHAPE;
  const int nchunks = (p.V + p.chunk - 1) / p.chunk;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nchunks, p.B);
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t err;
  if (p.dtype == JX_BF16)
    err = launch_ex(&cfg, sample_kernel<bf16>, p);
  else if (p.dtype == JX_F32)
    err = launch_ex(&cfg, sample_kernel<float>, p);
  else
    return JX_ERR_DTYPE;
  return err == cudaSuccess ? JX_OK : JX_ERR_CUDA;
}

int run_sample_finalize(const SampleArgs& p, const unsigned long long* gathered, int n_shards, cudaStream_t stream) {
  if (p.B <= 0 || p.B > 1024) return JX_ERR_SHAPE;
  sample_finalize_kernel<<<1, ((p.B + 31) / 32) * 32, 0, stream>>>(p, gathered, n_shards);
  return cudaGetLastError() == cudaSuccess ? JX_OK : JX_ERR_CUDA;
}

}  // namespace jxb
