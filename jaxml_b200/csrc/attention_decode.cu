// GQA decode attention on tensor cores (bfloat16, head_dim 64 / 128 / 256), split over the key axis.
//
// Reproduces Attention.mha for one query token per row (nn/attention.py:321-400, decode branch): for
// the n_rep = Hq/Hkv query heads of one KV head (repeat_kv by indexing, :294-319)
//   s_t = bf16(bf16(q . k_t) * bf16(attn_scale))                      (einsum output and scale in dtype)
//   keys: t < len (prefix padding mask) and, for sliding-window layers, t >= len - window
//   p_t = bf16(exp(s_t - max) / sum exp(s - max))                     (float32 softmax, cast to dtype)
//   o   = bf16(sum_t p_t v_t)                                          (float32 accumulation)
// Only the valid (or in-window) keys are read, not the whole padded buffer.
//
// Two forms.  The single-pass cluster form (dattn_fused_kernel, below) covers key ranges up to 8 CTAs x
// 1024 keys per (row, KV head) and is selected explicitly.  The default split form runs two kernels per
// layer, each a grid of (key split, KV head, batch row) CTAs of 128 keys:
//   scores: K tiles arrive by TMA (2-D tensor map over the [L*B*T, Hkv*hd] cache, 128-byte swizzle);
//           Q.K^T on mma.sync; the rounded scores go to a float32 workspace with per-split (max, sum).
//   pv:     combines the split statistics into the exact softmax normaliser, forms the bf16
//           probabilities, P.V on mma.sync with V tiles by TMA, and the last CTA of a head group sums
//           the split partials in split order (deterministic) into the bf16 output (K128 layout).
#include <cudaTypedefs.h>

#include "common.cuh"

namespace jxb {

constexpr int kDaKeys = 128;        // keys per CTA
constexpr int kDaTile = 64;         // keys per TMA tile
constexpr int kPLd = kDaKeys + 8;   // padded row stride (bf16) of the probability tile: conflict-free ldmatrix

struct DAttnParams {
  int B, Hq, Hkv, n_rep, T, n_splits;
  long long layer_row0;
  const bf16* q;         // [B, Hq, HD]
  const int* len_ptr;
  int len_add, window;
  float scale_bf16;      // attn_scale rounded to bf16
  bf16* out;
  long long out_rp;
  float* sc;             // [B, Hq, T]
  float* stats;          // [B, Hq, n_splits, 2]
  float* opart;          // [B, Hq, n_splits, HD]
  int* counters;         // [B * Hkv]
  int* status;
};

// Address of the 16-byte chunk `c` (8 bf16 columns) of row r in a [rows x 64] block stored with the
// 128-byte swizzle (chunk index XOR row % 8), the layout TMA writes with CU_TENSOR_MAP_SWIZZLE_128B.
__device__ __forceinline__ uint32_t swz(uint32_t block_base, int r, int c) {
  return block_base + r * 128 + ((c ^ (r & 7)) << 4);
}

__device__ __forceinline__ void key_range(const DAttnParams& p, int b, int& lo, int& valid) {
  valid = p.len_ptr[b] + p.len_add;
  if (valid > p.T) {
    set_status(p.status, JX_ERR_RANGE);
    valid = p.T;
  }
  lo = (p.window > 0 && valid > p.window) ? valid - p.window : 0;
}

template <int HD>
__global__ void __launch_bounds__(128) dattn_scores_kernel(const __grid_constant__ CUtensorMap kmap, DAttnParams p) {
  constexpr int NB = HD / 64;                 // 64-column blocks per head
  constexpr int TILE_BYTES = kDaTile * HD * 2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ktile = smem;                                   // 2 tiles, each NB blocks of [64 x 64]
  uint8_t* qs = smem + 2 * TILE_BYTES;                     // NB blocks of [16 x 64]
  uint64_t* bar = reinterpret_cast<uint64_t*>(qs + NB * 2048);
  float* red = reinterpret_cast<float*>(bar + 2);          // [4 warps][16 rows]

  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_trigger();
  pdl_wait();
  int lo, valid;
  key_range(p, b, lo, valid);
  const int t0 = lo + split * kDaKeys;
  if (t0 >= valid) return;
  const int t1 = min(t0 + kDaKeys, valid);
  const int n_tiles = (t1 - t0 + kDaTile - 1) / kDaTile;
  if (threadIdx.x == 0) {
    prefetch_tmap(&kmap);
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    fence_barrier_init();
    for (int i = 0; i < n_tiles; ++i) {
      mbar_arrive_expect_tx(&bar[i], TILE_BYTES);
      const int y = (int)(p.layer_row0 + (long long)b * p.T + t0 + i * kDaTile);
#pragma unroll
      for (int c = 0; c < NB; ++c) tma_load_2d(ktile + i * TILE_BYTES + c * 8192, &kmap, kvh * HD + c * 64, y, &bar[i]);
    }
  }
  // Q rows of this head group (rows >= n_rep are zero) into the swizzled layout.
  for (int idx = threadIdx.x; idx < 16 * (HD / 8); idx += 128) {
    const int r = idx / (HD / 8), cg = idx % (HD / 8);
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < p.n_rep)
      v = *reinterpret_cast<const uint4*>(p.q + ((long long)b * p.Hq + kvh * p.n_rep + r) * HD + cg * 8);
    const uint32_t a = swz(smem_u32(qs + (cg >> 3) * 2048), r, cg & 7);
    asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(a), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w));
  }
  __syncthreads();

  const int mi = lane >> 3, r8 = lane & 7;
  float s[2][2][4];          // [tile][n8 tile][frag]
  float mrow[2] = {-INFINITY, -INFINITY};   // rows lane/4 and lane/4 + 8
  bool ok = true;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[i][nt][e] = -INFINITY;
    if (i >= n_tiles || !ok) continue;
    if (!mbar_wait_bounded(&bar[i], 0)) {
      set_status(p.status, JX_ERR_TIMEOUT);
      ok = false;
      continue;
    }
    float acc[2][4] = {};
    const uint32_t kb = smem_u32(ktile + i * TILE_BYTES);
#pragma unroll
    for (int ks = 0; ks < HD / 16; ++ks) {
      uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
      {
        const int row = (mi & 1) * 8 + r8, ch = ks * 2 + (mi >> 1);
        ldsm_x4(swz(smem_u32(qs + (ch >> 3) * 2048), row, ch & 7), a0, a1, a2, a3);
      }
      {
        const int row = warp * 16 + (mi >> 1) * 8 + r8, ch = ks * 2 + (mi & 1);
        ldsm_x4(swz(kb + (ch >> 3) * 8192, row, ch & 7), b0, b1, b2, b3);
      }
      mma_bf16(acc[0], a0, a1, a2, a3, b0, b1);
      mma_bf16(acc[1], a0, a1, a2, a3, b2, b3);
    }
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int t = t0 + i * kDaTile + warp * 16 + nt * 8 + (lane & 3) * 2 + (e & 1);
        if (t < t1) {
          const float v = rnd<bf16>(rnd<bf16>(acc[nt][e]) * p.scale_bf16);
          s[i][nt][e] = v;
          mrow[e >> 1] = fmaxf(mrow[e >> 1], v);
        }
      }
  }
  if (!__syncthreads_and(ok)) return;
  // row maxima over the CTA
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    mrow[h] = fmaxf(mrow[h], __shfl_xor_sync(0xffffffffu, mrow[h], 1));
    mrow[h] = fmaxf(mrow[h], __shfl_xor_sync(0xffffffffu, mrow[h], 2));
  }
  if ((lane & 3) == 0) {
    red[warp * 16 + (lane >> 2)] = mrow[0];
    red[warp * 16 + (lane >> 2) + 8] = mrow[1];
  }
  __syncthreads();
  float m[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int row = (lane >> 2) + h * 8;
    m[h] = fmaxf(fmaxf(red[row], red[16 + row]), fmaxf(red[32 + row], red[48 + row]));
  }
  __syncthreads();
  float l[2] = {0.f, 0.f};
  const long long sc_row = ((long long)b * p.Hq + kvh * p.n_rep) * p.T;
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int row = (lane >> 2) + (e >> 1) * 8;
        const int t = t0 + i * kDaTile + warp * 16 + nt * 8 + (lane & 3) * 2 + (e & 1);
        if (t < t1 && row < p.n_rep) {
          const float v = s[i][nt][e];
          p.sc[sc_row + (long long)row * p.T + t] = v;
          l[e >> 1] += expf(v - m[e >> 1]);
        }
      }
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    l[h] += __shfl_xor_sync(0xffffffffu, l[h], 1);
    l[h] += __shfl_xor_sync(0xffffffffu, l[h], 2);
  }
  if ((lane & 3) == 0) {
    red[warp * 16 + (lane >> 2)] = l[0];
    red[warp * 16 + (lane >> 2) + 8] = l[1];
  }
  __syncthreads();
  // (max, sum) of this split for each query row: warp 0's lanes with lane % 4 == 0 own rows lane/4, +8
  if (warp == 0 && (lane & 3) == 0) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int row = (lane >> 2) + h * 8;
      if (row < p.n_rep) {
        float* st = p.stats + (((long long)b * p.Hq + kvh * p.n_rep + row) * p.n_splits + split) * 2;
        st[0] = m[h];
        st[1] = (red[row] + red[16 + row]) + (red[32 + row] + red[48 + row]);
      }
    }
  }
}

template <int HD>
__global__ void __launch_bounds__(128) dattn_pv_kernel(const __grid_constant__ CUtensorMap vmap, DAttnParams p) {
  constexpr int NB = HD / 64;
  constexpr int TILE_BYTES = kDaTile * HD * 2;
  constexpr int WCOLS = HD / 4;             // output columns per warp
  constexpr int NT = WCOLS / 8;             // n8 tiles per warp
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* vtile = smem;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + 2 * TILE_BYTES);
  float* Ms = reinterpret_cast<float*>(bar + 2);   // [16]
  float* Ls = Ms + 16;                             // [16]
  bf16* ptile = reinterpret_cast<bf16*>(Ls + 16);  // [16][kPLd]
  __shared__ int last_flag;

  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_trigger();
  pdl_wait();
  int lo, valid;
  key_range(p, b, lo, valid);
  const int t0 = lo + split * kDaKeys;
  const int n_active = (valid - lo + kDaKeys - 1) / kDaKeys;
  if (t0 >= valid) return;
  const int t1 = min(t0 + kDaKeys, valid);
  const int n_tiles = (t1 - t0 + kDaTile - 1) / kDaTile;
  if (threadIdx.x == 0) {
    prefetch_tmap(&vmap);
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    fence_barrier_init();
    for (int i = 0; i < n_tiles; ++i) {
      mbar_arrive_expect_tx(&bar[i], TILE_BYTES);
      const int y = (int)(p.layer_row0 + (long long)b * p.T + t0 + i * kDaTile);
#pragma unroll
      for (int c = 0; c < NB; ++c) tma_load_2d(vtile + i * TILE_BYTES + c * 8192, &vmap, kvh * HD + c * 64, y, &bar[i]);
    }
  }
  // exact softmax normaliser of each row from the split statistics
  if (threadIdx.x < 16) {
    const int row = threadIdx.x;
    float M = -INFINITY, L = 0.f;
    if (row < p.n_rep) {
      const float* st = p.stats + ((long long)b * p.Hq + kvh * p.n_rep + row) * p.n_splits * 2;
      for (int s2 = 0; s2 < n_active; ++s2) M = fmaxf(M, st[s2 * 2]);
      for (int s2 = 0; s2 < n_active; ++s2) L += st[s2 * 2 + 1] * expf(st[s2 * 2] - M);
    }
    Ms[row] = M;
    Ls[row] = L;
  }
  __syncthreads();

  const int mi = lane >> 3, r8 = lane & 7;
  const int r_lo = lane >> 2, r_hi = r_lo + 8;
  // Probabilities of this CTA's keys, computed once (coalesced score reads) into a padded bf16 tile
  // [16 rows][kDaKeys + 8] that every warp reads with ldmatrix.
  for (int idx = threadIdx.x; idx < 16 * kDaKeys; idx += 128) {
    const int row = idx / kDaKeys, k = idx % kDaKeys, t = t0 + k;
    float pv = 0.f;
    if (row < p.n_rep && t < t1) {
      const float s = __ldcg(p.sc + ((long long)b * p.Hq + kvh * p.n_rep + row) * p.T + t);
      pv = rnd<bf16>(expf(s - Ms[row]) / Ls[row]);
    }
    ptile[row * kPLd + k] = __float2bfloat16_rn(pv);
  }
  __syncthreads();
  float acc[NT][4] = {};
  bool ok = true;
  for (int i = 0; i < n_tiles && ok; ++i) {
    if (!mbar_wait_bounded(&bar[i], 0)) {
      set_status(p.status, JX_ERR_TIMEOUT);
      ok = false;
      continue;
    }
    const uint32_t vb = smem_u32(vtile + i * TILE_BYTES);
#pragma unroll
    for (int kk = 0; kk < kDaTile / 16; ++kk) {
      uint32_t a0, a1, a2, a3;
      {
        const int row = (mi & 1) * 8 + r8, col = i * kDaTile + kk * 16 + (mi >> 1) * 8;
        ldsm_x4(smem_u32(ptile + row * kPLd + col), a0, a1, a2, a3);
      }
#pragma unroll
      for (int n16 = 0; n16 < NT / 2; ++n16) {
        uint32_t b0, b1, b2, b3;
        const int row = kk * 16 + (mi & 1) * 8 + r8;
        const int ch = (warp * WCOLS) / 8 + n16 * 2 + (mi >> 1);
        ldsm_x4_t(swz(vb + (ch >> 3) * 8192, row, ch & 7), b0, b1, b2, b3);
        mma_bf16(acc[n16 * 2], a0, a1, a2, a3, b0, b1);
        mma_bf16(acc[n16 * 2 + 1], a0, a1, a2, a3, b2, b3);
      }
    }
  }
  if (!__syncthreads_and(ok)) return;
  // split partial -> workspace
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int row = (e >> 1) ? r_hi : r_lo;
      const int col = warp * WCOLS + nt * 8 + (lane & 3) * 2 + (e & 1);
      if (row < p.n_rep)
        p.opart[(((long long)b * p.Hq + kvh * p.n_rep + row) * p.n_splits + split) * HD + col] = acc[nt][e];
    }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int prev = atomicAdd(&p.counters[b * p.Hkv + kvh], 1);
    last_flag = (prev == n_active - 1);
  }
  __syncthreads();
  if (!last_flag) return;
  __threadfence();
  for (int idx = threadIdx.x; idx < p.n_rep * HD; idx += 128) {
    const int row = idx / HD, col = idx % HD;
    const float* src = p.opart + (((long long)b * p.Hq + kvh * p.n_rep + row) * p.n_splits) * HD + col;
    float sum = 0.f;
    for (int s2 = 0; s2 < n_active; ++s2) sum += __ldcg(src + (long long)s2 * HD);
    const long long ocol = (long long)(kvh * p.n_rep + row) * HD + col;
    p.out[k128_offset(b, ocol, p.out_rp)] = __float2bfloat16_rn(sum);
  }
  if (threadIdx.x == 0) p.counters[b * p.Hkv + kvh] = 0;
}

// ------------------------------------------------------------------------------------------------
// Single-pass form: one thread-block cluster per (batch row, KV head), its CS CTAs splitting the key
// range into contiguous runs of 64-key tiles.  Every CTA issues its K and V tiles at once (one
// memory round trip when they fit the ring), keeps its rounded scores in shared memory, and the
// cluster exchanges the per-row maxima and exp-sums through distributed shared memory, so each CTA
// forms the exact probabilities bf16(exp(s - max) / sum) itself.  The partial outputs sum_t p_t v_t
// are added across the cluster in rank order (deterministic) by the CTA that owns each column slice.
// ------------------------------------------------------------------------------------------------
constexpr int kFaKT = 64;                 // keys per tile
constexpr int kFaMaxTiles = 16;           // tiles per CTA this form holds scores for (1024 keys)
constexpr int kFaPLd = kFaKT + 8;         // padded bf16 row stride of the probability tile

struct FAttnParams {
  int B, Hq, Hkv, n_rep, T, window;
  int kt_cap;            // tiles per CTA the shared memory was sized for
  int n_stages;          // ring stages
  long long layer_row0;
  const bf16* q;         // [B, Hq, HD]
  const int* len_ptr;
  int len_add;
  float scale_bf16;
  bf16* out;
  long long out_rp;
  int* status;
};

template <int HD>
struct FaSmem {
  static constexpr int NB = HD / 64;
  static constexpr int kTileBytes = kFaKT * HD * 2;
  // byte offsets from the 1024-aligned base; `kt` = tiles per CTA, `ns` = ring stages
  static __host__ __device__ int q_off(int ns) { return ns * kTileBytes; }
  static __host__ __device__ int sc_off(int ns) { return q_off(ns) + NB * 2048; }
  static __host__ __device__ int sc_ld(int kt) { return kt * kFaKT + 8; }
  static __host__ __device__ int p_off(int ns, int kt) { return sc_off(ns) + 16 * sc_ld(kt) * 2; }
  static __host__ __device__ int red_off(int ns, int kt) { return p_off(ns, kt) + 16 * kFaPLd * 2; }
  static __host__ __device__ int bar_off(int ns, int kt) { return red_off(ns, kt) + (64 + 16 + 16 + 16 + 16) * 4; }
  static __host__ __device__ int bytes(int ns, int kt) { return 1024 + bar_off(ns, kt) + ns * 8 + 16; }
};

template <int HD>
__global__ void __launch_bounds__(128) dattn_fused_kernel(const __grid_constant__ CUtensorMap kmap,
                                                          const __grid_constant__ CUtensorMap vmap, FAttnParams p) {
  using S = FaSmem<HD>;
  constexpr int NB = S::NB;
  constexpr int WCOLS = HD / 4;
  constexpr int NT = WCOLS / 8;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int ns = p.n_stages, kt_cap = p.kt_cap;
  uint8_t* ring = smem;
  uint8_t* qs = smem + S::q_off(ns);
  bf16* sc = reinterpret_cast<bf16*>(smem + S::sc_off(ns));
  const int sc_ld = S::sc_ld(kt_cap);
  bf16* ptile = reinterpret_cast<bf16*>(smem + S::p_off(ns, kt_cap));
  float* red = reinterpret_cast<float*>(smem + S::red_off(ns, kt_cap));   // [4 warps][16]
  float* cmax = red + 64;        // [16] this CTA's row maxima (read by the cluster)
  float* csum = cmax + 16;       // [16] this CTA's row exp-sums (read by the cluster)
  float* Mrow = csum + 16;       // [16] cluster row maxima
  float* Lrow = Mrow + 16;       // [16] cluster row sums
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::bar_off(ns, kt_cap));
  float* opart = reinterpret_cast<float*>(ring);   // [16][HD], reuses the ring once every tile is consumed

  const int CS = gridDim.x;
  const uint32_t rank = cluster_ctarank();
  const int kvh = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_wait();

  int valid = p.len_ptr[b] + p.len_add;
  if (valid > p.T) {
    set_status(p.status, JX_ERR_RANGE);
    valid = p.T;
  }
  const int lo = (p.window > 0 && valid > p.window) ? valid - p.window : 0;
  const int n_tiles = valid > lo ? (valid - lo + kFaKT - 1) / kFaKT : 0;
  int tpc = (n_tiles + CS - 1) / CS;
  if (tpc > kt_cap) {
    set_status(p.status, JX_ERR_RANGE);
    tpc = kt_cap;
  }
  const int my0 = (int)rank * tpc;
  const int my_n = max(0, min(tpc, n_tiles - my0));       // tiles of this CTA
  const int key0 = lo + my0 * kFaKT;                       // first key of this CTA
  const int n_loads = 2 * my_n;                            // K tiles, then V tiles
  const long long row0 = p.layer_row0 + (long long)b * p.T;

  auto issue = [&](int ld) {
    const int s = ld % ns;
    const bool is_v = ld >= my_n;
    const int i = is_v ? ld - my_n : ld;
    mbar_arrive_expect_tx(&full[s], S::kTileBytes);
    const int y = (int)(row0 + key0 + i * kFaKT);
#pragma unroll
    for (int c = 0; c < NB; ++c)
      tma_load_2d(ring + s * S::kTileBytes + c * 8192, is_v ? &vmap : &kmap, kvh * HD + c * 64, y, &full[s]);
  };
  if (threadIdx.x == 0) {
    prefetch_tmap(&kmap);
    prefetch_tmap(&vmap);
    for (int s = 0; s < ns; ++s) mbar_init(&full[s], 1);
    fence_barrier_init();
    for (int ld = 0; ld < min(ns, n_loads); ++ld) issue(ld);
  }
  pdl_trigger();
  // Q rows of this head group (rows >= n_rep are zero) into the swizzled layout.
  for (int idx = threadIdx.x; idx < 16 * (HD / 8); idx += 128) {
    const int r = idx / (HD / 8), cg = idx % (HD / 8);
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < p.n_rep) v = *reinterpret_cast<const uint4*>(p.q + ((long long)b * p.Hq + kvh * p.n_rep + r) * HD + cg * 8);
    const uint32_t a = swz(smem_u32(qs + (cg >> 3) * 2048), r, cg & 7);
    asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(a), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w));
  }
  __syncthreads();

  const int mi = lane >> 3, r8 = lane & 7;
  bool ok = true;
  float mrow[2] = {-INFINITY, -INFINITY};   // rows lane/4 and lane/4 + 8
  // ---- scores of this CTA's keys ----
  for (int i = 0; i < my_n; ++i) {
    const int s = i % ns;
    if (ok && !mbar_wait_bounded(&full[s], (i / ns) & 1)) {
      set_status(p.status, JX_ERR_TIMEOUT);
      ok = false;
    }
    float acc[2][4] = {};
    if (ok) {
      const uint32_t kb = smem_u32(ring + s * S::kTileBytes);
#pragma unroll
      for (int ks = 0; ks < HD / 16; ++ks) {
        uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
        {
          const int row = (mi & 1) * 8 + r8, ch = ks * 2 + (mi >> 1);
          ldsm_x4(swz(smem_u32(qs + (ch >> 3) * 2048), row, ch & 7), a0, a1, a2, a3);
        }
        {
          const int row = warp * 16 + (mi >> 1) * 8 + r8, ch = ks * 2 + (mi & 1);
          ldsm_x4(swz(kb + (ch >> 3) * 8192, row, ch & 7), b0, b1, b2, b3);
        }
        mma_bf16(acc[0], a0, a1, a2, a3, b0, b1);
        mma_bf16(acc[1], a0, a1, a2, a3, b2, b3);
      }
    }
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int kl = warp * 16 + nt * 8 + (lane & 3) * 2 + (e & 1);   // key within the tile
        const int row = (lane >> 2) + (e >> 1) * 8;
        float v = -INFINITY;
        if (key0 + i * kFaKT + kl < valid) {
          v = rnd<bf16>(rnd<bf16>(acc[nt][e]) * p.scale_bf16);
          mrow[e >> 1] = fmaxf(mrow[e >> 1], v);
        }
        sc[row * sc_ld + i * kFaKT + kl] = __float2bfloat16_rn(v);
      }
    __syncthreads();   // every warp is done with stage s
    if (threadIdx.x == 0 && i + ns < n_loads) issue(i + ns);
  }
  // ---- cluster row maxima ----
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    mrow[h] = fmaxf(mrow[h], __shfl_xor_sync(0xffffffffu, mrow[h], 1));
    mrow[h] = fmaxf(mrow[h], __shfl_xor_sync(0xffffffffu, mrow[h], 2));
  }
  if ((lane & 3) == 0) {
    red[warp * 16 + (lane >> 2)] = mrow[0];
    red[warp * 16 + (lane >> 2) + 8] = mrow[1];
  }
  __syncthreads();
  if (threadIdx.x < 16) {
    const int r = threadIdx.x;
    cmax[r] = fmaxf(fmaxf(red[r], red[16 + r]), fmaxf(red[32 + r], red[48 + r]));
  }
  cluster_sync_all();
  if (threadIdx.x < 16) {
    const int r = threadIdx.x;
    float M = -INFINITY;
    for (int cr = 0; cr < CS; ++cr) M = fmaxf(M, dsmem_ld_f32(dsmem_map(smem_u32(cmax + r), cr)));
    Mrow[r] = M;
  }
  __syncthreads();
  // ---- cluster row sums of exp(s - max): warp w sums rows 4w .. 4w+3 over this CTA's keys ----
  const int my_keys = max(0, min(my_n * kFaKT, valid - key0));
#pragma unroll
  for (int rr = 0; rr < 4; ++rr) {
    const int r = warp * 4 + rr;
    const float M = Mrow[r];
    float l = 0.f;
    if (r < p.n_rep && M != -INFINITY)
      for (int k = lane; k < my_keys; k += 32) l += expf(__bfloat162float(sc[r * sc_ld + k]) - M);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    if (lane == 0) csum[r] = l;
  }
  cluster_sync_all();
  if (threadIdx.x < 16) {
    const int r = threadIdx.x;
    float L = 0.f;
    for (int cr = 0; cr < CS; ++cr) L += dsmem_ld_f32(dsmem_map(smem_u32(csum + r), cr));
    Lrow[r] = L;
  }
  __syncthreads();

  // ---- P . V over this CTA's keys ----
  float acc[NT][4] = {};
  for (int i = 0; i < my_n; ++i) {
    for (int idx = threadIdx.x; idx < 16 * kFaKT; idx += 128) {
      const int r = idx / kFaKT, k = idx % kFaKT;
      float pv = 0.f;
      const float M = Mrow[r], L = Lrow[r];
      if (r < p.n_rep && key0 + i * kFaKT + k < valid && M != -INFINITY && L > 0.f)
        pv = rnd<bf16>(expf(__bfloat162float(sc[r * sc_ld + i * kFaKT + k]) - M) / L);
      ptile[r * kFaPLd + k] = __float2bfloat16_rn(pv);
    }
    __syncthreads();
    const int ld = my_n + i, s = ld % ns;
    if (ok && !mbar_wait_bounded(&full[s], (ld / ns) & 1)) {
      set_status(p.status, JX_ERR_TIMEOUT);
      ok = false;
    }
    if (ok) {
      const uint32_t vb = smem_u32(ring + s * S::kTileBytes);
#pragma unroll
      for (int kk = 0; kk < kFaKT / 16; ++kk) {
        uint32_t a0, a1, a2, a3;
        {
          const int row = (mi & 1) * 8 + r8, col = kk * 16 + (mi >> 1) * 8;
          ldsm_x4(smem_u32(ptile + row * kFaPLd + col), a0, a1, a2, a3);
        }
#pragma unroll
        for (int n16 = 0; n16 < NT / 2; ++n16) {
          uint32_t b0, b1, b2, b3;
          const int row = kk * 16 + (mi & 1) * 8 + r8;
          const int ch = (warp * WCOLS) / 8 + n16 * 2 + (mi >> 1);
          ldsm_x4_t(swz(vb + (ch >> 3) * 8192, row, ch & 7), b0, b1, b2, b3);
          mma_bf16(acc[n16 * 2], a0, a1, a2, a3, b0, b1);
          mma_bf16(acc[n16 * 2 + 1], a0, a1, a2, a3, b2, b3);
        }
      }
    }
    __syncthreads();   // stage s and the probability tile are free again
    if (threadIdx.x == 0 && ld + ns < n_loads) issue(ld + ns);
  }
  // ---- partial outputs -> shared memory (the ring is idle: every issued tile has been consumed) ----
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int row = (lane >> 2) + (e >> 1) * 8;
      const int col = warp * WCOLS + nt * 8 + (lane & 3) * 2 + (e & 1);
      opart[row * HD + col] = acc[nt][e];
    }
  cluster_sync_all();
  // ---- each CTA sums one slice of the [n_rep, HD] output over the cluster, in rank order ----
  const int total = p.n_rep * HD;
  const int chunk = (total + CS - 1) / CS;
  const int e0 = (int)rank * chunk, e1 = min(total, e0 + chunk);
  for (int idx = e0 + threadIdx.x; idx < e1; idx += 128) {
    const uint32_t la = smem_u32(opart + idx);
    float sum = 0.f;
    for (int cr = 0; cr < CS; ++cr) sum += dsmem_ld_f32(dsmem_map(la, cr));
    const int row = idx / HD, col = idx % HD;
    const long long ocol = (long long)(kvh * p.n_rep + row) * HD + col;
    p.out[k128_offset(b, ocol, p.out_rp)] = __float2bfloat16_rn(sum);
  }
  cluster_sync_all();   // no CTA leaves while another may still read its shared memory
}

// ------------------------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// 2-D bf16 tensor map over a row-major [rows, cols] matrix with a [box_rows x 64] box and 128-byte swizzle.
int make_tmap_2d_bf16_box(CUtensorMap* map, const void* base, long long rows, long long cols,
                          long long row_stride_elems, int box_rows) {
  auto enc = tmap_encoder();
  if (!enc) return JX_ERR_CUDA;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || ((row_stride_elems * 2) & 15) || cols % 64) return JX_ERR_ARG;
  if (box_rows <= 0 || box_rows > 256) return JX_ERR_ARG;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(row_stride_elems * 2)};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? JX_OK : JX_ERR_ARG;
}

int make_tmap_2d_bf16(CUtensorMap* map, const void* base, long long rows, long long cols, long long row_stride_elems) {
  return make_tmap_2d_bf16_box(map, base, rows, cols, row_stride_elems, 64);
}

long long dattn_workspace_bytes(int B, int Hq, int T, int hd, int n_splits) {
  const long long sc = (long long)B * Hq * T;
  const long long st = (long long)B * Hq * n_splits * 2;
  const long long op = (long long)B * Hq * n_splits * hd;
  return (sc + st + op) * 4;
}

int dattn_n_splits(int T, int window) {
  const int range = (window > 0 && window < T) ? window : T;
  return (range + kDaKeys - 1) / kDaKeys;
}

template <int HD>
static int launch_dattn(const CUtensorMap& km, const CUtensorMap& vm, const DAttnParams& p, bool pdl, cudaStream_t s) {
  const int smem_a = 1024 + 2 * kDaTile * HD * 2 + (HD / 64) * 2048 + 16 + 4 * 16 * 4;
  const int smem_b = 1024 + 2 * kDaTile * HD * 2 + 16 + 32 * 4 + 16 * kPLd * 2;
  static bool configured = false;
  if (!configured) {
    if (cudaFuncSetAttribute(dattn_scores_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_a) != cudaSuccess ||
        cudaFuncSetAttribute(dattn_pv_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_b) != cudaSuccess)
      return JX_ERR_CUDA;
    configured = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.n_splits, p.Hkv, p.B);
  cfg.blockDim = dim3(128);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cfg.dynamicSmemBytes = smem_a;
  if (cudaLaunchKernelEx(&cfg, dattn_scores_kernel<HD>, km, p) != cudaSuccess) return JX_ERR_CUDA;
  cfg.dynamicSmemBytes = smem_b;
  if (cudaLaunchKernelEx(&cfg, dattn_pv_kernel<HD>, vm, p) != cudaSuccess) return JX_ERR_CUDA;
  return JX_OK;
}

// Cluster shape of the single-pass form for a key range of `range` keys: up to 8 CTAs of up to
// kFaMaxTiles 64-key tiles each.  Returns false when the range needs more (the split form runs then).
static bool fused_shape(int range, int hd, int& cs, int& kt, int& ns) {
  const int n128 = (range + 127) / 128;
  cs = n128 < 1 ? 1 : (n128 > 8 ? 8 : n128);
  const int tiles = (range + kFaKT - 1) / kFaKT;
  kt = (tiles + cs - 1) / cs;
  const int ns_max = hd == 256 ? 3 : 4;
  ns = 2 * kt < ns_max ? 2 * kt : ns_max;
  return kt <= kFaMaxTiles;
}

template <int HD>
static int launch_dattn_fused(const CUtensorMap& km, const CUtensorMap& vm, const FAttnParams& p, int cs, bool pdl,
                              cudaStream_t s) {
  using S = FaSmem<HD>;
  static bool configured = false;
  if (!configured) {
    const int max_bytes = S::bytes(HD == 256 ? 3 : 4, kFaMaxTiles);
    if (cudaFuncSetAttribute(dattn_fused_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_bytes) !=
        cudaSuccess)
      return JX_ERR_CUDA;
    configured = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(cs, p.Hkv, p.B);
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = S::bytes(p.n_stages, p.kt_cap);
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cs;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, dattn_fused_kernel<HD>, km, vm, p) == cudaSuccess ? JX_OK : JX_ERR_CUDA;
}

// 0: by shape (the split form; the cluster form measured slower on the Llama-8B decode shapes), 1: split
// form, 2: cluster form.
static int g_dattn_impl = 0;
void set_dattn_impl(int impl) { g_dattn_impl = impl; }

int run_decode_attention(const jx_dattn_args& a, bool pdl, cudaStream_t stream) {
  if (a.B <= 0 || a.Hkv <= 0 || a.Hq % a.Hkv || a.T <= 0) return JX_ERR_SHAPE;
  const int n_rep = a.Hq / a.Hkv;
  if (n_rep > 16) return JX_ERR_SHAPE;
  if (a.hd != 64 && a.hd != 128 && a.hd != 256) return JX_ERR_SHAPE;
  if (reinterpret_cast<uintptr_t>(a.q) & 15) return JX_ERR_ARG;
  CUtensorMap km, vm;
  const long long cols = (long long)a.Hkv * a.hd;
  int rc = make_tmap_2d_bf16(&km, a.k_base, a.cache_rows, cols, cols);
  if (rc == JX_OK) rc = make_tmap_2d_bf16(&vm, a.v_base, a.cache_rows, cols, cols);
  if (rc != JX_OK) return rc;

  const int range = (a.window > 0 && a.window < a.T) ? a.window : a.T;
  int cs, kt, ns;
  const bool fits = fused_shape(range, a.hd, cs, kt, ns);
  if (g_dattn_impl == 2 && !fits) return JX_ERR_SHAPE;
  if (fits && g_dattn_impl == 2) {
    FAttnParams f;
    f.B = a.B;
    f.Hq = a.Hq;
    f.Hkv = a.Hkv;
    f.n_rep = n_rep;
    f.T = a.T;
    f.window = a.window;
    f.kt_cap = kt;
    f.n_stages = ns;
    f.layer_row0 = a.layer_row0;
    f.q = reinterpret_cast<const bf16*>(a.q);
    f.len_ptr = a.len_ptr;
    f.len_add = a.len_add;
    f.scale_bf16 = __bfloat162float(__float2bfloat16_rn(a.scale));
    f.out = reinterpret_cast<bf16*>(a.out);
    f.out_rp = a.out_rp;
    f.status = a.status;
    switch (a.hd) {
      case 64: return launch_dattn_fused<64>(km, vm, f, cs, pdl, stream);
      case 128: return launch_dattn_fused<128>(km, vm, f, cs, pdl, stream);
      default: return launch_dattn_fused<256>(km, vm, f, cs, pdl, stream);
    }
  }

  const int n_splits = dattn_n_splits(a.T, a.window);
  if (dattn_workspace_bytes(a.B, a.Hq, a.T, a.hd, n_splits) > a.ws_bytes) return JX_ERR_ARG;
  DAttnParams p;
  p.B = a.B;
  p.Hq = a.Hq;
  p.Hkv = a.Hkv;
  p.n_rep = n_rep;
  p.T = a.T;
  p.n_splits = n_splits;
  p.layer_row0 = a.layer_row0;
  p.q = reinterpret_cast<const bf16*>(a.q);
  p.len_ptr = a.len_ptr;
  p.len_add = a.len_add;
  p.window = a.window;
  p.scale_bf16 = __bfloat162float(__float2bfloat16_rn(a.scale));
  p.out = reinterpret_cast<bf16*>(a.out);
  p.out_rp = a.out_rp;
  float* ws = reinterpret_cast<float*>(a.ws);
  p.sc = ws;
  p.stats = p.sc + (long long)a.B * a.Hq * a.T;
  p.opart = p.stats + (long long)a.B * a.Hq * n_splits * 2;
  p.counters = a.counters;
  p.status = a.status;
  switch (a.hd) {
    case 64: return launch_dattn<64>(km, vm, p, pdl, stream);
    case 128: return launch_dattn<128>(km, vm, p, pdl, stream);
    default: return launch_dattn<256>(km, vm, p, pdl, stream);
  }
}

}  // namespace jxb
