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
// The default split form runs two kernels per layer, each a grid of (KV head, batch row, key split) CTAs
// of 128 keys (the split varying slowest, so the splits past the valid keys are dispatched last):
//   scores: K tiles arrive by TMA (2-D tensor map over the [L*B*T, Hkv*hd] cache, 128-byte swizzle);
//           Q.K^T on mma.sync; the rounded scores go to a float32 workspace with per-split (max, sum).
//   pv:     combines the split statistics into the exact softmax normaliser, forms the bf16
//           probabilities, P.V on mma.sync with V tiles by TMA, and the last CTA of a head group sums
//           the split partials in split order (deterministic) into the bf16 output (K128 layout).
// Selectable alternatives (jx_set_decode_attention_impl; all tested, none faster at the decode shapes):
// the column pv (one CTA per 64 output columns over all keys), the single-pass cluster form
// (dattn_warp_kernel: a thread-block cluster per (row, KV head), key ranges up to 8 CTAs x 2048 keys), the
// cluster-split form (the split form's CTAs of a head group as one cluster exchanging statistics and
// partials through distributed shared memory) and the queue form (the split form's work as one
// persistent kernel whose CTAs claim score and pv items from a counter).
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
  // RoPE + cache append fused in (qkv != nullptr): see jx_dattn_args
  const bf16* qkv;
  long long ld_qkv;
  const bf16* cos;
  const bf16* sin;
  int rd, max_pos;
  bf16* k_cache;         // the cache allocations, written at this step's position
  bf16* v_cache;
  // queue form: [0] item claims, [1] finished CTAs, [2, 2 + B * Hkv) scored splits per head group
  int* qsync;
};

// 8 consecutive elements [j0, j0 + 8) of one head of the projection output, rotated on its first rd
// dims at table row `pos` exactly as qkv_rope_append_kernel does (rotate_half, products and sum each
// rounded to bf16), packed as bf16.
__device__ __forceinline__ uint4 rope8(const bf16* head, int j0, int hd, int rd, const bf16* cos, const bf16* sin,
                                       int pos) {
  const int half = rd >> 1;
  float o[8];
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    const int j = j0 + u;
    const float x = __bfloat162float(head[j]);
    if (j < rd) {
      const float rot = j < half ? -__bfloat162float(head[j + half]) : __bfloat162float(head[j - half]);
      const float a = rnd<bf16>(x * __bfloat162float(cos[(long long)pos * rd + j]));
      const float c = rnd<bf16>(rot * __bfloat162float(sin[(long long)pos * rd + j]));
      o[u] = rnd<bf16>(a + c);
    } else {
      o[u] = x;
    }
  }
  (void)hd;
  return make_uint4(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]), pack_bf16x2(o[4], o[5]),
                    pack_bf16x2(o[6], o[7]));
}

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

// Exact softmax normaliser of each query row of a head group from its split statistics st[row][split]
// (max, sum): M = max over the splits, L = sum over the splits in split order of sum * exp(max - M).  All
// 128 threads: 8 lanes per row (rows tid / 8 < 16) load the statistics at once; the ordered sum passes
// each split's (sum, exp) to the row's lanes by shuffles, so L is accumulated in split order with one
// fused multiply-add a split, as a loop over the splits compiles (bit-identical).  Writes Ms[row], Ls[row] for rows < 16 (rows >= n_rep: -inf, 0).
__device__ __forceinline__ void split_normaliser(const float* st_group, int n_rep, int n_splits, int n_active,
                                                 float* Ms, float* Ls) {
  const int row = threadIdx.x >> 3, j = threadIdx.x & 7, base = (threadIdx.x & 31) & ~7;
  const bool on = row < n_rep;
  const float* st = st_group + (long long)row * n_splits * 2;
  // chunks of 64 splits: lane j holds splits c0 + 8 i + j, i < 8, all loaded before they are used
  float M = -INFINITY;
  for (int c0 = 0; c0 < n_active; c0 += 64) {
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int sj = c0 + 8 * i + j;
      v[i] = on && sj < n_active ? __ldcg(st + sj * 2) : -INFINITY;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) M = fmaxf(M, v[i]);
  }
  M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, 4));
  M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, 2));
  M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, 1));
  float L = 0.f;
  for (int c0 = 0; c0 < n_active; c0 += 64) {
    float mx[8], sm[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int sj = c0 + 8 * i + j;
      const bool in = on && sj < n_active;
      mx[i] = in ? __ldcg(st + sj * 2) : 0.f;
      sm[i] = in ? __ldcg(st + sj * 2 + 1) : 0.f;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float e = expf(mx[i] - M);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        // L += sum * e as one fused multiply-add, as the compiler contracts it in a loop over the splits
        const float sk = __shfl_sync(0xffffffffu, sm[i], base + k);
        const float ek = __shfl_sync(0xffffffffu, e, base + k);
        if (c0 + 8 * i + k < n_active) L = fmaf(sk, ek, L);
      }
    }
  }
  if (j == 0) {
    Ms[row] = on ? M : -INFINITY;
    Ls[row] = on ? L : 0.f;
  }
}

// The last pv CTA of a head group: out = bf16(sum over the splits, in split order, of the float32
// partials), four outputs a thread at a time with their partials' loads issued together.
template <int HD>
__device__ __forceinline__ void sum_split_partials(const float* opart_group, int n_rep, int n_splits, int n_active,
                                                   bf16* out, long long out_rp, int b, long long col0) {
  const int total = n_rep * HD;
  for (int i0 = threadIdx.x; i0 < total; i0 += 4 * 128) {
    float sum[4] = {0.f, 0.f, 0.f, 0.f};
    for (int s0 = 0; s0 < n_active; s0 += 8) {
      float v[4][8];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int idx = i0 + q * 128;
        const int row = idx / HD, col = idx % HD;
        const float* src = opart_group + ((long long)row * n_splits) * HD + col;
#pragma unroll
        for (int k = 0; k < 8; ++k)
          v[q][k] = idx < total && s0 + k < n_active ? __ldcg(src + (long long)(s0 + k) * HD) : 0.f;
      }
#pragma unroll
      for (int q = 0; q < 4; ++q)
#pragma unroll
        for (int k = 0; k < 8; ++k)
          if (s0 + k < n_active) sum[q] += v[q][k];
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int idx = i0 + q * 128;
      if (idx >= total) continue;
      const int row = idx / HD, col = idx % HD;
      out[k128_offset(b, col0 + (long long)row * HD + col, out_rp)] = __float2bfloat16_rn(sum[q]);
    }
  }
}

// RQ: rows of the query (scores) / probability (pv) tile in shared memory, 16 or, when a head group has
// at most 8 query heads, 8 (the MMA's rows 8-15 are then zero registers).  The smaller tiles let 6 CTAs
// share an SM instead of 5, so a 768-slot cache (6 splits x 128 head groups) runs in one wave.
template <int HD, int RQ>
__global__ void __launch_bounds__(128) dattn_scores_kernel(const __grid_constant__ CUtensorMap kmap, DAttnParams p) {
  constexpr int NB = HD / 64;                 // 64-column blocks per head
  constexpr int TILE_BYTES = kDaTile * HD * 2;
  constexpr int QB = RQ * 128;                // bytes of one [RQ x 64] query block
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ktile = smem;                                   // 2 tiles, each NB blocks of [64 x 64]
  uint8_t* qs = smem + 2 * TILE_BYTES;                     // NB blocks of [RQ x 64]
  uint64_t* bar = reinterpret_cast<uint64_t*>(qs + NB * QB);
  float* red = reinterpret_cast<float*>(bar + 2);          // [4 warps][16 rows]

  const int kvh = blockIdx.x, b = blockIdx.y, split = blockIdx.z;   // split-major launch order
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // The kernel before this one (RoPE + cache append) releases it only after its own wait, so the
  // positions and the keys of earlier steps are complete here: tiles that end before this step's key
  // (position valid - 1) are loaded before waiting; the rest, and q, after.
  int lo, valid;
  key_range(p, b, lo, valid);
  const int t0 = lo + split * kDaKeys;
  if (t0 >= valid) return;
  const int t1 = min(t0 + kDaKeys, valid);
  const int n_tiles = (t1 - t0 + kDaTile - 1) / kDaTile;
  auto issue = [&](int i) {
    mbar_arrive_expect_tx(&bar[i], TILE_BYTES);
    const int y = (int)(p.layer_row0 + (long long)b * p.T + t0 + i * kDaTile);
#pragma unroll
    for (int c = 0; c < NB; ++c) tma_load_2d(ktile + i * TILE_BYTES + c * 8192, &kmap, kvh * HD + c * 64, y, &bar[i]);
  };
  int n_early = 0;
  if (threadIdx.x == 0) {
    prefetch_tmap(&kmap);
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    fence_barrier_init();
    // with the append fused in, this kernel writes this step's key itself and patches it into the
    // loaded tile, so that tile loads early too; otherwise the kernel before wrote it
    const bool fused_append = p.qkv != nullptr;
    while (n_early < n_tiles && (fused_append || t0 + (n_early + 1) * kDaTile <= valid - 1)) issue(n_early++);
  }
  pdl_wait();
  // the pv kernel after this one loads values before its own wait: release it only now
  pdl_trigger();
  if (threadIdx.x == 0)
    for (int i = n_early; i < n_tiles; ++i) issue(i);
  // Fused RoPE: this step's position, its table row (row 0 with a range error beyond the table)
  const bool fused = p.qkv != nullptr;
  int pos = valid - 1;
  if (fused && pos >= p.max_pos) {
    if (threadIdx.x == 0) set_status(p.status, JX_ERR_RANGE);
    pos = 0;
  }
  const bf16* qkv_row = fused ? p.qkv + (long long)b * p.ld_qkv : nullptr;
  // Q rows of this head group (rows >= n_rep are zero) into the swizzled layout.
  for (int idx = threadIdx.x; idx < RQ * (HD / 8); idx += 128) {
    const int r = idx / (HD / 8), cg = idx % (HD / 8);
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < p.n_rep) {
      if (fused)
        v = rope8(qkv_row + (long long)(kvh * p.n_rep + r) * HD, cg * 8, HD, p.rd, p.cos, p.sin, pos);
      else
        v = *reinterpret_cast<const uint4*>(p.q + ((long long)b * p.Hq + kvh * p.n_rep + r) * HD + cg * 8);
    }
    const uint32_t a = swz(smem_u32(qs + (cg >> 3) * QB), r, cg & 7);
    asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(a), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w));
  }
  // The CTA holding this step's key appends the rotated k and the v of this KV head to the cache and
  // puts the k into its loaded tile (whose row was read from the cache before the append).
  if (fused && valid - 1 >= t0 && valid - 1 < t1) {
    const int kpos = valid - 1;
    const int tile = (kpos - t0) / kDaTile, trow = (kpos - t0) % kDaTile;
    const long long crow = (p.layer_row0 + (long long)b * p.T + kpos) * ((long long)p.Hkv * HD) + (long long)kvh * HD;
    uint4 k8 = make_uint4(0, 0, 0, 0);
    const int j0 = threadIdx.x * 8;
    if (j0 < HD) {
      k8 = rope8(qkv_row + (long long)(p.Hq + kvh) * HD, j0, HD, p.rd, p.cos, p.sin, pos);
      const uint4 v8 = *reinterpret_cast<const uint4*>(qkv_row + (long long)(p.Hq + p.Hkv + kvh) * HD + j0);
      *reinterpret_cast<uint4*>(p.k_cache + crow + j0) = k8;
      *reinterpret_cast<uint4*>(p.v_cache + crow + j0) = v8;
    }
    const bool landed = mbar_wait_bounded(&bar[tile], 0);
    if (!landed && threadIdx.x == 0) set_status(p.status, JX_ERR_TIMEOUT);
    if (landed && j0 < HD) {
      const uint32_t a = swz(smem_u32(ktile + tile * TILE_BYTES + (j0 >> 6) * 8192), trow, (j0 & 63) >> 3);
      asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(a), "r"(k8.x), "r"(k8.y), "r"(k8.z), "r"(k8.w));
    }
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
      uint32_t a0, a1 = 0, a2, a3 = 0, b0, b1, b2, b3;
      if (RQ == 16) {
        const int row = (mi & 1) * 8 + r8, ch = ks * 2 + (mi >> 1);
        ldsm_x4(swz(smem_u32(qs + (ch >> 3) * QB), row, ch & 7), a0, a1, a2, a3);
      } else {
        const int ch = ks * 2 + (mi & 1);   // (lanes 16-31 give no address for .x2)
        ldsm_x2(swz(smem_u32(qs + (ch >> 3) * QB), r8, ch & 7), a0, a2);
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

template <int HD, int RQ>
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
  bf16* ptile = reinterpret_cast<bf16*>(Ls + 16);  // [RQ][kPLd]
  __shared__ int last_flag;

  const int kvh = blockIdx.x, b = blockIdx.y, split = blockIdx.z;   // split-major launch order
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_trigger();
  // The scores kernel before this one releases it only after its own wait, so every value of the cache
  // (this step's included) and the positions are complete: the value tiles load while it finishes.
  int lo, valid;
  key_range(p, b, lo, valid);
  const int t0 = lo + split * kDaKeys;
  const int n_active = (valid - lo + kDaKeys - 1) / kDaKeys;
  if (t0 >= valid) return;
  const int t1 = min(t0 + kDaKeys, valid);
  const int n_tiles = (t1 - t0 + kDaTile - 1) / kDaTile;
  // With the append fused into the scores kernel, the tile holding this step's value loads after the wait.
  auto issue = [&](int i) {
    mbar_arrive_expect_tx(&bar[i], TILE_BYTES);
    const int y = (int)(p.layer_row0 + (long long)b * p.T + t0 + i * kDaTile);
#pragma unroll
    for (int c = 0; c < NB; ++c) tma_load_2d(vtile + i * TILE_BYTES + c * 8192, &vmap, kvh * HD + c * 64, y, &bar[i]);
  };
  int n_early = n_tiles;
  if (p.qkv != nullptr)
    for (n_early = 0; n_early < n_tiles && t0 + (n_early + 1) * kDaTile <= valid - 1;) ++n_early;
  if (threadIdx.x == 0) {
    prefetch_tmap(&vmap);
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    fence_barrier_init();
    for (int i = 0; i < n_early; ++i) issue(i);
  }
  pdl_wait();
  if (threadIdx.x == 0)
    for (int i = n_early; i < n_tiles; ++i) issue(i);
  // this CTA's scores (coalesced reads, issued before the statistics are combined; with 16-row tiles they
  // are read afterwards, which keeps the kernel at 5 CTAs per SM)
  constexpr bool kEarly = RQ == 8;
  auto score = [&](int i) {
    const int idx = threadIdx.x + i * 128;
    const int row = idx / kDaKeys, t = t0 + idx % kDaKeys;
    return row < p.n_rep && t < t1 ? __ldcg(p.sc + ((long long)b * p.Hq + kvh * p.n_rep + row) * p.T + t) : 0.f;
  };
  float sv[kEarly ? RQ : 1];
#pragma unroll
  for (int i = 0; i < (kEarly ? RQ : 0); ++i) sv[i] = score(i);
  // exact softmax normaliser of each row from the split statistics
  split_normaliser(p.stats + ((long long)b * p.Hq + kvh * p.n_rep) * p.n_splits * 2, p.n_rep, p.n_splits, n_active,
                   Ms, Ls);
  __syncthreads();

  const int mi = lane >> 3, r8 = lane & 7;
  const int r_lo = lane >> 2, r_hi = r_lo + 8;
  // Probabilities of this CTA's keys, computed once into a padded bf16 tile [RQ rows][kDaKeys + 8] that
  // every warp reads with ldmatrix.
#pragma unroll
  for (int i = 0; i < RQ; ++i) {
    const int idx = threadIdx.x + i * 128;
    const int row = idx / kDaKeys, k = idx % kDaKeys, t = t0 + k;
    float pv = 0.f;
    if (row < p.n_rep && t < t1) pv = rnd<bf16>(expf((kEarly ? sv[kEarly ? i : 0] : score(i)) - Ms[row]) / Ls[row]);
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
      uint32_t a0, a1 = 0, a2, a3 = 0;
      if (RQ == 16) {
        const int row = (mi & 1) * 8 + r8, col = i * kDaTile + kk * 16 + (mi >> 1) * 8;
        ldsm_x4(smem_u32(ptile + row * kPLd + col), a0, a1, a2, a3);
      } else {
        ldsm_x2(smem_u32(ptile + r8 * kPLd + i * kDaTile + kk * 16 + (mi & 1) * 8), a0, a2);
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
  // one fence after the barrier releases every thread's partial stores (cumulativity), then the arrival
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const int prev = atomicAdd(&p.counters[b * p.Hkv + kvh], 1);
    last_flag = (prev == n_active - 1);
  }
  __syncthreads();
  if (!last_flag) return;
  __threadfence();
  sum_split_partials<HD>(p.opart + (((long long)b * p.Hq + kvh * p.n_rep) * p.n_splits) * HD, p.n_rep, p.n_splits,
                         n_active, p.out, p.out_rp, b, (long long)kvh * p.n_rep * HD);
  if (threadIdx.x == 0) p.counters[b * p.Hkv + kvh] = 0;
}

// ------------------------------------------------------------------------------------------------
// Cluster-split form: the split form's decomposition (one CTA per 128 keys of a (KV head, batch row))
// in one kernel, the key splits of a head group forming one thread-block cluster (co-scheduled), so
// the softmax statistics and the output partials are exchanged through distributed shared memory
// instead of global memory and a second kernel.  Per CTA: K tiles (those of earlier steps before the
// wait, as in the scores kernel), q.k on mma.sync with the scores kept in registers, this CTA's row
// (max, sum) published in shared memory, the V tiles loaded into the freed K slots while the cluster
// exchanges the statistics, exact bf16 probabilities from the cluster-wide (max, sum) in rank order,
// P.V, and the partials summed over the cluster in rank order (the same sums as the split form).
// ------------------------------------------------------------------------------------------------
template <int HD>
__global__ void __launch_bounds__(128) dattn_csplit_kernel(const __grid_constant__ CUtensorMap kmap,
                                                           const __grid_constant__ CUtensorMap vmap, DAttnParams p) {
  constexpr int NB = HD / 64;
  constexpr int TILE_BYTES = kDaTile * HD * 2;
  constexpr int WCOLS = HD / 4;             // output columns per warp in P.V
  constexpr int NT = WCOLS / 8;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ktile = smem;                                   // 2 tiles: K, then V, then the output partial
  uint8_t* qs = smem + 2 * TILE_BYTES;                     // NB blocks of [16 x 64]
  bf16* ptile = reinterpret_cast<bf16*>(qs + NB * 2048);   // [16][kPLd]
  uint64_t* bar = reinterpret_cast<uint64_t*>(ptile + 16 * kPLd);   // [0,1] K tiles, [2,3] V tiles
  float* red = reinterpret_cast<float*>(bar + 4);          // [4 warps][16 rows]
  __shared__ float cmax[16], csum[16], Ms[16], Ls[16];

  const int kvh = blockIdx.y, b = blockIdx.z;
  const int rank = (int)cluster_ctarank(), CS = (int)gridDim.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_trigger();
  int lo, valid;
  key_range(p, b, lo, valid);
  const int t0 = lo + rank * kDaKeys;
  const int t1 = min(t0 + kDaKeys, valid);
  const int n_tiles = t0 < valid ? (t1 - t0 + kDaTile - 1) / kDaTile : 0;
  auto issue = [&](const CUtensorMap* map, int i, uint64_t* bb) {
    mbar_arrive_expect_tx(bb, TILE_BYTES);
    const int y = (int)(p.layer_row0 + (long long)b * p.T + t0 + i * kDaTile);
#pragma unroll
    for (int c = 0; c < NB; ++c) tma_load_2d(ktile + i * TILE_BYTES + c * 8192, map, kvh * HD + c * 64, y, bb);
  };
  int n_early = 0;
  if (threadIdx.x == 0) {
    prefetch_tmap(&kmap);
    prefetch_tmap(&vmap);
    for (int i = 0; i < 4; ++i) mbar_init(&bar[i], 1);
    fence_barrier_init();
    while (n_early < n_tiles && t0 + (n_early + 1) * kDaTile <= valid - 1) issue(&kmap, n_early, &bar[n_early]), ++n_early;
  }
  pdl_wait();
  if (threadIdx.x == 0)
    for (int i = n_early; i < n_tiles; ++i) issue(&kmap, i, &bar[i]);
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
  const int r_lo = lane >> 2, r_hi = r_lo + 8;
  float s[2][2][4];
  float mrow[2] = {-INFINITY, -INFINITY};
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
  ok = __syncthreads_and(ok) != 0;   // every warp is done with the K tiles
  // the V tiles go into the freed K slots while the statistics are exchanged
  if (threadIdx.x == 0 && ok) {
    fence_proxy_async();
    for (int i = 0; i < n_tiles; ++i) issue(&vmap, i, &bar[2 + i]);
  }
  // this CTA's row maxima and exp-sums (as the scores kernel computes them)
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    mrow[h] = fmaxf(mrow[h], __shfl_xor_sync(0xffffffffu, mrow[h], 1));
    mrow[h] = fmaxf(mrow[h], __shfl_xor_sync(0xffffffffu, mrow[h], 2));
  }
  if ((lane & 3) == 0) {
    red[warp * 16 + r_lo] = mrow[0];
    red[warp * 16 + r_hi] = mrow[1];
  }
  __syncthreads();
  float m[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int row = r_lo + h * 8;
    m[h] = fmaxf(fmaxf(red[row], red[16 + row]), fmaxf(red[32 + row], red[48 + row]));
  }
  __syncthreads();
  float l[2] = {0.f, 0.f};
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int row = r_lo + (e >> 1) * 8;
        const int t = t0 + i * kDaTile + warp * 16 + nt * 8 + (lane & 3) * 2 + (e & 1);
        if (t < t1 && row < p.n_rep) l[e >> 1] += expf(s[i][nt][e] - m[e >> 1]);
      }
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    l[h] += __shfl_xor_sync(0xffffffffu, l[h], 1);
    l[h] += __shfl_xor_sync(0xffffffffu, l[h], 2);
  }
  if ((lane & 3) == 0) {
    red[warp * 16 + r_lo] = l[0];
    red[warp * 16 + r_hi] = l[1];
  }
  __syncthreads();
  if (warp == 0 && (lane & 3) == 0) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int row = r_lo + h * 8;
      cmax[row] = m[h];
      csum[row] = (red[row] + red[16 + row]) + (red[32 + row] + red[48 + row]);
    }
  }
  cluster_sync_all();
  // cluster-wide normaliser of each row, over the ranks in order (the split statistics of the split form)
  if (threadIdx.x < 16) {
    const int row = threadIdx.x;
    float M = -INFINITY, L = 0.f;
    if (row < p.n_rep) {
      const uint32_t am = smem_u32(cmax + row), as = smem_u32(csum + row);
      for (int cr = 0; cr < CS; ++cr) M = fmaxf(M, dsmem_ld_f32(dsmem_map(am, cr)));
      for (int cr = 0; cr < CS; ++cr)
        L += dsmem_ld_f32(dsmem_map(as, cr)) * expf(dsmem_ld_f32(dsmem_map(am, cr)) - M);
    }
    Ms[row] = M;
    Ls[row] = L;
  }
  __syncthreads();
  // exact bf16 probabilities of this CTA's keys into the probability tile
  for (int idx = threadIdx.x; idx < 16 * kPLd; idx += 128) ptile[idx] = __float2bfloat16_rn(0.f);
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int row = r_lo + (e >> 1) * 8;
        const int k = i * kDaTile + warp * 16 + nt * 8 + (lane & 3) * 2 + (e & 1);
        if (t0 + k < t1 && row < p.n_rep)
          ptile[row * kPLd + k] = __float2bfloat16_rn(rnd<bf16>(expf(s[i][nt][e] - Ms[row]) / Ls[row]));
      }
  __syncthreads();
  float acc[NT][4] = {};
  for (int i = 0; i < n_tiles && ok; ++i) {
    if (!mbar_wait_bounded(&bar[2 + i], 0)) {
      set_status(p.status, JX_ERR_TIMEOUT);
      ok = false;
      continue;
    }
    const uint32_t vb = smem_u32(ktile + i * TILE_BYTES);
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
  __syncthreads();   // every warp is done with the V tiles: the slots take the partial
  float* part = reinterpret_cast<float*>(ktile);   // [16][HD]
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int row = (e >> 1) ? r_hi : r_lo;
      part[row * HD + warp * WCOLS + nt * 8 + (lane & 3) * 2 + (e & 1)] = acc[nt][e];
    }
  cluster_sync_all();
  // rank r sums its slice of the outputs over the ranks in order and rounds it once
  {
    const int total = p.n_rep * HD, chunk = (total + CS - 1) / CS;
    const int e0 = rank * chunk, e1 = min(e0 + chunk, total);
    for (int idx = e0 + threadIdx.x; idx < e1; idx += 128) {
      const int row = idx / HD, col = idx % HD;
      const uint32_t la = smem_u32(part + row * HD + col);
      float sum = 0.f;
      for (int cr = 0; cr < CS; ++cr) sum += dsmem_ld_f32(dsmem_map(la, cr));
      const long long ocol = (long long)(kvh * p.n_rep + row) * HD + col;
      if (ok) p.out[k128_offset(b, ocol, p.out_rp)] = __float2bfloat16_rn(sum);
    }
  }
  cluster_sync_all();   // no CTA leaves while another may still read its shared memory
}

// ------------------------------------------------------------------------------------------------
// Column form of the pv step: one CTA per (64-column block of the head, KV head, batch row) runs over
// all valid keys, so no split partials and no cross-CTA reduction are needed.  The value tiles
// [64 keys x 64 columns] stream through a ring of kPcStages stages; warp w consumes tiles w, w+4, ...
// and refills the stages it owns (kPcStages % 4 == 0) as it frees them.  The first kPcStages tiles are
// issued before the wait on the scores kernel (which releases dependents after its own wait, so the
// values are complete).  Each warp forms the exact bf16 probabilities of its tile from the scores and
// the split statistics, accumulates P.V on mma.sync, and the four warp partials are added in warp order
// (deterministic), rounded once to bf16 (K128 layout).
// ------------------------------------------------------------------------------------------------
constexpr int kPcStages = 8;
constexpr int kPcLd = 64 + 8;   // padded row stride (bf16) of a warp's probability tile

template <int HD>
__global__ void __launch_bounds__(128) dattn_pvcol_kernel(const __grid_constant__ CUtensorMap vmap, DAttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* vring = smem;                                             // kPcStages x [64 x 64] bf16, 128B swizzle
  bf16* ptiles = reinterpret_cast<bf16*>(smem + kPcStages * 8192);   // [4 warps][16][kPcLd]
  uint64_t* full = reinterpret_cast<uint64_t*>(ptiles + 4 * 16 * kPcLd);
  __shared__ float Ms[16], Ls[16];

  const int cb = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_trigger();
  int lo, valid;
  key_range(p, b, lo, valid);
  const int n_tiles = valid > lo ? (valid - lo + 63) / 64 : 0;
  auto issue = [&](int i) {
    const int st = i % kPcStages;
    mbar_arrive_expect_tx(&full[st], 8192);
    tma_load_2d(vring + st * 8192, &vmap, kvh * HD + cb * 64, (int)(p.layer_row0 + (long long)b * p.T + lo + i * 64),
                &full[st]);
  };
  if (threadIdx.x == 0) {
    prefetch_tmap(&vmap);
    for (int st = 0; st < kPcStages; ++st) mbar_init(&full[st], 1);
    fence_barrier_init();
    for (int i = 0; i < n_tiles && i < kPcStages; ++i) issue(i);
  }
  __syncthreads();
  pdl_wait();
  // exact softmax normaliser of each row from the split statistics
  if (threadIdx.x < 16) {
    const int row = threadIdx.x;
    float M = -INFINITY, L = 0.f;
    if (row < p.n_rep) {
      const int n_active = (valid - lo + kDaKeys - 1) / kDaKeys;
      const float* st = p.stats + ((long long)b * p.Hq + kvh * p.n_rep + row) * p.n_splits * 2;
      for (int s2 = 0; s2 < n_active; ++s2) M = fmaxf(M, st[s2 * 2]);
      for (int s2 = 0; s2 < n_active; ++s2) L += st[s2 * 2 + 1] * expf(st[s2 * 2] - M);
    }
    Ms[row] = M;
    Ls[row] = L;
  }
  __syncthreads();

  const int mi = lane >> 3, r8 = lane & 7;
  bf16* pt = ptiles + warp * 16 * kPcLd;
  const float* sc = p.sc + ((long long)b * p.Hq + kvh * p.n_rep) * p.T;
  float acc[8][4] = {};
  bool ok = true;
  for (int i = warp; i < n_tiles; i += 4) {
    const int st = i % kPcStages;
    const int t0 = lo + i * 64;
    // probabilities of this tile's keys (rows >= n_rep and keys past the range are zero)
    for (int idx = lane; idx < 16 * 64; idx += 32) {
      const int row = idx >> 6, k = idx & 63, t = t0 + k;
      float pv = 0.f;
      if (row < p.n_rep && t < valid) pv = rnd<bf16>(expf(__ldcg(sc + (long long)row * p.T + t) - Ms[row]) / Ls[row]);
      pt[row * kPcLd + k] = __float2bfloat16_rn(pv);
    }
    __syncwarp();
    if (!mbar_wait_bounded(&full[st], (i / kPcStages) & 1)) {
      // this warp's only other copy in flight is tile i + 4: let it land (bounded) before leaving
      if (lane == 0) set_status(p.status, JX_ERR_TIMEOUT);
      if (i + 4 < n_tiles) mbar_wait_bounded(&full[(i + 4) % kPcStages], ((i + 4) / kPcStages) & 1);
      ok = false;
      break;
    }
    {
      const uint32_t vb = smem_u32(vring + st * 8192);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4(smem_u32(pt + ((mi & 1) * 8 + r8) * kPcLd + kk * 16 + (mi >> 1) * 8), a0, a1, a2, a3);
#pragma unroll
        for (int n16 = 0; n16 < 4; ++n16) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(swz(vb, kk * 16 + (mi & 1) * 8 + r8, n16 * 2 + (mi >> 1)), b0, b1, b2, b3);
          mma_bf16(acc[n16 * 2], a0, a1, a2, a3, b0, b1);
          mma_bf16(acc[n16 * 2 + 1], a0, a1, a2, a3, b2, b3);
        }
      }
    }
    __syncwarp();
    // refill the stage just freed with this warp's tile i + kPcStages
    if (lane == 0 && i + kPcStages < n_tiles) {
      fence_proxy_async();
      issue(i + kPcStages);
    }
  }
  if (!__syncthreads_and(ok)) return;
  // warp partials into the (now idle) ring, then summed in warp order
  float* red = reinterpret_cast<float*>(vring);   // [4 warps][16][64]
  {
    const int r_lo = lane >> 2;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e)
        red[(warp * 16 + r_lo + (e >> 1) * 8) * 64 + nt * 8 + (lane & 3) * 2 + (e & 1)] = acc[nt][e];
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < p.n_rep * 64; idx += 128) {
    const int row = idx >> 6, col = idx & 63;
    const float sum = ((red[row * 64 + col] + red[(16 + row) * 64 + col]) + red[(32 + row) * 64 + col]) +
                      red[(48 + row) * 64 + col];
    const long long ocol = (long long)(kvh * p.n_rep + row) * HD + cb * 64 + col;
    p.out[k128_offset(b, ocol, p.out_rp)] = __float2bfloat16_rn(sum);
  }
}

// ------------------------------------------------------------------------------------------------
// Single-pass form: a thread-block cluster of CS CTAs per (batch row, KV head) (CS = 1 when there are
// at least as many head groups as SMs), the CTAs splitting the valid keys into contiguous runs of tiles.
// Inside a CTA the 4 warps are independent pipelines: warp w owns tiles w, w+4, ... of the CTA's run,
// streams their K and then their V tiles through its own two shared-memory slots (TMA, one mbarrier per
// slot, refilled by the same warp), so no CTA-wide barrier is taken per tile.  Q stays in registers.
//   scores : rounded like the reference, kept as bf16 in shared memory (exact: they are bf16 values)
//   softmax: row maxima and exp-sums over the warps in warp order, then over the cluster in rank
//            order through distributed shared memory; every CTA then forms the exact probabilities
//            bf16(exp(s - max) / sum) of its keys directly as mma.sync A fragments
//   output : each warp's partial sum_t p_t v_t, added over the warps in warp order and over the
//            cluster in rank order (deterministic), rounded once to bf16 (K128 layout)
// ------------------------------------------------------------------------------------------------
constexpr int kWaMaxKeys = 2048;          // keys per CTA this form keeps scores for

struct FAttnParams {
  int B, Hq, Hkv, n_rep, T, window;
  int kt_cap;            // tiles per CTA the shared memory was sized for
  int _pad0;
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
struct WaCfg {
  static constexpr int KT = HD == 256 ? 32 : 64;     // keys per tile
  static constexpr int NB = HD / 64;                 // 64-column blocks of a row
  static constexpr int kBlockBytes = KT * 128;       // one [KT x 64] block, 128-byte swizzle
  static constexpr int kTileBytes = NB * kBlockBytes;
  static constexpr int NSW = HD == 64 ? 4 : 2;       // ring slots per warp
  static constexpr int kRing = 4 * NSW * kTileBytes; // 128 KB
  static constexpr int NKS = HD / 16;                // k-steps of q . k
  static constexpr int NT = KT / 8;                  // n8 key tiles per tile
  static constexpr int kMaxTiles = kWaMaxKeys / KT;
  // byte offsets from the 1024-aligned base for `kt` tiles per CTA
  static __host__ __device__ int q_off() { return kRing; }
  static __host__ __device__ int sc_off() { return kRing + NB * 2048; }
  static __host__ __device__ int sc_ld(int kt) { return kt * KT + 8; }
  static __host__ __device__ int red_off(int kt) { return sc_off() + 16 * sc_ld(kt) * 2; }
  static __host__ __device__ int bar_off(int kt) { return red_off(kt) + 192 * 4; }
  static __host__ __device__ int bytes(int kt) { return 1024 + bar_off(kt) + 4 * NSW * 8 + 16; }
};

template <int HD>
__global__ void __launch_bounds__(128) dattn_warp_kernel(const __grid_constant__ CUtensorMap kmap,
                                                         const __grid_constant__ CUtensorMap vmap, FAttnParams p) {
  using C = WaCfg<HD>;
  constexpr int KT = C::KT, NSW = C::NSW;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int kt_cap = p.kt_cap;
  uint8_t* ring = smem;
  uint8_t* qs = smem + C::q_off();
  bf16* sc = reinterpret_cast<bf16*>(smem + C::sc_off());
  const int sc_ld = C::sc_ld(kt_cap);
  float* redm = reinterpret_cast<float*>(smem + C::red_off(kt_cap));   // [4 warps][16] row maxima
  float* reds = redm + 64;                                               // [4 warps][16] row exp-sums
  float* cmax = reds + 64;       // [16] this CTA's row maxima (read by the cluster)
  float* csum = cmax + 16;       // [16] this CTA's row exp-sums (read by the cluster)
  float* Mrow = csum + 16;       // [16] cluster row maxima
  float* Lrow = Mrow + 16;       // [16] cluster row sums
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::bar_off(kt_cap));
  float* opart = reinterpret_cast<float*>(ring);   // [4 warps][16][HD], once every tile is consumed

  const int CS = gridDim.x;
  const uint32_t rank = cluster_ctarank();
  const int kvh = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_trigger();
  pdl_wait();

  int valid = p.len_ptr[b] + p.len_add;
  if (valid > p.T) {
    set_status(p.status, JX_ERR_RANGE);
    valid = p.T;
  }
  const int lo = (p.window > 0 && valid > p.window) ? valid - p.window : 0;
  const int n_tiles = valid > lo ? (valid - lo + KT - 1) / KT : 0;
  int tpc = (n_tiles + CS - 1) / CS;
  if (tpc > kt_cap) {
    set_status(p.status, JX_ERR_RANGE);
    tpc = kt_cap;
  }
  const int my0 = (int)rank * tpc;
  const int my_n = max(0, min(tpc, n_tiles - my0));         // tiles of this CTA
  const int key0 = lo + my0 * KT;                           // first key of this CTA
  const int nw = my_n > warp ? (my_n - warp + 3) / 4 : 0;   // tiles of this warp: warp, warp+4, ...
  const long long row0 = p.layer_row0 + (long long)b * p.T;
  uint64_t* wbar = bars + warp * NSW;
  uint8_t* wring = ring + warp * NSW * C::kTileBytes;

  // load q of this warp: K tiles j = 0..nw-1, then V tiles (tile index warp + 4j)
  auto issue = [&](int q) {
    const int slot = q % NSW;
    const bool is_v = q >= nw;
    const int i = warp + 4 * (is_v ? q - nw : q);
    mbar_arrive_expect_tx(&wbar[slot], C::kTileBytes);
    const int y = (int)(row0 + key0 + i * KT);
#pragma unroll
    for (int c = 0; c < C::NB; ++c)
      tma_load_2d(wring + slot * C::kTileBytes + c * C::kBlockBytes, is_v ? &vmap : &kmap, kvh * HD + c * 64, y,
                  &wbar[slot]);
  };
  if (lane == 0) {
    if (warp == 0) {
      prefetch_tmap(&kmap);
      prefetch_tmap(&vmap);
    }
    for (int s = 0; s < NSW; ++s) mbar_init(&wbar[s], 1);
    fence_barrier_init();
    for (int q = 0; q < min(NSW, 2 * nw); ++q) issue(q);
  }
  // Q rows of this head group (rows >= n_rep are zero) into the swizzled layout, then into registers.
  for (int idx = threadIdx.x; idx < 16 * (HD / 8); idx += 128) {
    const int r = idx / (HD / 8), cg = idx % (HD / 8);
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < p.n_rep) v = *reinterpret_cast<const uint4*>(p.q + ((long long)b * p.Hq + kvh * p.n_rep + r) * HD + cg * 8);
    const uint32_t a = swz(smem_u32(qs + (cg >> 3) * 2048), r, cg & 7);
    asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(a), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w));
  }
  __syncthreads();
  const int mi = lane >> 3, r8 = lane & 7;
  uint32_t qf[C::NKS][4];
#pragma unroll
  for (int ks = 0; ks < C::NKS; ++ks) {
    const int row = (mi & 1) * 8 + r8, ch = ks * 2 + (mi >> 1);
    ldsm_x4(swz(smem_u32(qs + (ch >> 3) * 2048), row, ch & 7), qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3]);
  }

  bool ok = true;
  // ---- scores of this warp's tiles ----
  float mrow[2] = {-INFINITY, -INFINITY};   // rows lane/4 and lane/4 + 8
  for (int j = 0; j < nw; ++j) {
    const int slot = j % NSW, i = warp + 4 * j;
    if (ok && !mbar_wait_bounded(&wbar[slot], (j / NSW) & 1)) {
      set_status(p.status, JX_ERR_TIMEOUT);
      ok = false;
    }
    ok = __all_sync(0xffffffffu, ok);
    float acc[C::NT][4];
#pragma unroll
    for (int t = 0; t < C::NT; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.f;
    if (ok) {
      const uint32_t kb = smem_u32(wring + slot * C::kTileBytes);
#pragma unroll
      for (int ks = 0; ks < C::NKS; ++ks)
#pragma unroll
        for (int n16 = 0; n16 < C::NT / 2; ++n16) {
          uint32_t b0, b1, b2, b3;
          const int row = n16 * 16 + (mi >> 1) * 8 + r8, ch = ks * 2 + (mi & 1);
          ldsm_x4(swz(kb + (ch >> 3) * C::kBlockBytes, row, ch & 7), b0, b1, b2, b3);
          mma_bf16(acc[2 * n16], qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3], b0, b1);
          mma_bf16(acc[2 * n16 + 1], qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3], b2, b3);
        }
    }
#pragma unroll
    for (int t = 0; t < C::NT; ++t)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int kl = t * 8 + (lane & 3) * 2 + (e & 1);
        const int row = (lane >> 2) + (e >> 1) * 8;
        float v = -INFINITY;
        if (key0 + i * KT + kl < valid) {
          v = rnd<bf16>(rnd<bf16>(acc[t][e]) * p.scale_bf16);
          mrow[e >> 1] = fmaxf(mrow[e >> 1], v);
        }
        sc[row * sc_ld + i * KT + kl] = __float2bfloat16_rn(v);
      }
    __syncwarp();   // every lane is done reading the slot
    if (lane == 0 && ok && j + NSW < 2 * nw) {
      fence_proxy_async();
      issue(j + NSW);
    }
  }
  // ---- row maxima: warps, then the cluster ----
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    mrow[h] = fmaxf(mrow[h], __shfl_xor_sync(0xffffffffu, mrow[h], 1));
    mrow[h] = fmaxf(mrow[h], __shfl_xor_sync(0xffffffffu, mrow[h], 2));
  }
  if ((lane & 3) == 0) {
    redm[warp * 16 + (lane >> 2)] = mrow[0];
    redm[warp * 16 + (lane >> 2) + 8] = mrow[1];
  }
  __syncthreads();
  if (threadIdx.x < 16) {
    const int r = threadIdx.x;
    cmax[r] = fmaxf(fmaxf(redm[r], redm[16 + r]), fmaxf(redm[32 + r], redm[48 + r]));
  }
  cluster_sync_all();
  if (threadIdx.x < 16) {
    const int r = threadIdx.x;
    float v[8];   // every remote read is issued before any is used
#pragma unroll
    for (int cr = 0; cr < 8; ++cr) v[cr] = cr < CS ? dsmem_ld_f32(dsmem_map(smem_u32(cmax + r), cr)) : -INFINITY;
    float M = v[0];
#pragma unroll
    for (int cr = 1; cr < 8; ++cr) M = fmaxf(M, v[cr]);
    Mrow[r] = M;
  }
  __syncthreads();
  // ---- row sums of exp(s - max) over this warp's keys, then the warps, then the cluster ----
  for (int r = 0; r < p.n_rep; ++r) {
    const float M = Mrow[r];
    float l = 0.f;
    if (M != -INFINITY)
      for (int j = 0; j < nw; ++j) {
        const int i = warp + 4 * j;
        for (int kl = lane; kl < KT; kl += 32)
          if (key0 + i * KT + kl < valid) l += expf(__bfloat162float(sc[r * sc_ld + i * KT + kl]) - M);
      }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    if (lane == 0) reds[warp * 16 + r] = l;
  }
  __syncthreads();
  if (threadIdx.x < 16) {
    const int r = threadIdx.x;
    csum[r] = r < p.n_rep ? ((reds[r] + reds[16 + r]) + reds[32 + r]) + reds[48 + r] : 0.f;   // warp order
  }
  cluster_sync_all();
  if (threadIdx.x < 16) {
    const int r = threadIdx.x;
    float v[8];
#pragma unroll
    for (int cr = 0; cr < 8; ++cr) v[cr] = cr < CS ? dsmem_ld_f32(dsmem_map(smem_u32(csum + r), cr)) : 0.f;
    float L = v[0];   // rank order
#pragma unroll
    for (int cr = 1; cr < 8; ++cr) L += v[cr];
    Lrow[r] = L;
  }
  __syncthreads();

  // ---- P . V over this warp's tiles ----
  const int g = lane >> 2, t4 = lane & 3;
  const bool lo_row = g < p.n_rep, hi_row = g + 8 < p.n_rep;
  const float Mlo = lo_row ? Mrow[g] : 0.f, Llo = lo_row ? Lrow[g] : 0.f;
  const float Mhi = hi_row ? Mrow[g + 8] : 0.f, Lhi = hi_row ? Lrow[g + 8] : 0.f;
  auto prob = [&](bool row_ok, int r, float M, float L, int i, int kl) -> float {
    if (!row_ok || key0 + i * KT + kl >= valid || M == -INFINITY || !(L > 0.f)) return 0.f;
    return rnd<bf16>(expf(__bfloat162float(sc[r * sc_ld + i * KT + kl]) - M) / L);
  };
  float oacc[HD / 8][4];
#pragma unroll
  for (int t = 0; t < HD / 8; ++t) oacc[t][0] = oacc[t][1] = oacc[t][2] = oacc[t][3] = 0.f;
  for (int j = 0; j < nw; ++j) {
    const int q = nw + j, slot = q % NSW, i = warp + 4 * j;
    if (ok && !mbar_wait_bounded(&wbar[slot], (q / NSW) & 1)) {
      set_status(p.status, JX_ERR_TIMEOUT);
      ok = false;
    }
    ok = __all_sync(0xffffffffu, ok);
    if (ok) {
      const uint32_t vb = smem_u32(wring + slot * C::kTileBytes);
#pragma unroll
      for (int kk = 0; kk < KT / 16; ++kk) {
        // A fragment of the probabilities: rows g, g+8; keys c, c+1 and c+8, c+9 of this 16-key step
        const int c = kk * 16 + t4 * 2;
        const uint32_t a0 = pack_bf16x2(prob(lo_row, g, Mlo, Llo, i, c), prob(lo_row, g, Mlo, Llo, i, c + 1));
        const uint32_t a1 = pack_bf16x2(prob(hi_row, g + 8, Mhi, Lhi, i, c), prob(hi_row, g + 8, Mhi, Lhi, i, c + 1));
        const uint32_t a2 = pack_bf16x2(prob(lo_row, g, Mlo, Llo, i, c + 8), prob(lo_row, g, Mlo, Llo, i, c + 9));
        const uint32_t a3 =
            pack_bf16x2(prob(hi_row, g + 8, Mhi, Lhi, i, c + 8), prob(hi_row, g + 8, Mhi, Lhi, i, c + 9));
#pragma unroll
        for (int n16 = 0; n16 < HD / 16; ++n16) {
          uint32_t b0, b1, b2, b3;
          const int row = kk * 16 + (mi & 1) * 8 + r8;
          const int ch = n16 * 2 + (mi >> 1);
          ldsm_x4_t(swz(vb + (ch >> 3) * C::kBlockBytes, row, ch & 7), b0, b1, b2, b3);
          mma_bf16(oacc[n16 * 2], a0, a1, a2, a3, b0, b1);
          mma_bf16(oacc[n16 * 2 + 1], a0, a1, a2, a3, b2, b3);
        }
      }
    }
    __syncwarp();
    if (lane == 0 && ok && q + NSW < 2 * nw) {
      fence_proxy_async();
      issue(q + NSW);
    }
  }
  // ---- partial outputs: warps in warp order, then the cluster in rank order ----
  __syncthreads();   // every warp is done with its slots: the ring becomes the partial-output buffer
#pragma unroll
  for (int t = 0; t < HD / 8; ++t)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int row = g + (e >> 1) * 8;
      const int col = t * 8 + t4 * 2 + (e & 1);
      opart[(warp * 16 + row) * HD + col] = oacc[t][e];
    }
  __syncthreads();
  for (int idx = threadIdx.x; idx < 16 * HD; idx += 128)
    opart[idx] = ((opart[idx] + opart[16 * HD + idx]) + opart[32 * HD + idx]) + opart[48 * HD + idx];
  cluster_sync_all();
  const int total = p.n_rep * HD;
  const int chunk = (total + CS - 1) / CS;
  const int e0 = (int)rank * chunk, e1 = min(total, e0 + chunk);
  for (int idx = e0 + threadIdx.x; idx < e1; idx += 128) {
    const uint32_t la = smem_u32(opart + idx);
    float v[8];
#pragma unroll
    for (int cr = 0; cr < 8; ++cr) v[cr] = cr < CS ? dsmem_ld_f32(dsmem_map(la, cr)) : 0.f;
    float sum = v[0];   // rank order
#pragma unroll
    for (int cr = 1; cr < 8; ++cr) sum += v[cr];
    const int row = idx / HD, col = idx % HD;
    const long long ocol = (long long)(kvh * p.n_rep + row) * HD + col;
    p.out[k128_offset(b, ocol, p.out_rp)] = __float2bfloat16_rn(sum);
  }
  cluster_sync_all();   // no CTA leaves while another may still read its shared memory
}


// ------------------------------------------------------------------------------------------------
// Queue form: the split form's two kernels as one persistent kernel.  The work is a list of items, the
// score items of every (head group, key split) and then the pv items of the same; each CTA claims
// items in list order from a global counter and, while it works on one item, has the TMA tiles of the
// next one in flight in its second shared-memory slot, so K tiles and then V tiles stream without a
// kernel boundary between the two phases.  A score item writes its rounded scores and (max, sum) as the
// scores kernel does and counts itself done for its head group (release); a pv item waits (bounded,
// acquire) until every split of its head group is scored, then forms the exact bf16 probabilities and
// P.V as the pv kernel does, and the last pv item of a group sums the split partials in split order.
// CTA c starts with score item c (so that its K tiles load before the wait on the previous kernel, as
// the scores kernel's do); the rest are claimed after that wait.  No deadlock: only score items are
// assigned up front, every score item precedes every pv item in the list and a CTA finishes an item
// before it starts the next, so when a pv item waits, the score items it waits for are held by CTAs
// that run them without waiting on anything, or that become resident as soon as an SM frees up (the
// grid is sized by occupancy).  After any error status, CTAs stop waiting and claiming, so a failure
// costs one bounded wait.  The sums, roundings and workspace are the split form's, so the outputs are
// bit-identical to it.
// ------------------------------------------------------------------------------------------------
template <int HD>
struct DqCfg {
  static constexpr int NB = HD / 64;
  static constexpr int TILE_BYTES = kDaTile * HD * 2;
  static constexpr int SLOT_BYTES = 2 * TILE_BYTES;      // one item: 128 keys
  static constexpr int OFF_QS = 2 * SLOT_BYTES;
  static constexpr int OFF_PT = OFF_QS + NB * 2048;
  static constexpr int OFF_BAR = OFF_PT + 16 * kPLd * 2;  // 4 mbarriers: [slot][tile]
  static constexpr int OFF_RED = OFF_BAR + 4 * 8;         // [4 warps][16 rows]
  static constexpr int OFF_ML = OFF_RED + 64 * 4;         // M[16], L[16]
  static constexpr int OFF_IT = OFF_ML + 32 * 4;          // claimed items of the two slots, ok flag
  static constexpr int BYTES = OFF_IT + 16 + 1024;         // + alignment of the dynamic base to 1 KB
};

template <int HD>
__global__ void __launch_bounds__(128) dattn_queue_kernel(const __grid_constant__ CUtensorMap kmap,
                                                          const __grid_constant__ CUtensorMap vmap, DAttnParams p) {
  using C = DqCfg<HD>;
  constexpr int NB = C::NB;
  constexpr int WCOLS = HD / 4;
  constexpr int NT = WCOLS / 8;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* qs = smem + C::OFF_QS;
  bf16* ptile = reinterpret_cast<bf16*>(smem + C::OFF_PT);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  float* red = reinterpret_cast<float*>(smem + C::OFF_RED);
  float* Ms = reinterpret_cast<float*>(smem + C::OFF_ML);
  float* Ls = Ms + 16;
  volatile int* items = reinterpret_cast<volatile int*>(smem + C::OFF_IT);   // [2] items, [2] ok flag

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.B * p.Hkv;
  const int n_score = G * p.n_splits, total = 2 * n_score;
  int* claim_ctr = p.qsync;
  int* done_ctas = p.qsync + 1;
  int* scored = p.qsync + 2;
  const bool fused = p.qkv != nullptr;

  // Item -> (pv?, batch row, KV head, split, key range).  Items whose split holds no valid key are
  // skipped at claim time.
  struct Item {
    int pv, b, kvh, split, t0, t1, valid, n_tiles, n_active;
  };
  auto decode = [&](int it) {
    Item x;
    x.pv = it >= n_score;
    const int r = x.pv ? it - n_score : it;
    const int g = r / p.n_splits;
    x.split = r - g * p.n_splits;
    x.b = g / p.Hkv;
    x.kvh = g - x.b * p.Hkv;
    int lo;
    key_range(p, x.b, lo, x.valid);
    x.t0 = lo + x.split * kDaKeys;
    x.t1 = min(x.t0 + kDaKeys, x.valid);
    x.n_tiles = x.t0 < x.valid ? (x.t1 - x.t0 + kDaTile - 1) / kDaTile : 0;
    x.n_active = (x.valid - lo + kDaKeys - 1) / kDaKeys;
    return x;
  };
  // CTA c starts with score item c (c < S0, no shared state: its tiles load before the wait on the
  // previous kernel); every later item is claimed from the counter, after that wait.  The counter and the
  // group counts belong to the previous launch until it has completed (a back-to-back launch of this
  // kernel on the same workspace starts while the previous one runs), so nothing shared is touched before.
  const int S0 = (int)gridDim.x < n_score ? (int)gridDim.x : n_score;
  auto claim = [&]() {
    for (;;) {
      if (p.status && *reinterpret_cast<volatile int*>(p.status) != 0) return -1;   // an error: stop taking work
      const int it = S0 + atomicAdd(claim_ctr, 1);
      if (it >= total) return -1;
      if (decode(it).n_tiles > 0) return it;
    }
  };
  // tile i of item x holds this step's key (position valid - 1)
  auto holds_new = [&](const Item& x, int i) {
    return x.t0 + i * kDaTile <= x.valid - 1 && x.valid - 1 < x.t0 + (i + 1) * kDaTile;
  };
  auto issue_tile = [&](const Item& x, int slot, int i) {
    uint64_t* bb = &bar[slot * 2 + i];
    mbar_arrive_expect_tx(bb, C::TILE_BYTES);
    const int y = (int)(p.layer_row0 + (long long)x.b * p.T + x.t0 + i * kDaTile);
    uint8_t* dst = smem + slot * C::SLOT_BYTES + i * C::TILE_BYTES;
#pragma unroll
    for (int c = 0; c < NB; ++c) tma_load_2d(dst + c * 8192, x.pv ? &vmap : &kmap, x.kvh * HD + c * 64, y, bb);
  };
  // Thread 0: every barrier of the slot gets one arrival per item (a tile, or a plain arrive for a
  // tile the item does not have).  Returns the tile left to issue later (-1: none): this step's key or
  // value when it is not complete yet (before the wait on the previous kernel without the fused
  // append; the fused append's value, written by a score item of this kernel).
  auto issue_item = [&](int it, int slot, bool before_wait) {
    const Item x = decode(it);
    fence_proxy_async();   // the slot's previous contents were read through the generic proxy
    int late = -1;
    for (int i = 0; i < 2; ++i) {
      if (i >= x.n_tiles) {
        mbar_arrive(&bar[slot * 2 + i]);
      } else if (holds_new(x, i) && ((x.pv && fused) || (!fused && before_wait))) {
        late = i;
      } else {
        issue_tile(x, slot, i);
      }
    }
    return late;
  };

  int late0 = -1, late1 = -1;   // thread 0 only: the tile left to issue later, per slot
  if (threadIdx.x == 0) {
    prefetch_tmap(&kmap);
    prefetch_tmap(&vmap);
    for (int i = 0; i < 4; ++i) mbar_init(&bar[i], 1);
    fence_barrier_init();
    const int first = (int)blockIdx.x < S0 && decode(blockIdx.x).n_tiles > 0 ? (int)blockIdx.x : -1;
    items[0] = first;
    if (first >= 0) late0 = issue_item(first, 0, true);
  }
  pdl_wait();
  pdl_trigger();
  if (threadIdx.x == 0) {
    if (items[0] < 0) {
      const int it = claim();
      items[0] = it;
      if (it >= 0) late0 = issue_item(it, 0, false);
    } else if (late0 >= 0) {
      issue_tile(decode(items[0]), 0, late0);   // (a score item: this step's key after the wait)
      late0 = -1;
    }
  }
  if (threadIdx.x == 0) items[2] = 1;
  __syncthreads();

  const int mi = lane >> 3, r8 = lane & 7;
  const int r_lo = lane >> 2, r_hi = r_lo + 8;
  uint32_t phases = 0;   // bit s: parity of slot s's barriers for its next item
  int slot = 0;
  for (int cur = items[0]; cur >= 0;) {
    if (threadIdx.x == 0) {
      const int nxt = claim();
      items[slot ^ 1] = nxt;
      if (nxt >= 0) {
        const int lt = issue_item(nxt, slot ^ 1, false);
        if (slot) late0 = lt;
        else late1 = lt;
      }
    }
    const Item x = decode(cur);
    const int g = x.b * p.Hkv + x.kvh;
    uint8_t* tiles = smem + slot * C::SLOT_BYTES;
    uint64_t* sb = &bar[slot * 2];
    const uint32_t par = (phases >> slot) & 1u;
    if (!x.pv) {
      // ---------------- score item (the scores kernel's work on one split) ----------------
      int pos = x.valid - 1;
      if (fused && pos >= p.max_pos) {
        if (threadIdx.x == 0) set_status(p.status, JX_ERR_RANGE);
        pos = 0;
      }
      const bf16* qkv_row = fused ? p.qkv + (long long)x.b * p.ld_qkv : nullptr;
      for (int idx = threadIdx.x; idx < 16 * (HD / 8); idx += 128) {
        const int r = idx / (HD / 8), cg = idx % (HD / 8);
        uint4 v = make_uint4(0, 0, 0, 0);
        if (r < p.n_rep) {
          if (fused)
            v = rope8(qkv_row + (long long)(x.kvh * p.n_rep + r) * HD, cg * 8, HD, p.rd, p.cos, p.sin, pos);
          else
            v = *reinterpret_cast<const uint4*>(p.q + ((long long)x.b * p.Hq + x.kvh * p.n_rep + r) * HD + cg * 8);
        }
        const uint32_t a = swz(smem_u32(qs + (cg >> 3) * 2048), r, cg & 7);
        asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(a), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w));
      }
      if (fused && x.valid - 1 >= x.t0 && x.valid - 1 < x.t1) {
        // append this step's rotated k and its v to the cache; patch k into the loaded tile
        const int kpos = x.valid - 1;
        const int tile = (kpos - x.t0) / kDaTile, trow = (kpos - x.t0) % kDaTile;
        const long long crow =
            (p.layer_row0 + (long long)x.b * p.T + kpos) * ((long long)p.Hkv * HD) + (long long)x.kvh * HD;
        uint4 k8 = make_uint4(0, 0, 0, 0);
        const int j0 = threadIdx.x * 8;
        if (j0 < HD) {
          k8 = rope8(qkv_row + (long long)(p.Hq + x.kvh) * HD, j0, HD, p.rd, p.cos, p.sin, pos);
          const uint4 v8 = *reinterpret_cast<const uint4*>(qkv_row + (long long)(p.Hq + p.Hkv + x.kvh) * HD + j0);
          *reinterpret_cast<uint4*>(p.k_cache + crow + j0) = k8;
          *reinterpret_cast<uint4*>(p.v_cache + crow + j0) = v8;
        }
        const bool landed = mbar_wait_bounded(&sb[tile], par);
        if (!landed) {
          set_status(p.status, JX_ERR_TIMEOUT);
          items[2] = 0;
        }
        if (landed && j0 < HD) {
          const uint32_t a = swz(smem_u32(tiles + tile * C::TILE_BYTES + (j0 >> 6) * 8192), trow, (j0 & 63) >> 3);
          asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(a), "r"(k8.x), "r"(k8.y), "r"(k8.z), "r"(k8.w));
        }
      }
      __syncthreads();
      float sv[2][2][4];
      float mrow[2] = {-INFINITY, -INFINITY};
      bool ok = items[2] != 0;
#pragma unroll
      for (int i = 0; i < 2; ++i) {
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) sv[i][nt][e] = -INFINITY;
        if (i >= x.n_tiles || !ok) continue;
        if (!mbar_wait_bounded(&sb[i], par)) {
          set_status(p.status, JX_ERR_TIMEOUT);
          ok = false;
          continue;
        }
        float acc[2][4] = {};
        const uint32_t kb = smem_u32(tiles + i * C::TILE_BYTES);
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
            const int t = x.t0 + i * kDaTile + warp * 16 + nt * 8 + (lane & 3) * 2 + (e & 1);
            if (t < x.t1) {
              const float v = rnd<bf16>(rnd<bf16>(acc[nt][e]) * p.scale_bf16);
              sv[i][nt][e] = v;
              mrow[e >> 1] = fmaxf(mrow[e >> 1], v);
            }
          }
      }
      ok = __syncthreads_and(ok) != 0;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        mrow[h] = fmaxf(mrow[h], __shfl_xor_sync(0xffffffffu, mrow[h], 1));
        mrow[h] = fmaxf(mrow[h], __shfl_xor_sync(0xffffffffu, mrow[h], 2));
      }
      if ((lane & 3) == 0) {
        red[warp * 16 + r_lo] = mrow[0];
        red[warp * 16 + r_hi] = mrow[1];
      }
      __syncthreads();
      float m[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int row = r_lo + h * 8;
        m[h] = fmaxf(fmaxf(red[row], red[16 + row]), fmaxf(red[32 + row], red[48 + row]));
      }
      __syncthreads();
      float l[2] = {0.f, 0.f};
      const long long sc_row = ((long long)x.b * p.Hq + x.kvh * p.n_rep) * p.T;
#pragma unroll
      for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int row = r_lo + (e >> 1) * 8;
            const int t = x.t0 + i * kDaTile + warp * 16 + nt * 8 + (lane & 3) * 2 + (e & 1);
            if (t < x.t1 && row < p.n_rep) {
              const float v = sv[i][nt][e];
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
        red[warp * 16 + r_lo] = l[0];
        red[warp * 16 + r_hi] = l[1];
      }
      __syncthreads();
      if (warp == 0 && (lane & 3) == 0) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int row = r_lo + h * 8;
          if (row < p.n_rep) {
            float* st = p.stats + (((long long)x.b * p.Hq + x.kvh * p.n_rep + row) * p.n_splits + x.split) * 2;
            st[0] = m[h];
            st[1] = (red[row] + red[16 + row]) + (red[32 + row] + red[48 + row]);
          }
        }
      }
      __threadfence();
      __syncthreads();
      // counted done even after a timeout (the status is set), so the group's pv items do not wait
      if (threadIdx.x == 0) atomicAdd(&scored[g], 1);
    } else {
      // ---------------- pv item (the pv kernel's work on one split) ----------------
      if (threadIdx.x == 0) {
        bool ok = true;
        if (ld_acquire_gpu(&scored[g]) < x.n_active) {
          const uint64_t w0 = globaltimer_ns();
          while (ld_acquire_gpu(&scored[g]) < x.n_active) {
            if (p.status && *reinterpret_cast<volatile int*>(p.status) != 0) {   // another CTA failed: give up
              ok = false;
              break;
            }
            if (globaltimer_ns() - w0 > kWaitLimitNs) {
              set_status(p.status, JX_ERR_TIMEOUT);
              ok = false;
              break;
            }
          }
        }
        const int lt = slot ? late1 : late0;
        if (lt >= 0) {
          // this step's value was written by a score item of this kernel: order it before the copy
          fence_proxy_async_global();
          issue_tile(x, slot, lt);
          if (slot) late1 = -1;
          else late0 = -1;
        }
        items[2] = ok ? 1 : 0;
      }
      __syncthreads();
      bool ok = items[2] != 0;
      if (threadIdx.x < 16) {
        const int row = threadIdx.x;
        float M = -INFINITY, L = 0.f;
        if (row < p.n_rep) {
          const float* st = p.stats + ((long long)x.b * p.Hq + x.kvh * p.n_rep + row) * p.n_splits * 2;
          for (int s2 = 0; s2 < x.n_active; ++s2) M = fmaxf(M, __ldcg(st + s2 * 2));
          for (int s2 = 0; s2 < x.n_active; ++s2) L += __ldcg(st + s2 * 2 + 1) * expf(__ldcg(st + s2 * 2) - M);
        }
        Ms[row] = M;
        Ls[row] = L;
      }
      __syncthreads();
      for (int idx = threadIdx.x; idx < 16 * kDaKeys; idx += 128) {
        const int row = idx / kDaKeys, k = idx % kDaKeys, t = x.t0 + k;
        float pv = 0.f;
        if (row < p.n_rep && t < x.t1) {
          const float sc = __ldcg(p.sc + ((long long)x.b * p.Hq + x.kvh * p.n_rep + row) * p.T + t);
          pv = rnd<bf16>(expf(sc - Ms[row]) / Ls[row]);
        }
        ptile[row * kPLd + k] = __float2bfloat16_rn(pv);
      }
      __syncthreads();
      float acc[NT][4] = {};
      for (int i = 0; i < x.n_tiles; ++i) {
        if (!mbar_wait_bounded(&sb[i], par)) {
          set_status(p.status, JX_ERR_TIMEOUT);
          ok = false;
          break;
        }
        if (!ok) continue;
        const uint32_t vb = smem_u32(tiles + i * C::TILE_BYTES);
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
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int row = (e >> 1) ? r_hi : r_lo;
          const int col = warp * WCOLS + nt * 8 + (lane & 3) * 2 + (e & 1);
          if (row < p.n_rep)
            p.opart[(((long long)x.b * p.Hq + x.kvh * p.n_rep + row) * p.n_splits + x.split) * HD + col] = acc[nt][e];
        }
      __threadfence();
      __syncthreads();
      if (threadIdx.x == 0) items[3] = atomicAdd(&p.counters[g], 1) == x.n_active - 1;
      __syncthreads();
      if (items[3]) {
        __threadfence();
        for (int idx = threadIdx.x; idx < p.n_rep * HD; idx += 128) {
          const int row = idx / HD, col = idx % HD;
          const float* src = p.opart + (((long long)x.b * p.Hq + x.kvh * p.n_rep + row) * p.n_splits) * HD + col;
          float sum = 0.f;
          for (int s2 = 0; s2 < x.n_active; ++s2) sum += __ldcg(src + (long long)s2 * HD);
          const long long ocol = (long long)(x.kvh * p.n_rep + row) * HD + col;
          p.out[k128_offset(x.b, ocol, p.out_rp)] = __float2bfloat16_rn(sum);
        }
        if (threadIdx.x == 0) {
          p.counters[g] = 0;
          scored[g] = 0;
        }
      }
    }
    phases ^= 1u << slot;
    if (threadIdx.x == 0) items[2] = 1;
    __syncthreads();   // the slot is free; the next item's claim is visible
    slot ^= 1;
    cur = items[slot];
  }
  if (threadIdx.x == 0 && atomicAdd(done_ctas, 1) == (int)gridDim.x - 1) {
    // every CTA has made its last claim: reset the queue for the next call
    *claim_ctr = 0;
    *done_ctas = 0;
  }
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

// scores [B, Hq, T], split statistics [B, Hq, n_splits, 2], split partials [B, Hq, n_splits, hd] (float32),
// then the queue form's counters (2 + B * Hkv ints; B * Hq bounds B * Hkv).
long long dattn_workspace_bytes(int B, int Hq, int T, int hd, int n_splits) {
  const long long sc = (long long)B * Hq * T;
  const long long st = (long long)B * Hq * n_splits * 2;
  const long long op = (long long)B * Hq * n_splits * hd;
  return (sc + st + op) * 4 + (2 + (long long)B * Hq) * 4;
}

int dattn_n_splits(int T, int window) {
  const int range = (window > 0 && window < T) ? window : T;
  return (range + kDaKeys - 1) / kDaKeys;
}

template <int HD, int RQ>
static int launch_dattn_rq(const CUtensorMap& km, const CUtensorMap& vm, const DAttnParams& p, bool column_pv,
                           bool pdl, cudaStream_t s) {
  const int smem_a = 1024 + 2 * kDaTile * HD * 2 + (HD / 64) * RQ * 128 + 16 + 4 * 16 * 4;
  const int smem_b = 1024 + 2 * kDaTile * HD * 2 + 16 + 32 * 4 + RQ * kPLd * 2;
  const int smem_c = 1024 + kPcStages * 8192 + 4 * 16 * kPcLd * 2 + kPcStages * 8;
  static bool configured = false;
  if (!configured) {
    if (cudaFuncSetAttribute(dattn_scores_kernel<HD, RQ>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_a) !=
            cudaSuccess ||
        cudaFuncSetAttribute(dattn_pv_kernel<HD, RQ>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_b) != cudaSuccess ||
        cudaFuncSetAttribute(dattn_pvcol_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_c) != cudaSuccess)
      return JX_ERR_CUDA;
    configured = true;
  }
  cudaLaunchConfig_t cfg = {};
  // Splits vary slowest: CTAs are dispatched in linear block order, so the splits past the valid keys
  // (the grid is sized by the buffer length; they exit at once) come last, and a grid larger than one
  // wave of resident CTAs leaves only those to the second wave.
  cfg.gridDim = dim3(p.Hkv, p.B, p.n_splits);
  cfg.blockDim = dim3(128);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cfg.dynamicSmemBytes = smem_a;
  if (launch_ex(&cfg, dattn_scores_kernel<HD, RQ>, km, p) != cudaSuccess) return JX_ERR_CUDA;
  if (column_pv) {
    cfg.gridDim = dim3(HD / 64, p.Hkv, p.B);
    cfg.dynamicSmemBytes = smem_c;
    return launch_ex(&cfg, dattn_pvcol_kernel<HD>, vm, p) == cudaSuccess ? JX_OK : JX_ERR_CUDA;
  }
  cfg.dynamicSmemBytes = smem_b;
  if (launch_ex(&cfg, dattn_pv_kernel<HD, RQ>, vm, p) != cudaSuccess) return JX_ERR_CUDA;
  return JX_OK;
}

template <int HD>
static int launch_dattn(const CUtensorMap& km, const CUtensorMap& vm, const DAttnParams& p, bool column_pv, bool pdl,
                        cudaStream_t s) {
  return p.n_rep <= 8 ? launch_dattn_rq<HD, 8>(km, vm, p, column_pv, pdl, s)
                      : launch_dattn_rq<HD, 16>(km, vm, p, column_pv, pdl, s);
}

// Cluster shape of the single-pass form for B x Hkv head groups over a key range of `range` keys: as
// many CTAs per head group as fill the SMs once (one CTA per group when there are at least as many
// groups as SMs), more when a CTA would hold more than kWaMaxKeys keys, at most 8.  Returns false when
// the range needs more (the split form runs then).
static bool fused_shape(int range, int kt_keys, int max_tiles, int groups, int sms, int& cs, int& kt) {
  const int tiles = (range + kt_keys - 1) / kt_keys;
  cs = groups >= sms ? 1 : sms / groups;
  const int need = (tiles + max_tiles - 1) / max_tiles;
  if (cs < need) cs = need;
  if (cs > tiles) cs = tiles;
  if (cs > 8) cs = 8;
  if (cs < 1) cs = 1;
  kt = (tiles + cs - 1) / cs;
  return kt <= max_tiles;
}

template <int HD>
static int launch_dattn_fused(const jx_dattn_args& a, FAttnParams& p, int sms, bool pdl, cudaStream_t s) {
  using C = WaCfg<HD>;
  const int range = (a.window > 0 && a.window < a.T) ? a.window : a.T;
  int cs, kt;
  if (!fused_shape(range, C::KT, C::kMaxTiles, a.B * a.Hkv, sms, cs, kt)) return JX_ERR_SHAPE;
  CUtensorMap km, vm;
  const long long cols = (long long)a.Hkv * a.hd;
  int rc = make_tmap_2d_bf16_box(&km, a.k_base, a.cache_rows, cols, cols, C::KT);
  if (rc == JX_OK) rc = make_tmap_2d_bf16_box(&vm, a.v_base, a.cache_rows, cols, cols, C::KT);
  if (rc != JX_OK) return rc;
  static bool configured = false;
  if (!configured) {
    if (cudaFuncSetAttribute(dattn_warp_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             C::bytes(C::kMaxTiles)) != cudaSuccess)
      return JX_ERR_CUDA;
    configured = true;
  }
  p.kt_cap = kt;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(cs, p.Hkv, p.B);
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = C::bytes(kt);
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
  return launch_ex(&cfg, dattn_warp_kernel<HD>, km, vm, p) == cudaSuccess ? JX_OK : JX_ERR_CUDA;
}

template <int HD>
static int launch_dattn_csplit(const CUtensorMap& km, const CUtensorMap& vm, const DAttnParams& p, bool pdl,
                               cudaStream_t s) {
  const int smem = 1024 + 2 * kDaTile * HD * 2 + (HD / 64) * 2048 + 16 * kPLd * 2 + 4 * 8 + 64 * 4;
  static bool configured = false;
  if (!configured) {
    if (cudaFuncSetAttribute(dattn_csplit_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess ||
        cudaFuncSetAttribute(dattn_csplit_kernel<HD>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
      return JX_ERR_CUDA;
    configured = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.n_splits, p.Hkv, p.B);
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = p.n_splits;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  return launch_ex(&cfg, dattn_csplit_kernel<HD>, km, vm, p) == cudaSuccess ? JX_OK : JX_ERR_CUDA;
}

template <int HD>
static int launch_dattn_queue(const CUtensorMap& km, const CUtensorMap& vm, const DAttnParams& p, bool pdl,
                              cudaStream_t s) {
  using C = DqCfg<HD>;
  static int per_sm = 0, sms = 0;
  if (!per_sm) {
    if (cudaFuncSetAttribute(dattn_queue_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::BYTES) !=
        cudaSuccess)
      return JX_ERR_CUDA;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, dattn_queue_kernel<HD>, 128, C::BYTES) != cudaSuccess)
      return JX_ERR_CUDA;
    if (per_sm < 1) per_sm = 1;
  }
  const long long items = 2LL * p.B * p.Hkv * p.n_splits;
  const long long cap = (long long)per_sm * sms;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(items < cap ? items : cap));
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = C::BYTES;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return launch_ex(&cfg, dattn_queue_kernel<HD>, km, vm, p) == cudaSuccess ? JX_OK : JX_ERR_CUDA;
}

// 0: by shape (the split form), 1: split form (split pv), 2: single-pass form, 3: split scores + column
// pv, 4: cluster-split form (key ranges up to 16 splits of 128 keys), 5: queue form.  No alternative is chosen by
// shape: the cluster-split form measured 23.1 / 50.3 us against 17.6 / 43.5 us for the split form at
// context 640 / 2000 (B=16; its T-sized grid of clusters does not fit one wave), the single-pass form
// 22.7 us against 20.4 us at context 640 (its fewer warps leave the mma.sync latency exposed), and the
// column pv 22.4 / 122.7 us against 17.6 / 87.4 us at context 640 / 4096 (each
// warp forms the probabilities of its tiles serially, one L2 round trip per tile), and the queue form
// 30.0 / 153 us against 17.8 / 88 us (each CTA works through its items one after another).
static int g_dattn_impl = 0;
void set_dattn_impl(int impl) { g_dattn_impl = impl; }

int run_decode_attention(const jx_dattn_args& a, bool pdl, cudaStream_t stream) {
  if (a.B <= 0 || a.Hkv <= 0 || a.Hq % a.Hkv || a.T <= 0) return JX_ERR_SHAPE;
  const int n_rep = a.Hq / a.Hkv;
  if (n_rep > 16) return JX_ERR_SHAPE;
  if (a.hd != 64 && a.hd != 128 && a.hd != 256) return JX_ERR_SHAPE;
  if (a.qkv) {
    // fused RoPE + append: the split and queue forms; 16-byte rows of the projection output and tables
    if (g_dattn_impl >= 2 && g_dattn_impl != 5) return JX_ERR_UNSUPPORTED;
    if (!a.cos || !a.sin || a.rd <= 0 || a.rd > a.hd || (a.rd & 1) || a.max_pos <= 0 ||
        a.ld_qkv < (long long)(a.Hq + 2 * a.Hkv) * a.hd || (a.ld_qkv & 7) || (reinterpret_cast<uintptr_t>(a.qkv) & 15))
      return JX_ERR_ARG;
  } else if (reinterpret_cast<uintptr_t>(a.q) & 15) {
    return JX_ERR_ARG;
  }
  if (a.out_rp < a.B || a.out_rp % 8) return JX_ERR_ARG;   // the K128 output must hold every batch row

  if (g_dattn_impl == 2) {
    int sms = 148, dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    FAttnParams f;
    f.B = a.B;
    f.Hq = a.Hq;
    f.Hkv = a.Hkv;
    f.n_rep = n_rep;
    f.T = a.T;
    f.window = a.window;
    f.kt_cap = 0;
    f._pad0 = 0;
    f.layer_row0 = a.layer_row0;
    f.q = reinterpret_cast<const bf16*>(a.q);
    f.len_ptr = a.len_ptr;
    f.len_add = a.len_add;
    f.scale_bf16 = __bfloat162float(__float2bfloat16_rn(a.scale));
    f.out = reinterpret_cast<bf16*>(a.out);
    f.out_rp = a.out_rp;
    f.status = a.status;
    int frc;
    switch (a.hd) {
      case 64: frc = launch_dattn_fused<64>(a, f, sms, pdl, stream); break;
      case 128: frc = launch_dattn_fused<128>(a, f, sms, pdl, stream); break;
      default: frc = launch_dattn_fused<256>(a, f, sms, pdl, stream); break;
    }
    if (frc != JX_ERR_SHAPE || g_dattn_impl == 2) return frc;   // key range too long: the split form
  }

  CUtensorMap km, vm;
  const long long cols = (long long)a.Hkv * a.hd;
  int rc = make_tmap_2d_bf16(&km, a.k_base, a.cache_rows, cols, cols);
  if (rc == JX_OK) rc = make_tmap_2d_bf16(&vm, a.v_base, a.cache_rows, cols, cols);
  if (rc != JX_OK) return rc;

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
  p.qkv = reinterpret_cast<const bf16*>(a.qkv);
  p.ld_qkv = a.ld_qkv;
  p.cos = reinterpret_cast<const bf16*>(a.cos);
  p.sin = reinterpret_cast<const bf16*>(a.sin);
  p.rd = a.rd;
  p.max_pos = a.max_pos;
  p.k_cache = reinterpret_cast<bf16*>(const_cast<void*>(a.k_base));
  p.v_cache = reinterpret_cast<bf16*>(const_cast<void*>(a.v_base));
  p.qsync = reinterpret_cast<int*>(p.opart + (long long)a.B * a.Hq * n_splits * a.hd);
  if (g_dattn_impl == 5) {
    switch (a.hd) {
      case 64: return launch_dattn_queue<64>(km, vm, p, pdl, stream);
      case 128: return launch_dattn_queue<128>(km, vm, p, pdl, stream);
      default: return launch_dattn_queue<256>(km, vm, p, pdl, stream);
    }
  }
  if (g_dattn_impl == 4) {
    if (n_splits > 16) return JX_ERR_SHAPE;
    switch (a.hd) {
      case 64: return launch_dattn_csplit<64>(km, vm, p, pdl, stream);
      case 128: return launch_dattn_csplit<128>(km, vm, p, pdl, stream);
      default: return launch_dattn_csplit<256>(km, vm, p, pdl, stream);
    }
  }
  const bool column_pv = g_dattn_impl == 3;
  switch (a.hd) {
    case 64: return launch_dattn<64>(km, vm, p, column_pv, pdl, stream);
    case 128: return launch_dattn<128>(km, vm, p, column_pv, pdl, stream);
    default: return launch_dattn<256>(km, vm, p, column_pv, pdl, stream);
  }
}

}  // namespace jxb
