// Prefill attention on tensor cores (bfloat16, head_dim 64 / 128 / 256): causal, sliding-window and
// prefix-padding masks over the KV cache, with the reference's rounding points reproduced exactly.
//
// Attention.mha for q_len > 1 (nn/attention.py:321-400): scores = bf16(bf16(q.k) * bf16(attn_scale)),
// key j visible to query i iff j <= i (causal, :366-368), j > i - window (sliding window, :371-372) and
// j < len (right-padded mask, :382-383); softmax in float32 cast to bf16 (:388-389); o = bf16(p.v).
// A query row with no visible key attends uniformly to every slot of the buffer (:385-386): the first
// uniform_T slots, the reference's cache length when the prompt ran (the rest are zero then).
//
// One CTA per (64 query rows, HPC query heads of one KV head, batch row), the last query tiles (the
// most key tiles) first; each warp owns 16 rows of one head, so the HPC heads' warps share every K / V
// tile the CTA loads (HPC = 4, 2 or 1: the largest that divides the heads per KV head).  To round the normalised
// probabilities exactly as the reference does, the kernel makes two passes over the key tiles: pass 1
// finds each row's max and exp-sum, pass 2 recomputes the identical scores, forms bf16(exp(s-m)/l) and
// accumulates P.V.  K and V tiles arrive by TMA (the cache's 2-D tensor maps, 128-byte swizzle) in a
// two-stage ring; QK^T and PV run on mma.sync.
#include "common.cuh"

namespace jxb {

int make_tmap_2d_bf16_box(CUtensorMap* map, const void* base, long long rows, long long cols,
                          long long row_stride_elems, int box_rows);

struct PAttnParams {
  int B, S, Hq, Hkv, n_rep, T;
  int uniform_T;         // slots of the all-masked rows' uniform attention (<= T)
  long long layer_row0;
  const bf16* q;         // [B*S, Hq, HD]
  const bf16* v_plain;   // cache base of V (row-major [rows, Hkv*HD]) for the all-masked fallback
  const int* len_ptr;
  int len_add, window;
  float scale_bf16;
  bf16* out;
  long long out_rp;
  int* status;
};

__device__ __forceinline__ uint32_t pswz(uint32_t block_base, int r, int c) {
  return block_base + r * 128 + ((c ^ (r & 7)) << 4);
}

template <int HD, int KT, int HPC>
__global__ void __launch_bounds__(128 * HPC) pattn_kernel(const __grid_constant__ CUtensorMap kmap,
                                                          const __grid_constant__ CUtensorMap vmap, PAttnParams p) {
  constexpr int NT = 128 * HPC;                  // threads
  constexpr int NB = HD / 64;                    // 64-column blocks per head
  constexpr int QBLK = 64 * 128;                 // bytes of one [64 rows x 64 cols] Q block
  constexpr int TBLK = KT * 128;                 // bytes of one [KT rows x 64 cols] K/V block
  constexpr int TILE = KT * HD * 2;
  constexpr int NS = KT / 8;                     // score n8 tiles per warp
  constexpr int NO = HD / 8;                     // output n8 tiles per warp
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* qs_all = smem;                        // HPC heads x NB * QBLK
  uint8_t* ks = qs_all + HPC * NB * QBLK;        // 2 stages
  uint8_t* vs = ks + 2 * TILE;                   // 2 stages
  uint64_t* bar = reinterpret_cast<uint64_t*>(vs + 2 * TILE);
  int* dead_rows = reinterpret_cast<int*>(bar + 2);   // [HPC][64]

  // CTAs start in linear grid order; the query tiles with the most key tiles (the last ones, causal) go
  // first, so that the short ones fill in at the end instead of a long one starting last.
  const int per_qt = gridDim.y * gridDim.z;
  const int lin = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
  const int qt = gridDim.x - 1 - lin / per_qt, rest = lin % per_qt;
  const int b = rest / gridDim.y;
  const int h0 = (rest % gridDim.y) * HPC;       // first query head of this CTA
  const int kvh = h0 / p.n_rep;
  const int hw = (threadIdx.x >> 5) >> 2;        // this warp's head within the CTA
  const int h = h0 + hw;
  const int warp = (threadIdx.x >> 5) & 3, lane = threadIdx.x & 31;   // warp within its head's rows
  uint8_t* qs = qs_all + hw * NB * QBLK;
  const int s0 = qt * 64;
  pdl_trigger();
  pdl_wait();
  int valid = p.len_ptr[b] + p.len_add;
  if (valid > p.T) {
    set_status(p.status, JX_ERR_RANGE);
    valid = p.T;
  }
  const int s_max = min(s0 + 63, p.S - 1);
  const int j_hi = min(s_max, valid - 1);
  const int j_lo = p.window > 0 ? max(0, s0 - p.window + 1) : 0;
  const int n_tiles = j_hi >= j_lo ? (j_hi - j_lo + KT) / KT : 0;
  const int n_loads = 2 * n_tiles;

  auto issue = [&](int i) {
    const int st = i & 1;
    const int t = i % n_tiles;
    const bool with_v = i >= n_tiles;
    mbar_arrive_expect_tx(&bar[st], with_v ? 2 * TILE : TILE);
    const int y = (int)(p.layer_row0 + (long long)b * p.T + j_lo + t * KT);
#pragma unroll
    for (int c = 0; c < NB; ++c) {
      tma_load_2d(ks + st * TILE + c * TBLK, &kmap, kvh * HD + c * 64, y, &bar[st]);
      if (with_v) tma_load_2d(vs + st * TILE + c * TBLK, &vmap, kvh * HD + c * 64, y, &bar[st]);
    }
  };
  if (threadIdx.x == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    fence_barrier_init();
    if (n_loads > 0) issue(0);
    if (n_loads > 1) issue(1);
  }
  if (threadIdx.x < 64 * HPC) dead_rows[threadIdx.x] = 0;
  // Q tiles of the CTA's heads (rows past S are zero)
  for (int idx = threadIdx.x; idx < HPC * 64 * (HD / 8); idx += NT) {
    const int hl = idx / (64 * (HD / 8)), rem = idx % (64 * (HD / 8));
    const int r = rem / (HD / 8), cg = rem % (HD / 8);
    uint4 v = make_uint4(0, 0, 0, 0);
    if (s0 + r < p.S)
      v = *reinterpret_cast<const uint4*>(p.q + (((long long)b * p.S + s0 + r) * p.Hq + h0 + hl) * HD + cg * 8);
    const uint32_t a = pswz(smem_u32(qs_all + hl * NB * QBLK + (cg >> 3) * QBLK), r, cg & 7);
    asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(a), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w));
  }
  __syncthreads();

  const int mi = lane >> 3, r8 = lane & 7;
  const int row_lo = s0 + warp * 16 + (lane >> 2), row_hi = row_lo + 8;
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
  float o[NO][4];
#pragma unroll
  for (int i = 0; i < NO; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[i][e] = 0.f;
  bool ok = true;

  for (int i = 0; i < n_loads; ++i) {
    const int st = i & 1;
    const int t = i % n_tiles;
    const bool pass2 = i >= n_tiles;
    if (ok && !mbar_wait_bounded(&bar[st], (i >> 1) & 1)) {
      set_status(p.status, JX_ERR_TIMEOUT);
      ok = false;
    }
    if (ok) {
      const int jb = j_lo + t * KT;
      // S = Q K^T for this warp's 16 rows and the KT keys of the tile
      float sacc[NS][4];
#pragma unroll
      for (int n = 0; n < NS; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) sacc[n][e] = 0.f;
      const uint32_t kb = smem_u32(ks + st * TILE);
#pragma unroll
      for (int kk = 0; kk < HD / 16; ++kk) {
        uint32_t a0, a1, a2, a3;
        {
          const int row = warp * 16 + (mi & 1) * 8 + r8, ch = kk * 2 + (mi >> 1);
          ldsm_x4(pswz(smem_u32(qs + (ch >> 3) * QBLK), row, ch & 7), a0, a1, a2, a3);
        }
#pragma unroll
        for (int g = 0; g < NS / 2; ++g) {
          uint32_t b0, b1, b2, b3;
          const int row = g * 16 + (mi >> 1) * 8 + r8, ch = kk * 2 + (mi & 1);
          ldsm_x4(pswz(kb + (ch >> 3) * TBLK, row, ch & 7), b0, b1, b2, b3);
          mma_bf16(sacc[2 * g], a0, a1, a2, a3, b0, b1);
          mma_bf16(sacc[2 * g + 1], a0, a1, a2, a3, b2, b3);
        }
      }
      // reference rounding and masks
#pragma unroll
      for (int n = 0; n < NS; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int row = (e >> 1) ? row_hi : row_lo;
          const int j = jb + n * 8 + (lane & 3) * 2 + (e & 1);
          bool vis = j <= row && j < valid && j <= j_hi;
          if (p.window > 0 && j <= row - p.window) vis = false;
          sacc[n][e] = vis ? rnd<bf16>(rnd<bf16>(sacc[n][e]) * p.scale_bf16) : -INFINITY;
        }
      if (!pass2) {
        // online row max / exp-sum
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          float tm = -INFINITY;
#pragma unroll
          for (int n = 0; n < NS; ++n) tm = fmaxf(tm, fmaxf(sacc[n][hh * 2], sacc[n][hh * 2 + 1]));
          tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, 1));
          tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, 2));
          const float mn = fmaxf(m[hh], tm);
          // Rows differ in whether they see any key of this tile (sliding window), so every lane
          // must still reach the full-warp shuffles below: guard the arithmetic, not the shuffles.
          const bool live = mn != -INFINITY;
          float ts = 0.f;
#pragma unroll
          for (int n = 0; n < NS; ++n) {
            if (live && sacc[n][hh * 2] != -INFINITY) ts += expf(sacc[n][hh * 2] - mn);
            if (live && sacc[n][hh * 2 + 1] != -INFINITY) ts += expf(sacc[n][hh * 2 + 1] - mn);
          }
          ts += __shfl_xor_sync(0xffffffffu, ts, 1);
          ts += __shfl_xor_sync(0xffffffffu, ts, 2);
          if (live) {
            l[hh] = (m[hh] == -INFINITY ? 0.f : l[hh] * expf(m[hh] - mn)) + ts;
            m[hh] = mn;
          }
        }
      } else {
        // probabilities rounded as the reference does, then O += P V
        uint32_t pa[NS / 2][4];
#pragma unroll
        for (int g = 0; g < NS / 2; ++g) {
          float pv[2][4];
#pragma unroll
          for (int q2 = 0; q2 < 2; ++q2)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float x = sacc[2 * g + q2][e];
              const int hh = e >> 1;
              pv[q2][e] = (x == -INFINITY) ? 0.f : rnd<bf16>(expf(x - m[hh]) / l[hh]);
            }
          pa[g][0] = pack_bf16x2(pv[0][0], pv[0][1]);
          pa[g][1] = pack_bf16x2(pv[0][2], pv[0][3]);
          pa[g][2] = pack_bf16x2(pv[1][0], pv[1][1]);
          pa[g][3] = pack_bf16x2(pv[1][2], pv[1][3]);
        }
        const uint32_t vb = smem_u32(vs + st * TILE);
#pragma unroll
        for (int kk = 0; kk < KT / 16; ++kk) {
#pragma unroll
          for (int g = 0; g < NO / 2; ++g) {
            uint32_t b0, b1, b2, b3;
            const int row = kk * 16 + (mi & 1) * 8 + r8, ch = g * 2 + (mi >> 1);
            ldsm_x4_t(pswz(vb + (ch >> 3) * TBLK, row, ch & 7), b0, b1, b2, b3);
            mma_bf16(o[2 * g], pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3], b0, b1);
            mma_bf16(o[2 * g + 1], pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3], b2, b3);
          }
        }
      }
    }
    __syncthreads();
    if (threadIdx.x == 0 && ok && i + 2 < n_loads) issue(i + 2);
  }
  if (!__syncthreads_and(ok)) return;

  // output rows (K128 layout); rows with no visible key are finished below
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    const int row = hh ? row_hi : row_lo;
    if (row >= p.S) continue;
    if (m[hh] == -INFINITY) {
      if ((lane & 3) == 0) dead_rows[hw * 64 + row - s0] = 1;
      continue;
    }
    const long long orow = (long long)b * p.S + row;
#pragma unroll
    for (int n = 0; n < NO; ++n)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const long long col = (long long)h * HD + n * 8 + (lane & 3) * 2 + e;
        p.out[k128_offset(orow, col, p.out_rp)] = __float2bfloat16_rn(o[n][hh * 2 + e]);
      }
  }
  __syncthreads();
  // all-masked rows: uniform weights bf16(1/Tu) over the first Tu slots of the buffer
  const float pu = rnd<bf16>(1.0f / (float)p.uniform_T);
  for (int r = 0; r < 64 * HPC; ++r) {
    if (!dead_rows[r]) continue;
    const long long orow = (long long)b * p.S + s0 + (r & 63);
    for (int d = threadIdx.x; d < HD; d += NT) {
      float acc = 0.f;
      const bf16* vcol = p.v_plain + ((p.layer_row0 + (long long)b * p.T) * p.Hkv + kvh) * HD + d;
      for (int j = 0; j < p.uniform_T; ++j) acc += pu * __bfloat162float(vcol[(long long)j * p.Hkv * HD]);
      p.out[k128_offset(orow, (long long)(h0 + (r >> 6)) * HD + d, p.out_rp)] = __float2bfloat16_rn(acc);
    }
  }
}

template <int HD, int KT, int HPC>
static int launch_pattn_h(const jx_pattn_args& a, const PAttnParams& p, bool pdl, cudaStream_t s) {
  CUtensorMap km, vm;
  const long long cols = (long long)a.Hkv * HD;
  int rc = make_tmap_2d_bf16_box(&km, a.k_base, a.cache_rows, cols, cols, KT);
  if (rc == JX_OK) rc = make_tmap_2d_bf16_box(&vm, a.v_base, a.cache_rows, cols, cols, KT);
  if (rc != JX_OK) return rc;
  const int smem = 1024 + HPC * (HD / 64) * 64 * 128 + 4 * KT * HD * 2 + 16 + HPC * 64 * 4;
  static bool configured = false;
  if (!configured) {
    if (cudaFuncSetAttribute(pattn_kernel<HD, KT, HPC>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
        cudaSuccess)
      return JX_ERR_CUDA;
    configured = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((a.S + 63) / 64, a.Hq / HPC, a.B);
  cfg.blockDim = dim3(128 * HPC);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return launch_ex(&cfg, pattn_kernel<HD, KT, HPC>, km, vm, p) == cudaSuccess ? JX_OK : JX_ERR_CUDA;
}

// Heads per CTA: the largest of 4, 2, 1 that divides the heads per KV head (all of a CTA's heads read
// the same K / V tiles).
template <int HD, int KT>
static int launch_pattn(const jx_pattn_args& a, const PAttnParams& p, bool pdl, cudaStream_t s) {
  if (p.n_rep % 4 == 0) return launch_pattn_h<HD, KT, 4>(a, p, pdl, s);
  if (p.n_rep % 2 == 0) return launch_pattn_h<HD, KT, 2>(a, p, pdl, s);
  return launch_pattn_h<HD, KT, 1>(a, p, pdl, s);
}

int run_prefill_attention_tc(const jx_pattn_args& a, bool pdl, cudaStream_t stream);

// 0 = by shape (this file's kernel), 1 = this file's kernel, 2 = the tcgen05 kernel (attention_prefill_tc.cu)
static int g_pattn_impl = 0;
void set_pattn_impl(int impl) { g_pattn_impl = impl; }

int run_prefill_attention(const jx_pattn_args& a, bool pdl, cudaStream_t stream) {
  if (g_pattn_impl == 2) return run_prefill_attention_tc(a, pdl, stream);
  if (a.B <= 0 || a.S <= 0 || a.Hkv <= 0 || a.Hq % a.Hkv || a.T <= 0 || a.S > a.T) return JX_ERR_SHAPE;
  if (a.B > 65535 || a.Hq > 65535) return JX_ERR_SHAPE;
  if (reinterpret_cast<uintptr_t>(a.q) & 15) return JX_ERR_ARG;
  PAttnParams p;
  p.B = a.B;
  p.S = a.S;
  p.Hq = a.Hq;
  p.Hkv = a.Hkv;
  p.n_rep = a.Hq / a.Hkv;
  p.T = a.T;
  p.uniform_T = a.uniform_T > 0 && a.uniform_T < a.T ? a.uniform_T : a.T;
  p.layer_row0 = a.layer_row0;
  p.q = reinterpret_cast<const bf16*>(a.q);
  p.v_plain = reinterpret_cast<const bf16*>(a.v_base);
  p.len_ptr = a.len_ptr;
  p.len_add = a.len_add;
  p.window = a.window;
  p.scale_bf16 = __bfloat162float(__float2bfloat16_rn(a.scale));
  p.out = reinterpret_cast<bf16*>(a.out);
  p.out_rp = a.out_rp;
  p.status = a.status;
  switch (a.hd) {
    case 64: return launch_pattn<64, 64>(a, p, pdl, stream);
    case 128: return launch_pattn<128, 64>(a, p, pdl, stream);
    case 256: return launch_pattn<256, 32>(a, p, pdl, stream);
    default: return JX_ERR_SHAPE;
  }
}

}  // namespace jxb
