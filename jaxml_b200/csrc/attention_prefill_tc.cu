// Prefill attention on the 5th-generation tensor cores (tcgen05 + TMEM), head_dim 64 / 128 / 256: the masks
// and rounding points of attention_prefill.cu (Attention.mha for q_len > 1, nn/attention.py:321-400):
// scores = bf16(bf16(q.k) * bf16(attn_scale)) over the visible keys (causal, sliding window, right
// padding), probabilities bf16(exp(s - m) / l) with the row's final max m and exp-sum l (a first pass
// over the key tiles finds them, a second recomputes the scores, rounds the probabilities and
// accumulates P.V), o = bf16(P.V); a row with no visible key attends uniformly to the first uniform_T
// slots of the buffer.
//
// One CTA per (query block, head set, batch row): its 128 query rows are HPT heads x RPH positions
// (rows [head][position]; HPT = 4, 2 or 1, the largest that divides the heads per KV head, RPH =
// 128 / HPT), so the HPT heads share every K / V tile.  Warps: 0..15 softmax (warp w reads TMEM lane
// quadrant w % 4, i.e. rows 32 (w % 4) .. +31, and column group w / 4, a quarter of each tile), 16 the
// TMA producer, 17 the MMA issuer (and TMEM owner).  Shared memory holds every operand as 64-column blocks of
// [rows][128 bytes] with the 128-byte swizzle (16-byte chunk c of row r at chunk c ^ (r % 8)), the
// layout the K / V tensor maps produce: Q and P (written by threads) and K are K-major operands, V is
// the MN-major B operand of P.V.  TMEM: two KT-column score buffers (the MMA of the next tile overlaps
// the softmax of this one) and the HD-column output accumulator; KT = 128 keys per tile for head_dim
// 64 / 128, 64 for 256 (shared memory).
//
// The query tiles with the most key tiles start first (the CTA order is reversed over query blocks).
// Every wait is bounded; on a timeout the kernel records JX_ERR_TIMEOUT and returns.
#include <cudaTypedefs.h>

#include "common.cuh"

namespace jxb {

int make_tmap_2d_bf16_box(CUtensorMap* map, const void* base, long long rows, long long cols,
                          long long row_stride_elems, int box_rows);

struct PTcParams {
  int B, S, Hq, Hkv, n_rep, T;
  int hpt, rph;          // heads per CTA, query positions per head (hpt * rph = 128)
  int uniform_T;
  long long layer_row0;
  const bf16* q;         // [B*S, Hq, HD]
  const bf16* v_plain;   // V cache base, row-major [rows, Hkv*HD] (uniform fallback)
  const int* len_ptr;
  int len_add, window;
  float scale_bf16;
  bf16* out;
  long long out_rp;
  int* status;
};

constexpr int kPtRows = 128;                       // query rows per CTA (MMA M)
constexpr int kPtSoftWarps = 16;                   // 4 per TMEM lane quadrant
constexpr int kPtGroups = kPtSoftWarps / 4;        // column groups of a row (one warp of each quadrant)
constexpr int kPtThreads = 32 * (kPtSoftWarps + 2);
constexpr uint32_t kPtTmemCols = 512;              // scores 2 x KT columns, output at column 2 KT
constexpr int kPtBlk = kPtRows * 128;              // bytes of one [128 rows][128 B] block

// KT keys per tile (MMA N of the scores): 128 for head_dim 64 / 128, 64 for 256 (shared memory).
template <int HD, int KT>
struct PtCfg {
  static constexpr int kCB = HD / 64;                    // 64-column blocks of a head
  static constexpr int kQBytes = kCB * kPtBlk;           // Q: [kCB][128 rows][128 B]
  static constexpr int kTileBytes = kCB * KT * 128;      // one K or V tile: [kCB][KT keys][128 B]
  static constexpr int kPBytes = (KT / 64) * kPtBlk;     // P: [KT / 64 key blocks][128 rows][128 B]
  static constexpr int kOffK = kQBytes;                  // 2 stages
  static constexpr int kOffV = kOffK + 2 * kTileBytes;   // 2 stages
  static constexpr int kOffP = kOffV + 2 * kTileBytes;
  static constexpr int kOffStat = kOffP + kPBytes;       // float m[kPtGroups][128], l[kPtGroups][128]
  static constexpr int kOffBar = kOffStat + 2 * kPtGroups * kPtRows * 4;
  static constexpr int kNBar = 17;
  static constexpr int kOffMisc = kOffBar + kNBar * 8;   // tmem slot, dead flag, dead rows [128]
  static constexpr int kSmem = 1024 + kOffMisc + 16 + kPtRows * 4;
  static_assert(HD % 64 == 0 && KT % 64 == 0 && KT <= 256, "64-column blocks, at most a 256-row TMA box");
  static_assert(kOffK % 1024 == 0 && kOffV % 1024 == 0 && kOffP % 1024 == 0 && kTileBytes % 1024 == 0,
                "swizzled operand blocks start on 1024-byte boundaries");
  static_assert(2 * KT + HD <= (int)kPtTmemCols, "two score buffers and the output fit the TMEM allocation");
  static_assert(kSmem <= 227 * 1024, "shared memory per CTA");
  static_assert(HD <= 256 && KT <= 256, "MMA N <= 256");
  static_assert((KT / kPtGroups) % 16 == 0 && (HD / kPtGroups) % 16 == 0, "16-column TMEM loads per group");
};

// Shared-memory descriptor of a K-major operand in 128-byte-swizzled [rows][128 B] blocks: 8-row groups
// 1024 bytes apart (SBO), the leading offset unused (1); layout type SWIZZLE_128B (2) at [61,64).  A
// K step of 16 elements advances the start address by 32 bytes inside the block.
__device__ __forceinline__ uint64_t umma_desc_kmajor_sw128(uint32_t smem_addr) {
  return (uint64_t)((smem_addr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) |
         (2ull << 61);
}

// Shared-memory descriptor of an MN-major operand in the same blocks (rows = K, 64 MN elements per
// 128-byte row): 8-row K groups 1024 bytes apart (SBO), 64-element MN blocks `lbo` bytes apart (LBO).
__device__ __forceinline__ uint64_t umma_desc_mnmajor_sw128(uint32_t smem_addr, uint32_t lbo) {
  return (uint64_t)((smem_addr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
         ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}

// Byte offset of 16-byte chunk c of row r in a swizzled [rows][128 B] block.
__device__ __forceinline__ uint32_t sw128_off(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }

template <int HD, int KT>
__global__ void __launch_bounds__(kPtThreads, 1)
    pattn_tc_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap, PTcParams p) {
  using C = PtCfg<HD, KT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* qs = smem;
  uint8_t* ks = smem + C::kOffK;
  uint8_t* vs = smem + C::kOffV;
  uint8_t* ps = smem + C::kOffP;
  float* stat = reinterpret_cast<float*>(smem + C::kOffStat);   // m[kPtGroups][128], l[kPtGroups][128]
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
  uint64_t* kfull = bar;
  uint64_t* kempty = bar + 2;
  uint64_t* vfull = bar + 4;
  uint64_t* vempty = bar + 6;
  uint64_t* sfull = bar + 8;
  uint64_t* sempty = bar + 10;
  uint64_t* pfull = bar + 12;
  uint64_t* pempty = bar + 13;
  uint64_t* ofull = bar + 14;
  uint64_t* done = bar + 15;
  uint64_t* fin = bar + 16;     // every MMA this CTA issued has completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kOffMisc);
  volatile int* dead = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* dead_rows = reinterpret_cast<int*>(smem + C::kOffMisc + 16);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // query blocks in reverse order: the blocks with the most key tiles start first
  const int nqb = gridDim.x, per_qb = gridDim.y * gridDim.z;
  const int lin = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
  const int qb = nqb - 1 - lin / per_qb, rest = lin % per_qb;
  const int b = rest / gridDim.y;
  const int h0 = (rest % gridDim.y) * p.hpt;
  const int kvh = h0 / p.n_rep;
  const int q0 = qb * p.rph;

  if (threadIdx.x == 0) {
    prefetch_tmap(&kmap);
    prefetch_tmap(&vmap);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kfull[i], 1);
      mbar_init(&kempty[i], 1);
      mbar_init(&vfull[i], 1);
      mbar_init(&vempty[i], 1);
      mbar_init(&sfull[i], 1);
      mbar_init(&sempty[i], kPtSoftWarps);
    }
    mbar_init(pfull, kPtSoftWarps);
    mbar_init(pempty, 1);
    mbar_init(ofull, 1);
    mbar_init(done, kPtSoftWarps);
    mbar_init(fin, 1);
    *dead = 0;
    fence_barrier_init();
  }
  if (warp == kPtSoftWarps + 1) {
    tmem_alloc(tmem_slot, kPtTmemCols);
    tmem_relinquish();
  }
  pdl_trigger();
  pdl_wait();
  int valid = p.len_ptr[b] + p.len_add;
  if (valid > p.T) {
    if (threadIdx.x == 0) set_status(p.status, JX_ERR_RANGE);
    valid = p.T;
  }
  const int s_max = min(q0 + p.rph - 1, p.S - 1);
  const int j_hi = min(s_max, valid - 1);
  const int j_lo = p.window > 0 ? max(0, q0 - p.window + 1) : 0;
  const int n = j_hi >= j_lo ? (j_hi - j_lo + KT) / KT : 0;   // key tiles per pass

  // Q rows [head][position] (positions past S are zero) in 64-column swizzled blocks
  for (int idx = threadIdx.x; idx < kPtRows * (HD / 8); idx += kPtThreads) {
    const int r = idx / (HD / 8), cg = idx % (HD / 8);
    const int hl = r / p.rph, pos = q0 + r % p.rph;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (pos < p.S)
      v = *reinterpret_cast<const uint4*>(p.q + (((long long)b * p.S + pos) * p.Hq + h0 + hl) * HD + cg * 8);
    *reinterpret_cast<uint4*>(qs + (cg >> 3) * kPtBlk + sw128_off(r, cg & 7)) = v;
  }
  if (threadIdx.x < kPtRows) dead_rows[threadIdx.x] = 0;
  fence_proxy_async();   // the generic-proxy writes of Q are read by the tensor core (async proxy)
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kPtSoftWarps) {
    // ---------------- TMA producer: K tiles of pass 1, then K and V tiles of pass 2 ----------------
    if (lane == 0) {
      int issued = 0, v_issued = 0;
      for (int i = 0; i < 2 * n && !*dead; ++i) {
        const int st = i & 1, t = i < n ? i : i - n;
        const int y = (int)(p.layer_row0 + (long long)b * p.T + j_lo + t * KT);
        if (i >= 2 && !mbar_wait_bounded(&kempty[st], ((i >> 1) - 1) & 1)) {
          set_status(p.status, JX_ERR_TIMEOUT);
          *dead = 1;
          break;
        }
        mbar_arrive_expect_tx(&kfull[st], C::kTileBytes);
#pragma unroll
        for (int c = 0; c < C::kCB; ++c)
          tma_load_2d(ks + st * C::kTileBytes + c * KT * 128, &kmap, kvh * HD + c * 64, y, &kfull[st]);
        issued = i + 1;
        if (i >= n) {
          const int vst = t & 1;
          if (t >= 2 && !mbar_wait_bounded(&vempty[vst], ((t >> 1) - 1) & 1)) {
            set_status(p.status, JX_ERR_TIMEOUT);
            *dead = 1;
            break;
          }
          mbar_arrive_expect_tx(&vfull[vst], C::kTileBytes);
#pragma unroll
          for (int c = 0; c < C::kCB; ++c)
            tma_load_2d(vs + vst * C::kTileBytes + c * KT * 128, &vmap, kvh * HD + c * 64, y, &vfull[vst]);
          v_issued = t + 1;
        }
      }
      // every issued copy lands before this CTA's shared memory is released
      for (int i = (issued > 2 ? issued - 2 : 0); i < issued; ++i)
        if (!mbar_wait_bounded(&kfull[i & 1], (i >> 1) & 1)) break;
      for (int t = (v_issued > 2 ? v_issued - 2 : 0); t < v_issued; ++t)
        if (!mbar_wait_bounded(&vfull[t & 1], (t >> 1) & 1)) break;
    }
  } else if (warp == kPtSoftWarps + 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0 && n > 0) {
      const uint32_t idesc_s = umma_idesc_bf16_f32(kPtRows, KT);
      const uint32_t idesc_o = umma_idesc_bf16_f32(kPtRows, HD) | (1u << 16);   // B (V) MN-major
      const uint32_t qa = smem_u32(qs);
      bool ok = true;
      // S(i) = Q K(i)^T into score buffer i % 2 (i < n: pass 1, i >= n: pass 2 tile i - n)
      auto scores = [&](int i) -> bool {
        const int st = i & 1, buf = i & 1;
        if (!mbar_wait_bounded(&kfull[st], (i >> 1) & 1)) return false;
        if (i >= 2 && !mbar_wait_bounded(&sempty[buf], ((i >> 1) - 1) & 1)) return false;
        tc_fence_after();
        const uint32_t kb = smem_u32(ks + st * C::kTileBytes);
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) {
          const uint32_t off = (uint32_t)((k >> 2) * kPtBlk + (k & 3) * 32);
          const uint32_t koff = (uint32_t)((k >> 2) * KT * 128 + (k & 3) * 32);
          umma_bf16(tmem + (uint32_t)(buf * KT), umma_desc_kmajor_sw128(qa + off), umma_desc_kmajor_sw128(kb + koff),
                    idesc_s, k > 0 ? 1u : 0u);
        }
        umma_commit(&sfull[buf]);
        umma_commit(&kempty[st]);
        return true;
      };
      for (int i = 0; i < n && ok; ++i) ok = scores(i);
      if (ok) ok = scores(n);
      for (int t = 0; t < n && ok; ++t) {
        if (t + 1 < n) ok = scores(n + t + 1);
        const int vst = t & 1;
        if (ok && !(mbar_wait_bounded(&pfull[0], t & 1) && mbar_wait_bounded(&vfull[vst], (t >> 1) & 1))) ok = false;
        if (!ok) break;
        tc_fence_after();
        const uint32_t pa = smem_u32(ps), vb = smem_u32(vs + vst * C::kTileBytes);
#pragma unroll
        for (int k = 0; k < KT / 16; ++k) {
          const uint32_t aoff = (uint32_t)((k >> 2) * kPtBlk + (k & 3) * 32);
          umma_bf16(tmem + (uint32_t)(2 * KT), umma_desc_kmajor_sw128(pa + aoff),
                    umma_desc_mnmajor_sw128(vb + (uint32_t)(k * 16 * 128), (uint32_t)(KT * 128)), idesc_o,
                    (t > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(pempty);
        umma_commit(&vempty[vst]);
      }
      if (ok) {
        umma_commit(ofull);
      } else {
        set_status(p.status, JX_ERR_TIMEOUT);
        *dead = 1;
      }
      umma_commit(fin);
    }
  } else {
    // ------------- softmax warps: row r = 32 (warp % 4) + lane, column group cg = warp / 4 -------------
    const int quad = warp & 3, cg = warp >> 2;
    const int r = quad * 32 + lane;
    const int hl = r / p.rph, pos = q0 + r % p.rph;
    const uint32_t trow = tmem + ((uint32_t)(quad * 32) << 16);
    bool ok = true;
    constexpr int kCols = KT / kPtGroups;   // this thread's columns of a tile
    float x[kCols];
    // scores of tile t (score buffer `buf`) for this thread's 64 columns, masked and rounded
    auto load_scores = [&](int i, int t) -> bool {
      const int buf = i & 1;
      bool w = mbar_wait_bounded(&sfull[buf], (i >> 1) & 1);
      w = __all_sync(0xffffffffu, w);   // tcgen05.ld is warp-wide
      if (w) {
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < kCols / 16; ++c) tmem_ld16(trow + (uint32_t)(buf * KT + cg * kCols + c * 16), x + c * 16);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sempty[buf]);
      const int jb = j_lo + t * KT + cg * kCols;
#pragma unroll
      for (int e = 0; e < kCols; ++e) {
        const int j = jb + e;
        bool vis = j <= pos && j < valid && j <= j_hi;
        if (p.window > 0 && j <= pos - p.window) vis = false;
        x[e] = vis ? rnd<bf16>(rnd<bf16>(x[e]) * p.scale_bf16) : -INFINITY;
      }
      return w;
    };
    // pass 1: online max / exp-sum of this column group of the row
    float m = -INFINITY, l = 0.f;
    for (int t = 0; t < n && ok; ++t) {
      ok = load_scores(t, t);
      if (!ok) break;
      float tm = -INFINITY;
#pragma unroll
      for (int e = 0; e < kCols; ++e) tm = fmaxf(tm, x[e]);
      const float mn = fmaxf(m, tm);
      if (mn != -INFINITY) {
        float ts = 0.f;
#pragma unroll
        for (int e = 0; e < kCols; ++e)
          if (x[e] != -INFINITY) ts += expf(x[e] - mn);
        l = (m == -INFINITY ? 0.f : l * expf(m - mn)) + ts;
        m = mn;
      }
    }
    // the column groups of the row: final max and exp-sum, combined in group order (every group of the
    // row computes the same values)
    stat[cg * kPtRows + r] = m;
    stat[(kPtGroups + cg) * kPtRows + r] = l;
    named_bar_sync(1, 32 * kPtSoftWarps);
    m = -INFINITY;
#pragma unroll
    for (int g = 0; g < kPtGroups; ++g) m = fmaxf(m, stat[g * kPtRows + r]);
    l = 0.f;
#pragma unroll
    for (int g = 0; g < kPtGroups; ++g) {
      const float mg = stat[g * kPtRows + r];
      l += mg == -INFINITY ? 0.f : stat[(kPtGroups + g) * kPtRows + r] * expf(mg - m);
    }
    // pass 2: probabilities rounded as the reference does, into P for the P.V MMA
    for (int t = 0; t < n && ok; ++t) {
      ok = load_scores(n + t, t);
      if (!ok) break;
      uint32_t pk[kCols / 2];
#pragma unroll
      for (int e = 0; e < kCols; e += 2) {
        const float a = x[e] == -INFINITY ? 0.f : rnd<bf16>(expf(x[e] - m) / l);
        const float c = x[e + 1] == -INFINITY ? 0.f : rnd<bf16>(expf(x[e + 1] - m) / l);
        pk[e >> 1] = pack_bf16x2(a, c);
      }
      if (t > 0) {
        bool w = mbar_wait_bounded(pempty, (t - 1) & 1);
        if (!__all_sync(0xffffffffu, w)) {
          ok = false;
          break;
        }
      }
#pragma unroll
      for (int c = 0; c < kCols / 8; ++c) {
        const int kk = cg * kCols + 8 * c;   // first key of the chunk within the tile
        *reinterpret_cast<uint4*>(ps + (kk >> 6) * kPtBlk + sw128_off(r, (kk & 63) >> 3)) =
            make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
      }
      fence_proxy_async();   // generic-proxy writes of P, read by the tensor core
      __syncwarp();
      if (lane == 0) mbar_arrive(pfull);
    }
    // output accumulator: this thread's row, columns cg * HD / kPtGroups .., read and stored 16 at a time
    constexpr int kHalf = HD / kPtGroups;
    if (ok && n > 0) {
      bool w = mbar_wait_bounded(ofull, 0);
      w = __all_sync(0xffffffffu, w);
      if (w) {
        tc_fence_after();
        const bool store = pos < p.S && m != -INFINITY;
        const long long orow = (long long)b * p.S + pos;
        const long long col0 = (long long)(h0 + hl) * HD + cg * kHalf;
#pragma unroll
        for (int c = 0; c < kHalf / 16; ++c) {
          float o[16];
          tmem_ld16(trow + (uint32_t)(2 * KT + cg * kHalf + c * 16), o);   // warp-wide: every lane loads
          if (store) {
#pragma unroll
            for (int h2 = 0; h2 < 2; ++h2) {
              uint4 v;
              v.x = pack_bf16x2(o[8 * h2], o[8 * h2 + 1]);
              v.y = pack_bf16x2(o[8 * h2 + 2], o[8 * h2 + 3]);
              v.z = pack_bf16x2(o[8 * h2 + 4], o[8 * h2 + 5]);
              v.w = pack_bf16x2(o[8 * h2 + 6], o[8 * h2 + 7]);
              *reinterpret_cast<uint4*>(p.out + k128_offset(orow, col0 + 16 * c + 8 * h2, p.out_rp)) = v;
            }
          }
        }
      } else {
        ok = false;
      }
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(done);
    if (!ok) {
      set_status(p.status, JX_ERR_TIMEOUT);
      *dead = 1;
    }
    if (pos < p.S && m == -INFINITY && cg == 0) dead_rows[r] = 1;
    // rows with no visible key: uniform weights bf16(1/Tu) over the first Tu slots of the buffer
    named_bar_sync(1, 32 * kPtSoftWarps);
    if (ok) {
      const float pu = rnd<bf16>(1.0f / (float)p.uniform_T);
      for (int rr = 0; rr < kPtRows; ++rr) {
        if (!dead_rows[rr]) continue;
        const int pos2 = q0 + rr % p.rph;
        if (pos2 >= p.S) continue;
        const long long orow = (long long)b * p.S + pos2;
        for (int d = threadIdx.x; d < HD; d += 32 * kPtSoftWarps) {
          float acc = 0.f;
          const bf16* vcol = p.v_plain + ((p.layer_row0 + (long long)b * p.T) * p.Hkv + kvh) * HD + d;
          for (int j = 0; j < p.uniform_T; ++j) acc += pu * __bfloat162float(vcol[(long long)j * p.Hkv * HD]);
          p.out[k128_offset(orow, (long long)(h0 + rr / p.rph) * HD + d, p.out_rp)] = __float2bfloat16_rn(acc);
        }
      }
    }
  }
  // TMEM is freed by its owner once every softmax warp has read its last cells
  if (warp == kPtSoftWarps + 1) {
    __syncwarp();
    bool w = mbar_wait_bounded(done, 0);
    if (n > 0) w = mbar_wait_bounded(fin, 0) && w;
    if (!w && lane == 0) set_status(p.status, JX_ERR_TIMEOUT);
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, kPtTmemCols);
  }
}

// ------------------------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------------------------
template <int HD, int KT>
static int launch_pattn_tc(const jx_pattn_args& a, const PTcParams& p, bool pdl, cudaStream_t s) {
  CUtensorMap km, vm;
  const long long cols = (long long)a.Hkv * HD;
  int rc = make_tmap_2d_bf16_box(&km, a.k_base, a.cache_rows, cols, cols, KT);
  if (rc == JX_OK) rc = make_tmap_2d_bf16_box(&vm, a.v_base, a.cache_rows, cols, cols, KT);
  if (rc != JX_OK) return rc;
  static bool configured = false;
  if (!configured) {
    if (cudaFuncSetAttribute(pattn_tc_kernel<HD, KT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             PtCfg<HD, KT>::kSmem) != cudaSuccess)
      return JX_ERR_CUDA;
    configured = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((a.S + p.rph - 1) / p.rph, a.Hq / p.hpt, a.B);
  cfg.blockDim = dim3(kPtThreads);
  cfg.dynamicSmemBytes = PtCfg<HD, KT>::kSmem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return launch_ex(&cfg, pattn_tc_kernel<HD, KT>, km, vm, p) == cudaSuccess ? JX_OK : JX_ERR_CUDA;
}

bool prefill_attention_tc_supported(const jx_pattn_args& a) {
  return (a.hd == 64 || a.hd == 128 || a.hd == 256) && a.Hkv > 0 && a.Hq % a.Hkv == 0 && a.S > 0 && a.S <= a.T && a.B > 0 &&
         a.B <= 65535 && a.Hq <= 65535 && (reinterpret_cast<uintptr_t>(a.q) & 15) == 0 && a.out_rp > 0;
}

int run_prefill_attention_tc(const jx_pattn_args& a, bool pdl, cudaStream_t stream) {
  if (!prefill_attention_tc_supported(a)) return JX_ERR_SHAPE;
  PTcParams p;
  p.B = a.B;
  p.S = a.S;
  p.Hq = a.Hq;
  p.Hkv = a.Hkv;
  p.n_rep = a.Hq / a.Hkv;
  p.T = a.T;
  p.hpt = p.n_rep % 4 == 0 ? 4 : (p.n_rep % 2 == 0 ? 2 : 1);
  p.rph = kPtRows / p.hpt;
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
  if (a.hd == 64) return launch_pattn_tc<64, 128>(a, p, pdl, stream);
  if (a.hd == 128) return launch_pattn_tc<128, 128>(a, p, pdl, stream);
  return launch_pattn_tc<256, 64>(a, p, pdl, stream);
}

}  // namespace jxb
