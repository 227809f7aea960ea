// One decode step of a Llama-family bf16 stack in one persistent kernel (jx_decode_step).
//
// The per-op decode path launches 8 kernels per layer; each small projection then pays a few
// microseconds of ramp-up (first TMA data) and of split-K drain (the last arrivers summing partial
// tiles) while most SMs idle, and nothing streams weights across the kernel boundary.  Here one
// cooperative launch (one CTA per SM) runs the whole step as a fixed sequence of phases,
//     per layer: input norm, QKV projection, attention scores, attention P.V, o_proj (+ residual),
//                post-attention norm, gate/up projection (+ SiLU . up), down projection (+ residual)
//     then:      final norm, LM head projection,
// separated by grid-wide barriers (a monotonic arrival counter in global memory).  The warp roles are
//     warp 0     TMA producer: streams this CTA's share of every phase through one ring of shared-memory
//                stages (weight tiles, or K / V tiles of the attention phases).  Weights do not depend on
//                the step, so it loads the next phases' weights as soon as stages free up and waits on
//                the grid barrier only before loading a projection's activations;
//     warp 1     MMA issuer (tcgen05.mma, weight tile as A = 128 rows, 16 token rows as B, float32
//                accumulators double-buffered in TMEM);
//     warps 2-5  workers: projection epilogues (TMEM -> shared memory, deterministic split-K fix-up by the
//                last arriver, fused epilogue), the norm rows, the attention work items (mma.sync on the
//                K / V tiles the producer staged).
// Projections split (128-row weight block x 128-wide K chunk) iterations evenly over the CTAs
// (stream-K, as gemv_tc.cu).  Attention work items are (batch row, KV head, 128-key split), dealt
// round-robin; RoPE and the cache append are fused into the scores items (the item holding this step's
// position rotates k, appends k and v, and patches k into its staged tile; the P.V item patches v), and
// the P.V items form the exact bf16 probabilities from the split statistics, as attention_decode.cu.
//
// Every rounding point is the per-op path's (and the reference's): projection results rounded to bf16
// before the residual add / activation, RMSNorm y = bf16(w * bf16(x / sqrt(mean(x^2) + eps))), scores
// bf16(bf16(q.k) * bf16(scale)), float32 softmax with a true division, probabilities rounded to bf16.
//
// Waits are bounded (2 s): on a timeout a CTA sets the status word and a global abort flag that every
// other wait checks, drains its own TMA copies in flight, frees its TMEM and returns.
#include <cudaTypedefs.h>

#include "common.cuh"

namespace jxb {

int make_tmap_2d_bf16(CUtensorMap* map, const void* base, long long rows, long long cols, long long row_stride_elems);
long long dattn_workspace_bytes(int B, int Hq, int T, int hd, int n_splits);
int dattn_n_splits(int T, int window);
int fail(int code, const char* msg);
int note_cuda(const char* where);

namespace ds {
constexpr int kThreads = 192;
constexpr int kStages = 5;
constexpr int kWBytes = 128 * 128 * 2;          // a 128-row x 128-k weight tile, or 128 keys x 128 dims of K / V
constexpr int kXBytes = 16 * 128 * 2;           // 16 token rows x 128 k of activations
constexpr int kStageBytes = kWBytes + kXBytes;  // 36 KB (a multiple of 1 KB: 128-byte-swizzle alignment holds)
constexpr int kTileLd = 132;                    // float32 staging tile [16 tokens][128 weight rows + pad]
constexpr int kTileBytes = 16 * kTileLd * 4;
constexpr int kHD = 128;
constexpr int kKeys = 128;                      // keys per attention work item
constexpr int kPLd = kKeys + 8;                 // bf16 row stride of the probability tile
constexpr int kOffTile = kStages * kStageBytes;
constexpr int kOffQ = kOffTile + kTileBytes;    // [2 x (16 rows x 64 dims)] swizzled q
constexpr int kOffP = kOffQ + 4096;             // [16][kPLd] bf16 probabilities
constexpr int kOffRed = kOffP + 16 * kPLd * 2;  // 64 floats of reductions, 16 + 16 softmax statistics
constexpr int kOffS = kOffRed + 96 * 4;         // bf16 scores of the single-pass attention
constexpr int kSBufBytes = 28 * 1024;           // n_rep x keys <= 14336
constexpr int kOffBar = kOffS + kSBufBytes;     // mbarriers
constexpr int kNumBars = 2 * kStages + 6;
constexpr int kOffMisc = kOffBar + kNumBars * 8;
constexpr int kSmem = 1024 + kOffMisc + 256;
static_assert(kOffBar % 8 == 0, "mbarrier alignment");
static_assert(kSmem <= 227 * 1024, "shared memory");
enum Kind { NORM = 0, PROJ = 1, SCORES = 2, PV = 3, ATTN = 4 };
enum Epi { E_QKV = 0, E_RESID = 1, E_GLU = 2, E_LOGITS = 3 };
}  // namespace ds

struct DsParams {
  int M, L, d, Hq, Hkv, n_rep, T, rd, max_pos, V, vocab, F, nqkv, n_splits;
  long long Np_qkv, Np_d, Np_gu, Np_v, Kp_d, Kp_o, Kp_f;
  float eps, scale_bf16;
  const bf16* const* layers;   // [L][6]
  const bf16* embed;
  const int* ids;
  const bf16* final_norm;
  const bf16* lm_head;
  bf16* h;
  bf16* xn;
  bf16* qkv;
  bf16* attn;
  bf16* act;
  bf16* logits;
  bf16* k_cache;
  bf16* v_cache;
  const bf16* cos;
  const bf16* sin;
  const int* pos_id;
  float* ws;
  int* counters;
  float* sc;       // [M, Hq, T] scores
  float* stats;    // [M, Hq, n_splits, 2] per-split (max, sum)
  float* opart;    // [M, Hq, n_splits, 128] per-split P.V partials
  int* acnt;       // [M * Hkv] split arrivals
  int* sync;       // [0] arrivals, [1] abort, [2..5] where a wait gave up (site, phase, counter, CTA)
  int* status;
  int l2_ahead;    // projection weight tiles per CTA prefetched into L2 ahead of the ring
};

// ---------------------------------------------------------------------------------------------------
// phases
// ---------------------------------------------------------------------------------------------------
// Phases per layer: 8 with the two-phase attention (scores items, a grid barrier, then P.V items), 7 with
// the single-pass attention.  ds_lj gives the phase's index in the 8-phase numbering: 0 input norm,
// 1 QKV, 2 attention (scores), 3 P.V, 4 o_proj, 5 post-attention norm, 6 gate/up, 7 down.
__device__ __forceinline__ int ds_lj(int q, int ppl) {
  const int j = q % ppl;
  return (ppl == 8 || j < 3) ? j : j + 1;
}

__device__ __forceinline__ int ds_kind(const DsParams& p, int q, int ppl) {
  if (q >= ppl * p.L) return q == ppl * p.L ? ds::NORM : ds::PROJ;
  switch (ds_lj(q, ppl)) {
    case 0:
    case 5: return ds::NORM;
    case 2: return ppl == 8 ? ds::SCORES : ds::ATTN;
    case 3: return ds::PV;
    default: return ds::PROJ;
  }
}

struct DsProj {
  const bf16* W;
  const bf16* X;
  long long Np, Kp;
  int epi;
};

__device__ __forceinline__ DsProj ds_proj(const DsParams& p, int q, int ppl) {
  DsProj r;
  if (q >= ppl * p.L) {
    r.W = p.lm_head, r.X = p.xn, r.Np = p.Np_v, r.Kp = p.Kp_d, r.epi = ds::E_LOGITS;
    return r;
  }
  const bf16* const* lw = p.layers + (q / ppl) * 6;
  switch (ds_lj(q, ppl)) {
    case 1: r.W = lw[0], r.X = p.xn, r.Np = p.Np_qkv, r.Kp = p.Kp_d, r.epi = ds::E_QKV; break;
    case 4: r.W = lw[1], r.X = p.attn, r.Np = p.Np_d, r.Kp = p.Kp_o, r.epi = ds::E_RESID; break;
    case 6: r.W = lw[2], r.X = p.xn, r.Np = p.Np_gu, r.Kp = p.Kp_d, r.epi = ds::E_GLU; break;
    default: r.W = lw[3], r.X = p.act, r.Np = p.Np_d, r.Kp = p.Kp_f, r.epi = ds::E_RESID; break;
  }
  return r;
}

// stream-K split of `total` iterations over G CTAs
__device__ __forceinline__ long long ds_begin(long long total, int G, int c) { return total * c / G; }
__device__ __forceinline__ int ds_cta_of(long long it, long long total, int G) {
  return (int)(((it + 1) * G + total - 1) / total) - 1;
}
// A phase with fewer iterations than CTAs runs on the first `total` CTAs only (one iteration each), so
// every CTA between a block's first and last contributor has a share of it.  Returns the phase's CTA
// count and this CTA's range [it0, it1) (empty beyond that count).
__device__ __forceinline__ int ds_range(long long total, int G, int c, long long& it0, long long& it1) {
  const int Gp = total < G ? (int)total : G;
  if (c >= Gp) {
    it0 = it1 = 0;
  } else {
    it0 = ds_begin(total, Gp, c);
    it1 = ds_begin(total, Gp, c + 1);
  }
  return Gp;
}

// Attention work item i = ((b * Hkv + kvh) * S + split): live when its first key is below the row's length.
__device__ __forceinline__ bool ds_item(int i, int S, int Hkv, const volatile int* valid, int& b, int& kvh, int& split) {
  split = i % S;
  const int r = i / S;
  kvh = r % Hkv;
  b = r / Hkv;
  return split * ds::kKeys < valid[b];
}

// ---------------------------------------------------------------------------------------------------
// grid barrier and bounded waits that also stop on the global abort flag
// ---------------------------------------------------------------------------------------------------
// Where a wait gave up: the first one records (site, phase, stage / block counter, CTA) in sync[2..5].
enum DsSite { S_PROD_EMPTY_PRE = 1, S_PROD_GRID, S_PROD_EMPTY, S_PROD_EMPTY_ATTN, S_MMA_ACCE, S_MMA_FULL,
              S_WORK_GRID, S_WORK_ACCF, S_WORK_SCORES, S_WORK_PV, S_END };
__device__ __forceinline__ void ds_abort(const DsParams& p, int site = 0, int q = -1, long long g = -1) {
  set_status(p.status, JX_ERR_TIMEOUT);
  if (site && atomicCAS(p.sync + 2, 0, site) == 0) {
    p.sync[3] = q;
    p.sync[4] = (int)g;
    p.sync[5] = (int)blockIdx.x;
  }
  atomicExch(p.sync + 1, 1);
}

__device__ __forceinline__ bool ds_aborted(const DsParams& p) {
  return *reinterpret_cast<const volatile int*>(p.sync + 1) != 0;
}

// Wait until `target` arrivals (every CTA has finished the phases before the one about to start).
__device__ __noinline__ bool ds_grid_wait(const DsParams& p, int target, int site, int q) {
  if (ld_acquire_gpu(p.sync) >= target) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    __nanosleep(32);
    if (ld_acquire_gpu(p.sync) >= target) return true;
    if (ds_aborted(p)) return false;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      ds_abort(p, site, q, *reinterpret_cast<const volatile int*>(p.sync));
      return false;
    }
  }
}

// One arrival of this CTA (called by one thread after every thread of the phase's work has stored).
__device__ __forceinline__ void ds_grid_arrive(const DsParams& p) {
  __threadfence();
  asm volatile("red.release.gpu.global.add.s32 [%0], 1;" ::"l"(p.sync) : "memory");
}

__device__ __noinline__ bool ds_mbar_wait(uint64_t* bar, uint32_t parity, const DsParams& p, int site, int q,
                                          long long g) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (int spin = 0;; ++spin) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((spin & 255) == 255) {
      if (ds_aborted(p)) return false;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        ds_abort(p, site, q, g);
        return false;
      }
    }
  }
}

// Wait for global stage g in ring slot s.  The ring has two consumers (the MMA warp takes projection
// stages, the workers take K / V tiles), so each skips the other's stages, and a parity wait alone could
// see the slot's full barrier two phases behind (an earlier use of the slot still in flight reads as the
// phase it waits for).  The producer tags a slot with the stage index only after the slot's previous
// occupant was released, so once the tag reads g the barrier is at most one phase behind and its parity
// is exact.  (The tag is a plain shared-memory store: the producer writes it after its wait on the empty
// barrier saw the previous occupant released, which the consumer did after seeing that occupant land; the
// consumer reads it with an acquire load before its wait on the full barrier.)  A consumer whose previous
// stage in the slot was its own can skip the tag: it saw that use complete.
// Bounded wait with the common case (already complete) inline: the slow path is a call.
__device__ __forceinline__ bool ds_wait(uint64_t* bar, uint32_t parity, const DsParams& p, int site, int q,
                                        long long g) {
  return mbar_try_wait(bar, parity) || ds_mbar_wait(bar, parity, p, site, q, g);
}

__device__ __forceinline__ int ld_acquire_cta_shared(const volatile int* p) {
  int v;
  asm volatile("ld.acquire.cta.shared::cta.b32 %0, [%1];" : "=r"(v) : "r"(smem_u32((const void*)p)) : "memory");
  return v;
}

__device__ __forceinline__ bool ds_stage_wait(const volatile int* tag, uint64_t* full, int s, long long g,
                                              const DsParams& p, int site, int q) {
  if (ld_acquire_cta_shared(tag + s) != (int)g) {
    const uint64_t t0 = globaltimer_ns();
    for (int spin = 0; ld_acquire_cta_shared(tag + s) != (int)g; ++spin) {
      if ((spin & 255) == 255) {
        if (ds_aborted(p)) return false;
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          ds_abort(p, site, q, g);
          return false;
        }
      }
    }
  }
  if (mbar_try_wait(full + s, (uint32_t)((g / ds::kStages) & 1))) return true;
  return ds_mbar_wait(full + s, (uint32_t)((g / ds::kStages) & 1), p, site, q, g);
}

// ---------------------------------------------------------------------------------------------------
// worker helpers (128 threads: warps 2..5, named barrier 1)
// ---------------------------------------------------------------------------------------------------
__device__ __forceinline__ void ds_wsync() { named_bar_sync(1, 128); }

__device__ __forceinline__ uint4 pack8(const float* y) {
  return make_uint4(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]), pack_bf16x2(y[4], y[5]),
                    pack_bf16x2(y[6], y[7]));
}

// Elements [j0, j0 + 8) of one head of the projection output (written earlier in this launch: read
// from L2), rotated on the first rd dims at table row `pos` (rotate_half; products and sum rounded
// to bf16, nn/position.py:130-132).  rd % 16 == 0.
__device__ __forceinline__ uint4 ds_rope8(const bf16* head, int j0, int rd, const bf16* cos, const bf16* sin, int pos) {
  const uint4 xv = __ldcg(reinterpret_cast<const uint4*>(head + j0));
  if (j0 >= rd) return xv;
  const int half = rd >> 1;
  const uint4 pv = __ldcg(reinterpret_cast<const uint4*>(head + (j0 < half ? j0 + half : j0 - half)));
  const uint4 cv = *reinterpret_cast<const uint4*>(cos + (long long)pos * rd + j0);
  const uint4 sv = *reinterpret_cast<const uint4*>(sin + (long long)pos * rd + j0);
  float x[8], pr[8], co[8], si[8], o[8];
  unpack8(xv, x);
  unpack8(pv, pr);
  unpack8(cv, co);
  unpack8(sv, si);
  const float sgn = j0 < half ? -1.0f : 1.0f;
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    const float a = rnd<bf16>(x[u] * co[u]);
    const float c = rnd<bf16>((sgn * pr[u]) * si[u]);
    o[u] = rnd<bf16>(a + c);
  }
  return pack8(o);
}

__device__ __forceinline__ uint32_t ds_swz(uint32_t block_base, int r, int c) {
  return block_base + r * 128 + ((c ^ (r & 7)) << 4);
}

__device__ __forceinline__ void st_shared_v4(uint32_t a, const uint4& v) {
  asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(a), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w));
}

// RMSNorm of row m (norms.py:110-117) into the K128 activations xn: from the residual stream h, or for
// the first layer from the embedding row of ids[m] (written to h first; ids < 0 read row 0,
// models/llama.py:188).
__device__ __noinline__ void ds_norm_row(const DsParams& p, int m, const bf16* w, bool embed, int wtid, float* red) {
  const int d = p.d;
  const bf16* src;
  if (embed) {
    int id = p.ids[m];
    if (id < 0) id = 0;
    if (id >= p.vocab) {
      if (wtid == 0) set_status(p.status, JX_ERR_RANGE);
      id = 0;
    }
    src = p.embed + (long long)id * d;
  } else {
    src = p.h + (long long)m * d;
  }
  // this thread's 8 x 8 elements of the row and of the weights, kept packed between the two passes; every
  // load is issued before any store (the stores could alias them as far as the compiler knows)
  uint4 raw[8], wraw[8];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int j = (wtid + k * 128) * 8;
    raw[k] = wraw[k] = make_uint4(0, 0, 0, 0);
    if (j < d) {
      raw[k] = embed ? *reinterpret_cast<const uint4*>(src + j) : __ldcg(reinterpret_cast<const uint4*>(src + j));
      wraw[k] = *reinterpret_cast<const uint4*>(w + j);
    }
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int j = (wtid + k * 128) * 8;
    if (j < d) {
      if (embed) *reinterpret_cast<uint4*>(p.h + (long long)m * d + j) = raw[k];
      float x[8];
      unpack8(raw[k], x);
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += x[i] * x[i];
    }
  }
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((wtid & 31) == 0) red[wtid >> 5] = ss;
  ds_wsync();
  const float tot = (red[0] + red[1]) + (red[2] + red[3]);
  ds_wsync();
  const float den = sqrtf(tot / (float)d + p.eps);
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int j = (wtid + k * 128) * 8;
    if (j < d) {
      float wv[8], x[8], y[8];
      unpack8(wraw[k], wv);
      unpack8(raw[k], x);
#pragma unroll
      for (int i = 0; i < 8; ++i) y[i] = rnd<bf16>(wv[i] * rnd<bf16>(x[i] / den));
      *reinterpret_cast<uint4*>(p.xn + k128_offset(m, j, 16)) = pack8(y);
    }
  }
}

// Fused projection epilogue of one finished 128-row block (tile[m][j], m < 16 token rows).  Thread t
// owns token row t / 8 and 16 consecutive weight rows (t % 8) * 16: its tile values come as four
// float4 reads, a residual row is read with two 16-byte loads before anything is stored, and results
// leave as 16-byte stores (scalar only at a ragged edge).
__device__ __noinline__ void ds_epilogue(const DsParams& p, int epi, long long n0, const float* tile, int wtid) {
  using namespace ds;
  const int m = wtid >> 3, j0 = (wtid & 7) * 16;
  float v[16];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float4 f = *reinterpret_cast<const float4*>(tile + m * kTileLd + j0 + 4 * i);
    v[4 * i] = f.x, v[4 * i + 1] = f.y, v[4 * i + 2] = f.z, v[4 * i + 3] = f.w;
  }
  if (epi == E_GLU) {
    // packed rows come in groups of 64: 32 gate rows, then the 32 up rows of the same columns; this
    // thread's 16 rows are gate (j0 % 64 < 32) or up: pair them through the lane that holds the other half
    float o[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) o[i] = __shfl_xor_sync(0xffffffffu, v[i], 2);   // lane ^ 2: the row 32 away
    if (m >= p.M || ((j0 & 63) >> 5) != 0) return;                                // up-row threads are done
    const int grp = j0 >> 6, jj = j0 & 31;
    const long long col = ((n0 >> 6) + grp) * 32 + jj;
    float y[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float g = rnd<bf16>(v[i]), u = rnd<bf16>(o[i]);
      y[i] = rnd<bf16>(silu_f(g)) * u;
    }
    if (col + 16 <= p.F) {
      *reinterpret_cast<uint4*>(p.act + k128_offset(m, col, 16)) = pack8(y);
      *reinterpret_cast<uint4*>(p.act + k128_offset(m, col + 8, 16)) = pack8(y + 8);
    } else {
      #pragma unroll
      for (int i = 0; i < 16; ++i)
        if (col + i < p.F) p.act[k128_offset(m, col + i, 16)] = __float2bfloat16_rn(y[i]);
    }
    return;
  }
  if (m >= p.M) return;
  const long long n = n0 + j0;
  if (epi == E_RESID) {
    bf16* hp = p.h + (long long)m * p.d + n;
    if (n + 16 <= p.d) {
      const uint4 r0 = __ldcg(reinterpret_cast<const uint4*>(hp)), r1 = __ldcg(reinterpret_cast<const uint4*>(hp + 8));
      float r[16], y[16];
      unpack8(r0, r);
      unpack8(r1, r + 8);
#pragma unroll
      for (int i = 0; i < 16; ++i) y[i] = rnd<bf16>(v[i]) + r[i];
      *reinterpret_cast<uint4*>(hp) = pack8(y);
      *reinterpret_cast<uint4*>(hp + 8) = pack8(y + 8);
    } else {
      #pragma unroll
      for (int i = 0; i < 16; ++i)
        if (n + i < p.d) hp[i] = __float2bfloat16_rn(rnd<bf16>(v[i]) + __bfloat162float(__ldcg(hp + i)));
    }
    return;
  }
  bf16* out = epi == E_QKV ? p.qkv : p.logits;
  const long long ld = epi == E_QKV ? p.nqkv : p.V;
  bf16* op = out + m * ld + n;
  if (n + 16 <= ld && (ld & 7) == 0) {
    *reinterpret_cast<uint4*>(op) = pack8(v);
    *reinterpret_cast<uint4*>(op + 8) = pack8(v + 8);
  } else {
    #pragma unroll
      for (int i = 0; i < 16; ++i)
      if (n + i < ld) op[i] = __float2bfloat16_rn(v[i]);
  }
}

// One attention scores item: keys [t0, t1) of KV head kvh of row b, K tile staged in `kt` (two 64-key
// halves of two [64 x 64] swizzled blocks).  Returns false if the tile wait failed.
__device__ __noinline__ bool ds_scores_item(const DsParams& p, int layer, int b, int kvh, int split, int valid, uint8_t* kt,
                               const volatile int* tag, uint64_t* full, int slot, long long g, uint64_t* empty,
                               uint8_t* qs, float* red, volatile int* flag, int wtid, int w4, int lane) {
  using namespace ds;
  const int t0 = split * kKeys, t1 = min(t0 + kKeys, valid);
  const int n_tiles = (t1 - t0 + 63) / 64;
  int pos = valid - 1;
  if (pos >= p.max_pos) {
    if (wtid == 0) set_status(p.status, JX_ERR_RANGE);
    pos = 0;
  }
  const bf16* qkv_row = p.qkv + (long long)b * p.nqkv;
  for (int idx = wtid; idx < 16 * 16; idx += 128) {
    const int r = idx >> 4, cg = idx & 15;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < p.n_rep) v = ds_rope8(qkv_row + (long long)(kvh * p.n_rep + r) * kHD, cg * 8, p.rd, p.cos, p.sin, pos);
    st_shared_v4(ds_swz(smem_u32(qs + (cg >> 3) * 2048), r, cg & 7), v);
  }
  const bool landed = ds_stage_wait(tag, full, slot, g, p, S_WORK_SCORES, 8 * layer + 2);
  if (!landed) *flag = 1;
  if (valid - 1 >= t0 && valid - 1 < t1) {
    // this step's key: rotate, append k and v to the cache, patch k into the staged tile
    const int kpos = valid - 1, half = (kpos - t0) >> 6, trow = (kpos - t0) & 63;
    const long long crow = (((long long)layer * p.M + b) * p.T + kpos) * ((long long)p.Hkv * kHD) + (long long)kvh * kHD;
    const int j0 = wtid * 8;
    if (j0 < kHD) {
      const uint4 k8 = ds_rope8(qkv_row + (long long)(p.Hq + kvh) * kHD, j0, p.rd, p.cos, p.sin, pos);
      const uint4 v8 = __ldcg(reinterpret_cast<const uint4*>(qkv_row + (long long)(p.Hq + p.Hkv + kvh) * kHD + j0));
      *reinterpret_cast<uint4*>(p.k_cache + crow + j0) = k8;
      *reinterpret_cast<uint4*>(p.v_cache + crow + j0) = v8;
      if (landed) st_shared_v4(ds_swz(smem_u32(kt + half * 16384 + (j0 >> 6) * 8192), trow, (j0 & 63) >> 3), k8);
    }
  }
  ds_wsync();
  const bool ok = *flag == 0;
  const int mi = lane >> 3, r8 = lane & 7;
  float s[2][2][4];
  float mrow[2] = {-INFINITY, -INFINITY};
#pragma unroll
  for (int i = 0; i < 2; ++i) {
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[i][nt][e] = -INFINITY;
    if (i >= n_tiles || !ok) continue;
    float acc[2][4] = {};
    const uint32_t kb = smem_u32(kt + i * 16384);
#pragma unroll
    for (int ks = 0; ks < kHD / 16; ++ks) {
      uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
      {
        const int row = (mi & 1) * 8 + r8, ch = ks * 2 + (mi >> 1);
        ldsm_x4(ds_swz(smem_u32(qs + (ch >> 3) * 2048), row, ch & 7), a0, a1, a2, a3);
      }
      {
        const int row = w4 * 16 + (mi >> 1) * 8 + r8, ch = ks * 2 + (mi & 1);
        ldsm_x4(ds_swz(kb + (ch >> 3) * 8192, row, ch & 7), b0, b1, b2, b3);
      }
      mma_bf16(acc[0], a0, a1, a2, a3, b0, b1);
      mma_bf16(acc[1], a0, a1, a2, a3, b2, b3);
    }
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int t = t0 + i * 64 + w4 * 16 + nt * 8 + (lane & 3) * 2 + (e & 1);
        if (t < t1) {
          const float v = rnd<bf16>(rnd<bf16>(acc[nt][e]) * p.scale_bf16);
          s[i][nt][e] = v;
          mrow[e >> 1] = fmaxf(mrow[e >> 1], v);
        }
      }
  }
  // every warp is done with the staged tile: hand the stage back to the producer
  ds_wsync();
  if (wtid == 0) mbar_arrive(empty);
  if (!ok) return false;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    mrow[h] = fmaxf(mrow[h], __shfl_xor_sync(0xffffffffu, mrow[h], 1));
    mrow[h] = fmaxf(mrow[h], __shfl_xor_sync(0xffffffffu, mrow[h], 2));
  }
  if ((lane & 3) == 0) {
    red[w4 * 16 + (lane >> 2)] = mrow[0];
    red[w4 * 16 + (lane >> 2) + 8] = mrow[1];
  }
  ds_wsync();
  float m[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int row = (lane >> 2) + h * 8;
    m[h] = fmaxf(fmaxf(red[row], red[16 + row]), fmaxf(red[32 + row], red[48 + row]));
  }
  ds_wsync();
  float l[2] = {0.f, 0.f};
  const long long sc_row = ((long long)b * p.Hq + kvh * p.n_rep) * p.T;
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int row = (lane >> 2) + (e >> 1) * 8;
        const int t = t0 + i * 64 + w4 * 16 + nt * 8 + (lane & 3) * 2 + (e & 1);
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
    red[w4 * 16 + (lane >> 2)] = l[0];
    red[w4 * 16 + (lane >> 2) + 8] = l[1];
  }
  ds_wsync();
  if (w4 == 0 && (lane & 3) == 0) {
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
  ds_wsync();
  return true;
}

// One attention P.V item (V tile staged in `vt`): exact probabilities from every split's statistics,
// P.V, the split partial to the workspace; the last split of a (row, KV head) to arrive sums the
// partials in split order into the bf16 output (K128 layout).
__device__ __noinline__ bool ds_pv_item(const DsParams& p, int layer, int b, int kvh, int split, int valid, uint8_t* vt,
                           const volatile int* tag, uint64_t* full, int slot, long long g, uint64_t* empty,
                           bf16* ptile, float* Ms, float* Ls, volatile int* flag, volatile int* last, int wtid, int w4,
                           int lane) {
  using namespace ds;
  constexpr int WCOLS = kHD / 4, NT = WCOLS / 8;
  const int t0 = split * kKeys, t1 = min(t0 + kKeys, valid);
  const int n_tiles = (t1 - t0 + 63) / 64;
  const int n_active = (valid + kKeys - 1) / kKeys;
  if (wtid < 16) {
    const int row = wtid;
    float Mx = -INFINITY, Lx = 0.f;
    if (row < p.n_rep) {
      const float* st = p.stats + ((long long)b * p.Hq + kvh * p.n_rep + row) * p.n_splits * 2;
      for (int s2 = 0; s2 < n_active; ++s2) Mx = fmaxf(Mx, __ldcg(st + s2 * 2));
      for (int s2 = 0; s2 < n_active; ++s2) Lx += __ldcg(st + s2 * 2 + 1) * expf(__ldcg(st + s2 * 2) - Mx);
    }
    Ms[row] = Mx;
    Ls[row] = Lx;
  }
  ds_wsync();
  for (int idx = wtid; idx < 16 * kKeys; idx += 128) {
    const int row = idx / kKeys, k = idx % kKeys, t = t0 + k;
    float pv = 0.f;
    if (row < p.n_rep && t < t1) {
      const float s = __ldcg(p.sc + ((long long)b * p.Hq + kvh * p.n_rep + row) * p.T + t);
      pv = rnd<bf16>(expf(s - Ms[row]) / Ls[row]);
    }
    ptile[row * kPLd + k] = __float2bfloat16_rn(pv);
  }
  const bool landed = ds_stage_wait(tag, full, slot, g, p, S_WORK_PV, 8 * layer + 3);
  if (!landed) *flag = 1;
  if (landed && valid - 1 >= t0 && valid - 1 < t1) {
    // this step's value (appended to the cache by the scores item, possibly after the tile was staged)
    const int kpos = valid - 1, half = (kpos - t0) >> 6, trow = (kpos - t0) & 63;
    const int j0 = wtid * 8;
    if (j0 < kHD) {
      const bf16* vsrc = p.qkv + (long long)b * p.nqkv + (long long)(p.Hq + p.Hkv + kvh) * kHD + j0;
      st_shared_v4(ds_swz(smem_u32(vt + half * 16384 + (j0 >> 6) * 8192), trow, (j0 & 63) >> 3),
                   __ldcg(reinterpret_cast<const uint4*>(vsrc)));
    }
  }
  ds_wsync();
  const bool ok = *flag == 0;
  const int mi = lane >> 3, r8 = lane & 7;
  const int r_lo = lane >> 2, r_hi = r_lo + 8;
  float acc[NT][4] = {};
  for (int i = 0; i < n_tiles && ok; ++i) {
    const uint32_t vb = smem_u32(vt + i * 16384);
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t a0, a1, a2, a3;
      {
        const int row = (mi & 1) * 8 + r8, col = i * 64 + kk * 16 + (mi >> 1) * 8;
        ldsm_x4(smem_u32(ptile + row * kPLd + col), a0, a1, a2, a3);
      }
#pragma unroll
      for (int n16 = 0; n16 < NT / 2; ++n16) {
        uint32_t b0, b1, b2, b3;
        const int row = kk * 16 + (mi & 1) * 8 + r8;
        const int ch = (w4 * WCOLS) / 8 + n16 * 2 + (mi >> 1);
        ldsm_x4_t(ds_swz(vb + (ch >> 3) * 8192, row, ch & 7), b0, b1, b2, b3);
        mma_bf16(acc[n16 * 2], a0, a1, a2, a3, b0, b1);
        mma_bf16(acc[n16 * 2 + 1], a0, a1, a2, a3, b2, b3);
      }
    }
  }
  ds_wsync();
  if (wtid == 0) mbar_arrive(empty);
  if (!ok) return false;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int row = (e >> 1) ? r_hi : r_lo;
      const int col = w4 * WCOLS + nt * 8 + (lane & 3) * 2 + (e & 1);
      if (row < p.n_rep)
        p.opart[(((long long)b * p.Hq + kvh * p.n_rep + row) * p.n_splits + split) * kHD + col] = acc[nt][e];
    }
  __threadfence();
  ds_wsync();
  if (wtid == 0) {
    const int prev = atomicAdd(&p.acnt[b * p.Hkv + kvh], 1);
    *last = (prev == n_active - 1);
  }
  ds_wsync();
  if (*last) {
    __threadfence();
    for (int idx = wtid; idx < p.n_rep * kHD; idx += 128) {
      const int row = idx / kHD, col = idx % kHD;
      const float* src = p.opart + (((long long)b * p.Hq + kvh * p.n_rep + row) * p.n_splits) * kHD + col;
      float sum = 0.f;
      for (int s2 = 0; s2 < n_active; ++s2) sum += __ldcg(src + (long long)s2 * kHD);
      const long long ocol = (long long)(kvh * p.n_rep + row) * kHD + col;
      p.attn[k128_offset(b, ocol, 16)] = __float2bfloat16_rn(sum);
    }
    if (wtid == 0) p.acnt[b * p.Hkv + kvh] = 0;
  }
  ds_wsync();
  return true;
}

// Single-pass attention for all keys [0, valid) of KV head kvh of row b: the K tiles, then the V tiles,
// of this item arrive as stages g0 .. g0 + 2 nk - 1.  The rounded scores of the n_rep query rows stay in
// shared memory (bf16: they are bf16 values), so the exact normaliser comes from the whole row without a
// second phase: row max and sum of exp(s - max) over every key, then bf16 probabilities per 128-key tile,
// P.V accumulated in float32 over all tiles and rounded once into the output (K128 layout).  `cap` is the
// row stride of the score buffer (keys).  Returns false if a stage wait failed.
__device__ __noinline__ bool ds_attn_item(const DsParams& p, int layer, int b, int kvh, int valid, int cap, uint8_t* ring,
                             const volatile int* tag, uint64_t* full, uint64_t* empty, long long g0, uint8_t* qs,
                             float* red, bf16* sbuf, bf16* ptile, float* Ms, float* Ls, volatile int* flag, int wtid,
                             int w4, int lane) {
  using namespace ds;
  constexpr int WCOLS = kHD / 4, NT = WCOLS / 8;
  const int nk = (valid + kKeys - 1) / kKeys;
  const int mi = lane >> 3, r8 = lane & 7;
  int pos = valid - 1;
  if (pos >= p.max_pos) {
    if (wtid == 0) set_status(p.status, JX_ERR_RANGE);
    pos = 0;
  }
  const bf16* qkv_row = p.qkv + (long long)b * p.nqkv;
  for (int idx = wtid; idx < 16 * 16; idx += 128) {
    const int r = idx >> 4, cg = idx & 15;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < p.n_rep) v = ds_rope8(qkv_row + (long long)(kvh * p.n_rep + r) * kHD, cg * 8, p.rd, p.cos, p.sin, pos);
    st_shared_v4(ds_swz(smem_u32(qs + (cg >> 3) * 2048), r, cg & 7), v);
  }
  float mrow[2] = {-INFINITY, -INFINITY};   // query rows lane / 4 and lane / 4 + 8
  // ---- scores: q . k over every K tile ----
  for (int j = 0; j < nk; ++j) {
    const long long g = g0 + j;
    const int slot = (int)(g % kStages);
    uint8_t* kt = ring + slot * kStageBytes;
    const int t0 = j * kKeys, t1 = min(t0 + kKeys, valid);
    const bool landed = ds_stage_wait(tag, full, slot, g, p, S_WORK_SCORES, -1);
    if (!landed) *flag = 1;
    if (valid - 1 >= t0 && valid - 1 < t1) {
      // this step's key: rotate, append k and v to the cache, patch k into the staged tile
      const int kpos = valid - 1, half = (kpos - t0) >> 6, trow = (kpos - t0) & 63;
      const long long crow =
          (((long long)layer * p.M + b) * p.T + kpos) * ((long long)p.Hkv * kHD) + (long long)kvh * kHD;
      const int j0 = wtid * 8;
      if (j0 < kHD) {
        const uint4 k8 = ds_rope8(qkv_row + (long long)(p.Hq + kvh) * kHD, j0, p.rd, p.cos, p.sin, pos);
        const uint4 v8 = __ldcg(reinterpret_cast<const uint4*>(qkv_row + (long long)(p.Hq + p.Hkv + kvh) * kHD + j0));
        *reinterpret_cast<uint4*>(p.k_cache + crow + j0) = k8;
        *reinterpret_cast<uint4*>(p.v_cache + crow + j0) = v8;
        if (landed) st_shared_v4(ds_swz(smem_u32(kt + half * 16384 + (j0 >> 6) * 8192), trow, (j0 & 63) >> 3), k8);
      }
    }
    ds_wsync();
    const bool ok = *flag == 0;
    const int n_half = (t1 - t0 + 63) / 64;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      if (i >= n_half || !ok) continue;
      float acc[2][4] = {};
      const uint32_t kb = smem_u32(kt + i * 16384);
#pragma unroll
      for (int ks = 0; ks < kHD / 16; ++ks) {
        uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
        {
          const int row = (mi & 1) * 8 + r8, ch = ks * 2 + (mi >> 1);
          ldsm_x4(ds_swz(smem_u32(qs + (ch >> 3) * 2048), row, ch & 7), a0, a1, a2, a3);
        }
        {
          const int row = w4 * 16 + (mi >> 1) * 8 + r8, ch = ks * 2 + (mi & 1);
          ldsm_x4(ds_swz(kb + (ch >> 3) * 8192, row, ch & 7), b0, b1, b2, b3);
        }
        mma_bf16(acc[0], a0, a1, a2, a3, b0, b1);
        mma_bf16(acc[1], a0, a1, a2, a3, b2, b3);
      }
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int row = (lane >> 2) + (e >> 1) * 8;
          const int t = t0 + i * 64 + w4 * 16 + nt * 8 + (lane & 3) * 2 + (e & 1);
          if (t < t1 && row < p.n_rep) {
            const float v = rnd<bf16>(rnd<bf16>(acc[nt][e]) * p.scale_bf16);
            sbuf[row * cap + t] = __float2bfloat16_rn(v);
            mrow[e >> 1] = fmaxf(mrow[e >> 1], v);
          }
        }
    }
    // every warp is done with the staged tile: hand the stage back to the producer
    ds_wsync();
    if (wtid == 0) mbar_arrive(&empty[slot]);
    if (!ok) return false;
  }
  // ---- exact softmax statistics over the whole row ----
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    mrow[h] = fmaxf(mrow[h], __shfl_xor_sync(0xffffffffu, mrow[h], 1));
    mrow[h] = fmaxf(mrow[h], __shfl_xor_sync(0xffffffffu, mrow[h], 2));
  }
  if ((lane & 3) == 0) {
    red[w4 * 16 + (lane >> 2)] = mrow[0];
    red[w4 * 16 + (lane >> 2) + 8] = mrow[1];
  }
  ds_wsync();
  if (wtid < 16) Ms[wtid] = fmaxf(fmaxf(red[wtid], red[16 + wtid]), fmaxf(red[32 + wtid], red[48 + wtid]));
  ds_wsync();
  // sum of exp(s - max): warp w4 takes rows w4, w4 + 4, ... (lanes stride over the keys, in order)
  for (int row = w4; row < p.n_rep; row += 4) {
    float l = 0.f;
    const float mx = Ms[row];
    for (int t = lane; t < valid; t += 32) l += expf(__bfloat162float(sbuf[row * cap + t]) - mx);
    for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    if (lane == 0) Ls[row] = l;
  }
  ds_wsync();
  // ---- P.V over every V tile ----
  float acc[NT][4] = {};
  for (int j = 0; j < nk; ++j) {
    const long long g = g0 + nk + j;
    const int slot = (int)(g % kStages);
    uint8_t* vt = ring + slot * kStageBytes;
    const int t0 = j * kKeys, t1 = min(t0 + kKeys, valid);
    for (int idx = wtid; idx < 16 * kKeys; idx += 128) {
      const int row = idx / kKeys, k = idx % kKeys, t = t0 + k;
      float pv = 0.f;
      if (row < p.n_rep && t < t1) pv = rnd<bf16>(expf(__bfloat162float(sbuf[row * cap + t]) - Ms[row]) / Ls[row]);
      ptile[row * kPLd + k] = __float2bfloat16_rn(pv);
    }
    const bool landed = ds_stage_wait(tag, full, slot, g, p, S_WORK_PV, -1);
    if (!landed) *flag = 1;
    if (landed && valid - 1 >= t0 && valid - 1 < t1) {
      // this step's value (appended above, possibly after the tile was staged)
      const int kpos = valid - 1, half = (kpos - t0) >> 6, trow = (kpos - t0) & 63;
      const int j0 = wtid * 8;
      if (j0 < kHD)
        st_shared_v4(ds_swz(smem_u32(vt + half * 16384 + (j0 >> 6) * 8192), trow, (j0 & 63) >> 3),
                     __ldcg(reinterpret_cast<const uint4*>(qkv_row + (long long)(p.Hq + p.Hkv + kvh) * kHD + j0)));
    }
    ds_wsync();
    const bool ok = *flag == 0;
    const int n_half = (t1 - t0 + 63) / 64;
    for (int i = 0; i < n_half && ok; ++i) {
      const uint32_t vb = smem_u32(vt + i * 16384);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t a0, a1, a2, a3;
        {
          const int row = (mi & 1) * 8 + r8, col = i * 64 + kk * 16 + (mi >> 1) * 8;
          ldsm_x4(smem_u32(ptile + row * kPLd + col), a0, a1, a2, a3);
        }
#pragma unroll
        for (int n16 = 0; n16 < NT / 2; ++n16) {
          uint32_t b0, b1, b2, b3;
          const int row = kk * 16 + (mi & 1) * 8 + r8;
          const int ch = (w4 * WCOLS) / 8 + n16 * 2 + (mi >> 1);
          ldsm_x4_t(ds_swz(vb + (ch >> 3) * 8192, row, ch & 7), b0, b1, b2, b3);
          mma_bf16(acc[n16 * 2], a0, a1, a2, a3, b0, b1);
          mma_bf16(acc[n16 * 2 + 1], a0, a1, a2, a3, b2, b3);
        }
      }
    }
    ds_wsync();
    if (wtid == 0) mbar_arrive(&empty[slot]);
    if (!ok) return false;
  }
  const int r_lo = lane >> 2, r_hi = r_lo + 8;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int row = (e >> 1) ? r_hi : r_lo;
      const int col = w4 * WCOLS + nt * 8 + (lane & 3) * 2 + (e & 1);
      if (row < p.n_rep)
        p.attn[k128_offset(b, (long long)(kvh * p.n_rep + row) * kHD + col, 16)] = __float2bfloat16_rn(acc[nt][e]);
    }
  ds_wsync();
  return true;
}

// Split-K fix-up of block nb by its last arriver: the partial tiles of CTAs c_first .. c_last summed in CTA
// order into the staging tile (own = this CTA when its own partial is still in the tile, else -1).  Each
// thread owns 4 float4 of the [16 x 128] tile; the loads of up to 4 contributors are issued before any is
// added, so their L2 round trips overlap.  (Inlined, 4 at a time: a call, or 8 at a time, measured slower.)
__device__ __forceinline__ void ds_splitk_sum(const DsParams& p, long long nb, int c_first, int c_last, int own,
                                           long long total, int kc, int Gp, float* tile, int wtid) {
  using namespace ds;
  float4 acc4[4];
  for (int cc0 = c_first; cc0 <= c_last; cc0 += 4) {
    float4 vv[4][4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int cc = cc0 + u;
      if (cc > c_last) break;
      if (cc == own) {
#pragma unroll
        for (int qq = 0; qq < 4; ++qq) {
          const int e0 = (wtid + qq * 128) * 4;
          vv[u][qq] = *reinterpret_cast<const float4*>(tile + (e0 >> 7) * kTileLd + (e0 & 127));
        }
      } else {
        const long long nbf = ds_begin(total, Gp, cc) / kc;
        const int slot = cc * 2 + (nb == nbf ? 0 : 1);
        const float4* src = reinterpret_cast<const float4*>(p.ws + (long long)slot * 16 * 128);
#pragma unroll
        for (int qq = 0; qq < 4; ++qq) vv[u][qq] = __ldcg(src + wtid + qq * 128);
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (cc0 + u > c_last) break;
#pragma unroll
      for (int qq = 0; qq < 4; ++qq) {
        if (cc0 + u == c_first) {
          acc4[qq] = vv[u][qq];
        } else {
          acc4[qq].x += vv[u][qq].x;
          acc4[qq].y += vv[u][qq].y;
          acc4[qq].z += vv[u][qq].z;
          acc4[qq].w += vv[u][qq].w;
        }
      }
    }
  }
  ds_wsync();   // every thread's reads of its own tile values are done
#pragma unroll
  for (int qq = 0; qq < 4; ++qq) {
    const int e0 = (wtid + qq * 128) * 4;
    *reinterpret_cast<float4*>(tile + (e0 >> 7) * kTileLd + (e0 & 127)) = acc4[qq];
  }
}

// ---------------------------------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(ds::kThreads, 1)
    decode_step_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                       const __grid_constant__ DsParams p) {
  using namespace ds;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;
  float* tile = reinterpret_cast<float*>(smem + kOffTile);
  uint8_t* qs = smem + kOffQ;
  bf16* ptile = reinterpret_cast<bf16*>(smem + kOffP);
  float* red = reinterpret_cast<float*>(smem + kOffRed);
  float* Ms = red + 64;
  float* Ls = Ms + 16;
  bf16* sbuf = reinterpret_cast<bf16*>(smem + kOffS);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* empty = full + kStages;
  uint64_t* accf = empty + kStages;   // [2]
  uint64_t* acce = accf + 2;          // [2]
  uint64_t* done = acce + 2;          // workers finished with TMEM
  uint64_t* mmadone = done + 1;       // every MMA issued has completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffMisc);
  // [0] S, [1] flag, [2] last, [3] wait ok, [4] phases per layer
  volatile int* sh = reinterpret_cast<volatile int*>(smem + kOffMisc + 16);
  volatile int* valid = sh + 8;                                                  // [16]
  volatile int* tag = sh + 24;                                                   // [kStages] stage in each slot

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x, c = blockIdx.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf[b], 1);
      mbar_init(&acce[b], 4);
    }
    mbar_init(done, 4);
    mbar_init(mmadone, 1);
    int S = 0;
    for (int b = 0; b < p.M; ++b) {
      int v = p.pos_id[b] + 2;   // keys after this step's append
      if (v < 1 || v > p.T) {
        set_status(p.status, JX_ERR_RANGE);
        v = v < 1 ? 1 : p.T;
      }
      valid[b] = v;
      S = max(S, (v + kKeys - 1) / kKeys);
    }
    sh[0] = S;
    sh[1] = 0;
    // single-pass attention when one item per (row, KV head) keeps at least half the CTAs busy and the
    // rounded scores of a row fit the shared buffer; otherwise split items over 128-key ranges
    const bool single = 2 * p.M * p.Hkv >= (int)gridDim.x && p.n_rep * S * kKeys * 2 <= kSBufBytes;
    sh[4] = single ? 7 : 8;
    for (int s = 0; s < kStages; ++s) tag[s] = -1;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 32);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int S = sh[0];
  const int ppl = sh[4];
  const int NP = ppl * p.L + 2;
  const int n_items = p.M * p.Hkv * S;        // split items (two-phase attention)
  const int n_pairs = p.M * p.Hkv;            // single-pass items

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      prefetch_tmap(&kmap);
      prefetch_tmap(&vmap);
      const uint64_t pol = l2_policy_evict_first();   // weights and K/V are read once per step
      const uint64_t pol_keep = l2_policy_evict_last();
      long long g = 0;                                 // stages issued
      bool dead = false;
      // L2 lookahead: before every wait, the weight tiles of this CTA's next l2_ahead projection stages
      // (across phase boundaries) are prefetched into L2, so HBM keeps streaming through phase tails,
      // grid barriers and the attention phase, and those stages then load from L2.
      long long proj_issued = 0;                       // projection stages issued to the ring
      long long pf_n = 0, pf_it = 0, pf_it1 = 0;       // cursor: stages passed, range in its phase
      int pf_q = 0, pf_kc = 1;
      long long pf_np = 0;
      const bf16* pf_w = nullptr;
      auto lookahead = [&]() {
        while (pf_n < proj_issued + p.l2_ahead) {
          if (pf_it >= pf_it1) {   // the cursor moves on to the next projection phase this CTA has a share of
            bool found = false;
            while (!found && pf_q < NP) {
              const int qq = pf_q++;
              if (ds_kind(p, qq, ppl) != PROJ) continue;
              const DsProj pp = ds_proj(p, qq, ppl);
              pf_kc = (int)(pp.Kp >> 7);
              ds_range((pp.Np >> 7) * pf_kc, G, c, pf_it, pf_it1);
              pf_w = pp.W;
              pf_np = pp.Np;
              found = pf_it < pf_it1;
            }
            if (!found) return;
          }
          if (pf_n >= proj_issued) {
            const long long nb = pf_it / pf_kc, kk = pf_it - nb * pf_kc;
            bulk_prefetch_l2(pf_w + ((kk * (pf_np >> 3) + nb * 16) << 10), kWBytes, pol_keep);
          }
          ++pf_it;
          ++pf_n;
        }
      };
      for (int q = 0; q < NP && !dead; ++q) {
        const int kind = ds_kind(p, q, ppl);
        if (kind == PROJ) {
          const DsProj pr = ds_proj(p, q, ppl);
          const int kc = (int)(pr.Kp >> 7);
          const long long total = (pr.Np >> 7) * kc;
          long long it0, it1;
          ds_range(total, G, c, it0, it1);
          const int n = (int)(it1 - it0);
          if (n == 0) continue;
          auto wsrc = [&](long long it) {
            const long long nb = it / kc, kk = it - nb * kc;
            return pr.W + ((kk * (pr.Np >> 3) + nb * 16) << 10);
          };
          auto xsrc = [&](long long it) { return pr.X + (((it % kc) * 2) << 10); };
          // weights first (they do not depend on this step), as far as the ring allows
          const int pre = n < kStages ? n : kStages;
          int nw = 0;
          for (; nw < pre; ++nw) {
            const long long gg = g + nw;
            const int s = (int)(gg % kStages);
            lookahead();
            if (gg >= kStages && !ds_wait(&empty[s], (uint32_t)(((gg / kStages) - 1) & 1), p, S_PROD_EMPTY_PRE, q, gg)) {
              dead = true;
              break;
            }
            tag[s] = (int)gg;
            mbar_arrive_expect_tx(&full[s], kStageBytes);
            bulk_g2s_hint(ring + s * kStageBytes, wsrc(it0 + nw), kWBytes, &full[s], pol);
            ++proj_issued;
          }
          lookahead();
          // the activations exist once every CTA has finished the phases before this one
          const bool ok = !dead && ds_grid_wait(p, q * G, S_PROD_GRID, q);
          if (ok) {
            asm volatile("fence.acq_rel.gpu;" ::: "memory");
            fence_proxy_async_global();
          }
          // (issued even after a failure, so every stage that expects them completes before the drain)
          for (int i = 0; i < nw; ++i) {
            const int s = (int)((g + i) % kStages);
            bulk_g2s(ring + s * kStageBytes + kWBytes, xsrc(it0 + i), kXBytes, &full[s]);
          }
          if (!ok) {
            dead = true;
            g += nw;
            break;
          }
          for (int i = pre; i < n; ++i) {
            const long long gg = g + i;
            const int s = (int)(gg % kStages);
            lookahead();
            if (!ds_wait(&empty[s], (uint32_t)(((gg / kStages) - 1) & 1), p, S_PROD_EMPTY, q, gg)) {
              dead = true;
              g += i;
              break;
            }
            tag[s] = (int)gg;
            mbar_arrive_expect_tx(&full[s], kStageBytes);
            bulk_g2s_hint(ring + s * kStageBytes, wsrc(it0 + i), kWBytes, &full[s], pol);
            bulk_g2s(ring + s * kStageBytes + kWBytes, xsrc(it0 + i), kXBytes, &full[s]);
            ++proj_issued;
          }
          if (!dead) g += n;
        } else if (kind == ATTN) {
          const long long row0 = (long long)(q / ppl) * p.M * p.T;
          for (int i = c; i < n_pairs && !dead; i += G) {
            const int b = i / p.Hkv, kvh = i % p.Hkv;
            const int nk = (valid[b] + kKeys - 1) / kKeys;
            for (int j = 0; j < 2 * nk; ++j) {
              const int s = (int)(g % kStages);
              lookahead();
              if (g >= kStages && !ds_wait(&empty[s], (uint32_t)(((g / kStages) - 1) & 1), p, S_PROD_EMPTY_ATTN, q, g)) {
                dead = true;
                break;
              }
              tag[s] = (int)g;
              mbar_arrive_expect_tx(&full[s], kWBytes);
              const CUtensorMap* map = j < nk ? &kmap : &vmap;
              const int y0 = (int)(row0 + (long long)b * p.T + (j < nk ? j : j - nk) * kKeys);
#pragma unroll
              for (int hh = 0; hh < 2; ++hh)
#pragma unroll
                for (int cb = 0; cb < 2; ++cb)
                  tma_load_2d(ring + s * kStageBytes + hh * 16384 + cb * 8192, map, kvh * kHD + cb * 64, y0 + hh * 64,
                              &full[s]);
              ++g;
            }
          }
        } else if (kind == SCORES || kind == PV) {
          const CUtensorMap* map = kind == SCORES ? &kmap : &vmap;
          const long long row0 = (long long)(q / ppl) * p.M * p.T;
          for (int i = c; i < n_items; i += G) {
            int b, kvh, split;
            if (!ds_item(i, S, p.Hkv, valid, b, kvh, split)) continue;
            const int s = (int)(g % kStages);
            lookahead();
            if (g >= kStages && !ds_wait(&empty[s], (uint32_t)(((g / kStages) - 1) & 1), p, S_PROD_EMPTY_ATTN, q, g)) {
              dead = true;
              break;
            }
            tag[s] = (int)g;
            mbar_arrive_expect_tx(&full[s], kWBytes);
            const int y0 = (int)(row0 + (long long)b * p.T + split * kKeys);
#pragma unroll
            for (int hh = 0; hh < 2; ++hh)
#pragma unroll
              for (int cb = 0; cb < 2; ++cb)
                tma_load_2d(ring + s * kStageBytes + hh * 16384 + cb * 8192, map, kvh * kHD + cb * 64, y0 + hh * 64,
                            &full[s]);
            ++g;
          }
        }
      }
      // every copy issued must land before this CTA's shared memory is released
      for (long long gg = (g > kStages ? g - kStages : 0); gg < g; ++gg)
        if (!mbar_wait_bounded(&full[gg % kStages], (uint32_t)((gg / kStages) & 1))) break;
      if (dead) ds_abort(p, S_END, -1, g);
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer ------------------------------
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16_f32(128, 16);
      long long g = 0;
      long long g_foreign_end = 0;   // first stage after the last attention stages (which the workers consume)
      int blk = -1;
      bool dead = false;
      for (int q = 0; q < NP && !dead; ++q) {
        const int kind = ds_kind(p, q, ppl);
        if (kind == PROJ) {
          const DsProj pr = ds_proj(p, q, ppl);
          const int kc = (int)(pr.Kp >> 7);
          const long long total = (pr.Np >> 7) * kc;
          long long it0, it1;
          ds_range(total, G, c, it0, it1);
          long long cur_nb = -1;
          uint32_t dcol = 0;
          bool first = true;
          for (long long it = it0; it < it1; ++it, ++g) {
            const long long nb = it / kc, kk = it - nb * kc;
            if (nb != cur_nb) {
              cur_nb = nb;
              ++blk;
              const int buf = blk & 1;
              if (blk >= 2 && !ds_wait(&acce[buf], (uint32_t)(((blk >> 1) - 1) & 1), p, S_MMA_ACCE, q, blk)) {
                dead = true;
                break;
              }
              tc_fence_after();
              dcol = (uint32_t)(buf * 16);
              first = true;
            }
            const int s = (int)(g % kStages);
            const bool ok_full = (g - kStages >= g_foreign_end)
                                     ? ds_wait(&full[s], (uint32_t)((g / kStages) & 1), p, S_MMA_FULL, q, g)
                                     : ds_stage_wait(tag, full, s, g, p, S_MMA_FULL, q);
            if (!ok_full) {
              dead = true;
              break;
            }
            tc_fence_after();
            const uint32_t sw = smem_u32(ring + s * kStageBytes);
            const uint32_t sx = sw + kWBytes;
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {
              const uint64_t ad = umma_desc_kmajor(sw + ks * 256, 128, 2048);
              const uint64_t bd = umma_desc_kmajor(sx + ks * 256, 128, 2048);
              umma_bf16(tmem + dcol, ad, bd, idesc, (first && ks == 0) ? 0u : 1u);
            }
            first = false;
            umma_commit(&empty[s]);
            if (kk == kc - 1 || it == it1 - 1) umma_commit(&accf[blk & 1]);
          }
        } else if (kind == ATTN) {
          for (int i = c; i < n_pairs; i += G) g += 2 * ((valid[i / p.Hkv] + kKeys - 1) / kKeys);
          g_foreign_end = g;
        } else if (kind == SCORES || kind == PV) {
          for (int i = c; i < n_items; i += G) {
            int b, kvh, split;
            if (ds_item(i, S, p.Hkv, valid, b, kvh, split)) ++g;
          }
          g_foreign_end = g;
        }
      }
      // every MMA issued has completed before TMEM is freed
      umma_commit(mmadone);
      mbar_wait_bounded(mmadone, 0);
      if (dead) ds_abort(p, S_END, -2, g);
    }
  } else {
    // ------------------------------ workers (warps 2..5) ------------------------------
    const int wtid = threadIdx.x - 64, w4 = warp - 2;
    const int quad = warp & 3;                 // TMEM lane quadrant this warp may read
    long long g = 0;
    int blk = -1;
    bool dead = false;
    for (int q = 0; q < NP && !dead; ++q) {
      const int kind = ds_kind(p, q, ppl);
      // Every phase starts once every CTA has arrived for the phases before it (count >= q * G).  No CTA
      // arrives for phase q before that, so the count reaches q * G only when each CTA has arrived once
      // for each earlier phase.  (A projection's epilogue needs its activations anyway; the wait matters
      // for CTAs with no share of the phase, which would otherwise arrive early.)
      if (wtid == 0) sh[3] = ds_grid_wait(p, q * G, S_WORK_GRID, q) ? 1 : 0;
      ds_wsync();
      if (!sh[3]) {
        dead = true;
        break;
      }
      if (kind == PROJ) {
        const DsProj pr = ds_proj(p, q, ppl);
        const int kc = (int)(pr.Kp >> 7);
        const long long total = (pr.Np >> 7) * kc;
        long long it0, it1;
        const int Gp = ds_range(total, G, c, it0, it1);
        g += it1 - it0;
        long long cur_nb = -1;
        bool started_at_zero = false;
        for (long long it = it0; it < it1 && !dead; ++it) {
          const long long nb = it / kc, kk = it - nb * kc;
          if (nb != cur_nb) {
            cur_nb = nb;
            ++blk;
            started_at_zero = (kk == 0);
          }
          const bool block_end = (kk == kc - 1) || (it == it1 - 1);
          if (!block_end) continue;
          const int buf = blk & 1;
          bool ok = ds_wait(&accf[buf], (uint32_t)((blk >> 1) & 1), p, S_WORK_ACCF, q, blk);
          ok = __all_sync(0xffffffffu, ok);   // tcgen05.ld is warp-wide
          tc_fence_after();
          if (ok) {
            float v[16];
            tmem_ld16(tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(buf * 16), v);
            const int row = quad * 32 + lane;
#pragma unroll
            for (int j = 0; j < 16; ++j) tile[j * kTileLd + row] = v[j];
          } else if (lane == 0) {
            sh[1] = 1;
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acce[buf]);
          ds_wsync();
          if (sh[1]) {
            dead = true;
            break;
          }
          const bool whole = started_at_zero && (kk == kc - 1);
          bool do_epi = whole;
          if (!whole) {
            const int c_first = ds_cta_of(nb * kc, total, Gp), c_last = ds_cta_of(nb * kc + kc - 1, total, Gp);
            auto slot_of = [&](int cc) {
              const long long nbf = ds_begin(total, Gp, cc) / kc;
              return cc * 2 + (nb == nbf ? 0 : 1);
            };
            bool fast = false;
            if (c == c_first) {
              if (wtid == 0) sh[2] = (ld_acquire_gpu(&p.counters[nb]) == c_last - c_first) ? 1 : 0;
              ds_wsync();
              fast = sh[2] != 0;
              ds_wsync();
            }
            if (fast) {
              do_epi = true;
            } else {
              float4* my = reinterpret_cast<float4*>(p.ws + (long long)slot_of(c) * 16 * 128);
#pragma unroll
              for (int qq = 0; qq < 4; ++qq) {
                const int e0 = (wtid + qq * 128) * 4;
                my[wtid + qq * 128] = *reinterpret_cast<const float4*>(tile + (e0 >> 7) * kTileLd + (e0 & 127));
              }
              __threadfence();
              ds_wsync();
              if (wtid == 0) {
                const int prev = atomicAdd(&p.counters[nb], 1);
                sh[2] = (prev == c_last - c_first) ? 1 : 0;
              }
              ds_wsync();
              do_epi = sh[2] != 0;
            }
            if (do_epi) {
              __threadfence();
              ds_splitk_sum(p, nb, c_first, c_last, fast ? c : -1, total, kc, Gp, tile, wtid);
              if (wtid == 0) p.counters[nb] = 0;
              ds_wsync();
            }
          }
          if (do_epi) ds_epilogue(p, pr.epi, nb * 128, tile, wtid);
          ds_wsync();
        }
      } else {
        if (kind == NORM) {
          if (c < p.M) {
            const bool fin = q == ppl * p.L;
            const bf16* w = fin ? p.final_norm : p.layers[(q / ppl) * 6 + (ds_lj(q, ppl) == 0 ? 4 : 5)];
            ds_norm_row(p, c, w, q == 0, wtid, red);
          }
        } else if (kind == ATTN) {
          for (int i = c; i < n_pairs; i += G) {
            const int b = i / p.Hkv, kvh = i % p.Hkv;
            const int nk = (valid[b] + kKeys - 1) / kKeys;
            const bool ok = ds_attn_item(p, q / ppl, b, kvh, valid[b], S * kKeys, ring, tag, full, empty, g, qs, red,
                                         sbuf, ptile, Ms, Ls, &sh[1], wtid, w4, lane);
            g += 2 * nk;
            if (!ok) {
              dead = true;
              break;
            }
          }
          if (dead) break;
        } else {
          for (int i = c; i < n_items; i += G) {
            int b, kvh, split;
            if (!ds_item(i, S, p.Hkv, valid, b, kvh, split)) continue;
            const int s = (int)(g % kStages);
            const long long gi = g++;
            const bool ok = kind == SCORES
                                ? ds_scores_item(p, q / ppl, b, kvh, split, valid[b], ring + s * kStageBytes, tag, full,
                                                 s, gi, &empty[s], qs, red, &sh[1], wtid, w4, lane)
                                : ds_pv_item(p, q / ppl, b, kvh, split, valid[b], ring + s * kStageBytes, tag, full, s,
                                             gi, &empty[s], ptile, Ms, Ls, &sh[1], &sh[2], wtid, w4, lane);
            if (!ok) {
              dead = true;
              break;
            }
          }
          if (dead) break;
        }
      }
      // this CTA's part of phase q is done and stored
      ds_wsync();
      if (wtid == 0) ds_grid_arrive(p);
    }
    if (dead && wtid == 0) ds_abort(p, S_END, -3, g);
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(done);
  }
  // TMEM is freed once the workers' reads and every MMA are complete
  if (warp == 1) {
    __syncwarp();
    if (!mbar_wait_bounded(done, 0)) set_status(p.status, JX_ERR_TIMEOUT);
    tc_fence_after();
    tmem_dealloc(tmem, 32);
  }
}

}  // namespace jxb

using namespace jxb;

static int g_l2_ahead = 0;
extern "C" int jx_set_decode_step_lookahead(int stages) {
  if (stages < 0 || stages > 64) return fail(JX_ERR_ARG, "jx_set_decode_step_lookahead: stages must be in [0, 64]");
  g_l2_ahead = stages;
  return JX_OK;
}

extern "C" int jx_decode_step(const jx_step_args* a, void* stream) {
  using namespace ds;
  if (!a) return fail(JX_ERR_ARG, "jx_decode_step: null arguments");
  if (a->M < 1 || a->M > 16 || a->L < 1 || a->hd != kHD || a->Hkv < 1 || a->Hq % a->Hkv || a->Hq / a->Hkv > 16)
    return fail(JX_ERR_SHAPE, "jx_decode_step: needs 1 <= M <= 16, head_dim 128, Hq a multiple of Hkv, n_rep <= 16");
  if (a->d < 8 || a->d % 8 || a->d > 8192 || a->F < 1 || a->V < 1 || a->vocab < 1 || a->T < 2)
    return fail(JX_ERR_SHAPE, "jx_decode_step: needs d % 8 == 0, d <= 8192, F, V, vocab >= 1, T >= 2");
  if (a->rd <= 0 || a->rd > kHD || a->rd % 16 || a->max_pos < 1)
    return fail(JX_ERR_SHAPE, "jx_decode_step: rotary dims must be a positive multiple of 16, at most 128");
  const long long nqkv = (long long)(a->Hq + 2 * a->Hkv) * kHD;
  const long long nps[4] = {a->Np_qkv, a->Np_d, a->Np_gu, a->Np_v};
  const long long kps[3] = {a->Kp_d, a->Kp_o, a->Kp_f};
  for (long long v : nps)
    if (v <= 0 || v % 128) return fail(JX_ERR_SHAPE, "jx_decode_step: padded rows must be positive multiples of 128");
  for (long long v : kps)
    if (v <= 0 || v % 128) return fail(JX_ERR_SHAPE, "jx_decode_step: padded K must be positive multiples of 128");
  if (a->Np_qkv < nqkv || a->Np_d < a->d || a->Np_gu < 2 * ((a->F + 31) / 32 * 32) || a->Np_v < a->V ||
      a->Kp_d < a->d || a->Kp_o < (long long)a->Hq * kHD || a->Kp_f < a->F)
    return fail(JX_ERR_SHAPE, "jx_decode_step: padded extents smaller than the model");
  const void* ptrs[] = {a->layers, a->embed, a->ids, a->final_norm, a->lm_head, a->h, a->xn, a->qkv, a->attn, a->act,
                        a->logits, a->k_cache, a->v_cache, a->cos, a->sin, a->pos_id, a->ws, a->counters,
                        a->attn_ws, a->attn_counters, a->sync};
  for (const void* q : ptrs)
    if (!q) return fail(JX_ERR_ARG, "jx_decode_step: null pointer");
  uintptr_t al = 0;
  const void* aligned[] = {a->embed, a->final_norm, a->lm_head, a->h, a->xn, a->qkv, a->attn, a->act, a->k_cache,
                           a->v_cache, a->cos, a->sin, a->ws, a->attn_ws};
  for (const void* q : aligned) al |= reinterpret_cast<uintptr_t>(q);
  if ((al & 15) || (a->d % 8) || (nqkv % 8))
    return fail(JX_ERR_ARG, "jx_decode_step: buffers must be 16-byte aligned");

  static int sms = 0, occ = 0;
  if (!sms) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return note_cuda("jx_decode_step: device query");
    if (cudaFuncSetAttribute(decode_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, decode_step_kernel, kThreads, kSmem) != cudaSuccess)
      return note_cuda("jx_decode_step: kernel attributes");
  }
  if (occ < 1) return fail(JX_ERR_UNSUPPORTED, "jx_decode_step: the kernel does not fit on an SM");
  int grid = a->grid > 0 ? a->grid : sms;
  if (grid > sms * occ) grid = sms * occ;
  if (a->ws_floats < (long long)grid * 2 * 16 * 128) return fail(JX_ERR_ARG, "jx_decode_step: split-K workspace too small");
  const int n_splits = dattn_n_splits(a->T, 0);
  if (a->attn_ws_bytes < dattn_workspace_bytes(a->M, a->Hq, a->T, kHD, n_splits))
    return fail(JX_ERR_ARG, "jx_decode_step: attention workspace too small");

  CUtensorMap km, vm;
  const long long rows = (long long)a->L * a->M * a->T, cols = (long long)a->Hkv * kHD;
  if (make_tmap_2d_bf16(&km, a->k_cache, rows, cols, cols) != JX_OK ||
      make_tmap_2d_bf16(&vm, a->v_cache, rows, cols, cols) != JX_OK)
    return fail(JX_ERR_ARG, "jx_decode_step: cache tensor maps");

  DsParams p;
  p.M = a->M, p.L = a->L, p.d = a->d, p.Hq = a->Hq, p.Hkv = a->Hkv, p.n_rep = a->Hq / a->Hkv, p.T = a->T;
  p.rd = a->rd, p.max_pos = a->max_pos, p.V = a->V, p.vocab = a->vocab, p.F = a->F, p.nqkv = (int)nqkv;
  p.n_splits = n_splits;
  p.Np_qkv = a->Np_qkv, p.Np_d = a->Np_d, p.Np_gu = a->Np_gu, p.Np_v = a->Np_v;
  p.Kp_d = a->Kp_d, p.Kp_o = a->Kp_o, p.Kp_f = a->Kp_f;
  p.eps = a->eps;
  p.scale_bf16 = __bfloat162float(__float2bfloat16_rn(a->scale));
  p.layers = reinterpret_cast<const bf16* const*>(a->layers);
  p.embed = (const bf16*)a->embed, p.ids = a->ids, p.final_norm = (const bf16*)a->final_norm;
  p.lm_head = (const bf16*)a->lm_head;
  p.h = (bf16*)a->h, p.xn = (bf16*)a->xn, p.qkv = (bf16*)a->qkv, p.attn = (bf16*)a->attn, p.act = (bf16*)a->act;
  p.logits = (bf16*)a->logits, p.k_cache = (bf16*)a->k_cache, p.v_cache = (bf16*)a->v_cache;
  p.cos = (const bf16*)a->cos, p.sin = (const bf16*)a->sin, p.pos_id = a->pos_id;
  p.ws = a->ws, p.counters = a->counters;
  float* aw = reinterpret_cast<float*>(a->attn_ws);
  p.sc = aw;
  p.stats = p.sc + (long long)a->M * a->Hq * a->T;
  p.opart = p.stats + (long long)a->M * a->Hq * n_splits * 2;
  p.acnt = a->attn_counters;
  p.sync = a->sync, p.status = a->status;
  p.l2_ahead = g_l2_ahead;

  cudaStream_t s = (cudaStream_t)stream;
  if (cudaMemsetAsync(a->sync, 0, 6 * sizeof(int), s) != cudaSuccess) return note_cuda("jx_decode_step: clearing sync");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, decode_step_kernel, km, vm, p) != cudaSuccess) return note_cuda("jx_decode_step");
  return JX_OK;
}
