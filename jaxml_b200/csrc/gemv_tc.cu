// Decode projection on the 5th-generation tensor cores (tcgen05 + TMEM): Y[M, N] = X[M, K] . W[N, K]^T
// for M <= 64 token rows, bfloat16 operands in the K128 tiled layout, float32 accumulation in TMEM.
//
// Same work split as gemv.cu (persistent, stream-K over 128-row weight blocks x 128-wide K chunks,
// deterministic last-arriver fix-up of split blocks, fused epilogue), but the contraction runs as
// tcgen05.mma with the weight tile as A (M = 128 rows) and the activations as B (N = 16/32/64 tokens),
// reading both operands straight from shared memory (the K128 layout is the canonical K-major
// no-swizzle operand layout).  One thread issues all MMAs, so the SM's issue slots stay free and the
// kernel follows the TMA weight stream.  Warp roles: 0 = TMA producer, 1 = MMA issuer (and TMEM
// owner), 2..5 = epilogue (one TMEM lane quadrant each).  The accumulator is double-buffered in TMEM so
// the epilogue of one block overlaps the MMAs of the next.
#include "common.cuh"
#include "epilogue.cuh"

namespace jxb {

constexpr int kTcThreads = 192;
constexpr int kTcBN = 128;
constexpr int kTcBK = 128;

template <int MT>
struct TcCfg {
  static constexpr int N = MT * 16;                       // tokens = MMA N
  static constexpr int kWBytes = kTcBN * kTcBK * 2;        // 32 KB
  static constexpr int kXBytes = N * kTcBK * 2;            // 4 / 8 / 16 KB
  static constexpr int kStageBytes = kWBytes + kXBytes;
  // As many stages as shared memory holds (see gemv.cu).
  static constexpr int kStages = MT == 1 ? 5 : (MT == 2 ? 5 : 4);
  static constexpr int kLd = kTcBN + 4;                    // staging tile [N][128 rows] float32
  static constexpr int kTileBytes = N * kLd * 4;
  static constexpr int kBars = 2 * kStages + 5;
  static constexpr int kSmem = kStages * kStageBytes + kTileBytes + kBars * 8 + 32;
  static constexpr uint32_t kTmemCols = N <= 16 ? 32 : (N <= 32 ? 64 : 128);
};

__device__ __forceinline__ long long tc_it_begin(long long total, int G, int c) { return total * c / G; }
__device__ __forceinline__ int tc_cta_of(long long it, long long total, int G) {
  return (int)(((it + 1) * G + total - 1) / total) - 1;
}

template <int MT>
__global__ void __launch_bounds__(kTcThreads, 1)
    gemv_tc_kernel(const bf16* __restrict__ W, const bf16* __restrict__ X, long long Np, long long Kp, EpiParams e,
                   float* __restrict__ ws, int* __restrict__ counters, int* status) {
  using C = TcCfg<MT>;
  extern __shared__ __align__(1024) uint8_t smem[];
  float* tile = reinterpret_cast<float*>(smem + C::kStages * C::kStageBytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kStages * C::kStageBytes + C::kTileBytes);
  uint64_t* empty = full + C::kStages;
  uint64_t* accf = empty + C::kStages;      // [2] accumulator ready
  uint64_t* acce = accf + 2;                // [2] accumulator drained
  uint64_t* done = acce + 2;                // epilogue finished with TMEM
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* sh = reinterpret_cast<volatile int*>(tmem_slot + 1);   // [0] dead, [1] last-arriver

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_blocks = (int)(Np / kTcBN), kc = (int)(Kp / kTcBK);
  const long long total = (long long)n_blocks * kc;
  const int G = gridDim.x, c = blockIdx.x;
  const long long it0 = tc_it_begin(total, G, c), it1 = tc_it_begin(total, G, c + 1);
  const int n_it = (int)(it1 - it0);
  constexpr long long Np8 = 0;  // (unused) keeps the layout formula below explicit
  (void)Np8;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf[b], 1);
      mbar_init(&acce[b], 4);
    }
    mbar_init(done, 4);
    sh[0] = 0;
    sh[1] = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Dependents are released only by threads past their own wait on the previous kernel (the producer
  // and the epilogue warps; the MMA warp never waits), so a kernel launched behind this one finds
  // every kernel before this one complete.

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0 && n_it > 0) {
      auto wsrc = [&](long long it) {
        const long long nb = it / kc, kk = it - nb * kc;
        return W + ((kk * (Np >> 3) + nb * (kTcBN / 8)) << 10);
      };
      auto xsrc = [&](long long it) { return X + (((it % kc) * (C::N >> 3)) << 10); };
      const int pre = n_it < C::kStages ? n_it : C::kStages;
      const uint64_t pol_w = l2_policy_evict_first();   // weights are read once per step
      for (int i = 0; i < pre; ++i) {
        mbar_arrive_expect_tx(&full[i], C::kStageBytes);
        bulk_g2s_hint(smem + i * C::kStageBytes, wsrc(it0 + i), C::kWBytes, &full[i], pol_w);
      }
      pdl_wait();
      pdl_trigger();
      // normalisation prologue: the activations exist once CTAs 0..M-1 have written them
      if (e.pn_h && !prologue_wait(e, *reinterpret_cast<volatile int*>(e.pn_sync))) set_status(status, JX_ERR_TIMEOUT);
      for (int i = 0; i < pre; ++i)
        bulk_g2s(smem + i * C::kStageBytes + C::kWBytes, xsrc(it0 + i), C::kXBytes, &full[i]);
      int issued = pre;
      for (int i = pre; i < n_it; ++i) {
        const int s = i % C::kStages;
        if (sh[0] || !mbar_wait_bounded(&empty[s], ((i / C::kStages) - 1) & 1)) {
          set_status(status, JX_ERR_TIMEOUT);
          sh[0] = 1;
          break;
        }
        mbar_arrive_expect_tx(&full[s], C::kStageBytes);
        bulk_g2s_hint(smem + s * C::kStageBytes, wsrc(it0 + i), C::kWBytes, &full[s], pol_w);
        bulk_g2s(smem + s * C::kStageBytes + C::kWBytes, xsrc(it0 + i), C::kXBytes, &full[s]);
        issued = i + 1;
      }
      for (int i = (issued > C::kStages ? issued - C::kStages : 0); i < issued; ++i)
        if (!mbar_wait_bounded(&full[i % C::kStages], (i / C::kStages) & 1)) break;
      // Every own load has landed: warm L2 with what this CTA of the next projection reads first, while
      // this CTA's split-K finish and epilogue run.
      if (!sh[0]) prefetch_next_weights(e, c);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0 && n_it > 0) {
      constexpr uint32_t idesc = umma_idesc_bf16_f32(kTcBN, C::N);
      long long cur_nb = -1;
      int blk = -1;
      uint32_t dcol = 0;
      bool first = true;
      for (int i = 0; i < n_it && !sh[0]; ++i) {
        const long long it = it0 + i;
        const long long nb = it / kc, kk = it - nb * kc;
        if (nb != cur_nb) {
          cur_nb = nb;
          ++blk;
          const int buf = blk & 1;
          if (blk >= 2 && !mbar_wait_bounded(&acce[buf], ((blk >> 1) - 1) & 1)) {
            set_status(status, JX_ERR_TIMEOUT);
            sh[0] = 1;
            break;
          }
          tc_fence_after();
          dcol = (uint32_t)(buf * C::N);
          first = true;
        }
        const int s = i % C::kStages;
        if (!mbar_wait_bounded(&full[s], (i / C::kStages) & 1)) {
          set_status(status, JX_ERR_TIMEOUT);
          sh[0] = 1;
          break;
        }
        tc_fence_after();
        const uint32_t sw = smem_u32(smem + s * C::kStageBytes);
        const uint32_t sx = sw + C::kWBytes;
#pragma unroll
        for (int ks = 0; ks < kTcBK / 16; ++ks) {
          const uint64_t ad = umma_desc_kmajor(sw + ks * 256, 128, 2048);
          const uint64_t bd = umma_desc_kmajor(sx + ks * 256, 128, 2048);
          umma_bf16(tmem + dcol, ad, bd, idesc, (first && ks == 0) ? 0u : 1u);
        }
        first = false;
        umma_commit(&empty[s]);
        const bool block_end = (kk == kc - 1) || (i == n_it - 1);
        if (block_end) umma_commit(&accf[blk & 1]);
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5, 128 threads) ----------------
    pdl_wait();
    pdl_trigger();
    const int tid = threadIdx.x - 64;
    __shared__ float pn_red[4];
    const int pn_ep = e.pn_h ? *reinterpret_cast<volatile int*>(e.pn_sync) : 0;
    if (e.pn_h) prologue_rows(e, const_cast<bf16*>(X), C::N, c, pn_ep, tid, 128, 1, pn_red);
    const int quad = warp & 3;                 // TMEM lane quadrant this warp may read
    const int row = quad * 32 + lane;          // weight row within the block
    const long long Mp = C::N;
    long long cur_nb = -1;
    int blk = -1;
    bool started_at_zero = false;
    for (int i = 0; i < n_it; ++i) {
      const long long it = it0 + i;
      const long long nb = it / kc, kk = it - nb * kc;
      if (nb != cur_nb) {
        cur_nb = nb;
        ++blk;
        started_at_zero = (kk == 0);
      }
      const bool block_end = (kk == kc - 1) || (i == n_it - 1);
      if (!block_end) continue;
      const int buf = blk & 1;
      bool ok = !sh[0] && mbar_wait_bounded(&accf[buf], (blk >> 1) & 1);
      if (!ok) {
        set_status(status, JX_ERR_TIMEOUT);
        sh[0] = 1;
      }
      ok = __all_sync(0xffffffffu, ok);   // tcgen05.ld is a warp-wide instruction
      tc_fence_after();
      if (ok) {
#pragma unroll
        for (int c0 = 0; c0 < C::N; c0 += 16) {
          float v[16];
          tmem_ld16(tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(buf * C::N + c0), v);
#pragma unroll
          for (int j = 0; j < 16; ++j) tile[(c0 + j) * C::kLd + row] = v[j];
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acce[buf]);
      named_bar_sync(1, 128);

      const bool whole = started_at_zero && (kk == kc - 1);
      bool do_epi = whole;
      if (!whole) {
        const int c_first = tc_cta_of(nb * kc, total, G), c_last = tc_cta_of(nb * kc + kc - 1, total, G);
        auto slot_of = [&](int cc) {
          const int nbf = (int)(tc_it_begin(total, G, cc) / kc);
          return cc * 2 + (nb == nbf ? 0 : 1);
        };
        // The CTA holding the block's first K chunks reaches the block last (they end its range, while
        // the other contributors' parts start theirs).  When every other contributor has already
        // published, it sums without publishing its own partial: its own values come from the tile.
        bool fast = false;
        if (c == c_first) {
          if (tid == 0) sh[1] = (ld_acquire_gpu(&counters[nb]) == c_last - c_first) ? 1 : 0;
          named_bar_sync(1, 128);
          fast = sh[1] != 0;
          named_bar_sync(1, 128);
        }
        if (fast) {
          do_epi = true;
        } else {
          float* my = ws + (long long)slot_of(c) * Mp * kTcBN;
          for (int idx = tid; idx < Mp * kTcBN; idx += 128) my[idx] = tile[(idx >> 7) * C::kLd + (idx & 127)];
          __threadfence();
          named_bar_sync(1, 128);
          if (tid == 0) {
            const int prev = atomicAdd(&counters[nb], 1);
            sh[1] = (prev == c_last - c_first) ? 1 : 0;
          }
          named_bar_sync(1, 128);
          do_epi = sh[1] != 0;
        }
        if (do_epi) {
          __threadfence();
          // Sum every contribution (this CTA's too) in CTA order.  Each
          // thread owns 4*MT float4 groups of the tile, taken 4 at a time; the loads of up to 4
          // contributors are all issued before any is added, so the L2 round trips overlap.
#pragma unroll
          for (int q0 = 0; q0 < 4 * MT; q0 += 4) {
            float4 acc4[4];
            for (int cc0 = c_first; cc0 <= c_last; cc0 += 4) {
              float4 v[4][4];
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                if (cc0 + u > c_last) break;
                if (fast && cc0 + u == c) {   // this CTA's own partial, still in the tile
#pragma unroll
                  for (int q = 0; q < 4; ++q) {
                    const int e0 = (tid + (q0 + q) * 128) * 4;
                    v[u][q] = *reinterpret_cast<const float4*>(tile + (e0 >> 7) * C::kLd + (e0 & 127));
                  }
                } else {
                  const float4* src = reinterpret_cast<const float4*>(ws + (long long)slot_of(cc0 + u) * Mp * kTcBN);
#pragma unroll
                  for (int q = 0; q < 4; ++q) v[u][q] = __ldcg(src + tid + (q0 + q) * 128);
                }
              }
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                if (cc0 + u > c_last) break;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                  if (cc0 + u == c_first) {
                    acc4[q] = v[u][q];
                  } else {
                    acc4[q].x += v[u][q].x;
                    acc4[q].y += v[u][q].y;
                    acc4[q].z += v[u][q].z;
                    acc4[q].w += v[u][q].w;
                  }
                }
              }
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int e0 = (tid + (q0 + q) * 128) * 4;   // 4 consecutive weight rows of one token
              float* t = tile + (e0 >> 7) * C::kLd + (e0 & 127);
              t[0] = acc4[q].x;
              t[1] = acc4[q].y;
              t[2] = acc4[q].z;
              t[3] = acc4[q].w;
            }
          }
          if (tid == 0) counters[nb] = 0;
          named_bar_sync(1, 128);
        }
      }
      if (do_epi && !sh[0])
        run_epilogue<bf16>(e, 0, (int)Mp, nb * kTcBN, kTcBN, [&](int m, int j) { return tile[m * C::kLd + j]; },
                           tid, 128);
      named_bar_sync(1, 128);
      if (do_epi && !sh[0] && e.kind == JX_EPI_PUSH_F32 && tid == 0) push_signal(e, nb * kTcBN, kTcBN);
    }
    if (e.pn_h) {
      named_bar_sync(1, 128);
      if (tid == 0) prologue_arrive(e, pn_ep);
    }
  }
  // Teardown without a CTA-wide barrier (the roles above leave their warps at different points): the
  // epilogue warps arrive on `done` when their last TMEM read is complete; warp 1 waits for that and
  // frees TMEM.  The producer warp just exits.
  __syncwarp();
  if (warp >= 2) {
    tc_fence_before();
    if (lane == 0) mbar_arrive(done);
  } else if (warp == 1) {
    if (!mbar_wait_bounded(done, 0)) set_status(status, JX_ERR_TIMEOUT);
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

template <int MT>
static int launch_gemv_tc(const bf16* W, const bf16* X, long long Np, long long Kp, const EpiParams& e, float* ws,
                          int* counters, int* status, int grid, bool pdl, cudaStream_t stream) {
  using C = TcCfg<MT>;
  static bool configured = false;
  if (!configured) {
    if (cudaFuncSetAttribute(gemv_tc_kernel<MT>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem) != cudaSuccess)
      return JX_ERR_CUDA;
    configured = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = C::kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return launch_ex(&cfg, gemv_tc_kernel<MT>, W, X, Np, Kp, e, ws, counters, status) == cudaSuccess
             ? JX_OK
             : JX_ERR_CUDA;
}

int run_gemv_tc(const bf16* W, const bf16* X, long long Np, long long Kp, int M, const EpiParams& e, float* ws,
                long long ws_floats, int* counters, int* status, int grid, bool pdl, cudaStream_t stream) {
  if (M <= 0 || M > 64) return JX_ERR_SHAPE;
  if (Np % kTcBN || Kp % kTcBK || Np <= 0 || Kp <= 0) return JX_ERR_SHAPE;
  const int mt = M <= 16 ? 1 : (M <= 32 ? 2 : 4);
  const long long total = (Np / kTcBN) * (Kp / kTcBK);
  if (grid <= 0) grid = 148;
  if (grid > total) grid = (int)total;
  if ((long long)grid * 2 * mt * 16 * kTcBN > ws_floats) return JX_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(W) | reinterpret_cast<uintptr_t>(X)) & 15) return JX_ERR_ARG;
  switch (mt) {
    case 1: return launch_gemv_tc<1>(W, X, Np, Kp, e, ws, counters, status, grid, pdl, stream);
    case 2: return launch_gemv_tc<2>(W, X, Np, Kp, e, ws, counters, status, grid, pdl, stream);
    default: return launch_gemv_tc<4>(W, X, Np, Kp, e, ws, counters, status, grid, pdl, stream);
  }
}

}  // namespace jxb
