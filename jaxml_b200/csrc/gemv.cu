// Decode projection kernel: Y[M, N] = X[M, K] . W[N, K]^T for M <= 64 (one decode step of B <= 64
// sequences), bfloat16 operands in the K128 tiled layout, float32 accumulation.
//
// At decode batch sizes the projection is a weight stream: every weight byte is read once from HBM
// and used M times.  The kernel is persistent (one CTA per SM) and splits the flat iteration space
// (64-row weight block x 128-wide K chunk) evenly across CTAs ("stream-K"), so every SM streams the
// same number of bytes whatever N and K are.  A producer warp feeds a ring of shared-memory stages
// with 1-D TMA bulk copies (16 KB of weights + the matching activation chunk per stage); eight consumer
// warps (16 rows x half the K steps each) run mma.sync m16n8k16 over the stage.  A weight block that is
// split across CTAs is finished by whichever CTA arrives last: the partial tiles are summed in CTA
// order (deterministic) and the fused epilogue runs once.
#include "common.cuh"
#include "epilogue.cuh"

namespace jxb {

// warp 0: producer; warps 1..8: consumers.  Consumer warp c owns weight rows [(c%4)*16, +16) of each
// 64-row block and the K steps [(c/4)*4, +4) of each 128-wide chunk: two warps per SM sub-partition
// keep enough independent ldmatrix / mma instructions in flight to follow the memory stream.
constexpr int kGemvConsumers = 256;
constexpr int kGemvThreads = 32 + kGemvConsumers;
constexpr int kGemvBN = 64;
constexpr int kGemvBK = 128;
constexpr int kTileLd = 68;         // padded float32 row stride of the staging tile

template <int MT>
struct GemvCfg {
  // 5 stages at M <= 16 (104 KB).  Doubling them (10 stages, 205 KB) made every mma.sync projection of
  // the Llama-8B decode step slower (o_proj 12.3 -> 13.3 us, qkv 15.2 -> 16.4, down 27.2 -> 28.2) and
  // the step 4.35 -> 4.41 ms: a smaller CTA starts beside the tail of the kernel before it.
  static constexpr int kStages = MT == 1 ? 5 : (MT == 2 ? 4 : 3);
  static constexpr int kWBytes = kGemvBN * kGemvBK * 2;   // 16 KB
  static constexpr int kXBytes = MT * 16 * kGemvBK * 2;   // 4 KB per m16 tile
  static constexpr int kStageBytes = kWBytes + kXBytes;
  static constexpr int kTileBytes = MT * 16 * kTileLd * 4;
  static constexpr int kSmem = kStages * kStageBytes + kTileBytes + 2 * kStages * 8 + 16;
};

__device__ __forceinline__ long long it_begin(long long total, int G, int c) { return total * c / G; }
__device__ __forceinline__ int cta_of(long long it, long long total, int G) {
  return (int)(((it + 1) * G + total - 1) / total) - 1;
}

template <int MT>
__global__ void __launch_bounds__(kGemvThreads, 1)
    gemv_k128_kernel(const bf16* __restrict__ W, const bf16* __restrict__ X, long long Np, long long Kp,
                     EpiParams e, float* __restrict__ ws, int* __restrict__ counters, int* status) {
  using C = GemvCfg<MT>;
  extern __shared__ __align__(128) uint8_t smem[];
  float* tile = reinterpret_cast<float*>(smem + C::kStages * C::kStageBytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kStages * C::kStageBytes + C::kTileBytes);
  uint64_t* empty = full + C::kStages;
  volatile int* sh = reinterpret_cast<volatile int*>(empty + C::kStages);  // [0]: dead flag, [1]: last-arriver flag

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_blocks = (int)(Np / kGemvBN), kc = (int)(Kp / kGemvBK);
  const long long total = (long long)n_blocks * kc;
  const int G = gridDim.x, c = blockIdx.x;
  const long long it0 = it_begin(total, G, c), it1 = it_begin(total, G, c + 1);
  const int n_it = (int)(it1 - it0);
  const long long Mp = MT * 16;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kGemvConsumers / 32);
    }
    sh[0] = 0;
    sh[1] = 0;
    fence_barrier_init();
  }
  __syncthreads();

  // Dependents are released only by threads past their own wait on the previous kernel, so a kernel
  // launched behind this one finds every kernel before this one complete.
  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0 && n_it > 0) {
      const int pre = n_it < C::kStages ? n_it : C::kStages;
      auto wsrc = [&](long long it) {
        const long long nb = it / kc, kk = it - nb * kc;
        return W + ((kk * (Np >> 3) + nb * 8) << 10);
      };
      auto xsrc = [&](long long it) {
        const long long kk = it % kc;
        return X + ((kk * (Mp >> 3)) << 10);
      };
      const uint64_t pol_w = l2_policy_evict_first();   // weights are read once per step
      // Weights do not depend on the previous kernel: start streaming them before waiting on it.
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
        const uint32_t round = i / C::kStages;
        if (!mbar_wait_bounded(&empty[s], (round - 1) & 1)) {
          set_status(status, JX_ERR_TIMEOUT);
          sh[0] = 1;
          break;
        }
        mbar_arrive_expect_tx(&full[s], C::kStageBytes);
        bulk_g2s_hint(smem + s * C::kStageBytes, wsrc(it0 + i), C::kWBytes, &full[s], pol_w);
        bulk_g2s(smem + s * C::kStageBytes + C::kWBytes, xsrc(it0 + i), C::kXBytes, &full[s]);
        issued = i + 1;
      }
      // Drain: every issued copy must land before this CTA's shared memory is released.
      for (int i = (issued > C::kStages ? issued - C::kStages : 0); i < issued; ++i) {
        const int s = i % C::kStages;
        if (!mbar_wait_bounded(&full[s], (i / C::kStages) & 1)) {
          set_status(status, JX_ERR_TIMEOUT);
          break;
        }
      }
      // Every own load has landed: warm L2 with what this CTA of the next projection reads first, while
      // this CTA's split-K finish and epilogue run.
      if (!sh[0]) prefetch_next_weights(e, c);
    }
    return;
  }

  // ---------------- consumers ----------------
  pdl_wait();
  pdl_trigger();
  const int cw = (warp - 1) & 3;       // owns weight rows [cw*16, cw*16+16) of each 64-row block
  const int khalf = (warp - 1) >> 2;   // and K steps [khalf*4, khalf*4+4) of each chunk
  const int tid = threadIdx.x - 32;    // 0..255
  __shared__ float pn_red[kGemvConsumers / 32];
  const int pn_ep = e.pn_h ? *reinterpret_cast<volatile int*>(e.pn_sync) : 0;
  if (e.pn_h) prologue_rows(e, const_cast<bf16*>(X), Mp, c, pn_ep, tid, kGemvConsumers, 1, pn_red);
  float acc[MT][2][4];
  bool dead = false;

  long long cur_nb = -1;
  bool started_at_zero = false;

  for (int i = 0; i < n_it; ++i) {
    const long long it = it0 + i;
    const long long nb = it / kc, kk = it - nb * kc;
    if (nb != cur_nb) {
      cur_nb = nb;
      started_at_zero = (kk == 0);
#pragma unroll
      for (int a = 0; a < MT; ++a)
#pragma unroll
        for (int b = 0; b < 2; ++b)
#pragma unroll
          for (int q = 0; q < 4; ++q) acc[a][b][q] = 0.f;
    }
    const int s = i % C::kStages;
    if (!dead) {
      if (sh[0] || !mbar_wait_bounded(&full[s], (i / C::kStages) & 1)) {
        dead = true;
        sh[0] = 1;
        set_status(status, JX_ERR_TIMEOUT);
      }
    }
    if (!dead) {
      const uint32_t sW = smem_u32(smem + s * C::kStageBytes);
      const uint32_t sX = sW + C::kWBytes;
      const int mi = lane >> 3, r8 = lane & 7;
#pragma unroll
      for (int kq = 0; kq < 4; ++kq) {
        const int ks = khalf * 4 + kq;
        uint32_t b0, b1, b2, b3;
        {
          const int rg = cw * 2 + (mi >> 1), kcore = ks * 2 + (mi & 1);
          ldsm_x4(sW + (uint32_t)((rg * 1024 + kcore * 64 + r8 * 8) * 2), b0, b1, b2, b3);
        }
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          uint32_t a0, a1, a2, a3;
          const int rg = mt * 2 + (mi & 1), kcore = ks * 2 + (mi >> 1);
          ldsm_x4(sX + (uint32_t)((rg * 1024 + kcore * 64 + r8 * 8) * 2), a0, a1, a2, a3);
          mma_bf16(acc[mt][0], a0, a1, a2, a3, b0, b1);
          mma_bf16(acc[mt][1], a0, a1, a2, a3, b2, b3);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }

    const bool block_end = (kk == kc - 1) || (i == n_it - 1);
    if (!block_end) continue;

    // ---- this CTA's share of weight block nb is done: stage the tile in shared memory ----
    // (the K-half 0 warps store, then the K-half 1 warps add: a fixed summation order)
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      if (khalf == half) {
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
          for (int nt = 0; nt < 2; ++nt) {
            const int r = mt * 16 + (lane >> 2);
            const int col = cw * 16 + nt * 8 + (lane & 3) * 2;
            float* t0 = tile + r * kTileLd + col;
            float* t1 = tile + (r + 8) * kTileLd + col;
            if (half == 0) {
              t0[0] = acc[mt][nt][0];
              t0[1] = acc[mt][nt][1];
              t1[0] = acc[mt][nt][2];
              t1[1] = acc[mt][nt][3];
            } else {
              t0[0] += acc[mt][nt][0];
              t0[1] += acc[mt][nt][1];
              t1[0] += acc[mt][nt][2];
              t1[1] += acc[mt][nt][3];
            }
          }
      }
      named_bar_sync(1, kGemvConsumers);
    }

    const bool whole = started_at_zero && (kk == kc - 1);
    bool do_epi = whole;
    if (!whole) {
      const long long blk_first_it = nb * kc, blk_last_it = nb * kc + kc - 1;
      const int c_first = cta_of(blk_first_it, total, G), c_last = cta_of(blk_last_it, total, G);
      auto slot_of = [&](int cc) {
        const int nbf = (int)(it_begin(total, G, cc) / kc);
        return cc * 2 + (nb == nbf ? 0 : 1);
      };
      // The CTA holding the block's first K chunks reaches the block last (they end its range, while the
      // other contributors' parts start theirs).  When every other contributor has already published, it
      // sums without publishing its own partial: its own values come from the tile.
      bool fast = false;
      if (c == c_first) {
        if (tid == 0) sh[1] = (ld_acquire_gpu(&counters[nb]) == c_last - c_first) ? 1 : 0;
        named_bar_sync(1, kGemvConsumers);
        fast = sh[1] != 0;
        named_bar_sync(1, kGemvConsumers);
      }
      if (fast) {
        do_epi = true;
      } else {
        float* my = ws + (long long)slot_of(c) * Mp * kGemvBN;
        for (int idx = tid; idx < Mp * kGemvBN; idx += kGemvConsumers) my[idx] = tile[(idx >> 6) * kTileLd + (idx & 63)];
        __threadfence();
        named_bar_sync(1, kGemvConsumers);
        if (tid == 0) {
          const int prev = atomicAdd(&counters[nb], 1);
          sh[1] = (prev == c_last - c_first) ? 1 : 0;
        }
        named_bar_sync(1, kGemvConsumers);
        do_epi = sh[1] != 0;
      }
      if (do_epi) {
        __threadfence();
        // Sum every contribution (this CTA's too) in CTA order.  Each thread
        // owns MT float4 groups of the tile; the loads of up to 4 contributors are all issued before
        // any is added, so the L2 round trips overlap instead of following one another.
        float4 acc4[MT];
        for (int cc0 = c_first; cc0 <= c_last; cc0 += 4) {
          float4 v[4][MT];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            if (cc0 + u > c_last) break;
            if (fast && cc0 + u == c) {   // this CTA's own partial, still in the tile
#pragma unroll
              for (int q = 0; q < MT; ++q) {
                const int e0 = (tid + q * kGemvConsumers) * 4;
                v[u][q] = *reinterpret_cast<const float4*>(tile + (e0 >> 6) * kTileLd + (e0 & 63));
              }
            } else {
              const float4* src = reinterpret_cast<const float4*>(ws + (long long)slot_of(cc0 + u) * Mp * kGemvBN);
#pragma unroll
              for (int q = 0; q < MT; ++q) v[u][q] = __ldcg(src + tid + q * kGemvConsumers);
            }
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            if (cc0 + u > c_last) break;
#pragma unroll
            for (int q = 0; q < MT; ++q) {
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
        for (int q = 0; q < MT; ++q) {
          const int e0 = (tid + q * kGemvConsumers) * 4;           // 4 consecutive columns of one row
          float* t = tile + (e0 >> 6) * kTileLd + (e0 & 63);
          t[0] = acc4[q].x;
          t[1] = acc4[q].y;
          t[2] = acc4[q].z;
          t[3] = acc4[q].w;
        }
        if (tid == 0) counters[nb] = 0;
        named_bar_sync(1, kGemvConsumers);
      }
    }
    if (do_epi && !dead) {
      run_epilogue<bf16>(e, 0, (int)Mp, nb * kGemvBN, kGemvBN,
                         [&](int m, int j) { return tile[m * kTileLd + j]; }, tid, kGemvConsumers);
    }
    named_bar_sync(1, kGemvConsumers);
    if (do_epi && !dead && e.kind == JX_EPI_PUSH_F32 && tid == 0) push_signal(e, nb * kGemvBN, kGemvBN);
  }
  if (e.pn_h) {
    named_bar_sync(1, kGemvConsumers);
    if (tid == 0) prologue_arrive(e, pn_ep);
  }
}

template <int MT>
static int launch_gemv(const bf16* W, const bf16* X, long long Np, long long Kp, const EpiParams& e, float* ws,
                       int* counters, int* status, int grid, bool pdl, cudaStream_t stream) {
  using C = GemvCfg<MT>;
  static bool configured = false;
  if (!configured) {
    if (cudaFuncSetAttribute(gemv_k128_kernel<MT>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem) !=
        cudaSuccess)
      return JX_ERR_CUDA;
    configured = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kGemvThreads);
  cfg.dynamicSmemBytes = C::kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t err = launch_ex(&cfg, gemv_k128_kernel<MT>, W, X, Np, Kp, e, ws, counters, status);
  return err == cudaSuccess ? JX_OK : JX_ERR_CUDA;
}

// Split-K partial tiles: two slots per CTA of (16 * mt) rows x 128 columns (the larger of the two
// kernels' weight blocks).
int gemv_workspace_floats(int grid, int mt) { return grid * 2 * mt * 16 * 128; }

int run_gemv_tc(const bf16* W, const bf16* X, long long Np, long long Kp, int M, const EpiParams& e, float* ws,
                long long ws_floats, int* counters, int* status, int grid, bool pdl, cudaStream_t stream);

int gemv_rows_groups(long long Np, int sms);
int run_gemv_rows(const bf16* W, const bf16* X, long long Np, long long Kp, int M, const EpiParams& e, int* status,
                  int sms, bool pdl, cudaStream_t stream);

// 0: by shape (default), 1: mma.sync kernel, 2: tcgen05 kernel, 3: row-split kernel (gemv_rows.cu).
// By shape: the tcgen05 kernel streams the large projections fastest (one thread issues every MMA),
// but its 128-row blocks leave too few blocks per SM on the small ones, where the split-block
// fix-up dominates; it is used once there are at least as many 128-row blocks as SMs.
static int g_gemv_impl = 0;
void set_gemv_impl(int impl) { g_gemv_impl = impl; }
// "By shape" picks the row-split kernel for the shapes it takes (Llama-3-8B decode, batch 16: qkv 15.3 ->
// 9.8 us, o_proj 12.5 -> 8.8 us, down 27.3 -> 23.8 us against the stream-K mma.sync kernel).
static bool g_rows_by_shape = true;

static bool gemv_uses_tc(long long Np, int grid) {
  return Np % 128 == 0 && (g_gemv_impl == 2 || (g_gemv_impl == 0 && Np / 128 >= (grid > 0 ? grid : 148)));
}

int run_gemv(const bf16* W, const bf16* X, long long Np, long long Kp, int M, const EpiParams& e_in, float* ws,
             long long ws_floats, int* counters, int* status, int grid, bool pdl, cudaStream_t stream) {
  // L2 prefetch plan of the next decode projection (jx_epilogue.pf_w): the kernel and grid that call
  // will get by the same rules, or no prefetch when its sizes or alignment are not a decode projection's.
  EpiParams e = e_in;
  if (e.pn_h) {
    // normalisation prologue: one CTA per token row, rows of whole 16-byte vectors
    // (CTAs 0..M-1 must exist: the grid the chosen kernel gets is at least M)
    const long long tot = gemv_uses_tc(Np, grid) ? (Np / 128) * (Kp / 128) : (Np / kGemvBN) * (Kp / kGemvBK);
    const long long g = grid > 0 ? grid : 148;
    if (M > 16 || !e.pn_w || !e.pn_sync || e.pn_d <= 0 || e.pn_d % 8 || e.pn_d > Kp || (e.pn_ldh & 7) ||
        e.pn_ldh < e.pn_d || (e.pn_kind != JX_NORM_RMS && e.pn_kind != JX_NORM_GEMMA && e.pn_kind != JX_NORM_LAYER) ||
        ((reinterpret_cast<uintptr_t>(e.pn_h) | reinterpret_cast<uintptr_t>(e.pn_w) |
          reinterpret_cast<uintptr_t>(e.pn_b) | reinterpret_cast<uintptr_t>(X)) & 15) ||
        (reinterpret_cast<uintptr_t>(e.pn_sync) & 3) || (g < tot ? g : tot) < M)
      return JX_ERR_ARG;
  }
  if (e.kind == JX_EPI_PUSH_F32) {
    // every rank's receive slot and flags sit at the same offsets of its region; units of 64 columns
    if (!e.peer_bases || e.peer_world < 1 || e.peer_world > 8 || e.peer_rank < 0 || e.peer_rank >= e.peer_world ||
        e.N <= 0 || e.N % 64 || e.N > Np || Np / 64 > kPushMaxUnits || (e.ldo & 3) || e.ldo < e.N ||
        (e.peer_recv_off & 15) || (e.peer_slot_bytes & 15) || (long long)e.M * e.ldo * 4 > e.peer_slot_bytes ||
        (e.peer_flag_off & 3) || (e.peer_seq_off & 7) ||
        (reinterpret_cast<uintptr_t>(e.peer_bases) & 7))
      return JX_ERR_ARG;
  }
  e.pf_rows = 0;
  e.pf_grid = 0;
  if (e.pf_w && e.pf_iters > 0 && e.pf_np > 0 && e.pf_kp > 0) {
    const int rows = gemv_uses_tc(e.pf_np, grid) ? 128 : 64;
    const long long tot = (e.pf_np / rows) * (e.pf_kp / 128);
    const int g = grid > 0 ? grid : 148;
    if (e.pf_np % rows == 0 && e.pf_kp % 128 == 0 && !(reinterpret_cast<uintptr_t>(e.pf_w) & 15)) {
      e.pf_rows = rows;
      e.pf_grid = (int)(tot < g ? tot : g);
    } else {
      e.pf_w = nullptr;
    }
  } else {
    e.pf_w = nullptr;
  }
  // Row-split kernel: M <= 16, element-wise epilogues (not the 64-row GLU / push units), no prologue or
  // prefetch, and a grid of at most one CTA per SM.  The float32 partial sums of a row-parallel
  // projection (tensor parallelism) stay on the stream-K kernel, which the push epilogue needs, so the
  // pull and the push exchange sum the same partials (bit-identical results).
  const bool rows_ok = M <= 16 && e.kind != JX_EPI_GLU_SILU && e.kind != JX_EPI_GLU_GELU_TANH &&
                       e.kind != JX_EPI_PUSH_F32 && e.kind != JX_EPI_STORE_F32 && e.kind != JX_EPI_ACC_F32 &&
                       !e.pn_h && !e.pf_w && gemv_rows_groups(Np, grid > 0 ? grid : 148) > 0;
  if (e.tn_x) {
    // the normalisation tail runs in the row-split kernel only
    const bool rows_taken = rows_ok && (g_gemv_impl == 3 || (g_gemv_impl == 0 && g_rows_by_shape && !gemv_uses_tc(Np, grid)));
    if (!rows_taken) return JX_ERR_UNSUPPORTED;
    if ((e.kind != JX_EPI_STORE && e.kind != JX_EPI_RESID) || e.out_rp > 0 || e.N % 256 || e.N > 8192 || e.ldo % 8 ||
        !e.tn_w || !e.tn_sync || e.tn_rp < M || e.tn_rp % 8 ||
        (e.tn_kind != JX_NORM_RMS && e.tn_kind != JX_NORM_GEMMA && e.tn_kind != JX_NORM_LAYER) ||
        ((reinterpret_cast<uintptr_t>(e.out) | reinterpret_cast<uintptr_t>(e.tn_x) |
          reinterpret_cast<uintptr_t>(e.tn_w) | reinterpret_cast<uintptr_t>(e.tn_b)) & 15))
      return JX_ERR_ARG;
  }
  if (g_gemv_impl == 3) {
    if (!rows_ok) return JX_ERR_SHAPE;
    return run_gemv_rows(W, X, Np, Kp, M, e, status, grid > 0 ? grid : 148, pdl, stream);
  }
  // By shape, more than 16 token rows over a long K also take the tcgen05 kernel: at M = 64 the down
  // projection (4096 x 14336) took 37.8 us against 45.2 us on mma.sync, while o_proj (K = 4096) took
  // 25.4 against 19.4 us and qkv 24.6 against 24.2 us.
  const bool tc_by_k = g_gemv_impl == 0 && M > 16 && Kp >= 8192 && Np % 128 == 0 && !e.pn_h;
  if (gemv_uses_tc(Np, grid) || tc_by_k)
    return run_gemv_tc(W, X, Np, Kp, M, e, ws, ws_floats, counters, status, grid, pdl, stream);
  if (g_gemv_impl == 0 && g_rows_by_shape && rows_ok)
    return run_gemv_rows(W, X, Np, Kp, M, e, status, grid > 0 ? grid : 148, pdl, stream);
  if (M <= 0 || M > 64) return JX_ERR_SHAPE;
  if (Np % kGemvBN || Kp % kGemvBK || Np <= 0 || Kp <= 0) return JX_ERR_SHAPE;
  const int mt = M <= 16 ? 1 : (M <= 32 ? 2 : 4);
  const long long total = (Np / kGemvBN) * (Kp / kGemvBK);
  if (grid <= 0) grid = 148;
  if (grid > total) grid = (int)total;
  if ((long long)gemv_workspace_floats(grid, mt) > ws_floats) return JX_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(W) | reinterpret_cast<uintptr_t>(X)) & 15) return JX_ERR_ARG;
  switch (mt) {
    case 1: return launch_gemv<1>(W, X, Np, Kp, e, ws, counters, status, grid, pdl, stream);
    case 2: return launch_gemv<2>(W, X, Np, Kp, e, ws, counters, status, grid, pdl, stream);
    default: return launch_gemv<4>(W, X, Np, Kp, e, ws, counters, status, grid, pdl, stream);
  }
}

}  // namespace jxb
