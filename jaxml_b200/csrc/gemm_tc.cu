// Prefill projections on the 5th-generation tensor cores (tcgen05 + TMEM):
// Y[M, N] = X[M, K] . W[N, K]^T for M > 64 token rows, bfloat16 operands in the K128 tiled layout,
// float32 accumulation in TMEM, the fused epilogues of epilogue.cuh.
//
// Persistent kernel, one CTA per SM, output tiles of 128 weight rows (MMA M) x 256 tokens (MMA N; a
// 128-token last block uses N = 128), tile t -> (token block t % nM, weight block t / nM).  Warp roles:
// 0 = TMA producer, 1 = MMA issuer (and TMEM owner), 2..5 = epilogue, one TMEM lane quadrant each.
//
// Operand staging: a 64-wide K half of one 128-wide K chunk is, in the K128 layout, the first or second
// 1 KB of every 2 KB unit (8 rows x 128 k).  A 3-D tensor map (64 elements, 16 K-cores, units) moves
// the 16 (A) or 32 (B) unit halves of a stage with one TMA each; shared memory then holds [8-row group]
// [8 K-cores][8 x 8], the canonical K-major no-swizzle operand layout with LBO = 128 B between K-cores
// and SBO = 1 KB between 8-row groups.  Four such stages (48 KB each) are in flight.  The accumulator is
// double-buffered in TMEM (2 x 256 columns), so the epilogue of one tile overlaps the MMAs of the next;
// the epilogue moves 32-token slices through a shared-memory staging tile into run_epilogue.
#include <cudaTypedefs.h>

#include "common.cuh"
#include "epilogue.cuh"

namespace jxb {

constexpr int kGtThreads = 192;
constexpr int kGtBM = 128;                      // weight rows per tile (MMA M)
constexpr int kGtBN = 256;                      // tokens per tile (MMA N)
constexpr int kGtBK = 64;                       // K per stage
constexpr int kGtStages = 4;
constexpr int kGtABytes = kGtBM * kGtBK * 2;    // 16 KB
constexpr int kGtBBytes = kGtBN * kGtBK * 2;    // 32 KB (the full box is always written)
constexpr int kGtStageBytes = kGtABytes + kGtBBytes;
constexpr int kGtSlice = 32;                    // tokens per epilogue slice
constexpr int kGtLd = kGtBM + 4;                // staging tile [32 tokens][128 rows + 4] float32
constexpr int kGtTileBytes = kGtSlice * kGtLd * 4;
constexpr int kGtBars = 2 * kGtStages + 5;
constexpr int kGtSmem = 1024 + kGtStages * kGtStageBytes + kGtTileBytes + kGtBars * 8 + 32;
constexpr uint32_t kGtTmemCols = 512;

struct GtParams {
  long long Mp, Np, Kp;
  int nM, nN, tiles;
  int gm;                // token blocks per tile group (0: token blocks fastest over the whole grid)
  EpiParams e;
  int* status;
};

// Tile t -> (token block mb, weight block nb).  With tile groups, the tiles of gm token blocks x all
// weight blocks come first (token block fastest inside the group), so the activations of a group stay
// in L2 while the weights stream past; otherwise token blocks are fastest over the whole grid.
__device__ __forceinline__ void gt_tile(const GtParams& p, int t, int& mb, int& nb) {
  if (p.gm <= 0 || p.gm >= p.nM) {
    mb = t % p.nM;
    nb = t / p.nM;
    return;
  }
  const int per_group = p.gm * p.nN;
  const int g = t / per_group, r = t - g * per_group;
  const int width = min(p.gm, p.nM - g * p.gm);   // the last group may hold fewer token blocks
  mb = g * p.gm + r % width;
  nb = r / width;
}

__global__ void __launch_bounds__(kGtThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap, GtParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* stile = reinterpret_cast<float*>(smem + kGtStages * kGtStageBytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kGtStages * kGtStageBytes + kGtTileBytes);
  uint64_t* empty = full + kGtStages;
  uint64_t* accf = empty + kGtStages;   // [2] accumulator ready
  uint64_t* acce = accf + 2;            // [2] accumulator drained
  uint64_t* done = acce + 2;            // epilogue finished with TMEM
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* dead = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x;
  const int ksteps = (int)(p.Kp / kGtBK);

  if (threadIdx.x == 0) {
    prefetch_tmap(&wmap);
    prefetch_tmap(&xmap);
    for (int s = 0; s < kGtStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf[b], 1);
      mbar_init(&acce[b], 4);
    }
    mbar_init(done, 4);
    *dead = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kGtTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_trigger();

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      pdl_wait();
      int cnt = 0;
      for (int t = blockIdx.x; t < p.tiles && !*dead; t += G) {
        int mb, nb;
        gt_tile(p, t, mb, nb);
        const int wz = nb * (kGtBM / 8), xz = mb * (kGtBN / 8);
        for (int j = 0; j < ksteps; ++j, ++cnt) {
          const int s = cnt % kGtStages;
          if (cnt >= kGtStages && !mbar_wait_bounded(&empty[s], ((cnt / kGtStages) - 1) & 1)) {
            set_status(p.status, JX_ERR_TIMEOUT);
            *dead = 1;
            break;
          }
          const int kk = j >> 1, kh = (j & 1) * 8;
          mbar_arrive_expect_tx(&full[s], kGtStageBytes);
          tma_load_3d(smem + s * kGtStageBytes, &wmap, 0, kh, kk * (int)(p.Np >> 3) + wz, &full[s]);
          tma_load_3d(smem + s * kGtStageBytes + kGtABytes, &xmap, 0, kh, kk * (int)(p.Mp >> 3) + xz, &full[s]);
        }
      }
      // Drain: every issued copy lands before this CTA's shared memory is released.
      for (int i = (cnt > kGtStages ? cnt - kGtStages : 0); i < cnt; ++i)
        if (!mbar_wait_bounded(&full[i % kGtStages], (i / kGtStages) & 1)) break;
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      int cnt = 0, ti = 0;
      for (int t = blockIdx.x; t < p.tiles && !*dead; t += G, ++ti) {
        int mb, nb;
        gt_tile(p, t, mb, nb);
        (void)nb;
        const bool half = (p.Mp - (long long)mb * kGtBN) < kGtBN;   // 128-token last block
        const uint32_t idesc = half ? umma_idesc_bf16_f32(kGtBM, 128) : umma_idesc_bf16_f32(kGtBM, kGtBN);
        const int buf = ti & 1;
        if (ti >= 2 && !mbar_wait_bounded(&acce[buf], ((ti >> 1) - 1) & 1)) {
          set_status(p.status, JX_ERR_TIMEOUT);
          *dead = 1;
          break;
        }
        tc_fence_after();
        const uint32_t dtm = tmem + (uint32_t)(buf * kGtBN);
        bool ok = true;
        for (int j = 0; j < ksteps; ++j, ++cnt) {
          const int s = cnt % kGtStages;
          if (!mbar_wait_bounded(&full[s], (cnt / kGtStages) & 1)) {
            set_status(p.status, JX_ERR_TIMEOUT);
            *dead = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * kGtStageBytes);
          const uint32_t sb = sa + kGtABytes;
#pragma unroll
          for (int ks = 0; ks < kGtBK / 16; ++ks) {
            const uint64_t ad = umma_desc_kmajor(sa + ks * 256, 128, 1024);
            const uint64_t bd = umma_desc_kmajor(sb + ks * 256, 128, 1024);
            umma_bf16(dtm, ad, bd, idesc, (j > 0 || ks > 0) ? 1u : 0u);
          }
          umma_commit(&empty[s]);
        }
        if (!ok) break;
        umma_commit(&accf[buf]);
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int tid = threadIdx.x - 64;
    const int quad = warp & 3;            // TMEM lane quadrant = weight rows quad*32 .. +31
    const int row = quad * 32 + lane;
    int ti = 0;
    for (int t = blockIdx.x; t < p.tiles; t += G, ++ti) {
      int mb, nb;
        gt_tile(p, t, mb, nb);
      const int buf = ti & 1;
      const int ntok = (p.Mp - (long long)mb * kGtBN) < kGtBN ? 128 : kGtBN;
      bool ok = !*dead && mbar_wait_bounded(&accf[buf], (ti >> 1) & 1);
      if (!ok) {
        set_status(p.status, JX_ERR_TIMEOUT);
        *dead = 1;
      }
      ok = __all_sync(0xffffffffu, ok);   // tcgen05.ld is a warp-wide instruction
      tc_fence_after();
      for (int c0 = 0; c0 < ntok; c0 += kGtSlice) {
        if (ok) {
#pragma unroll
          for (int h = 0; h < kGtSlice; h += 16) {
            float v[16];
            tmem_ld16(tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(buf * kGtBN + c0 + h), v);
#pragma unroll
            for (int q = 0; q < 16; ++q) stile[(h + q) * kGtLd + row] = v[q];
          }
        }
        if (c0 + kGtSlice >= ntok) {
          // last TMEM read of this tile: hand the accumulator buffer back to the MMA warp
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acce[buf]);
        }
        named_bar_sync(1, 128);
        if (ok)
          run_epilogue<bf16>(p.e, (long long)mb * kGtBN + c0, kGtSlice, (long long)nb * kGtBM, kGtBM,
                             [&](int m, int j) { return stile[m * kGtLd + j]; }, tid, 128);
        named_bar_sync(1, 128);
      }
      // no early exit on a failed wait: every epilogue thread keeps the same sequence of named barriers
    }
  }
  // Teardown without a CTA-wide barrier: the epilogue warps arrive on `done` after their last TMEM
  // read; warp 1 waits for that and frees TMEM.  The producer warp just exits.
  __syncwarp();
  if (warp >= 2) {
    tc_fence_before();
    if (lane == 0) mbar_arrive(done);
  } else if (warp == 1) {
    if (!mbar_wait_bounded(done, 0)) set_status(p.status, JX_ERR_TIMEOUT);
    tc_fence_after();
    tmem_dealloc(tmem, kGtTmemCols);
  }
}

// ------------------------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 gt_encoder() {
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

// 3-D view of a K128 operand [Kp/128][Rp/8][16 K-cores][8 x 8]: (64 elements, 16 K-cores, units) with a
// (64, 8, box_rows / 8) box = one 64-wide K half of box_rows rows.
static int make_tmap_k128_half(CUtensorMap* map, const void* base, long long Rp, long long Kp, int box_rows) {
  auto enc = gt_encoder();
  if (!enc) return JX_ERR_CUDA;
  if (reinterpret_cast<uintptr_t>(base) & 15) return JX_ERR_ARG;
  cuuint64_t dims[3] = {64, 16, (cuuint64_t)((Kp / 128) * (Rp / 8))};
  cuuint64_t strides[2] = {128, 2048};
  cuuint32_t box[3] = {64, 8, (cuuint32_t)(box_rows / 8)};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? JX_OK : JX_ERR_ARG;
}

bool gemm_tc_supported(long long Mp, long long Np, long long Kp) {
  return Mp >= 128 && Mp % 128 == 0 && Np % kGtBM == 0 && Kp % 128 == 0 && Np > 0 && Kp > 0 &&
         (Kp / 128) * (Np / 8) < (1LL << 31) && (Kp / 128) * (Mp / 8) < (1LL << 31);
}

static int g_tile_group = 0;
void set_gemm_tile_group(int gm) { g_tile_group = gm; }

int run_gemm_tc(const bf16* X, const bf16* W, long long Mp, long long Np, long long Kp, const EpiParams& e,
                int* status, bool pdl, cudaStream_t stream) {
  if (!gemm_tc_supported(Mp, Np, Kp)) return JX_ERR_SHAPE;
  CUtensorMap wm, xm;
  int rc = make_tmap_k128_half(&wm, W, Np, Kp, kGtBM);
  if (rc == JX_OK) rc = make_tmap_k128_half(&xm, X, Mp, Kp, kGtBN);
  if (rc != JX_OK) return rc;
  static bool configured = false;
  if (!configured) {
    if (cudaFuncSetAttribute(gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kGtSmem) != cudaSuccess)
      return JX_ERR_CUDA;
    configured = true;
  }
  GtParams p;
  p.Mp = Mp;
  p.Np = Np;
  p.Kp = Kp;
  p.nM = (int)((Mp + kGtBN - 1) / kGtBN);
  p.nN = (int)(Np / kGtBM);
  p.tiles = p.nM * p.nN;
  p.gm = g_tile_group;
  p.e = e;
  p.status = status;
  int sms = 148;
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.tiles < sms ? p.tiles : sms);
  cfg.blockDim = dim3(kGtThreads);
  cfg.dynamicSmemBytes = kGtSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return launch_ex(&cfg, gemm_tc_kernel, wm, xm, p) == cudaSuccess ? JX_OK : JX_ERR_CUDA;
}

}  // namespace jxb
