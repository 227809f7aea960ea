// Prefill projections (M > 64 token rows): Y[M, N] = X[M, K] . W[N, K]^T with the fused epilogues.
//
// bfloat16: the tcgen05 kernel (gemm_tc.cu) runs every shape it supports; this mma.sync kernel is the
// fallback and the comparison path.  Both operands in the K128 tiled layout, so a 128 x 128 operand tile of one K chunk is a
// single contiguous 32 KB run that one TMA bulk copy moves into shared memory.  A producer warp keeps
// three stages in flight; eight consumer warps (2 x 4, 64 x 32 each) run mma.sync m16n8k16 with
// conflict-free ldmatrix reads of the 8x8 core matrices.
//
// float32 (GPT-NeoX parity path): plain row-major X and the reference's [K, N] kernel layout, shared
// memory tiled CUDA-core FMA (true float32, no TF32).
#include "common.cuh"
#include "epilogue.cuh"

namespace jxb {

// ------------------------------------------------------------------------------------------------
// bfloat16 tensor-core GEMM on K128 operands
// ------------------------------------------------------------------------------------------------
constexpr int kGemmBM = 128, kGemmBN = 128, kGemmBK = 128;
constexpr int kGemmStages = 3;
constexpr int kGemmThreads = 288;   // warp 0 producer + 8 consumer warps
constexpr int kGemmTileBytes = kGemmBM * kGemmBK * 2;   // 32 KB (same for B)
constexpr int kGemmStageBytes = 2 * kGemmTileBytes;
constexpr int kGemmCLd = kGemmBN + 4;
constexpr int kGemmSmem = kGemmStages * kGemmStageBytes + 2 * kGemmStages * 8 + 16;

__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_k128_kernel(const bf16* __restrict__ X, const bf16* __restrict__ W, long long Mp, long long Np, long long Kp,
                     EpiParams e, int* status) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kGemmStages * kGemmStageBytes);
  uint64_t* empty = full + kGemmStages;
  volatile int* dead_flag = reinterpret_cast<volatile int*>(empty + kGemmStages);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long m0 = (long long)blockIdx.y * kGemmBM, n0 = (long long)blockIdx.x * kGemmBN;
  const int kc = (int)(Kp / kGemmBK);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kGemmStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 8);
    }
    *dead_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  pdl_trigger();

  if (warp == 0) {
    if (lane == 0) {
      auto asrc = [&](int kk) { return X + (((long long)kk * (Mp >> 3) + (m0 >> 3)) << 10); };
      auto bsrc = [&](int kk) { return W + (((long long)kk * (Np >> 3) + (n0 >> 3)) << 10); };
      const int pre = kc < kGemmStages ? kc : kGemmStages;
      for (int i = 0; i < pre; ++i) {
        mbar_arrive_expect_tx(&full[i], kGemmStageBytes);
        bulk_g2s(smem + i * kGemmStageBytes + kGemmTileBytes, bsrc(i), kGemmTileBytes, &full[i]);
      }
      pdl_wait();
      for (int i = 0; i < pre; ++i) bulk_g2s(smem + i * kGemmStageBytes, asrc(i), kGemmTileBytes, &full[i]);
      int issued = pre;
      for (int i = pre; i < kc; ++i) {
        const int s = i % kGemmStages;
        if (!mbar_wait_bounded(&empty[s], ((i / kGemmStages) - 1) & 1)) {
          set_status(status, JX_ERR_TIMEOUT);
          *dead_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&full[s], kGemmStageBytes);
        bulk_g2s(smem + s * kGemmStageBytes, asrc(i), kGemmTileBytes, &full[s]);
        bulk_g2s(smem + s * kGemmStageBytes + kGemmTileBytes, bsrc(i), kGemmTileBytes, &full[s]);
        issued = i + 1;
      }
      for (int i = (issued > kGemmStages ? issued - kGemmStages : 0); i < issued; ++i) {
        if (!mbar_wait_bounded(&full[i % kGemmStages], (i / kGemmStages) & 1)) {
          set_status(status, JX_ERR_TIMEOUT);
          break;
        }
      }
    }
    return;
  }

  pdl_wait();
  const int cw = warp - 1;
  const int wm = cw >> 2, wn = cw & 3;   // warp tile: rows wm*64.., cols wn*32..
  float acc[4][4][4];
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b)
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[a][b][q] = 0.f;
  bool dead = false;
  const int mi = lane >> 3, r8 = lane & 7;
  for (int i = 0; i < kc; ++i) {
    const int s = i % kGemmStages;
    if (!dead && (*dead_flag || !mbar_wait_bounded(&full[s], (i / kGemmStages) & 1))) {
      dead = true;
      *dead_flag = 1;
      set_status(status, JX_ERR_TIMEOUT);
    }
    if (dead) continue;
    const uint32_t sA = smem_u32(smem + s * kGemmStageBytes);
    const uint32_t sB = sA + kGemmTileBytes;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      uint32_t bfr[4][2];
#pragma unroll
      for (int nb = 0; nb < 2; ++nb) {
        const int rg = (wn * 32 + nb * 16) / 8 + (mi >> 1), kcore = ks * 2 + (mi & 1);
        uint32_t r0, r1, r2, r3;
        ldsm_x4(sB + (uint32_t)((rg * 1024 + kcore * 64 + r8 * 8) * 2), r0, r1, r2, r3);
        bfr[nb * 2][0] = r0;
        bfr[nb * 2][1] = r1;
        bfr[nb * 2 + 1][0] = r2;
        bfr[nb * 2 + 1][1] = r3;
      }
#pragma unroll
      for (int mt = 0; mt < 4; ++mt) {
        uint32_t a0, a1, a2, a3;
        const int rg = (wm * 64 + mt * 16) / 8 + (mi & 1), kcore = ks * 2 + (mi >> 1);
        ldsm_x4(sA + (uint32_t)((rg * 1024 + kcore * 64 + r8 * 8) * 2), a0, a1, a2, a3);
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) mma_bf16(acc[mt][nt], a0, a1, a2, a3, bfr[nt][0], bfr[nt][1]);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
  // All consumer warps are past the last stage: reuse the stage memory as the float32 output tile.
  named_bar_sync(1, 256);
  float* ct = reinterpret_cast<float*>(smem);
#pragma unroll
  for (int mt = 0; mt < 4; ++mt)
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      const int r = wm * 64 + mt * 16 + (lane >> 2);
      const int c = wn * 32 + nt * 8 + (lane & 3) * 2;
      ct[r * kGemmCLd + c] = acc[mt][nt][0];
      ct[r * kGemmCLd + c + 1] = acc[mt][nt][1];
      ct[(r + 8) * kGemmCLd + c] = acc[mt][nt][2];
      ct[(r + 8) * kGemmCLd + c + 1] = acc[mt][nt][3];
    }
  named_bar_sync(1, 256);
  if (!dead)
    run_epilogue<bf16>(e, m0, kGemmBM, n0, kGemmBN, [&](int m, int j) { return ct[m * kGemmCLd + j]; },
                       threadIdx.x - 32, 256);
}

bool gemm_tc_supported(long long Mp, long long Np, long long Kp);
int run_gemm_tc(const bf16* X, const bf16* W, long long Mp, long long Np, long long Kp, const EpiParams& e,
                int* status, bool pdl, cudaStream_t stream);

// 0: by shape (the tcgen05 kernel whenever it supports the shape), 1: mma.sync kernel, 2: tcgen05 kernel.
static int g_gemm_impl = 0;
void set_gemm_impl(int impl) { g_gemm_impl = impl; }

int run_gemm_k128(const bf16* X, const bf16* W, long long Mp, long long Np, long long Kp, const EpiParams& e,
                  int* status, bool pdl, cudaStream_t stream) {
  if (g_gemm_impl != 1 && gemm_tc_supported(Mp, Np, Kp)) return run_gemm_tc(X, W, Mp, Np, Kp, e, status, pdl, stream);
  if (g_gemm_impl == 2) return JX_ERR_SHAPE;
  if (Mp % kGemmBM || Np % kGemmBN || Kp % kGemmBK || Mp <= 0 || Np <= 0 || Kp <= 0) return JX_ERR_SHAPE;
  if ((Np / kGemmBN) > 65535 * 1024LL || (Mp / kGemmBM) > 65535) return JX_ERR_SHAPE;
  static bool configured = false;
  if (!configured) {
    if (cudaFuncSetAttribute(gemm_k128_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemmSmem) != cudaSuccess)
      return JX_ERR_CUDA;
    configured = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(Np / kGemmBN), (unsigned)(Mp / kGemmBM));
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = kGemmSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return launch_ex(&cfg, gemm_k128_kernel, X, W, Mp, Np, Kp, e, status) == cudaSuccess ? JX_OK
                                                                                              : JX_ERR_CUDA;
}

// ------------------------------------------------------------------------------------------------
// float32 GEMM: X [M, K] (row stride ldx) times W [K, N] (row stride N), CUDA-core FMA
// ------------------------------------------------------------------------------------------------
constexpr int kF32BM = 32, kF32BN = 128, kF32BK = 32;

__global__ void __launch_bounds__(256) gemm_f32_kernel(const float* __restrict__ X, long long ldx,
                                                       const float* __restrict__ W, int M, int N, int K,
                                                       EpiParams e) {
  __shared__ float xs[kF32BK][kF32BM + 1];
  __shared__ float ws[kF32BK][kF32BN];
  __shared__ float ct[kF32BM][kF32BN + 1];
  const int tid = threadIdx.x;
  const int tr = tid / 32, tc = tid % 32;  // 8 x 32 threads: 4 rows x 4 cols each
  const long long m0 = (long long)blockIdx.y * kF32BM, n0 = (long long)blockIdx.x * kF32BN;
  pdl_trigger();
  pdl_wait();
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += kF32BK) {
    for (int i = tid; i < kF32BM * kF32BK; i += 256) {
      const int r = i / kF32BK, kk = i % kF32BK;
      const long long m = m0 + r, k = k0 + kk;
      xs[kk][r] = (m < M && k < K) ? X[m * ldx + k] : 0.f;
    }
    for (int i = tid; i < kF32BK * kF32BN; i += 256) {
      const int kk = i / kF32BN, c = i % kF32BN;
      const long long k = k0 + kk, n = n0 + c;
      ws[kk][c] = (k < K && n < N) ? W[k * N + n] : 0.f;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < kF32BK; ++kk) {
      float xv[4], wv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) xv[i] = xs[kk][tr * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) wv[j] = ws[kk][tc + 32 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(xv[i], wv[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) ct[tr * 4 + i][tc + 32 * j] = acc[i][j];
  __syncthreads();
  run_epilogue<float>(e, m0, kF32BM, n0, kF32BN, [&](int m, int j) { return ct[m][j]; }, tid, 256);
}

// float32 projection for up to 64 token rows (decode steps, short prompts).  The tiled kernel above gives a decode-sized M only N / 128
// CTAs, each streaming its whole K x 128 panel with synchronous loads.  Here a CTA owns NC output columns
// (lane = column, so each W row segment is one coalesced 128-byte load per 32 columns; NC = 64 keeps a
// GLU epilogue's 32 gate + 32 up columns together) and a K slice; the CS CTAs of one column tile form a
// thread-block cluster over K.  Sums are deterministic: each warp sums its K range in order, the 8 warps
// are added in warp order, then rank 0 adds the cluster's CTAs in rank order through distributed shared
// memory and runs the epilogue.  Rows come in blocks of 16 (grid y), each block reading W again (from
// L2 at these sizes).  Plain float32 FMA, no TF32.
constexpr int kF32vWarps = 8;

template <int NC>
__global__ void __launch_bounds__(kF32vWarps * 32) gemv_f32_kernel(const float* __restrict__ X, long long ldx,
                                                                   const float* __restrict__ W, int M, int N, int K,
                                                                   EpiParams e) {
  constexpr int CPL = NC / 32;   // columns per lane
  __shared__ float red[kF32vWarps][16][NC + 1];
  __shared__ float fin[16][NC + 1];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int CS = (int)cluster_nctarank(), rank = (int)cluster_ctarank();
  const long long n0 = (long long)(blockIdx.x / CS) * NC;
  const int m0 = blockIdx.y * 16;
  X += (long long)m0 * ldx;
  M = M - m0 < 16 ? M - m0 : 16;
  const int q = rank * kF32vWarps + warp, nq = CS * kF32vWarps;
  const int k0 = (int)((long long)K * q / nq), k1 = (int)((long long)K * (q + 1) / nq);
  bool col_ok[CPL];
#pragma unroll
  for (int c = 0; c < CPL; ++c) col_ok[c] = n0 + c * 32 + lane < N;
  // the weights do not depend on the previous kernel: pull this warp's rows towards L2 before waiting on it
  for (int k = k0 + lane; k < k1; k += 32) prefetch_l2(W + (long long)k * N + n0);
  pdl_trigger();
  pdl_wait();
  float acc[16][CPL];
#pragma unroll
  for (int m = 0; m < 16; ++m)
#pragma unroll
    for (int c = 0; c < CPL; ++c) acc[m][c] = 0.f;
#pragma unroll 8
  for (int k = k0; k < k1; ++k) {
    float wv[CPL];
#pragma unroll
    for (int c = 0; c < CPL; ++c) wv[c] = col_ok[c] ? __ldg(W + (long long)k * N + n0 + c * 32 + lane) : 0.f;
#pragma unroll
    for (int m = 0; m < 16; ++m)
      if (m < M) {
        const float xv = __ldg(X + m * ldx + k);
#pragma unroll
        for (int c = 0; c < CPL; ++c) acc[m][c] = fmaf(xv, wv[c], acc[m][c]);
      }
  }
#pragma unroll
  for (int m = 0; m < 16; ++m)
    if (m < M)
#pragma unroll
      for (int c = 0; c < CPL; ++c) red[warp][m][c * 32 + lane] = acc[m][c];
  __syncthreads();
  for (int idx = threadIdx.x; idx < M * NC; idx += kF32vWarps * 32) {
    const int m = idx / NC, j = idx - m * NC;
    float v = red[0][m][j];
#pragma unroll
    for (int w = 1; w < kF32vWarps; ++w) v += red[w][m][j];
    if (CS == 1)
      fin[m][j] = v;
    else
      red[0][m][j] = v;
  }
  if (CS > 1) {
    cluster_sync_all();   // every CTA's warp sums are in its red[0]
    if (rank == 0) {
      const uint32_t base = smem_u32(&red[0][0][0]);
      for (int idx = threadIdx.x; idx < M * NC; idx += kF32vWarps * 32) {
        const int m = idx / NC, j = idx - m * NC;
        const uint32_t off = (uint32_t)((m * (NC + 1) + j) * 4);
        float v = red[0][m][j];
        for (int r = 1; r < CS; ++r) v += dsmem_ld_f32(dsmem_map(base + off, (uint32_t)r));
        fin[m][j] = v;
      }
    }
    cluster_sync_all();   // no CTA leaves while rank 0 may still read its shared memory
    if (rank != 0) return;
  } else {
    __syncthreads();
  }
  run_epilogue<float>(e, m0, 16, n0, NC, [&](int m, int j) { return fin[m][j]; }, threadIdx.x, kF32vWarps * 32);
}

template <int NC>
static int launch_gemv_f32(const float* X, long long ldx, const float* W, int M, int N, int K, const EpiParams& e,
                           bool pdl, cudaStream_t stream) {
  const int tiles = (N + NC - 1) / NC;
  // enough CTAs for two per SM, at most 8 per cluster (portable), at least 8 K steps per warp
  const int mb = (M + 15) / 16;
  int cs = (2 * 148 + tiles * mb - 1) / (tiles * mb);
  cs = cs > 8 ? 8 : cs;
  while (cs > 1 && K < cs * kF32vWarps * 8) --cs;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(tiles * cs), (unsigned)mb);
  cfg.blockDim = dim3(kF32vWarps * 32);
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cs;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  return launch_ex(&cfg, gemv_f32_kernel<NC>, X, ldx, W, M, N, K, e) == cudaSuccess ? JX_OK : JX_ERR_CUDA;
}

int run_gemm_f32(const float* X, long long ldx, const float* W, int M, int N, int K, const EpiParams& e, bool pdl,
                 cudaStream_t stream) {
  if (M <= 0 || N <= 0 || K <= 0) return JX_ERR_SHAPE;
  if (M <= 64) {
    const bool glu = e.kind == JX_EPI_GLU_SILU || e.kind == JX_EPI_GLU_GELU_TANH;
    return glu ? launch_gemv_f32<64>(X, ldx, W, M, N, K, e, pdl, stream)
               : launch_gemv_f32<32>(X, ldx, W, M, N, K, e, pdl, stream);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((N + kF32BN - 1) / kF32BN, (M + kF32BM - 1) / kF32BM);
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return launch_ex(&cfg, gemm_f32_kernel, X, ldx, W, M, N, K, e) == cudaSuccess ? JX_OK : JX_ERR_CUDA;
}

}  // namespace jxb
