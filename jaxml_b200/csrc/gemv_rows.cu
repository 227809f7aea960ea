// Decode projection split by output rows: Y[M, N] = X[M, K] . W[N, K]^T for M <= 16 token rows, bfloat16
// operands in the K128 tiled layout, float32 accumulation on mma.sync.
//
// The stream-K kernels (gemv.cu, gemv_tc.cu) give every SM the same number of bytes by splitting K
// across CTAs, and pay for it at the end: the CTAs sharing a weight block publish float32 partial tiles
// and the last to arrive sums them (two L2 round trips and an atomic before the epilogue can run), while
// the kernel's last CTAs finish.  For the projections with fewer 128-row blocks than SMs (the decode
// qkv, o_proj and down projections of a Llama-3-8B-shaped layer) this kernel instead gives CTA c the
// output rows [c * ROWS, (c + 1) * ROWS) over the whole K: no partial tiles, no arrival counters, and a
// CTA's epilogue follows its own last MMA.  ROWS (32 or 48) is chosen so that the grid is at most one
// CTA per SM; at the shapes above that is 128 CTAs, each streaming ROWS x K weights through a ring of
// TMA bulk copies (every ROWS-row run of one 128-wide K chunk is one contiguous block of the layout).
//
// Warp roles: warp 0 = TMA producer; consumer warp w (RG row groups x 4 K slices) owns weight rows
// [(w % RG) * 16, + 16) and K steps [(w / RG) * 2, + 2) of every 128-wide chunk.  The 4 K-slice partials
// are summed in slice order through shared memory (deterministic), then the shared fused epilogue runs.
#include "common.cuh"
#include "epilogue.cuh"

namespace jxb {

// ---- normalisation tail (jx_epilogue.tn_*) ----
// One warp normalises row m of the projection's [M, ldo] bf16 output into the K128 operand tn_x with
// jx_norm's vectorised arithmetic and summation order: there a block of d / 8 threads holds 8 values
// each, sums them in order, adds over the lanes of each warp with an xor butterfly, stores each warp's
// lane-0 value and adds those with a second butterfly, every lane keeping its own result.  Here lane l
// plays lane l of every one of those d / 256 warps (w), so it holds the same partial sums, takes the
// same lane-0 values from the butterflies and ends with the same per-lane totals: bit-identical output.
constexpr int kTnMaxWarps = 32;   // d <= 8192

__device__ __forceinline__ uint4 tn_ld(const bf16* p) {
  return __ldcg(reinterpret_cast<const uint4*>(p));   // written by other CTAs of this grid
}
__device__ __forceinline__ void tn_unpack(const uint4& u, float* v) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

// jx_norm's two-stage block sum of per-(virtual warp, lane) partials part[w] (zero for w >= nw).  The
// 32 butterflies are independent chains (no early exit), so their shuffles overlap.
__device__ __forceinline__ float tn_block_sum(const float* part, int lane) {
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < kTnMaxWarps; ++w) {
    float v = part[w];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const float lane0 = __shfl_sync(0xffffffffu, v, 0);
    if (lane == w) t = lane0;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  return t;
}

// Per-(virtual warp, lane) partial sums of row h: sum of x (mode 0), of x^2 (mode 1) or of (x - mean)^2
// (mode 2).  Loads go out 8 at a time (predicated, no early exit) so that they overlap.
__device__ __forceinline__ void tn_partials(const bf16* h, int nw, int lane, int mode, float mean, float* part) {
#pragma unroll
  for (int c0 = 0; c0 < kTnMaxWarps; c0 += 8) {
    uint4 u[8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
      u[j] = c0 + j < nw ? tn_ld(h + ((c0 + j) * 32 + lane) * 8) : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float x[8];
      tn_unpack(u[j], x);
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) s += mode == 0 ? x[i] : (mode == 1 ? x[i] * x[i] : (x[i] - mean) * (x[i] - mean));
      part[c0 + j] = c0 + j < nw ? s : 0.f;
    }
  }
}

__device__ __forceinline__ void tail_norm_row(const EpiParams& e, int m, int lane) {
  const int d = e.N, nw = d >> 8;
  const bf16* h = reinterpret_cast<const bf16*>(e.out) + (long long)m * e.ldo;
  const bf16* w = reinterpret_cast<const bf16*>(e.tn_w);
  const bf16* b = reinterpret_cast<const bf16*>(e.tn_b);
  bf16* X = reinterpret_cast<bf16*>(e.tn_x);
  const bool layer = e.tn_kind == JX_NORM_LAYER;
  float part[kTnMaxWarps];
  float mean = 0.f;
  if (layer) {
    tn_partials(h, nw, lane, 0, 0.f, part);
    mean = tn_block_sum(part, lane) / (float)d;
  }
  tn_partials(h, nw, lane, layer ? 2 : 1, mean, part);
  const float den = sqrtf(tn_block_sum(part, lane) / (float)d + e.tn_eps);
  const float inv = 1.0f / den;
#pragma unroll
  for (int c0 = 0; c0 < kTnMaxWarps; c0 += 4) {
    uint4 uh[4], uw[4], ub[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int j0 = ((c0 + j) * 32 + lane) * 8;
      const bool on = c0 + j < nw;
      uh[j] = on ? tn_ld(h + j0) : make_uint4(0, 0, 0, 0);
      uw[j] = on ? tn_ld(w + j0) : make_uint4(0, 0, 0, 0);
      ub[j] = on && b ? tn_ld(b + j0) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (c0 + j >= nw) continue;
      const int j0 = ((c0 + j) * 32 + lane) * 8;
      float x[8], wv[8], bv[8], y[8];
      tn_unpack(uh[j], x);
      tn_unpack(uw[j], wv);
      tn_unpack(ub[j], bv);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (layer)
          y[i] = rnd<bf16>((x[i] - mean) / den * wv[i] + (b ? bv[i] : 0.f));
        else if (e.tn_kind == JX_NORM_RMS)
          y[i] = rnd<bf16>(wv[i] * rnd<bf16>(x[i] / den));
        else
          y[i] = rnd<bf16>((wv[i] + 1.0f) * (x[i] * inv));
      }
      uint4 o;
      o.x = pack_bf16x2(y[0], y[1]);
      o.y = pack_bf16x2(y[2], y[3]);
      o.z = pack_bf16x2(y[4], y[5]);
      o.w = pack_bf16x2(y[6], y[7]);
      *reinterpret_cast<uint4*>(X + k128_offset(m, j0, e.tn_rp)) = o;
    }
  }
}

// K chunks per ring stage and in flight.  The consumers' mbarrier wait and arrival per stage, not the
// bytes in flight, limited this kernel: with one 128-wide chunk a stage (10 in flight) qkv / o_proj / down
// took 10.6 / 9.5 / 26.2 us and the step 3.72 ms; 2 a stage (10 in flight) 9.6 / 8.0 / 21.6 us, 3.54 ms;
// 3 a stage (9) 9.7 / 7.9 / 21.4 us; 5 a stage (10) 10.3 / 8.5 / 23.0 us; 2 a stage with 12 in flight
// 9.6 / 8.2 / 21.7 us; 4 a stage with 12 in flight 9.7 / 7.5 / 19.5 us (down at 0.92 of the measured
// copy bandwidth) and 3.49 ms; 4 a stage with 16 in flight for the 32-row CTAs (o_proj, down; the 48-row
// ones keep 12, the shared memory holds no more) 9.7 / 7.5 / 19.0 us and 3.42 ms; 8 a stage (16 / 8 in
// flight) 13.0 / 8.0 / 20.2 us, 3.56-3.60 ms (same calls).
constexpr int kRowsChunksPerStage = 4;
constexpr int kRowsChunksInFlight = 12;
constexpr int kRowsChunksInFlight32 = 16;   // 32-row CTAs

template <int RG>
struct RowsCfg {
  static constexpr int ROWS = 16 * RG;
  static constexpr int kConsumers = RG * 4;                 // warps
  static constexpr int kThreads = 32 * (1 + kConsumers);
  static constexpr int kWBytes = ROWS * 128 * 2;            // 8 / 12 KB: one 128-wide K chunk of weights
  static constexpr int kXBytes = 16 * 128 * 2;              // 4 KB: one chunk of activations
  static constexpr int kCps = kRowsChunksPerStage;          // K chunks per ring stage
  // a stage: kCps weight chunks, then their kCps activation chunks (contiguous in the K128 layout)
  static constexpr int kStageBytes = kCps * (kWBytes + kXBytes);
  // 10 chunks in flight (120 / 160 KB): 16 / 12 measured slower on every decode shape with one chunk a
  // stage (e.g. o_proj 8.8 -> 9.4 us): the next kernel's CTAs start later behind a larger one.
  static constexpr int kStages = (RG == 2 ? kRowsChunksInFlight32 : kRowsChunksInFlight) / kCps;
  static constexpr int kLd = ROWS + 4;                      // float32 row stride of the staging tiles
  static constexpr int kPartBytes = 4 * 16 * kLd * 4;       // [4 K slices][16 tokens][ROWS]
  static constexpr int kSmem = kStages * kStageBytes + kPartBytes + 2 * kStages * 8 + 16;
};

// TAIL: the normalisation tail is compiled in (its code roughly doubles the kernel's registers, so the
// kernel without it is a separate instantiation).
template <int RG, bool TAIL>
__global__ void __launch_bounds__(RowsCfg<RG>::kThreads, 1)
    gemv_rows_kernel(const bf16* __restrict__ W, const bf16* __restrict__ X, long long Np, long long Kp, EpiParams e,
                     int* status) {
  using C = RowsCfg<RG>;
  extern __shared__ __align__(128) uint8_t smem[];
  float* part = reinterpret_cast<float*>(smem + C::kStages * C::kStageBytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kStages * C::kStageBytes + C::kPartBytes);
  uint64_t* empty = full + C::kStages;
  volatile int* dead = reinterpret_cast<volatile int*>(empty + C::kStages);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long r0 = (long long)blockIdx.x * C::ROWS;
  const int kc = (int)(Kp >> 7);

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], C::kConsumers);
    }
    *dead = 0;
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      auto wsrc = [&](int kk) { return W + (((long long)kk * (Np >> 3) + (r0 >> 3)) << 10); };
      auto xsrc = [&](int kk) { return X + ((long long)kk << 11); };   // 16 rows x 128 k per chunk
      const uint64_t pol_w = l2_policy_evict_first();   // weights are read once per step
      const int ns = (kc + C::kCps - 1) / C::kCps;      // stages of the whole K
      auto nch = [&](int st) { return kc - st * C::kCps < C::kCps ? kc - st * C::kCps : C::kCps; };
      auto issue_w = [&](int st, int s) {
        mbar_arrive_expect_tx(&full[s], nch(st) * (C::kWBytes + C::kXBytes));
        for (int j = 0; j < nch(st); ++j)
          bulk_g2s_hint(smem + s * C::kStageBytes + j * C::kWBytes, wsrc(st * C::kCps + j), C::kWBytes, &full[s],
                        pol_w);
      };
      auto issue_x = [&](int st, int s) {
        bulk_g2s(smem + s * C::kStageBytes + C::kCps * C::kWBytes, xsrc(st * C::kCps), nch(st) * C::kXBytes,
                 &full[s]);
      };
      const int pre = ns < C::kStages ? ns : C::kStages;
      // Weights do not depend on the previous kernel: start streaming them before waiting on it.
      for (int st = 0; st < pre; ++st) issue_w(st, st);
      pdl_wait();
      pdl_trigger();
      for (int st = 0; st < pre; ++st) issue_x(st, st);
      int issued = pre;
      for (int st = pre; st < ns; ++st) {
        const int s = st % C::kStages;
        if (!mbar_wait_bounded(&empty[s], ((st / C::kStages) - 1) & 1)) {
          set_status(status, JX_ERR_TIMEOUT);
          *dead = 1;
          break;
        }
        issue_w(st, s);
        issue_x(st, s);
        issued = st + 1;
      }
      // every issued copy lands before this CTA's shared memory is released
      for (int i = (issued > C::kStages ? issued - C::kStages : 0); i < issued; ++i)
        if (!mbar_wait_bounded(&full[i % C::kStages], (i / C::kStages) & 1)) break;
    }
    return;
  }

  // ---------------- consumers ----------------
  pdl_wait();
  pdl_trigger();
  const int cw = (warp - 1) % RG;     // weight rows [cw * 16, + 16)
  const int ksl = (warp - 1) / RG;    // K steps [ksl * 2, + 2) of every chunk
  const int tid = threadIdx.x - 32;
  // The tensor-core accumulator is folded into an IEEE float32 sum every 4 chunks (8 MMAs): one chain over
  // the whole K rounds noticeably worse than float32 sums (bf16 results flip more often).  Every 8 chunks
  // saved up to 0.8 us on the down projection but took a small bf16 model's decode logits to 1.5 ulps
  // (0.0234) from the oracle's, past the 2e-2 bound that every 4 chunks meets.
  float acc[2][4] = {}, sum[2][4] = {};
  bool ok = true;
  const int mi = lane >> 3, r8 = lane & 7;
  const int ns = (kc + C::kCps - 1) / C::kCps;
  for (int st = 0; st < ns; ++st) {
    const int s = st % C::kStages;
    if (ok && (*dead || !mbar_wait_bounded(&full[s], (st / C::kStages) & 1))) {
      ok = false;
      *dead = 1;
      set_status(status, JX_ERR_TIMEOUT);
    }
#pragma unroll
    for (int j = 0; j < C::kCps; ++j) {
    const int i = st * C::kCps + j;
    if (i >= kc) break;
    if (ok) {
      const uint32_t sW = smem_u32(smem + s * C::kStageBytes + j * C::kWBytes);
      const uint32_t sX = smem_u32(smem + s * C::kStageBytes + C::kCps * C::kWBytes + j * C::kXBytes);
#pragma unroll
      for (int kq = 0; kq < 2; ++kq) {
        const int ks = ksl * 2 + kq;
        uint32_t b0, b1, b2, b3, a0, a1, a2, a3;
        {
          const int rg = cw * 2 + (mi >> 1), kcore = ks * 2 + (mi & 1);
          ldsm_x4(sW + (uint32_t)((rg * 1024 + kcore * 64 + r8 * 8) * 2), b0, b1, b2, b3);
        }
        {
          const int rg = mi & 1, kcore = ks * 2 + (mi >> 1);
          ldsm_x4(sX + (uint32_t)((rg * 1024 + kcore * 64 + r8 * 8) * 2), a0, a1, a2, a3);
        }
        mma_bf16(acc[0], a0, a1, a2, a3, b0, b1);
        mma_bf16(acc[1], a0, a1, a2, a3, b2, b3);
      }
    }
    if ((i & 3) == 3 || i == kc - 1) {
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          sum[nt][q] += acc[nt][q];
          acc[nt][q] = 0.f;
        }
    }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
  // this warp's partial: tokens lane / 4 (+ 8) x weight rows cw * 16 + nt * 8 + (lane % 4) * 2 (+ 1)
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    const int t = lane >> 2, col = cw * 16 + nt * 8 + (lane & 3) * 2;
    float* p0 = part + (ksl * 16 + t) * C::kLd + col;
    float* p1 = part + (ksl * 16 + t + 8) * C::kLd + col;
    p0[0] = sum[nt][0];
    p0[1] = sum[nt][1];
    p1[0] = sum[nt][2];
    p1[1] = sum[nt][3];
  }
  named_bar_sync(1, C::kConsumers * 32);
  // the K slices summed in slice order into slice 0
  for (int idx = tid; idx < 16 * C::ROWS; idx += C::kConsumers * 32) {
    const int m = idx / C::ROWS, j = idx - m * C::ROWS;
    float v = part[m * C::kLd + j];
#pragma unroll
    for (int q = 1; q < 4; ++q) v += part[(q * 16 + m) * C::kLd + j];
    part[m * C::kLd + j] = v;
  }
  named_bar_sync(1, C::kConsumers * 32);
  if (ok && !*dead)
    run_epilogue<bf16>(e, 0, 16, r0, C::ROWS, [&](int m, int j) { return part[m * C::kLd + j]; }, tid,
                       C::kConsumers * 32);
  if (TAIL && e.tn_x) {
    // the last CTA to finish its columns normalises the rows (see tail_norm_row)
    __shared__ int tn_last;
    __threadfence();
    named_bar_sync(1, C::kConsumers * 32);
    if (tid == 0) tn_last = atomicAdd(e.tn_sync, 1) == (int)gridDim.x - 1;
    named_bar_sync(1, C::kConsumers * 32);
    if (tn_last) {
      __threadfence();
      for (int m = tid >> 5; m < e.M; m += C::kConsumers) tail_norm_row(e, m, lane);
      if (tid == 0) *e.tn_sync = 0;
    }
  }
}

template <int RG, bool TAIL>
static int launch_rows_t(const bf16* W, const bf16* X, long long Np, long long Kp, const EpiParams& e, int* status,
                       bool pdl, cudaStream_t stream) {
  using C = RowsCfg<RG>;
  static bool configured = false;
  if (!configured) {
    if (cudaFuncSetAttribute(gemv_rows_kernel<RG, TAIL>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem) !=
        cudaSuccess)
      return JX_ERR_CUDA;
    configured = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(Np / C::ROWS));
  cfg.blockDim = dim3(C::kThreads);
  cfg.dynamicSmemBytes = C::kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return launch_ex(&cfg, gemv_rows_kernel<RG, TAIL>, W, X, Np, Kp, e, status) == cudaSuccess ? JX_OK : JX_ERR_CUDA;
}

template <int RG>
static int launch_rows(const bf16* W, const bf16* X, long long Np, long long Kp, const EpiParams& e, int* status,
                       bool pdl, cudaStream_t stream) {
  return e.tn_x ? launch_rows_t<RG, true>(W, X, Np, Kp, e, status, pdl, stream)
                : launch_rows_t<RG, false>(W, X, Np, Kp, e, status, pdl, stream);
}

// Row-group count (2 -> 32 rows, 3 -> 48 rows per CTA) for an Np-row projection on `sms` SMs: the
// smallest whose grid fits one CTA per SM and divides Np; 0 when none does.
int gemv_rows_groups(long long Np, int sms) {
  for (int rg = 2; rg <= 3; ++rg)
    if (Np % (16 * rg) == 0 && Np / (16 * rg) <= sms) return rg;
  return 0;
}

int run_gemv_rows(const bf16* W, const bf16* X, long long Np, long long Kp, int M, const EpiParams& e, int* status,
                  int sms, bool pdl, cudaStream_t stream) {
  if (M <= 0 || M > 16 || Kp % 128 || Kp <= 0) return JX_ERR_SHAPE;
  if ((reinterpret_cast<uintptr_t>(W) | reinterpret_cast<uintptr_t>(X)) & 15) return JX_ERR_ARG;
  switch (gemv_rows_groups(Np, sms)) {
    case 2: return launch_rows<2>(W, X, Np, Kp, e, status, pdl, stream);
    case 3: return launch_rows<3>(W, X, Np, Kp, e, status, pdl, stream);
    default: return JX_ERR_SHAPE;
  }
}

}  // namespace jxb
