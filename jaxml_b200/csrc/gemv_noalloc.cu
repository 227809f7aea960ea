// Decode projection for callers that cannot allocate device memory.
//
// jx_linear_decode needs a scratch buffer (split-K partial tiles and per-block arrival counters) that the
// caller allocates.  Some callers cannot: code that runs inside a host framework's custom-call / FFI
// handler, where the framework owns every device allocation and the handler may only use the buffers
// it is handed, or a plugin that must not call cudaMalloc at all (allocation can synchronise the device
// and break the caller's stream ordering or its CUDA-graph capture).  jx_linear_decode_noalloc runs the
// same kernel with its scratch in a fixed-size array compiled into this library instead.
//
// The array lives in device global memory of every GPU that loads the library, from module load until
// the process exits.  It is sized for up to 148 CTAs, M <= 16 token rows and N <= 262144 weight rows.
// All calls share it and it keeps the previous call's contents, so the arrival counters are cleared at
// the start of every call; two calls that run at the same time on the GPU (different streams) race on
// the shared array and must not overlap.
#include <mutex>

#include "common.cuh"
#include "epilogue.cuh"

namespace jxb {

int run_gemv(const bf16* W, const bf16* X, long long Np, long long Kp, int M, const EpiParams& e, float* ws,
             long long ws_floats, int* counters, int* status, int grid, bool pdl, cudaStream_t stream);
int gemv_workspace_floats(int grid, int mt);
int fail(int code, const char* msg);
int note_cuda(const char* where);

constexpr int kNoAllocMaxGrid = 148;
constexpr int kNoAllocMaxRows = 16;
constexpr long long kNoAllocPartials = (long long)kNoAllocMaxGrid * 2 * kNoAllocMaxRows * 128;  // floats
constexpr int kNoAllocMaxCounters = 4096;      // one per 64-row weight block: N <= 262144
// Partial tiles (2.3 MiB) followed by the arrival counters (16 KiB), 256-byte aligned.
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocPartials + kNoAllocMaxCounters];

static std::mutex g_noalloc_mutex;
static float* g_noalloc_ptr[64] = {};

// Device address of the scratch array on the current device, looked up once per device.
static int noalloc_scratch(float** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return note_cuda("jx_linear_decode_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(JX_ERR_UNSUPPORTED, "jx_linear_decode_noalloc: device index >= 64");
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p)
      return note_cuda("jx_linear_decode_noalloc: cudaGetSymbolAddress");
    g_noalloc_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return JX_OK;
}

}  // namespace jxb

using namespace jxb;

extern "C" int jx_linear_decode_noalloc(const void* W, const void* X, long long Np, long long Kp, int M,
                                        const jx_epilogue* epi, int* status, int grid, int pdl, void* stream) {
  if (!W || !X || !epi) return fail(JX_ERR_ARG, "jx_linear_decode_noalloc: null pointer");
  if (M <= 0 || M > kNoAllocMaxRows)
    return fail(JX_ERR_SHAPE, "jx_linear_decode_noalloc: M must be in [1, 16] (fixed scratch size)");
  if (Np <= 0 || Np % 64 || Np / 64 + 1 > kNoAllocMaxCounters)
    return fail(JX_ERR_SHAPE, "jx_linear_decode_noalloc: Np must be a positive multiple of 64 and <= 262080");
  if (grid > kNoAllocMaxGrid)
    return fail(JX_ERR_SHAPE, "jx_linear_decode_noalloc: grid must be at most 148 CTAs (fixed scratch size)");
  if (grid <= 0) grid = kNoAllocMaxGrid;
  if ((long long)gemv_workspace_floats(grid, 1) > kNoAllocPartials)
    return fail(JX_ERR_SHAPE, "jx_linear_decode_noalloc: grid exceeds the fixed scratch size");
  float* scratch = nullptr;
  int rc = noalloc_scratch(&scratch);
  if (rc != JX_OK) return rc;
  int* counters = reinterpret_cast<int*>(scratch + kNoAllocPartials);
  // The counters must start at zero; the array keeps whatever the previous call (or an aborted one) left.
  // This clear is a stream operation of its own ahead of the kernel, so pdl = 1 cannot overlap the
  // kernel's start with the kernel before it on this entry point.
  if (cudaMemsetAsync(counters, 0, (size_t)(Np / 64 + 1) * sizeof(int), (cudaStream_t)stream) != cudaSuccess)
    return note_cuda("jx_linear_decode_noalloc: clearing counters");
  rc = run_gemv((const bf16*)W, (const bf16*)X, Np, Kp, M, *epi, scratch, kNoAllocPartials, counters, status, grid,
                pdl != 0, (cudaStream_t)stream);
  if (rc == JX_ERR_CUDA) return note_cuda("jx_linear_decode_noalloc");
  if (rc != JX_OK) return fail(rc, "jx_linear_decode_noalloc: bad shape (Kp % 128) or alignment");
  return JX_OK;
}
