// Tensor-parallel all-reduce of the row-parallel projections' float32 partial sums over NVLink peer
// memory (the reference all-reduces the o_proj / down_proj outputs of its "heads"/"intermediate"
// sharding through XLA's GSPMD collectives, inference_engine/engine.py:258-267 and models/llama.py:133-137).
//
// Every rank owns one device region (cudaMalloc'd here, shared with the other ranks through CUDA IPC):
//   [header: flags, counters, the ranks' base table][partials buffer 0][partials buffer 1][push slots]
// One-shot algorithm with one handshake, CTA b of every rank working on the same slice:
//   1. pdl wait (the partial in buffer `which` was written by the previous kernel), read seq; v = seq + 1
//   2. write v into flags[b][my rank] of every rank (release, system scope); wait until this rank's
//      flags[b][r] == v for every r (acquire) -> every rank's partial is complete
//   3. read the slice of buffer `which` from every rank (peer loads over NVLink), sum in rank order
//      0..world-1 (every rank computes bit-identical values) and write the sums to this rank's `out`
//   4. the last CTA advances seq
// Consecutive calls alternate the two buffers, so no second ("done reading") handshake is needed: a
// rank rewrites buffer `which` only two calls later, after every rank has passed the handshake of the
// call in between, which every rank enters only once its reads of this call are complete.
// All waits are bounded: on timeout the status word gets JX_ERR_TIMEOUT and the kernel returns.  No
// multicast object and no NVLS are involved: plain peer loads and stores only.
#include "common.cuh"

namespace jxb {

constexpr int kArMaxRanks = 8;
constexpr int kArMaxCtas = 64;
constexpr int kArThreads = 512;
constexpr long long kArFlagBytes = (long long)kArMaxCtas * kArMaxRanks * 4;
// Region header: all-reduce flags, all-reduce counters (+0 seq, +4 finished CTAs), push counters (+0 epoch,
// +4 finished CTAs), the table of every rank's region base as mapped in this process, push flags
// [2 calls][kPushMaxUnits 64-column units][kArMaxRanks sources].
constexpr long long kArCtrOff = kArFlagBytes;
constexpr long long kPushSeqOff = kArCtrOff + 256;
constexpr long long kBasesOff = kPushSeqOff + 256;
constexpr long long kPushFlagOff = kBasesOff + 256;
constexpr long long kPushFlagBytes = 2LL * kPushMaxUnits * kArMaxRanks * 4;
constexpr long long kArHeaderBytes = kPushFlagOff + kPushFlagBytes;

struct ArParams {
  unsigned char* base[kArMaxRanks];   // every rank's region (this rank's own included)
  int rank, world;
  long long n;                        // floats
  long long data_off;                 // byte offset of the partials buffer of this call in every region
  float* out;                         // this rank's result
  int* status;
};

// Signal CTA b's readiness to every rank and wait for every rank's.  Thread r < world does rank r.
// Returns false on timeout.
__device__ __forceinline__ bool ar_handshake(const ArParams& p, unsigned int v) {
  bool ok = true;
  const int b = blockIdx.x;
  if (threadIdx.x < p.world) {
    const int r = threadIdx.x;
    st_release_sys(reinterpret_cast<unsigned int*>(p.base[r]) + b * kArMaxRanks + p.rank, v);
    const unsigned int* mine = reinterpret_cast<const unsigned int*>(p.base[p.rank]) + b * kArMaxRanks + r;
    if (ld_acquire_sys(mine) != v) {
      const uint64_t t0 = globaltimer_ns();
      while (ld_acquire_sys(mine) != v) {
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          ok = false;
          break;
        }
      }
    }
  }
  return __syncthreads_and(ok) != 0;
}

__global__ void __launch_bounds__(kArThreads) allreduce_f32_kernel(ArParams p) {
  __shared__ unsigned int s_seq;
  pdl_trigger();
  pdl_wait();
  unsigned int* ctr = reinterpret_cast<unsigned int*>(p.base[p.rank] + kArCtrOff);   // [0] seq, [1] finished
  if (threadIdx.x == 0) s_seq = *reinterpret_cast<volatile unsigned int*>(ctr);
  __syncthreads();
  const unsigned int v = s_seq + 1;
  if (!ar_handshake(p, v)) {
    if (threadIdx.x == 0) set_status(p.status, JX_ERR_TIMEOUT);
    return;
  }
  // float4 groups: thread t of CTA b takes b * threads + t, then every gridDim.x * threads
  const long long n4 = p.n >> 2;
  const long long stride = (long long)gridDim.x * kArThreads;
  for (long long i = (long long)blockIdx.x * kArThreads + threadIdx.x; i < n4; i += stride) {
    float4 vals[kArMaxRanks];
#pragma unroll
    for (int r = 0; r < kArMaxRanks; ++r)
      if (r < p.world) vals[r] = __ldcv(reinterpret_cast<const float4*>(p.base[r] + p.data_off) + i);
    float4 s = vals[0];
#pragma unroll
    for (int r = 1; r < kArMaxRanks; ++r)
      if (r < p.world) {
        s.x += vals[r].x;
        s.y += vals[r].y;
        s.z += vals[r].z;
        s.w += vals[r].w;
      }
    reinterpret_cast<float4*>(p.out)[i] = s;
  }
  // the last CTA to finish advances seq for the next call
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(ctr + 1, 1u) == gridDim.x - 1) {
      ctr[1] = 0;
      ctr[0] = v;
      __threadfence();
    }
  }
}

static long long ar_buffer_bytes(long long max_floats) { return ((max_floats * 4 + 255) / 256) * 256; }
// Layout: header, all-reduce partials buffers 0 and 1, push receive slots [2 calls][world sources].
long long ar_region_bytes(long long max_floats, int world) {
  return kArHeaderBytes + (2 + 2LL * world) * ar_buffer_bytes(max_floats);
}
long long ar_data_offset(long long max_floats, int which) { return kArHeaderBytes + which * ar_buffer_bytes(max_floats); }
void comm_layout(long long max_floats, int world, long long* out) {
  const long long buf = ar_buffer_bytes(max_floats);
  out[0] = ar_region_bytes(max_floats, world);
  out[1] = ar_data_offset(max_floats, 0);
  out[2] = ar_data_offset(max_floats, 1);
  out[3] = kArHeaderBytes + 2 * buf;   // push receive slots: + ((which * world + source) * recv_stride)
  out[4] = buf;                        // recv_stride (bytes between source slots)
  out[5] = kPushFlagOff;               // push flags: + which * kPushMaxUnits * kArMaxRanks * 4
  out[6] = (long long)kPushMaxUnits * kArMaxRanks * 4;
  out[7] = kPushSeqOff;
  out[8] = kBasesOff;
  out[9] = kPushMaxUnits;
}

int run_allreduce_f32(void* const* bases, int rank, int world, long long max_floats, int which, long long n,
                      float* out, int* status, bool pdl, cudaStream_t s) {
  if (world < 1 || world > kArMaxRanks || rank < 0 || rank >= world || n <= 0 || (n & 3) || n > max_floats ||
      (which != 0 && which != 1) || !out || (reinterpret_cast<uintptr_t>(out) & 15))
    return JX_ERR_ARG;
  ArParams p;
  for (int r = 0; r < kArMaxRanks; ++r) p.base[r] = r < world ? reinterpret_cast<unsigned char*>(bases[r]) : nullptr;
  for (int r = 0; r < world; ++r)
    if (!p.base[r] || (reinterpret_cast<uintptr_t>(p.base[r]) & 255)) return JX_ERR_ARG;
  p.rank = rank;
  p.world = world;
  p.n = n;
  p.data_off = ar_data_offset(max_floats, which);
  p.out = out;
  p.status = status;
  // one float4 group per thread while kArMaxCtas CTAs suffice, then loop
  const long long groups = n >> 2;
  long long ctas = (groups + kArThreads - 1) / kArThreads;
  if (ctas > kArMaxCtas) ctas = kArMaxCtas;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)ctas);
  cfg.blockDim = dim3(kArThreads);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return launch_ex(&cfg, allreduce_f32_kernel, p) == cudaSuccess ? JX_OK : JX_ERR_CUDA;
}

}  // namespace jxb
