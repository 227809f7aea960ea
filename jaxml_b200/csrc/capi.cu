// C ABI of libjxb200: argument checks, layout packing and dispatch to the kernels.
#include <stdio.h>
#include <string.h>

#include "common.cuh"

namespace jxb {
int run_norm(int dtype, const jx_norm_args& p, bool pdl, cudaStream_t stream);
int run_gemv(const bf16* W, const bf16* X, long long Np, long long Kp, int M, const jx_epilogue& e, float* ws,
             long long ws_floats, int* counters, int* status, int grid, bool pdl, cudaStream_t stream);
int gemv_workspace_floats(int grid, int mt);
int run_gemm_k128(const bf16* X, const bf16* W, long long Mp, long long Np, long long Kp, const jx_epilogue& e,
                  int* status, bool pdl, cudaStream_t stream);
int run_gemm_f32(const float* X, long long ldx, const float* W, int M, int N, int K, const jx_epilogue& e, bool pdl,
                 cudaStream_t stream);
int run_qkv_rope_append(int dtype, const jx_qkv_args& p, bool pdl, cudaStream_t stream);
int run_attention_generic(int dtype, const jx_attn_args& p, bool pdl, cudaStream_t stream);
int run_rope_apply(int dtype, const jx_rope_args& p, bool pdl, cudaStream_t stream);
int run_sample(const jx_sample_args& p, bool pdl, cudaStream_t stream);
int run_decode_attention(const jx_dattn_args& a, bool pdl, cudaStream_t stream);
void set_gemv_impl(int impl);
void set_dattn_impl(int impl);
void set_gemm_impl(int impl);
void set_gemm_tile_group(int gm);
int run_prefill_attention(const jx_pattn_args& a, bool pdl, cudaStream_t stream);
void set_pattn_impl(int impl);
long long dattn_workspace_bytes(int B, int Hq, int T, int hd, int n_splits);
int dattn_n_splits(int T, int window);
int run_filter_logits(const jx_filter_args& p, cudaStream_t stream);
int run_sample_finalize(const jx_sample_args& p, const unsigned long long* gathered, int n_shards,
                        cudaStream_t stream);

static thread_local char g_err[512] = "";

int note_cuda(const char* where) {
  const cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) return JX_OK;
  snprintf(g_err, sizeof(g_err), "%s: %s", where, cudaGetErrorString(e));
  return JX_ERR_CUDA;
}

int fail(int code, const char* msg) {
  snprintf(g_err, sizeof(g_err), "%s", msg);
  return code;
}

// ------------------------------------------------------------------------------------------------
// K128 pack / unpack
// ------------------------------------------------------------------------------------------------
template <typename S>
__global__ void pack_k128_kernel(const S* __restrict__ src, long long rows, long long cols, long long ld, int transposed,
                                 bf16* __restrict__ dst, long long rp, long long cp) {
  const long long total = rp * cp;
  for (long long o = blockIdx.x * (long long)blockDim.x + threadIdx.x; o < total; o += (long long)gridDim.x * blockDim.x) {
    // invert k128_offset
    const long long unit = o >> 10, within = o & 1023;
    const long long groups = rp >> 3;
    const long long kchunk = unit / groups, rg = unit - kchunk * groups;
    const long long kcore = within >> 6, r8 = (within >> 3) & 7, k8 = within & 7;
    const long long r = rg * 8 + r8, k = kchunk * 128 + kcore * 8 + k8;
    float v = 0.f;
    if (r < rows && k < cols) v = to_f(transposed ? src[k * ld + r] : src[r * ld + k]);
    dst[o] = __float2bfloat16_rn(v);
  }
}

template <typename D>
__global__ void unpack_k128_kernel(const bf16* __restrict__ src, long long rows, long long cols, long long rp,
                                   D* __restrict__ dst, long long ld) {
  const long long total = rows * cols;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / cols, k = i - r * cols;
    dst[r * ld + k] = from_f<D>(__bfloat162float(src[k128_offset(r, k, rp)]));
  }
}

}  // namespace jxb

using namespace jxb;

extern "C" {

const char* jx_version(void) { return "jxb200 0.1 (sm_100a)"; }
const char* jx_last_error(void) { return g_err; }

int jx_device_sm_count(int* out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return note_cuda("cudaGetDevice");
  if (cudaDeviceGetAttribute(out, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return note_cuda("cudaDeviceGetAttribute");
  return JX_OK;
}

int jx_memset_async(void* ptr, int value, long long bytes, void* stream) {
  if (!ptr || bytes < 0) return fail(JX_ERR_ARG, "jx_memset_async: bad pointer or size");
  if (cudaMemsetAsync(ptr, value, (size_t)bytes, (cudaStream_t)stream) != cudaSuccess) return note_cuda("cudaMemsetAsync");
  return JX_OK;
}

int jx_pack_k128(const void* src, int src_dtype, long long rows, long long cols, long long src_ld, int transposed,
                 void* dst, long long rp, long long cp, void* stream) {
  if (!src || !dst) return fail(JX_ERR_ARG, "jx_pack_k128: null pointer");
  if (rp % 8 || cp % 128 || rows > rp || cols > cp || rows < 0 || cols < 0)
    return fail(JX_ERR_SHAPE, "jx_pack_k128: padded sizes must be multiples of 8 (rows) / 128 (cols) and cover the matrix");
  const long long total = rp * cp;
  const int threads = 256;
  const long long blocks = (total + threads - 1) / threads;
  const int grid = (int)(blocks < 65535 * 16 ? blocks : 65535 * 16);
  cudaStream_t s = (cudaStream_t)stream;
  if (src_dtype == JX_F32)
    pack_k128_kernel<float><<<grid, threads, 0, s>>>((const float*)src, rows, cols, src_ld, transposed, (bf16*)dst, rp, cp);
  else if (src_dtype == JX_BF16)
    pack_k128_kernel<bf16><<<grid, threads, 0, s>>>((const bf16*)src, rows, cols, src_ld, transposed, (bf16*)dst, rp, cp);
  else
    return fail(JX_ERR_DTYPE, "jx_pack_k128: dtype must be JX_F32 or JX_BF16");
  return note_cuda("jx_pack_k128");
}

int jx_unpack_k128(const void* src, long long rows, long long cols, long long rp, void* dst, int dst_dtype,
                   long long dst_ld, void* stream) {
  if (!src || !dst) return fail(JX_ERR_ARG, "jx_unpack_k128: null pointer");
  if (rp % 8 || rows > rp) return fail(JX_ERR_SHAPE, "jx_unpack_k128: bad row padding");
  const long long total = rows * cols;
  if (total == 0) return JX_OK;
  const long long blocks = (total + 255) / 256;
  const int grid = (int)(blocks < 65535 * 16 ? blocks : 65535 * 16);
  cudaStream_t s = (cudaStream_t)stream;
  if (dst_dtype == JX_F32)
    unpack_k128_kernel<float><<<grid, 256, 0, s>>>((const bf16*)src, rows, cols, rp, (float*)dst, dst_ld);
  else if (dst_dtype == JX_BF16)
    unpack_k128_kernel<bf16><<<grid, 256, 0, s>>>((const bf16*)src, rows, cols, rp, (bf16*)dst, dst_ld);
  else
    return fail(JX_ERR_DTYPE, "jx_unpack_k128: dtype must be JX_F32 or JX_BF16");
  return note_cuda("jx_unpack_k128");
}

int jx_norm(const jx_norm_args* args, int dtype, int pdl, void* stream) {
  if (!args || !args->h) return fail(JX_ERR_ARG, "jx_norm: args and h are required");
  if (args->out && args->kind == JX_NORM_NONE) return fail(JX_ERR_ARG, "jx_norm: an output needs a norm kind");
  if ((args->out_rp > 0 || args->out2_rp > 0) && dtype != JX_BF16)
    return fail(JX_ERR_DTYPE, "jx_norm: K128 outputs are bfloat16 only");
  const int rc = run_norm(dtype, *args, pdl != 0, (cudaStream_t)stream);
  if (rc != JX_OK) return rc == JX_ERR_CUDA ? note_cuda("jx_norm") : fail(rc, "jx_norm: unsupported sizes or dtype");
  return JX_OK;
}

int jx_set_decode_linear_impl(int impl) {
  if (impl < 0 || impl > 3)
    return fail(JX_ERR_ARG, "jx_set_decode_linear_impl: 0 (by shape), 1 (mma.sync), 2 (tcgen05), 3 (row split)");
  set_gemv_impl(impl);
  return JX_OK;
}

int jx_linear_decode_workspace(int grid, int M, long long* floats_out) {
  if (!floats_out || M <= 0 || M > 64) return fail(JX_ERR_SHAPE, "jx_linear_decode_workspace: M must be in [1, 64]");
  const int mt = M <= 16 ? 1 : (M <= 32 ? 2 : 4);
  *floats_out = gemv_workspace_floats(grid <= 0 ? 148 : grid, mt);
  return JX_OK;
}

int jx_linear_decode(const void* W, const void* X, long long Np, long long Kp, int M, const jx_epilogue* epi,
                     float* ws, long long ws_floats, int* counters, int* status, int grid, int pdl, void* stream) {
  if (!W || !X || !epi || !ws || !counters) return fail(JX_ERR_ARG, "jx_linear_decode: null pointer");
  const int rc = run_gemv((const bf16*)W, (const bf16*)X, Np, Kp, M, *epi, ws, ws_floats, counters, status, grid,
                          pdl != 0, (cudaStream_t)stream);
  if (rc == JX_ERR_CUDA) return note_cuda("jx_linear_decode");
  if (rc != JX_OK)
    return fail(rc, "jx_linear_decode: bad shape (M<=64, Np%64, Kp%128), alignment, workspace or push fields");
  return JX_OK;
}

int jx_linear_prefill(const void* X, const void* W, long long Mp, long long Np, long long Kp, const jx_epilogue* epi,
                      int* status, int pdl, void* stream) {
  if (!W || !X || !epi) return fail(JX_ERR_ARG, "jx_linear_prefill: null pointer");
  if (epi->kind == JX_EPI_PUSH_F32) return fail(JX_ERR_UNSUPPORTED, "jx_linear_prefill: the push epilogue is decode-only");
  const int rc = run_gemm_k128((const bf16*)X, (const bf16*)W, Mp, Np, Kp, *epi, status, pdl != 0, (cudaStream_t)stream);
  if (rc == JX_ERR_CUDA) return note_cuda("jx_linear_prefill");
  if (rc != JX_OK) return fail(rc, "jx_linear_prefill: Mp, Np and Kp must be multiples of 128");
  return JX_OK;
}

int jx_linear_f32(const float* X, long long ldx, const float* W, int M, int N, int K, const jx_epilogue* epi, int pdl,
                  void* stream) {
  if (!X || !W || !epi) return fail(JX_ERR_ARG, "jx_linear_f32: null pointer");
  if (epi->kind == JX_EPI_PUSH_F32) return fail(JX_ERR_UNSUPPORTED, "jx_linear_f32: the push epilogue is decode-only");
  const int rc = run_gemm_f32(X, ldx, W, M, N, K, *epi, pdl != 0, (cudaStream_t)stream);
  if (rc == JX_ERR_CUDA) return note_cuda("jx_linear_f32");
  if (rc != JX_OK) return fail(rc, "jx_linear_f32: bad shape");
  return JX_OK;
}

int jx_qkv_rope_append(const jx_qkv_args* args, int dtype, int pdl, void* stream) {
  if (!args || !args->qkv || !args->q_out || !args->k_cache || !args->v_cache || !args->cos || !args->sin)
    return fail(JX_ERR_ARG, "jx_qkv_rope_append: null pointer");
  if (args->decode && !args->pos_id) return fail(JX_ERR_ARG, "jx_qkv_rope_append: decode needs pos_id");
  const int rc = run_qkv_rope_append(dtype, *args, pdl != 0, (cudaStream_t)stream);
  if (rc == JX_ERR_CUDA) return note_cuda("jx_qkv_rope_append");
  if (rc != JX_OK) return fail(rc, "jx_qkv_rope_append: unsupported head size / rotary dim / dtype");
  return JX_OK;
}

int jx_rope_apply(const jx_rope_args* args, int dtype, int pdl, void* stream) {
  if (!args || !args->cos || !args->sin || !args->pos || (args->Hq > 0 && (!args->q || !args->q_out)) ||
      (args->Hk > 0 && (!args->k || !args->k_out)))
    return fail(JX_ERR_ARG, "jx_rope_apply: null pointer");
  const int rc = run_rope_apply(dtype, *args, pdl != 0, (cudaStream_t)stream);
  if (rc == JX_ERR_CUDA) return note_cuda("jx_rope_apply");
  if (rc != JX_OK) return fail(rc, "jx_rope_apply: unsupported head size / rotary dim / dtype");
  return JX_OK;
}

int jx_attention(const jx_attn_args* args, int dtype, int pdl, void* stream) {
  if (!args || !args->q || !args->k || !args->v || !args->out) return fail(JX_ERR_ARG, "jx_attention: null pointer");
  if (args->out_rp > 0 && dtype != JX_BF16) return fail(JX_ERR_DTYPE, "jx_attention: K128 output is bfloat16 only");
  const int rc = run_attention_generic(dtype, *args, pdl != 0, (cudaStream_t)stream);
  if (rc == JX_ERR_CUDA) return note_cuda("jx_attention");
  if (rc != JX_OK) return fail(rc, "jx_attention: unsupported sizes or dtype");
  return JX_OK;
}

int jx_decode_attention_workspace(int B, int Hq, int hd, int T, int window, long long* bytes_out) {
  if (!bytes_out || B <= 0 || Hq <= 0 || hd <= 0 || T <= 0) return fail(JX_ERR_SHAPE, "jx_decode_attention_workspace: bad sizes");
  *bytes_out = dattn_workspace_bytes(B, Hq, T, hd, dattn_n_splits(T, window));
  return JX_OK;
}

int jx_decode_attention(const jx_dattn_args* args, int pdl, void* stream) {
  if (!args || !(args->q || args->qkv) || !args->k_base || !args->v_base || !args->out || !args->ws || !args->counters ||
      !args->len_ptr)
    return fail(JX_ERR_ARG, "jx_decode_attention: null pointer");
  const int rc = run_decode_attention(*args, pdl != 0, (cudaStream_t)stream);
  if (rc == JX_ERR_CUDA) return note_cuda("jx_decode_attention");
  if (rc == JX_ERR_UNSUPPORTED) return fail(rc, "jx_decode_attention: the fused RoPE inputs (qkv) need the split form");
  if (rc != JX_OK)
    return fail(rc, "jx_decode_attention: head_dim must be 64/128/256, Hq/Hkv <= 16, out_rp >= B and a multiple "
                    "of 8, workspace large enough, 16-byte aligned q/cache, and with qkv: tables, 0 < rd <= hd "
                    "even, ld_qkv >= (Hq + 2 Hkv) hd and a multiple of 8");
  return JX_OK;
}

int jx_set_prefill_tile_group(int gm) {
  if (gm < 0) return fail(JX_ERR_ARG, "jx_set_prefill_tile_group: gm >= 0");
  set_gemm_tile_group(gm);
  return JX_OK;
}

int jx_set_prefill_linear_impl(int impl) {
  if (impl < 0 || impl > 2)
    return fail(JX_ERR_ARG, "jx_set_prefill_linear_impl: 0 (by shape), 1 (mma.sync), 2 (tcgen05)");
  set_gemm_impl(impl);
  return JX_OK;
}

int jx_set_decode_attention_impl(int impl) {
  if (impl < 0 || impl > 5)
    return fail(JX_ERR_ARG, "jx_set_decode_attention_impl: 0 (by shape), 1 (split), 2 (cluster), 3 (column pv), "
                            "4 (cluster-split), 5 (queue)");
  set_dattn_impl(impl);
  return JX_OK;
}

int jx_set_prefill_attention_impl(int impl) {
  if (impl < 0 || impl > 2)
    return fail(JX_ERR_ARG, "jx_set_prefill_attention_impl: 0 (by shape), 1 (mma.sync), 2 (tcgen05)");
  set_pattn_impl(impl);
  return JX_OK;
}

int jx_prefill_attention(const jx_pattn_args* args, int pdl, void* stream) {
  if (!args || !args->q || !args->k_base || !args->v_base || !args->out || !args->len_ptr)
    return fail(JX_ERR_ARG, "jx_prefill_attention: null pointer");
  const int rc = run_prefill_attention(*args, pdl != 0, (cudaStream_t)stream);
  if (rc == JX_ERR_CUDA) return note_cuda("jx_prefill_attention");
  if (rc != JX_OK) return fail(rc, "jx_prefill_attention: head_dim must be 64/128/256, Hq % Hkv == 0, S <= T");
  return JX_OK;
}

int jx_filter_logits(const jx_filter_args* args, void* stream) {
  if (!args || !args->logits || !args->out) return fail(JX_ERR_ARG, "jx_filter_logits: null pointer");
  const int rc = run_filter_logits(*args, (cudaStream_t)stream);
  if (rc == JX_ERR_CUDA) return note_cuda("jx_filter_logits");
  if (rc == JX_ERR_DTYPE) return fail(rc, "jx_filter_logits: logits must be float32 or bfloat16");
  if (rc != JX_OK) return fail(rc, "jx_filter_logits: B <= 8191, 0 < V <= 393216 and V <= each leading dimension");
  return JX_OK;
}

int jx_sample(const jx_sample_args* args, int pdl, void* stream) {
  if (!args || !args->logits || !args->ws || !args->counters) return fail(JX_ERR_ARG, "jx_sample: null pointer");
  if (!args->greedy && (!args->rng || (args->dtype == JX_BF16 && !args->gumbel_tab)))
    return fail(JX_ERR_ARG, "jx_sample: temperature sampling needs rng state and the Gumbel table");
  if (!args->greedy && !(args->temp > 0.f)) return fail(JX_ERR_ARG, "jx_sample: temperature must be positive");
  if (!args->finalize && !args->row_best) return fail(JX_ERR_ARG, "jx_sample: finalize == 0 needs row_best");
  const int rc = run_sample(*args, pdl != 0, (cudaStream_t)stream);
  if (rc == JX_ERR_CUDA) return note_cuda("jx_sample");
  if (rc != JX_OK) return fail(rc, "jx_sample: bad sizes or dtype");
  return JX_OK;
}

int jx_sample_finalize(const jx_sample_args* args, const unsigned long long* gathered, int n_shards, void* stream) {
  if (!args || !gathered || n_shards <= 0) return fail(JX_ERR_ARG, "jx_sample_finalize: bad arguments");
  const int rc = run_sample_finalize(*args, gathered, n_shards, (cudaStream_t)stream);
  if (rc == JX_ERR_CUDA) return note_cuda("jx_sample_finalize");
  if (rc != JX_OK) return fail(rc, "jx_sample_finalize: bad sizes");
  return JX_OK;
}

}  // extern "C"

// ------------------------------------------------------------------------------------------------
// tensor-parallel peer memory and all-reduce
// ------------------------------------------------------------------------------------------------
namespace jxb {
long long ar_region_bytes(long long max_floats, int world);
long long ar_data_offset(long long max_floats, int which);
void comm_layout(long long max_floats, int world, long long* out);
int run_allreduce_f32(void* const* bases, int rank, int world, long long max_floats, int which, long long n,
                      float* out, int* status, bool pdl, cudaStream_t s);
}  // namespace jxb

extern "C" {

int jx_comm_alloc(long long bytes, void** ptr_out) {
  if (!ptr_out || bytes <= 0) return fail(JX_ERR_ARG, "jx_comm_alloc: null output or non-positive size");
  void* p = nullptr;
  if (cudaMalloc(&p, (size_t)bytes) != cudaSuccess) return note_cuda("jx_comm_alloc");
  if (cudaMemset(p, 0, (size_t)bytes) != cudaSuccess) {
    cudaFree(p);
    return note_cuda("jx_comm_alloc");
  }
  *ptr_out = p;
  return JX_OK;
}

int jx_comm_free(void* ptr) {
  if (!ptr) return JX_OK;
  return cudaFree(ptr) == cudaSuccess ? JX_OK : note_cuda("jx_comm_free");
}

int jx_ipc_get_handle(const void* ptr, unsigned char* handle_out) {
  if (!ptr || !handle_out) return fail(JX_ERR_ARG, "jx_ipc_get_handle: null pointer");
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, const_cast<void*>(ptr)) != cudaSuccess) return note_cuda("jx_ipc_get_handle");
  memcpy(handle_out, &h, sizeof(h));
  return JX_OK;
}

int jx_ipc_open_handle(const unsigned char* handle, void** ptr_out) {
  if (!handle || !ptr_out) return fail(JX_ERR_ARG, "jx_ipc_open_handle: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return note_cuda("jx_ipc_open_handle");
  *ptr_out = p;
  return JX_OK;
}

int jx_ipc_close_handle(void* ptr) {
  if (!ptr) return JX_OK;
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? JX_OK : note_cuda("jx_ipc_close_handle");
}

int jx_comm_layout(long long max_floats, int world, long long* out10) {
  if (max_floats <= 0 || world < 1 || world > 8 || !out10)
    return fail(JX_ERR_ARG, "jx_comm_layout: max_floats > 0, 1 <= world <= 8, non-null output");
  jxb::comm_layout(max_floats, world, out10);
  return JX_OK;
}

int jx_allreduce_f32(void* const* bases, int rank, int world, long long max_floats, int which, long long n,
                     float* out, int* status, int pdl, void* stream) {
  if (!bases) return fail(JX_ERR_ARG, "jx_allreduce_f32: null region table");
  const int rc =
      jxb::run_allreduce_f32(bases, rank, world, max_floats, which, n, out, status, pdl != 0, (cudaStream_t)stream);
  if (rc == JX_ERR_CUDA) return note_cuda("jx_allreduce_f32");
  if (rc != JX_OK)
    return fail(rc, "jx_allreduce_f32: 1 <= world <= 8, 0 <= rank < world, which 0 or 1, n a positive multiple "
                    "of 4 and at most max_floats, every region 256-byte aligned, out 16-byte aligned");
  return JX_OK;
}

}  // extern "C"
