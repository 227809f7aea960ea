// Element-wise MLP activations of the reference's MLP blocks, for callers that hold the projection
// outputs separately (the module-level decoder layers; the decode/prefill runtime fuses the same
// arithmetic into the gate/up projection's epilogue instead):
//   GLU kinds  out = dtype(dtype(act(gate)) * up)   models/llama.py:90-95 (silu), gemma3.py:85-90 (gelu tanh)
//   GELU_ERF   out = dtype(gelu_erf(x))             models/gpt_neox.py:84-88
// gate / up / x are already in the model dtype (the projections round their outputs).  One thread per
// element, rows of F elements with their own leading dimensions.
#include "common.cuh"

namespace jxb {

int fail(int code, const char* msg);
int note_cuda(const char* where);

struct ActParams {
  const void* gate;
  long long ldg;
  const void* up;
  long long ldu;
  void* out;
  long long ldo;
  long long M, F;
  int kind;
};

template <typename T>
__global__ void __launch_bounds__(256) mlp_act_kernel(ActParams p) {
  pdl_wait();
  pdl_trigger();
  const long long n = p.M * p.F;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long m = i / p.F, j = i - m * p.F;
    const float g = to_f(reinterpret_cast<const T*>(p.gate)[m * p.ldg + j]);
    float r;
    if (p.kind == JX_EPI_ACT_GELU_ERF) {
      r = gelu_erf_f(g);
    } else {
      const float a = rnd<T>(p.kind == JX_EPI_GLU_SILU ? silu_f(g) : gelu_tanh_f(g));
      r = a * to_f(reinterpret_cast<const T*>(p.up)[m * p.ldu + j]);
    }
    reinterpret_cast<T*>(p.out)[m * p.ldo + j] = from_f<T>(r);
  }
}

int run_mlp_act(int dtype, const ActParams& p, bool pdl, cudaStream_t stream) {
  const bool glu = p.kind == JX_EPI_GLU_SILU || p.kind == JX_EPI_GLU_GELU_TANH;
  if (!glu && p.kind != JX_EPI_ACT_GELU_ERF) return JX_ERR_ARG;
  if (p.M <= 0 || p.F <= 0 || p.ldg < p.F || p.ldo < p.F || (glu && p.ldu < p.F)) return JX_ERR_SHAPE;
  const long long n = p.M * p.F;
  long long blocks = (n + 255) / 256;
  if (blocks > 148LL * 64) blocks = 148LL * 64;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)blocks);
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t err;
  if (dtype == JX_BF16)
    err = launch_ex(&cfg, mlp_act_kernel<bf16>, p);
  else if (dtype == JX_F32)
    err = launch_ex(&cfg, mlp_act_kernel<float>, p);
  else
    return JX_ERR_DTYPE;
  return err == cudaSuccess ? JX_OK : JX_ERR_CUDA;
}

}  // namespace jxb

extern "C" int jx_mlp_act(const void* gate, long long ldg, const void* up, long long ldu, void* out, long long ldo,
                          long long M, long long F, int kind, int dtype, int pdl, void* stream) {
  if (!gate || !out || ((kind == JX_EPI_GLU_SILU || kind == JX_EPI_GLU_GELU_TANH) && !up))
    return jxb::fail(JX_ERR_ARG, "jx_mlp_act: null pointer");
  jxb::ActParams p{gate, ldg, up, ldu, out, ldo, M, F, kind};
  const int rc = jxb::run_mlp_act(dtype, p, pdl != 0, (cudaStream_t)stream);
  if (rc == JX_ERR_CUDA) return jxb::note_cuda("jx_mlp_act");
  if (rc != JX_OK) return jxb::fail(rc, "jx_mlp_act: kind must be a GLU or GELU_ERF kind, M, F > 0, leading dims >= F, dtype f32 or bf16");
  return JX_OK;
}
