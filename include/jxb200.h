/*
 * libjxb200 -- C ABI of the B200 (sm_100a) decode/prefill path that stands in for jaxml's
 * JAX/XLA compute.  Every entry point takes plain device pointers, sizes and a cudaStream_t passed as
 * void*, launches asynchronously on that stream and returns a status code (0 = JX_OK).  The compute
 * entry points allocate no device memory (scratch buffers are passed in by the caller); only the
 * tensor-parallel set-up call jx_comm_alloc allocates (its peer region).  Device-side failures (index
 * out of range, a bounded wait that ran out) are reported through an int status word in device
 * memory that the caller reads after synchronising.
 *
 * The reference has no native code: each entry point replaces a piece of the Flax/XLA program named
 * in its comment (paths relative to the reference's src/jaxml/).
 */
#ifndef JXB200_H_
#define JXB200_H_

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---- */
#define JX_OK 0
#define JX_ERR_ARG 1          /* bad pointer / alignment / workspace size */
#define JX_ERR_SHAPE 2        /* unsupported or inconsistent sizes */
#define JX_ERR_DTYPE 3        /* unsupported dtype */
#define JX_ERR_RANGE 4        /* token id / position / cache slot out of range (device status) */
#define JX_ERR_TIMEOUT 5      /* a bounded device wait ran out (device status) */
#define JX_ERR_CUDA 6         /* a CUDA runtime call failed; see jx_last_error() */
#define JX_ERR_UNSUPPORTED 7

/* ---- enums ---- */
#define JX_F32 0
#define JX_BF16 1

#define JX_NORM_NONE 0
#define JX_NORM_RMS 1         /* nn/norms.py:83-117 */
#define JX_NORM_GEMMA 2       /* models/gemma3.py:89-106 */
#define JX_NORM_LAYER 3       /* nn/norms.py:120-168 */

#define JX_EPI_STORE 0            /* out = dtype(acc) (+ bias)                              nn/linear.py:161-182 */
#define JX_EPI_RESID 1            /* out = dtype(dtype(acc) + res)                          models/llama.py:133,137 */
#define JX_EPI_GLU_SILU 2         /* out = dtype(silu(gate) * up), K128 output              models/llama.py:82-88 */
#define JX_EPI_GLU_GELU_TANH 3    /* out = dtype(gelu_tanh(gate) * up), K128 output         models/gemma3.py:80-86 */
#define JX_EPI_ACT_GELU_ERF 4     /* out = dtype(gelu_erf(acc + b))                         models/gpt_neox.py:75-80 */
#define JX_EPI_RESID2 5           /* out = dtype(dtype(acc + res2) + res)  (parallel resid.) models/gpt_neox.py:126-129 */
#define JX_EPI_STORE_F32 6        /* float out = acc + bias: a tensor-parallel partial sum, all-reduced in float32 */
#define JX_EPI_ACC_F32 7          /* float out += acc + bias (GPT-NeoX parallel residual partials)            */
#define JX_EPI_PUSH_F32 8         /* float acc + bias stored into every rank's receive slot (peer_* fields)   */

/* Fused epilogue of a projection.  Output column n of a plain output lives at out[m*ldo + n]; a K128
 * output (out_rp > 0) is the tiled layout described in jx_pack_k128. */
typedef struct jx_epilogue {
  int kind;
  int M;                 /* valid output rows */
  int N;                 /* valid output columns (GLU: F) */
  int pf_iters;          /* decode projections: see pf_w (0: no prefetch) */
  const void* bias;      /* per packed weight row, model dtype, or NULL */
  void* out;
  long long ldo;
  long long out_rp;      /* > 0: K128 output with this row padding */
  const void* res;       /* RESID/RESID2 residual (may alias out) */
  long long ldr;
  const void* res2;      /* RESID2 second addend */
  long long ldr2;
  /* Decode projections only (jx_linear_decode): once this call has issued its own weight loads, each
   * CTA prefetches into L2 the first pf_iters 128-wide K chunks that the same CTA of the NEXT decode
   * projection will read (its K128 weights pf_w [pf_np, pf_kp], same grid), so that call starts from L2
   * while this one finishes.  A cache hint only: results are unchanged.  No counterpart in the reference. */
  const void* pf_w;
  long long pf_np, pf_kp;
  int pf_rows;           /* set by the library: weight rows per block of the next call's kernel */
  int pf_grid;           /* set by the library: CTAs of the next call */
  /* JX_EPI_PUSH_F32 (tensor parallelism, decode projections): a row-parallel projection and its
   * all-reduce in one kernel.  Each finished block's float32 partial (M rows x 64 columns) is stored
   * over NVLink into this rank's receive slot of every rank's peer region, then the block's 64-column
   * units are flagged at every rank; a jx_norm with peer_recv set consumes the sum (no counterpart in the
   * reference, which all-reduces through XLA).  Offsets are bytes within every rank's region (layout
   * from jx_comm_layout); `ldo` gives the element index (row * ldo + column) inside the slot.  Calls
   * alternate between two sets of slots and flags by the parity of the push epoch, which the device
   * keeps, so captured CUDA graphs replay correctly whatever number of pushes a pass makes. */
  const void* peer_bases;      /* device array [peer_world] of the ranks' region bases, mapped here */
  long long peer_recv_off;     /* receive slots: slot (set s, source r) at + (s * peer_world + r) * peer_slot_bytes */
  long long peer_slot_bytes;
  long long peer_flag_off;     /* flags: [2 sets][256 units][8 sources] uint32 */
  long long peer_seq_off;      /* push epoch counter */
  int peer_rank, peer_world;
  /* Normalisation prologue (decode projections at M <= 16; pn_h != NULL): before the activations are
   * loaded, CTA m < M writes row m of the activation operand X (K128 layout) as the norm of row m of h
   * (jx_norm's kinds RMS / GEMMA / LAYER, no residual input), and every CTA waits for those rows: the
   * RMSNorm / LayerNorm of models/llama.py:133-137 and gpt_neox.py run in the projection's prologue
   * instead of a separate jx_norm launch.  pn_sync: [2 + 16] ints, zero-initialised once, shared by the
   * prologue calls on one stream ([0] epoch, [1] arrivals, [2 + m] row flags). */
  const void* pn_h;            /* [M, pn_ldh] model dtype (bf16) */
  long long pn_ldh;
  const void* pn_w;            /* [pn_d] */
  const void* pn_b;            /* [pn_d] (LayerNorm) or NULL */
  int* pn_sync;
  int pn_kind, pn_d;
  float pn_eps;
  int _pad1;
  /* Normalisation tail (the row-split decode projection, jx_set_decode_linear_impl 3 or chosen by shape;
   * tn_x != NULL, JX_ERR_UNSUPPORTED when another kernel would run): once every CTA has stored its output
   * columns of the residual stream (kind JX_EPI_STORE or JX_EPI_RESID, bf16, plain [M, ldo] output), the
   * last CTA to finish normalises the M rows of that output into the next projection's activation
   * operand tn_x (K128, tn_rp rows) with the arithmetic and summation order of jx_norm (kinds RMS /
   * GEMMA / LAYER, weights tn_w, bias tn_b, over the N columns; N % 256 == 0, N <= 8192): the RMSNorm
   * after a residual add of models/llama.py:133-137 without a separate launch.  tn_sync: one int,
   * zero-initialised once, self-resetting.  No counterpart in the reference. */
  void* tn_x;
  long long tn_rp;
  const void* tn_w;
  const void* tn_b;
  int* tn_sync;
  int tn_kind;
  float tn_eps;
} jx_epilogue;

/* Row-wise embedding gather / residual add / normalisation (one launch per call). */
typedef struct jx_norm_args {
  int M, d;
  float eps;
  int kind;              /* JX_NORM_* of the main norm */
  int kind_pre;          /* JX_NORM_* applied to `a` before it is added into h (NONE: plain add) */
  int vocab;
  const int* ids;        /* embedding ids [M] or NULL */
  const void* table;     /* embedding table [vocab, d] */
  float embed_scale;     /* multiply gathered rows by this (0: none) */
  int a_f32;             /* `a` is float32 (an all-reduced partial sum): round it to the model dtype first */
  const int* row_map;    /* read h[row_map[m]] instead of h[m] (no write back) */
  const void* a;
  long long lda;
  void* h;
  long long ldh;
  const void* w_pre;
  const void* b_pre;
  const void* w;
  const void* b;
  void* out;
  long long ldo, out_rp;
  const void* w2;
  const void* b2;
  void* out2;
  long long ldo2, out2_rp;
  int* status;
  /* Tensor parallelism, push mode (peer_recv set): `a` is the rank-order sum of the float32 partials that
   * the row-parallel projection (JX_EPI_PUSH_F32) stored into this rank's receive slots; the kernel
   * first waits, bounded, for the flags of every 64-column unit from every rank, and its last CTA
   * advances the push epoch.  bfloat16 models with d / 8 a multiple of 32 (the vectorised kernel). */
  const void* peer_recv;       /* this rank's receive slots: [2 sets][peer_world sources][peer_stride floats] */
  long long peer_stride;
  const unsigned* peer_flags;  /* this rank's push flags: [2 sets][256 units][8 sources] */
  unsigned* peer_seq;          /* this rank's push epoch counter ([0] epoch, [1] finished CTAs) */
  int peer_world, peer_units;
} jx_norm_args;

typedef struct jx_qkv_args {
  int M, S;              /* token rows, tokens per sequence (rows are b*S + s) */
  int Hq, Hkv, hd, rd;   /* heads, head dim, rotary dim */
  const void* qkv;       /* [M, (Hq + 2 Hkv) hd] projection output */
  long long ld_qkv;
  const void* qn_w;      /* [hd] QK-norm weights (Gemma3) or NULL */
  const void* kn_w;
  float eps;
  int max_pos;           /* rows of the rotary tables */
  const void* cos;       /* [max_pos, rd] in the model dtype */
  const void* sin;
  const int* pos_id;     /* decode: [B] last valid cache slot */
  int decode;
  int T;                 /* cache slots */
  void* q_out;           /* [M, Hq, hd] */
  void* k_cache;         /* [B, T, Hkv, hd] */
  void* v_cache;
  int* status;
} jx_qkv_args;

typedef struct jx_attn_args {
  int B, S, Hq, Hkv, hd;
  int T;                 /* key slots in the cache buffer */
  const void* q;         /* [B*S, Hq, hd] */
  const void* k;         /* [B, T, Hkv, hd] */
  const void* v;
  const int* len_ptr;    /* [B]: keys j < len_ptr[b] + len_add are valid (prefix mask) */
  int len_add;
  int causal;            /* 1 for prefill with S > 1 */
  int window;            /* sliding window, 0 = none */
  float scale;           /* attn_scale (rounded to the model dtype inside) */
  void* out;             /* [B*S, Hq*hd]; K128 when out_rp > 0 */
  long long ldo, out_rp;
  int* status;
  void* weights;         /* optional [B, Hq, S, T] softmax probabilities in the dtype (output_attentions), or NULL */
  int uniform_T;         /* slots a query row with no visible key attends over, uniformly (0 = T) */
  int _pad1;
} jx_attn_args;

/* Standalone rotary embedding: q [M, Hq, hd] and k [M, Hk, hd] rows at positions pos[M] (outputs may
 * alias the inputs). */
typedef struct jx_rope_args {
  int M;                 /* token rows */
  int Hq, Hk, hd, rd;    /* heads of q and of k, head dim (<= 256), rotary dim (even, <= hd) */
  int n_pos;             /* rows of the cos / sin tables; a position outside [0, n_pos) -> JX_ERR_RANGE */
  const void* q;
  const void* k;
  void* q_out;
  void* k_out;
  const void* cos;       /* [n_pos, rd] in the dtype of q and k */
  const void* sin;
  const int* pos;        /* [M] */
  int* status;
} jx_rope_args;

/* Decode attention on tensor cores: one query token per batch row, head_dim 64/128/256, n_rep <= 16. */
typedef struct jx_dattn_args {
  int B, Hq, Hkv, hd;
  int T;                 /* cache slots per row */
  int window;            /* sliding window, 0 = none */
  long long cache_rows;  /* rows of the whole cache allocation viewed as [cache_rows, Hkv*hd] */
  long long layer_row0;  /* first row of this layer (layer * B * T) */
  const void* q;         /* [B, Hq, hd] */
  const void* k_base;    /* cache allocation base (row 0) */
  const void* v_base;
  const int* len_ptr;    /* [B]: valid keys = len_ptr[b] + len_add */
  int len_add;
  float scale;
  void* out;             /* K128 output [out_rp rows, Hq*hd] */
  long long out_rp;
  void* ws;              /* scratch, jx_decode_attention_workspace bytes */
  long long ws_bytes;
  int* counters;         /* [B * Hkv], zero-initialised once, self-resetting */
  int* status;
  /* RoPE and the cache append fused in (qkv != NULL; the split form only, no QK norm): q and this
   * step's k and v are read unrotated from the fused projection output, q and k are rotated on their
   * first rd dims like jx_qkv_rope_append (rotate_half, in bf16), and k and v are written into the
   * cache at position len_ptr[b] + len_add - 1 (JX_ERR_RANGE beyond max_pos); `q` is then unused. */
  const void* qkv;       /* [B, ld_qkv] bf16: Hq q heads, Hkv k heads, Hkv v heads of hd each */
  long long ld_qkv;
  const void* cos;       /* [max_pos, rd] bf16 */
  const void* sin;
  int rd, max_pos;
} jx_dattn_args;

/* Prefill attention on tensor cores: S query tokens per row (rows b*S + s), head_dim 64/128/256. */
typedef struct jx_pattn_args {
  int B, S, Hq, Hkv, hd;
  int T;                 /* cache slots per row (S <= T) */
  int window;            /* sliding window, 0 = none */
  int uniform_T;         /* slots a query row with no visible key attends over, uniformly (0 = T): the
                            reference's cache length when the prompt ran (engine.py:543-557) */
  long long cache_rows;  /* rows of the whole cache allocation viewed as [cache_rows, Hkv*hd] */
  long long layer_row0;  /* first row of this layer (layer * B * T) */
  const void* q;         /* [B*S, Hq, hd] */
  const void* k_base;
  const void* v_base;
  const int* len_ptr;    /* [B]: valid keys = len_ptr[b] + len_add (right-padded prompt mask) */
  int len_add;
  float scale;
  void* out;             /* K128 output [out_rp rows, Hq*hd] */
  long long out_rp;
  int* status;
} jx_pattn_args;

typedef struct jx_sample_args {
  int B, V;              /* rows, local vocabulary columns */
  const void* logits;
  long long ld;
  int dtype;
  int greedy;
  float temp;
  int chunk;             /* columns per CTA */
  long long vocab_offset;
  long long vocab_total;
  unsigned int* rng;     /* [4] device: key[2], subkey[2] */
  const float* gumbel_tab; /* [256] bfloat16 Gumbel values (as float) */
  unsigned long long* ws;  /* [B * ceil(V/chunk)] */
  unsigned long long* row_best; /* [B] when finalize == 0 */
  int* counters;         /* [B + 1], zero-initialised once */
  int finalize;
  int ld_tok;
  int* tokens_out;       /* [B, ld_tok], column = *step */
  int* step;
  int* next_ids;         /* [B] */
  int* pos_id;           /* [B] */
  unsigned char* mask;   /* [B, T_mask] */
  int T_mask;
  int update_pos;
  int advance_rng;
  int _pad0;
  int* status;
} jx_sample_args;

typedef struct jx_filter_args {
  int B, V;              /* rows, vocabulary columns (V <= 393216) */
  const void* logits;    /* [B, ld_in] */
  long long ld_in;
  void* out;             /* [B, ld_out]; may alias logits */
  long long ld_out;
  int dtype;             /* JX_F32 or JX_BF16 */
  int top_k;             /* <= 0: off */
  float top_p;           /* >= 1: off */
  float min_p;           /* <= 0: off */
} jx_filter_args;

/* ---- library ---- */
const char* jx_version(void);
const char* jx_last_error(void);
int jx_device_sm_count(int* out);

/* ---- layout ----
 * K128 tiled layout of a [rows, cols] matrix padded to [rp, cp] (rp % 8 == 0, cp % 128 == 0):
 * element (r, k) at ((k/128)*(rp/8) + r/8)*1024 + ((k%128)/8)*64 + (r%8)*8 + k%8.
 * Packs the reference's DenseGeneral kernels ([in, out], nn/linear.py:150-157) and activations into the
 * operand layout of the projection kernels.  transposed = 1 reads src as [cols, rows] (kernel layout). */
int jx_pack_k128(const void* src, int src_dtype, long long rows, long long cols, long long src_ld, int transposed,
                 void* dst, long long rp, long long cp, void* stream);
int jx_unpack_k128(const void* src, long long rows, long long cols, long long rp, void* dst, int dst_dtype,
                   long long dst_ld, void* stream);

/* ---- compute ---- */
/* Embed (nn/embedding.py:60-111) + residual add + RMSNorm/LayerNorm (nn/norms.py:83-168, gemma3.py:89-106). */
int jx_norm(const jx_norm_args* args, int dtype, int pdl, void* stream);

/* Decode projection (M <= 64): DenseGeneral (nn/linear.py:119-182) with fused epilogue.  W and X are
 * bfloat16 K128 ([Np, Kp] and [16*ceil(M/16) (or 64), Kp]); workspace from jx_linear_decode_workspace. */
int jx_linear_decode_workspace(int grid, int M, long long* floats_out);
/* Kernel behind jx_linear_decode: 0 = by shape (default: tcgen05/TMEM when Np/128 >= grid or when M > 16
 * and Kp >= 8192; else the row split where it applies; else mma.sync stream-K), 1 = mma.sync,
 * 2 = tcgen05/TMEM (needs Np % 128 == 0), 3 = row split (M <= 16: each CTA takes 32 or 48 output rows over
 * the whole K, so no split-K partials; needs a grid of at most `grid` CTAs, an element-wise bf16 epilogue
 * (not the float32 partial sums of tensor parallelism) and no prologue / prefetch; JX_ERR_SHAPE otherwise). */
int jx_set_decode_linear_impl(int impl);
int jx_linear_decode(const void* W, const void* X, long long Np, long long Kp, int M, const jx_epilogue* epi,
                     float* ws, long long ws_floats, int* counters, int* status, int grid, int pdl, void* stream);

/* jx_linear_decode for callers that cannot allocate device memory (no counterpart in the reference):
 * for example a handler running inside a host framework's custom-call / FFI hook, which may only use
 * the buffers it is handed, or a plugin that must not call cudaMalloc.  The split-K scratch is a
 * fixed array compiled into this library (2.3 MiB of every GPU that loads it, until exit), so the
 * sizes are capped: M <= 16 token rows, Np <= 262080 weight rows, grid <= 148 CTAs (grid <= 0 means 148);
 * larger requests fail with JX_ERR_SHAPE.  The first call on a device looks the array's address up (make
 * it before any stream capture).  Every call clears the array's arrival counters with a stream operation
 * ahead of the kernel, so pdl gives no overlap with the preceding kernel here.  All calls share the
 * array: calls that overlap on the GPU race and must not. */
int jx_linear_decode_noalloc(const void* W, const void* X, long long Np, long long Kp, int M, const jx_epilogue* epi,
                             int* status, int grid, int pdl, void* stream);

/* Prefill projection (any M): bfloat16 K128 operands X [Mp, Kp], W [Np, Kp] (Mp, Np multiples of 128). */
int jx_linear_prefill(const void* X, const void* W, long long Mp, long long Np, long long Kp, const jx_epilogue* epi,
                      int* status, int pdl, void* stream);
/* Kernel behind jx_linear_prefill: 0 = by shape (default: tcgen05/TMEM whenever the shape allows),
 * 1 = mma.sync, 2 = tcgen05/TMEM (JX_ERR_SHAPE when the shape does not allow it). */
int jx_set_prefill_linear_impl(int impl);

/* Tile order of the tcgen05 prefill projection (process-wide): gm > 0 runs the tiles of gm 256-token
 * blocks x all weight blocks before the next gm token blocks; 0 = token blocks fastest over the grid. */
int jx_set_prefill_tile_group(int gm);

/* float32 projection: X [M, K] (row stride ldx) times the reference's kernel layout W [K, N]. */
int jx_linear_f32(const float* X, long long ldx, const float* W, int M, int N, int K, const jx_epilogue* epi, int pdl,
                  void* stream);

/* QK-norm + RoPE (nn/position.py:78-141) + KV-cache append (cache.py:183-243). */
int jx_qkv_rope_append(const jx_qkv_args* args, int dtype, int pdl, void* stream);

/* RotaryEmbedding.apply_rotary_pos_emb (nn/position.py:78-141) for any positions. */
int jx_rope_apply(const jx_rope_args* args, int dtype, int pdl, void* stream);

/* Element-wise MLP activation on separate projection outputs [M, F] (leading dims ldg / ldu / ldo):
 * kind JX_EPI_GLU_SILU / JX_EPI_GLU_GELU_TANH: out = dtype(dtype(act(gate)) * up) (models/llama.py:90-95,
 * models/gemma3.py:85-90); JX_EPI_ACT_GELU_ERF: out = dtype(gelu_erf(gate)), up unused
 * (models/gpt_neox.py:84-88).  dtype JX_F32 or JX_BF16. */
int jx_mlp_act(const void* gate, long long ldg, const void* up, long long ldu, void* out, long long ldo, long long M,
               long long F, int kind, int dtype, int pdl, void* stream);

/* Attention.mha (nn/attention.py:321-400) on the cache, any head size (CUDA cores). */
int jx_attention(const jx_attn_args* args, int dtype, int pdl, void* stream);

/* Attention.mha decode branch (nn/attention.py:321-400) for bf16 caches on tensor cores: split over
 * the valid keys, TMA-staged K/V tiles, exact reference rounding (see csrc/attention_decode.cu).
 * With pdl = 1 the kernel loads the keys of earlier positions before waiting on the kernel launched
 * just before it on the stream, so that kernel must release its dependents only after its own wait
 * (jx_qkv_rope_append does); otherwise pass pdl = 0. */
int jx_decode_attention_workspace(int B, int Hq, int hd, int T, int window, long long* bytes_out);
int jx_decode_attention(const jx_dattn_args* args, int pdl, void* stream);
/* Form behind jx_decode_attention: 0 = by shape (default: the two-kernel split form), 1 = split scores
 * + split pv,
 * 2 = the single-pass thread-block-cluster form (key range (T, or the window) up to 8 CTAs x 2048 keys;
 * JX_ERR_SHAPE otherwise), 3 = split scores + column pv, 4 = the cluster-split form (one kernel, the
 * key splits of a head group in one thread-block cluster; up to 16 splits of 128 keys, JX_ERR_SHAPE
 * otherwise), 5 = the queue form (the split form's score and pv work as one persistent kernel whose CTAs
 * claim items from a counter in the workspace; outputs bit-identical to the split form). */
int jx_set_decode_attention_impl(int impl);

/* Attention.mha prefill branch (causal + window + padding masks, nn/attention.py:321-400) for bf16
 * caches on tensor cores, exact reference rounding (see csrc/attention_prefill.cu). */
int jx_prefill_attention(const jx_pattn_args* args, int pdl, void* stream);
/* Kernel behind jx_prefill_attention (process-wide): 0 = by shape (the mma.sync kernel), 1 = mma.sync
 * (csrc/attention_prefill.cu), 2 = tcgen05/TMEM (csrc/attention_prefill_tc.cu: head_dim 64 / 128 / 256, a
 * K128 output; JX_ERR_SHAPE otherwise; not yet the by-shape choice). */
int jx_set_prefill_attention_impl(int impl);

/* greedy_fn / categorical sampling (inference_engine/sampling.py:75-188) + end-of-step bookkeeping. */
int jx_sample(const jx_sample_args* args, int pdl, void* stream);
int jx_sample_finalize(const jx_sample_args* args, const unsigned long long* gathered, int n_shards, void* stream);

/* min_p_filtering, then top_k_filtering, then top_p_filtering (inference_engine/sampling.py:34-75, order
 * :169-188) of full-vocabulary rows, filtered entries -inf: probabilities in float32 rounded to the logits'
 * dtype, ties at the top-k cutoff kept, the top-p cutoff from exact (fixed-point) cumulative masses.  One
 * thread-block cluster per row (see csrc/filter.cu). */
int jx_filter_logits(const jx_filter_args* args, void* stream);

/* Clear the split-K counters after an error (they are self-resetting otherwise). */
int jx_memset_async(void* ptr, int value, long long bytes, void* stream);

/* ---- one decode step of a Llama-family stack in one persistent kernel ----
 * Replaces, for one token per row, the whole of LlamaModelWithHead.__call__ with a populated cache
 * (models/llama.py:112-143 per layer: input RMSNorm, q/k/v projections, RoPE (nn/position.py:78-141),
 * cache append (cache.py:183-243), Attention.mha decode branch (nn/attention.py:321-400), o_proj +
 * residual, post-attention RMSNorm, SwiGLU MLP (models/llama.py:82-88) + residual; then the final norm
 * and lm_head, models/llama.py:245-273), with the reference's bf16 rounding points.  One cooperative
 * launch of one CTA per SM runs every layer: the weights of the next phase stream into shared memory
 * while the current phase finishes, and the phases are separated by grid-wide barriers (bounded waits:
 * JX_ERR_TIMEOUT in *status).  Embedding rows are gathered from ids[M]; logits [M, V] bf16 are left for
 * jx_sample.  Requirements: bf16, head_dim 128, M <= 16, Hq / Hkv <= 16, no sliding window, rd % 16 == 0,
 * weights in the K128 layout (the gate/up rows interleaved in groups of 32, as for JX_EPI_GLU_SILU),
 * activations h [M, d] row-major and xn / attn / act in the K128 layout with 16 padded rows. */
typedef struct jx_step_args {
  int M, L;                  /* token rows (<= 16), layers */
  int d, Hq, Hkv, hd;        /* hidden size, heads, head size (128) */
  int F, V, vocab;           /* intermediate size, lm_head columns, embedding rows */
  int T, rd, max_pos;        /* cache slots per row, rotary dims, rows of the cos / sin tables */
  long long Np_qkv, Np_d, Np_gu, Np_v, Kp_d, Kp_o, Kp_f;   /* padded K128 extents */
  float eps, scale;          /* RMSNorm epsilon, attention scale */
  const void* layers;        /* device array of L x 6 pointers: wqkv, wo, wgu, wd, input / post-attention norm weights */
  const void* embed;         /* [vocab, d] */
  const int* ids;            /* [M] this step's token ids */
  const void* final_norm;    /* [d] */
  const void* lm_head;       /* K128 [Np_v, Kp_d] */
  void* h;                   /* residual stream [M, d] (rows 0..M-1) */
  void* xn;                  /* normalised activations, K128 [16, Kp_d] */
  void* qkv;                 /* fused projection output [M, (Hq + 2 Hkv) hd] */
  void* attn;                /* attention output, K128 [16, Kp_o] */
  void* act;                 /* GLU product, K128 [16, Kp_f] */
  void* logits;              /* [M, V] */
  void* k_cache, *v_cache;   /* [L, M, T, Hkv, hd] */
  const void* cos, *sin;     /* [max_pos, rd] */
  const int* pos_id;         /* [M]: this step writes position pos_id + 1 */
  float* ws;                 /* split-K partial tiles, >= grid x 2 x 16 x 128 floats */
  long long ws_floats;
  int* counters;             /* >= Np_v / 128 + 1 ints, zero (left zero) */
  void* attn_ws;             /* jx_decode_attention_workspace(M, Hq, 128, T, 0) bytes */
  long long attn_ws_bytes;
  int* attn_counters;        /* [M x Hkv] ints, zero (left zero) */
  int* sync;                 /* 6 ints: grid barrier counter, abort flag, where a bounded wait gave up (cleared by the call) */
  int* status;
  int grid;                  /* CTAs (<= 0: one per SM) */
} jx_step_args;
int jx_decode_step(const jx_step_args* args, void* stream);
/* L2 lookahead of jx_decode_step (process-wide): each CTA prefetches into L2 the weight tiles of its next
 * `stages` projection stages (32 KB each) beyond those in shared memory, across phase boundaries, so HBM
 * keeps streaming while the step waits at grid barriers and in the attention phase.  0 (the default)
 * disables it: on the Llama-3-8B decode step every depth tried made the step slower.  A
 * cache hint only: results are unchanged.  No counterpart in the reference. */
int jx_set_decode_step_lookahead(int stages);

/* ---- tensor parallelism over NVLink peer memory ----
 * The reference all-reduces the row-parallel o_proj / down_proj outputs through XLA's GSPMD collectives
 * (inference_engine/engine.py:258-267 sharding rules, models/llama.py:133-137 residual adds); these
 * calls replace that collective for decode-sized messages.  Each rank allocates one region with
 * jx_comm_alloc (layout from jx_comm_layout), shares it with jx_ipc_get_handle (64-byte handle,
 * exchanged by the caller), maps the other ranks' regions with jx_ipc_open_handle and writes the table
 * of mapped bases into its own region (base_table offset).  Two forms:
 *   - jx_allreduce_f32: sums the first n floats of partials buffer `which` of every region in rank order
 *     into `out` (every rank gets bit-identical values);
 *   - the push form: a decode projection with JX_EPI_PUSH_F32 followed by a jx_norm with peer_recv set.
 * Consecutive calls (of either form) alternate `which`; all ranks make the same sequence of calls; every
 * device wait is bounded (JX_ERR_TIMEOUT in *status).
 * jx_comm_layout fills out10: [0] region bytes, [1] / [2] all-reduce buffers 0 / 1, [3] push receive
 * slots (+ (which * world + source) * [4]), [4] receive slot stride, [5] push flags (+ which * [6]),
 * [6] flags bytes per call, [7] push epoch counter, [8] base table, [9] units per call at most. */
int jx_comm_alloc(long long bytes, void** ptr_out);
int jx_comm_free(void* ptr);
int jx_ipc_get_handle(const void* ptr, unsigned char* handle_out);
int jx_ipc_open_handle(const unsigned char* handle, void** ptr_out);
int jx_ipc_close_handle(void* ptr);
int jx_comm_layout(long long max_floats, int world, long long* out10);
int jx_allreduce_f32(void* const* bases, int rank, int world, long long max_floats, int which, long long n,
                     float* out, int* status, int pdl, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* JXB200_H_ */
