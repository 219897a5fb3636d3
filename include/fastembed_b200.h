/*
 * fastembed_b200.h — C ABI of the B200 (sm_100a) encoder forward path.
 *
 * Drop-in boundary for fastEmbed's op classes and model runtime.  The reference
 * has no C ABI: its boundary is the C++ classes CUDAMatrixOps
 * (include/ops/cuda/cuda_matrix_ops.h:4-45), CUDAAttentionOps
 * (include/ops/cuda/cuda_attention_ops.cuh:6-22) and SentenceTransformer
 * (include/sentence_transformers.h:12-40).  Each entry point below names the
 * reference routine it replaces.  The C++ classes of the same names in this
 * repository (the headers under include/ops/cuda and include/sentence_transformers.h) are thin
 * wrappers over these functions.
 *
 * Conventions
 *   - Plain pointers and sizes only.  "device" pointers are CUDA device memory
 *     owned by the caller; "host" pointers are ordinary host memory.
 *   - Op entry points (fe_* without _engine) are stream-ordered, allocate nothing
 *     and do not synchronise; the stream is a cudaStream_t (NULL = default).
 *   - Every call returns an fe_status; fe_last_error_message() gives the detail
 *     for the calling thread.  Nothing here calls exit() (the reference's matrix
 *     ops do, src/ops/cuda/cuda_matrix_ops.cu:13-19).
 *   - Device-side waits are bounded: a kernel whose wait runs out records
 *     FE_ERR_DEVICE_TIMEOUT in a per-device status word and returns; read it with
 *     fe_device_status().
 */
#ifndef FASTEMBED_B200_H
#define FASTEMBED_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *fe_stream_t; /* identical to cudaStream_t */

typedef enum fe_status {
    FE_OK = 0,
    FE_ERR_INVALID_ARGUMENT = 1, /* reference: std::invalid_argument */
    FE_ERR_CUDA = 2,             /* reference: std::runtime_error from CUDA calls */
    FE_ERR_OUT_OF_MEMORY = 3,
    FE_ERR_UNSUPPORTED = 4,      /* shape or device this build does not handle */
    FE_ERR_DEVICE_TIMEOUT = 5,   /* a bounded device-side wait ran out */
    FE_ERR_IO = 6,               /* file missing or malformed */
    FE_ERR_NOT_FOUND = 7         /* unknown tensor name */
} fe_status;

/* Epilogues fused into the tensor-core linear layer. */
typedef enum fe_epilogue {
    FE_EPI_NONE = 0,          /* y = x W^T                          */
    FE_EPI_BIAS = 1,          /* y = x W^T + b                      */
    FE_EPI_BIAS_GELU = 2,     /* y = gelu_tanh(x W^T + b)           */
    FE_EPI_BIAS_RELU = 3,     /* y = relu(x W^T + b)                */
    FE_EPI_BIAS_SWISH = 4,    /* y = swish(x W^T + b)               */
    FE_EPI_BIAS_RESIDUAL = 5, /* y = x W^T + b + residual (fp32)    */
    /* Gated MLP (not in the reference; Qwen3 / Gemma3 shapes): W has n rows that
     * alternate 32 gate rows and 32 up rows; y has n/2 columns, bf16, y = act(x Wg^T) * (x Wu^T)
     * with act = silu or gelu_tanh; no bias.  n % 128 == 0. */
    FE_EPI_SWIGLU = 6,
    FE_EPI_GEGLU = 7
} fe_epilogue;

typedef enum fe_dtype { FE_DTYPE_F32 = 0, FE_DTYPE_BF16 = 1 } fe_dtype;

typedef enum fe_pooling {
    FE_POOL_CLS = 0,  /* first token of each sentence (src/sentence_transformers_impl.cpp:289-290) */
    FE_POOL_MEAN = 1, /* mean over valid tokens */
    FE_POOL_LAST = 2  /* last valid token */
} fe_pooling;

typedef enum fe_activation { FE_ACT_GELU = 0, FE_ACT_RELU = 1, FE_ACT_SWISH = 2 } fe_activation;

/* ---------------------------------------------------------------- status */
const char *fe_status_string(fe_status s);
/* Detail of the last failing call on this thread ("" if none). */
const char *fe_last_error_message(void);
/* Synchronises `device` and returns (then clears) its device-side status word:
 * FE_OK, or FE_ERR_DEVICE_TIMEOUT when a kernel's bounded wait ran out.  The word and
 * the library's other per-device state (scratch and counter addresses, kernel
 * attributes) belong to the device's current CUDA context and are set up again in a
 * new one: a device may be reset (cudaDeviceReset) while no call of this library is in
 * flight on it. */
fe_status fe_device_status(int device);
/* Sets the limit, in nanoseconds, of the device-side waits that guard work (a TMA stage,
 * a TMEM accumulator, another CTA's row statistics) in every tcgen05 kernel launched on
 * `device` from now on; default 2,000,000,000 (2 s).  A wait that runs out makes its
 * kernel record FE_ERR_DEVICE_TIMEOUT, let its own in-flight copies and MMAs land (those
 * drain waits keep the 2 s limit), free its TMEM and return.  Limits under 1 ms are
 * checked at every poll.  Call it with no kernel of this library running on the device.
 * The reference has no counterpart: its CUDA ops exit() on a CUDA error
 * (src/ops/cuda/cuda_matrix_ops.cu:13-19).  limit_ns must be > 0. */
fe_status fe_set_wait_limit(int device, uint64_t limit_ns);
/* Library version string. */
const char *fe_version(void);

/* ------------------------------------------- FP32 ops (legacy op API) ---
 * Accurate FP32 SIMT kernels behind CUDAMatrixOps / CUDAAttentionOps, which
 * the reference's GTests compare against the CPU ops at 1e-5 / 1e-3 absolute. */

/* C[m,k] = A[m,n] · B[n,k].  Replaces CUDAMatrixOps::matrix_multiply
 * (include/ops/cuda/cuda_matrix_ops.h:7-8, src/ops/cuda/cuda_matrix_ops.cu:192-219). */
fe_status fe_sgemm_nn(const float *a, const float *b, float *c, int64_t m, int64_t n, int64_t k,
                      fe_stream_t stream);
/* C[m,k] = A[m,n] · B[k,n]^T (+ bias[k] when bias != NULL).  Replaces
 * CUDAMatrixOps::matrix_multiply_transpose (cuda_matrix_ops.h:10-11, .cu:221-248). */
fe_status fe_sgemm_nt(const float *a, const float *b, const float *bias, float *c, int64_t m,
                      int64_t n, int64_t k, fe_stream_t stream);
/* Elementwise activations.  Replace CUDAMatrixOps::gelu / relu / swish
 * (cuda_matrix_ops.h:13-16, .cu:250-305); GELU is the tanh form. */
fe_status fe_gelu_f32(const float *x, float *y, int64_t count, fe_stream_t stream);
fe_status fe_relu_f32(const float *x, float *y, int64_t count, fe_stream_t stream);
fe_status fe_swish_f32(const float *x, float *y, int64_t count, fe_stream_t stream);
/* Row LayerNorm over `dim`, any dim >= 1.  Replaces CUDAMatrixOps::layer_norm
 * (cuda_matrix_ops.h:18-22, .cu:307-362; the reference kernel needs dim <= 1024). */
fe_status fe_layer_norm_f32(const float *x, const float *gamma, const float *beta, float *y,
                            int64_t rows, int64_t dim, float eps, fe_stream_t stream);
/* Row RMSNorm.  Replaces CUDAMatrixOps::rms_norm (cuda_matrix_ops.h:24-27, .cu:464-520). */
fe_status fe_rms_norm_f32(const float *x, const float *weight, float *y, int64_t rows,
                          int64_t dim, float eps, fe_stream_t stream);
/* Row softmax, any dim.  Replaces CUDAMatrixOps::softmax(axis = 1)
 * (cuda_matrix_ops.h:29, .cu:364-389). */
fe_status fe_softmax_rows_f32(const float *x, float *y, int64_t rows, int64_t dim,
                              fe_stream_t stream);
/* In-place softmax over the last axis of [heads, seq_len, seq_len] device scores.
 * Replaces CUDAMatrixOps::apply_softmax (cuda_matrix_ops.h:32, .cu:417-422). */
fe_status fe_softmax_scores_inplace_f32(float *scores, int64_t heads, int64_t seq_len,
                                        fe_stream_t stream);
/* Bytes of device workspace fe_mha_f32 needs. */
size_t fe_mha_f32_workspace_bytes(int64_t seq_len, int64_t dim, int64_t heads);
/* Single-sequence MHA: Q,K,V = X·W^T + b, per head softmax(Q K^T / sqrt(hd)) V,
 * heads concatenated.  Replaces CUDAAttentionOps::multi_head_attention
 * (include/ops/cuda/cuda_attention_ops.cuh:10-20, src/ops/cuda/cuda_attention_ops.cu:164-342). */
fe_status fe_mha_f32(const float *x, const float *wq, const float *wk, const float *wv,
                     const float *bq, const float *bk, const float *bv, float *out,
                     int64_t seq_len, int64_t dim, int64_t heads, void *workspace,
                     size_t workspace_bytes, fe_stream_t stream);
/* fe_mha_f32 without a workspace argument and without allocating: Q, K and V live in
 * a fixed 3 MiB scratch array inside the library (one per device, kept until process
 * exit), for callers that cannot allocate device memory on demand.  No counterpart in
 * the reference (its attention op allocates per call).  Requires seq_len * dim <=
 * 262144 (FE_ERR_UNSUPPORTED otherwise).  All calls on a device share the scratch, so
 * calls whose GPU work overlaps race; order them on one stream.  The first call on a
 * device looks up the scratch address and should precede any stream capture. */
fe_status fe_mha_f32_noalloc(const float *x, const float *wq, const float *wk, const float *wv,
                             const float *bq, const float *bk, const float *bv, float *out,
                             int64_t seq_len, int64_t dim, int64_t heads, fe_stream_t stream);

/* ----------------------------------- BF16 tensor-core hot-path ops -----
 * tcgen05 (TMEM accumulator, TMA-fed) kernels of the model pipeline. */

/* y[m,n] = epilogue(x[m,k] · w[n,k]^T): bf16 x and w (nn.Linear layout), FP32
 * accumulation, fused bias / activation / residual; y is bf16 or fp32 (the
 * residual form writes fp32).  Requires k % 8 == 0, n % 8 == 0, 16-byte aligned
 * pointers.  Replaces the model's matrix_multiply_transpose calls plus their host
 * bias / activation / residual loops (src/sentence_transformers_impl.cpp:250-263,
 * :403-436). */
fe_status fe_linear_bf16(const void *x, const void *w, const float *bias, const float *residual,
                         void *y, int64_t m, int64_t n, int64_t k, fe_epilogue epilogue,
                         fe_dtype y_dtype, fe_stream_t stream);
/* Variable-length bidirectional attention over a packed batch.  qkv is bf16
 * [total_tokens, 3*heads*head_dim] (Q | K | V column blocks, head h at h*head_dim);
 * cu_seqlens (device, int32 [batch+1]) are sentence offsets; out is bf16
 * [total_tokens, heads*head_dim].  Keys past a sentence's end are masked, which is
 * the unpadded per-sentence attention of src/ops/cpu/cpu_attention_ops.cpp:33-85.
 * head_dim must be 64; max_len <= 4096. */
fe_status fe_attention_varlen_bf16(const void *qkv, const int32_t *cu_seqlens, int32_t batch,
                                   int32_t max_len, int32_t heads, int32_t head_dim, void *out,
                                   int64_t total_tokens, fe_stream_t stream);
/* Grouped-query variable-length attention for head_dim 128 or 256 (the Qwen3 and Gemma3
 * shapes; these models are not in the reference, whose attention is
 * src/ops/cpu/cpu_attention_ops.cpp:33-85 with one key-value head per query head).
 * qkv is bf16 [total_tokens, (q_heads + 2*kv_heads)*head_dim]: the query heads, then the
 * key heads, then the value heads; query head h reads key-value head
 * h / (q_heads / kv_heads).  out [total_tokens, q_heads*head_dim] bf16 =
 * softmax(Q K^T * scale) V per sentence; causal != 0 keeps key j for query i only when
 * j <= i.  Requires q_heads % kv_heads == 0. */
fe_status fe_attention_varlen_gqa_bf16(const void *qkv, const int32_t *cu_seqlens, int32_t batch, int32_t max_len,
                                       int32_t q_heads, int32_t kv_heads, int32_t head_dim, int32_t causal, float scale,
                                       void *out, int64_t total_tokens, fe_stream_t stream);
/* Fused embedding sum + LayerNorm over a packed batch: x_t = word[id_t] +
 * pos[t - start(s)] + type[0]; writes LN(x) as fp32 (h32) and bf16 (h16).
 * Replaces src/sentence_transformers_impl.cpp:30-44, :155-194.  Out-of-range ids
 * and positions set FE_ERR_INVALID_ARGUMENT in the device status word and write
 * zeros for that token. */
fe_status fe_embed_layernorm(const int32_t *ids, const int32_t *cu_seqlens, int32_t batch,
                             int64_t total_tokens, const float *word, const float *pos,
                             const float *type, const float *gamma, const float *beta,
                             int32_t dim, int32_t vocab, int32_t max_pos, float eps,
                             float *h32, void *h16, fe_stream_t stream);
/* The same with the bge-m3 / XLM-R position rows (FE_POSITIONS_XLMR above), replacing
 * the BGE_M3 branch of bge_forward's embedding (src/sentence_transformers_impl.cpp:139-155
 * with create_position_ids_from_input_ids, :101-123).  Requires pad_token_id >= 0. */
fe_status fe_embed_layernorm_xlmr(const int32_t *ids, const int32_t *cu_seqlens, int32_t batch,
                                  int64_t total_tokens, const float *word, const float *pos,
                                  const float *type, const float *gamma, const float *beta,
                                  int32_t dim, int32_t vocab, int32_t max_pos, int32_t pad_token_id,
                                  float eps, float *h32, void *h16, fe_stream_t stream);
/* h = LayerNorm(x + residual) (residual may be NULL) writing fp32 and (when
 * h16 != NULL) bf16 copies: the residual add and post-residual norms of
 * src/sentence_transformers_impl.cpp:255-266 and :429-437.  h32 may alias residual. */
fe_status fe_layernorm_dual(const float *x, const float *residual, const float *gamma, const float *beta,
                            float *h32, void *h16, int64_t rows, int32_t dim, float eps, fe_stream_t stream);
/* Projection, residual add and LayerNorm in one launch:
 *     h32 <- LayerNorm((x[m,k] · w[n,k]^T + bias) + h32) * gamma + beta   (in place)
 *     h16 <- bf16(h32)                                                  (when h16 != NULL)
 * The out-projection and FFN-down steps of a post-LN encoder layer, each with the
 * residual add and LayerNorm that follow it (src/sentence_transformers_impl.cpp:250-266
 * and :403-437; LayerNorm as in src/ops/cpu/cpu_matrix_ops.cpp:64-92).  Requires
 * k % 8 == 0 and n in {128, 256, 384, 512, 768, 1024, 1536, 2048}; 16-byte aligned
 * pointers.  `workspace` holds fe_linear_layernorm_workspace_bytes(m, n) bytes and
 * must be zero-filled before its first use; it then serves any number of calls, with
 * any m up to the one it was sized for.  Calls that share a workspace must not run
 * concurrently. */
/* Pre-norm RMSNorm form of the same step (Qwen3-shaped encoders; not in the reference):
 *     h32 <- (x[m,k] · w[n,k]^T + bias) + h32      (in place: the residual stream)
 *     h16 <- bf16(h32 / sqrt(mean(h32^2) + eps) * rms_w)   (the next layer input; may be NULL)
 * bias is required (zeros for models without one).  Workspace as above. */
fe_status fe_linear_rmsnorm_bf16(const void *x, const void *w, const float *bias, const float *rms_w, float *h32,
                                 void *h16, int64_t m, int64_t n, int64_t k, float eps, void *workspace,
                                 size_t workspace_bytes, fe_stream_t stream);
/* The same pre-norm step with the RMSNorm deferred to the next projection (Qwen3-shaped
 * encoders; not in the reference):
 *     h32 <- (x[m,k] · w[n,k]^T + bias) + h32                     (in place: the residual stream)
 *     h16 <- bf16(h32 * rms_w)                                     (may be NULL)
 *     row_ss[i][p] <- sum of h32[i][j]^2 over the p-th of fe_linear_rmsnorm_deferred_parts(n)
 *                     equal column ranges                          (fp32 [m][parts])
 * The next projection of h16 takes row_ss (fe_linear_row_scaled_bf16,
 * fe_linear_qk_norm_rope_scaled_bf16) and multiplies row i of its product by
 * 1 / sqrt(sum_p row_ss[i][p] / n + eps): the RMSNorm factor, applied after that GEMM, so
 * this step needs no exchange of row statistics between the CTAs of a row.  n a multiple
 * of 256 up to 2048, k % 8 == 0, bias required (zeros for models without one), 16-byte
 * aligned pointers, no workspace. */
fe_status fe_linear_rmsnorm_deferred_bf16(const void *x, const void *w, const float *bias, const float *rms_w,
                                          float *h32, void *h16, float *row_ss, int64_t m, int64_t n, int64_t k,
                                          fe_stream_t stream);
/* Partials per row of fe_linear_rmsnorm_deferred_bf16 for n columns (0 if n is unsupported). */
int32_t fe_linear_rmsnorm_deferred_parts(int64_t n);
/* fe_linear_bf16 on an input whose rows still need their RMSNorm factor: row i of
 * x · w^T is multiplied by 1 / sqrt(sum_p row_ss[i][p] / k + eps) before the epilogue
 * (row_ss [m][ss_parts], ss_parts 1..8, from fe_linear_rmsnorm_deferred_bf16 with n = k). */
fe_status fe_linear_row_scaled_bf16(const void *x, const void *w, const float *bias, const float *residual, void *y,
                                    int64_t m, int64_t n, int64_t k, fe_epilogue epilogue, fe_dtype y_dtype,
                                    const float *row_ss, int32_t ss_parts, float eps, fe_stream_t stream);
fe_status fe_linear_layernorm_workspace_bytes(int64_t m, int64_t n, size_t *bytes);
fe_status fe_linear_layernorm_bf16(const void *x, const void *w, const float *bias, const float *gamma,
                                   const float *beta, float *h32, void *h16, int64_t m, int64_t n, int64_t k,
                                   float eps, void *workspace, size_t workspace_bytes, fe_stream_t stream);
/* ---- RMSNorm / RoPE encoders (Qwen3, Gemma3 shapes; not in the reference) ----
 * dim in {256, 384, 512, 768, 1024, 1536, 2048}; one_plus != 0 uses (1 + w) as the
 * norm weight (Gemma3), else w (Qwen3).  All statistics in fp32. */
/* h32[t] = word[ids[t]] * scale (fp32 [total, dim]). */
fe_status fe_embed_scale(const int32_t *ids, int64_t total_tokens, const float *word, int32_t vocab, int32_t dim,
                         float scale, float *h32, fe_stream_t stream);
/* out = x / sqrt(mean(x^2) + eps) * w, written as fp32 (o32) and / or bf16 (o16). */
fe_status fe_rms_norm_rows(const float *x, const float *w, int32_t one_plus, float eps, int64_t rows, int32_t dim,
                           float *o32, void *o16, fe_stream_t stream);
/* h32 += RMSNorm(y; w_post), then out = RMSNorm(h32; w_next) as fp32 and / or bf16. */
/* fe_rms_sandwich with y in bf16 (a projection written in bf16, as the Gemma3-shaped
 * engine writes o_proj and down_proj): same arithmetic in fp32 after widening y. */
fe_status fe_rms_sandwich_bf16(const void *y, const float *w_post, float *h32, const float *w_next,
                               int32_t one_plus, float eps, int64_t rows, int32_t dim, float *o32, void *o16,
                               fe_stream_t stream);
fe_status fe_rms_sandwich(const float *y, const float *w_post, float *h32, const float *w_next, int32_t one_plus,
                          float eps, int64_t rows, int32_t dim, float *o32, void *o16, fe_stream_t stream);
/* The Qwen3 / Gemma3 QKV projection with its q/k norms and RoPE fused into the GEMM
 * epilogue: qkv [m, (q_heads + 2 kv_heads) * head_dim] bf16 = x [m, k] W^T ([N, k] bf16,
 * query | key | value rows, no bias), where each query and key head is RMS-normalised in
 * fp32 straight from the accumulator (weights q_w / k_w, or 1 + w when one_plus), then
 * rotated (rotate-half RoPE, inverse frequencies theta^(-2i/head_dim), position
 * positions[row]) before the single bf16 rounding; value heads are stored as they are.
 * Replaces fe_linear_bf16 followed by fe_qk_norm_rope_bf16 (one pass over qkv fewer).
 * head_dim 128 or 256; q_heads * head_dim and kv_heads * head_dim multiples of 256
 * (FE_ERR_UNSUPPORTED otherwise).  Not in the reference (no Qwen3 / Gemma forward). */
fe_status fe_linear_qk_norm_rope_bf16(const void *x, const void *w, const float *q_w, const float *k_w,
                                      const int32_t *positions, void *qkv, int64_t m, int64_t k, int32_t q_heads,
                                      int32_t kv_heads, int32_t head_dim, int32_t one_plus, float eps, float theta,
                                      fe_stream_t stream);
/* fe_linear_qk_norm_rope_bf16 on an input whose rows still need their RMSNorm factor
 * (row_ss, ss_parts as in fe_linear_row_scaled_bf16; the same eps for both norms). */
fe_status fe_linear_qk_norm_rope_scaled_bf16(const void *x, const void *w, const float *q_w, const float *k_w,
                                             const int32_t *positions, void *qkv, int64_t m, int64_t k,
                                             int32_t q_heads, int32_t kv_heads, int32_t head_dim, int32_t one_plus,
                                             float eps, float theta, const float *row_ss, int32_t ss_parts,
                                             fe_stream_t stream);
/* positions[t] = position of token t in its sentence (0, 1, ...) for the packed batch of
 * cu_seqlens [batch + 1]: the positions fe_linear_qk_norm_rope_bf16 reads. */
fe_status fe_token_positions(const int32_t *cu_seqlens, int32_t batch, int32_t *positions, fe_stream_t stream);
/* In place on qkv [total, (q_heads + 2*kv_heads)*head_dim] bf16: per-head RMSNorm of the
 * query (q_w) and key (k_w) heads, then the rotate-half rotary embedding with inverse
 * frequencies theta^(-2i/head_dim) at positions 0.. within each sentence.  head_dim 128 / 256. */
fe_status fe_qk_norm_rope_bf16(void *qkv, const int32_t *cu_seqlens, int32_t batch, int64_t total_tokens,
                               int32_t q_heads, int32_t kv_heads, int32_t head_dim, const float *q_w, const float *k_w,
                               int32_t one_plus, float eps, float theta, fe_stream_t stream);
/* Per-sentence pooling + L2 normalisation of packed hidden states h [total, dim]
 * into out [batch, dim].  Replaces src/sentence_transformers_impl.cpp:289-341. */
fe_status fe_pool_l2(const float *h, const int32_t *cu_seqlens, int32_t batch, int32_t dim,
                     fe_pooling mode, float *out, fe_stream_t stream);

/* --------------------------------------------------------- model engine
 * Device-resident post-LN BERT encoder (the reference's bge_forward,
 * src/sentence_transformers_impl.cpp:126-344, batched and packed). */
/* Position rows of the embedding (src/sentence_transformers_impl.cpp:139-163):
 *   FE_POSITIONS_BERT  token i of a sentence takes row i (model_type "bge" / "bert");
 *   FE_POSITIONS_XLMR  bge-m3 / XLM-R (model_type "bge-m3" / "xlm-roberta", :101-123,
 *                      :146-149): a token equal to pad_token_id takes row 0, the others
 *                      rows 2, 3, ... in order; a row at or past max_position becomes 0. */
typedef enum fe_positions { FE_POSITIONS_BERT = 0, FE_POSITIONS_XLMR = 1 } fe_positions;

typedef struct fe_encoder_config {
    int32_t vocab_size, hidden, layers, heads, intermediate, max_position, type_vocab;
    float layer_norm_eps;
    int32_t activation; /* fe_activation */
    int32_t pooling;    /* fe_pooling */
    int32_t positions;  /* fe_positions (0, the BERT rows, when zero-initialised) */
    int32_t pad_token_id; /* FE_POSITIONS_XLMR only: config.json pad_token_id (0 if absent, :141) */
} fe_encoder_config;

/* Pre-RMSNorm rotary encoders, the Qwen3 and Gemma3 shapes (not in the reference; the
 * forward follows the model definitions):
 *   FE_FAMILY_QWEN3   x <- x + Wo attn(rope(qknorm(Wqkv rms(x))), causal);
 *                     x <- x + Wd (silu(Wg rms(x)) * Wu rms(x)); final RMSNorm; w weights
 *   FE_FAMILY_GEMMA3  embeddings scaled by sqrt(hidden);
 *                     x <- x + rms(Wo attn(rope(qknorm(Wqkv rms(x)))), bidirectional);
 *                     x <- x + rms(Wd (gelu_tanh(Wg rms(x)) * Wu rms(x))); final RMSNorm;
 *                     (1 + w) weights; layers l with (l + 1) % full_attention_every == 0 use
 *                     rope_theta, the others rope_theta_local.
 * Weights by HF name (embed_tokens.weight, layers.N.self_attn.{q,k,v,o}_proj.weight,
 * layers.N.self_attn.{q,k}_norm.weight, layers.N.mlp.{gate,up,down}_proj.weight,
 * layers.N.{input,post_attention}_layernorm.weight, Gemma3 also
 * layers.N.{pre,post}_feedforward_layernorm.weight, norm.weight), with or without a
 * leading "model.". */
typedef enum fe_family { FE_FAMILY_BERT = 0, FE_FAMILY_QWEN3 = 1, FE_FAMILY_GEMMA3 = 2 } fe_family;

typedef struct fe_rms_encoder_config {
    int32_t family; /* FE_FAMILY_QWEN3 or FE_FAMILY_GEMMA3 */
    int32_t vocab_size, hidden, layers, q_heads, kv_heads, head_dim, intermediate, max_position;
    float rms_norm_eps;
    float rope_theta;             /* global-attention layers */
    float rope_theta_local;       /* sliding-window layers (Gemma3) */
    int32_t full_attention_every; /* Gemma3 layer pattern; 0: every layer uses rope_theta */
    float query_scale;            /* attention scale; 0: head_dim^-0.5 */
    int32_t pooling;              /* fe_pooling: FE_POOL_LAST (Qwen3), FE_POOL_MEAN (Gemma3) */
} fe_rms_encoder_config;

typedef struct fe_engine fe_engine;

typedef struct fe_engine_stats {
    int64_t launches;      /* kernels launched by the last encode call            */
    int64_t gemm_launches; /* of which tcgen05 linear-layer kernels               */
    int64_t tokens;        /* packed tokens of the last encode call               */
    double gemm_ms;        /* summed device time of the linear-layer kernels      */
    double attention_ms;   /* summed device time of the attention kernels         */
    double other_ms;       /* summed device time of the memory-bound kernels      */
    double gemm_flops;     /* algorithmic FLOPs of the linear layers (valid rows) */
    double attention_flops;/* algorithmic FLOPs of QK^T and PV (valid keys)       */
} fe_engine_stats;

/* Creates an engine on `device` and allocates its weight storage.  Mirrors the
 * SentenceTransformerImpl constructor (src/sentence_transformers_impl.cpp:46-98). */
fe_status fe_engine_create(const fe_encoder_config *cfg, int device, fe_engine **out);
fe_status fe_engine_destroy(fe_engine *e);
/* Creates an engine for a pre-RMSNorm rotary encoder (Qwen3 / Gemma3 shapes).  Requires
 * head_dim 128 or 256, q_heads % kv_heads == 0, hidden in {256, 384, 512, 768, 1024, 1536,
 * 2048}, intermediate % 64 == 0; Gemma3 sentences up to 1024 tokens. */
fe_status fe_engine_create_rms(const fe_rms_encoder_config *cfg, int device, fe_engine **out);

/* Uploads one FP32 tensor by its HF name (the keys of the reference's weights map,
 * src/sentence_transformers_impl.cpp:201-218).  `data` is host memory unless
 * data_on_device != 0.  Unknown names return FE_ERR_NOT_FOUND; a wrong element
 * count FE_ERR_INVALID_ARGUMENT. */
fe_status fe_engine_set_weight(fe_engine *e, const char *name, const float *data, size_t count,
                               int data_on_device);
/* Loads every tensor of a model.safetensors file (F32 or BF16 entries); returns
 * FE_ERR_IO on a malformed file.  Replaces load_single_safetensors_file
 * (src/safetensors.cpp:31-95). */
fe_status fe_engine_load_safetensors(fe_engine *e, const char *path);
/* Number of weights still unset (0 = ready). */
int32_t fe_engine_missing_weights(const fe_engine *e);
/* Encodes a packed batch already resident on the engine's device: ids (int32
 * [total]) and cu_seqlens (int32 [batch+1]) are device pointers; cu_seqlens_host
 * is the same offsets in host memory (they size the launches); out is device
 * fp32 [batch, hidden].  Stream-ordered on `stream` (NULL = the engine's stream);
 * does not synchronise. */
fe_status fe_engine_encode_packed(fe_engine *e, const int32_t *ids, const int32_t *cu_seqlens,
                                  const int32_t *cu_seqlens_host, int32_t batch, float *out,
                                  fe_stream_t stream);
/* End-to-end encode from host buffers: ids is host int32 [batch, stride] (right
 * padded), lengths host int32 [batch]; out is host fp32 [batch, hidden].  Copies
 * in, runs, copies out and synchronises.  Consecutive sentences run as one device
 * pass of at most FE_MAX_TOKENS_PER_PASS tokens (default 262,144; a longer sentence
 * runs alone) and 65,535 sentences, so device memory stays bounded for any batch, as
 * the reference's one-sentence-at-a-time loop does.  The device status word is read
 * after every pass: a bad token id (FE_ERR_INVALID_ARGUMENT) or a wait that ran out
 * (FE_ERR_DEVICE_TIMEOUT) ends the call before the next pass.  The word is per device,
 * not per engine, so it also reports such an error recorded since its last read by
 * another engine's or op's kernel on the same device.  The token-id form of
 * SentenceTransformerImpl::encode_batch (src/sentence_transformers_impl.cpp:359-365). */
fe_status fe_engine_encode_host(fe_engine *e, const int32_t *ids, const int32_t *lengths,
                                int32_t batch, int32_t stride, float *out);
/* Per-kernel device timing of subsequent encode calls (CUDA events on the
 * launching stream); off by default. */
fe_status fe_engine_set_profiling(fe_engine *e, int enabled);
fe_status fe_engine_get_stats(const fe_engine *e, fe_engine_stats *stats);

/* ------------------------------------------------------ host-only helpers */
/* Contiguous cut points of a length-sorted batch into `parts` slices of near-equal
 * algorithmic FLOPs (parts-1 cuts written to `cuts`).  Host only; no GPU needed. */
fe_status fe_plan_shards(const fe_encoder_config *cfg, const int32_t *sorted_lengths,
                         int32_t batch, int32_t parts, int32_t *cuts);
/* The same cut rule over explicit per-sentence costs (any model family, e.g. the
 * Qwen3 / Gemma3 shapes' FLOPs): parts-1 contiguous cut points giving slices of
 * near-equal total cost.  Costs must be finite and non-negative.  Host only. */
fe_status fe_plan_shards_costs(const double *costs, int32_t batch, int32_t parts, int32_t *cuts);
/* Packs right-padded host ids [batch, stride] with lengths into ids_packed
 * [sum(lengths)] and cu_seqlens [batch+1].  Host only. */
fe_status fe_pack_batch(const int32_t *ids, const int32_t *lengths, int32_t batch,
                        int32_t stride, int32_t *ids_packed, int32_t *cu_seqlens);

/* BGE WordPiece tokenizer, host only: replaces BGETokenizer (include/tokenizer.h:11-23;
 * tokenize + encode, src/tokenizer.cpp:9-160).  The vocabulary is vocab.txt, one token per
 * line, its line number the id (a repeated line keeps its last id); it must hold [UNK]
 * (FE_ERR_IO otherwise, or when the file cannot be read). */
typedef struct fe_wordpiece fe_wordpiece;
fe_status fe_wordpiece_create(const char *vocab_path, fe_wordpiece **out);
fe_status fe_wordpiece_destroy(fe_wordpiece *t);
/* The ids of `text` (`len` bytes, any bytes) with [CLS]=101 in front and [SEP]=102
 * behind, as SentenceTransformerImpl::tokenize frames them
 * (src/sentence_transformers_impl.cpp:11-27).  *count receives the number of ids; at most
 * `capacity` are written to ids (call with capacity 0 to size the buffer). */
fe_status fe_wordpiece_encode(const fe_wordpiece *t, const char *text, size_t len, int32_t *ids,
                              size_t capacity, size_t *count);

#ifdef __cplusplus
}
#endif
#endif /* FASTEMBED_B200_H */
