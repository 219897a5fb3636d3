// fe_internal.h — host-side declarations shared by the library's translation units:
// error reporting, the per-device status word, TMA descriptor encoding and the
// kernel launchers behind the C ABI.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "fastembed_b200.h"

namespace fe {

// Codes kernels write into the per-device status word.
enum : int { DEV_OK = 0, DEV_BAD_INPUT = 1, DEV_TIMEOUT = 5 };

// Records `msg` as this thread's last error and returns `s`.
fe_status fail(fe_status s, const std::string &msg);
// Maps a CUDA error to a status (recording its text); cudaSuccess -> FE_OK.
fe_status check_cuda(cudaError_t err, const char *what);

#define FE_TRY_CUDA(expr)                                             \
    do {                                                              \
        cudaError_t fe_err_ = (expr);                                 \
        if (fe_err_ != cudaSuccess) return ::fe::check_cuda(fe_err_, #expr); \
    } while (0)

#define FE_TRY(expr)                          \
    do {                                      \
        fe_status fe_st_ = (expr);            \
        if (fe_st_ != FE_OK) return fe_st_;   \
    } while (0)

// Per-device int32 status word that kernels write on bounded-wait timeout or bad
// input (allocated once per device on first use).
int *device_status_word(int device);
int *current_device_status_word();
// Unique id of the CUDA context current on this thread (making the current device's
// primary context current if none is): per-device caches (the status word, scratch and
// counter addresses, kernel attributes) record it and are set up again when it changes,
// so that nothing set up before a cudaDeviceReset is used in the device's next context.
// 1 when the driver cannot tell (the caches then never refresh).
uint64_t current_context_id();
// The work-wait limit of the kernels of one .cu file, on the current device
// (fe_common.cuh c_wait_limit_ns); fe_set_wait_limit calls all of them.
cudaError_t set_wait_limit_linear(uint64_t ns);
cudaError_t set_wait_limit_attention(uint64_t ns);
cudaError_t set_wait_limit_attention_wide(uint64_t ns);
int current_sm_count();
// Programmatic dependent launch for the kernels that call grid_dep_wait(): on with
// FE_PDL=1 (read once per process), off by default.  On bge-large, Qwen3- and
// Gemma3-shaped forwards it measured 0.5-2 % slower than plain stream order: those
// steps run at the power cap, so shorter gaps between kernels buy no time, and the
// successor's waiting CTAs share SMs with the running kernel.
bool pdl_enabled();

// TMA descriptor for a row-major 2-D tensor [rows, cols] of `elem_bytes` elements
// with row stride `ld` elements, box [box_rows, box_cols], swizzled as `swizzle`
// (the box row must then be exactly the swizzle width in bytes).
fe_status make_tmap_2d(CUtensorMap *map, const void *base, CUtensorMapDataType dtype,
                       int elem_bytes, uint64_t rows, uint64_t cols, uint64_t ld,
                       uint32_t box_rows, uint32_t box_cols,
                       CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B);

// TMA descriptor for a head-major tensor [heads, rows, 64] of bf16 (each head's
// rows contiguous), box [1, box_rows, 64], 128B swizzle.
fe_status make_tmap_heads(CUtensorMap *map, const void *base, uint64_t heads, uint64_t rows,
                          uint32_t box_rows);

// ---- launchers (no argument validation; the C ABI validates) ----
// row_ss (optional): deferred RMSNorm row scale of the input, [m][ss_parts] partial sums of
// squares from launch_linear_rms_deferred; each accumulator row i is multiplied by
// 1 / sqrt(sum_p row_ss[i][p] / k + ss_eps) before the epilogue.
cudaError_t launch_linear_bf16(const void *x, const void *w, const float *bias,
                               const float *residual, void *y, int64_t m, int64_t n, int64_t k,
                               int epilogue, int y_dtype, cudaStream_t s, fe_status *st,
                               const float *row_ss = nullptr, int ss_parts = 0, float ss_eps = 0.f);
// True when launch_linear_layernorm runs the step as linear_ln_cluster (LayerNorm, n a
// multiple of 256 from 512 to 1024, k a multiple of 64; by default only where the pair kernel
// would not fuse: pair_fused is that decision).
bool ln_cluster_applies(int64_t n, int64_t k, bool rms, bool pair_fused);
// QKV projection y = x W^T [m, (q_heads + 2 kv_heads) * head_dim] in bf16, no bias, with the
// per-head RMSNorm (w, or 1 + w when one_plus) and rotate-half RoPE (positions pos[m], base
// theta) of the query and key heads applied in the GEMM epilogue; value heads as they are.
// Needs (q_heads * head_dim) % 256 == 0 and (kv_heads * head_dim) % 256 == 0 (not checked).
cudaError_t launch_linear_qk_norm_rope(const void *x, const void *w, void *y, int64_t m, int64_t k, int q_heads,
                                       int kv_heads, int head_dim, const float *q_w, const float *k_w,
                                       const int32_t *pos, bool one_plus, float eps, float theta, cudaStream_t s,
                                       fe_status *st, const float *row_ss = nullptr, int ss_parts = 0);
// Pre-norm projection + residual with the RMSNorm deferred to the consumer:
//     h32 <- (x W^T + bias) + h32,   h16 <- bf16(h32 * gamma) (h16 may be null),
//     row_ss[i][p] <- sum of h32[i][j]^2 over part p of the columns (linear_rms_deferred_parts(n)
// parts); the next projection of h16 takes row_ss (launch_linear_bf16 /
// launch_linear_qk_norm_rope) and applies the factor 1 / sqrt(mean(h32^2) + eps) per row.
// n a multiple of 256, at most 2048.
int linear_rms_deferred_parts(int64_t n);
cudaError_t launch_linear_rms_deferred(const void *x, const void *w, const float *bias, const float *gamma, float *h32,
                                       void *h16, float *row_ss, int64_t m, int64_t n, int64_t k, cudaStream_t s,
                                       fe_status *st);
// h32 <- LayerNorm((x W^T + bias) + h32) * gamma + beta; h16 <- bf16 of it (h16 may be
// null).  stats / y_fallback come from linear_layernorm_split_workspace; the stats
// region must be zero-filled before its first launch.
size_t linear_layernorm_workspace_bytes(int64_t m, int64_t n);
size_t linear_layernorm_stats_bytes(int64_t m, int64_t n);  // the statistics head of it
void linear_layernorm_split_workspace(void *ws, int64_t m, int64_t n, void **stats, float **y);
// rms: pre-norm RMSNorm form instead: h32 <- (x W^T + bias) + h32, h16 <- RMSNorm(h32) * gamma.
cudaError_t launch_linear_layernorm(const void *x, const void *w, const float *bias, const float *gamma,
                                    const float *beta, float *h32, void *h16, int64_t m, int64_t n, int64_t k,
                                    float eps, void *stats, float *y_fallback, cudaStream_t s, fe_status *st,
                                    bool rms = false);
// qkv / out layouts: token-major [T, 3*H*64] / [T, H*64], or head-major
// [3*H, T, 64] / [H, T, 64] when head_major is true.
cudaError_t launch_attention_varlen(const void *qkv, const int32_t *cu_seqlens, int batch,
                                    int max_len, int heads, int head_dim, void *out,
                                    int64_t total_tokens, bool head_major, cudaStream_t s,
                                    fe_status *st);
// Grouped-query attention for head_dim 128 / 256: qkv [T, (q_heads + 2 kv_heads) * head_dim]
// (Q heads, then K heads, then V heads), out [T, q_heads * head_dim].
cudaError_t launch_attention_wide(const void *qkv, const int32_t *cu_seqlens, int batch, int max_len, int q_heads,
                                  int kv_heads, int head_dim, bool causal, float scale, void *out,
                                  int64_t total_tokens, cudaStream_t s, fe_status *st);
// Row kernels of the RMSNorm / RoPE encoders (k_decoder.cu); one_plus selects the
// (1 + w) weight form.  dim in {256, 384, 512, 768, 1024, 1536, 2048}.
cudaError_t launch_embed_scale(const int32_t *ids, int64_t total, const float *word, int vocab, int dim, float scale,
                               float *h32, cudaStream_t s);
cudaError_t launch_rms_norm_rows(const float *x, const float *w, bool one_plus, float eps, int64_t rows, int dim,
                                 float *o32, void *o16, cudaStream_t s);
cudaError_t launch_rms_sandwich(const void *y, const float *w_post, float *h32, const float *w_next, bool one_plus,
                                float eps, int64_t rows, int dim, float *o32, void *o16, cudaStream_t s,
                                bool y_bf16 = false);
// pos: the positions array of launch_token_positions, or null to search cu for each token
cudaError_t launch_qk_norm_rope(void *qkv, const int32_t *cu, int batch, int64_t total, int q_heads, int kv_heads,
                                int head_dim, const float *q_w, const float *k_w, bool one_plus, float eps, float theta,
                                cudaStream_t s, const int32_t *pos = nullptr);
// pos[t] = position of token t in its sentence, for the packed batch of cu [batch + 1]
cudaError_t launch_token_positions(const int32_t *cu, int batch, int32_t *pos, cudaStream_t s);
cudaError_t launch_embed_layernorm(const int32_t *ids, const int32_t *cu, int batch, int64_t total,
                                   const float *word, const float *pos, const float *type,
                                   const float *g, const float *b, int dim, int vocab,
                                   int max_pos, float eps, float *h32, void *h16, cudaStream_t s,
                                   int pad_id = -1);
// h = LayerNorm(x [+ res]); res may be null, h32 may alias res.
cudaError_t launch_layernorm_dual(const float *x, const float *res, const float *g, const float *b,
                                  float *h32, void *h16, int64_t rows, int dim, float eps, cudaStream_t s);
// The same with x in bf16 (a projection written in bf16).
cudaError_t launch_layernorm_dual_bf16in(const void *x, const float *res, const float *g, const float *b, float *h32,
                                         void *h16, int64_t rows, int dim, float eps, cudaStream_t s);
cudaError_t launch_pool_l2(const float *h, const int32_t *cu, int batch, int dim, int mode,
                           float *out, cudaStream_t s);
cudaError_t launch_f32_to_bf16(const float *x, void *y, int64_t count, cudaStream_t s);

cudaError_t launch_sgemm(const float *a, const float *b, const float *bias, float *c, int64_t m,
                         int64_t n, int64_t k, bool b_transposed, cudaStream_t s);
cudaError_t launch_unary(int op, const float *x, float *y, int64_t count, cudaStream_t s);
cudaError_t launch_layer_norm_f32(const float *x, const float *g, const float *b, float *y,
                                  int64_t rows, int64_t dim, float eps, cudaStream_t s);
cudaError_t launch_rms_norm_f32(const float *x, const float *w, float *y, int64_t rows,
                                int64_t dim, float eps, cudaStream_t s);
cudaError_t launch_softmax_rows_f32(const float *x, float *y, int64_t rows, int64_t dim,
                                    cudaStream_t s);
cudaError_t launch_mha_core_f32(const float *q, const float *k, const float *v, float *out,
                                int64_t seq_len, int64_t dim, int64_t heads, cudaStream_t s);

}  // namespace fe
