// capi_ops.cpp — extern "C" op entry points: argument validation, then the launchers.
// Validation mirrors the reference's checks where it has them (shape errors are
// std::invalid_argument there: src/ops/cuda/cuda_matrix_ops.cu:314-319, :365-373,
// :470-481; src/ops/cuda/cuda_attention_ops.cu:182-187) and returns
// FE_ERR_INVALID_ARGUMENT instead of throwing or exiting.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <string>
#include <vector>

#include "fe_internal.h"

using fe::fail;

namespace {

inline cudaStream_t cs(fe_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

inline fe_status done(cudaError_t e, const char *what) { return fe::check_cuda(e, what); }

inline bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Row widths with a register-resident warp-per-row kernel (dim = 128 * v).
bool supported_row_dim(int32_t dim)
{
    const int v = dim / 128;
    return dim > 0 && dim % 128 == 0 && (v == 1 || v == 2 || v == 3 || v == 4 || v == 6 || v == 8 || v == 12 || v == 16);
}


}  // namespace

extern "C" {

fe_status fe_sgemm_nn(const float *a, const float *b, float *c, int64_t m, int64_t n, int64_t k,
                      fe_stream_t stream)
{
    if (m < 0 || n < 0 || k < 0) return fail(FE_ERR_INVALID_ARGUMENT, "fe_sgemm_nn: negative size");
    if (m && k && (!c || (n && (!a || !b)))) return fail(FE_ERR_INVALID_ARGUMENT, "fe_sgemm_nn: null pointer");
    return done(fe::launch_sgemm(a, b, nullptr, c, m, n, k, false, cs(stream)), "fe_sgemm_nn");
}

fe_status fe_sgemm_nt(const float *a, const float *b, const float *bias, float *c, int64_t m, int64_t n,
                      int64_t k, fe_stream_t stream)
{
    if (m < 0 || n < 0 || k < 0) return fail(FE_ERR_INVALID_ARGUMENT, "fe_sgemm_nt: negative size");
    if (m && k && (!c || (n && (!a || !b)))) return fail(FE_ERR_INVALID_ARGUMENT, "fe_sgemm_nt: null pointer");
    return done(fe::launch_sgemm(a, b, bias, c, m, n, k, true, cs(stream)), "fe_sgemm_nt");
}

static fe_status unary(int op, const float *x, float *y, int64_t count, fe_stream_t stream, const char *name)
{
    if (count < 0) return fail(FE_ERR_INVALID_ARGUMENT, std::string(name) + ": negative count");
    if (count && (!x || !y)) return fail(FE_ERR_INVALID_ARGUMENT, std::string(name) + ": null pointer");
    return done(fe::launch_unary(op, x, y, count, cs(stream)), name);
}

fe_status fe_gelu_f32(const float *x, float *y, int64_t count, fe_stream_t s) { return unary(FE_ACT_GELU, x, y, count, s, "fe_gelu_f32"); }
fe_status fe_relu_f32(const float *x, float *y, int64_t count, fe_stream_t s) { return unary(FE_ACT_RELU, x, y, count, s, "fe_relu_f32"); }
fe_status fe_swish_f32(const float *x, float *y, int64_t count, fe_stream_t s) { return unary(FE_ACT_SWISH, x, y, count, s, "fe_swish_f32"); }

fe_status fe_layer_norm_f32(const float *x, const float *gamma, const float *beta, float *y, int64_t rows,
                            int64_t dim, float eps, fe_stream_t stream)
{
    if (rows < 0 || dim <= 0) return fail(FE_ERR_INVALID_ARGUMENT, "fe_layer_norm_f32: bad shape");
    if (rows && (!x || !gamma || !beta || !y)) return fail(FE_ERR_INVALID_ARGUMENT, "fe_layer_norm_f32: null pointer");
    if (rows > 0x7fffffff) return fail(FE_ERR_UNSUPPORTED, "fe_layer_norm_f32: too many rows");
    return done(fe::launch_layer_norm_f32(x, gamma, beta, y, rows, dim, eps, cs(stream)), "fe_layer_norm_f32");
}

fe_status fe_rms_norm_f32(const float *x, const float *weight, float *y, int64_t rows, int64_t dim, float eps,
                          fe_stream_t stream)
{
    if (rows < 0 || dim <= 0) return fail(FE_ERR_INVALID_ARGUMENT, "fe_rms_norm_f32: bad shape");
    if (rows && (!x || !weight || !y)) return fail(FE_ERR_INVALID_ARGUMENT, "fe_rms_norm_f32: null pointer");
    if (rows > 0x7fffffff) return fail(FE_ERR_UNSUPPORTED, "fe_rms_norm_f32: too many rows");
    return done(fe::launch_rms_norm_f32(x, weight, y, rows, dim, eps, cs(stream)), "fe_rms_norm_f32");
}

fe_status fe_softmax_rows_f32(const float *x, float *y, int64_t rows, int64_t dim, fe_stream_t stream)
{
    if (rows < 0 || dim <= 0) return fail(FE_ERR_INVALID_ARGUMENT, "fe_softmax_rows_f32: bad shape");
    if (rows && (!x || !y)) return fail(FE_ERR_INVALID_ARGUMENT, "fe_softmax_rows_f32: null pointer");
    if (rows > 0x7fffffff) return fail(FE_ERR_UNSUPPORTED, "fe_softmax_rows_f32: too many rows");
    return done(fe::launch_softmax_rows_f32(x, y, rows, dim, cs(stream)), "fe_softmax_rows_f32");
}

fe_status fe_softmax_scores_inplace_f32(float *scores, int64_t heads, int64_t seq_len, fe_stream_t stream)
{
    if (heads < 0 || seq_len < 0) return fail(FE_ERR_INVALID_ARGUMENT, "fe_softmax_scores_inplace_f32: bad shape");
    if (heads * seq_len == 0) return FE_OK;
    if (!scores) return fail(FE_ERR_INVALID_ARGUMENT, "fe_softmax_scores_inplace_f32: null pointer");
    return done(fe::launch_softmax_rows_f32(scores, scores, heads * seq_len, seq_len, cs(stream)),
                "fe_softmax_scores_inplace_f32");
}

size_t fe_mha_f32_workspace_bytes(int64_t seq_len, int64_t dim, int64_t heads)
{
    (void)heads;
    if (seq_len <= 0 || dim <= 0) return 0;
    return static_cast<size_t>(3 * seq_len * dim) * sizeof(float);
}

fe_status fe_mha_f32(const float *x, const float *wq, const float *wk, const float *wv, const float *bq,
                     const float *bk, const float *bv, float *out, int64_t seq_len, int64_t dim, int64_t heads,
                     void *workspace, size_t workspace_bytes, fe_stream_t stream)
{
    if (heads <= 0 || dim <= 0 || seq_len < 0)
        return fail(FE_ERR_INVALID_ARGUMENT, "fe_mha_f32: bad shape");
    if (dim % heads != 0)
        return fail(FE_ERR_INVALID_ARGUMENT, "Embedding dimension must be divisible by number of heads");
    if (seq_len == 0) return FE_OK;
    if (!x || !wq || !wk || !wv || !bq || !bk || !bv || !out)
        return fail(FE_ERR_INVALID_ARGUMENT, "fe_mha_f32: null pointer");
    if (!workspace || workspace_bytes < fe_mha_f32_workspace_bytes(seq_len, dim, heads))
        return fail(FE_ERR_INVALID_ARGUMENT, "fe_mha_f32: workspace too small");
    if (seq_len > 0xffff || static_cast<size_t>(seq_len) * 4 > 200 * 1024)
        return fail(FE_ERR_UNSUPPORTED, "fe_mha_f32: sequence too long for the fp32 path");
    float *q = static_cast<float *>(workspace);
    float *k = q + seq_len * dim;
    float *v = k + seq_len * dim;
    cudaStream_t s = cs(stream);
    FE_TRY_CUDA(fe::launch_sgemm(x, wq, bq, q, seq_len, dim, dim, true, s));
    FE_TRY_CUDA(fe::launch_sgemm(x, wk, bk, k, seq_len, dim, dim, true, s));
    FE_TRY_CUDA(fe::launch_sgemm(x, wv, bv, v, seq_len, dim, dim, true, s));
    return done(fe::launch_mha_core_f32(q, k, v, out, seq_len, dim, heads, s), "fe_mha_f32");
}

static fe_status linear_call(const char *name, const void *x, const void *w, const float *bias, const float *residual,
                             void *y, int64_t m, int64_t n, int64_t k, fe_epilogue epilogue, fe_dtype y_dtype,
                             const float *row_ss, int32_t ss_parts, float ss_eps, fe_stream_t stream)
{
    if (m < 0 || n <= 0 || k <= 0) return fail(FE_ERR_INVALID_ARGUMENT, std::string(name) + ": bad shape");
    if (k % 8 != 0 || n % 8 != 0) return fail(FE_ERR_INVALID_ARGUMENT, std::string(name) + ": k and n must be multiples of 8");
    if (m > 0x7fffffff || n > 0x7fffffff || k > 0x7fffffff) return fail(FE_ERR_UNSUPPORTED, std::string(name) + ": size too large");
    if (epilogue < FE_EPI_NONE || epilogue > FE_EPI_GEGLU)
        return fail(FE_ERR_INVALID_ARGUMENT, std::string(name) + ": unknown epilogue");
    const bool glu = epilogue == FE_EPI_SWIGLU || epilogue == FE_EPI_GEGLU;
    if (glu && (n % 128 != 0 || y_dtype != FE_DTYPE_BF16))
        return fail(FE_ERR_INVALID_ARGUMENT, std::string(name) + ": gated epilogues need n % 128 == 0 and bf16 output");
    if (y_dtype != FE_DTYPE_F32 && y_dtype != FE_DTYPE_BF16)
        return fail(FE_ERR_INVALID_ARGUMENT, std::string(name) + ": unknown output dtype");
    if (epilogue == FE_EPI_BIAS_RESIDUAL && y_dtype != FE_DTYPE_F32)
        return fail(FE_ERR_INVALID_ARGUMENT, std::string(name) + ": the residual epilogue writes fp32");
    if (m == 0) return FE_OK;
    if (!x || !w || !y) return fail(FE_ERR_INVALID_ARGUMENT, std::string(name) + ": null pointer");
    if (epilogue != FE_EPI_NONE && !glu && !bias)
        return fail(FE_ERR_INVALID_ARGUMENT, std::string(name) + ": epilogue needs a bias");
    if (epilogue == FE_EPI_BIAS_RESIDUAL && !residual)
        return fail(FE_ERR_INVALID_ARGUMENT, std::string(name) + ": residual epilogue needs a residual");
    if (!aligned16(x) || !aligned16(w) || !aligned16(y) || (bias && !aligned16(bias)) ||
        (residual && !aligned16(residual)))
        return fail(FE_ERR_INVALID_ARGUMENT, std::string(name) + ": pointers must be 16-byte aligned");
    fe_status st = FE_OK;
    cudaError_t e = fe::launch_linear_bf16(x, w, bias, residual, y, m, n, k, epilogue, y_dtype,
                                           reinterpret_cast<cudaStream_t>(stream), &st, row_ss, ss_parts, ss_eps);
    if (st != FE_OK) return st;
    return done(e, name);
}

fe_status fe_linear_bf16(const void *x, const void *w, const float *bias, const float *residual, void *y,
                         int64_t m, int64_t n, int64_t k, fe_epilogue epilogue, fe_dtype y_dtype,
                         fe_stream_t stream)
{
    return linear_call("fe_linear_bf16", x, w, bias, residual, y, m, n, k, epilogue, y_dtype, nullptr, 0, 0.f, stream);
}

fe_status fe_linear_row_scaled_bf16(const void *x, const void *w, const float *bias, const float *residual, void *y,
                                    int64_t m, int64_t n, int64_t k, fe_epilogue epilogue, fe_dtype y_dtype,
                                    const float *row_ss, int32_t ss_parts, float eps, fe_stream_t stream)
{
    if (ss_parts < 1 || ss_parts > 8) return fail(FE_ERR_INVALID_ARGUMENT, "fe_linear_row_scaled_bf16: ss_parts must be 1..8");
    if (m > 0 && !row_ss) return fail(FE_ERR_INVALID_ARGUMENT, "fe_linear_row_scaled_bf16: null pointer");
    return linear_call("fe_linear_row_scaled_bf16", x, w, bias, residual, y, m, n, k, epilogue, y_dtype, row_ss, ss_parts,
                       eps, stream);
}

fe_status fe_attention_varlen_bf16(const void *qkv, const int32_t *cu_seqlens, int32_t batch, int32_t max_len,
                                   int32_t heads, int32_t head_dim, void *out, int64_t total_tokens,
                                   fe_stream_t stream)
{
    if (batch < 0 || max_len < 0 || heads <= 0 || total_tokens < 0)
        return fail(FE_ERR_INVALID_ARGUMENT, "fe_attention_varlen_bf16: bad shape");
    if (head_dim != 64) return fail(FE_ERR_UNSUPPORTED, "fe_attention_varlen_bf16: head_dim must be 64");
    if (max_len > 4096 || heads > 65535 || batch > 65535)
        return fail(FE_ERR_UNSUPPORTED, "fe_attention_varlen_bf16: batch, heads or max_len too large");
    if (batch == 0 || total_tokens == 0) return FE_OK;
    if (static_cast<int64_t>(4096) * ((max_len + 127) / 128) * heads > 0x7fffffff)
        return fail(FE_ERR_UNSUPPORTED, "fe_attention_varlen_bf16: too many (sentence, tile, head) units");
    if (!qkv || !cu_seqlens || !out) return fail(FE_ERR_INVALID_ARGUMENT, "fe_attention_varlen_bf16: null pointer");
    if (!aligned16(qkv) || !aligned16(out))
        return fail(FE_ERR_INVALID_ARGUMENT, "fe_attention_varlen_bf16: pointers must be 16-byte aligned");
    fe_status st = FE_OK;
    cudaError_t e = fe::launch_attention_varlen(qkv, cu_seqlens, batch, max_len, heads, head_dim, out, total_tokens,
                                                false, reinterpret_cast<cudaStream_t>(stream), &st);
    if (st != FE_OK) return st;
    return done(e, "fe_attention_varlen_bf16");
}

fe_status fe_attention_varlen_gqa_bf16(const void *qkv, const int32_t *cu_seqlens, int32_t batch, int32_t max_len,
                                       int32_t q_heads, int32_t kv_heads, int32_t head_dim, int32_t causal, float scale,
                                       void *out, int64_t total_tokens, fe_stream_t stream)
{
    if (batch < 0 || max_len < 0 || q_heads <= 0 || kv_heads <= 0 || total_tokens < 0)
        return fail(FE_ERR_INVALID_ARGUMENT, "fe_attention_varlen_gqa_bf16: bad shape");
    if (q_heads % kv_heads != 0)
        return fail(FE_ERR_INVALID_ARGUMENT, "fe_attention_varlen_gqa_bf16: q_heads must be a multiple of kv_heads");
    if (head_dim != 128 && head_dim != 256)
        return fail(FE_ERR_UNSUPPORTED, "fe_attention_varlen_gqa_bf16: head_dim must be 128 or 256");
    if (max_len > 65536 || batch > 1 << 24 || q_heads > 1024)
        return fail(FE_ERR_UNSUPPORTED, "fe_attention_varlen_gqa_bf16: batch, heads or max_len too large");
    if (batch == 0 || total_tokens == 0) return FE_OK;
    if (!qkv || !cu_seqlens || !out) return fail(FE_ERR_INVALID_ARGUMENT, "fe_attention_varlen_gqa_bf16: null pointer");
    if (!aligned16(qkv) || !aligned16(out))
        return fail(FE_ERR_INVALID_ARGUMENT, "fe_attention_varlen_gqa_bf16: pointers must be 16-byte aligned");
    fe_status st = FE_OK;
    cudaError_t e = fe::launch_attention_wide(qkv, cu_seqlens, batch, max_len, q_heads, kv_heads, head_dim, causal != 0,
                                              scale, out, total_tokens, reinterpret_cast<cudaStream_t>(stream), &st);
    if (st != FE_OK) return st;
    return done(e, "fe_attention_varlen_gqa_bf16");
}

fe_status fe_embed_layernorm(const int32_t *ids, const int32_t *cu_seqlens, int32_t batch, int64_t total_tokens,
                             const float *word, const float *pos, const float *type, const float *gamma,
                             const float *beta, int32_t dim, int32_t vocab, int32_t max_pos, float eps, float *h32,
                             void *h16, fe_stream_t stream)
{
    if (batch < 0 || total_tokens < 0 || vocab <= 0 || max_pos <= 0)
        return fail(FE_ERR_INVALID_ARGUMENT, "fe_embed_layernorm: bad shape");
    if (!supported_row_dim(dim) || dim == 128)
        return fail(FE_ERR_UNSUPPORTED, "fe_embed_layernorm: dim must be 256, 384, 512, 768, 1024, 1536 or 2048");
    if (total_tokens == 0) return FE_OK;
    if (batch == 0) return fail(FE_ERR_INVALID_ARGUMENT, "fe_embed_layernorm: tokens without sentences");
    if (!ids || !cu_seqlens || !word || !pos || !type || !gamma || !beta || !h32)
        return fail(FE_ERR_INVALID_ARGUMENT, "fe_embed_layernorm: null pointer");
    return done(fe::launch_embed_layernorm(ids, cu_seqlens, batch, total_tokens, word, pos, type, gamma, beta, dim,
                                           vocab, max_pos, eps, h32, h16, reinterpret_cast<cudaStream_t>(stream)),
                "fe_embed_layernorm");
}

fe_status fe_embed_layernorm_xlmr(const int32_t *ids, const int32_t *cu_seqlens, int32_t batch, int64_t total_tokens,
                                  const float *word, const float *pos, const float *type, const float *gamma,
                                  const float *beta, int32_t dim, int32_t vocab, int32_t max_pos, int32_t pad_token_id,
                                  float eps, float *h32, void *h16, fe_stream_t stream)
{
    if (batch < 0 || total_tokens < 0 || vocab <= 0 || max_pos <= 0 || pad_token_id < 0)
        return fail(FE_ERR_INVALID_ARGUMENT, "fe_embed_layernorm_xlmr: bad shape or pad_token_id");
    if (!supported_row_dim(dim) || dim == 128)
        return fail(FE_ERR_UNSUPPORTED, "fe_embed_layernorm_xlmr: dim must be 256, 384, 512, 768, 1024, 1536 or 2048");
    if (total_tokens == 0) return FE_OK;
    if (batch == 0) return fail(FE_ERR_INVALID_ARGUMENT, "fe_embed_layernorm_xlmr: tokens without sentences");
    if (!ids || !cu_seqlens || !word || !pos || !type || !gamma || !beta || !h32)
        return fail(FE_ERR_INVALID_ARGUMENT, "fe_embed_layernorm_xlmr: null pointer");
    return done(fe::launch_embed_layernorm(ids, cu_seqlens, batch, total_tokens, word, pos, type, gamma, beta, dim,
                                           vocab, max_pos, eps, h32, h16, reinterpret_cast<cudaStream_t>(stream),
                                           pad_token_id),
                "fe_embed_layernorm_xlmr");
}

fe_status fe_layernorm_dual(const float *x, const float *residual, const float *gamma, const float *beta, float *h32,
                            void *h16, int64_t rows, int32_t dim, float eps, fe_stream_t stream)
{
    if (rows < 0 || dim <= 0) return fail(FE_ERR_INVALID_ARGUMENT, "fe_layernorm_dual: bad shape");
    if (residual && !supported_row_dim(dim))
        return fail(FE_ERR_UNSUPPORTED, "fe_layernorm_dual: the residual form needs dim in {128, 256, 384, 512, 768, "
                                        "1024, 1536, 2048}");
    if (rows > 0x7fffffff) return fail(FE_ERR_UNSUPPORTED, "fe_layernorm_dual: too many rows");
    if (rows == 0) return FE_OK;
    if (!x || !gamma || !beta || !h32) return fail(FE_ERR_INVALID_ARGUMENT, "fe_layernorm_dual: null pointer");
    return done(fe::launch_layernorm_dual(x, residual, gamma, beta, h32, h16, rows, dim, eps,
                                          reinterpret_cast<cudaStream_t>(stream)),
                "fe_layernorm_dual");
}

fe_status fe_linear_layernorm_workspace_bytes(int64_t m, int64_t n, size_t *bytes)
{
    if (!bytes) return fail(FE_ERR_INVALID_ARGUMENT, "fe_linear_layernorm_workspace_bytes: null pointer");
    if (m < 0 || n <= 0) return fail(FE_ERR_INVALID_ARGUMENT, "fe_linear_layernorm_workspace_bytes: bad shape");
    *bytes = fe::linear_layernorm_workspace_bytes(m, n);
    return FE_OK;
}

fe_status fe_linear_layernorm_bf16(const void *x, const void *w, const float *bias, const float *gamma,
                                   const float *beta, float *h32, void *h16, int64_t m, int64_t n, int64_t k,
                                   float eps, void *workspace, size_t workspace_bytes, fe_stream_t stream)
{
    if (m < 0 || n <= 0 || k <= 0) return fail(FE_ERR_INVALID_ARGUMENT, "fe_linear_layernorm_bf16: bad shape");
    if (k % 8 != 0) return fail(FE_ERR_INVALID_ARGUMENT, "fe_linear_layernorm_bf16: k must be a multiple of 8");
    if (n > 0x7fffffff || !supported_row_dim(static_cast<int32_t>(n)))
        return fail(FE_ERR_UNSUPPORTED, "fe_linear_layernorm_bf16: n must be 128, 256, 384, 512, 768, 1024, 1536 "
                                        "or 2048");
    if (m > 0x7fffffff || k > 0x7fffffff) return fail(FE_ERR_UNSUPPORTED, "fe_linear_layernorm_bf16: size too large");
    if (m == 0) return FE_OK;
    if (!x || !w || !bias || !gamma || !beta || !h32 || !workspace)
        return fail(FE_ERR_INVALID_ARGUMENT, "fe_linear_layernorm_bf16: null pointer");
    if (workspace_bytes < fe::linear_layernorm_workspace_bytes(m, n))
        return fail(FE_ERR_INVALID_ARGUMENT, "fe_linear_layernorm_bf16: workspace too small");
    if (!aligned16(x) || !aligned16(w) || !aligned16(bias) || !aligned16(gamma) || !aligned16(beta) ||
        !aligned16(h32) || (h16 && !aligned16(h16)) || !aligned16(workspace))
        return fail(FE_ERR_INVALID_ARGUMENT, "fe_linear_layernorm_bf16: pointers must be 16-byte aligned");
    void *stats = nullptr;
    float *y = nullptr;
    fe::linear_layernorm_split_workspace(workspace, m, n, &stats, &y);
    fe_status st = FE_OK;
    cudaError_t e = fe::launch_linear_layernorm(x, w, bias, gamma, beta, h32, h16, m, n, k, eps, stats, y,
                                                reinterpret_cast<cudaStream_t>(stream), &st);
    if (st != FE_OK) return st;
    return done(e, "fe_linear_layernorm_bf16");
}

fe_status fe_linear_rmsnorm_bf16(const void *x, const void *w, const float *bias, const float *rms_w, float *h32,
                                 void *h16, int64_t m, int64_t n, int64_t k, float eps, void *workspace,
                                 size_t workspace_bytes, fe_stream_t stream)
{
    if (m < 0 || n <= 0 || k <= 0) return fail(FE_ERR_INVALID_ARGUMENT, "fe_linear_rmsnorm_bf16: bad shape");
    if (k % 8 != 0) return fail(FE_ERR_INVALID_ARGUMENT, "fe_linear_rmsnorm_bf16: k must be a multiple of 8");
    if (n > 0x7fffffff || !supported_row_dim(static_cast<int32_t>(n)) || n == 128)
        return fail(FE_ERR_UNSUPPORTED, "fe_linear_rmsnorm_bf16: n must be 256, 384, 512, 768, 1024, 1536 or 2048");
    if (m > 0x7fffffff || k > 0x7fffffff) return fail(FE_ERR_UNSUPPORTED, "fe_linear_rmsnorm_bf16: size too large");
    if (m == 0) return FE_OK;
    if (!x || !w || !bias || !rms_w || !h32 || !workspace)
        return fail(FE_ERR_INVALID_ARGUMENT, "fe_linear_rmsnorm_bf16: null pointer");
    if (workspace_bytes < fe::linear_layernorm_workspace_bytes(m, n))
        return fail(FE_ERR_INVALID_ARGUMENT, "fe_linear_rmsnorm_bf16: workspace too small");
    if (!aligned16(x) || !aligned16(w) || !aligned16(bias) || !aligned16(rms_w) || !aligned16(h32) ||
        (h16 && !aligned16(h16)) || !aligned16(workspace))
        return fail(FE_ERR_INVALID_ARGUMENT, "fe_linear_rmsnorm_bf16: pointers must be 16-byte aligned");
    void *stats = nullptr;
    float *y = nullptr;
    fe::linear_layernorm_split_workspace(workspace, m, n, &stats, &y);
    fe_status st = FE_OK;
    cudaError_t e = fe::launch_linear_layernorm(x, w, bias, rms_w, nullptr, h32, h16, m, n, k, eps, stats, y,
                                                reinterpret_cast<cudaStream_t>(stream), &st, true);
    if (st != FE_OK) return st;
    return done(e, "fe_linear_rmsnorm_bf16");
}

int32_t fe_linear_rmsnorm_deferred_parts(int64_t n)
{
    return n > 0 && n % 256 == 0 && n <= 2048 ? fe::linear_rms_deferred_parts(n) : 0;
}

fe_status fe_linear_rmsnorm_deferred_bf16(const void *x, const void *w, const float *bias, const float *rms_w,
                                          float *h32, void *h16, float *row_ss, int64_t m, int64_t n, int64_t k,
                                          fe_stream_t stream)
{
    if (m < 0 || n <= 0 || k <= 0) return fail(FE_ERR_INVALID_ARGUMENT, "fe_linear_rmsnorm_deferred_bf16: bad shape");
    if (k % 8 != 0) return fail(FE_ERR_INVALID_ARGUMENT, "fe_linear_rmsnorm_deferred_bf16: k must be a multiple of 8");
    if (n % 256 != 0 || n > 2048)
        return fail(FE_ERR_UNSUPPORTED, "fe_linear_rmsnorm_deferred_bf16: n must be a multiple of 256, at most 2048");
    if (m > 0x7fffffff || k > 0x7fffffff) return fail(FE_ERR_UNSUPPORTED, "fe_linear_rmsnorm_deferred_bf16: size too large");
    if (m == 0) return FE_OK;
    if (!x || !w || !bias || !rms_w || !h32 || !row_ss)
        return fail(FE_ERR_INVALID_ARGUMENT, "fe_linear_rmsnorm_deferred_bf16: null pointer");
    if (!aligned16(x) || !aligned16(w) || !aligned16(bias) || !aligned16(rms_w) || !aligned16(h32) ||
        (h16 && !aligned16(h16)) || !aligned16(row_ss))
        return fail(FE_ERR_INVALID_ARGUMENT, "fe_linear_rmsnorm_deferred_bf16: pointers must be 16-byte aligned");
    fe_status st = FE_OK;
    cudaError_t e = fe::launch_linear_rms_deferred(x, w, bias, rms_w, h32, h16, row_ss, m, n, k,
                                                   reinterpret_cast<cudaStream_t>(stream), &st);
    if (st != FE_OK) return st;
    return done(e, "fe_linear_rmsnorm_deferred_bf16");
}

static bool rms_dim_ok(int32_t dim) { return supported_row_dim(dim) && dim != 128; }

fe_status fe_embed_scale(const int32_t *ids, int64_t total_tokens, const float *word, int32_t vocab, int32_t dim,
                         float scale, float *h32, fe_stream_t stream)
{
    if (total_tokens < 0 || vocab <= 0) return fail(FE_ERR_INVALID_ARGUMENT, "fe_embed_scale: bad shape");
    if (!rms_dim_ok(dim)) return fail(FE_ERR_UNSUPPORTED, "fe_embed_scale: unsupported dim");
    if (total_tokens == 0) return FE_OK;
    if (!ids || !word || !h32) return fail(FE_ERR_INVALID_ARGUMENT, "fe_embed_scale: null pointer");
    return done(fe::launch_embed_scale(ids, total_tokens, word, vocab, dim, scale, h32,
                                       reinterpret_cast<cudaStream_t>(stream)),
                "fe_embed_scale");
}

fe_status fe_rms_norm_rows(const float *x, const float *w, int32_t one_plus, float eps, int64_t rows, int32_t dim,
                           float *o32, void *o16, fe_stream_t stream)
{
    if (rows < 0) return fail(FE_ERR_INVALID_ARGUMENT, "fe_rms_norm_rows: bad shape");
    if (!rms_dim_ok(dim)) return fail(FE_ERR_UNSUPPORTED, "fe_rms_norm_rows: unsupported dim");
    if (rows == 0) return FE_OK;
    if (!x || !w || (!o32 && !o16)) return fail(FE_ERR_INVALID_ARGUMENT, "fe_rms_norm_rows: null pointer");
    return done(fe::launch_rms_norm_rows(x, w, one_plus != 0, eps, rows, dim, o32, o16,
                                         reinterpret_cast<cudaStream_t>(stream)),
                "fe_rms_norm_rows");
}

fe_status fe_rms_sandwich_bf16(const void *y, const float *w_post, float *h32, const float *w_next,
                               int32_t one_plus, float eps, int64_t rows, int32_t dim, float *o32, void *o16,
                               fe_stream_t stream)
{
    if (rows < 0) return fail(FE_ERR_INVALID_ARGUMENT, "fe_rms_sandwich_bf16: bad shape");
    if (!rms_dim_ok(dim)) return fail(FE_ERR_UNSUPPORTED, "fe_rms_sandwich_bf16: unsupported dim");
    if (rows == 0) return FE_OK;
    if (!y || !w_post || !h32 || !w_next || (!o32 && !o16))
        return fail(FE_ERR_INVALID_ARGUMENT, "fe_rms_sandwich_bf16: null pointer");
    return done(fe::launch_rms_sandwich(y, w_post, h32, w_next, one_plus != 0, eps, rows, dim, o32, o16,
                                        reinterpret_cast<cudaStream_t>(stream), true),
                "fe_rms_sandwich_bf16");
}

fe_status fe_rms_sandwich(const float *y, const float *w_post, float *h32, const float *w_next, int32_t one_plus,
                          float eps, int64_t rows, int32_t dim, float *o32, void *o16, fe_stream_t stream)
{
    if (rows < 0) return fail(FE_ERR_INVALID_ARGUMENT, "fe_rms_sandwich: bad shape");
    if (!rms_dim_ok(dim)) return fail(FE_ERR_UNSUPPORTED, "fe_rms_sandwich: unsupported dim");
    if (rows == 0) return FE_OK;
    if (!y || !w_post || !h32 || !w_next || (!o32 && !o16))
        return fail(FE_ERR_INVALID_ARGUMENT, "fe_rms_sandwich: null pointer");
    return done(fe::launch_rms_sandwich(y, w_post, h32, w_next, one_plus != 0, eps, rows, dim, o32, o16,
                                        reinterpret_cast<cudaStream_t>(stream)),
                "fe_rms_sandwich");
}

fe_status fe_qk_norm_rope_bf16(void *qkv, const int32_t *cu_seqlens, int32_t batch, int64_t total_tokens,
                               int32_t q_heads, int32_t kv_heads, int32_t head_dim, const float *q_w, const float *k_w,
                               int32_t one_plus, float eps, float theta, fe_stream_t stream)
{
    if (batch < 0 || total_tokens < 0 || q_heads <= 0 || kv_heads <= 0 || !(theta > 1.0f))
        return fail(FE_ERR_INVALID_ARGUMENT, "fe_qk_norm_rope_bf16: bad shape");
    if (head_dim != 128 && head_dim != 256) return fail(FE_ERR_UNSUPPORTED, "fe_qk_norm_rope_bf16: head_dim 128 or 256");
    if (total_tokens == 0) return FE_OK;
    if (batch == 0 || !qkv || !cu_seqlens || !q_w || !k_w)
        return fail(FE_ERR_INVALID_ARGUMENT, "fe_qk_norm_rope_bf16: null pointer or no sentences");
    return done(fe::launch_qk_norm_rope(qkv, cu_seqlens, batch, total_tokens, q_heads, kv_heads, head_dim, q_w, k_w,
                                        one_plus != 0, eps, theta, reinterpret_cast<cudaStream_t>(stream)),
                "fe_qk_norm_rope_bf16");
}

static fe_status qk_norm_rope_call(const char *name, const void *x, const void *w, const float *q_w, const float *k_w,
                                   const int32_t *positions, void *qkv, int64_t m, int64_t k, int32_t q_heads,
                                   int32_t kv_heads, int32_t head_dim, int32_t one_plus, float eps, float theta,
                                   const float *row_ss, int32_t ss_parts, fe_stream_t stream)
{
    if (m < 0 || k <= 0 || q_heads <= 0 || kv_heads <= 0 || !(theta > 1.0f))
        return fail(FE_ERR_INVALID_ARGUMENT, std::string(name) + ": bad shape");
    if (k % 8 != 0) return fail(FE_ERR_INVALID_ARGUMENT, std::string(name) + ": k must be a multiple of 8");
    if (head_dim != 128 && head_dim != 256)
        return fail(FE_ERR_UNSUPPORTED, std::string(name) + ": head_dim must be 128 or 256");
    if ((static_cast<int64_t>(q_heads) * head_dim) % 256 != 0 || (static_cast<int64_t>(kv_heads) * head_dim) % 256 != 0)
        return fail(FE_ERR_UNSUPPORTED,
                    std::string(name) + ": q_heads * head_dim and kv_heads * head_dim must be multiples of 256");
    if (m > 0x7fffffff || k > 0x7fffffff || static_cast<int64_t>(q_heads + 2 * kv_heads) * head_dim > 0x7fffffff)
        return fail(FE_ERR_UNSUPPORTED, std::string(name) + ": size too large");
    if (m == 0) return FE_OK;
    if (!x || !w || !q_w || !k_w || !positions || !qkv)
        return fail(FE_ERR_INVALID_ARGUMENT, std::string(name) + ": null pointer");
    if (!aligned16(x) || !aligned16(w) || !aligned16(qkv))
        return fail(FE_ERR_INVALID_ARGUMENT, std::string(name) + ": pointers must be 16-byte aligned");
    fe_status st = FE_OK;
    cudaError_t e = fe::launch_linear_qk_norm_rope(x, w, qkv, m, k, q_heads, kv_heads, head_dim, q_w, k_w, positions,
                                                   one_plus != 0, eps, theta, reinterpret_cast<cudaStream_t>(stream),
                                                   &st, row_ss, ss_parts);
    if (st != FE_OK) return st;
    return done(e, name);
}

fe_status fe_linear_qk_norm_rope_bf16(const void *x, const void *w, const float *q_w, const float *k_w,
                                      const int32_t *positions, void *qkv, int64_t m, int64_t k, int32_t q_heads,
                                      int32_t kv_heads, int32_t head_dim, int32_t one_plus, float eps, float theta,
                                      fe_stream_t stream)
{
    return qk_norm_rope_call("fe_linear_qk_norm_rope_bf16", x, w, q_w, k_w, positions, qkv, m, k, q_heads, kv_heads,
                             head_dim, one_plus, eps, theta, nullptr, 0, stream);
}

fe_status fe_linear_qk_norm_rope_scaled_bf16(const void *x, const void *w, const float *q_w, const float *k_w,
                                             const int32_t *positions, void *qkv, int64_t m, int64_t k,
                                             int32_t q_heads, int32_t kv_heads, int32_t head_dim, int32_t one_plus,
                                             float eps, float theta, const float *row_ss, int32_t ss_parts,
                                             fe_stream_t stream)
{
    if (ss_parts < 1 || ss_parts > 8)
        return fail(FE_ERR_INVALID_ARGUMENT, "fe_linear_qk_norm_rope_scaled_bf16: ss_parts must be 1..8");
    if (m > 0 && !row_ss) return fail(FE_ERR_INVALID_ARGUMENT, "fe_linear_qk_norm_rope_scaled_bf16: null pointer");
    return qk_norm_rope_call("fe_linear_qk_norm_rope_scaled_bf16", x, w, q_w, k_w, positions, qkv, m, k, q_heads,
                             kv_heads, head_dim, one_plus, eps, theta, row_ss, ss_parts, stream);
}

fe_status fe_token_positions(const int32_t *cu_seqlens, int32_t batch, int32_t *positions, fe_stream_t stream)
{
    if (batch < 0) return fail(FE_ERR_INVALID_ARGUMENT, "fe_token_positions: bad batch");
    if (batch == 0) return FE_OK;
    if (!cu_seqlens || !positions) return fail(FE_ERR_INVALID_ARGUMENT, "fe_token_positions: null pointer");
    return done(fe::launch_token_positions(cu_seqlens, batch, positions, reinterpret_cast<cudaStream_t>(stream)),
                "fe_token_positions");
}

fe_status fe_pool_l2(const float *h, const int32_t *cu_seqlens, int32_t batch, int32_t dim, fe_pooling mode,
                     float *out, fe_stream_t stream)
{
    if (batch < 0 || dim <= 0) return fail(FE_ERR_INVALID_ARGUMENT, "fe_pool_l2: bad shape");
    if (mode != FE_POOL_CLS && mode != FE_POOL_MEAN && mode != FE_POOL_LAST)
        return fail(FE_ERR_INVALID_ARGUMENT, "fe_pool_l2: unknown pooling mode");
    if (batch == 0) return FE_OK;
    if (!h || !cu_seqlens || !out) return fail(FE_ERR_INVALID_ARGUMENT, "fe_pool_l2: null pointer");
    return done(fe::launch_pool_l2(h, cu_seqlens, batch, dim, mode, out, reinterpret_cast<cudaStream_t>(stream)),
                "fe_pool_l2");
}

// ------------------------------------------------------------ host-only helpers
}  // extern "C"

namespace {
// Greedy prefix cuts: cut r goes to the sentence boundary nearest total * r / parts
// (ties to the earlier boundary), never before the previous cut.
void cut_prefix(const std::vector<double> &prefix, int32_t batch, int32_t parts, int32_t *cuts)
{
    const double total = prefix[batch];
    int32_t lo = 0;
    for (int32_t r = 1; r < parts; ++r) {
        const double target = total * r / parts;
        int32_t i = static_cast<int32_t>(std::lower_bound(prefix.begin(), prefix.end(), target) - prefix.begin());
        if (i > 0 && (i > batch || target - prefix[i - 1] <= prefix[i] - target)) --i;
        i = std::min(std::max(i, lo), batch);
        cuts[r - 1] = i;
        lo = i;
    }
}
}  // namespace

extern "C" {

fe_status fe_plan_shards(const fe_encoder_config *cfg, const int32_t *sorted_lengths, int32_t batch, int32_t parts,
                         int32_t *cuts)
{
    if (!cfg || batch < 0 || parts < 1 || (batch && !sorted_lengths) || (parts > 1 && !cuts))
        return fail(FE_ERR_INVALID_ARGUMENT, "fe_plan_shards: bad arguments");
    // A sentence's cost in projection FLOPs: its GEMM FLOPs plus, per head and layer, one
    // attention-tile cost for each (128-query, 128-key) tile it occupies.  The attention
    // kernel's time goes by tiles, not FLOPs (a 40-token sentence takes a whole tile), and a
    // tile takes about the time of three times its full-tile FLOPs (4 x 128 x 128 x head_dim)
    // at the projections' rate (bge-large batch on a B200: 2.23 ms for 7,952 tiles against
    // 14.98 ms for 16.0 TFLOP of projections).  Slices of equal cost finish together.
    const double D = cfg->hidden, F = cfg->intermediate, hd = static_cast<double>(cfg->hidden) / cfg->heads;
    const double tile = 3.0 * 4.0 * 128.0 * 128.0 * hd;
    std::vector<double> prefix(static_cast<size_t>(batch) + 1, 0.0);
    for (int32_t i = 0; i < batch; ++i) {
        const double L = sorted_lengths[i];
        if (i && sorted_lengths[i] > sorted_lengths[i - 1])
            return fail(FE_ERR_INVALID_ARGUMENT, "fe_plan_shards: lengths must be sorted in descending order");
        const double tiles = std::ceil(L / 128.0);
        prefix[i + 1] = prefix[i] + cfg->layers * (2.0 * L * (4 * D * D + 2 * D * F) + cfg->heads * tiles * tiles * tile);
    }
    cut_prefix(prefix, batch, parts, cuts);
    return FE_OK;
}

fe_status fe_plan_shards_costs(const double *costs, int32_t batch, int32_t parts, int32_t *cuts)
{
    if (batch < 0 || parts < 1 || (batch && !costs) || (parts > 1 && !cuts))
        return fail(FE_ERR_INVALID_ARGUMENT, "fe_plan_shards_costs: bad arguments");
    std::vector<double> prefix(static_cast<size_t>(batch) + 1, 0.0);
    for (int32_t i = 0; i < batch; ++i) {
        if (!std::isfinite(costs[i]) || costs[i] < 0)
            return fail(FE_ERR_INVALID_ARGUMENT, "fe_plan_shards_costs: costs must be finite and non-negative");
        prefix[i + 1] = prefix[i] + costs[i];
    }
    cut_prefix(prefix, batch, parts, cuts);
    return FE_OK;
}

fe_status fe_pack_batch(const int32_t *ids, const int32_t *lengths, int32_t batch, int32_t stride,
                        int32_t *ids_packed, int32_t *cu_seqlens)
{
    if (batch < 0 || stride < 0 || (batch && (!ids || !lengths || !cu_seqlens)))
        return fail(FE_ERR_INVALID_ARGUMENT, "fe_pack_batch: bad arguments");
    int64_t off = 0;
    if (cu_seqlens) cu_seqlens[0] = 0;
    for (int32_t b = 0; b < batch; ++b) {
        const int32_t L = lengths[b];
        if (L < 0 || L > stride) return fail(FE_ERR_INVALID_ARGUMENT, "fe_pack_batch: length outside [0, stride]");
        if (off + L > 0x7fffffff) return fail(FE_ERR_UNSUPPORTED, "fe_pack_batch: too many tokens");
        if (L && !ids_packed) return fail(FE_ERR_INVALID_ARGUMENT, "fe_pack_batch: null output");
        std::copy(ids + static_cast<int64_t>(b) * stride, ids + static_cast<int64_t>(b) * stride + L, ids_packed + off);
        off += L;
        cu_seqlens[b + 1] = static_cast<int32_t>(off);
    }
    return FE_OK;
}

}  // extern "C"
