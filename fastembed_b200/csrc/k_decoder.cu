// k_decoder.cu — row kernels of the RMSNorm / RoPE encoders (Qwen3, Gemma3 shapes).
// These models are not in the reference; the arithmetic follows their model
// definitions: RMSNorm y = x / sqrt(mean(x^2) + eps) * w (Qwen3) or * (1 + w) (Gemma3),
// computed in fp32; rotary embeddings in the rotate-half form with inverse frequencies
// theta^(-2i/d), positions counted from 0 within each sentence.  One warp per row or per
// token; HBM-bound.
#include <cuda_bf16.h>

#include "fe_common.cuh"
#include "fe_internal.h"

namespace fe {
namespace {

unsigned grid_rows(int64_t rows, int per_block) { return static_cast<unsigned>((rows + per_block - 1) / per_block); }

// Sentence of token t: last s with cu[s] <= t.
__device__ __forceinline__ int sentence_of(const int32_t *cu, int batch, int64_t t)
{
    int lo = 0, hi = batch - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (cu[mid] <= t) lo = mid;
        else hi = mid - 1;
    }
    return lo;
}

// h32[t] = word[ids[t]] * scale.  Out-of-range ids record FE_ERR_INVALID_ARGUMENT and
// write zeros.
template <int VPT>
__global__ void __launch_bounds__(256)
    embed_scale(const int32_t *__restrict__ ids, int64_t total, const float *__restrict__ word, int vocab, float scale,
                float *__restrict__ h32, int *status)
{
    constexpr int dim = 128 * VPT;
    const int64_t t = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    grid_dep_wait();
    grid_dep_launch();
    if (t >= total) return;
    const int id = ids[t];
    float *o = h32 + t * dim;
    const bool ok = id >= 0 && id < vocab;
    if (!ok && lane == 0) report(status, DEV_BAD_INPUT);
    const float *w = word + static_cast<int64_t>(ok ? id : 0) * dim;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        const int col = (i * 32 + lane) * 4;
        float4 a = ok ? __ldg(reinterpret_cast<const float4 *>(w + col)) : make_float4(0.f, 0.f, 0.f, 0.f);
        a.x *= scale;
        a.y *= scale;
        a.z *= scale;
        a.w *= scale;
        *reinterpret_cast<float4 *>(o + col) = a;
    }
}

// x (registers) -> x / sqrt(mean(x^2) + eps) * (w or 1 + w), written as fp32 and / or bf16.
template <int VPT>
__device__ __forceinline__ void rms_store(float4 (&x)[VPT], const float *__restrict__ w, int one_plus, float eps,
                                          int lane, float *o32, __nv_bfloat16 *o16)
{
    constexpr int dim = 128 * VPT;
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) s += (x[i].x * x[i].x + x[i].y * x[i].y) + (x[i].z * x[i].z + x[i].w * x[i].w);
    const float r = rsqrtf(warp_sum(s) / static_cast<float>(dim) + eps);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        const int col = (i * 32 + lane) * 4;
        float4 g = __ldg(reinterpret_cast<const float4 *>(w + col));
        if (one_plus) {
            g.x += 1.f;
            g.y += 1.f;
            g.z += 1.f;
            g.w += 1.f;
        }
        const float4 y = make_float4(x[i].x * r * g.x, x[i].y * r * g.y, x[i].z * r * g.z, x[i].w * r * g.w);
        if (o32) *reinterpret_cast<float4 *>(o32 + col) = y;
        if (o16) *reinterpret_cast<uint2 *>(o16 + col) = make_uint2(pack_bf16x2(y.x, y.y), pack_bf16x2(y.z, y.w));
    }
}

// out = RMSNorm(x) as fp32 and / or bf16.
template <int VPT>
__global__ void __launch_bounds__(256)
    rms_norm_rows(const float *__restrict__ x, const float *__restrict__ w, int one_plus, float eps, int64_t rows,
                  float *__restrict__ o32, __nv_bfloat16 *__restrict__ o16)
{
    constexpr int dim = 128 * VPT;
    const int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    grid_dep_wait();
    grid_dep_launch();
    if (r >= rows) return;
    float4 v[VPT];
#pragma unroll
    for (int i = 0; i < VPT; ++i) v[i] = *reinterpret_cast<const float4 *>(x + r * dim + (i * 32 + lane) * 4);
    rms_store<VPT>(v, w, one_plus, eps, lane, o32 ? o32 + r * dim : nullptr, o16 ? o16 + r * dim : nullptr);
}

// Sandwich norm step: h32 += RMSNorm(y; w_post), then out = RMSNorm(h32; w_next) as fp32
// and / or bf16 (the post-attention / post-FFN norms of Gemma3 followed by the next pre-norm).
// YT: the type of y (float, or __nv_bfloat16 for a projection written in bf16).
template <int VPT, class YT>
__global__ void __launch_bounds__(256)
    rms_sandwich(const YT *__restrict__ y, const float *__restrict__ w_post, float *__restrict__ h32,
                 const float *__restrict__ w_next, int one_plus, float eps, int64_t rows, float *__restrict__ o32,
                 __nv_bfloat16 *__restrict__ o16)
{
    constexpr int dim = 128 * VPT;
    const int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    grid_dep_wait();
    grid_dep_launch();
    if (r >= rows) return;
    float4 v[VPT];
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        if constexpr (sizeof(YT) == 4) {
            v[i] = *reinterpret_cast<const float4 *>(y + r * dim + (i * 32 + lane) * 4);
        } else {
            const uint2 u = *reinterpret_cast<const uint2 *>(y + r * dim + (i * 32 + lane) * 4);
            const float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y);
            v[i] = make_float4(a.x, a.y, b.x, b.y);
        }
    }
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) s += (v[i].x * v[i].x + v[i].y * v[i].y) + (v[i].z * v[i].z + v[i].w * v[i].w);
    const float rr = rsqrtf(warp_sum(s) / static_cast<float>(dim) + eps);
    float *hr = h32 + r * dim;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        const int col = (i * 32 + lane) * 4;
        float4 g = __ldg(reinterpret_cast<const float4 *>(w_post + col));
        if (one_plus) {
            g.x += 1.f;
            g.y += 1.f;
            g.z += 1.f;
            g.w += 1.f;
        }
        const float4 h = *reinterpret_cast<const float4 *>(hr + col);
        v[i] = make_float4(h.x + v[i].x * rr * g.x, h.y + v[i].y * rr * g.y, h.z + v[i].z * rr * g.z,
                           h.w + v[i].w * rr * g.w);
        *reinterpret_cast<float4 *>(hr + col) = v[i];
    }
    rms_store<VPT>(v, w_next, one_plus, eps, lane, o32 ? o32 + r * dim : nullptr, o16 ? o16 + r * dim : nullptr);
}

// Per-head RMSNorm and rotary embedding of the query and key heads, in place on the bf16
// qkv buffer [T, (q_heads + 2 kv_heads) * HD].  One warp per token: the rotation angles
// depend only on (position, frequency), so each lane computes the cos / sin of its E = HD/32
// elements once and applies them to every query and key head of the token.  Lane l holds
// elements [E * l, E * (l + 1)) of a head; its rotation partner (i +- HD/2) is in lane l ^ 16.
template <int HD>
__device__ __forceinline__ void load_head(const __nv_bfloat16 *p, float (&x)[HD / 32])
{
    if constexpr (HD == 128) {
        const uint2 u = *reinterpret_cast<const uint2 *>(p);
        const float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y);
        x[0] = a.x, x[1] = a.y, x[2] = b.x, x[3] = b.y;
    } else {
        const uint4 u = *reinterpret_cast<const uint4 *>(p);
        const float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y), c = unpack_bf16x2(u.z), d = unpack_bf16x2(u.w);
        x[0] = a.x, x[1] = a.y, x[2] = b.x, x[3] = b.y, x[4] = c.x, x[5] = c.y, x[6] = d.x, x[7] = d.y;
    }
}

template <int HD>
__device__ __forceinline__ void store_head(__nv_bfloat16 *p, const float (&y)[HD / 32])
{
    if constexpr (HD == 128) {
        *reinterpret_cast<uint2 *>(p) = make_uint2(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]));
    } else {
        *reinterpret_cast<uint4 *>(p) = make_uint4(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]),
                                                   pack_bf16x2(y[4], y[5]), pack_bf16x2(y[6], y[7]));
    }
}

// pos[t] = t - (first token of t's sentence) for the packed batch: one warp per sentence.
// Built once per forward pass; every layer's qk_norm_rope then reads a token's position
// instead of searching cu_seqlens for its sentence.
__global__ void __launch_bounds__(256)
    token_positions(const int32_t *__restrict__ cu, int batch, int32_t *__restrict__ pos)
{
    const int s = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    grid_dep_wait();
    grid_dep_launch();
    if (s >= batch) return;
    const int start = cu[s], len = cu[s + 1] - start;
    for (int i = lane; i < len; i += 32) pos[start + i] = i;
}

// At head_dim 256, five resident blocks per SM (48 registers) measured 5 % faster than four
// (59 registers); at 128 the same bound made it 10 % slower, and grouping 2 or 4 heads per
// pass (more loads in flight, more registers) made 256 slower.
template <int HD>
__global__ void __launch_bounds__(256, HD == 256 ? 5 : 0)
    qk_norm_rope(__nv_bfloat16 *qkv, const int32_t *__restrict__ cu, const int32_t *__restrict__ tpos, int batch,
                 int64_t total, int q_heads, int kv_heads, const float *__restrict__ q_w, const float *__restrict__ k_w,
                 int one_plus, float eps, float log2_theta)
{
    constexpr int E = HD / 32;
    const int64_t t = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    grid_dep_wait();
    grid_dep_launch();
    if (t >= total) return;
    // the token's position in its sentence: from the positions array when given, else by
    // binary search of cu_seqlens
    const int pos = tpos ? tpos[t] : static_cast<int>(t - cu[sentence_of(cu, batch, t)]);
    float cs[E], sn[E], wq[E], wk[E];
    const int f0 = (E * lane) & (HD / 2 - 1);  // this lane's first frequency index (E in a row)
#pragma unroll
    for (int i = 0; i < E; ++i) rope_angle<HD>(pos, f0 + i, log2_theta, sn[i], cs[i]);
#pragma unroll
    for (int i = 0; i < E; ++i) {
        const int e = E * lane + i;
        wq[i] = q_w[e] + (one_plus ? 1.f : 0.f);
        wk[i] = k_w[e] + (one_plus ? 1.f : 0.f);
    }
    const bool lo = lane < 16;  // elements i < HD/2
    __nv_bfloat16 *row = qkv + t * static_cast<int64_t>(q_heads + 2 * kv_heads) * HD + E * lane;
    const int nh = q_heads + kv_heads;
    // Heads in groups of G: the group's loads are issued together and its G row
    // reductions run interleaved.
    constexpr int G = HD == 128 ? 4 : 1;
#pragma unroll(HD == 128 ? 1 : 2)
    for (int h0 = 0; h0 < nh; h0 += G) {
        float x[G][E];
        float ss[G];
#pragma unroll
        for (int g = 0; g < G; ++g) {
            ss[g] = 0.f;
            if (h0 + g < nh) load_head<HD>(row + (h0 + g) * HD, x[g]);
        }
#pragma unroll
        for (int g = 0; g < G; ++g)
            if (h0 + g < nh) {
#pragma unroll
                for (int i = 0; i < E; ++i) ss[g] += x[g][i] * x[g][i];
            }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
            for (int g = 0; g < G; ++g) ss[g] += __shfl_xor_sync(0xffffffffu, ss[g], o);
#pragma unroll
        for (int g = 0; g < G; ++g) {
            if (h0 + g >= nh) continue;
            const float r = rsqrtf(ss[g] / static_cast<float>(HD) + eps);
            const bool is_q = h0 + g < q_heads;
            float xs[E], y[E];
#pragma unroll
            for (int i = 0; i < E; ++i) xs[i] = x[g][i] * r * (is_q ? wq[i] : wk[i]);
#pragma unroll
            for (int i = 0; i < E; ++i) {
                const float partner = __shfl_xor_sync(0xffffffffu, xs[i], 16);
                y[i] = lo ? xs[i] * cs[i] - partner * sn[i] : xs[i] * cs[i] + partner * sn[i];
            }
            store_head<HD>(row + (h0 + g) * HD, y);
        }
    }
}

}  // namespace

#define FE_ROW_DISPATCH2(KERNEL, T2, DIM, ...)                                                        \
    {                                                                                                 \
        cudaError_t fe_e_ = cudaSuccess;                                                              \
        switch (DIM) {                                                                                \
        case 256: fe_e_ = launch_k(KERNEL<2, T2>, dim3(grid), dim3(256), 0, s, __VA_ARGS__); break;   \
        case 384: fe_e_ = launch_k(KERNEL<3, T2>, dim3(grid), dim3(256), 0, s, __VA_ARGS__); break;   \
        case 512: fe_e_ = launch_k(KERNEL<4, T2>, dim3(grid), dim3(256), 0, s, __VA_ARGS__); break;   \
        case 768: fe_e_ = launch_k(KERNEL<6, T2>, dim3(grid), dim3(256), 0, s, __VA_ARGS__); break;   \
        case 1024: fe_e_ = launch_k(KERNEL<8, T2>, dim3(grid), dim3(256), 0, s, __VA_ARGS__); break;  \
        case 1536: fe_e_ = launch_k(KERNEL<12, T2>, dim3(grid), dim3(256), 0, s, __VA_ARGS__); break; \
        case 2048: fe_e_ = launch_k(KERNEL<16, T2>, dim3(grid), dim3(256), 0, s, __VA_ARGS__); break; \
        default: return cudaErrorInvalidValue;                                                        \
        }                                                                                             \
        if (fe_e_ != cudaSuccess) return fe_e_;                                                       \
    }

#define FE_ROW_DISPATCH(KERNEL, DIM, ...)                                                         \
    {                                                                                             \
        cudaError_t fe_e_ = cudaSuccess;                                                          \
        switch (DIM) {                                                                            \
        case 256: fe_e_ = launch_k(KERNEL<2>, dim3(grid), dim3(256), 0, s, __VA_ARGS__); break;   \
        case 384: fe_e_ = launch_k(KERNEL<3>, dim3(grid), dim3(256), 0, s, __VA_ARGS__); break;   \
        case 512: fe_e_ = launch_k(KERNEL<4>, dim3(grid), dim3(256), 0, s, __VA_ARGS__); break;   \
        case 768: fe_e_ = launch_k(KERNEL<6>, dim3(grid), dim3(256), 0, s, __VA_ARGS__); break;   \
        case 1024: fe_e_ = launch_k(KERNEL<8>, dim3(grid), dim3(256), 0, s, __VA_ARGS__); break;  \
        case 1536: fe_e_ = launch_k(KERNEL<12>, dim3(grid), dim3(256), 0, s, __VA_ARGS__); break; \
        case 2048: fe_e_ = launch_k(KERNEL<16>, dim3(grid), dim3(256), 0, s, __VA_ARGS__); break; \
        default: return cudaErrorInvalidValue;                                                    \
        }                                                                                         \
        if (fe_e_ != cudaSuccess) return fe_e_;                                                   \
    }

cudaError_t launch_embed_scale(const int32_t *ids, int64_t total, const float *word, int vocab, int dim, float scale,
                               float *h32, cudaStream_t s)
{
    if (total == 0) return cudaSuccess;
    const unsigned grid = grid_rows(total, 8);
    int *st = current_device_status_word();
    FE_ROW_DISPATCH(embed_scale, dim, ids, total, word, vocab, scale, h32, st)
    return cudaGetLastError();
}

cudaError_t launch_rms_norm_rows(const float *x, const float *w, bool one_plus, float eps, int64_t rows, int dim,
                                 float *o32, void *o16, cudaStream_t s)
{
    if (rows == 0) return cudaSuccess;
    const unsigned grid = grid_rows(rows, 8);
    auto *b16 = static_cast<__nv_bfloat16 *>(o16);
    FE_ROW_DISPATCH(rms_norm_rows, dim, x, w, one_plus ? 1 : 0, eps, rows, o32, b16)
    return cudaGetLastError();
}

cudaError_t launch_rms_sandwich(const void *y, const float *w_post, float *h32, const float *w_next, bool one_plus,
                                float eps, int64_t rows, int dim, float *o32, void *o16, cudaStream_t s, bool y_bf16)
{
    if (rows == 0) return cudaSuccess;
    const unsigned grid = grid_rows(rows, 8);
    auto *b16 = static_cast<__nv_bfloat16 *>(o16);
    if (y_bf16) {
        const auto *yb = static_cast<const __nv_bfloat16 *>(y);
        FE_ROW_DISPATCH2(rms_sandwich, __nv_bfloat16, dim, yb, w_post, h32, w_next, one_plus ? 1 : 0, eps, rows, o32,
                         b16)
    } else {
        const auto *yf = static_cast<const float *>(y);
        FE_ROW_DISPATCH2(rms_sandwich, float, dim, yf, w_post, h32, w_next, one_plus ? 1 : 0, eps, rows, o32, b16)
    }
    return cudaGetLastError();
}
#undef FE_ROW_DISPATCH
#undef FE_ROW_DISPATCH2

cudaError_t launch_token_positions(const int32_t *cu, int batch, int32_t *pos, cudaStream_t s)
{
    if (batch == 0) return cudaSuccess;
    return launch_k(token_positions, dim3(grid_rows(batch, 8)), dim3(256), 0, s, cu, batch, pos);
}

cudaError_t launch_qk_norm_rope(void *qkv, const int32_t *cu, int batch, int64_t total, int q_heads, int kv_heads,
                                int head_dim, const float *q_w, const float *k_w, bool one_plus, float eps, float theta,
                                cudaStream_t s, const int32_t *pos)
{
    if (total == 0) return cudaSuccess;
    const unsigned grid = grid_rows(total, 8);
    auto *p = static_cast<__nv_bfloat16 *>(qkv);
    const float lt = log2f(theta);
    if (head_dim == 128)
        return launch_k(qk_norm_rope<128>, dim3(grid), dim3(256), 0, s, p, cu, pos, batch, total, q_heads, kv_heads,
                        q_w, k_w, one_plus ? 1 : 0, eps, lt);
    if (head_dim == 256)
        return launch_k(qk_norm_rope<256>, dim3(grid), dim3(256), 0, s, p, cu, pos, batch, total, q_heads, kv_heads,
                        q_w, k_w, one_plus ? 1 : 0, eps, lt);
    return cudaErrorInvalidValue;
}

}  // namespace fe
