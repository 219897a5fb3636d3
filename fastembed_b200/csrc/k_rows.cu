// k_rows.cu — memory-bound row kernels of the encoder pipeline: fused embedding
// sum + LayerNorm, LayerNorm with fp32 + bf16 outputs, pooling + L2 normalise, and
// the fp32 -> bf16 weight conversion.  All are HBM-bound: one warp per row, float4
// loads, two-pass statistics held in registers, warp-shuffle reductions.
#include <cuda_bf16.h>

#include "fe_common.cuh"
#include "fe_internal.h"

namespace fe {
namespace {

// Row LayerNorm of VPT float4 per lane (dim = 128 * VPT), values already in
// registers; writes fp32 and (optionally) bf16.  Two-pass mean / variance as in
// src/ops/cpu/cpu_matrix_ops.cpp:64-92, normalised with a true division.
template <int VPT>
__device__ __forceinline__ void ln_store(float4 (&x)[VPT], const float *__restrict__ g,
                                         const float *__restrict__ b, float *__restrict__ y32,
                                         __nv_bfloat16 *__restrict__ y16, int dim, float eps, int lane)
{
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) s += (x[i].x + x[i].y) + (x[i].z + x[i].w);
    const float mean = warp_sum(s) / static_cast<float>(dim);
    float v = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        const float a = x[i].x - mean, bb = x[i].y - mean, c = x[i].z - mean, d = x[i].w - mean;
        v += (a * a + bb * bb) + (c * c + d * d);
    }
    const float var = warp_sum(v) / static_cast<float>(dim);
    const float sd = sqrtf(var + eps);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        const int col = (i * 32 + lane) * 4;
        const float4 gg = __ldg(reinterpret_cast<const float4 *>(g + col));
        const float4 bv = __ldg(reinterpret_cast<const float4 *>(b + col));
        float4 o;
        o.x = (x[i].x - mean) / sd * gg.x + bv.x;
        o.y = (x[i].y - mean) / sd * gg.y + bv.y;
        o.z = (x[i].z - mean) / sd * gg.z + bv.z;
        o.w = (x[i].w - mean) / sd * gg.w + bv.w;
        *reinterpret_cast<float4 *>(y32 + col) = o;
        if (y16) {
            uint2 p;
            p.x = pack_bf16x2(o.x, o.y);
            p.y = pack_bf16x2(o.z, o.w);
            *reinterpret_cast<uint2 *>(y16 + col) = p;
        }
    }
}

// Token t of sentence s: x = word[id] + pos[row] + type[0] (summed in that order,
// src/sentence_transformers_impl.cpp:30-44, :139-188), then LayerNorm (:189-194).  The
// position row is t - start(s) (BERT), or with pad_id >= 0 the bge-m3 / XLM-R row
// (:101-123, :146-149): 0 for a token equal to pad_id, else 2 + the number of non-pad
// tokens before it in the sentence (counted by the warp, 32 ids per step), a row at or
// past max_pos becoming 0.
template <int VPT>
__global__ void __launch_bounds__(256)
    embed_ln(const int32_t *__restrict__ ids, const int32_t *__restrict__ cu, int batch, int64_t total,
             const float *__restrict__ word, const float *__restrict__ pos, const float *__restrict__ type,
             const float *__restrict__ g, const float *__restrict__ b, int vocab, int max_pos, int pad_id, float eps,
             float *__restrict__ h32, __nv_bfloat16 *__restrict__ h16, int *status)
{
    constexpr int dim = 128 * VPT;
    const int64_t t = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    grid_dep_wait();
    grid_dep_launch();
    if (t >= total) return;
    // sentence of token t: last s with cu[s] <= t
    int lo = 0, hi = batch - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (cu[mid] <= t) lo = mid; else hi = mid - 1;
    }
    const int id = ids[t];
    int p = static_cast<int>(t - cu[lo]);
    if (pad_id >= 0) {
        int before = 0;  // non-pad tokens in [start(s), t)
        for (int64_t j0 = cu[lo]; j0 < t; j0 += 32) {
            const int64_t j = j0 + lane;
            before += __popc(__ballot_sync(0xffffffffu, j < t && ids[j] != pad_id));
        }
        p = id == pad_id ? 0 : 2 + before;
        if (p >= max_pos) p = 0;
    }
    float *o32 = h32 + t * dim;
    __nv_bfloat16 *o16 = h16 ? h16 + t * dim : nullptr;
    if (id < 0 || id >= vocab || p < 0 || p >= max_pos) {
        if (lane == 0) report(status, DEV_BAD_INPUT);
#pragma unroll
        for (int i = 0; i < VPT; ++i) {
            const int col = (i * 32 + lane) * 4;
            *reinterpret_cast<float4 *>(o32 + col) = make_float4(0.f, 0.f, 0.f, 0.f);
            if (o16) *reinterpret_cast<uint2 *>(o16 + col) = make_uint2(0u, 0u);
        }
        return;
    }
    const float *wr = word + static_cast<int64_t>(id) * dim;
    const float *pr = pos + static_cast<int64_t>(p) * dim;
    float4 x[VPT];
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        const int col = (i * 32 + lane) * 4;
        const float4 a = __ldg(reinterpret_cast<const float4 *>(wr + col));
        const float4 c = __ldg(reinterpret_cast<const float4 *>(pr + col));
        const float4 d = __ldg(reinterpret_cast<const float4 *>(type + col));
        x[i] = make_float4((a.x + c.x) + d.x, (a.y + c.y) + d.y, (a.z + c.z) + d.z, (a.w + c.w) + d.w);
    }
    ln_store<VPT>(x, g, b, o32, o16, dim, eps, lane);
}

// h = LayerNorm(y [+ res]) with fp32 and bf16 outputs.  With `res`, the sum y + res is
// formed here (y already holds x W^T + b), the order of the reference's residual add
// (src/sentence_transformers_impl.cpp:255-263, :429-436).  h32 may alias res: every
// element is read before the thread that owns it writes it.
template <int VPT, class IT = float>
__global__ void __launch_bounds__(256)
    ln_dual(const IT *__restrict__ in, const float *res, const float *__restrict__ g, const float *__restrict__ b,
            float *h32, __nv_bfloat16 *__restrict__ h16, int64_t rows, float eps)
{
    constexpr int dim = 128 * VPT;
    const int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    grid_dep_wait();
    grid_dep_launch();
    if (r >= rows) return;
    const IT *src = in + r * dim;
    float4 x[VPT];
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        if constexpr (sizeof(IT) == 4) {
            x[i] = *reinterpret_cast<const float4 *>(src + (i * 32 + lane) * 4);
        } else {  // a projection written in bf16, widened
            const uint2 u = *reinterpret_cast<const uint2 *>(src + (i * 32 + lane) * 4);
            const float2 p = unpack_bf16x2(u.x), q = unpack_bf16x2(u.y);
            x[i] = make_float4(p.x, p.y, q.x, q.y);
        }
    }
    if (res) {
        const float *rr = res + r * dim;
#pragma unroll
        for (int i = 0; i < VPT; ++i) {
            const float4 a = *reinterpret_cast<const float4 *>(rr + (i * 32 + lane) * 4);
            x[i].x += a.x;
            x[i].y += a.y;
            x[i].z += a.z;
            x[i].w += a.w;
        }
    }
    ln_store<VPT>(x, g, b, h32 + r * dim, h16 ? h16 + r * dim : nullptr, dim, eps, lane);
}

// Generic-width LayerNorm (any dim): one block per row, block reductions.
__device__ float block_sum(float v, float *red)
{
    v = warp_sum(v);
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) red[w] = v;
    __syncthreads();
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    if (w == 0) t = warp_sum(t);
    if (threadIdx.x == 0) red[32] = t;
    __syncthreads();
    return red[32];
}

__device__ float block_max(float v, float *red)
{
    v = warp_max(v);
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) red[w] = v;
    __syncthreads();
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : -INFINITY;
    if (w == 0) t = warp_max(t);
    if (threadIdx.x == 0) red[32] = t;
    __syncthreads();
    return red[32];
}

__global__ void __launch_bounds__(256)
    ln_generic(const float *__restrict__ in, const float *__restrict__ g, const float *__restrict__ b,
               float *__restrict__ h32, __nv_bfloat16 *__restrict__ h16, int64_t dim, float eps)
{
    __shared__ float red[33];
    const float *x = in + static_cast<int64_t>(blockIdx.x) * dim;  // (no residual form: dims the fast path lacks)
    float s = 0.f;
    for (int64_t i = threadIdx.x; i < dim; i += blockDim.x) s += x[i];
    const float mean = block_sum(s, red) / static_cast<float>(dim);
    float v = 0.f;
    for (int64_t i = threadIdx.x; i < dim; i += blockDim.x) {
        const float d = x[i] - mean;
        v += d * d;
    }
    const float var = block_sum(v, red) / static_cast<float>(dim);
    const float sd = sqrtf(var + eps);
    float *y = h32 + static_cast<int64_t>(blockIdx.x) * dim;
    for (int64_t i = threadIdx.x; i < dim; i += blockDim.x) {
        const float o = (x[i] - mean) / sd * g[i] + b[i];
        y[i] = o;
        if (h16) h16[static_cast<int64_t>(blockIdx.x) * dim + i] = __float2bfloat16_rn(o);
    }
}

// RMSNorm, src/ops/cpu/cpu_matrix_ops.cpp:95-121: inv = 1/sqrt(mean(x^2)+eps); y = inv*w*x.
__global__ void __launch_bounds__(256)
    rms_generic(const float *__restrict__ in, const float *__restrict__ w, float *__restrict__ out,
                int64_t dim, float eps)
{
    __shared__ float red[33];
    const float *x = in + static_cast<int64_t>(blockIdx.x) * dim;
    float s = 0.f;
    for (int64_t i = threadIdx.x; i < dim; i += blockDim.x) s += x[i] * x[i];
    float ms = block_sum(s, red) / static_cast<float>(dim);
    const float inv = 1.0f / sqrtf(ms + eps);
    float *y = out + static_cast<int64_t>(blockIdx.x) * dim;
    for (int64_t i = threadIdx.x; i < dim; i += blockDim.x) y[i] = inv * w[i] * x[i];
}

// Row softmax, src/ops/cpu/cpu_matrix_ops.cpp:141-163 (in == out allowed).
__global__ void __launch_bounds__(256)
    softmax_generic(const float *in, float *out, int64_t dim)
{
    __shared__ float red[33];
    const float *x = in + static_cast<int64_t>(blockIdx.x) * dim;
    float *y = out + static_cast<int64_t>(blockIdx.x) * dim;
    float m = -INFINITY;
    for (int64_t i = threadIdx.x; i < dim; i += blockDim.x) m = fmaxf(m, x[i]);
    m = block_max(m, red);
    float s = 0.f;
    for (int64_t i = threadIdx.x; i < dim; i += blockDim.x) {
        const float e = expf(x[i] - m);
        y[i] = e;
        s += e;
    }
    s = block_sum(s, red);
    for (int64_t i = threadIdx.x; i < dim; i += blockDim.x) y[i] = y[i] / s;
}

// Pooling + L2 (src/sentence_transformers_impl.cpp:289-341): one warp per sentence (the CLS
// and last-token rows; mean pooling of dims that pool_mean_l2 does not take).
__global__ void __launch_bounds__(256)
    pool_l2(const float *__restrict__ h, const int32_t *__restrict__ cu, int batch, int dim, int mode,
            float *__restrict__ out)
{
    const int s = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    grid_dep_wait();
    grid_dep_launch();
    if (s >= batch) return;
    const int start = cu[s], len = cu[s + 1] - cu[s];
    float *o = out + static_cast<int64_t>(s) * dim;
    if (len <= 0) {
        for (int c = lane; c < dim; c += 32) o[c] = 0.f;
        return;
    }
    float ss = 0.f;
    if (mode == FE_POOL_MEAN) {
        for (int c = lane; c < dim; c += 32) {
            float acc = 0.f;
            for (int t = 0; t < len; ++t) acc += h[static_cast<int64_t>(start + t) * dim + c];
            acc /= static_cast<float>(len);
            o[c] = acc;
            ss += acc * acc;
        }
    } else {
        const int row = mode == FE_POOL_LAST ? start + len - 1 : start;
        const float *src = h + static_cast<int64_t>(row) * dim;
        for (int c = lane; c < dim; c += 32) {
            const float v = src[c];
            o[c] = v;
            ss += v * v;
        }
    }
    const float nrm = sqrtf(warp_sum(ss));
    for (int c = lane; c < dim; c += 32) o[c] = o[c] / nrm;
}

// Mean pooling + L2 (src/sentence_transformers_impl.cpp:289-341, the mean branch), one
// block of W warps per sentence: warp w sums the sentence's tokens w, w + W, w + 2W, ... over
// float4 columns (four rows in flight), the W partial sums are added in warp order through
// shared memory ([W][dim] floats), and the mean is L2-normalised.  The summation order
// depends only on the sentence's length, so a sentence gives the same row in any batch.
// Needs dim % 4 == 0 and W * dim * 4 bytes of dynamic shared memory.
template <int W>
__global__ void __launch_bounds__(W * 32)
    pool_mean_l2(const float *__restrict__ h, const int32_t *__restrict__ cu, int dim, float *__restrict__ out)
{
    extern __shared__ float part[];  // [W][dim]
    __shared__ float red[W];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    grid_dep_wait();
    grid_dep_launch();
    const int s = blockIdx.x;
    const int start = cu[s], len = cu[s + 1] - cu[s];
    float *o = out + static_cast<int64_t>(s) * dim;
    if (len <= 0) {
        for (int c = threadIdx.x; c < dim; c += blockDim.x) o[c] = 0.f;
        return;
    }
    const int d4 = dim >> 2;
    const float4 *base = reinterpret_cast<const float4 *>(h + static_cast<int64_t>(start) * dim);
    for (int c4 = lane; c4 < d4; c4 += 32) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
        for (int t = warp; t < len; t += W) {
            const float4 v = __ldg(base + static_cast<int64_t>(t) * d4 + c4);
            acc.x += v.x;
            acc.y += v.y;
            acc.z += v.z;
            acc.w += v.w;
        }
        reinterpret_cast<float4 *>(part + warp * dim)[c4] = acc;
    }
    __syncthreads();
    float ss = 0.f;
    for (int c = threadIdx.x; c < dim; c += blockDim.x) {
        float a = 0.f;
#pragma unroll
        for (int w = 0; w < W; ++w) a += part[w * dim + c];
        a /= static_cast<float>(len);
        part[c] = a;  // column c is read and written by this thread only
        ss += a * a;
    }
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < W; ++w) tot += red[w];
    const float nrm = sqrtf(tot);
    for (int c = threadIdx.x; c < dim; c += blockDim.x) o[c] = part[c] / nrm;
}

__global__ void f32_to_bf16(const float *__restrict__ x, __nv_bfloat16 *__restrict__ y, int64_t n)
{
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        y[i] = __float2bfloat16_rn(x[i]);
}

inline unsigned grid_for(int64_t rows, int per_block) { return static_cast<unsigned>((rows + per_block - 1) / per_block); }

}  // namespace

cudaError_t launch_embed_layernorm(const int32_t *ids, const int32_t *cu, int batch, int64_t total,
                                   const float *word, const float *pos, const float *type,
                                   const float *g, const float *b, int dim, int vocab, int max_pos,
                                   float eps, float *h32, void *h16, cudaStream_t s, int pad_id)
{
    if (total == 0) return cudaSuccess;
    auto *o16 = static_cast<__nv_bfloat16 *>(h16);
    int *st = current_device_status_word();
    const unsigned grid = grid_for(total, 8);
    switch (dim) {
#define FE_EMB(V)                                                                                                \
    case 128 * V:                                                                                                \
        return launch_k(embed_ln<V>, dim3(grid), dim3(256), 0, s, ids, cu, batch, total, word, pos, type, g, b, vocab, \
                        max_pos, pad_id, eps, h32, o16, st);
        FE_EMB(2) FE_EMB(3) FE_EMB(4) FE_EMB(6) FE_EMB(8) FE_EMB(12) FE_EMB(16)
#undef FE_EMB
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_layernorm_dual_bf16in(const void *x, const float *res, const float *g, const float *b, float *h32,
                                         void *h16, int64_t rows, int dim, float eps, cudaStream_t s)
{
    if (rows == 0) return cudaSuccess;
    auto *o16 = static_cast<__nv_bfloat16 *>(h16);
    const auto *xb = static_cast<const __nv_bfloat16 *>(x);
    const unsigned grid = grid_for(rows, 8);
    switch (dim) {
#define FE_LN(V) \
    case 128 * V: return launch_k(ln_dual<V, __nv_bfloat16>, dim3(grid), dim3(256), 0, s, xb, res, g, b, h32, o16, rows, eps);
        FE_LN(1) FE_LN(2) FE_LN(3) FE_LN(4) FE_LN(6) FE_LN(8) FE_LN(12) FE_LN(16)
#undef FE_LN
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_layernorm_dual(const float *x, const float *res, const float *g, const float *b, float *h32,
                                  void *h16, int64_t rows, int dim, float eps, cudaStream_t s)
{
    if (rows == 0) return cudaSuccess;
    auto *o16 = static_cast<__nv_bfloat16 *>(h16);
    const unsigned grid = grid_for(rows, 8);
    switch (dim) {
#define FE_LN(V) \
    case 128 * V: return launch_k(ln_dual<V>, dim3(grid), dim3(256), 0, s, x, res, g, b, h32, o16, rows, eps);
        FE_LN(1) FE_LN(2) FE_LN(3) FE_LN(4) FE_LN(6) FE_LN(8) FE_LN(12) FE_LN(16)
#undef FE_LN
        default:
            if (res) return cudaErrorInvalidValue;
            ln_generic<<<static_cast<unsigned>(rows), 256, 0, s>>>(x, g, b, h32, o16, dim, eps);
    }
    return cudaGetLastError();
}

cudaError_t launch_layer_norm_f32(const float *x, const float *g, const float *b, float *y, int64_t rows,
                                  int64_t dim, float eps, cudaStream_t s)
{
    if (rows == 0) return cudaSuccess;
    ln_generic<<<static_cast<unsigned>(rows), 256, 0, s>>>(x, g, b, y, nullptr, dim, eps);
    return cudaGetLastError();
}

cudaError_t launch_rms_norm_f32(const float *x, const float *w, float *y, int64_t rows, int64_t dim,
                                float eps, cudaStream_t s)
{
    if (rows == 0) return cudaSuccess;
    rms_generic<<<static_cast<unsigned>(rows), 256, 0, s>>>(x, w, y, dim, eps);
    return cudaGetLastError();
}

cudaError_t launch_softmax_rows_f32(const float *x, float *y, int64_t rows, int64_t dim, cudaStream_t s)
{
    if (rows == 0) return cudaSuccess;
    softmax_generic<<<static_cast<unsigned>(rows), 256, 0, s>>>(x, y, dim);
    return cudaGetLastError();
}

cudaError_t launch_pool_l2(const float *h, const int32_t *cu, int batch, int dim, int mode, float *out,
                           cudaStream_t s)
{
    if (batch == 0) return cudaSuccess;
    if (mode == FE_POOL_MEAN && dim % 4 == 0 && (reinterpret_cast<uintptr_t>(h) & 15) == 0) {
        // one block per sentence (float4 rows: dim % 4 == 0 and h 16-byte aligned); W warps so
        // that the [W][dim] partial sums and the W-float reduction array fit in 48 KB
        const size_t row = static_cast<size_t>(dim) * sizeof(float), cap = 48 * 1024;
        if (8 * row + 8 * 4 <= cap)
            return launch_k(pool_mean_l2<8>, dim3(batch), dim3(256), 8 * row, s, h, cu, dim, out);
        if (4 * row + 4 * 4 <= cap)
            return launch_k(pool_mean_l2<4>, dim3(batch), dim3(128), 4 * row, s, h, cu, dim, out);
        if (2 * row + 2 * 4 <= cap)
            return launch_k(pool_mean_l2<2>, dim3(batch), dim3(64), 2 * row, s, h, cu, dim, out);
    }
    return launch_k(pool_l2, dim3(grid_for(batch, 8)), dim3(256), 0, s, h, cu, batch, dim, mode, out);
}

cudaError_t launch_f32_to_bf16(const float *x, void *y, int64_t count, cudaStream_t s)
{
    if (count == 0) return cudaSuccess;
    int64_t blocks = (count + 255) / 256;
    if (blocks > 4096) blocks = 4096;
    f32_to_bf16<<<static_cast<unsigned>(blocks), 256, 0, s>>>(x, static_cast<__nv_bfloat16 *>(y), count);
    return cudaGetLastError();
}

}  // namespace fe
