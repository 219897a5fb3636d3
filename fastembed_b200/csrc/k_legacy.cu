// k_legacy.cu — FP32 kernels behind the host-vector op API (CUDAMatrixOps /
// CUDAAttentionOps).  The reference's GTests compare these ops with its CPU ops at
// 1e-5 (matrix) and 1e-3 (attention) absolute, which BF16/TF32 tensor-core inputs
// cannot meet, so these stay in FP32 SIMT.  Dot products accumulate in the CPU
// ops' order (p = 0, 1, ..., each product rounded, then added: no FMA
// contraction), so the GEMMs reproduce src/ops/cpu/cpu_matrix_ops.cpp:7-32 bit for bit.
#include "fe_common.cuh"
#include "fe_internal.h"

namespace fe {
namespace {

constexpr int TM = 64, TN = 64, TKK = 16;

// C[m,k] = A[m,n] · B  with B = [k,n] (transposed, nn.Linear) or [n,k]; 4x4 outputs
// per thread, 64x64 tile per block, operands staged through shared memory.
template <bool BT>
__global__ void __launch_bounds__(256)
    sgemm_exact(const float *__restrict__ A, const float *__restrict__ B, const float *__restrict__ bias,
                float *__restrict__ C, int64_t m, int64_t n, int64_t k)
{
    __shared__ float As[TKK][TM + 1];
    __shared__ float Bs[TKK][TN + 1];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int64_t row0 = static_cast<int64_t>(blockIdx.y) * TM;
    const int64_t col0 = static_cast<int64_t>(blockIdx.x) * TN;
    float acc[4][4] = {};
    for (int64_t p0 = 0; p0 < n; p0 += TKK) {
        for (int i = threadIdx.x; i < TM * TKK; i += 256) {
            const int r = i / TKK, c = i % TKK;
            const int64_t gr = row0 + r, gc = p0 + c;
            As[c][r] = (gr < m && gc < n) ? A[gr * n + gc] : 0.f;
        }
        for (int i = threadIdx.x; i < TN * TKK; i += 256) {
            int r, c;  // r: output column within tile, c: reduction index within chunk
            if (BT) { r = i / TKK; c = i % TKK; } else { c = i / TN; r = i % TN; }
            const int64_t gcol = col0 + r, gp = p0 + c;
            float v = 0.f;
            if (gcol < k && gp < n) v = BT ? B[gcol * n + gp] : B[gp * k + gcol];
            Bs[c][r] = v;
        }
        __syncthreads();
        const int pend = static_cast<int>(n - p0 < TKK ? n - p0 : TKK);
        for (int p = 0; p < pend; ++p) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = As[p][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; ++j) b[j] = Bs[p][tx * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(a[i], b[j]));
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int64_t r = row0 + ty * 4 + i, c = col0 + tx * 4 + j;
            if (r < m && c < k) C[r * k + c] = bias ? __fadd_rn(acc[i][j], bias[c]) : acc[i][j];
        }
}

// Elementwise activations (src/ops/cpu/cpu_matrix_ops.cpp:35-61), full-precision tanhf / expf.
__global__ void unary(int op, const float *__restrict__ x, float *__restrict__ y, int64_t n)
{
    const float k_s2pi = sqrtf(2.0f / 3.14159265358979323846f);
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const float v = x[i];
        float r;
        if (op == FE_ACT_GELU) {
            const float cube = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, v), v), v);
            r = __fmul_rn(__fmul_rn(0.5f, v), __fadd_rn(1.0f, tanhf(__fmul_rn(k_s2pi, __fadd_rn(v, cube)))));
        } else if (op == FE_ACT_RELU) {
            r = v > 0.f ? v : 0.f;
        } else {
            r = v / __fadd_rn(1.0f, expf(-v));
        }
        y[i] = r;
    }
}

// Per (query row, head) attention of one sequence in FP32 with the CPU op's order
// (src/ops/cpu/cpu_attention_ops.cpp:40-85): scores = (q . k_j) / sqrt(hd),
// softmax, out = sum_j p_j v_j.  Scores live in dynamic shared memory [L].
__global__ void __launch_bounds__(128)
    mha_rows(const float *__restrict__ q, const float *__restrict__ kx, const float *__restrict__ v,
             float *__restrict__ out, int64_t L, int64_t dim, int64_t hd)
{
    extern __shared__ float sc[];
    __shared__ float red[2];
    const int64_t i = blockIdx.x;
    const int64_t h = blockIdx.y;
    const float denom = sqrtf(static_cast<float>(hd));
    const float *qi = q + i * dim + h * hd;
    for (int64_t j = threadIdx.x; j < L; j += blockDim.x) {
        const float *kj = kx + j * dim + h * hd;
        float acc = 0.f;
        for (int64_t d = 0; d < hd; ++d) acc = __fadd_rn(acc, __fmul_rn(qi[d], kj[d]));
        sc[j] = acc / denom;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float mx = sc[0];
        for (int64_t j = 1; j < L; ++j) mx = fmaxf(mx, sc[j]);
        red[0] = mx;
    }
    __syncthreads();
    const float mx = red[0];
    for (int64_t j = threadIdx.x; j < L; j += blockDim.x) sc[j] = expf(sc[j] - mx);
    __syncthreads();
    if (threadIdx.x == 0) {
        float s = 0.f;
        for (int64_t j = 0; j < L; ++j) s = __fadd_rn(s, sc[j]);
        red[1] = s;
    }
    __syncthreads();
    const float s = red[1];
    for (int64_t j = threadIdx.x; j < L; j += blockDim.x) sc[j] = sc[j] / s;
    __syncthreads();
    for (int64_t d = threadIdx.x; d < hd; d += blockDim.x) {
        float acc = 0.f;
        for (int64_t j = 0; j < L; ++j) acc = __fadd_rn(acc, __fmul_rn(sc[j], v[j * dim + h * hd + d]));
        out[i * dim + h * hd + d] = acc;
    }
}

}  // namespace

cudaError_t launch_sgemm(const float *a, const float *b, const float *bias, float *c, int64_t m, int64_t n,
                         int64_t k, bool b_transposed, cudaStream_t s)
{
    if (m == 0 || k == 0) return cudaSuccess;
    dim3 grid(static_cast<unsigned>((k + TN - 1) / TN), static_cast<unsigned>((m + TM - 1) / TM));
    if (b_transposed)
        sgemm_exact<true><<<grid, 256, 0, s>>>(a, b, bias, c, m, n, k);
    else
        sgemm_exact<false><<<grid, 256, 0, s>>>(a, b, bias, c, m, n, k);
    return cudaGetLastError();
}

cudaError_t launch_unary(int op, const float *x, float *y, int64_t count, cudaStream_t s)
{
    if (count == 0) return cudaSuccess;
    int64_t blocks = (count + 255) / 256;
    if (blocks > 65535) blocks = 65535;
    unary<<<static_cast<unsigned>(blocks), 256, 0, s>>>(op, x, y, count);
    return cudaGetLastError();
}

cudaError_t launch_mha_core_f32(const float *q, const float *k, const float *v, float *out, int64_t seq_len,
                                int64_t dim, int64_t heads, cudaStream_t s)
{
    if (seq_len == 0) return cudaSuccess;
    const size_t smem = static_cast<size_t>(seq_len) * sizeof(float);
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(mha_rows, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem));
        if (e != cudaSuccess) return e;
    }
    dim3 grid(static_cast<unsigned>(seq_len), static_cast<unsigned>(heads));
    mha_rows<<<grid, 128, smem, s>>>(q, k, v, out, seq_len, dim, dim / heads);
    return cudaGetLastError();
}

}  // namespace fe
