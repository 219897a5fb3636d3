// ops_classes.cpp — the drop-in op classes CUDAMatrixOps and CUDAAttentionOps over the
// C ABI.  Each call stages the host vectors into cached device buffers on the object's
// own stream, runs one fe_* entry point, copies the result back and synchronises.
// Argument checks and exception types follow the reference
// (src/ops/cuda/cuda_matrix_ops.cu:307-319, :364-373, :464-481;
// src/ops/cuda/cuda_attention_ops.cu:182-187).
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "fastembed_b200.h"
#include "ops/cuda/cuda_attention_ops.cuh"
#include "ops/cuda/cuda_matrix_ops.h"

namespace {

void throw_status(fe_status st, const char *where)
{
    if (st == FE_OK) return;
    const std::string msg = std::string(where) + ": " + fe_last_error_message();
    if (st == FE_ERR_INVALID_ARGUMENT) throw std::invalid_argument(msg);
    throw std::runtime_error(msg);
}

void throw_cuda(cudaError_t e, const char *where)
{
    if (e != cudaSuccess) throw std::runtime_error(std::string(where) + ": " + cudaGetErrorString(e));
}

// A growable device buffer.
struct Buf {
    float *p = nullptr;
    size_t n = 0;
    ~Buf() { if (p) cudaFree(p); }
    float *get(size_t count)
    {
        if (count > n) {
            if (p) cudaFree(p);
            p = nullptr;
            n = 0;
            throw_cuda(cudaMalloc(&p, std::max<size_t>(count, 1) * sizeof(float)), "cudaMalloc");
            n = count;
        }
        return p;
    }
};

// Device state shared by both op classes: a stream and a few staging buffers.
struct Staging {
    std::mutex mu;
    cudaStream_t stream = nullptr;
    int device = 0;
    Buf b[8];
    Staging()
    {
        throw_cuda(cudaGetDevice(&device), "cudaGetDevice");
        throw_cuda(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "cudaStreamCreate");
    }
    ~Staging()
    {
        if (stream) {
            cudaStreamSynchronize(stream);
            cudaStreamDestroy(stream);
        }
    }
    fe_stream_t s() const { return reinterpret_cast<fe_stream_t>(stream); }
    float *up(int slot, const std::vector<float> &v)
    {
        float *d = b[slot].get(v.size());
        if (!v.empty())
            throw_cuda(cudaMemcpyAsync(d, v.data(), v.size() * sizeof(float), cudaMemcpyHostToDevice, stream),
                       "cudaMemcpyAsync");
        return d;
    }
    std::vector<float> down(const float *d, size_t count)
    {
        std::vector<float> out(count);
        if (count)
            throw_cuda(cudaMemcpyAsync(out.data(), d, count * sizeof(float), cudaMemcpyDeviceToHost, stream),
                       "cudaMemcpyAsync");
        throw_cuda(cudaStreamSynchronize(stream), "cudaStreamSynchronize");
        return out;
    }
};

void need(bool ok, const char *msg)
{
    if (!ok) throw std::invalid_argument(msg);
}

}  // namespace

struct CUDAMatrixOps::Impl : Staging {};

CUDAMatrixOps::CUDAMatrixOps() : impl_(new Impl()) {}
CUDAMatrixOps::~CUDAMatrixOps() = default;

std::vector<float> CUDAMatrixOps::matrix_multiply(const std::vector<float> &a, const std::vector<float> &b, size_t m,
                                                  size_t n, size_t k)
{
    need(a.size() >= m * n && b.size() >= n * k, "matrix_multiply: input smaller than m*n or n*k");
    std::lock_guard<std::mutex> lk(impl_->mu);
    float *da = impl_->up(0, a), *db = impl_->up(1, b), *dc = impl_->b[2].get(m * k);
    throw_status(fe_sgemm_nn(da, db, dc, m, n, k, impl_->s()), "matrix_multiply");
    return impl_->down(dc, m * k);
}

std::vector<float> CUDAMatrixOps::matrix_multiply_transpose(const std::vector<float> &a, const std::vector<float> &b,
                                                            size_t m, size_t n, size_t k)
{
    need(a.size() >= m * n && b.size() >= n * k, "matrix_multiply_transpose: input smaller than m*n or k*n");
    std::lock_guard<std::mutex> lk(impl_->mu);
    float *da = impl_->up(0, a), *db = impl_->up(1, b), *dc = impl_->b[2].get(m * k);
    throw_status(fe_sgemm_nt(da, db, nullptr, dc, m, n, k, impl_->s()), "matrix_multiply_transpose");
    return impl_->down(dc, m * k);
}

namespace {
template <class F>
std::vector<float> unary(Staging &st, const std::vector<float> &in, F fn, const char *name)
{
    std::lock_guard<std::mutex> lk(st.mu);
    float *dx = st.up(0, in), *dy = st.b[1].get(in.size());
    throw_status(fn(dx, dy, static_cast<int64_t>(in.size()), st.s()), name);
    return st.down(dy, in.size());
}
}  // namespace

std::vector<float> CUDAMatrixOps::gelu(const std::vector<float> &input) { return unary(*impl_, input, fe_gelu_f32, "gelu"); }
std::vector<float> CUDAMatrixOps::relu(const std::vector<float> &input) { return unary(*impl_, input, fe_relu_f32, "relu"); }
std::vector<float> CUDAMatrixOps::swish(const std::vector<float> &input) { return unary(*impl_, input, fe_swish_f32, "swish"); }

std::vector<float> CUDAMatrixOps::layer_norm(const std::vector<float> &input, const std::vector<float> &gamma,
                                             const std::vector<float> &beta, size_t embedding_dim, float epsilon)
{
    need(!input.empty() && !gamma.empty() && !beta.empty(), "Input vectors cannot be empty");
    need(gamma.size() == embedding_dim && beta.size() == embedding_dim,
         "Gamma and beta must match embedding dimension size");
    std::lock_guard<std::mutex> lk(impl_->mu);
    const size_t rows = input.size() / embedding_dim;
    float *dx = impl_->up(0, input), *dg = impl_->up(1, gamma), *db = impl_->up(2, beta);
    float *dy = impl_->b[3].get(input.size());
    throw_status(fe_layer_norm_f32(dx, dg, db, dy, rows, embedding_dim, epsilon, impl_->s()), "layer_norm");
    std::vector<float> out = impl_->down(dy, rows * embedding_dim);
    // a trailing partial row (input.size() not a multiple of embedding_dim) is passed through
    out.insert(out.end(), input.begin() + rows * embedding_dim, input.end());
    return out;
}

std::vector<float> CUDAMatrixOps::rms_norm(const std::vector<float> &input, const std::vector<float> &weight,
                                           size_t embedding_dim, float epsilon)
{
    need(!input.empty() && !weight.empty(), "Input vectors cannot be empty");
    need(weight.size() == embedding_dim, "Weight must match embedding dimension size");
    need(input.size() % embedding_dim == 0, "Input size is not divisible by embedding_dim");
    std::lock_guard<std::mutex> lk(impl_->mu);
    float *dx = impl_->up(0, input), *dw = impl_->up(1, weight), *dy = impl_->b[2].get(input.size());
    throw_status(fe_rms_norm_f32(dx, dw, dy, input.size() / embedding_dim, embedding_dim, epsilon, impl_->s()),
                 "rms_norm");
    return impl_->down(dy, input.size());
}

std::vector<float> CUDAMatrixOps::softmax(const std::vector<float> &input, size_t axis, size_t dim_size)
{
    if (axis != 1) throw std::invalid_argument("Only axis=1 is supported for CUDA softmax");
    if (dim_size == 0) dim_size = 768;
    need(input.size() % dim_size == 0, "Input size must be divisible by dim_size");
    std::lock_guard<std::mutex> lk(impl_->mu);
    float *dx = impl_->up(0, input), *dy = impl_->b[1].get(input.size());
    throw_status(fe_softmax_rows_f32(dx, dy, input.size() / dim_size, dim_size, impl_->s()), "softmax");
    return impl_->down(dy, input.size());
}

void CUDAMatrixOps::apply_softmax(float *input, size_t num_heads, size_t seq_len)
{
    std::lock_guard<std::mutex> lk(impl_->mu);
    throw_status(fe_softmax_scores_inplace_f32(input, num_heads, seq_len, impl_->s()), "apply_softmax");
    throw_cuda(cudaStreamSynchronize(impl_->stream), "cudaStreamSynchronize");
}

// ------------------------------------------------------------------ attention
struct CUDAAttentionOps::Impl : Staging {
    void *ws = nullptr;
    size_t ws_bytes = 0;
    ~Impl() { if (ws) cudaFree(ws); }
};

CUDAAttentionOps::CUDAAttentionOps() : impl_(new Impl()) {}
CUDAAttentionOps::~CUDAAttentionOps() = default;

std::vector<float> CUDAAttentionOps::multi_head_attention(const std::vector<float> &input,
                                                          const std::vector<float> &weight_q,
                                                          const std::vector<float> &weight_k,
                                                          const std::vector<float> &weight_v,
                                                          const std::vector<float> &query_bias,
                                                          const std::vector<float> &key_bias,
                                                          const std::vector<float> &value_bias, size_t num_heads,
                                                          size_t embedding_dim)
{
    need(num_heads > 0 && embedding_dim % num_heads == 0, "Embedding dimension must be divisible by number of heads");
    const size_t seq_len = input.size() / embedding_dim;
    need(seq_len == 0 || input.size() % (seq_len * embedding_dim) == 0, "Invalid input size for given dimensions");
    const size_t DD = embedding_dim * embedding_dim;
    need(weight_q.size() >= DD && weight_k.size() >= DD && weight_v.size() >= DD,
         "multi_head_attention: weight smaller than embed_dim^2");
    need(query_bias.size() >= embedding_dim && key_bias.size() >= embedding_dim && value_bias.size() >= embedding_dim,
         "multi_head_attention: bias smaller than embed_dim");
    std::lock_guard<std::mutex> lk(impl_->mu);
    Impl &st = *impl_;
    float *dx = st.up(0, input), *dq = st.up(1, weight_q), *dk = st.up(2, weight_k), *dv = st.up(3, weight_v);
    float *bq = st.up(4, query_bias), *bk = st.up(5, key_bias), *bv = st.up(6, value_bias);
    float *dout = st.b[7].get(seq_len * embedding_dim);
    const size_t need_ws = fe_mha_f32_workspace_bytes(seq_len, embedding_dim, num_heads);
    if (need_ws > st.ws_bytes) {
        if (st.ws) cudaFree(st.ws);
        st.ws = nullptr;
        st.ws_bytes = 0;
        throw_cuda(cudaMalloc(&st.ws, need_ws), "cudaMalloc");
        st.ws_bytes = need_ws;
    }
    throw_status(fe_mha_f32(dx, dq, dk, dv, bq, bk, bv, dout, seq_len, embedding_dim, num_heads, st.ws, st.ws_bytes,
                            st.s()),
                 "multi_head_attention");
    return st.down(dout, seq_len * embedding_dim);
}
