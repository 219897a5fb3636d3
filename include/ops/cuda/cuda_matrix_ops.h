// cuda_matrix_ops.h — drop-in for fastEmbed's CUDAMatrixOps
// (include/ops/cuda/cuda_matrix_ops.h:4-45 of the reference): same class name, same
// public methods and argument meaning, host std::vector<float> in and out.
//
// Each method runs a B200 kernel through the C ABI (include/fastembed_b200.h) in FP32
// (the reference's GTests compare these ops with the CPU ops at 1e-5 absolute).
// Shape errors throw std::invalid_argument as the reference does; CUDA errors throw
// std::runtime_error (the reference calls exit()).  Device buffers are cached per
// object and grown on demand; an object may be used from several threads.
#pragma once
#include <cstddef>
#include <memory>
#include <vector>

class CUDAMatrixOps {
public:
    CUDAMatrixOps();
    ~CUDAMatrixOps();
    CUDAMatrixOps(const CUDAMatrixOps &) = delete;
    CUDAMatrixOps &operator=(const CUDAMatrixOps &) = delete;

    // C[m,k] = A[m,n] · B[n,k]
    std::vector<float> matrix_multiply(const std::vector<float> &a, const std::vector<float> &b, size_t m, size_t n,
                                       size_t k);
    // C[m,k] = A[m,n] · B[k,n]^T
    std::vector<float> matrix_multiply_transpose(const std::vector<float> &a, const std::vector<float> &b, size_t m,
                                                 size_t n, size_t k);
    // tanh-form GELU
    std::vector<float> gelu(const std::vector<float> &input);
    std::vector<float> relu(const std::vector<float> &input);
    std::vector<float> swish(const std::vector<float> &input);
    // row LayerNorm over embedding_dim (any width)
    std::vector<float> layer_norm(const std::vector<float> &input, const std::vector<float> &gamma,
                                  const std::vector<float> &beta, size_t embedding_dim, float epsilon = 1e-5);
    std::vector<float> rms_norm(const std::vector<float> &input, const std::vector<float> &weight,
                                size_t embedding_dim, float epsilon = 1e-5);
    // row softmax (axis 1 only); dim_size 0 means 768, as in the reference
    std::vector<float> softmax(const std::vector<float> &input, size_t axis = 1, size_t dim_size = 0);
    // in-place softmax of device scores [num_heads, seq_len, seq_len]
    void apply_softmax(float *input, size_t num_heads, size_t seq_len);

private:
    struct Impl;
    std::unique_ptr<Impl> impl_;
};
