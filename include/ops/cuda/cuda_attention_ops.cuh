// cuda_attention_ops.cuh — drop-in for fastEmbed's CUDAAttentionOps
// (include/ops/cuda/cuda_attention_ops.cuh:6-22 of the reference): single-sequence
// multi-head attention over host vectors, Q,K,V = X·W^T + b, per head
// softmax(Q K^T / sqrt(hd)) V, heads concatenated.  Runs the FP32 attention of the C ABI
// (fe_mha_f32); shape errors throw std::invalid_argument, CUDA errors std::runtime_error.
#ifndef CUDA_ATTENTION_OPS_CUH
#define CUDA_ATTENTION_OPS_CUH

#include <cstddef>
#include <memory>
#include <vector>

class CUDAAttentionOps {
public:
    CUDAAttentionOps();
    ~CUDAAttentionOps();
    CUDAAttentionOps(const CUDAAttentionOps &) = delete;
    CUDAAttentionOps &operator=(const CUDAAttentionOps &) = delete;

    std::vector<float> multi_head_attention(const std::vector<float> &input,       // [seq_len, embed_dim]
                                            const std::vector<float> &weight_q,    // [embed_dim, embed_dim]
                                            const std::vector<float> &weight_k,    // [embed_dim, embed_dim]
                                            const std::vector<float> &weight_v,    // [embed_dim, embed_dim]
                                            const std::vector<float> &query_bias,  // [embed_dim]
                                            const std::vector<float> &key_bias,    // [embed_dim]
                                            const std::vector<float> &value_bias,  // [embed_dim]
                                            size_t num_heads, size_t embedding_dim);

private:
    struct Impl;
    std::unique_ptr<Impl> impl_;
};

#endif  // CUDA_ATTENTION_OPS_CUH
