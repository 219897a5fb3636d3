// ref_forward.cpp — drives the reference's own CPU ops (compiled from the reference
// sources by oracle/Makefile into oracle/_ref/) through a restatement of its
// bge_forward, to pin the C restatement in fe_oracle.c and to serve as the timed
// CPU baseline.
//
// TEST INFRASTRUCTURE ONLY.  The product library never links this.
//
// The op order restates src/sentence_transformers_impl.cpp:126-344 and :389-440,
// with CPUAttentionOps / CPUMatrixOps (src/ops/cpu/*.cpp) where the reference
// binary calls its CUDA classes; every op takes and returns std::vector<float>
// exactly as the reference's op API does.
#include <atomic>
#include <cmath>
#include <cstring>
#include <thread>
#include <vector>

#include "fe_oracle.h"
#include "ops/cpu/cpu_attention_ops.h"
#include "ops/cpu/cpu_matrix_ops.h"

namespace {

std::vector<float> vec(const float *p, size_t n) { return std::vector<float>(p, p + n); }

int forward_one(const fe_oracle_bert *m, const int32_t *ids, int len, float *out)
{
    const size_t D = (size_t)m->hidden, F = (size_t)m->intermediate, L = (size_t)len;
    if (len <= 0 || len > m->max_pos) return -1;
    for (int t = 0; t < len; ++t)
        if (ids[t] < 0 || ids[t] >= m->vocab) return -2;
    CPUMatrixOps mops;
    CPUAttentionOps aops;

    // word gather (:30-44), += position row (:139-163), += token type 0 (:166-188).
    // bge-m3 / XLM-R rows (:101-123, :146-149): pad tokens row 0, the others 2, 3, ...;
    // a row outside the table becomes row 0.
    std::vector<float> x(L * D);
    for (size_t t = 0; t < L; ++t)
        std::memcpy(&x[t * D], m->word + (size_t)ids[t] * D, sizeof(float) * D);
    int next_row = 2;
    for (size_t t = 0; t < L; ++t) {
        int row = static_cast<int>(t);
        if (m->pad_id >= 0) {
            row = ids[t] == m->pad_id ? 0 : next_row++;
            if (row >= m->max_pos) row = 0;
        }
        for (size_t j = 0; j < D; ++j) x[t * D + j] += m->pos[(size_t)row * D + j];
    }
    for (size_t t = 0; t < L; ++t)
        for (size_t j = 0; j < D; ++j) x[t * D + j] += m->type[j];
    x = mops.layer_norm(x, vec(m->emb_ln_g, D), vec(m->emb_ln_b, D), D, m->eps);

    for (int l = 0; l < m->layers; ++l) {
        const fe_oracle_layer &w = m->layer[l];
        std::vector<float> attn = aops.multi_head_attention(
            x, vec(w.wq, D * D), vec(w.wk, D * D), vec(w.wv, D * D), vec(w.bq, D), vec(w.bk, D),
            vec(w.bv, D), (size_t)m->heads, D);
        attn = mops.matrix_multiply_transpose(attn, vec(w.wo, D * D), L, D, D);
        for (size_t i = 0; i < attn.size(); ++i) attn[i] += w.bo[i % D];
        for (size_t i = 0; i < attn.size(); ++i) attn[i] += x[i];
        x = mops.layer_norm(attn, vec(w.ln1_g, D), vec(w.ln1_b, D), D, m->eps);

        std::vector<float> hidden = mops.matrix_multiply_transpose(x, vec(w.w1, F * D), L, D, F);
        for (size_t i = 0; i < hidden.size(); ++i) hidden[i] += w.b1[i % F];
        if (m->act == FE_ORACLE_ACT_RELU) hidden = mops.relu(hidden);
        else if (m->act == FE_ORACLE_ACT_SWISH) hidden = mops.swish(hidden);
        else hidden = mops.gelu(hidden);
        std::vector<float> y = mops.matrix_multiply_transpose(hidden, vec(w.w2, D * F), L, F, D);
        for (size_t i = 0; i < y.size(); ++i) y[i] += w.b2[i % D];
        for (size_t i = 0; i < y.size(); ++i) y[i] += x[i];
        x = mops.layer_norm(y, vec(w.ln2_g, D), vec(w.ln2_b, D), D, m->eps);
    }

    // CLS row, L2 normalised (:289-341)
    float norm = 0.0f;
    for (size_t j = 0; j < D; ++j) norm += x[j] * x[j];
    norm = std::sqrt(norm);
    for (size_t j = 0; j < D; ++j) out[j] = x[j] / norm;
    return 0;
}

}  // namespace

extern "C" {

int fe_ref_bert_forward(const fe_oracle_bert *m, const int32_t *ids, int len, float *out)
{
    return forward_one(m, ids, len, out);
}

// Sentence-parallel driver over std::thread; the reference's encode_batch
// (:359-365) is the serial special case threads = 1.
int fe_ref_bert_forward_batch(const fe_oracle_bert *m, const int32_t *ids, const int32_t *lengths,
                              int batch, int stride, float *out, int threads)
{
    std::atomic<int> next{0}, status{0};
    if (threads < 1) threads = 1;
    if (threads > batch) threads = batch > 0 ? batch : 1;
    std::vector<std::thread> pool;
    for (int i = 0; i < threads; ++i)
        pool.emplace_back([&] {
            for (int s; (s = next.fetch_add(1)) < batch;) {
                int rc = forward_one(m, ids + (size_t)s * stride, lengths[s],
                                     out + (size_t)s * m->hidden);
                if (rc != 0) {
                    int zero = 0;
                    status.compare_exchange_strong(zero, rc);
                }
            }
        });
    for (auto &t : pool) t.join();
    return status.load();
}

// Op-level entry points over the reference classes, for the op parity pins.
void fe_ref_matmul_nt(const float *a, const float *b, float *c, size_t m, size_t n, size_t k)
{
    CPUMatrixOps ops;
    auto r = ops.matrix_multiply_transpose(vec(a, m * n), vec(b, k * n), m, n, k);
    std::memcpy(c, r.data(), sizeof(float) * r.size());
}

void fe_ref_matmul_nn(const float *a, const float *b, float *c, size_t m, size_t n, size_t k)
{
    CPUMatrixOps ops;
    auto r = ops.matrix_multiply(vec(a, m * n), vec(b, n * k), m, n, k);
    std::memcpy(c, r.data(), sizeof(float) * r.size());
}

#define FE_REF_UNARY(name, method)                                        \
    void name(const float *x, float *y, size_t count)                     \
    {                                                                     \
        CPUMatrixOps ops;                                                 \
        auto r = ops.method(vec(x, count));                               \
        std::memcpy(y, r.data(), sizeof(float) * r.size());               \
    }
FE_REF_UNARY(fe_ref_gelu, gelu)
FE_REF_UNARY(fe_ref_relu, relu)
FE_REF_UNARY(fe_ref_swish, swish)
#undef FE_REF_UNARY

void fe_ref_layer_norm(const float *x, const float *g, const float *b, float *y, size_t count,
                       size_t dim, float eps)
{
    CPUMatrixOps ops;
    auto r = ops.layer_norm(vec(x, count), vec(g, dim), vec(b, dim), dim, eps);
    std::memcpy(y, r.data(), sizeof(float) * r.size());
}

void fe_ref_rms_norm(const float *x, const float *w, float *y, size_t count, size_t dim, float eps)
{
    CPUMatrixOps ops;
    auto r = ops.rms_norm(vec(x, count), vec(w, dim), dim, eps);
    std::memcpy(y, r.data(), sizeof(float) * r.size());
}

void fe_ref_softmax_rows(const float *x, float *y, size_t count, size_t dim)
{
    CPUMatrixOps ops;
    auto r = ops.softmax(vec(x, count), 1, dim);
    std::memcpy(y, r.data(), sizeof(float) * r.size());
}

void fe_ref_mha(const float *x, const float *wq, const float *wk, const float *wv, const float *bq,
                const float *bk, const float *bv, size_t heads, size_t dim, size_t seq_len,
                float *out)
{
    CPUAttentionOps ops;
    auto r = ops.multi_head_attention(vec(x, seq_len * dim), vec(wq, dim * dim), vec(wk, dim * dim),
                                      vec(wv, dim * dim), vec(bq, dim), vec(bk, dim), vec(bv, dim),
                                      heads, dim);
    std::memcpy(out, r.data(), sizeof(float) * r.size());
}

}  // extern "C"
