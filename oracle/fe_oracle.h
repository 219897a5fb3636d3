/*
 * fe_oracle.h — CPU restatement of fastEmbed's FP32 encoder path.
 *
 * TEST INFRASTRUCTURE ONLY. This is the parity checker for the CUDA path in
 * fastembed_b200/. Only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg load it; the product library never links or calls it.
 *
 * Every function restates one reference routine with the same floating-point
 * operation order, so that (compiled with the same flags, no FMA contraction)
 * results are bit-identical to the reference's CPU ops.  The pin is checked in
 * tests/test_oracle.py against oracle/_ref (the reference's own CPU sources
 * compiled by oracle/Makefile) and against the committed golden vectors under
 * tests/golden/.
 */
#ifndef FE_ORACLE_H
#define FE_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Hidden activation selector, config.json "hidden_act"
 * (src/sentence_transformers_impl.cpp:413-421). */
enum { FE_ORACLE_ACT_GELU = 0, FE_ORACLE_ACT_RELU = 1, FE_ORACLE_ACT_SWISH = 2 };

/* One post-LN BERT layer, HF tensor names as read at
 * src/sentence_transformers_impl.cpp:201-218. Weights are nn.Linear [out,in]. */
typedef struct fe_oracle_layer {
    const float *wq, *bq, *wk, *bk, *wv, *bv; /* attention.self.{query,key,value} */
    const float *wo, *bo;                     /* attention.output.dense            */
    const float *ln1_g, *ln1_b;               /* attention.output.LayerNorm        */
    const float *w1, *b1;                     /* intermediate.dense  [F, D]        */
    const float *w2, *b2;                     /* output.dense        [D, F]        */
    const float *ln2_g, *ln2_b;               /* output.LayerNorm                  */
} fe_oracle_layer;

typedef struct fe_oracle_bert {
    int vocab, hidden, heads, intermediate, layers, max_pos, type_vocab;
    int act;   /* FE_ORACLE_ACT_* */
    float eps; /* config.json layer_norm_eps */
    const float *word, *pos, *type, *emb_ln_g, *emb_ln_b;
    const fe_oracle_layer *layer; /* [layers] */
    int pad_id; /* -1: position row i for token i (BERT / BGE); >= 0: the bge-m3 / XLM-R
                 * rows of fe_oracle_position_rows with this pad_token_id */
} fe_oracle_bert;

/* Position rows of one sentence (src/sentence_transformers_impl.cpp:101-123, :139-155):
 * pad_id < 0: row t; pad_id >= 0: a token equal to pad_id takes row 0, the others rows
 * 2, 3, ... in order, and a row at or past max_pos becomes row 0. */
void fe_oracle_position_rows(const int32_t *ids, int len, int pad_id, int max_pos, int32_t *rows);

/* --- op-level restatements (src/ops/cpu/cpu_matrix_ops.cpp) --- */
void fe_oracle_matmul_nt(const float *a, const float *b, float *c, size_t m, size_t n, size_t k);
void fe_oracle_matmul_nn(const float *a, const float *b, float *c, size_t m, size_t n, size_t k);
void fe_oracle_gelu(const float *x, float *y, size_t count);
void fe_oracle_relu(const float *x, float *y, size_t count);
void fe_oracle_swish(const float *x, float *y, size_t count);
void fe_oracle_layer_norm(const float *x, const float *g, const float *b, float *y,
                          size_t count, size_t dim, float eps);
void fe_oracle_rms_norm(const float *x, const float *w, float *y, size_t count, size_t dim,
                        float eps);
void fe_oracle_softmax_rows(const float *x, float *y, size_t count, size_t dim);

/* --- src/ops/cpu/cpu_attention_ops.cpp:8-98 --- */
void fe_oracle_mha(const float *x, const float *wq, const float *wk, const float *wv,
                   const float *bq, const float *bk, const float *bv, size_t heads, size_t dim,
                   size_t seq_len, float *out);

/* --- src/sentence_transformers_impl.cpp:126-344 (one unpadded sentence) --- */
int fe_oracle_bert_forward(const fe_oracle_bert *m, const int32_t *ids, int len, float *out);

/* Sentence-parallel batch driver: sentence s has ids[s*stride .. s*stride+lengths[s]).
 * Returns 0 on success, or the first non-zero per-sentence status. */
int fe_oracle_bert_forward_batch(const fe_oracle_bert *m, const int32_t *ids,
                                 const int32_t *lengths, int batch, int stride, float *out,
                                 int threads);

/* std::mt19937(seed) + std::uniform_real_distribution<float>(lo, hi), the input
 * generator of tests/matrix_ops_test.cpp:20-26 and tests/attention_ops_test.cpp:17-32. */
void fe_oracle_fill_uniform_mt19937(uint32_t seed, float lo, float hi, float *out, size_t count);

#ifdef __cplusplus
}
#endif
#endif
