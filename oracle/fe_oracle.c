/*
 * fe_oracle.c — CPU restatement of fastEmbed's FP32 encoder path.
 *
 * TEST INFRASTRUCTURE ONLY: the parity checker for the CUDA path.  Not linked
 * into, nor called by, the product library.  See fe_oracle.h.
 *
 * Each routine keeps the reference's floating-point operation order (sums run
 * front to back from 0.0f, scalars combine left to right) because bit-exact
 * agreement with the reference CPU ops is what pins this oracle.  Build with
 * plain -O3 and no FMA contraction (oracle/Makefile), as the reference is.
 */
#include "fe_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* C[m,k] = A[m,n] · B[k,n]^T  — CPUMatrixOps::matrix_multiply_transpose,
 * src/ops/cpu/cpu_matrix_ops.cpp:7-18 (dot product accumulated p = 0..n-1). */
void fe_oracle_matmul_nt(const float *a, const float *b, float *c, size_t m, size_t n, size_t k)
{
    for (size_t row = 0; row < m; ++row) {
        const float *arow = a + row * n;
        for (size_t col = 0; col < k; ++col) {
            const float *brow = b + col * n;
            float acc = 0.0f;
            for (size_t p = 0; p < n; ++p) acc += arow[p] * brow[p];
            c[row * k + col] = acc;
        }
    }
}

/* C[m,k] = A[m,n] · B[n,k] — CPUMatrixOps::matrix_multiply, cpu_matrix_ops.cpp:21-32. */
void fe_oracle_matmul_nn(const float *a, const float *b, float *c, size_t m, size_t n, size_t k)
{
    for (size_t row = 0; row < m; ++row) {
        for (size_t col = 0; col < k; ++col) {
            float acc = 0.0f;
            for (size_t p = 0; p < n; ++p) acc += a[row * n + p] * b[p * k + col];
            c[row * k + col] = acc;
        }
    }
}

/* tanh-form GELU, cpu_matrix_ops.cpp:35-43.  The constant is sqrt(2/pi) computed
 * entirely in float (float pi literal, float division, float sqrt). */
void fe_oracle_gelu(const float *x, float *y, size_t count)
{
    const float k_s2pi = sqrtf(2.0f / 3.14159265358979323846f);
    for (size_t i = 0; i < count; ++i) {
        const float v = x[i];
        const float cube = 0.044715f * v * v * v;
        y[i] = 0.5f * v * (1.0f + tanhf(k_s2pi * (v + cube)));
    }
}

/* cpu_matrix_ops.cpp:46-52 */
void fe_oracle_relu(const float *x, float *y, size_t count)
{
    for (size_t i = 0; i < count; ++i) y[i] = x[i] > 0.0f ? x[i] : 0.0f;
}

/* x / (1 + e^-x), cpu_matrix_ops.cpp:55-61 */
void fe_oracle_swish(const float *x, float *y, size_t count)
{
    for (size_t i = 0; i < count; ++i) y[i] = x[i] / (1.0f + expf(-x[i]));
}

/* Two-pass LayerNorm, cpu_matrix_ops.cpp:64-92: mean, then mean squared deviation,
 * then (x - mean) / sqrt(var + eps) * gamma + beta. `count` is the element total. */
void fe_oracle_layer_norm(const float *x, const float *g, const float *b, float *y,
                          size_t count, size_t dim, float eps)
{
    const size_t rows = count / dim;
    const float fdim = (float)dim;
    for (size_t r = 0; r < rows; ++r) {
        const float *xr = x + r * dim;
        float *yr = y + r * dim;
        float mean = 0.0f;
        for (size_t i = 0; i < dim; ++i) mean += xr[i];
        mean /= fdim;
        float var = 0.0f;
        for (size_t i = 0; i < dim; ++i) {
            const float d = xr[i] - mean;
            var += d * d;
        }
        var /= fdim;
        const float sd = sqrtf(var + eps);
        for (size_t i = 0; i < dim; ++i) yr[i] = (xr[i] - mean) / sd * g[i] + b[i];
    }
}

/* RMSNorm, cpu_matrix_ops.cpp:95-121: inv = 1/sqrt(mean(x^2) + eps); y = inv * w * x. */
void fe_oracle_rms_norm(const float *x, const float *w, float *y, size_t count, size_t dim,
                        float eps)
{
    const size_t rows = count / dim;
    const float fdim = (float)dim;
    for (size_t r = 0; r < rows; ++r) {
        const float *xr = x + r * dim;
        float *yr = y + r * dim;
        float ss = 0.0f;
        for (size_t i = 0; i < dim; ++i) ss += xr[i] * xr[i];
        ss /= fdim;
        ss += eps;
        const float inv = 1.0f / sqrtf(ss);
        for (size_t i = 0; i < dim; ++i) yr[i] = inv * w[i] * xr[i];
    }
}

/* Row softmax (axis = 1), cpu_matrix_ops.cpp:141-163. */
void fe_oracle_softmax_rows(const float *x, float *y, size_t count, size_t dim)
{
    const size_t rows = count / dim;
    for (size_t r = 0; r < rows; ++r) {
        const float *xr = x + r * dim;
        float *yr = y + r * dim;
        float mx = xr[0];
        for (size_t i = 1; i < dim; ++i)
            if (xr[i] > mx) mx = xr[i];
        float sum = 0.0f;
        for (size_t i = 0; i < dim; ++i) {
            yr[i] = expf(xr[i] - mx);
            sum += yr[i];
        }
        for (size_t i = 0; i < dim; ++i) yr[i] /= sum;
    }
}

/* Single-sequence multi-head attention, src/ops/cpu/cpu_attention_ops.cpp:8-98:
 * Q,K,V = X·W^T + b; per head scores = (Q_h K_h^T) / sqrt(hd) (a division, :35,:69);
 * row softmax; O_h = P V_h; heads concatenated at columns h*hd. */
void fe_oracle_mha(const float *x, const float *wq, const float *wk, const float *wv,
                   const float *bq, const float *bk, const float *bv, size_t heads, size_t dim,
                   size_t seq_len, float *out)
{
    const size_t hd = dim / heads;
    const size_t L = seq_len;
    float *q = malloc(sizeof(float) * L * dim);
    float *k = malloc(sizeof(float) * L * dim);
    float *v = malloc(sizeof(float) * L * dim);
    float *qh = malloc(sizeof(float) * L * hd);
    float *kt = malloc(sizeof(float) * hd * L);
    float *vh = malloc(sizeof(float) * L * hd);
    float *s = malloc(sizeof(float) * (L * L > 0 ? L * L : 1));
    float *p = malloc(sizeof(float) * (L * L > 0 ? L * L : 1));
    float *oh = malloc(sizeof(float) * L * hd);

    fe_oracle_matmul_nt(x, wq, q, L, dim, dim);
    fe_oracle_matmul_nt(x, wk, k, L, dim, dim);
    fe_oracle_matmul_nt(x, wv, v, L, dim, dim);
    for (size_t i = 0; i < L * dim; ++i) {
        q[i] += bq[i % dim];
        k[i] += bk[i % dim];
        v[i] += bv[i % dim];
    }
    const float denom = sqrtf((float)hd);
    for (size_t h = 0; h < heads; ++h) {
        for (size_t t = 0; t < L; ++t)
            for (size_t d = 0; d < hd; ++d) {
                const size_t src = t * dim + h * hd + d;
                qh[t * hd + d] = q[src];
                kt[d * L + t] = k[src];
                vh[t * hd + d] = v[src];
            }
        fe_oracle_matmul_nn(qh, kt, s, L, hd, L);
        for (size_t i = 0; i < L * L; ++i) s[i] /= denom;
        fe_oracle_softmax_rows(s, p, L * L, L);
        fe_oracle_matmul_nn(p, vh, oh, L, L, hd);
        for (size_t t = 0; t < L; ++t) memcpy(out + t * dim + h * hd, oh + t * hd, sizeof(float) * hd);
    }
    free(q); free(k); free(v); free(qh); free(kt); free(vh); free(s); free(p); free(oh);
}

/* src/sentence_transformers_impl.cpp:101-123 (create_position_ids_from_input_ids: the
 * count starts at 2, a pad token keeps 0) and :146-149 (a row outside the table is
 * replaced by row 0). */
void fe_oracle_position_rows(const int32_t *ids, int len, int pad_id, int max_pos, int32_t *rows)
{
    int next = 2;
    for (int t = 0; t < len; ++t) {
        if (pad_id < 0) {
            rows[t] = t;
            continue;
        }
        int r = ids[t] != pad_id ? next++ : 0;
        if (r < 0 || r >= max_pos) r = 0;
        rows[t] = r;
    }
}

/* Embedding + encoder + CLS/L2 for one unpadded sentence, following
 * src/sentence_transformers_impl.cpp op for op:
 *   :30-44 word gather; :139-163 += position row (row i, or the bge-m3 rows of
 *   fe_oracle_position_rows); :166-188 += token-type row 0;
 *   :189-194 LayerNorm(eps);
 *   per layer :199-281: MHA (:243-246) -> out-proj (:250-252) -> += bias (:255-257)
 *     -> += residual (:261-263) -> LayerNorm (:266) -> FFN (:389-440: GEMM1, += b1,
 *     activation, GEMM2, += b2, += residual, LayerNorm);
 *   :289-341 CLS row 0 divided by its L2 norm.
 * Returns 0, or -1 when the sentence is longer than the position table (:132-136). */
int fe_oracle_bert_forward(const fe_oracle_bert *m, const int32_t *ids, int len, float *out)
{
    const size_t D = (size_t)m->hidden, F = (size_t)m->intermediate, L = (size_t)len;
    if (len <= 0 || len > m->max_pos) return -1;
    for (int t = 0; t < len; ++t)
        if (ids[t] < 0 || ids[t] >= m->vocab) return -2;

    float *x = malloc(sizeof(float) * L * D);
    float *a = malloc(sizeof(float) * L * D);
    float *y = malloc(sizeof(float) * L * D);
    float *hmid = malloc(sizeof(float) * L * F);
    float *hact = malloc(sizeof(float) * L * F);

    for (size_t t = 0; t < L; ++t) memcpy(x + t * D, m->word + (size_t)ids[t] * D, sizeof(float) * D);
    int32_t *prow = malloc(sizeof(int32_t) * L);
    fe_oracle_position_rows(ids, len, m->pad_id, m->max_pos, prow);
    for (size_t t = 0; t < L; ++t)
        for (size_t j = 0; j < D; ++j) x[t * D + j] += m->pos[(size_t)prow[t] * D + j];
    free(prow);
    for (size_t t = 0; t < L; ++t)
        for (size_t j = 0; j < D; ++j) x[t * D + j] += m->type[j];
    fe_oracle_layer_norm(x, m->emb_ln_g, m->emb_ln_b, x, L * D, D, m->eps);

    for (int l = 0; l < m->layers; ++l) {
        const fe_oracle_layer *w = &m->layer[l];
        fe_oracle_mha(x, w->wq, w->wk, w->wv, w->bq, w->bk, w->bv, (size_t)m->heads, D, L, a);
        fe_oracle_matmul_nt(a, w->wo, y, L, D, D);
        for (size_t i = 0; i < L * D; ++i) y[i] += w->bo[i % D];
        for (size_t i = 0; i < L * D; ++i) y[i] += x[i];
        fe_oracle_layer_norm(y, w->ln1_g, w->ln1_b, x, L * D, D, m->eps);

        fe_oracle_matmul_nt(x, w->w1, hmid, L, D, F);
        for (size_t i = 0; i < L * F; ++i) hmid[i] += w->b1[i % F];
        if (m->act == FE_ORACLE_ACT_RELU) fe_oracle_relu(hmid, hact, L * F);
        else if (m->act == FE_ORACLE_ACT_SWISH) fe_oracle_swish(hmid, hact, L * F);
        else fe_oracle_gelu(hmid, hact, L * F);
        fe_oracle_matmul_nt(hact, w->w2, y, L, F, D);
        for (size_t i = 0; i < L * D; ++i) y[i] += w->b2[i % D];
        for (size_t i = 0; i < L * D; ++i) y[i] += x[i];
        fe_oracle_layer_norm(y, w->ln2_g, w->ln2_b, x, L * D, D, m->eps);
    }

    float ss = 0.0f;
    for (size_t j = 0; j < D; ++j) ss += x[j] * x[j];
    const float nrm = sqrtf(ss);
    for (size_t j = 0; j < D; ++j) out[j] = x[j] / nrm;

    free(x); free(a); free(y); free(hmid); free(hact);
    return 0;
}

/* ---- sentence-parallel driver (pthreads) ---- */
typedef struct {
    const fe_oracle_bert *m;
    const int32_t *ids, *lengths;
    int batch, stride;
    float *out;
    int next;          /* shared work counter */
    int status;
    pthread_mutex_t mu;
} batch_job;

static void *batch_worker(void *arg)
{
    batch_job *job = arg;
    for (;;) {
        pthread_mutex_lock(&job->mu);
        const int s = job->next++;
        pthread_mutex_unlock(&job->mu);
        if (s >= job->batch) break;
        const int rc = fe_oracle_bert_forward(job->m, job->ids + (size_t)s * job->stride,
                                              job->lengths[s], job->out + (size_t)s * job->m->hidden);
        if (rc != 0) {
            pthread_mutex_lock(&job->mu);
            if (job->status == 0) job->status = rc;
            pthread_mutex_unlock(&job->mu);
        }
    }
    return NULL;
}

int fe_oracle_bert_forward_batch(const fe_oracle_bert *m, const int32_t *ids,
                                 const int32_t *lengths, int batch, int stride, float *out,
                                 int threads)
{
    batch_job job = {m, ids, lengths, batch, stride, out, 0, 0};
    pthread_mutex_init(&job.mu, NULL);
    if (threads < 1) threads = 1;
    if (threads > batch) threads = batch > 0 ? batch : 1;
    pthread_t *tid = malloc(sizeof(pthread_t) * (size_t)threads);
    for (int i = 0; i < threads; ++i) pthread_create(&tid[i], NULL, batch_worker, &job);
    for (int i = 0; i < threads; ++i) pthread_join(tid[i], NULL);
    free(tid);
    pthread_mutex_destroy(&job.mu);
    return job.status;
}
