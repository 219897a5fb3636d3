// engine.cpp — device-resident post-LN BERT encoder over packed variable-length
// batches: the batched, unpadded form of the reference's bge_forward
// (src/sentence_transformers_impl.cpp:126-344) and feed_forward_network (:389-440).
//
// Per call: embed+LN, then per layer
//   QKV linear (bias)            -> qkv  bf16 [T, 3D]
//   varlen attention             -> attn bf16 [T, D]
//   out-proj linear (bias+resid) -> y    fp32 [T, D]   ; LN -> h fp32 + bf16
//   FFN1 linear (bias+act)       -> ff   bf16 [T, F]
//   FFN2 linear (bias+resid)     -> y    fp32 [T, D]   ; LN -> h fp32 + bf16
// then pooling + L2.  Weights are uploaded once (bf16 copies of the projection
// matrices, Q/K/V concatenated into one [3D, D] matrix; fp32 everything else).
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include <nvtx3/nvToolsExt.h>

#include "fe_internal.h"
#include "json_min.h"

using fe::fail;

namespace {

struct DevBuf {
    void *p = nullptr;
    size_t bytes = 0;
    ~DevBuf() { if (p) cudaFree(p); }
    cudaError_t ensure(size_t n)
    {
        if (n <= bytes) return cudaSuccess;
        if (p) cudaFree(p);
        p = nullptr;
        bytes = 0;
        cudaError_t e = cudaMalloc(&p, n);
        if (e == cudaSuccess) bytes = n;
        return e;
    }
    template <class T> T *as() const { return static_cast<T *>(p); }
};

struct PinnedBuf {
    void *p = nullptr;
    size_t bytes = 0;
    ~PinnedBuf() { if (p) cudaFreeHost(p); }
    cudaError_t ensure(size_t n)
    {
        if (n <= bytes) return cudaSuccess;
        if (p) cudaFreeHost(p);
        p = nullptr;
        bytes = 0;
        cudaError_t e = cudaMallocHost(&p, n);
        if (e == cudaSuccess) bytes = n;
        return e;
    }
    template <class T> T *as() const { return static_cast<T *>(p); }
};

struct Layer {
    DevBuf wqkv, wo, w1, w2;                 // bf16 [3D,D], [D,D], [F,D], [D,F]
    DevBuf bqkv, bo, b1, b2;                 // fp32
    DevBuf ln1_g, ln1_b, ln2_g, ln2_b;       // fp32 [D]
};

// Where an HF tensor goes: fp32 buffer (`f32`) or bf16 matrix (`bf16`) at element
// offset `offset`, with `count` elements.
struct Slot {
    DevBuf *buf;
    size_t offset;
    size_t count;
    bool bf16;
    // gated-MLP weights: 0 = contiguous; 1 / 2 = this [F, row] matrix goes to the even /
    // odd 32-row blocks of the interleaved [2F, row] gate-up matrix
    int interleave = 0;
    size_t row = 0;
};

// One layer of a pre-RMSNorm rotary encoder (Qwen3 / Gemma3 shapes).
struct RLayer {
    DevBuf wqkv, wo, wgu, wd;                        // bf16 [(Hq+2Hkv)hd, D], [D, Hq hd], [2F, D], [D, F]
    DevBuf q_norm, k_norm;                           // fp32 [hd]
    DevBuf in_norm, post_attn_norm, pre_ff_norm, post_ff_norm;  // fp32 [D]
};

enum Cat { CAT_GEMM = 0, CAT_ATTN = 1, CAT_OTHER = 2 };

}  // namespace

struct fe_engine {
    fe_encoder_config cfg{};
    int family = FE_FAMILY_BERT;
    fe_rms_encoder_config rc{};  // RMSNorm families
    std::vector<RLayer> rlayers;
    DevBuf final_norm, zero_bias, hfin;  // hfin: final-norm output [T, D] fp32 (RMSNorm families)
    DevBuf tpos;                         // int32 [T]: each token's position in its sentence (RMSNorm families)
    DevBuf staging16;  // bf16 conversion buffer of interleaved uploads
    int device = 0;
    cudaStream_t stream = nullptr;
    std::mutex mu;

    DevBuf word, pos, type, emb_g, emb_b;
    std::vector<Layer> layers;
    std::map<std::string, Slot> slots;
    std::map<std::string, bool> loaded;
    DevBuf staging;  // fp32 upload staging for bf16 conversion

    // activations, sized for the largest batch seen
    DevBuf h32, h16, qkv, attn, y32, ff;
    DevBuf ln_ws;  // row-statistics exchange of the fused linear + LayerNorm (zero-filled when allocated)
    DevBuf rss;    // fp32 [T][parts]: row sums of squares of the deferred pre-norm RMSNorm (Qwen3 shapes)
    int64_t cap_tokens = 0;
    // per-call inputs for the host path
    DevBuf d_ids, d_cu, d_out;
    PinnedBuf p_ids, p_cu, p_out, p_status;

    // profiling
    bool profiling = false;
    std::vector<cudaEvent_t> ev;  // pairs
    std::vector<int> ev_cat;
    size_t ev_used = 0;
    fe_engine_stats stats{};
};

namespace {

fe_status alloc_weights(fe_engine *e)
{
    const fe_encoder_config &c = e->cfg;
    const size_t D = c.hidden, F = c.intermediate;
    auto f32 = [&](DevBuf &b, size_t n) { return b.ensure(n * sizeof(float)); };
    auto b16 = [&](DevBuf &b, size_t n) { return b.ensure(n * sizeof(__nv_bfloat16)); };
    FE_TRY_CUDA(f32(e->word, static_cast<size_t>(c.vocab_size) * D));
    FE_TRY_CUDA(f32(e->pos, static_cast<size_t>(c.max_position) * D));
    FE_TRY_CUDA(f32(e->type, static_cast<size_t>(c.type_vocab) * D));
    FE_TRY_CUDA(f32(e->emb_g, D));
    FE_TRY_CUDA(f32(e->emb_b, D));
    e->slots["embeddings.word_embeddings.weight"] = {&e->word, 0, static_cast<size_t>(c.vocab_size) * D, false};
    e->slots["embeddings.position_embeddings.weight"] = {&e->pos, 0, static_cast<size_t>(c.max_position) * D, false};
    e->slots["embeddings.token_type_embeddings.weight"] = {&e->type, 0, static_cast<size_t>(c.type_vocab) * D, false};
    e->slots["embeddings.LayerNorm.weight"] = {&e->emb_g, 0, D, false};
    e->slots["embeddings.LayerNorm.bias"] = {&e->emb_b, 0, D, false};
    e->layers.resize(c.layers);
    for (int l = 0; l < c.layers; ++l) {
        Layer &L = e->layers[l];
        FE_TRY_CUDA(b16(L.wqkv, 3 * D * D));
        FE_TRY_CUDA(b16(L.wo, D * D));
        FE_TRY_CUDA(b16(L.w1, F * D));
        FE_TRY_CUDA(b16(L.w2, D * F));
        FE_TRY_CUDA(f32(L.bqkv, 3 * D));
        FE_TRY_CUDA(f32(L.bo, D));
        FE_TRY_CUDA(f32(L.b1, F));
        FE_TRY_CUDA(f32(L.b2, D));
        FE_TRY_CUDA(f32(L.ln1_g, D));
        FE_TRY_CUDA(f32(L.ln1_b, D));
        FE_TRY_CUDA(f32(L.ln2_g, D));
        FE_TRY_CUDA(f32(L.ln2_b, D));
        const std::string p = "encoder.layer." + std::to_string(l) + ".";
        e->slots[p + "attention.self.query.weight"] = {&L.wqkv, 0, D * D, true};
        e->slots[p + "attention.self.key.weight"] = {&L.wqkv, D * D, D * D, true};
        e->slots[p + "attention.self.value.weight"] = {&L.wqkv, 2 * D * D, D * D, true};
        e->slots[p + "attention.self.query.bias"] = {&L.bqkv, 0, D, false};
        e->slots[p + "attention.self.key.bias"] = {&L.bqkv, D, D, false};
        e->slots[p + "attention.self.value.bias"] = {&L.bqkv, 2 * D, D, false};
        e->slots[p + "attention.output.dense.weight"] = {&L.wo, 0, D * D, true};
        e->slots[p + "attention.output.dense.bias"] = {&L.bo, 0, D, false};
        e->slots[p + "attention.output.LayerNorm.weight"] = {&L.ln1_g, 0, D, false};
        e->slots[p + "attention.output.LayerNorm.bias"] = {&L.ln1_b, 0, D, false};
        e->slots[p + "intermediate.dense.weight"] = {&L.w1, 0, F * D, true};
        e->slots[p + "intermediate.dense.bias"] = {&L.b1, 0, F, false};
        e->slots[p + "output.dense.weight"] = {&L.w2, 0, D * F, true};
        e->slots[p + "output.dense.bias"] = {&L.b2, 0, D, false};
        e->slots[p + "output.LayerNorm.weight"] = {&L.ln2_g, 0, D, false};
        e->slots[p + "output.LayerNorm.bias"] = {&L.ln2_b, 0, D, false};
    }
    for (auto &kv : e->slots) e->loaded[kv.first] = false;
    return FE_OK;
}

fe_status ensure_activations(fe_engine *e, int64_t T)
{
    if (T <= e->cap_tokens) return FE_OK;
    const int64_t cap = std::max<int64_t>(T, 128);
    const size_t D = e->cfg.hidden, F = e->cfg.intermediate;
    FE_TRY_CUDA(e->h32.ensure(cap * D * 4));
    FE_TRY_CUDA(e->h16.ensure(cap * D * 2));
    FE_TRY_CUDA(e->qkv.ensure(cap * 3 * D * 2));
    FE_TRY_CUDA(e->attn.ensure(cap * D * 2));
    FE_TRY_CUDA(e->y32.ensure(cap * D * 4));
    FE_TRY_CUDA(e->ff.ensure(cap * F * 2));
    const size_t ws = fe::linear_layernorm_stats_bytes(cap, static_cast<int64_t>(D));
    FE_TRY_CUDA(e->ln_ws.ensure(ws));
    FE_TRY_CUDA(cudaMemset(e->ln_ws.p, 0, ws));
    e->cap_tokens = cap;
    return FE_OK;
}

// One launch of the forward: counted, optionally timed with CUDA events on its stream,
// and marked as an NVTX range (host side, for nsys and other NVTX tools; the range
// brackets the launch call, not the kernel's execution) named after the op.
struct Scope {
    fe_engine *e;
    int cat;
    cudaStream_t s;
    size_t idx = 0;
    Scope(fe_engine *e_, int cat_, cudaStream_t s_, const char *name = nullptr) : e(e_), cat(cat_), s(s_)
    {
        nvtxRangePushA(name ? name : cat == CAT_GEMM ? "fe.linear" : cat == CAT_ATTN ? "fe.attention" : "fe.rows");
        e->stats.launches++;
        if (cat == CAT_GEMM) e->stats.gemm_launches++;
        if (!e->profiling) return;
        idx = e->ev_used;
        if (idx + 2 > e->ev.size()) {
            for (int i = 0; i < 64; ++i) {
                cudaEvent_t x;
                cudaEventCreate(&x);
                e->ev.push_back(x);
            }
            e->ev_cat.resize(e->ev.size() / 2);
        }
        e->ev_cat[idx / 2] = cat;
        cudaEventRecord(e->ev[idx], s);
        e->ev_used += 2;
    }
    ~Scope()
    {
        if (e->profiling) cudaEventRecord(e->ev[idx + 1], s);
        nvtxRangePop();
    }
};

int act_epilogue(int act)
{
    if (act == FE_ACT_RELU) return FE_EPI_BIAS_RELU;
    if (act == FE_ACT_SWISH) return FE_EPI_BIAS_SWISH;
    return FE_EPI_BIAS_GELU;
}

fe_status linear(fe_engine *e, cudaStream_t s, const void *x, const DevBuf &w, const DevBuf &b, const float *res,
                 void *y, int64_t m, int64_t n, int64_t k, int epi, int dtype)
{
    Scope sc(e, CAT_GEMM, s);
    fe_status st = FE_OK;
    cudaError_t err = fe::launch_linear_bf16(x, w.p, b.as<float>(), res, y, m, n, k, epi, dtype, s, &st);
    if (st != FE_OK) return st;
    return fe::check_cuda(err, "linear");
}

// h32 <- LayerNorm((x W^T + b) + h32) * g + beta (and its bf16 copy): one fused launch
// where the shape allows it, else the linear and the LayerNorm separately (y32 scratch).
fe_status linear_ln(fe_engine *e, cudaStream_t s, const void *x, const DevBuf &w, const DevBuf &b, const DevBuf &g,
                    const DevBuf &beta, float *h32, void *h16, int64_t m, int64_t n, int64_t k)
{
    Scope sc(e, CAT_GEMM, s, "fe.linear_layernorm");
    fe_status st = FE_OK;
    cudaError_t err = fe::launch_linear_layernorm(x, w.p, b.as<float>(), g.as<float>(), beta.as<float>(), h32, h16, m,
                                                  n, k, e->cfg.layer_norm_eps, e->ln_ws.p, e->y32.as<float>(), s, &st);
    if (st != FE_OK) return st;
    return fe::check_cuda(err, "linear+LayerNorm");
}

fe_status forward(fe_engine *e, const int32_t *ids, const int32_t *cu, const int32_t *cu_host, int batch,
                  float *out, cudaStream_t s)
{
    const fe_encoder_config &c = e->cfg;
    const int64_t T = cu_host[batch];
    int max_len = 0;
    for (int b = 0; b < batch; ++b) {
        const int L = cu_host[b + 1] - cu_host[b];
        if (L < 0) return fail(FE_ERR_INVALID_ARGUMENT, "cu_seqlens must be non-decreasing");
        if (L > c.max_position)
            return fail(FE_ERR_INVALID_ARGUMENT, "sequence length exceeds the position embedding table");
        max_len = std::max(max_len, L);
    }
    if (cu_host[0] != 0) return fail(FE_ERR_INVALID_ARGUMENT, "cu_seqlens[0] must be 0");
    FE_TRY(ensure_activations(e, T));
    e->stats.launches = 0;
    e->stats.gemm_launches = 0;
    e->stats.tokens = T;
    e->ev_used = 0;
    const int64_t D = c.hidden, F = c.intermediate;
    double gemm_flops = 0, attn_flops = 0;
    for (int b = 0; b < batch; ++b) {
        const double L = cu_host[b + 1] - cu_host[b];
        gemm_flops += c.layers * 2.0 * L * (4.0 * D * D + 2.0 * D * F);
        attn_flops += c.layers * 4.0 * L * L * D;
    }
    e->stats.gemm_flops = gemm_flops;
    e->stats.attention_flops = attn_flops;
    if (T == 0) {
        if (batch > 0) FE_TRY_CUDA(cudaMemsetAsync(out, 0, sizeof(float) * batch * D, s));
        return FE_OK;
    }
    float *h32 = e->h32.as<float>();
    void *h16 = e->h16.p, *qkv = e->qkv.p, *attn = e->attn.p, *ff = e->ff.p;
    {
        Scope sc(e, CAT_OTHER, s, "fe.embed_layernorm");
        FE_TRY_CUDA(fe::launch_embed_layernorm(ids, cu, batch, T, e->word.as<float>(), e->pos.as<float>(),
                                               e->type.as<float>(), e->emb_g.as<float>(), e->emb_b.as<float>(),
                                               static_cast<int>(D), c.vocab_size, c.max_position, c.layer_norm_eps,
                                               h32, h16, s, c.positions == FE_POSITIONS_XLMR ? c.pad_token_id : -1));
    }
    const int act = act_epilogue(c.activation);
    for (int l = 0; l < c.layers; ++l) {
        const Layer &L = e->layers[l];
        const bool last = l + 1 == c.layers;
        FE_TRY(linear(e, s, h16, L.wqkv, L.bqkv, nullptr, qkv, T, 3 * D, D, FE_EPI_BIAS, FE_DTYPE_BF16));
        {
            Scope sc(e, CAT_ATTN, s, "fe.attention");
            fe_status st = FE_OK;
            cudaError_t err = fe::launch_attention_varlen(qkv, cu, batch, max_len, c.heads,
                                                          static_cast<int>(D / c.heads), attn, T, false, s, &st);
            if (st != FE_OK) return st;
            FE_TRY_CUDA(err);
        }
        if (fe::ln_cluster_applies(D, D, false, false)) {
            // out-proj + bias + residual + LayerNorm in one launch: one cluster per 128-row block
            FE_TRY(linear_ln(e, s, attn, L.wo, L.bo, L.ln1_g, L.ln1_b, h32, h16, T, D, D));
        } else {
            // out-proj + bias (bf16, into the y32 buffer) then residual + LayerNorm, in place on the fp32
            // residual stream
            FE_TRY(linear(e, s, attn, L.wo, L.bo, nullptr, e->y32.p, T, D, D, FE_EPI_BIAS, FE_DTYPE_BF16));
            Scope sc(e, CAT_GEMM, s, "fe.residual_layernorm");
            FE_TRY_CUDA(fe::launch_layernorm_dual_bf16in(e->y32.p, h32, L.ln1_g.as<float>(), L.ln1_b.as<float>(), h32,
                                                         h16, T, static_cast<int>(D), c.layer_norm_eps, s));
        }
        FE_TRY(linear(e, s, h16, L.w1, L.b1, nullptr, ff, T, F, D, act, FE_DTYPE_BF16));
        FE_TRY(linear_ln(e, s, ff, L.w2, L.b2, L.ln2_g, L.ln2_b, h32, last ? nullptr : h16, T, D, F));
    }
    {
        Scope sc(e, CAT_OTHER, s, "fe.pool_l2");
        FE_TRY_CUDA(fe::launch_pool_l2(h32, cu, batch, static_cast<int>(D), c.pooling, out, s));
    }
    return FE_OK;
}

// ---------------------------------------------------------------- RMSNorm families
bool is_gemma(const fe_engine *e) { return e->family == FE_FAMILY_GEMMA3; }

fe_status alloc_weights_rms(fe_engine *e)
{
    const fe_rms_encoder_config &c = e->rc;
    const size_t D = c.hidden, F = c.intermediate, hd = c.head_dim;
    const size_t QKV = static_cast<size_t>(c.q_heads + 2 * c.kv_heads) * hd, AO = static_cast<size_t>(c.q_heads) * hd;
    auto f32 = [&](DevBuf &b, size_t n) { return b.ensure(n * sizeof(float)); };
    auto b16 = [&](DevBuf &b, size_t n) { return b.ensure(n * sizeof(__nv_bfloat16)); };
    FE_TRY_CUDA(f32(e->word, static_cast<size_t>(c.vocab_size) * D));
    FE_TRY_CUDA(f32(e->final_norm, D));
    FE_TRY_CUDA(f32(e->zero_bias, std::max(D, 2 * F)));
    FE_TRY_CUDA(cudaMemset(e->zero_bias.p, 0, std::max(D, 2 * F) * sizeof(float)));
    e->slots["embed_tokens.weight"] = {&e->word, 0, static_cast<size_t>(c.vocab_size) * D, false};
    e->slots["norm.weight"] = {&e->final_norm, 0, D, false};
    e->rlayers.resize(c.layers);
    for (int l = 0; l < c.layers; ++l) {
        RLayer &L = e->rlayers[l];
        FE_TRY_CUDA(b16(L.wqkv, QKV * D));
        FE_TRY_CUDA(b16(L.wo, D * AO));
        FE_TRY_CUDA(b16(L.wgu, 2 * F * D));
        FE_TRY_CUDA(b16(L.wd, D * F));
        FE_TRY_CUDA(f32(L.q_norm, hd));
        FE_TRY_CUDA(f32(L.k_norm, hd));
        FE_TRY_CUDA(f32(L.in_norm, D));
        FE_TRY_CUDA(f32(L.post_attn_norm, D));
        const std::string p = "layers." + std::to_string(l) + ".";
        e->slots[p + "self_attn.q_proj.weight"] = {&L.wqkv, 0, AO * D, true};
        e->slots[p + "self_attn.k_proj.weight"] = {&L.wqkv, AO * D, c.kv_heads * hd * D, true};
        e->slots[p + "self_attn.v_proj.weight"] = {&L.wqkv, (AO + c.kv_heads * hd) * D, c.kv_heads * hd * D, true};
        e->slots[p + "self_attn.o_proj.weight"] = {&L.wo, 0, D * AO, true};
        e->slots[p + "self_attn.q_norm.weight"] = {&L.q_norm, 0, hd, false};
        e->slots[p + "self_attn.k_norm.weight"] = {&L.k_norm, 0, hd, false};
        Slot gate{&L.wgu, 0, F * D, true};
        gate.interleave = 1;
        gate.row = D;
        Slot up = gate;
        up.interleave = 2;
        e->slots[p + "mlp.gate_proj.weight"] = gate;
        e->slots[p + "mlp.up_proj.weight"] = up;
        e->slots[p + "mlp.down_proj.weight"] = {&L.wd, 0, D * F, true};
        e->slots[p + "input_layernorm.weight"] = {&L.in_norm, 0, D, false};
        e->slots[p + "post_attention_layernorm.weight"] = {&L.post_attn_norm, 0, D, false};
        if (is_gemma(e)) {
            FE_TRY_CUDA(f32(L.pre_ff_norm, D));
            FE_TRY_CUDA(f32(L.post_ff_norm, D));
            e->slots[p + "pre_feedforward_layernorm.weight"] = {&L.pre_ff_norm, 0, D, false};
            e->slots[p + "post_feedforward_layernorm.weight"] = {&L.post_ff_norm, 0, D, false};
        }
    }
    for (auto &kv : e->slots) e->loaded[kv.first] = false;
    return FE_OK;
}

fe_status ensure_activations_rms(fe_engine *e, int64_t T)
{
    if (T <= e->cap_tokens) return FE_OK;
    const fe_rms_encoder_config &c = e->rc;
    const int64_t cap = std::max<int64_t>(T, 128);
    const size_t D = c.hidden, F = c.intermediate, hd = c.head_dim;
    FE_TRY_CUDA(e->h32.ensure(cap * D * 4));
    FE_TRY_CUDA(e->h16.ensure(cap * D * 2));
    FE_TRY_CUDA(e->qkv.ensure(cap * (c.q_heads + 2 * c.kv_heads) * hd * 2));
    FE_TRY_CUDA(e->attn.ensure(cap * c.q_heads * hd * 2));
    FE_TRY_CUDA(e->y32.ensure(cap * D * 4));
    FE_TRY_CUDA(e->ff.ensure(cap * F * 2));
    FE_TRY_CUDA(e->hfin.ensure(cap * D * 4));
    FE_TRY_CUDA(e->tpos.ensure(cap * 4));
    FE_TRY_CUDA(e->rss.ensure(cap * 8 * 4));
    const size_t ws = fe::linear_layernorm_stats_bytes(cap, static_cast<int64_t>(D));
    FE_TRY_CUDA(e->ln_ws.ensure(ws));
    FE_TRY_CUDA(cudaMemset(e->ln_ws.p, 0, ws));
    e->cap_tokens = cap;
    return FE_OK;
}

// FE_RMS_DEFER=0 keeps the pre-norm RMSNorm of o_proj / down_proj inside those GEMMs (row
// statistics exchanged between the CTA pairs of a row, second pass over TMEM) instead of
// deferring the row factor to the next projection's epilogue (for comparison).
bool rms_defer_enabled()
{
    static const bool on = [] {
        const char *v = getenv("FE_RMS_DEFER");
        return !(v && v[0] == '0');
    }();
    return on;
}

bool qkrope_fuse_enabled()
{
    static const bool on = [] {
        const char *v = getenv("FE_QKROPE_FUSE");
        return !(v && v[0] == '0');
    }();
    return on;
}

// Theta of layer l (Gemma3: every full_attention_every-th layer is a global layer).
float layer_theta(const fe_rms_encoder_config &c, int l)
{
    if (c.full_attention_every <= 0) return c.rope_theta;
    return (l + 1) % c.full_attention_every == 0 ? c.rope_theta : c.rope_theta_local;
}

fe_status forward_rms(fe_engine *e, const int32_t *ids, const int32_t *cu, const int32_t *cu_host, int batch,
                      float *out, cudaStream_t s)
{
    const fe_rms_encoder_config &c = e->rc;
    const int64_t T = cu_host[batch];
    int max_len = 0;
    for (int b = 0; b < batch; ++b) {
        const int L = cu_host[b + 1] - cu_host[b];
        if (L < 0) return fail(FE_ERR_INVALID_ARGUMENT, "cu_seqlens must be non-decreasing");
        if (L > c.max_position) return fail(FE_ERR_INVALID_ARGUMENT, "sequence length exceeds max_position");
        if (is_gemma(e) && L > 1024)
            return fail(FE_ERR_UNSUPPORTED, "Gemma3 shapes: sentences up to 1024 tokens (no sliding-window mask)");
        max_len = std::max(max_len, L);
    }
    if (cu_host[0] != 0) return fail(FE_ERR_INVALID_ARGUMENT, "cu_seqlens[0] must be 0");
    FE_TRY(ensure_activations_rms(e, T));
    e->stats.launches = 0;
    e->stats.gemm_launches = 0;
    e->stats.tokens = T;
    e->ev_used = 0;
    const int64_t D = c.hidden, F = c.intermediate, hd = c.head_dim;
    const int64_t QKV = (c.q_heads + 2 * c.kv_heads) * hd, AO = static_cast<int64_t>(c.q_heads) * hd;
    const bool gemma = is_gemma(e);
    double gemm_flops = 0, attn_flops = 0;
    for (int b = 0; b < batch; ++b) {
        const double L = cu_host[b + 1] - cu_host[b];
        gemm_flops += c.layers * 2.0 * L * (static_cast<double>(D) * QKV + AO * D + 3.0 * D * F);
        const double pairs = gemma ? L * L : L * (L + 1) / 2;  // causal: the lower triangle
        attn_flops += c.layers * 4.0 * pairs * AO;
    }
    e->stats.gemm_flops = gemm_flops;
    e->stats.attention_flops = attn_flops;
    if (T == 0) {
        if (batch > 0) FE_TRY_CUDA(cudaMemsetAsync(out, 0, sizeof(float) * batch * D, s));
        return FE_OK;
    }
    float *h32 = e->h32.as<float>(), *y32 = e->y32.as<float>();
    void *x16 = e->h16.p, *qkv = e->qkv.p, *attn = e->attn.p, *ff = e->ff.p;
    const float eps = c.rms_norm_eps;
    const float qscale = c.query_scale > 0.f ? c.query_scale : 1.0f / sqrtf(static_cast<float>(hd));
    // Qwen3: the RMSNorms that follow o_proj and down_proj are deferred.  Those GEMMs write
    // bf16(h * w) and each row's partial sums of h^2 (rss); the next projection (gate_up,
    // or the next layer's QKV) multiplies its product's rows by 1 / rms(h).  Layer 0's QKV
    // reads rows normalised by the row kernel (no factor).
    const int ss_parts = fe::linear_rms_deferred_parts(D);
    const bool defer = !gemma && rms_defer_enabled() && D % 256 == 0 && D <= 2048;
    float *rss = defer ? e->rss.as<float>() : nullptr;
    auto gemm = [&](const void *x, const DevBuf &w, const float *bias, const float *res, void *y, int64_t n, int64_t k,
                    int epi, int dtype, const float *row_ss = nullptr) -> fe_status {
        Scope sc(e, CAT_GEMM, s);
        fe_status st = FE_OK;
        cudaError_t err = fe::launch_linear_bf16(x, w.p, bias, res, y, T, n, k, epi, dtype, s, &st, row_ss, ss_parts, eps);
        if (st != FE_OK) return st;
        return fe::check_cuda(err, "linear");
    };
    // pre-norm projection + residual + RMSNorm: fused where the launcher can (long K), else two launches
    auto linear_rms = [&](const void *x, const DevBuf &w, const DevBuf &norm_w, float *h, void *out16, int64_t n,
                          int64_t k) -> fe_status {
        Scope sc(e, CAT_GEMM, s, "fe.linear_rmsnorm");
        fe_status st = FE_OK;
        cudaError_t err = fe::launch_linear_layernorm(x, w.p, e->zero_bias.as<float>(), norm_w.as<float>(), nullptr, h,
                                                      out16, T, n, k, eps, e->ln_ws.p, nullptr, s, &st, true);
        if (st != FE_OK) return st;
        return fe::check_cuda(err, "linear+RMSNorm");
    };
    // the deferred form: h32 <- x W^T + h32, out16 <- bf16(h32 * norm_w), rss <- row sums of squares
    auto linear_rms_deferred = [&](const void *x, const DevBuf &w, const DevBuf &norm_w, float *h, void *out16,
                                   int64_t n, int64_t k) -> fe_status {
        Scope sc(e, CAT_GEMM, s, "fe.linear_rmsnorm_deferred");
        fe_status st = FE_OK;
        cudaError_t err = fe::launch_linear_rms_deferred(x, w.p, e->zero_bias.as<float>(), norm_w.as<float>(), h, out16,
                                                         rss, T, n, k, s, &st);
        if (st != FE_OK) return st;
        return fe::check_cuda(err, "linear+deferred RMSNorm");
    };
    {
        Scope sc(e, CAT_OTHER, s, "fe.embed_scale");
        // Gemma3 scales the embeddings by sqrt(hidden) (rounded to fp32); Qwen3 does not
        const float escale = gemma ? static_cast<float>(std::sqrt(static_cast<double>(D))) : 1.0f;
        FE_TRY_CUDA(fe::launch_embed_scale(ids, T, e->word.as<float>(), c.vocab_size, static_cast<int>(D), escale, h32, s));
        FE_TRY_CUDA(fe::launch_token_positions(cu, batch, e->tpos.as<int32_t>(), s));
    }
    {
        Scope sc(e, CAT_OTHER, s, "fe.rms_norm");
        FE_TRY_CUDA(fe::launch_rms_norm_rows(h32, e->rlayers[0].in_norm.as<float>(), gemma, eps, T, static_cast<int>(D),
                                             nullptr, x16, s));
    }
    float *fin = e->hfin.as<float>();  // the final-norm output (fp32) for pooling
    // The q/k norms and RoPE run in the QKV projection's epilogue when every head group
    // starts on a 256-column tile (FE_QKROPE_FUSE=0: the separate row kernel, for comparison)
    const bool fuse_rope = qkrope_fuse_enabled() && (static_cast<int64_t>(c.q_heads) * hd) % 256 == 0 &&
                           (static_cast<int64_t>(c.kv_heads) * hd) % 256 == 0;
    for (int l = 0; l < c.layers; ++l) {
        const RLayer &L = e->rlayers[l];
        const bool last = l + 1 == c.layers;
        const float *in_ss = defer && l > 0 ? rss : nullptr;  // this layer's input still needs 1 / rms
        if (fuse_rope) {
            // QKV projection with the q/k norms and RoPE in its epilogue
            Scope sc(e, CAT_GEMM, s, "fe.qkv_qk_norm_rope");
            fe_status st = FE_OK;
            cudaError_t err = fe::launch_linear_qk_norm_rope(x16, L.wqkv.p, qkv, T, D, c.q_heads, c.kv_heads,
                                                             static_cast<int>(hd), L.q_norm.as<float>(),
                                                             L.k_norm.as<float>(), e->tpos.as<int32_t>(), gemma, eps,
                                                             layer_theta(c, l), s, &st, in_ss, ss_parts);
            if (st != FE_OK) return st;
            FE_TRY_CUDA(err);
        } else {
            FE_TRY(gemm(x16, L.wqkv, nullptr, nullptr, qkv, QKV, D, FE_EPI_NONE, FE_DTYPE_BF16, in_ss));
            Scope sc(e, CAT_OTHER, s, "fe.qk_norm_rope");
            FE_TRY_CUDA(fe::launch_qk_norm_rope(qkv, cu, batch, T, c.q_heads, c.kv_heads, static_cast<int>(hd),
                                                L.q_norm.as<float>(), L.k_norm.as<float>(), gemma, eps,
                                                layer_theta(c, l), s, e->tpos.as<int32_t>()));
        }
        {
            Scope sc(e, CAT_ATTN, s, "fe.attention_gqa");
            fe_status st = FE_OK;
            cudaError_t err = fe::launch_attention_wide(qkv, cu, batch, max_len, c.q_heads, c.kv_heads,
                                                        static_cast<int>(hd), !gemma, qscale, attn, T, s, &st);
            if (st != FE_OK) return st;
            FE_TRY_CUDA(err);
        }
        const float *next_norm = last ? e->final_norm.as<float>() : e->rlayers[l + 1].in_norm.as<float>();
        if (!gemma && defer) {
            // x <- x + attn Wo^T, x16 <- bf16(x * post_attn_norm) and the row sums of squares;
            // gate_up applies the post-attention RMSNorm's row factor
            FE_TRY(linear_rms_deferred(attn, L.wo, L.post_attn_norm, h32, x16, D, AO));
            FE_TRY(gemm(x16, L.wgu, nullptr, nullptr, ff, 2 * F, D, FE_EPI_SWIGLU, FE_DTYPE_BF16, rss));
            // x <- x + ff Wd^T, x16 <- bf16(x * next input norm) for the next layer's QKV (the
            // final norm: below, in fp32, from h32)
            FE_TRY(linear_rms_deferred(ff, L.wd, last ? e->final_norm : e->rlayers[l + 1].in_norm, h32,
                                       last ? nullptr : x16, D, F));
            if (last) {
                Scope sc(e, CAT_OTHER, s, "fe.rms_norm");
                FE_TRY_CUDA(fe::launch_rms_norm_rows(h32, next_norm, false, eps, T, static_cast<int>(D), fin, nullptr,
                                                     s));
            }
        } else if (!gemma) {
            // x <- x + attn Wo^T and the post-attention RMSNorm into x16, one fused step
            FE_TRY(linear_rms(attn, L.wo, L.post_attn_norm, h32, x16, D, AO));
            FE_TRY(gemm(x16, L.wgu, nullptr, nullptr, ff, 2 * F, D, FE_EPI_SWIGLU, FE_DTYPE_BF16));
            // x <- x + ff Wd^T and the next layer's input RMSNorm (the final norm: below, in fp32)
            FE_TRY(linear_rms(ff, L.wd, last ? e->final_norm : e->rlayers[l + 1].in_norm, h32, last ? nullptr : x16, D,
                              F));
            if (last) {
                Scope sc(e, CAT_OTHER, s, "fe.rms_norm");
                FE_TRY_CUDA(fe::launch_rms_norm_rows(h32, next_norm, false, eps, T, static_cast<int>(D), fin, nullptr,
                                                     s));
            }
        } else {
            // x <- x + rms(attn Wo^T), then the pre-FFN norm, in one row kernel
            // o_proj and down_proj are written in bf16 (y16, in the y32 buffer): the sandwich
            // step normalises them before they reach the fp32 residual stream, and bf16 halves
            // both their store and the sandwich's read
            void *y16 = y32;
            FE_TRY(gemm(attn, L.wo, nullptr, nullptr, y16, D, AO, FE_EPI_NONE, FE_DTYPE_BF16));
            {
                Scope sc(e, CAT_OTHER, s, "fe.rms_sandwich");
                FE_TRY_CUDA(fe::launch_rms_sandwich(y16, L.post_attn_norm.as<float>(), h32, L.pre_ff_norm.as<float>(),
                                                    true, eps, T, static_cast<int>(D), nullptr, x16, s, true));
            }
            FE_TRY(gemm(x16, L.wgu, nullptr, nullptr, ff, 2 * F, D, FE_EPI_GEGLU, FE_DTYPE_BF16));
            FE_TRY(gemm(ff, L.wd, nullptr, nullptr, y16, D, F, FE_EPI_NONE, FE_DTYPE_BF16));
            {
                Scope sc(e, CAT_OTHER, s, "fe.rms_sandwich");
                FE_TRY_CUDA(fe::launch_rms_sandwich(y16, L.post_ff_norm.as<float>(), h32, next_norm, true, eps, T,
                                                    static_cast<int>(D), last ? fin : nullptr, last ? nullptr : x16,
                                                    s, true));
            }
        }
    }
    {
        Scope sc(e, CAT_OTHER, s, "fe.pool_l2");
        FE_TRY_CUDA(fe::launch_pool_l2(fin, cu, batch, static_cast<int>(D), c.pooling, out, s));
    }
    return FE_OK;
}

bool config_rms_ok(const fe_rms_encoder_config *c, std::string &why)
{
    if (c->family != FE_FAMILY_QWEN3 && c->family != FE_FAMILY_GEMMA3) {
        why = "family must be FE_FAMILY_QWEN3 or FE_FAMILY_GEMMA3";
        return false;
    }
    if (c->vocab_size <= 0 || c->hidden <= 0 || c->layers <= 0 || c->q_heads <= 0 || c->kv_heads <= 0 ||
        c->intermediate <= 0 || c->max_position <= 0) {
        why = "all sizes must be positive";
        return false;
    }
    if (c->head_dim != 128 && c->head_dim != 256) {
        why = "head_dim must be 128 or 256";
        return false;
    }
    if (c->q_heads % c->kv_heads != 0) {
        why = "q_heads must be a multiple of kv_heads";
        return false;
    }
    const int v = c->hidden / 128;
    if (c->hidden % 128 != 0 || !(v == 2 || v == 3 || v == 4 || v == 6 || v == 8 || v == 12 || v == 16)) {
        why = "hidden must be 256, 384, 512, 768, 1024, 1536 or 2048";
        return false;
    }
    if (c->intermediate % 64 != 0) {
        why = "intermediate must be a multiple of 64";
        return false;
    }
    if (!(c->rope_theta > 1.0f) || (c->full_attention_every > 0 && !(c->rope_theta_local > 1.0f))) {
        why = "rope_theta must be above 1";
        return false;
    }
    if (c->pooling < FE_POOL_CLS || c->pooling > FE_POOL_LAST) {
        why = "unknown pooling";
        return false;
    }
    return true;
}

bool config_ok(const fe_encoder_config *c, std::string &why)
{
    if (c->hidden <= 0 || c->layers <= 0 || c->heads <= 0 || c->intermediate <= 0 || c->vocab_size <= 0 ||
        c->max_position <= 0 || c->type_vocab <= 0) {
        why = "all sizes must be positive";
        return false;
    }
    if (c->hidden % c->heads != 0) {
        why = "Embedding dimension must be divisible by number of heads";
        return false;
    }
    if (c->positions != FE_POSITIONS_BERT && c->positions != FE_POSITIONS_XLMR) {
        why = "positions must be FE_POSITIONS_BERT or FE_POSITIONS_XLMR";
        return false;
    }
    if (c->positions == FE_POSITIONS_XLMR && c->pad_token_id < 0) {
        why = "pad_token_id must be >= 0 for the XLM-R position rows";
        return false;
    }
    if (c->hidden / c->heads != 64) {
        why = "head_dim must be 64";
        return false;
    }
    const int v = c->hidden / 128;
    if (c->hidden % 128 != 0 || !(v == 2 || v == 3 || v == 4 || v == 6 || v == 8 || v == 12 || v == 16)) {
        why = "hidden must be 256, 384, 512, 768, 1024, 1536 or 2048";
        return false;
    }
    if (c->intermediate % 8 != 0) {
        why = "intermediate must be a multiple of 8";
        return false;
    }
    if (c->activation < FE_ACT_GELU || c->activation > FE_ACT_SWISH) {
        why = "unknown activation";
        return false;
    }
    if (c->pooling < FE_POOL_CLS || c->pooling > FE_POOL_LAST) {
        why = "unknown pooling";
        return false;
    }
    return true;
}

struct DeviceGuard {
    int prev = 0;
    explicit DeviceGuard(int d) { cudaGetDevice(&prev); cudaSetDevice(d); }
    ~DeviceGuard() { cudaSetDevice(prev); }
};

// Tokens per device pass of fe_engine_encode_host: FE_MAX_TOKENS_PER_PASS, else 262,144
// (about 7 GB of bge-large activations).
int64_t max_tokens_per_pass()
{
    if (const char *v = std::getenv("FE_MAX_TOKENS_PER_PASS")) {
        const long long n = std::atoll(v);
        if (n > 0) return n;
    }
    return 262144;
}

}  // namespace

extern "C" {

fe_status fe_engine_create(const fe_encoder_config *cfg, int device, fe_engine **out)
{
    if (!cfg || !out) return fail(FE_ERR_INVALID_ARGUMENT, "fe_engine_create: null argument");
    *out = nullptr;
    std::string why;
    if (!config_ok(cfg, why)) return fail(FE_ERR_UNSUPPORTED, "fe_engine_create: " + why);
    int n = 0;
    FE_TRY_CUDA(cudaGetDeviceCount(&n));
    if (device < 0 || device >= n) return fail(FE_ERR_INVALID_ARGUMENT, "fe_engine_create: bad device index");
    cudaDeviceProp prop{};
    FE_TRY_CUDA(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10) return fail(FE_ERR_UNSUPPORTED, "fe_engine_create: this build targets sm_100a (B200)");
    DeviceGuard g(device);
    auto *e = new fe_engine();
    e->cfg = *cfg;
    e->device = device;
    cudaError_t err = cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking);
    if (err != cudaSuccess) {
        delete e;
        return fe::check_cuda(err, "cudaStreamCreate");
    }
    fe_status st = alloc_weights(e);
    if (st != FE_OK) {
        fe_engine_destroy(e);
        return st;
    }
    *out = e;
    return FE_OK;
}

fe_status fe_engine_create_rms(const fe_rms_encoder_config *cfg, int device, fe_engine **out)
{
    if (!cfg || !out) return fail(FE_ERR_INVALID_ARGUMENT, "fe_engine_create_rms: null argument");
    *out = nullptr;
    std::string why;
    if (!config_rms_ok(cfg, why)) return fail(FE_ERR_UNSUPPORTED, "fe_engine_create_rms: " + why);
    int n = 0;
    FE_TRY_CUDA(cudaGetDeviceCount(&n));
    if (device < 0 || device >= n) return fail(FE_ERR_INVALID_ARGUMENT, "fe_engine_create_rms: bad device index");
    cudaDeviceProp prop{};
    FE_TRY_CUDA(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10) return fail(FE_ERR_UNSUPPORTED, "fe_engine_create_rms: this build targets sm_100a (B200)");
    DeviceGuard g(device);
    auto *e = new fe_engine();
    e->family = cfg->family;
    e->rc = *cfg;
    e->device = device;
    cudaError_t err = cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking);
    if (err != cudaSuccess) {
        delete e;
        return fe::check_cuda(err, "cudaStreamCreate");
    }
    fe_status st = alloc_weights_rms(e);
    if (st != FE_OK) {
        fe_engine_destroy(e);
        return st;
    }
    *out = e;
    return FE_OK;
}

fe_status fe_engine_destroy(fe_engine *e)
{
    if (!e) return FE_OK;
    DeviceGuard g(e->device);
    if (e->stream) cudaStreamSynchronize(e->stream);
    for (auto x : e->ev) cudaEventDestroy(x);
    if (e->stream) cudaStreamDestroy(e->stream);
    delete e;
    return FE_OK;
}

fe_status fe_engine_set_weight(fe_engine *e, const char *name, const float *data, size_t count, int data_on_device)
{
    if (!e || !name || (count && !data)) return fail(FE_ERR_INVALID_ARGUMENT, "fe_engine_set_weight: null argument");
    auto it = e->slots.find(name);
    if (it == e->slots.end() && std::strncmp(name, "model.", 6) == 0) it = e->slots.find(name + 6);
    if (it == e->slots.end()) return fail(FE_ERR_NOT_FOUND, std::string("unknown tensor ") + name);
    const std::string key = it->first;
    const Slot &sl = it->second;
    if (count != sl.count)
        return fail(FE_ERR_INVALID_ARGUMENT, std::string("tensor ") + name + ": expected " + std::to_string(sl.count) +
                                                 " elements, got " + std::to_string(count));
    std::lock_guard<std::mutex> lk(e->mu);
    DeviceGuard g(e->device);
    const cudaMemcpyKind kind = data_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
    if (!sl.bf16) {
        FE_TRY_CUDA(cudaMemcpyAsync(static_cast<float *>(sl.buf->p) + sl.offset, data, count * sizeof(float), kind,
                                    e->stream));
    } else {
        const float *src = data;
        if (!data_on_device) {
            FE_TRY_CUDA(e->staging.ensure(count * sizeof(float)));
            FE_TRY_CUDA(cudaMemcpyAsync(e->staging.p, data, count * sizeof(float), kind, e->stream));
            src = e->staging.as<float>();
        }
        auto *dst = static_cast<__nv_bfloat16 *>(sl.buf->p) + sl.offset;
        if (!sl.interleave) {
            FE_TRY_CUDA(fe::launch_f32_to_bf16(src, dst, static_cast<int64_t>(count), e->stream));
        } else {
            // [F, row] into every other 32-row block of the [2F, row] gate-up matrix
            FE_TRY_CUDA(e->staging16.ensure(count * sizeof(__nv_bfloat16)));
            FE_TRY_CUDA(fe::launch_f32_to_bf16(src, e->staging16.as<__nv_bfloat16>(), static_cast<int64_t>(count),
                                               e->stream));
            const size_t block = 32 * sl.row * sizeof(__nv_bfloat16);
            FE_TRY_CUDA(cudaMemcpy2DAsync(dst + (sl.interleave == 2 ? 32 * sl.row : 0), 2 * block, e->staging16.p,
                                          block, block, count / (32 * sl.row), cudaMemcpyDeviceToDevice, e->stream));
        }
    }
    FE_TRY_CUDA(cudaStreamSynchronize(e->stream));
    e->loaded[key] = true;
    return FE_OK;
}

int32_t fe_engine_missing_weights(const fe_engine *e)
{
    if (!e) return -1;
    int32_t n = 0;
    for (auto &kv : e->loaded) n += kv.second ? 0 : 1;
    return n;
}

fe_status fe_engine_load_safetensors(fe_engine *e, const char *path)
{
    if (!e || !path) return fail(FE_ERR_INVALID_ARGUMENT, "fe_engine_load_safetensors: null argument");
    const int fd = ::open(path, O_RDONLY);
    if (fd < 0) return fail(FE_ERR_IO, std::string("cannot open ") + path);
    struct stat sb;
    if (fstat(fd, &sb) != 0 || sb.st_size < 8) {
        ::close(fd);
        return fail(FE_ERR_IO, std::string("not a safetensors file: ") + path);
    }
    const size_t size = static_cast<size_t>(sb.st_size);
    void *map = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (map == MAP_FAILED) return fail(FE_ERR_IO, std::string("mmap failed: ") + path);
    const uint8_t *base = static_cast<const uint8_t *>(map);
    fe_status result = FE_OK;
    try {
        uint64_t hlen = 0;
        std::memcpy(&hlen, base, 8);  // little-endian header length (src/safetensors.cpp:38-45)
        if (hlen > size - 8) throw std::runtime_error("header length past end of file");
        const fe::json::Value hdr = fe::json::parse(std::string(reinterpret_cast<const char *>(base + 8), hlen));
        const uint8_t *data = base + 8 + hlen;
        const size_t data_size = size - 8 - hlen;
        std::vector<float> buf;
        for (const auto &kv : hdr.obj) {
            if (kv.first == "__metadata__") continue;
            if (!e->slots.count(kv.first)) continue;  // e.g. pooler.* is read but unused by the forward
            const auto &t = kv.second;
            const std::string &dt = t.at("dtype").as_string();
            const auto &off = t.at("data_offsets").arr;
            if (off.size() != 2) throw std::runtime_error("bad data_offsets for " + kv.first);
            const size_t a = static_cast<size_t>(off[0].as_number()), b = static_cast<size_t>(off[1].as_number());
            if (a > b || b > data_size) throw std::runtime_error("data_offsets out of range for " + kv.first);
            size_t n = 0;
            if (dt == "F32") {
                n = (b - a) / 4;
                buf.resize(n);
                std::memcpy(buf.data(), data + a, n * 4);
            } else if (dt == "BF16") {  // widened by placing the 16 bits on top (src/safetensors.cpp:22-28)
                n = (b - a) / 2;
                buf.resize(n);
                for (size_t i = 0; i < n; ++i) {
                    uint16_t h;
                    std::memcpy(&h, data + a + 2 * i, 2);
                    const uint32_t u = static_cast<uint32_t>(h) << 16;
                    std::memcpy(&buf[i], &u, 4);
                }
            } else {
                continue;  // other dtypes are skipped, as the reference does (src/safetensors.cpp:85-87)
            }
            fe_status st = fe_engine_set_weight(e, kv.first.c_str(), buf.data(), n, 0);
            if (st != FE_OK) {
                result = st;
                break;
            }
        }
    } catch (const std::exception &ex) {
        result = fail(FE_ERR_IO, std::string("malformed safetensors file ") + path + ": " + ex.what());
    }
    munmap(map, size);
    return result;
}

fe_status fe_engine_encode_packed(fe_engine *e, const int32_t *ids, const int32_t *cu_seqlens,
                                  const int32_t *cu_seqlens_host, int32_t batch, float *out, fe_stream_t stream)
{
    if (!e || batch < 0 || (batch && (!ids || !cu_seqlens || !cu_seqlens_host || !out)))
        return fail(FE_ERR_INVALID_ARGUMENT, "fe_engine_encode_packed: bad arguments");
    if (fe_engine_missing_weights(e) != 0)
        return fail(FE_ERR_INVALID_ARGUMENT, "fe_engine_encode_packed: weights not loaded");
    if (batch > 65535) return fail(FE_ERR_UNSUPPORTED, "fe_engine_encode_packed: batch too large");
    std::lock_guard<std::mutex> lk(e->mu);
    DeviceGuard g(e->device);
    cudaStream_t s = stream ? reinterpret_cast<cudaStream_t>(stream) : e->stream;
    if (batch == 0) return FE_OK;
    if (e->family != FE_FAMILY_BERT) return forward_rms(e, ids, cu_seqlens, cu_seqlens_host, batch, out, s);
    return forward(e, ids, cu_seqlens, cu_seqlens_host, batch, out, s);
}

fe_status fe_engine_encode_host(fe_engine *e, const int32_t *ids, const int32_t *lengths, int32_t batch,
                                int32_t stride, float *out)
{
    if (!e || batch < 0 || stride < 0 || (batch && (!ids || !lengths || !out)))
        return fail(FE_ERR_INVALID_ARGUMENT, "fe_engine_encode_host: bad arguments");
    if (fe_engine_missing_weights(e) != 0)
        return fail(FE_ERR_INVALID_ARGUMENT, "fe_engine_encode_host: weights not loaded");
    if (batch == 0) return FE_OK;
    std::lock_guard<std::mutex> lk(e->mu);
    DeviceGuard g(e->device);
    for (int b = 0; b < batch; ++b)
        if (lengths[b] < 0 || lengths[b] > stride)
            return fail(FE_ERR_INVALID_ARGUMENT, "fe_engine_encode_host: length outside [0, stride]");
    const size_t D = e->family == FE_FAMILY_BERT ? e->cfg.hidden : e->rc.hidden;
    // Consecutive sentences run as one device pass of at most max_tokens_per_pass() tokens
    // (a longer single sentence runs alone) and kMaxPassSentences sentences (the device
    // path's batch limit): activation memory stays bounded for any batch.
    const int64_t cap = max_tokens_per_pass();
    constexpr int kMaxPassSentences = 65535;
    cudaStream_t s = e->stream;
    int *w = fe::device_status_word(e->device);
    if (!w) return fail(FE_ERR_CUDA, "fe_engine_encode_host: no device status word");
    FE_TRY_CUDA(e->p_status.ensure(sizeof(int)));
    for (int b0 = 0; b0 < batch;) {
        int b1 = b0;
        int64_t T = 0;
        while (b1 < batch && b1 - b0 < kMaxPassSentences && (b1 == b0 || T + lengths[b1] <= cap)) T += lengths[b1++];
        const int nb = b1 - b0;
        FE_TRY_CUDA(e->p_ids.ensure(std::max<int64_t>(T, 1) * 4));
        FE_TRY_CUDA(e->p_cu.ensure((nb + 1) * 4));
        FE_TRY_CUDA(e->p_out.ensure(nb * D * 4));
        FE_TRY_CUDA(e->d_ids.ensure(std::max<int64_t>(T, 1) * 4));
        FE_TRY_CUDA(e->d_cu.ensure((nb + 1) * 4));
        FE_TRY_CUDA(e->d_out.ensure(nb * D * 4));
        FE_TRY(fe_pack_batch(ids + static_cast<size_t>(b0) * stride, lengths + b0, nb, stride, e->p_ids.as<int32_t>(),
                             e->p_cu.as<int32_t>()));
        FE_TRY_CUDA(cudaMemcpyAsync(e->d_ids.p, e->p_ids.p, T * 4, cudaMemcpyHostToDevice, s));
        FE_TRY_CUDA(cudaMemcpyAsync(e->d_cu.p, e->p_cu.p, (nb + 1) * 4, cudaMemcpyHostToDevice, s));
        if (e->family != FE_FAMILY_BERT)
            FE_TRY(forward_rms(e, e->d_ids.as<int32_t>(), e->d_cu.as<int32_t>(), e->p_cu.as<int32_t>(), nb,
                               e->d_out.as<float>(), s));
        else
            FE_TRY(forward(e, e->d_ids.as<int32_t>(), e->d_cu.as<int32_t>(), e->p_cu.as<int32_t>(), nb,
                           e->d_out.as<float>(), s));
        FE_TRY_CUDA(cudaMemcpyAsync(e->p_out.p, e->d_out.p, nb * D * 4, cudaMemcpyDeviceToHost, s));
        // the device status word comes back with the embeddings: a pass whose kernels met a
        // bad token id or a wait that ran out ends the call before the next pass starts
        FE_TRY_CUDA(cudaMemcpyAsync(e->p_status.p, w, sizeof(int), cudaMemcpyDeviceToHost, s));
        FE_TRY_CUDA(cudaStreamSynchronize(s));  // the pinned buffers are reused by the next pass
        const int v = *e->p_status.as<int>();
        if (v != 0) {
            FE_TRY_CUDA(cudaMemsetAsync(w, 0, sizeof(int), s));
            FE_TRY_CUDA(cudaStreamSynchronize(s));
            if (v == fe::DEV_BAD_INPUT) return fail(FE_ERR_INVALID_ARGUMENT, "token id outside the vocabulary");
            return fail(FE_ERR_DEVICE_TIMEOUT, "a kernel's bounded wait ran out");
        }
        std::memcpy(out + static_cast<size_t>(b0) * D, e->p_out.p, nb * D * 4);
        b0 = b1;
    }
    return FE_OK;
}

fe_status fe_engine_set_profiling(fe_engine *e, int enabled)
{
    if (!e) return fail(FE_ERR_INVALID_ARGUMENT, "fe_engine_set_profiling: null engine");
    std::lock_guard<std::mutex> lk(e->mu);
    e->profiling = enabled != 0;
    return FE_OK;
}

fe_status fe_engine_get_stats(const fe_engine *ce, fe_engine_stats *stats)
{
    if (!ce || !stats) return fail(FE_ERR_INVALID_ARGUMENT, "fe_engine_get_stats: null argument");
    auto *e = const_cast<fe_engine *>(ce);
    std::lock_guard<std::mutex> lk(e->mu);
    DeviceGuard g(e->device);
    e->stats.gemm_ms = e->stats.attention_ms = e->stats.other_ms = 0;
    if (e->profiling && e->ev_used) {
        FE_TRY_CUDA(cudaEventSynchronize(e->ev[e->ev_used - 1]));
        for (size_t i = 0; i + 1 < e->ev_used; i += 2) {
            float ms = 0;
            FE_TRY_CUDA(cudaEventElapsedTime(&ms, e->ev[i], e->ev[i + 1]));
            const int cat = e->ev_cat[i / 2];
            if (cat == CAT_GEMM) e->stats.gemm_ms += ms;
            else if (cat == CAT_ATTN) e->stats.attention_ms += ms;
            else e->stats.other_ms += ms;
        }
    }
    *stats = e->stats;
    return FE_OK;
}

}  // extern "C"
