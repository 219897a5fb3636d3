// sentence_transformers.cpp — the drop-in SentenceTransformer over the device engine.
//
// Construction mirrors SentenceTransformerImpl's (src/sentence_transformers_impl.cpp:46-98):
// config.json, a WordPiece vocabulary (vocab.txt) and model.safetensors from one model
// directory.  encode / encode_batch tokenise on the host (BGE WordPiece, then [CLS]=101
// in front and [SEP]=102 behind, :11-27) and run every sentence of the batch in one
// packed device pass per GPU instead of a per-text loop (:359-365).  With FE_DEVICES
// listing several GPUs, a batch is sorted by length and cut into contiguous slices of
// equal estimated time (fe_plan_shards: projection FLOPs plus a per-tile attention cost),
// one per GPU, each run by its own host thread; there is no device-to-device traffic.
#include <cuda_runtime.h>

#include <algorithm>
#include <cctype>
#include <cstdio>
#include <cstdlib>
#include <exception>
#include <fstream>
#include <iostream>
#include <mutex>
#include <numeric>
#include <sstream>
#include <stdexcept>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include "coalescer.h"
#include "fastembed_b200.h"
#include "json_min.h"
#include "sentence_transformers.h"
#include "wordpiece.h"

namespace {

using fe::WordPiece;

void check(fe_status st, const std::string &where)
{
    if (st == FE_OK) return;
    const std::string msg = where + ": " + fe_last_error_message();
    if (st == FE_ERR_INVALID_ARGUMENT) throw std::invalid_argument(msg);
    throw std::runtime_error(msg);
}

std::string read_file(const std::string &path)
{
    std::ifstream f(path, std::ios::binary);
    if (!f.is_open()) throw std::runtime_error("cannot open " + path);
    std::stringstream ss;
    ss << f.rdbuf();
    return ss.str();
}

int cfg_int(const fe::json::Value &cfg, const char *key, int fallback)
{
    return cfg.has(key) ? static_cast<int>(cfg.at(key).as_number()) : fallback;
}

}  // namespace

class SentenceTransformerImpl {
public:
    explicit SentenceTransformerImpl(const std::string &model_path)
    {
        const fe::json::Value cfg = fe::json::parse(read_file(model_path + "/config.json"));
        std::string type = "bge";
        if (cfg.has("model_type")) type = cfg.at("model_type").as_string();
        else if (cfg.has("model") && cfg.at("model").has("model_type")) type = cfg.at("model").at("model_type").as_string();
        // (:64-72) "bge" / "bert" -> BGE; "bge-m3" / "xlm-roberta" -> BGE_M3; anything else
        // is taken as BGE_M3 with a warning
        const bool bert = type == "bge" || type == "bert";
        if (!bert && type != "bge-m3" && type != "xlm-roberta")
            std::cerr << "warning: unknown model_type '" << type << "', using bge-m3" << std::endl;
        fe_encoder_config c{};
        if (!bert) {  // position rows of create_position_ids_from_input_ids (:101-123, :139-155)
            c.positions = FE_POSITIONS_XLMR;
            c.pad_token_id = cfg_int(cfg, "pad_token_id", 0);
        }
        c.vocab_size = cfg_int(cfg, "vocab_size", 0);
        c.hidden = cfg_int(cfg, "hidden_size", 0);
        c.layers = cfg_int(cfg, "num_hidden_layers", 0);
        c.heads = cfg_int(cfg, "num_attention_heads", 0);
        c.intermediate = cfg_int(cfg, "intermediate_size", 0);
        c.max_position = cfg_int(cfg, "max_position_embeddings", 512);
        c.type_vocab = cfg_int(cfg, "type_vocab_size", 2);
        c.layer_norm_eps = cfg.has("layer_norm_eps") ? static_cast<float>(cfg.at("layer_norm_eps").as_number()) : 1e-12f;
        const std::string act = cfg.has("hidden_act") ? cfg.at("hidden_act").as_string() : "gelu";
        if (act == "gelu") c.activation = FE_ACT_GELU;
        else if (act == "relu") c.activation = FE_ACT_RELU;
        else if (act == "swish") c.activation = FE_ACT_SWISH;
        else throw std::runtime_error("Unsupported activation function");  // (:413-421)
        c.pooling = FE_POOL_CLS;
        cfg_ = c;
        // bge-m3 tokenises with SentencePiece (tokenizer.cpp:176-301), which this build does
        // not include: such models take token ids through encode_ids
        if (bert) tokenizer_.reset(new WordPiece(model_path + "/vocab.txt"));

        for (int dev : devices()) {
            check(cudaSetDevice(dev) == cudaSuccess ? FE_OK : FE_ERR_CUDA, "cudaSetDevice");
            fe_engine *e = nullptr;
            check(fe_engine_create(&cfg_, dev, &e), "fe_engine_create");
            engines_.push_back(e);
            fe_status st = fe_engine_load_safetensors(e, (model_path + "/model.safetensors").c_str());
            if (st == FE_OK && fe_engine_missing_weights(e) != 0)
                throw std::runtime_error("model.safetensors lacks some encoder weights");
            check(st, "load model.safetensors");
        }
    }

    ~SentenceTransformerImpl()
    {
        for (fe_engine *e : engines_) fe_engine_destroy(e);
    }

    size_t dim() const { return static_cast<size_t>(cfg_.hidden); }

    std::vector<int32_t> tokenize(const std::string &text) const
    {
        if (!tokenizer_)
            throw std::runtime_error("bge-m3 / XLM-R text needs the SentencePiece tokenizer, which this build does not "
                                     "include; pass token ids (<s> ... </s>) to encode_ids");
        std::vector<int32_t> ids = tokenizer_->ids(text);
        ids.insert(ids.begin(), 101);
        ids.push_back(102);
        return ids;
    }

    // A batch's texts tokenised on host threads: contiguous chunks of at least 32 texts, at
    // most 32 threads (WordPiece::ids only reads the vocabulary).
    std::vector<std::vector<int32_t>> tokenize_all(const std::vector<std::string> &texts) const
    {
        const size_t n = texts.size();
        std::vector<std::vector<int32_t>> seqs(n);
        const size_t hw = std::max<size_t>(1, std::thread::hardware_concurrency());
        const size_t workers = std::min<size_t>({hw, 32, (n + 31) / 32});
        if (workers <= 1) {
            for (size_t i = 0; i < n; ++i) seqs[i] = tokenize(texts[i]);
            return seqs;
        }
        std::vector<std::exception_ptr> errs(workers);
        std::vector<std::thread> pool;
        for (size_t w = 0; w < workers; ++w)
            pool.emplace_back([&, w] {
                try {
                    for (size_t i = n * w / workers; i < n * (w + 1) / workers; ++i) seqs[i] = tokenize(texts[i]);
                } catch (...) {
                    errs[w] = std::current_exception();
                }
            });
        for (auto &t : pool) t.join();
        for (const auto &e : errs)
            if (e) std::rethrow_exception(e);
        return seqs;
    }

    // Concurrent calls (threads sharing this object, as the reference's HTTP server does)
    // are merged into one device batch by the coalescer; the engine's outputs do not
    // depend on which other sentences share the batch.
    std::vector<std::vector<float>> run(const std::vector<std::vector<int32_t>> &seqs)
    {
        for (const auto &s : seqs)
            if (static_cast<int>(s.size()) > cfg_.max_position)
                throw std::runtime_error("sequence longer than the position embedding table");  // (:132-136)
        if (seqs.empty()) return {};
        return coalescer_.submit(seqs);
    }

private:
    // One packed pass per GPU over `seqs` (run by one thread at a time, the coalescer's leader).
    std::vector<std::vector<float>> run_batch(const std::vector<std::vector<int32_t>> &seqs)
    {
        const int B = static_cast<int>(seqs.size());
        std::vector<std::vector<float>> out(B, std::vector<float>(dim()));
        if (B == 0) return out;
        // longest first, so that contiguous slices are balanced by fe_plan_shards
        std::vector<int> order(B);
        std::iota(order.begin(), order.end(), 0);
        std::stable_sort(order.begin(), order.end(),
                         [&](int a, int b) { return seqs[a].size() > seqs[b].size(); });
        std::vector<int32_t> lens(B);
        int stride = 1;
        for (int i = 0; i < B; ++i) {
            lens[i] = static_cast<int32_t>(seqs[order[i]].size());
            stride = std::max(stride, static_cast<int>(lens[i]));
        }
        const int parts = std::min<int>(static_cast<int>(engines_.size()), B);
        std::vector<int32_t> cuts(std::max(parts - 1, 1));
        check(fe_plan_shards(&cfg_, lens.data(), B, parts, cuts.data()), "fe_plan_shards");
        std::vector<int> bounds{0};
        for (int p = 0; p + 1 < parts; ++p) bounds.push_back(cuts[p]);
        bounds.push_back(B);

        std::vector<fe_status> status(parts, FE_OK);
        std::vector<std::string> errors(parts);
        auto work = [&](int p) {
            const int b0 = bounds[p], nb = bounds[p + 1] - b0;
            if (nb == 0) return;
            std::vector<int32_t> ids(static_cast<size_t>(nb) * stride, 0), sl(nb);
            for (int i = 0; i < nb; ++i) {
                const auto &s = seqs[order[b0 + i]];
                std::copy(s.begin(), s.end(), ids.begin() + static_cast<size_t>(i) * stride);
                sl[i] = static_cast<int32_t>(s.size());
            }
            std::vector<float> emb(static_cast<size_t>(nb) * dim());
            status[p] = fe_engine_encode_host(engines_[p], ids.data(), sl.data(), nb, stride, emb.data());
            if (status[p] != FE_OK) {
                errors[p] = fe_last_error_message();
                return;
            }
            for (int i = 0; i < nb; ++i)
                std::copy(emb.begin() + static_cast<size_t>(i) * dim(), emb.begin() + static_cast<size_t>(i + 1) * dim(),
                          out[order[b0 + i]].begin());
        };
        if (parts == 1) {
            work(0);
        } else {
            std::vector<std::thread> pool;
            for (int p = 0; p < parts; ++p) pool.emplace_back(work, p);
            for (auto &t : pool) t.join();
        }
        for (int p = 0; p < parts; ++p)
            if (status[p] != FE_OK) {
                const std::string msg = "encode on GPU slice " + std::to_string(p) + ": " + errors[p];
                if (status[p] == FE_ERR_INVALID_ARGUMENT) throw std::invalid_argument(msg);
                throw std::runtime_error(msg);
            }
        return out;
    }

    fe_encoder_config cfg_{};
    std::unique_ptr<WordPiece> tokenizer_;
    std::vector<fe_engine *> engines_;
    fe::Coalescer<std::vector<int32_t>, std::vector<float>> coalescer_{
        [this](const std::vector<std::vector<int32_t>> &seqs) { return run_batch(seqs); }, coalesce_limit()};

    // Sentences per merged batch: FE_COALESCE_MAX (0 turns merging off), else 256 per GPU.
    static size_t coalesce_limit()
    {
        if (const char *env = std::getenv("FE_COALESCE_MAX")) return static_cast<size_t>(std::strtoul(env, nullptr, 10));
        return 256 * devices().size();
    }

    static std::vector<int> devices()
    {
        std::vector<int> out;
        if (const char *env = std::getenv("FE_DEVICES")) {
            std::stringstream ss(env);
            std::string tok;
            while (std::getline(ss, tok, ','))
                if (!tok.empty()) out.push_back(std::stoi(tok));
        }
        if (out.empty()) out.push_back(0);
        return out;
    }
};

SentenceTransformer::SentenceTransformer(const std::string &model_path) : impl(new SentenceTransformerImpl(model_path)) {}
SentenceTransformer::~SentenceTransformer() = default;
SentenceTransformer::SentenceTransformer(SentenceTransformer &&) noexcept = default;
SentenceTransformer &SentenceTransformer::operator=(SentenceTransformer &&) noexcept = default;

std::vector<float> SentenceTransformer::encode(const std::string &text)
{
    std::vector<int32_t> ids = impl->tokenize(text);
    if (const char *p = std::getenv("FE_PRINT_TOKENS"); p && p[0] == '1') {  // (:350-354)
        std::cout << "tokens: " << std::endl;
        for (int32_t t : ids) std::cout << t << " ";
        std::cout << std::endl;
    }
    return impl->run({ids})[0];
}

std::vector<std::vector<float>> SentenceTransformer::encode_batch(const std::vector<std::string> &texts)
{
    return impl->run(impl->tokenize_all(texts));
}

std::vector<std::vector<float>> SentenceTransformer::encode_ids(const std::vector<std::vector<int32_t>> &ids)
{
    return impl->run(ids);
}

size_t SentenceTransformer::get_embedding_dimension() const { return impl->dim(); }

std::vector<int32_t> SentenceTransformer::tokenize(const std::string &text) const { return impl->tokenize(text); }
