// sentence_transformers.h — drop-in for fastEmbed's SentenceTransformer
// (include/sentence_transformers.h:12-40 of the reference): same constructor and
// methods, move-only, pimpl.  A model directory holds config.json, vocab.txt and
// model.safetensors, as for the reference.
//
// Beyond the reference: encode_batch runs the whole batch in one device pass (packed,
// unpadded) instead of a loop over texts, encode_ids takes token ids directly, and the
// object is safe to share between threads (the reference's Crow server shares one
// unguarded instance).  FE_DEVICES="0,1,..." spreads each batch over several GPUs, one
// weight replica per GPU; FE_PRINT_TOKENS=1 prints the token ids from encode() as the
// reference does.
#ifndef SENTENCE_TRANSFORMERS_H
#define SENTENCE_TRANSFORMERS_H

#include <cstdint>
#include <memory>
#include <string>
#include <vector>

class SentenceTransformerImpl;

class SentenceTransformer {
public:
    explicit SentenceTransformer(const std::string &model_path);
    ~SentenceTransformer();

    std::vector<float> encode(const std::string &text);
    std::vector<std::vector<float>> encode_batch(const std::vector<std::string> &texts);
    size_t get_embedding_dimension() const;

    // token-id form of encode_batch ([CLS] ... [SEP] included by the caller)
    std::vector<std::vector<float>> encode_ids(const std::vector<std::vector<int32_t>> &ids);
    // the ids encode() runs for `text`: [CLS]=101, WordPiece ids, [SEP]=102
    std::vector<int32_t> tokenize(const std::string &text) const;

    SentenceTransformer(const SentenceTransformer &) = delete;
    SentenceTransformer &operator=(const SentenceTransformer &) = delete;
    SentenceTransformer(SentenceTransformer &&) noexcept;
    SentenceTransformer &operator=(SentenceTransformer &&) noexcept;

private:
    std::unique_ptr<SentenceTransformerImpl> impl;
};

#endif  // SENTENCE_TRANSFORMERS_H
