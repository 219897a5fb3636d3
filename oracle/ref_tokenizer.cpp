// ref_tokenizer.cpp — drives the reference's own BGETokenizer (src/tokenizer.cpp, compiled
// from its sources by oracle/Makefile into oracle/_ref/) with the [CLS] / [SEP] framing of
// SentenceTransformerImpl::tokenize (src/sentence_transformers_impl.cpp:11-27), to pin the
// drop-in tokenizer (fe_wordpiece_*) token for token.
//
// TEST INFRASTRUCTURE ONLY.  The product library never links this.
#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

#include "tokenizer.h"

extern "C" {

void *fe_ref_tok_create(const char *vocab_path)
{
    try {
        return new BGETokenizer(vocab_path);
    } catch (...) {
        return nullptr;
    }
}

void fe_ref_tok_destroy(void *t) { delete static_cast<BGETokenizer *>(t); }

// Number of ids of `text` (`len` bytes); at most `capacity` of them are written; -1 on error.
long fe_ref_tok_encode(void *t, const char *text, size_t len, int32_t *ids, size_t capacity)
{
    try {
        BGETokenizer &tok = *static_cast<BGETokenizer *>(t);
        std::vector<int> v = tok.encode(tok.tokenize(std::string(text, len)));
        v.insert(v.begin(), 101);
        v.push_back(102);
        for (size_t i = 0; i < v.size() && i < capacity; ++i) ids[i] = v[i];
        return static_cast<long>(v.size());
    } catch (...) {
        return -1;
    }
}

}  // extern "C"
