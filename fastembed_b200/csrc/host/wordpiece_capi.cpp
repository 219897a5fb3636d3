// wordpiece_capi.cpp — C ABI of the BGE WordPiece tokenizer (fe_wordpiece_*), host only:
// the reference's BGETokenizer (include/tokenizer.h:11-23) behind plain pointers, with
// the [CLS] / [SEP] framing of SentenceTransformerImpl::tokenize
// (src/sentence_transformers_impl.cpp:11-27).
#include <exception>
#include <new>
#include <string>

#include "fastembed_b200.h"
#include "fe_internal.h"
#include "wordpiece.h"

struct fe_wordpiece {
    fe::WordPiece wp;
    explicit fe_wordpiece(const std::string &path) : wp(path) {}
};

extern "C" {

fe_status fe_wordpiece_create(const char *vocab_path, fe_wordpiece **out)
{
    if (!vocab_path || !out) return fe::fail(FE_ERR_INVALID_ARGUMENT, "fe_wordpiece_create: null argument");
    *out = nullptr;
    try {
        *out = new fe_wordpiece(vocab_path);
    } catch (const std::bad_alloc &) {
        return fe::fail(FE_ERR_OUT_OF_MEMORY, "fe_wordpiece_create: out of host memory");
    } catch (const std::exception &ex) {
        return fe::fail(FE_ERR_IO, std::string("fe_wordpiece_create: ") + ex.what());
    }
    return FE_OK;
}

fe_status fe_wordpiece_destroy(fe_wordpiece *t)
{
    delete t;
    return FE_OK;
}

fe_status fe_wordpiece_encode(const fe_wordpiece *t, const char *text, size_t len, int32_t *ids, size_t capacity,
                              size_t *count)
{
    if (!t || !count || (len && !text) || (capacity && !ids))
        return fe::fail(FE_ERR_INVALID_ARGUMENT, "fe_wordpiece_encode: null argument");
    try {
        const std::vector<int32_t> v = t->wp.ids(std::string(text ? text : "", len));
        *count = v.size() + 2;
        size_t n = 0;
        if (n < capacity) ids[n] = 101;  // [CLS]
        ++n;
        for (int32_t id : v) {
            if (n < capacity) ids[n] = id;
            ++n;
        }
        if (n < capacity) ids[n] = 102;  // [SEP]
    } catch (const std::bad_alloc &) {
        return fe::fail(FE_ERR_OUT_OF_MEMORY, "fe_wordpiece_encode: out of host memory");
    }
    return FE_OK;
}

}  // extern "C"
