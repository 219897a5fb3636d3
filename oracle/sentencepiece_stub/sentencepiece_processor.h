// Stand-in for the SentencePiece C++ header (not installed here), so that the reference's
// src/tokenizer.cpp compiles unmodified for the BGE WordPiece checker (ref_tokenizer.cpp).
//
// TEST INFRASTRUCTURE ONLY.  Only the names tokenizer.cpp uses are declared; the checker
// never constructs an XLMRobertaTokenizer, and every method here reports failure.
#pragma once

#include <string>
#include <vector>

namespace sentencepiece {
namespace util {
class Status {
public:
    bool ok() const { return false; }
    std::string ToString() const { return "SentencePiece is not part of this checker"; }
};
}  // namespace util

class SentencePieceProcessor {
public:
    util::Status Load(const std::string &) { return {}; }
    util::Status Encode(const std::string &, std::vector<std::string> *) const { return {}; }
    util::Status Encode(const std::string &, std::vector<int> *) const { return {}; }
    util::Status Decode(const std::vector<int> &, std::string *) const { return {}; }
};
}  // namespace sentencepiece
