// wordpiece.h — the BGE WordPiece tokenizer of the drop-in SentenceTransformer, host only.
// Replaces the reference's BGETokenizer (include/tokenizer.h:11-23, src/tokenizer.cpp:9-160);
// the C ABI exposes it as fe_wordpiece_* (include/fastembed_b200.h).
#pragma once

#include <cctype>
#include <cstdint>
#include <fstream>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

namespace fe {

// BGE WordPiece tokenizer with the reference's behaviour (src/tokenizer.cpp:9-160):
// whitespace separates words; every non-ASCII UTF-8 character is a word of its own;
// ASCII letters and digits accumulate lower-cased; any other ASCII byte is a word of
// its own; each word is looked up whole, else split greedily into the longest known
// prefix then "##"-continuations, and becomes a single [UNK] if a piece is missing.
class WordPiece {
public:
    explicit WordPiece(const std::string &vocab_file)
    {
        std::ifstream f(vocab_file);
        if (!f.is_open()) throw std::runtime_error("cannot open vocabulary file: " + vocab_file);
        std::string line;
        int id = 0;
        while (std::getline(f, line)) vocab_[line] = id++;
        auto it = vocab_.find("[UNK]");
        if (it == vocab_.end()) throw std::runtime_error("vocabulary has no [UNK] token");
        unk_ = it->second;
    }

    std::vector<int32_t> ids(const std::string &text) const
    {
        std::vector<int32_t> out;
        for (const std::string &w : words(text)) pieces(w, out);
        return out;
    }

private:
    std::unordered_map<std::string, int32_t> vocab_;
    int32_t unk_ = 0;

    static std::vector<std::string> words(const std::string &text)
    {
        std::vector<std::string> out;
        std::string cur;
        auto flush = [&] {
            if (!cur.empty()) {
                out.push_back(cur);
                cur.clear();
            }
        };
        size_t i = 0;
        while (i < text.size()) {
            const unsigned char c = static_cast<unsigned char>(text[i]);
            if (std::isspace(c)) {
                flush();
                ++i;
                continue;
            }
            if (c & 0x80) {
                size_t n = 0;
                if ((c & 0xE0) == 0xC0) n = 2;
                else if ((c & 0xF0) == 0xE0) n = 3;
                else if ((c & 0xF8) == 0xF0) n = 4;
                if (n == 0 || i + n > text.size()) {  // stray or truncated byte
                    out.push_back("[UNK]");
                    ++i;
                    continue;
                }
                flush();
                out.push_back(text.substr(i, n));
                i += n;
                continue;
            }
            if (std::isalnum(c)) {
                cur.push_back(static_cast<char>(std::tolower(c)));
            } else {
                flush();
                out.push_back(std::string(1, static_cast<char>(c)));
            }
            ++i;
        }
        flush();
        return out;
    }

    void pieces(const std::string &w, std::vector<int32_t> &out) const
    {
        auto whole = vocab_.find(w);
        if (whole != vocab_.end()) {
            out.push_back(whole->second);
            return;
        }
        std::vector<int32_t> found;
        size_t start = 0;
        while (start < w.size()) {
            bool hit = false;
            for (size_t end = w.size(); end > start; --end) {
                const std::string sub = (start > 0 ? "##" : "") + w.substr(start, end - start);
                auto it = vocab_.find(sub);
                if (it != vocab_.end()) {
                    found.push_back(it->second);
                    start = end;
                    hit = true;
                    break;
                }
            }
            if (!hit) {
                out.push_back(unk_);
                return;
            }
        }
        out.insert(out.end(), found.begin(), found.end());
    }
};

}  // namespace fe
