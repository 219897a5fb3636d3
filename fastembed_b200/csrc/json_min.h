// json_min.h — a small JSON reader for config.json and safetensors headers (the
// reference uses nlohmann::json for both: src/sentence_transformers_impl.cpp:47-54,
// src/safetensors.cpp:31-60).  Parses objects, arrays, strings (with \u escapes),
// numbers, booleans and null into a tree; throws std::runtime_error on bad input.
#pragma once

#include <cctype>
#include <cstdint>
#include <cstdlib>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace fe {
namespace json {

struct Value {
    enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
    bool b = false;
    double num = 0.0;
    std::string str;
    std::vector<Value> arr;
    std::map<std::string, Value> obj;

    bool is_object() const { return kind == Object; }
    bool has(const std::string &k) const { return kind == Object && obj.count(k) != 0; }
    const Value &at(const std::string &k) const
    {
        auto it = obj.find(k);
        if (kind != Object || it == obj.end()) throw std::runtime_error("json: missing key '" + k + "'");
        return it->second;
    }
    double as_number() const
    {
        if (kind != Number) throw std::runtime_error("json: expected a number");
        return num;
    }
    const std::string &as_string() const
    {
        if (kind != String) throw std::runtime_error("json: expected a string");
        return str;
    }
};

class Parser {
public:
    Parser(const char *p, size_t n) : p_(p), end_(p + n) {}

    Value parse()
    {
        Value v = value(0);
        ws();
        if (p_ != end_) throw std::runtime_error("json: trailing characters");
        return v;
    }

private:
    const char *p_;
    const char *end_;

    void ws()
    {
        while (p_ < end_ && (*p_ == ' ' || *p_ == '\n' || *p_ == '\r' || *p_ == '\t')) ++p_;
    }
    char peek()
    {
        ws();
        if (p_ >= end_) throw std::runtime_error("json: unexpected end");
        return *p_;
    }
    void expect(char c)
    {
        if (peek() != c) throw std::runtime_error(std::string("json: expected '") + c + "'");
        ++p_;
    }
    Value value(int depth)
    {
        if (depth > 64) throw std::runtime_error("json: nesting too deep");
        const char c = peek();
        Value v;
        if (c == '{') {
            ++p_;
            v.kind = Value::Object;
            if (peek() == '}') { ++p_; return v; }
            for (;;) {
                if (peek() != '"') throw std::runtime_error("json: expected a key");
                std::string k = string();
                expect(':');
                v.obj[k] = value(depth + 1);
                const char d = peek();
                ++p_;
                if (d == '}') break;
                if (d != ',') throw std::runtime_error("json: expected ',' or '}'");
            }
        } else if (c == '[') {
            ++p_;
            v.kind = Value::Array;
            if (peek() == ']') { ++p_; return v; }
            for (;;) {
                v.arr.push_back(value(depth + 1));
                const char d = peek();
                ++p_;
                if (d == ']') break;
                if (d != ',') throw std::runtime_error("json: expected ',' or ']'");
            }
        } else if (c == '"') {
            v.kind = Value::String;
            v.str = string();
        } else if (c == 't' || c == 'f' || c == 'n') {
            const char *words[3] = {"true", "false", "null"};
            for (int i = 0; i < 3; ++i) {
                const size_t n = std::char_traits<char>::length(words[i]);
                if (static_cast<size_t>(end_ - p_) >= n && std::string(p_, n) == words[i]) {
                    p_ += n;
                    if (i == 2) v.kind = Value::Null;
                    else { v.kind = Value::Bool; v.b = (i == 0); }
                    return v;
                }
            }
            throw std::runtime_error("json: bad literal");
        } else {
            const char *s = p_;
            while (p_ < end_ && (std::isdigit(static_cast<unsigned char>(*p_)) || *p_ == '-' || *p_ == '+' ||
                                 *p_ == '.' || *p_ == 'e' || *p_ == 'E'))
                ++p_;
            if (s == p_) throw std::runtime_error("json: unexpected character");
            v.kind = Value::Number;
            v.num = std::strtod(std::string(s, p_).c_str(), nullptr);
        }
        return v;
    }
    std::string string()
    {
        expect('"');
        std::string out;
        while (p_ < end_ && *p_ != '"') {
            char c = *p_++;
            if (c != '\\') { out.push_back(c); continue; }
            if (p_ >= end_) break;
            c = *p_++;
            switch (c) {
                case 'n': out.push_back('\n'); break;
                case 't': out.push_back('\t'); break;
                case 'r': out.push_back('\r'); break;
                case 'b': out.push_back('\b'); break;
                case 'f': out.push_back('\f'); break;
                case 'u': {
                    if (end_ - p_ < 4) throw std::runtime_error("json: bad \\u escape");
                    unsigned cp = static_cast<unsigned>(std::strtoul(std::string(p_, 4).c_str(), nullptr, 16));
                    p_ += 4;
                    if (cp >= 0xD800 && cp <= 0xDBFF && end_ - p_ >= 6 && p_[0] == '\\' && p_[1] == 'u') {
                        unsigned lo = static_cast<unsigned>(std::strtoul(std::string(p_ + 2, 4).c_str(), nullptr, 16));
                        if (lo >= 0xDC00 && lo <= 0xDFFF) {
                            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                            p_ += 6;
                        }
                    }
                    if (cp < 0x80) out.push_back(static_cast<char>(cp));
                    else if (cp < 0x800) {
                        out.push_back(static_cast<char>(0xC0 | (cp >> 6)));
                        out.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
                    } else if (cp < 0x10000) {
                        out.push_back(static_cast<char>(0xE0 | (cp >> 12)));
                        out.push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
                        out.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
                    } else {
                        out.push_back(static_cast<char>(0xF0 | (cp >> 18)));
                        out.push_back(static_cast<char>(0x80 | ((cp >> 12) & 0x3F)));
                        out.push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
                        out.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
                    }
                    break;
                }
                default: out.push_back(c);
            }
        }
        if (p_ >= end_) throw std::runtime_error("json: unterminated string");
        ++p_;
        return out;
    }
};

inline Value parse(const std::string &text) { return Parser(text.data(), text.size()).parse(); }

}  // namespace json
}  // namespace fe
