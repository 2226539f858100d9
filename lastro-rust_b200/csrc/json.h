// Minimal JSON reader for the two documents the loader parses: a safetensors header and a Hugging Face config.json.
//
// A value is null, a bool, a number, a string, an array or an object.  Numbers keep both readings: a non-negative
// integer literal without fraction or exponent that fits in 64 bits is exact in `u` (safetensors offsets go up to
// 2^64 - 1); every number also has its double `d`.  Parsing never throws: a malformed document yields ok == false
// and a message.  Recursion depth is bounded, so hostile headers cannot exhaust the stack.
#pragma once

#include <cstdint>
#include <cstdlib>
#include <map>
#include <memory>
#include <string>
#include <vector>

namespace lastro_json {

struct Value {
    enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
    bool b = false;
    double d = 0.0;
    bool is_u64 = false;  // an exact non-negative integer literal
    uint64_t u = 0;
    std::string s;
    std::vector<Value> arr;
    std::vector<std::pair<std::string, Value>> obj;  // in document order

    const Value* get(const std::string& key) const {
        if (kind != Object) return nullptr;
        for (const auto& kv : obj)
            if (kv.first == key) return &kv.second;
        return nullptr;
    }
};

class Parser {
  public:
    Parser(const char* p, size_t n) : p_(p), end_(p + n) {}

    bool parse(Value* out, std::string* err) {
        skip();
        if (!value(out, 0)) {
            *err = err_.empty() ? "malformed JSON" : err_;
            return false;
        }
        skip();
        if (p_ != end_) {
            *err = "trailing bytes after the JSON value";
            return false;
        }
        return true;
    }

  private:
    static constexpr int kMaxDepth = 64;
    const char* p_;
    const char* end_;
    std::string err_;

    bool fail(const char* m) {
        if (err_.empty()) err_ = m;
        return false;
    }
    void skip() {
        while (p_ < end_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
    }
    bool lit(const char* w) {
        const char* q = p_;
        for (; *w; ++w, ++q)
            if (q >= end_ || *q != *w) return false;
        p_ = q;
        return true;
    }
    static void put_utf8(std::string& s, uint32_t c) {
        if (c < 0x80) {
            s += (char)c;
        } else if (c < 0x800) {
            s += (char)(0xC0 | (c >> 6));
            s += (char)(0x80 | (c & 0x3F));
        } else if (c < 0x10000) {
            s += (char)(0xE0 | (c >> 12));
            s += (char)(0x80 | ((c >> 6) & 0x3F));
            s += (char)(0x80 | (c & 0x3F));
        } else {
            s += (char)(0xF0 | (c >> 18));
            s += (char)(0x80 | ((c >> 12) & 0x3F));
            s += (char)(0x80 | ((c >> 6) & 0x3F));
            s += (char)(0x80 | (c & 0x3F));
        }
    }
    bool hex4(uint32_t* v) {
        if (end_ - p_ < 4) return fail("short \\u escape");
        uint32_t r = 0;
        for (int i = 0; i < 4; ++i) {
            const char c = *p_++;
            r <<= 4;
            if (c >= '0' && c <= '9') r |= (uint32_t)(c - '0');
            else if (c >= 'a' && c <= 'f') r |= (uint32_t)(c - 'a' + 10);
            else if (c >= 'A' && c <= 'F') r |= (uint32_t)(c - 'A' + 10);
            else return fail("bad \\u escape");
        }
        *v = r;
        return true;
    }
    bool string(std::string* s) {
        if (p_ >= end_ || *p_ != '"') return fail("expected a string");
        ++p_;
        while (p_ < end_ && *p_ != '"') {
            const char c = *p_++;
            if ((unsigned char)c < 0x20) return fail("control character in a string");
            if (c != '\\') {
                *s += c;
                continue;
            }
            if (p_ >= end_) return fail("unterminated escape");
            const char e = *p_++;
            switch (e) {
            case '"': *s += '"'; break;
            case '\\': *s += '\\'; break;
            case '/': *s += '/'; break;
            case 'b': *s += '\b'; break;
            case 'f': *s += '\f'; break;
            case 'n': *s += '\n'; break;
            case 'r': *s += '\r'; break;
            case 't': *s += '\t'; break;
            case 'u': {
                uint32_t c1;
                if (!hex4(&c1)) return false;
                if (c1 >= 0xD800 && c1 < 0xDC00 && end_ - p_ >= 6 && p_[0] == '\\' && p_[1] == 'u') {
                    p_ += 2;
                    uint32_t c2;
                    if (!hex4(&c2)) return false;
                    if (c2 < 0xDC00 || c2 > 0xDFFF) return fail("bad surrogate pair");
                    c1 = 0x10000 + ((c1 - 0xD800) << 10) + (c2 - 0xDC00);
                }
                put_utf8(*s, c1);
                break;
            }
            default: return fail("bad escape");
            }
        }
        if (p_ >= end_) return fail("unterminated string");
        ++p_;
        return true;
    }
    bool number(Value* v) {
        const char* q = p_;
        bool neg = false, frac = false;
        if (q < end_ && *q == '-') {
            neg = true;
            ++q;
        }
        if (q >= end_ || *q < '0' || *q > '9') return fail("bad number");
        uint64_t u = 0;
        bool exact = true;
        for (; q < end_ && *q >= '0' && *q <= '9'; ++q) {
            const uint64_t dgt = (uint64_t)(*q - '0');
            if (u > (UINT64_MAX - dgt) / 10) exact = false;
            else u = u * 10 + dgt;
        }
        if (q < end_ && *q == '.') {
            frac = true;
            ++q;
            if (q >= end_ || *q < '0' || *q > '9') return fail("bad number");
            while (q < end_ && *q >= '0' && *q <= '9') ++q;
        }
        if (q < end_ && (*q == 'e' || *q == 'E')) {
            frac = true;
            ++q;
            if (q < end_ && (*q == '+' || *q == '-')) ++q;
            if (q >= end_ || *q < '0' || *q > '9') return fail("bad number");
            while (q < end_ && *q >= '0' && *q <= '9') ++q;
        }
        const std::string text(p_, q);
        v->kind = Value::Number;
        v->d = std::strtod(text.c_str(), nullptr);
        v->is_u64 = !neg && !frac && exact;
        v->u = v->is_u64 ? u : 0;
        p_ = q;
        return true;
    }
    bool value(Value* v, int depth) {
        if (depth > kMaxDepth) return fail("JSON nested too deeply");
        skip();
        if (p_ >= end_) return fail("unexpected end of JSON");
        const char c = *p_;
        if (c == '{') {
            ++p_;
            v->kind = Value::Object;
            skip();
            if (p_ < end_ && *p_ == '}') {
                ++p_;
                return true;
            }
            while (true) {
                skip();
                std::string key;
                if (!string(&key)) return false;
                skip();
                if (p_ >= end_ || *p_ != ':') return fail("expected ':'");
                ++p_;
                Value item;
                if (!value(&item, depth + 1)) return false;
                v->obj.emplace_back(std::move(key), std::move(item));
                skip();
                if (p_ < end_ && *p_ == ',') {
                    ++p_;
                    continue;
                }
                if (p_ < end_ && *p_ == '}') {
                    ++p_;
                    return true;
                }
                return fail("expected ',' or '}'");
            }
        }
        if (c == '[') {
            ++p_;
            v->kind = Value::Array;
            skip();
            if (p_ < end_ && *p_ == ']') {
                ++p_;
                return true;
            }
            while (true) {
                Value item;
                if (!value(&item, depth + 1)) return false;
                v->arr.push_back(std::move(item));
                skip();
                if (p_ < end_ && *p_ == ',') {
                    ++p_;
                    continue;
                }
                if (p_ < end_ && *p_ == ']') {
                    ++p_;
                    return true;
                }
                return fail("expected ',' or ']'");
            }
        }
        if (c == '"') {
            v->kind = Value::String;
            return string(&v->s);
        }
        if (lit("true")) {
            v->kind = Value::Bool;
            v->b = true;
            return true;
        }
        if (lit("false")) {
            v->kind = Value::Bool;
            v->b = false;
            return true;
        }
        if (lit("null")) {
            v->kind = Value::Null;
            return true;
        }
        return number(v);
    }
};

inline bool parse(const char* p, size_t n, Value* out, std::string* err) { return Parser(p, n).parse(out, err); }

}  // namespace lastro_json
