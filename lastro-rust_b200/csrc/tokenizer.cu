// Text I/O of the decode path: the byte-level BPE tokenizer and the Granite 3.1 chat template, behind the C ABI
// (include/lastro_b200.h, "text" section).  Host code only.
//
// Restates rust/moe-rt/src/tokenizador.rs (Tokenizador, renderiza_chat, formata_data):
//   - a tokenizer.json of exactly the Granite 3.1 configuration is accepted (no normalizer; ByteLevel pre-tokenizer
//     with add_prefix_space false and the GPT-2 regex; BPE without dropout, unk token, byte fallback, subword affixes
//     or ignore_merges; ByteLevel decoder; added tokens that are plain literals); anything else is refused with the
//     field named (tokenizador.rs:221-278), instead of a silently different tokenization;
//   - encoding: added tokens are matched in the raw text, longest first at the leftmost position; the text between
//     them is split by the GPT-2 regex (tokenizador.rs:125-177), each piece mapped to byte-level symbols (a byte
//     whose symbol the vocabulary lacks is dropped, as `tokenizers` does without an unk token) and merged by merge
//     rank, lowest rank first and the leftmost pair on equal ranks (tokenizador.rs:350-403);
//   - decoding: the exact bytes (added tokens as their literal text), and a text form that replaces invalid UTF-8
//     over the whole sequence with U+FFFD per maximal invalid subsequence (tokenizador.rs:451-466);
//   - the chat template rendering for system / user / assistant messages (tokenizador.rs:512-541) and the
//     strftime("%B %d, %Y") date it embeds (tokenizador.rs:544-561).
// The regex classes \p{L}, \p{N} and \s come from unicode_tables.h, generated from the `tokenizers` pre-tokenizer
// itself by gen_unicode_tables.py (Rust's and C's character predicates differ from the regex's classes).
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <mutex>
#include <queue>
#include <sstream>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/lastro_b200.h"
#include "json.h"
#include "unicode_tables.h"

namespace lastro_text {
namespace {

template <size_t N>
bool in_ranges(const uint32_t (&t)[N][2], uint32_t cp) {
    size_t lo = 0, hi = N;
    while (lo < hi) {
        const size_t mid = (lo + hi) / 2;
        if (cp < t[mid][0]) hi = mid;
        else if (cp > t[mid][1]) lo = mid + 1;
        else return true;
    }
    return false;
}

enum CharClass { kSpaceClass = 0, kLetterClass = 1, kNumberClass = 2, kOtherClass = 3 };

CharClass classify(uint32_t cp) {
    if (in_ranges(kSpace, cp)) return kSpaceClass;
    if (in_ranges(kLetter, cp)) return kLetterClass;
    if (in_ranges(kNumber, cp)) return kNumberClass;
    return kOtherClass;
}

// UTF-8 -> code points with their byte offsets (offs has one more entry: the end); false on malformed input
bool decode_utf8(const unsigned char* s, size_t n, std::vector<uint32_t>* cps, std::vector<size_t>* offs) {
    size_t i = 0;
    while (i < n) {
        const unsigned char b = s[i];
        uint32_t cp;
        int len;
        if (b < 0x80) {
            cp = b;
            len = 1;
        } else if (b >= 0xC2 && b <= 0xDF) {
            cp = b & 0x1F;
            len = 2;
        } else if (b >= 0xE0 && b <= 0xEF) {
            cp = b & 0x0F;
            len = 3;
        } else if (b >= 0xF0 && b <= 0xF4) {
            cp = b & 0x07;
            len = 4;
        } else {
            return false;
        }
        if (i + len > n) return false;
        for (int k = 1; k < len; ++k) {
            const unsigned char c = s[i + k];
            if ((c & 0xC0) != 0x80) return false;
            cp = (cp << 6) | (c & 0x3F);
        }
        // overlong forms, surrogates and values past U+10FFFF are not UTF-8
        if ((len == 3 && cp < 0x800) || (len == 4 && (cp < 0x10000 || cp > 0x10FFFF)) || (cp >= 0xD800 && cp <= 0xDFFF))
            return false;
        cps->push_back(cp);
        offs->push_back(i);
        i += len;
    }
    offs->push_back(n);
    return true;
}

// bytes -> text with U+FFFD for each maximal subpart of an ill-formed sequence (the Unicode Standard's recommended
// practice, which Rust's String::from_utf8_lossy follows)
std::string utf8_lossy(const std::string& in) {
    static const char kRepl[] = "\xEF\xBF\xBD";
    std::string out;
    out.reserve(in.size());
    const unsigned char* s = reinterpret_cast<const unsigned char*>(in.data());
    const size_t n = in.size();
    size_t i = 0;
    while (i < n) {
        const unsigned char b = s[i];
        if (b < 0x80) {
            out.push_back((char)b);
            ++i;
            continue;
        }
        int len = 0;
        unsigned char lo = 0x80, hi = 0xBF;  // the valid range of the second byte
        if (b >= 0xC2 && b <= 0xDF) len = 2;
        else if (b == 0xE0) len = 3, lo = 0xA0;
        else if (b >= 0xE1 && b <= 0xEC) len = 3;
        else if (b == 0xED) len = 3, hi = 0x9F;
        else if (b >= 0xEE && b <= 0xEF) len = 3;
        else if (b == 0xF0) len = 4, lo = 0x90;
        else if (b >= 0xF1 && b <= 0xF3) len = 4;
        else if (b == 0xF4) len = 4, hi = 0x8F;
        if (len == 0) {
            out += kRepl;
            ++i;
            continue;
        }
        size_t k = 1;
        for (; k < (size_t)len && i + k < n; ++k) {
            const unsigned char c = s[i + k];
            const bool ok = k == 1 ? (c >= lo && c <= hi) : (c >= 0x80 && c <= 0xBF);
            if (!ok) break;
        }
        if (k == (size_t)len) {
            out.append(in, i, len);
        } else {
            out += kRepl;  // the valid prefix [i, i + k) is one maximal subpart
        }
        i += k;
    }
    return out;
}

void append_utf8(std::string* s, uint32_t cp) {
    if (cp < 0x80) {
        s->push_back((char)cp);
    } else if (cp < 0x800) {
        s->push_back((char)(0xC0 | (cp >> 6)));
        s->push_back((char)(0x80 | (cp & 0x3F)));
    } else if (cp < 0x10000) {
        s->push_back((char)(0xE0 | (cp >> 12)));
        s->push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
        s->push_back((char)(0x80 | (cp & 0x3F)));
    } else {
        s->push_back((char)(0xF0 | (cp >> 18)));
        s->push_back((char)(0x80 | ((cp >> 12) & 0x3F)));
        s->push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
        s->push_back((char)(0x80 | (cp & 0x3F)));
    }
}

// GPT-2's byte-level alphabet: printable bytes stand for themselves, the others for U+0100 onwards in byte order
void byte_alphabet(uint32_t (&cp_of_byte)[256]) {
    uint32_t next = 256;
    for (uint32_t b = 0; b < 256; ++b) {
        const bool printable = (b >= 33 && b <= 126) || (b >= 161 && b <= 172) || (b >= 174 && b <= 255);
        cp_of_byte[b] = printable ? b : next++;
    }
}

}  // namespace

// The GPT-2 pre-tokenizer regex 's|'t|'re|'ve|'m|'ll|'d| ?\p{L}+| ?\p{N}+| ?[^\s\p{L}\p{N}]+|\s+(?!\S)|\s+ applied
// left to right, the first alternative that matches winning; pieces as [start, end) byte ranges that tile the text.
void pretokenize(const std::vector<uint32_t>& cps, const std::vector<size_t>& offs, size_t base,
                 std::vector<std::pair<size_t, size_t>>* pieces) {
    const size_t n = cps.size();
    size_t i = 0;
    while (i < n) {
        const uint32_t c = cps[i];
        if (c == '\'' && i + 1 < n) {
            const uint32_t a = cps[i + 1], b = i + 2 < n ? cps[i + 2] : 0;
            size_t len = 0;
            if (a == 's' || a == 't' || a == 'm' || a == 'd') len = 2;
            else if ((a == 'r' && b == 'e') || (a == 'v' && b == 'e') || (a == 'l' && b == 'l')) len = 3;
            if (len) {
                pieces->push_back({base + offs[i], base + offs[i + len]});
                i += len;
                continue;
            }
        }
        // an optional U+0020 in front of a run of one class (letters, numbers, or neither of those nor space)
        const size_t j = (c == ' ' && i + 1 < n) ? i + 1 : i;
        const CharClass k = classify(cps[j]);
        if (k != kSpaceClass) {
            size_t e = j + 1;
            while (e < n && classify(cps[e]) == k) ++e;
            pieces->push_back({base + offs[i], base + offs[e]});
            i = e;
            continue;
        }
        // whitespace: \s+(?!\S) leaves the last one of a run that a non-space follows, \s+ takes the rest
        size_t e = i;
        while (e < n && classify(cps[e]) == kSpaceClass) ++e;
        const size_t stop = (e < n && e - i > 1) ? e - 1 : e;
        pieces->push_back({base + offs[i], base + offs[stop]});
        i = stop;
    }
}

struct Tokenizer {
    std::vector<std::string> bytes_of_id;  // what each id decodes to (empty + !has_bytes: no such id)
    std::vector<char> has_bytes;
    int32_t id_of_byte[256];               // -1: the vocabulary lacks that byte's symbol
    std::unordered_map<uint64_t, std::pair<uint32_t, uint32_t>> merges;  // (left, right) -> (rank, result)
    std::vector<std::pair<std::string, int32_t>> added;                  // literal, id
    mutable std::mutex cache_mu;
    mutable std::unordered_map<std::string, std::vector<int32_t>> cache;
    static constexpr size_t kCacheMax = 50000;

    static uint64_t key(uint32_t a, uint32_t b) { return ((uint64_t)a << 32) | b; }

    // merge-rank BPE over one piece's bytes.  The heap holds (rank, position, result) for adjacent pairs; an entry
    // is stale when its left symbol was merged away or when the pair now at its position merges into another token
    // (the check `tokenizers` makes, by result id)
    void bpe(const unsigned char* p, size_t n, std::vector<int32_t>* out) const {
        std::vector<int32_t> sym;
        sym.reserve(n);
        for (size_t i = 0; i < n; ++i)
            if (id_of_byte[p[i]] >= 0) sym.push_back(id_of_byte[p[i]]);
        const int m = (int)sym.size();
        if (m == 0) return;
        std::vector<int> nxt(m), prv(m);
        std::vector<char> live(m, 1);
        for (int i = 0; i < m; ++i) {
            nxt[i] = i + 1 < m ? i + 1 : -1;
            prv[i] = i - 1;
        }
        using Item = std::pair<uint64_t, uint32_t>;  // ((rank << 32) | pos, result id)
        std::priority_queue<Item, std::vector<Item>, std::greater<Item>> heap;
        auto push = [&](int pos) {
            const int q = nxt[pos];
            if (q < 0) return;
            auto it = merges.find(key((uint32_t)sym[pos], (uint32_t)sym[q]));
            if (it != merges.end()) heap.push({((uint64_t)it->second.first << 32) | (uint32_t)pos, it->second.second});
        };
        for (int i = 0; i + 1 < m; ++i) push(i);
        while (!heap.empty()) {
            const Item top = heap.top();
            heap.pop();
            const int pos = (int)(top.first & 0xFFFFFFFFu);
            if (!live[pos]) continue;
            const int q = nxt[pos];
            if (q < 0) continue;
            auto it = merges.find(key((uint32_t)sym[pos], (uint32_t)sym[q]));
            if (it == merges.end() || it->second.second != top.second) continue;
            sym[pos] = (int32_t)top.second;
            live[q] = 0;
            nxt[pos] = nxt[q];
            if (nxt[q] >= 0) prv[nxt[q]] = pos;
            if (prv[pos] >= 0) push(prv[pos]);
            push(pos);
        }
        for (int i = 0; i >= 0; i = nxt[i]) out->push_back(sym[i]);
    }

    void encode_piece(const char* p, size_t n, std::vector<int32_t>* out) const {
        const std::string k(p, n);
        {
            std::lock_guard<std::mutex> g(cache_mu);
            auto it = cache.find(k);
            if (it != cache.end()) {
                out->insert(out->end(), it->second.begin(), it->second.end());
                return;
            }
        }
        std::vector<int32_t> ids;
        bpe(reinterpret_cast<const unsigned char*>(p), n, &ids);
        out->insert(out->end(), ids.begin(), ids.end());
        std::lock_guard<std::mutex> g(cache_mu);
        if (cache.size() < kCacheMax) cache.emplace(k, std::move(ids));
    }

    void encode_span(const char* text, size_t a, size_t b, std::vector<int32_t>* out) const {
        if (a >= b) return;
        std::vector<uint32_t> cps;
        std::vector<size_t> offs;
        decode_utf8(reinterpret_cast<const unsigned char*>(text + a), b - a, &cps, &offs);
        std::vector<std::pair<size_t, size_t>> pieces;
        pretokenize(cps, offs, a, &pieces);
        for (const auto& pc : pieces) encode_piece(text + pc.first, pc.second - pc.first, out);
    }

    // text must be UTF-8 (checked by the caller)
    void encode(const char* text, size_t n, std::vector<int32_t>* out) const {
        size_t rest = 0, i = 0;
        while (i < n) {
            const unsigned char b = (unsigned char)text[i];
            int best = -1;
            if ((b & 0xC0) != 0x80) {  // a character boundary
                size_t best_len = 0;
                for (size_t t = 0; t < added.size(); ++t) {
                    const std::string& lit = added[t].first;
                    if (lit.size() > best_len && lit.size() <= n - i && std::memcmp(text + i, lit.data(), lit.size()) == 0) {
                        best = (int)t;
                        best_len = lit.size();
                    }
                }
            }
            if (best >= 0) {
                encode_span(text, rest, i, out);
                out->push_back(added[best].second);
                i += added[best].first.size();
                rest = i;
            } else {
                ++i;
            }
        }
        encode_span(text, rest, n, out);
    }
};

namespace {

bool is_null_or_missing(const lastro_json::Value* v) { return !v || v->kind == lastro_json::Value::Null; }
bool is_str(const lastro_json::Value* v, const char* s) {
    return v && v->kind == lastro_json::Value::String && v->s == s;
}
bool is_bool(const lastro_json::Value* v, bool b) { return v && v->kind == lastro_json::Value::Bool && v->b == b; }
bool empty_or_null_str(const lastro_json::Value* v) {
    return is_null_or_missing(v) || (v->kind == lastro_json::Value::String && v->s.empty());
}

// tokenizador.rs:221-345: parse and validate; returns a LASTRO_* status and a message
int build(const char* json, size_t len, Tokenizer* t, std::string* msg) {
    using lastro_json::Value;
    Value root;
    lastro_json::Parser parser(json, len);
    if (!parser.parse(&root, msg)) return LASTRO_E_ARG;
    if (root.kind != Value::Object) {
        *msg = "tokenizer.json is not an object";
        return LASTRO_E_ARG;
    }
    auto refuse = [&](const std::string& m) {
        *msg = "tokenizer.json outside the supported configuration: " + m;
        return LASTRO_E_UNSUPPORTED;
    };
    if (!is_null_or_missing(root.get("normalizer"))) return refuse("normalizer is not null");
    const Value* pre = root.get("pre_tokenizer");
    if (!pre || !is_str(pre->get("type"), "ByteLevel") || !is_bool(pre->get("add_prefix_space"), false) ||
        !is_bool(pre->get("use_regex"), true))
        return refuse("pre_tokenizer is not ByteLevel{add_prefix_space: false, use_regex: true}");
    const Value* dec = root.get("decoder");
    if (!dec || !is_str(dec->get("type"), "ByteLevel")) return refuse("decoder is not ByteLevel");
    const Value* model = root.get("model");
    if (!model || !is_str(model->get("type"), "BPE")) return refuse("model is not BPE");
    if (!is_null_or_missing(model->get("dropout"))) return refuse("model.dropout");
    if (!is_null_or_missing(model->get("unk_token"))) return refuse("model.unk_token");
    if (!empty_or_null_str(model->get("continuing_subword_prefix"))) return refuse("model.continuing_subword_prefix");
    if (!empty_or_null_str(model->get("end_of_word_suffix"))) return refuse("model.end_of_word_suffix");
    if (is_bool(model->get("byte_fallback"), true)) return refuse("model.byte_fallback");
    if (is_bool(model->get("ignore_merges"), true)) return refuse("model.ignore_merges");
    const Value* vocab = model->get("vocab");
    if (!vocab || vocab->kind != Value::Object) return refuse("model.vocab missing");

    uint64_t max_id = 0;
    for (const auto& kv : vocab->obj) {
        if (kv.second.kind != Value::Number || !kv.second.is_u64 || kv.second.u > 0xFFFFFFFFull)
            return refuse("bad id for a vocabulary entry");
        max_id = std::max(max_id, kv.second.u);
    }
    std::vector<std::pair<std::string, int32_t>> added;
    if (const Value* at = root.get("added_tokens")) {
        if (at->kind != Value::Array) return refuse("added_tokens is not an array");
        for (const Value& a : at->arr) {
            const Value* content = a.get("content");
            const Value* id = a.get("id");
            if (!content || content->kind != Value::String || !id || id->kind != Value::Number || !id->is_u64)
                return refuse("an added token without content or id");
            if (!is_bool(a.get("lstrip"), false) || !is_bool(a.get("rstrip"), false) ||
                !is_bool(a.get("single_word"), false) || !is_bool(a.get("normalized"), false) || content->s.empty())
                return refuse("added token " + content->s + " with lstrip/rstrip/single_word/normalized");
            if (id->u > 0x7FFFFFFFull) return refuse("added token id too large");
            max_id = std::max(max_id, id->u);
            added.push_back({content->s, (int32_t)id->u});
        }
    }
    // dense tables indexed by id: refuse sparse ids before allocating them
    const uint64_t entries = vocab->obj.size() + added.size();
    if (max_id + 1 > 2 * entries + 1024 || max_id > 0x7FFFFFFEull) return refuse("sparse ids");
    const size_t size = (size_t)max_id + 1;

    uint32_t cp_of_byte[256];
    byte_alphabet(cp_of_byte);
    std::unordered_map<uint32_t, int> byte_of_cp;
    for (int b = 0; b < 256; ++b) byte_of_cp[cp_of_byte[b]] = b;

    t->bytes_of_id.assign(size, std::string());
    t->has_bytes.assign(size, 0);
    std::unordered_map<std::string, int32_t> id_of_token;
    id_of_token.reserve(vocab->obj.size() * 2);
    for (const auto& kv : vocab->obj) {
        const int32_t id = (int32_t)kv.second.u;
        id_of_token[kv.first] = id;
        std::vector<uint32_t> cps;
        std::vector<size_t> offs;
        std::string bytes;
        bool ok = decode_utf8(reinterpret_cast<const unsigned char*>(kv.first.data()), kv.first.size(), &cps, &offs);
        for (uint32_t cp : cps) {
            auto it = byte_of_cp.find(cp);
            if (it == byte_of_cp.end()) ok = false;
            else bytes.push_back((char)it->second);
        }
        // a token with a symbol outside the byte-level alphabet has no byte form
        t->bytes_of_id[id] = ok ? bytes : std::string();
        t->has_bytes[id] = ok ? 1 : 0;
    }
    for (const auto& a : added) {
        t->bytes_of_id[a.second] = a.first;
        t->has_bytes[a.second] = 1;
    }
    for (int b = 0; b < 256; ++b) {
        std::string sym;
        append_utf8(&sym, cp_of_byte[b]);
        auto it = id_of_token.find(sym);
        t->id_of_byte[b] = it == id_of_token.end() ? -1 : it->second;
    }
    const Value* merges = model->get("merges");
    if (!merges || merges->kind != Value::Array) return refuse("model.merges missing");
    t->merges.reserve(merges->arr.size() * 2);
    for (size_t rank = 0; rank < merges->arr.size(); ++rank) {
        const Value& mg = merges->arr[rank];
        std::string a, b;
        if (mg.kind == Value::String) {
            const size_t sp = mg.s.find(' ');
            if (sp == std::string::npos) return refuse("merge " + std::to_string(rank) + " without a space");
            a = mg.s.substr(0, sp);
            b = mg.s.substr(sp + 1);
        } else if (mg.kind == Value::Array && mg.arr.size() == 2 && mg.arr[0].kind == Value::String &&
                   mg.arr[1].kind == Value::String) {
            a = mg.arr[0].s;
            b = mg.arr[1].s;
        } else {
            return refuse("merge " + std::to_string(rank) + " malformed");
        }
        auto ia = id_of_token.find(a), ib = id_of_token.find(b), ij = id_of_token.find(a + b);
        if (ia == id_of_token.end() || ib == id_of_token.end())
            return refuse("merge " + std::to_string(rank) + " uses a token outside the vocabulary");
        if (ij == id_of_token.end()) return refuse("merge " + std::to_string(rank) + " makes a token outside the vocabulary");
        // a repeated pair keeps the last rank, as `tokenizers` builds its map
        t->merges[Tokenizer::key((uint32_t)ia->second, (uint32_t)ib->second)] = {(uint32_t)rank, (uint32_t)ij->second};
    }
    t->added = std::move(added);
    return LASTRO_OK;
}

int put_err(char* err, int32_t errlen, const std::string& m) {
    if (err && errlen > 0) {
        const size_t n = std::min((size_t)errlen - 1, m.size());
        std::memcpy(err, m.data(), n);
        err[n] = '\0';
    }
    return 0;
}

const char* kStartRole = "<|start_of_role|>";
const char* kEndRole = "<|end_of_role|>";
const char* kEndText = "<|end_of_text|>";

int copy_out(const std::string& s, char* out, size_t cap, size_t* n_out) {
    if (n_out) *n_out = s.size();
    if (!out || cap < s.size()) return LASTRO_E_ARG;
    if (!s.empty()) std::memcpy(out, s.data(), s.size());
    return LASTRO_OK;
}

}  // namespace
}  // namespace lastro_text

struct lastro_tokenizer {
    lastro_text::Tokenizer t;
};

extern "C" int lastro_tokenizer_from_json(const char* json, size_t len, lastro_tokenizer** out, char* err, int32_t errlen) {
    if (!out || (!json && len)) return LASTRO_E_ARG;
    *out = nullptr;
    lastro_tokenizer* tk = new (std::nothrow) lastro_tokenizer;
    if (!tk) return LASTRO_E_NOMEM;
    std::string msg;
    int rc;
    try {
        rc = lastro_text::build(json, len, &tk->t, &msg);
    } catch (const std::bad_alloc&) {
        rc = LASTRO_E_NOMEM;
        msg = "out of host memory";
    }
    if (rc != LASTRO_OK) {
        lastro_text::put_err(err, errlen, msg);
        delete tk;
        return rc;
    }
    *out = tk;
    return LASTRO_OK;
}

extern "C" int lastro_tokenizer_load(const char* path, lastro_tokenizer** out, char* err, int32_t errlen) {
    if (!path || !out) return LASTRO_E_ARG;
    std::ifstream f(path, std::ios::binary);
    if (!f) {
        lastro_text::put_err(err, errlen, std::string("cannot read ") + path);
        return LASTRO_E_IO;
    }
    std::stringstream ss;
    ss << f.rdbuf();
    const std::string s = ss.str();
    return lastro_tokenizer_from_json(s.data(), s.size(), out, err, errlen);
}

extern "C" void lastro_tokenizer_destroy(lastro_tokenizer* tk) { delete tk; }

extern "C" int32_t lastro_tokenizer_vocab_size(const lastro_tokenizer* tk) {
    return tk ? (int32_t)tk->t.bytes_of_id.size() : 0;
}

extern "C" int lastro_tokenizer_encode(const lastro_tokenizer* tk, const char* text, size_t len, int32_t* ids, int32_t cap,
                                       int32_t* n_ids) {
    if (!tk || (!text && len) || !n_ids) return LASTRO_E_ARG;
    std::vector<uint32_t> cps;
    std::vector<size_t> offs;
    if (!lastro_text::decode_utf8(reinterpret_cast<const unsigned char*>(text), len, &cps, &offs)) return LASTRO_E_ARG;
    std::vector<int32_t> out;
    tk->t.encode(text, len, &out);
    *n_ids = (int32_t)out.size();
    if (!ids || cap < (int32_t)out.size()) return LASTRO_E_ARG;
    std::copy(out.begin(), out.end(), ids);
    return LASTRO_OK;
}

extern "C" int lastro_tokenizer_pretokenize(const char* text, size_t len, int32_t* ends, int32_t cap, int32_t* n_pieces) {
    if ((!text && len) || !n_pieces) return LASTRO_E_ARG;
    std::vector<uint32_t> cps;
    std::vector<size_t> offs;
    if (!lastro_text::decode_utf8(reinterpret_cast<const unsigned char*>(text), len, &cps, &offs)) return LASTRO_E_ARG;
    std::vector<std::pair<size_t, size_t>> pieces;
    lastro_text::pretokenize(cps, offs, 0, &pieces);
    *n_pieces = (int32_t)pieces.size();
    if (!ends || cap < (int32_t)pieces.size()) return LASTRO_E_ARG;
    for (size_t i = 0; i < pieces.size(); ++i) ends[i] = (int32_t)pieces[i].second;
    return LASTRO_OK;
}

static int decode_bytes(const lastro_tokenizer* tk, const int32_t* ids, int32_t n, std::string* s) {
    for (int32_t i = 0; i < n; ++i) {
        const int32_t id = ids[i];
        if (id < 0 || (size_t)id >= tk->t.bytes_of_id.size() || !tk->t.has_bytes[id]) return LASTRO_E_ARG;
        *s += tk->t.bytes_of_id[id];
    }
    return LASTRO_OK;
}

extern "C" int lastro_tokenizer_decode_bytes(const lastro_tokenizer* tk, const int32_t* ids, int32_t n, char* out,
                                             size_t cap, size_t* n_out) {
    if (!tk || (!ids && n) || n < 0) return LASTRO_E_ARG;
    std::string s;
    if (int rc = decode_bytes(tk, ids, n, &s)) return rc;
    return lastro_text::copy_out(s, out, cap, n_out);
}

extern "C" int lastro_tokenizer_decode(const lastro_tokenizer* tk, const int32_t* ids, int32_t n, char* out, size_t cap,
                                       size_t* n_out) {
    if (!tk || (!ids && n) || n < 0) return LASTRO_E_ARG;
    std::string s;
    if (int rc = decode_bytes(tk, ids, n, &s)) return rc;
    return lastro_text::copy_out(lastro_text::utf8_lossy(s), out, cap, n_out);
}

extern "C" int lastro_chat_render(const int32_t* roles, const char* const* contents, const size_t* lens, int32_t n,
                                  int32_t add_generation_prompt, const char* date, char* out, size_t cap, size_t* n_out) {
    using namespace lastro_text;
    if (n < 1 || !roles || !contents || !lens || !date) return LASTRO_E_ARG;  // the template reads messages[0]
    static const char* kRole[3] = {"system", "user", "assistant"};
    for (int32_t i = 0; i < n; ++i)
        if (roles[i] < LASTRO_ROLE_SYSTEM || roles[i] > LASTRO_ROLE_ASSISTANT || (!contents[i] && lens[i])) return LASTRO_E_ARG;
    std::string s;
    int32_t first = 0;
    s += kStartRole;
    s += "system";
    s += kEndRole;
    if (roles[0] == LASTRO_ROLE_SYSTEM) {
        s.append(contents[0], lens[0]);
        first = 1;
    } else {
        s += "Knowledge Cutoff Date: April 2024.\nToday's Date: ";
        s += date;
        s += ".\nYou are Granite, developed by IBM. You are a helpful AI assistant.";
    }
    s += kEndText;
    s += "\n";
    for (int32_t i = first; i < n; ++i) {
        s += kStartRole;
        s += kRole[roles[i]];
        s += kEndRole;
        s.append(contents[i], lens[i]);
        s += kEndText;
        s += "\n";
        if (i == n - 1 && add_generation_prompt) {
            s += kStartRole;
            s += "assistant";
            s += kEndRole;
        }
    }
    return copy_out(s, out, cap, n_out);
}

extern "C" int lastro_format_date(int32_t year, int32_t month, int32_t day, char* out, int32_t cap) {
    static const char* kMonth[12] = {"January", "February", "March",     "April",   "May",      "June",
                                     "July",    "August",   "September", "October", "November", "December"};
    if (month < 1 || month > 12 || year < 1 || year > 9999) return LASTRO_E_ARG;
    const bool leap = (year % 4 == 0 && year % 100 != 0) || year % 400 == 0;
    static const int kDays[12] = {31, 28, 31, 30, 31, 30, 31, 31, 30, 31, 30, 31};
    const int days = month == 2 && leap ? 29 : kDays[month - 1];
    if (day < 1 || day > days || !out) return LASTRO_E_ARG;
    char buf[48];
    const int n = std::snprintf(buf, sizeof buf, "%s %02d, %04d", kMonth[month - 1], day, year);
    if (n < 0 || n + 1 > cap) return LASTRO_E_ARG;
    std::memcpy(out, buf, (size_t)n + 1);
    return LASTRO_OK;
}
