// safetensors checkpoints and Granite config.json: the on-disk formats the C ABI accepts.
//
// Restates the reference's loader (rust/moe-rt/src/weights.rs:52-122 Checkpoint::open / Checkpoint::bf16, model.rs:34-61
// Config::from_json, model.rs:99-132 HostModel::load with block.rs:31-53 HostLayer::load) on the host, in C++: every
// *.safetensors file of a directory is indexed (8-byte little-endian header length, at most 100 MiB, then a JSON object
// name -> {dtype, shape, data_offsets}); only the index stays in memory and each tensor is read from disk when it is
// asked for.  Malformed headers are refused with a message, never a crash: missing or non-numeric fields, data_offsets
// that are not two numbers, offsets that overflow or point past the end of the file, and (on read) a wrong dtype or a
// byte count that does not match the shape, overflow included.  Host code only: nothing here needs a GPU except
// lastro_model_load_checkpoint, which hands each tensor to lastro_model_load_tensor.
#include <dirent.h>
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "../../include/lastro_b200.h"
#include "capi_internal.h"
#include "json.h"

namespace {

struct Entry {
    int file = 0;
    std::string dtype;
    std::vector<uint64_t> shape;
    uint64_t start = 0, end = 0;
};

int put_err(char* err, int32_t len, int code, const char* fmt, ...) {
    if (err && len > 0) {
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(err, (size_t)len, fmt, ap);
        va_end(ap);
    }
    return code;
}

bool read_at(int fd, void* dst, uint64_t n, uint64_t off) {
    unsigned char* p = static_cast<unsigned char*>(dst);
    while (n > 0) {
        const ssize_t r = pread(fd, p, n > (1u << 30) ? (1u << 30) : (size_t)n, (off_t)off);
        if (r <= 0) return false;
        p += r;
        n -= (uint64_t)r;
        off += (uint64_t)r;
    }
    return true;
}

std::string shape_text(const std::vector<uint64_t>& s) {
    std::string t = "[";
    for (size_t i = 0; i < s.size(); ++i) t += (i ? ", " : "") + std::to_string(s[i]);
    return t + "]";
}

}  // namespace

struct lastro_checkpoint {
    std::string dir;
    std::vector<std::string> paths;
    std::vector<int> fds;
    std::map<std::string, Entry> index;
    ~lastro_checkpoint() {
        for (int fd : fds)
            if (fd >= 0) close(fd);
    }
};

namespace {

// weights.rs:52-106: the index of one file (appended to ck), or a Format / I/O error
int index_file(lastro_checkpoint* ck, const std::string& path, char* err, int32_t len) {
    const int fd = open(path.c_str(), O_RDONLY | O_CLOEXEC);
    if (fd < 0) return put_err(err, len, LASTRO_E_IO, "I/O: cannot open %s", path.c_str());
    ck->fds.push_back(fd);
    ck->paths.push_back(path);
    const int fi = (int)ck->fds.size() - 1;
    struct stat st;
    if (fstat(fd, &st) != 0) return put_err(err, len, LASTRO_E_IO, "I/O: cannot stat %s", path.c_str());
    const uint64_t size = (uint64_t)st.st_size;
    unsigned char lb[8];
    if (!read_at(fd, lb, 8, 0)) return put_err(err, len, LASTRO_E_IO, "I/O: %s is shorter than 8 bytes", path.c_str());
    uint64_t n = 0;
    for (int i = 7; i >= 0; --i) n = (n << 8) | lb[i];
    if (n > (100ull << 20))
        return put_err(err, len, LASTRO_E_ARG, "safetensors: header of %llu bytes in %s", (unsigned long long)n,
                       path.c_str());
    if (8 + n > size) return put_err(err, len, LASTRO_E_ARG, "safetensors: header past the end of %s", path.c_str());
    std::vector<char> head(n);
    if (n && !read_at(fd, head.data(), n, 8)) return put_err(err, len, LASTRO_E_IO, "I/O: reading %s", path.c_str());
    lastro_json::Value j;
    std::string jerr;
    if (!lastro_json::parse(head.data(), head.size(), &j, &jerr))
        return put_err(err, len, LASTRO_E_ARG, "safetensors: %s in %s", jerr.c_str(), path.c_str());
    if (j.kind != lastro_json::Value::Object)
        return put_err(err, len, LASTRO_E_ARG, "safetensors: header is not an object");
    for (const auto& kv : j.obj) {
        const std::string& name = kv.first;
        if (name == "__metadata__") continue;
        const lastro_json::Value& v = kv.second;
        const lastro_json::Value* dt = v.get("dtype");
        if (!dt || dt->kind != lastro_json::Value::String)
            return put_err(err, len, LASTRO_E_ARG, "safetensors: %s: no dtype", name.c_str());
        const lastro_json::Value* sh = v.get("shape");
        if (!sh || sh->kind != lastro_json::Value::Array)
            return put_err(err, len, LASTRO_E_ARG, "safetensors: %s: no shape", name.c_str());
        Entry e;
        e.file = fi;
        e.dtype = dt->s;
        for (const auto& d : sh->arr) {
            if (d.kind != lastro_json::Value::Number || !d.is_u64)
                return put_err(err, len, LASTRO_E_ARG, "safetensors: %s: invalid shape", name.c_str());
            e.shape.push_back(d.u);
        }
        const lastro_json::Value* off = v.get("data_offsets");
        if (!off || off->kind != lastro_json::Value::Array)
            return put_err(err, len, LASTRO_E_ARG, "safetensors: %s: no data_offsets", name.c_str());
        if (off->arr.size() != 2)
            return put_err(err, len, LASTRO_E_ARG, "safetensors: %s: data_offsets with %zu values (expected 2)",
                           name.c_str(), off->arr.size());
        const lastro_json::Value &s0 = off->arr[0], &s1 = off->arr[1];
        if (s0.kind != lastro_json::Value::Number || !s0.is_u64 || s1.kind != lastro_json::Value::Number || !s1.is_u64)
            return put_err(err, len, LASTRO_E_ARG, "safetensors: %s: data_offsets not numeric", name.c_str());
        const uint64_t base = 8 + n;
        if (s0.u > UINT64_MAX - base || s1.u > UINT64_MAX - base)
            return put_err(err, len, LASTRO_E_ARG, "safetensors: %s: offsets outside the file", name.c_str());
        e.start = base + s0.u;
        e.end = base + s1.u;
        if (s0.u > s1.u || e.end > size)
            return put_err(err, len, LASTRO_E_ARG, "safetensors: %s: offsets outside the file", name.c_str());
        ck->index[name] = e;
    }
    return LASTRO_OK;
}

// bytes of a tensor of `shape` with `elem` bytes per element, or false on overflow
bool shape_bytes(const std::vector<uint64_t>& shape, uint64_t elem, uint64_t* out) {
    uint64_t b = elem;
    for (uint64_t d : shape) {
        if (d != 0 && b > UINT64_MAX / d) return false;
        b *= d;
    }
    *out = b;
    return true;
}

// weights.rs:108-122 Checkpoint::bf16, generalised to the one dtype the caller expects
int read_tensor(const lastro_checkpoint* ck, const char* name, const char* dtype, uint64_t elem, void* dst,
                uint64_t capacity_bytes, char* err, int32_t len, const Entry** entry_out = nullptr) {
    auto it = ck->index.find(name);
    if (it == ck->index.end()) return put_err(err, len, LASTRO_E_ARG, "safetensors: tensor absent: %s", name);
    const Entry& e = it->second;
    if (entry_out) *entry_out = &e;
    if (e.dtype != dtype)
        return put_err(err, len, LASTRO_E_ARG, "safetensors: %s: dtype %s (expected %s)", name, e.dtype.c_str(), dtype);
    uint64_t bytes = 0;
    if (!shape_bytes(e.shape, elem, &bytes) || bytes != e.end - e.start)
        return put_err(err, len, LASTRO_E_ARG, "safetensors: %s: size does not match the shape", name);
    if (!dst) return LASTRO_OK;
    if (bytes > capacity_bytes)
        return put_err(err, len, LASTRO_E_ARG, "%s: %llu bytes do not fit the %llu-byte buffer", name,
                       (unsigned long long)bytes, (unsigned long long)capacity_bytes);
    if (!read_at(ck->fds[e.file], dst, bytes, e.start))
        return put_err(err, len, LASTRO_E_IO, "I/O: reading %s from %s", name, ck->paths[e.file].c_str());
    return LASTRO_OK;
}

bool json_u32(const lastro_json::Value& v, const char* key, int32_t* out) {
    const lastro_json::Value* x = v.get(key);
    if (!x || x->kind != lastro_json::Value::Number || !x->is_u64 || x->u > 0x7fffffffull) return false;
    *out = (int32_t)x->u;
    return true;
}

bool json_f32(const lastro_json::Value& v, const char* key, float* out) {
    const lastro_json::Value* x = v.get(key);
    if (!x || x->kind != lastro_json::Value::Number) return false;
    *out = (float)x->d;
    return true;
}

}  // namespace

extern "C" int lastro_checkpoint_open(const char* dir, lastro_checkpoint** out, char* err, int32_t err_len) {
    if (!dir || !out) return put_err(err, err_len, LASTRO_E_ARG, "null argument");
    *out = nullptr;
    DIR* d = opendir(dir);
    if (!d) return put_err(err, err_len, LASTRO_E_IO, "I/O: cannot read the directory %s", dir);
    std::vector<std::string> paths;
    while (struct dirent* ent = readdir(d)) {
        const std::string n = ent->d_name;
        if (n.size() > 12 && n.compare(n.size() - 12, 12, ".safetensors") == 0) paths.push_back(std::string(dir) + "/" + n);
    }
    closedir(d);
    std::sort(paths.begin(), paths.end());
    if (paths.empty()) return put_err(err, err_len, LASTRO_E_ARG, "safetensors: no *.safetensors in %s", dir);
    lastro_checkpoint* ck = new lastro_checkpoint;
    ck->dir = dir;
    for (const std::string& p : paths) {
        const int rc = index_file(ck, p, err, err_len);
        if (rc) {
            delete ck;
            return rc;
        }
    }
    *out = ck;
    return LASTRO_OK;
}

extern "C" void lastro_checkpoint_close(lastro_checkpoint* ck) { delete ck; }

extern "C" int lastro_checkpoint_count(const lastro_checkpoint* ck) { return ck ? (int)ck->index.size() : 0; }

extern "C" int lastro_checkpoint_tensor(const lastro_checkpoint* ck, const char* name, char* dtype, int32_t dtype_len,
                                        int64_t* shape, int32_t max_ndim, int32_t* ndim) {
    if (!ck || !name || !ndim) return LASTRO_E_ARG;
    auto it = ck->index.find(name);
    if (it == ck->index.end()) return LASTRO_E_ARG;
    const Entry& e = it->second;
    if (dtype && dtype_len > 0) snprintf(dtype, (size_t)dtype_len, "%s", e.dtype.c_str());
    *ndim = (int32_t)e.shape.size();
    for (int32_t i = 0; shape && i < max_ndim && i < *ndim; ++i)
        shape[i] = e.shape[i] > (uint64_t)INT64_MAX ? -1 : (int64_t)e.shape[i];
    return LASTRO_OK;
}

extern "C" int lastro_checkpoint_read_bf16(const lastro_checkpoint* ck, const char* name, uint16_t* dst,
                                           int64_t capacity, char* err, int32_t err_len) {
    if (!ck || !name || capacity < 0) return put_err(err, err_len, LASTRO_E_ARG, "null argument");
    return read_tensor(ck, name, "BF16", 2, dst, (uint64_t)capacity * 2, err, err_len);
}

extern "C" int lastro_config_from_json(const char* json, lastro_model_desc* out, char* err, int32_t err_len) {
    if (!json || !out) return put_err(err, err_len, LASTRO_E_ARG, "null argument");
    lastro_json::Value v;
    std::string jerr;
    if (!lastro_json::parse(json, strlen(json), &v, &jerr) || v.kind != lastro_json::Value::Object)
        return put_err(err, err_len, LASTRO_E_ARG, "config.json: %s", jerr.empty() ? "not an object" : jerr.c_str());
    // model.rs:37-42: only the architecture the kernels implement
    const lastro_json::Value* mt = v.get("model_type");
    if (!mt || mt->kind != lastro_json::Value::String || mt->s != "granitemoe")
        return put_err(err, err_len, LASTRO_E_UNSUPPORTED, "model_type %s (expected granitemoe)",
                       mt && mt->kind == lastro_json::Value::String ? mt->s.c_str() : "missing");
    const lastro_json::Value* rs = v.get("rope_scaling");
    const lastro_json::Value* ab = v.get("attention_bias");
    const lastro_json::Value* te = v.get("tie_word_embeddings");
    if ((rs && rs->kind != lastro_json::Value::Null) || (ab && ab->kind == lastro_json::Value::Bool && ab->b) ||
        (te && te->kind == lastro_json::Value::Bool && !te->b))
        return put_err(err, err_len, LASTRO_E_UNSUPPORTED,
                       "unsupported variant (rope_scaling, attention_bias or untied embeddings)");
    lastro_model_desc d{};
    const struct {
        const char* key;
        int32_t* dst;
    } ints[] = {{"hidden_size", &d.hidden},         {"intermediate_size", &d.inter},
                {"num_hidden_layers", &d.layers},   {"num_attention_heads", &d.heads},
                {"num_key_value_heads", &d.kv_heads}, {"vocab_size", &d.vocab},
                {"num_local_experts", &d.experts},  {"num_experts_per_tok", &d.k}};
    for (const auto& f : ints)
        if (!json_u32(v, f.key, f.dst)) return put_err(err, err_len, LASTRO_E_ARG, "config.json without %s", f.key);
    const struct {
        const char* key;
        float* dst;
    } floats[] = {{"rope_theta", &d.rope_theta},
                  {"rms_norm_eps", &d.eps},
                  {"embedding_multiplier", &d.embedding_multiplier},
                  {"residual_multiplier", &d.residual_multiplier},
                  {"attention_multiplier", &d.attention_multiplier},
                  {"logits_scaling", &d.logits_scaling}};
    for (const auto& f : floats)
        if (!json_f32(v, f.key, f.dst)) return put_err(err, err_len, LASTRO_E_ARG, "config.json without %s", f.key);
    if (d.heads < 1) return put_err(err, err_len, LASTRO_E_ARG, "config.json: num_attention_heads 0");
    // model.rs:49: head_dim when present, else hidden / heads
    if (!json_u32(v, "head_dim", &d.head_dim)) d.head_dim = d.hidden / d.heads;
    d.weight_dtype = LASTRO_DTYPE_BF16;
    d.kv_dtype = LASTRO_DTYPE_BF16;
    *out = d;
    return LASTRO_OK;
}

extern "C" int lastro_checkpoint_config(const lastro_checkpoint* ck, lastro_model_desc* out, char* err,
                                        int32_t err_len) {
    if (!ck || !out) return put_err(err, err_len, LASTRO_E_ARG, "null argument");
    const std::string path = ck->dir + "/config.json";
    const int fd = open(path.c_str(), O_RDONLY | O_CLOEXEC);
    if (fd < 0) return put_err(err, err_len, LASTRO_E_IO, "I/O: cannot open %s", path.c_str());
    struct stat st;
    std::string text;
    bool ok = fstat(fd, &st) == 0 && st.st_size < (1 << 24);
    if (ok) {
        text.resize((size_t)st.st_size);
        ok = st.st_size == 0 || read_at(fd, &text[0], (uint64_t)st.st_size, 0);
    }
    close(fd);
    if (!ok) return put_err(err, err_len, LASTRO_E_IO, "I/O: reading %s", path.c_str());
    return lastro_config_from_json(text.c_str(), out, err, err_len);
}

// model.rs:99-132 + block.rs:31-53: every tensor the decode step needs, each checked for dtype, byte size and shape
// before it is read, then copied to the device by lastro_model_load_tensor.  bf16 models take BF16 tensors; a Q8_0
// model takes its linear weights as U8 tensors whose last axis holds each row's 34-byte blocks (fp16 scale, then 32
// int8 values) and its norms and embedding as BF16.
extern "C" int lastro_model_load_checkpoint(lastro_model* model, const lastro_checkpoint* ck) {
    if (!model) return LASTRO_E_ARG;
    lastro_ctx* ctx = model->ctx;
    if (!ck) return lastro_capi::set_err(ctx, LASTRO_E_ARG, "null checkpoint");
    const lastro_model_desc* d = &model->d;
    const uint64_t H = (uint64_t)d->hidden, I = (uint64_t)d->inter, E = (uint64_t)d->experts, V = (uint64_t)d->vocab;
    const uint64_t qd = (uint64_t)d->heads * d->head_dim, kvd = (uint64_t)d->kv_heads * d->head_dim;
    const bool q8 = d->weight_dtype == LASTRO_DTYPE_Q8_0;
    struct Want {
        std::string name;
        std::vector<uint64_t> shape;  // in weights (columns last)
        bool linear;
    };
    std::vector<Want> want = {{"model.embed_tokens.weight", {V, H}, false}, {"model.norm.weight", {H}, false}};
    for (int32_t l = 0; l < d->layers; ++l) {
        const std::string p = "model.layers." + std::to_string(l) + ".";
        want.push_back({p + "input_layernorm.weight", {H}, false});
        want.push_back({p + "post_attention_layernorm.weight", {H}, false});
        want.push_back({p + "self_attn.q_proj.weight", {qd, H}, true});
        want.push_back({p + "self_attn.k_proj.weight", {kvd, H}, true});
        want.push_back({p + "self_attn.v_proj.weight", {kvd, H}, true});
        want.push_back({p + "self_attn.o_proj.weight", {H, qd}, true});
        want.push_back({p + "block_sparse_moe.router.layer.weight", {E, H}, true});
        want.push_back({p + "block_sparse_moe.input_linear.weight", {E, 2 * I, H}, true});
        want.push_back({p + "block_sparse_moe.output_linear.weight", {E, H, I}, true});
    }
    std::vector<unsigned char> buf;
    char msg[512];
    for (const Want& w : want) {
        const bool as_q8 = q8 && w.linear;
        std::vector<uint64_t> file_shape = w.shape;
        if (as_q8) file_shape.back() = file_shape.back() / 32 * 34;  // the model requires whole blocks
        auto it = ck->index.find(w.name);
        if (it == ck->index.end())
            return lastro_capi::set_err(ctx, LASTRO_E_ARG, "safetensors: tensor absent: %s", w.name.c_str());
        if (it->second.shape != file_shape)
            return lastro_capi::set_err(ctx, LASTRO_E_ARG, "%s: shape %s (expected %s)", w.name.c_str(),
                                        shape_text(it->second.shape).c_str(), shape_text(file_shape).c_str());
        uint64_t bytes = 0;
        shape_bytes(file_shape, as_q8 ? 1 : 2, &bytes);
        buf.resize(bytes);
        int rc = read_tensor(ck, w.name.c_str(), as_q8 ? "U8" : "BF16", as_q8 ? 1 : 2, buf.data(), bytes, msg,
                             (int32_t)sizeof msg);
        if (rc) return lastro_capi::set_err(ctx, rc, "%s", msg);
        std::vector<int64_t> shape(w.shape.begin(), w.shape.end());
        rc = lastro_model_load_tensor(model, w.name.c_str(), as_q8 ? LASTRO_DTYPE_Q8_0 : LASTRO_DTYPE_BF16, shape.data(),
                                      (int32_t)shape.size(), buf.data());
        if (rc) return rc;  // lastro_model_load_tensor set the message
    }
    return LASTRO_OK;
}
