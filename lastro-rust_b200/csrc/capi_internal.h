// Internal to liblastro_b200.so: the context and model objects shared by the C-ABI translation units (capi.cu:
// context, MoE block and batch-1 model; batch_capi.cu: batched decode with expert parallelism).
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <string>
#include <vector>

#include "../../include/lastro_b200.h"
#include "batch.h"
#include "kernels.h"

// Reference-counted by its layers and models, so that the context and its objects may be destroyed in any order
// (a garbage-collected host language finalises objects in no fixed order).
struct lastro_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;
    bool own_stream = false;
    std::string err;
    std::atomic<int> refs{1};
    std::atomic<bool> closed{false};
};

namespace lastro_capi {

inline int set_err(lastro_ctx* c, int code, const char* fmt, ...) {
    if (c) {
        char buf[512];
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(buf, sizeof buf, fmt, ap);
        va_end(ap);
        c->err = buf;
    }
    return code;
}

// synthetic tensor seed: the same formula as the CPU oracle's lo_tensor_seed
inline uint64_t mix64_host(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

inline uint64_t tensor_seed(uint64_t base, int layer, int kind) {
    return mix64_host(base * 0x9E3779B97F4A7C15ull + ((uint64_t)(uint32_t)(layer + 1) << 8) + (uint64_t)kind + 1u);
}

inline float synth_scale(float sd) { return sd / 37837.2265f; }

enum { K_EMBED = 0, K_NORM, K_LN_ATTN, K_LN_MOE, K_Q, K_K, K_V, K_O, K_ROUTER, K_GATE_UP, K_DOWN, K_COUNT };

// Device allocations of one object, freed together.
struct Arena {
    std::vector<void*> ptrs;
    size_t bytes = 0;
    cudaError_t alloc(void** p, size_t n) {
        *p = nullptr;
        if (n == 0) n = 16;
        cudaError_t e = cudaMalloc(p, n);
        if (e == cudaSuccess) {
            ptrs.push_back(*p);
            bytes += n;
        }
        return e;
    }
    template <typename T>
    cudaError_t alloc(T** p, size_t count) {
        return alloc(reinterpret_cast<void**>(p), count * sizeof(T));
    }
    void release() {
        for (void* p : ptrs) cudaFree(p);
        ptrs.clear();
        bytes = 0;
    }
};


inline void ctx_retain(lastro_ctx* c) { c->refs.fetch_add(1); }

inline void ctx_release(lastro_ctx* c) {
    if (c->refs.fetch_sub(1) != 1) return;
    cudaSetDevice(c->device);
    if (c->stream) cudaStreamSynchronize(c->stream);
    if (c->own_stream) cudaStreamDestroy(c->stream);
    delete c;
}


// gpu.rs:345-355: synchronize the stream before reporting, then poison
inline int cuda_fail(lastro_ctx* c, bool* poisoned, cudaError_t e, const char* what) {
    cudaStreamSynchronize(c->stream);
    cudaGetLastError();
    *poisoned = true;
    return set_err(c, LASTRO_E_CUDA, "%s: %s", what, cudaGetErrorString(e));
}



struct LayerDev {
    float *ln_attn = nullptr, *ln_moe = nullptr;
    float* wr_t = nullptr;  // [H, E] router weight x ln_moe, transposed (fused router operand)
    bool fold_dirty = true;
    // linear weights: bf16 rows, or Q8_0 rows in the device layout (wrow_bytes): byte buffers either way
    unsigned char *wqkv = nullptr, *wo = nullptr, *router = nullptr, *gate_up = nullptr, *down = nullptr;
    void *k_pool = nullptr, *v_pool = nullptr;
};

constexpr int kPageSize = 64;

// model.rs:63-73: inv_freq = 1/theta^(2j/d) and cos/sin of pos*inv_freq, in f32 on the host; [max_len][d]: cos of the
// d/2 frequencies, then their sin
inline std::vector<float> rope_table(const lastro_model_desc& d, int max_len) {
    std::vector<float> cs((size_t)max_len * d.head_dim);
    const int half = d.head_dim / 2;
    for (int p = 0; p < max_len; ++p)
        for (int j = 0; j < half; ++j) {
            const float inv = 1.0f / powf(d.rope_theta, (float)(2 * j) / (float)d.head_dim);
            const float f = (float)p * inv;
            cs[(size_t)p * d.head_dim + j] = cosf(f);
            cs[(size_t)p * d.head_dim + half + j] = sinf(f);
        }
    return cs;
}

}  // namespace lastro_capi

struct lastro_model {
    lastro_ctx* ctx = nullptr;
    lastro_model_desc d{};
    int max_len = 0, qd = 0, kvd = 0, G = 1, max_pages = 0, head_grid = 1;
    int q8 = 0;  // linear weights are Q8_0
    bool poisoned = false;
    bool use_graphs = true, use_pdl = true;
    lastro_capi::Arena arena;
    uint16_t* embed = nullptr;
    float* norm = nullptr;
    std::vector<lastro_capi::LayerDev> L;
    float* rope_cs = nullptr;
    int* page_table = nullptr;
    // per-step state
    float *h = nullptr, *q = nullptr, *att = nullptr;
    float *part_acc = nullptr, *part_ml = nullptr;  // attention splits [heads, kAttnSplits, d] / [.., 2]
    float *rlogits = nullptr, *route_w = nullptr, *rnorm = nullptr, *a = nullptr, *logits = nullptr;
    // the router logits of each layer's input (qkv kernel), from which the experts the layer will most likely route
    // to are fetched before the routing is known (bf16 weights): 2 hinted into L2 by the output projection's CTAs
    // while the attention runs (LASTRO_TUNE_SPEC_L2), 1 staged into shared memory by the gate_up CTAs
    // (LASTRO_TUNE_SPEC_STAGE), 0 off (the default)
    float* spec_logits = nullptr;
    int spec_mode = 0;  // 3: the predicted top-k hinted into L2 by the attention kernel's CTAs (LASTRO_TUNE_SPEC_ATTN)
    int* spec_ids = nullptr;
    unsigned int* spec_ticket = nullptr;
    // the routing hand-off from gate_up to down: a step counter (advanced by the step's first kernel) and a flag per
    // layer; on unless LASTRO_TUNE_DOWN_ROUTES
    unsigned int* step_ctr = nullptr;
    unsigned int* route_flags = nullptr;
    bool route_handoff = true;
    int *route_ids = nullptr, *d_token = nullptr, *d_pos = nullptr, *d_step = nullptr, *d_out_ids = nullptr;
    int* d_prompt = nullptr;
    unsigned int *router_counter = nullptr, *head_counter = nullptr, *attn_counters = nullptr;
    unsigned long long* head_partial = nullptr;
    float* op_partial = nullptr;  // [oproj_grid(H), E + 1]
    int* d_err = nullptr;    // error word of the bounded waits
    int* h_token = nullptr;  // pinned
    int* h_err = nullptr;    // pinned copy of d_err
    int pos_host = 0;
    std::vector<char> loaded;  // per (layer, kind)
    cudaGraphExec_t graph = nullptr;
    // in-graph timeline (lastro_model_trace): stamp buffer and the step graph captured with the stamps on
    unsigned long long* d_trace = nullptr;
    cudaGraphExec_t trace_graph = nullptr;
    std::vector<unsigned long long> trace_host;  // the last traced step's stamps
    // fused step (one persistent launch per step) when the shapes fit it
    bool fused_ok = false, use_fused = false;
    lastro::FusedLayout flay{};
    lastro::FusedLayer* f_layers = nullptr;  // [layers] (device)
    unsigned int *f_ticket = nullptr, *f_epoch = nullptr, *f_count = nullptr;
    lastro::FusedExchange fx{};
    unsigned long long* f_best = nullptr;
    // bf16 KV: optional attention on tensor cores (the batched step's streaming kernel, 16 context splits) with TMA page
    // loads through these maps (per layer: K, V); the CUDA-core split kernel by default
    std::vector<CUtensorMap> kvmaps;
    bool attn_tc = false;
    // bf16 KV: the split attention kernel's staging maps (per layer: K, V; 8-row boxes, 128-byte swizzle) and
    // whether it uses them (LASTRO_TUNE_ATTN_TMA) or one bulk copy per page run (the default)
    std::vector<CUtensorMap> kvboxmaps;
    bool attn_tma = false;
    bool attn_mma = false;  // bf16 K/V scored and summed on tensor cores (LASTRO_TUNE_ATTN_MMA)
    // the MoE block as one persistent launch per layer (moe_kernel) where the shapes fit it and the option is on (off
    // by default), else the gate_up and down kernels; its grid barrier's counter
    lastro::MoePlan moe{};
    // batch-1 attention: context splits (8 or 16) and where the splits are merged (the attention kernel's last CTA, or
    // the output projection as it loads them); lastro_model_set_tuning
    int attn_splits = 16;
    int attn_merge = 0;  // 0: the attention's last CTA per KV head, 1: the output projection, 2: a cluster per KV head
    bool oproj_smem = false;  // the output projection's weights staged in shared memory (oproj_smem_kernel)
    bool gu_prefetch_down = false;  // gate_up hints the chosen experts' down slabs into L2
    bool moe_ok = false, use_moe = false;
    unsigned long long* moe_barrier = nullptr;
    // multi-position steps (lastro_model_step_positions): a batch of the model's own sequence on its KV cache
    lastro_batch* pbatch = nullptr;
};

namespace lastro_capi {
// positions of one multi-position step (cuda_backend.rs:264-266: 1..=32)
constexpr int kMaxStepPositions = 32;
// every tensor loaded, router folds current, not poisoned (defined in capi.cu)
int model_check_ready(lastro_model* m);
}  // namespace lastro_capi
