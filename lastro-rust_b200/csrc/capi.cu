// C ABI of liblastro_b200.so: context, MoE block (GpuLayer) and whole model (GpuModel).
//
// Host-side mirror of the reference's operator API (brenoperucchi/lastro-rust, rust/moe-rt/src/gpu.rs and
// gpu_model.rs): same objects, same argument meaning, same error policy -- argument errors are refused before any
// launch, runtime errors synchronize the stream and poison the object (gpu_model.rs:249-267).
//
// B200 layout: all weights resident in HBM (the reference's expert cache collapses: the 3B model is 6.4 GB of a
// 180 GB part), q/k/v projections concatenated into one [qd + 2 kvd, H] matrix, K/V in pages of 64 positions
// ([page][kv_head][slot][d], bf16 or f32) behind a page table, and the whole decode step captured once as a CUDA
// graph whose kernels read the token and position from device memory, so one graph serves every position.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "capi_internal.h"

using namespace lastro;
using namespace lastro_capi;

#define LASTRO_VERSION "lastro-b200 0.1.0 (sm_100a)"

// =====================================================================================================================
// context
// =====================================================================================================================
extern "C" const char* lastro_version(void) { return LASTRO_VERSION; }

extern "C" int lastro_ctx_create(int32_t device, void* stream, lastro_ctx** out) {
    if (!out) return LASTRO_E_ARG;
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        return LASTRO_E_CUDA;
    }
    if (device < 0 || device >= n) return LASTRO_E_ARG;
    if (cudaSetDevice(device) != cudaSuccess) return LASTRO_E_CUDA;
    lastro_ctx* c = new lastro_ctx();
    c->device = device;
    if (stream) {
        c->stream = static_cast<cudaStream_t>(stream);
    } else {
        if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess) {
            delete c;
            return LASTRO_E_CUDA;
        }
        c->own_stream = true;
    }
    *out = c;
    return LASTRO_OK;
}


extern "C" void lastro_ctx_destroy(lastro_ctx* c) {
    if (!c || c->closed.exchange(true)) return;
    ctx_release(c);
}

extern "C" int lastro_ctx_synchronize(lastro_ctx* c) {
    if (!c) return LASTRO_E_ARG;
    cudaError_t e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess) return set_err(c, LASTRO_E_CUDA, "synchronize: %s", cudaGetErrorString(e));
    return LASTRO_OK;
}

extern "C" const char* lastro_last_error(const lastro_ctx* c) { return c ? c->err.c_str() : "null context"; }

// =====================================================================================================================
// MoE block (GpuLayer)
// =====================================================================================================================
struct lastro_layer {
    lastro_ctx* ctx = nullptr;
    int E = 0, H = 0, I = 0, k = 0;
    int q8 = 0;  // weights are Q8_0 rows in the device layout (wrow_bytes)
    bool poisoned = false;
    Arena arena;
    unsigned char *router = nullptr, *gate_up = nullptr, *down = nullptr;
    float *x = nullptr, *y = nullptr, *logits = nullptr, *weights = nullptr, *a = nullptr;
    int* ids = nullptr;
    unsigned int* counter = nullptr;
    int* err = nullptr;  // device error word of the bounded waits
};

namespace {

int check_block_shape(lastro_ctx* c, int E, int H, int I, int k, int q8 = 0) {
    if (E < 1 || H < 8 || I < 8 || k < 1) return set_err(c, LASTRO_E_ARG, "block shape E=%d H=%d I=%d k=%d", E, H, I, k);
    if (k > E) return set_err(c, LASTRO_E_ARG, "k=%d > experts=%d", k, E);
    if (H % 8 || I % 8) return set_err(c, LASTRO_E_UNSUPPORTED, "H=%d and I=%d must be multiples of 8", H, I);
    if (H > kMaxHidden || I > kMaxInter || E > kMaxExperts || k > kMaxTopK)
        return set_err(c, LASTRO_E_UNSUPPORTED, "block shape beyond the kernels' limits (H<=%d I<=%d E<=%d k<=%d)",
                       kMaxHidden, kMaxInter, kMaxExperts, kMaxTopK);
    if (I % gate_up_rows_per_cta() || H % down_rows_per_cta())
        return set_err(c, LASTRO_E_UNSUPPORTED, "I=%d must be a multiple of %d and H=%d of %d", I, gate_up_rows_per_cta(),
                       H, down_rows_per_cta());
    if (q8 && (H % 32 || I % 32)) return set_err(c, LASTRO_E_UNSUPPORTED, "Q8_0: H=%d and I=%d must be multiples of 32", H, I);
    if (down_smem(H, I, k, q8) > kMaxSmemBytes || gate_up_smem(H, q8) > kMaxSmemBytes)
        return set_err(c, LASTRO_E_UNSUPPORTED, "k=%d, I=%d, H=%d: expert tiles exceed shared memory", k, I, H);
    return LASTRO_OK;
}

#define LASTRO_TRY(expr, what)                                                   \
    do {                                                                         \
        cudaError_t e_ = (expr);                                                 \
        if (e_ != cudaSuccess) return cuda_fail(ctx, &obj->poisoned, e_, what);  \
    } while (0)

// router -> gate_up -> down of one block; `xn` is the block input, `out` receives y (accumulate=0) or h += resid*y
int enqueue_block(lastro_layer* obj, const float* xn, float* out, float resid, int accumulate) {
    lastro_ctx* ctx = obj->ctx;
    cudaStream_t s = ctx->stream;
    RouterArgs ra{};
    ra.x = xn;
    ra.norm_mode = 0;
    ra.w = obj->router;
    ra.q8 = obj->q8;
    ra.logits = obj->logits;
    ra.ids = obj->ids;
    ra.weights = obj->weights;
    ra.counter = obj->counter;
    ra.E = obj->E;
    ra.H = obj->H;
    ra.k = obj->k;
    LASTRO_TRY(launch_router(ra, s, false), "router launch");
    GateUpArgs ga{};
    ga.x = xn;
    ga.ids = obj->ids;
    ga.w = obj->gate_up;
    ga.q8 = obj->q8;
    ga.a = obj->a;
    ga.err = obj->err;
    ga.H = obj->H;
    ga.I = obj->I;
    ga.k = obj->k;
    ga.E = obj->E;
    LASTRO_TRY(launch_gate_up(ga, s, true), "gate_up launch");
    DownArgs da{};
    da.a = obj->a;
    da.ids = obj->ids;
    da.weights = obj->weights;
    da.w = obj->down;
    da.q8 = obj->q8;
    da.out = out;
    da.resid = resid;
    da.accumulate = accumulate;
    da.err = obj->err;
    da.H = obj->H;
    da.I = obj->I;
    da.k = obj->k;
    da.E = obj->E;
    LASTRO_TRY(launch_down(da, s, true), "down launch");
    return LASTRO_OK;
}

}  // namespace

namespace {

// Q8_0 host rows (blocks of 34 bytes: fp16 scale, then 32 int8 values) -> the device row layout (wrow_bytes: the
// row's int8 values, then its fp16 scales, padded to 16 bytes)
std::vector<unsigned char> repack_q8_rows(const unsigned char* src, size_t rows, int cols) {
    const size_t nb = (size_t)cols / 32, rb = wrow_bytes(cols, 1);
    std::vector<unsigned char> buf(rows * rb, 0);
    for (size_t r = 0; r < rows; ++r)
        for (size_t b = 0; b < nb; ++b) {
            const unsigned char* blk = src + (r * nb + b) * 34;
            memcpy(&buf[r * rb + (size_t)cols + 2 * b], blk, 2);
            memcpy(&buf[r * rb + 32 * b], blk + 2, 32);
        }
    return buf;
}

int layer_create(lastro_ctx* ctx, int E, int H, int I, int k, int q8, const void* router, const void* gate_up,
                 const void* down, lastro_layer** out) {
    if (!ctx || !out) return LASTRO_E_ARG;
    *out = nullptr;
    if (!router || !gate_up || !down) return set_err(ctx, LASTRO_E_ARG, "null weight pointer");
    int rc = check_block_shape(ctx, E, H, I, k, q8);
    if (rc) return rc;
    cudaSetDevice(ctx->device);
    lastro_layer* obj = new lastro_layer();
    obj->ctx = ctx;
    obj->E = E;
    obj->H = H;
    obj->I = I;
    obj->k = k;
    obj->q8 = q8;
    Arena& A = obj->arena;
    const size_t rbh = wrow_bytes(H, q8), rbi = wrow_bytes(I, q8);
    const size_t nr = (size_t)E * rbh, ngu = (size_t)E * 2 * I * rbh, nd = (size_t)E * H * rbi;  // bytes
    if (A.alloc(&obj->router, nr) || A.alloc(&obj->gate_up, ngu) || A.alloc(&obj->down, nd) || A.alloc(&obj->x, H) ||
        A.alloc(&obj->y, H) || A.alloc(&obj->logits, E) || A.alloc(&obj->weights, k) || A.alloc(&obj->a, (size_t)k * I) ||
        A.alloc(&obj->ids, k) || A.alloc(&obj->counter, 1) || A.alloc(&obj->err, 1)) {
        cudaGetLastError();
        A.release();
        delete obj;
        return set_err(ctx, LASTRO_E_NOMEM, "layer allocation failed");
    }
    cudaError_t e = cudaSuccess;
    if (q8) {
        const auto* r8 = static_cast<const unsigned char*>(router);
        const auto* g8 = static_cast<const unsigned char*>(gate_up);
        const auto* d8 = static_cast<const unsigned char*>(down);
        const std::vector<unsigned char> br = repack_q8_rows(r8, E, H), bg = repack_q8_rows(g8, (size_t)E * 2 * I, H),
                                         bd = repack_q8_rows(d8, (size_t)E * H, I);
        e = cudaMemcpyAsync(obj->router, br.data(), nr, cudaMemcpyHostToDevice, ctx->stream);
        if (!e) e = cudaMemcpyAsync(obj->gate_up, bg.data(), ngu, cudaMemcpyHostToDevice, ctx->stream);
        if (!e) e = cudaMemcpyAsync(obj->down, bd.data(), nd, cudaMemcpyHostToDevice, ctx->stream);
        if (!e) e = cudaStreamSynchronize(ctx->stream);  // the staging vectors die with this scope
    } else {
        e = cudaMemcpyAsync(obj->router, router, nr, cudaMemcpyHostToDevice, ctx->stream);
        if (!e) e = cudaMemcpyAsync(obj->gate_up, gate_up, ngu, cudaMemcpyHostToDevice, ctx->stream);
        if (!e) e = cudaMemcpyAsync(obj->down, down, nd, cudaMemcpyHostToDevice, ctx->stream);
    }
    if (!e) e = cudaMemsetAsync(obj->counter, 0, sizeof(unsigned int), ctx->stream);
    if (!e) e = cudaMemsetAsync(obj->ids, 0, sizeof(int) * k, ctx->stream);
    if (!e) e = cudaMemsetAsync(obj->err, 0, sizeof(int), ctx->stream);
    if (!e) e = cudaMemsetAsync(obj->weights, 0, sizeof(float) * k, ctx->stream);
    if (!e) e = cudaStreamSynchronize(ctx->stream);
    if (e) {
        cudaGetLastError();
        A.release();
        delete obj;
        return set_err(ctx, LASTRO_E_CUDA, "layer upload: %s", cudaGetErrorString(e));
    }
    ctx_retain(ctx);
    *out = obj;
    return LASTRO_OK;
}

}  // namespace

extern "C" int lastro_layer_create(lastro_ctx* ctx, int32_t E, int32_t H, int32_t I, int32_t k, const uint16_t* router,
                                   const uint16_t* gate_up, const uint16_t* down, lastro_layer** out) {
    return layer_create(ctx, E, H, I, k, 0, router, gate_up, down, out);
}

extern "C" int lastro_layer_create_q8_0(lastro_ctx* ctx, int32_t E, int32_t H, int32_t I, int32_t k,
                                        const uint8_t* router, const uint8_t* gate_up, const uint8_t* down,
                                        lastro_layer** out) {
    return layer_create(ctx, E, H, I, k, 1, router, gate_up, down, out);
}

extern "C" int lastro_layer_forward(lastro_layer* obj, const float* x, float* y, int32_t* ids, float* weights,
                                    float* logits) {
    if (!obj) return LASTRO_E_ARG;
    lastro_ctx* ctx = obj->ctx;
    if (obj->poisoned) return set_err(ctx, LASTRO_E_POISONED, "layer unusable after an earlier error");
    if (!x) return set_err(ctx, LASTRO_E_ARG, "null x");
    cudaSetDevice(ctx->device);
    cudaStream_t s = ctx->stream;
    LASTRO_TRY(cudaMemcpyAsync(obj->x, x, sizeof(float) * obj->H, cudaMemcpyHostToDevice, s), "x upload");
    int rc = enqueue_block(obj, obj->x, obj->y, 0.0f, 0);
    if (rc) return rc;
    if (y) LASTRO_TRY(cudaMemcpyAsync(y, obj->y, sizeof(float) * obj->H, cudaMemcpyDeviceToHost, s), "y download");
    if (ids) LASTRO_TRY(cudaMemcpyAsync(ids, obj->ids, sizeof(int) * obj->k, cudaMemcpyDeviceToHost, s), "ids download");
    if (weights)
        LASTRO_TRY(cudaMemcpyAsync(weights, obj->weights, sizeof(float) * obj->k, cudaMemcpyDeviceToHost, s), "w download");
    if (logits)
        LASTRO_TRY(cudaMemcpyAsync(logits, obj->logits, sizeof(float) * obj->E, cudaMemcpyDeviceToHost, s), "logits");
    int err = 0;
    LASTRO_TRY(cudaMemcpyAsync(&err, obj->err, sizeof(int), cudaMemcpyDeviceToHost, s), "error word");
    LASTRO_TRY(cudaStreamSynchronize(s), "layer forward");
    if (err) {
        obj->poisoned = true;
        return set_err(ctx, LASTRO_E_CUDA, "a kernel wait gave up (code %d); layer poisoned", err);
    }
    return LASTRO_OK;
}

extern "C" int lastro_layer_add_into(lastro_layer* obj, const float* xn, float* h, float resid, int32_t* ids,
                                     float* weights) {
    if (!obj) return LASTRO_E_ARG;
    lastro_ctx* ctx = obj->ctx;
    if (obj->poisoned) return set_err(ctx, LASTRO_E_POISONED, "layer unusable after an earlier error");
    if (!xn || !h) return set_err(ctx, LASTRO_E_ARG, "null device pointer");
    cudaSetDevice(ctx->device);
    cudaStream_t s = ctx->stream;
    int rc = enqueue_block(obj, xn, h, resid, 1);
    if (rc) return rc;
    if (ids) LASTRO_TRY(cudaMemcpyAsync(ids, obj->ids, sizeof(int) * obj->k, cudaMemcpyDeviceToDevice, s), "ids copy");
    if (weights)
        LASTRO_TRY(cudaMemcpyAsync(weights, obj->weights, sizeof(float) * obj->k, cudaMemcpyDeviceToDevice, s), "w copy");
    return LASTRO_OK;
}

extern "C" void lastro_layer_destroy(lastro_layer* obj) {
    if (!obj) return;
    cudaSetDevice(obj->ctx->device);
    cudaStreamSynchronize(obj->ctx->stream);  // gpu.rs:544-550: kernels may still read the weights
    obj->arena.release();
    lastro_ctx* ctx = obj->ctx;
    delete obj;
    ctx_release(ctx);
}

// =====================================================================================================================
// whole model (GpuModel)
// =====================================================================================================================


namespace {

int model_fail(lastro_model* m, cudaError_t e, const char* what) { return cuda_fail(m->ctx, &m->poisoned, e, what); }

#define MTRY(expr, what)                                        \
    do {                                                        \
        cudaError_t e_ = (expr);                                \
        if (e_ != cudaSuccess) return model_fail(m, e_, what);  \
    } while (0)

size_t kv_elem_bytes(const lastro_model* m) { return m->d.kv_dtype == LASTRO_DTYPE_F32 ? 4 : 2; }

char& loaded_flag(lastro_model* m, int layer, int kind) { return m->loaded[(size_t)(layer + 1) * K_COUNT + kind]; }

const char* kind_name(int kind) {
    static const char* names[K_COUNT] = {"model.embed_tokens.weight",
                                         "model.norm.weight",
                                         "input_layernorm.weight",
                                         "post_attention_layernorm.weight",
                                         "self_attn.q_proj.weight",
                                         "self_attn.k_proj.weight",
                                         "self_attn.v_proj.weight",
                                         "self_attn.o_proj.weight",
                                         "block_sparse_moe.router.layer.weight",
                                         "block_sparse_moe.input_linear.weight",
                                         "block_sparse_moe.output_linear.weight"};
    return names[kind];
}

int missing_tensor(lastro_model* m) {
    if (!loaded_flag(m, -1, K_EMBED)) return set_err(m->ctx, LASTRO_E_STATE, "tensor %s not loaded", kind_name(K_EMBED));
    if (!loaded_flag(m, -1, K_NORM)) return set_err(m->ctx, LASTRO_E_STATE, "tensor %s not loaded", kind_name(K_NORM));
    for (int l = 0; l < m->d.layers; ++l)
        for (int k = K_LN_ATTN; k < K_COUNT; ++k)
            if (!loaded_flag(m, l, k))
                return set_err(m->ctx, LASTRO_E_STATE, "tensor model.layers.%d.%s not loaded", l, kind_name(k));
    return LASTRO_OK;
}

// Kernel kinds of one step, in launch order within a layer (the head closes the step).
enum { KK_QKV = 0, KK_ATTN, KK_OPROJ, KK_ROUTER, KK_GATE_UP, KK_DOWN, KK_HEAD, KK_FUSED, KK_MOE, KK_COUNT };

bool moe_on(const lastro_model* m) { return m->moe_ok && m->use_moe; }

FusedArgs fused_args(const lastro_model* m) {
    const lastro_model_desc& d = m->d;
    FusedArgs a{};
    a.layers = m->f_layers;
    a.L = d.layers;
    a.embed = m->embed;
    a.norm = m->norm;
    a.rope_cs = m->rope_cs;
    a.page_table = m->page_table;
    a.page_size = kPageSize;
    a.pos = m->d_pos;
    a.token = m->d_token;
    a.step = m->d_step;
    a.out_ids = m->d_out_ids;
    a.out_cap = m->max_len + 1;
    a.x = m->fx;
    a.logits = m->logits;
    a.route_ids = m->route_ids;
    a.route_w = m->route_w;
    a.rlogits = m->rlogits;
    a.best = m->f_best;
    a.ticket = m->f_ticket;
    a.count = m->f_count;
    a.epoch = m->f_epoch;
    a.err = m->d_err;
    a.H = d.hidden;
    a.I = d.inter;
    a.E = d.experts;
    a.k = d.k;
    a.qd = m->qd;
    a.kvd = m->kvd;
    a.kv_heads = d.kv_heads;
    a.G = m->G;
    a.V = d.vocab;
    a.eps = d.eps;
    a.emb_mult = d.embedding_multiplier;
    a.resid = d.residual_multiplier;
    a.attn_scale = d.attention_multiplier;
    a.logits_scaling = d.logits_scaling;
    a.lay = m->flay;
    return a;
}

// Optional per-launch events: ev[0] before the first launch, ev[i + 1] after launch i.
struct StepEvents {
    cudaEvent_t* ev = nullptr;
    int* kind = nullptr;  // kind of launch i (between ev[i] and ev[i + 1])
    int next = 0;
};

cudaError_t mark(StepEvents* pe, cudaStream_t s, int kind = -1) {
    if (!pe) return cudaSuccess;
    if (pe->next > 0) pe->kind[pe->next - 1] = kind;
    return cudaEventRecord(pe->ev[pe->next++], s);
}

// Enqueue the kernels of one decode step; the token is read from d_token, the position from d_pos.
// trace: with a timeline buffer ([launches][kTraceMaxCtas][3] words), launch i of the step stamps slot i
cudaError_t enqueue_step(lastro_model* m, cudaStream_t s, StepEvents* pe = nullptr, unsigned long long* trace = nullptr) {
    const lastro_model_desc& d = m->d;
    const bool pdl = m->use_pdl && !pe;
    cudaError_t e;
    int launch = 0;
    auto slot = [&]() -> unsigned long long* {
        return trace ? trace + (size_t)(launch++) * kTraceMaxCtas * kTraceWords : nullptr;
    };
    if ((e = mark(pe, s)) != cudaSuccess) return e;
    if (m->fused_ok && m->use_fused) {
        if ((e = launch_fused_step(fused_args(m), d.kv_dtype == LASTRO_DTYPE_F32, s)) != cudaSuccess) return e;
        return mark(pe, s, KK_FUSED);
    }
    for (int l = 0; l < d.layers; ++l) {
        const LayerDev& L = m->L[l];
        QkvArgs qa{};
        qa.h = m->h;
        qa.h_write = m->h;
        qa.embed = m->embed;
        qa.token = m->d_token;
        qa.emb_mult = d.embedding_multiplier;
        qa.embed_mode = (l == 0);
        qa.ln = L.ln_attn;
        qa.w = L.wqkv;
        qa.q8 = m->q8;
        qa.rope_cs = m->rope_cs;
        qa.pos = m->d_pos;
        qa.q_out = m->q;
        qa.k_pool = L.k_pool;
        qa.v_pool = L.v_pool;
        qa.page_table = m->page_table;
        qa.page_size = kPageSize;
        qa.kv_f32 = d.kv_dtype == LASTRO_DTYPE_F32;
        qa.H = d.hidden;
        qa.qd = m->qd;
        qa.kvd = m->kvd;
        qa.d = d.head_dim;
        qa.kv_heads = d.kv_heads;
        qa.eps = d.eps;
        qa.trace = slot();
        qa.step_ctr = m->step_ctr;
        const bool spec = m->spec_mode != 0 && !m->q8 && !moe_on(m);
        if (spec) {
            qa.spec_router = reinterpret_cast<const uint16_t*>(L.router);
            qa.spec_ln = L.ln_moe;
            qa.spec_out = m->spec_logits;
            qa.spec_E = d.experts;
            if (m->spec_mode == 3) {
                qa.spec_ids = m->spec_ids;
                qa.spec_ticket = m->spec_ticket;
                qa.spec_k = d.k;
            }
        }
        if ((e = launch_qkv_rope(qa, s, pdl && l > 0)) != cudaSuccess) return e;
        if ((e = mark(pe, s, KK_QKV)) != cudaSuccess) return e;

        AttnArgs aa{};
        aa.q = m->q;
        aa.k_pool = L.k_pool;
        aa.v_pool = L.v_pool;
        aa.page_table = m->page_table;
        aa.page_size = kPageSize;
        aa.kv_f32 = qa.kv_f32;
        aa.pos = m->d_pos;
        aa.part_acc = m->part_acc;
        aa.part_ml = m->part_ml;
        aa.counters = m->attn_counters;
        aa.att_out = m->att;
        aa.err = m->d_err;
        aa.kv_heads = d.kv_heads;
        aa.G = m->G;
        aa.d = d.head_dim;
        aa.max_len = m->max_len;
        aa.splits = m->attn_splits;
        aa.split_cap = attn_split_cap(m->max_len, aa.splits);
        aa.merge = m->attn_merge == 0 ? 1 : 0;
        aa.cluster = m->attn_merge == 2 ? 1 : 0;
        aa.scale = d.attention_multiplier;
        aa.trace = slot();
        if (m->attn_tc) {
            BAttnArgs ba{};
            ba.q = m->q;
            ba.k_pool = L.k_pool;
            ba.v_pool = L.v_pool;
            ba.page_table = m->page_table;
            ba.pt_stride = m->max_pages;
            ba.page_size = kPageSize;
            ba.kv_f32 = 0;
            ba.pos = m->d_pos;
            ba.part_acc = m->part_acc;
            ba.part_ml = m->part_ml;
            ba.counters = m->attn_counters;
            ba.att_out = m->att;
            ba.err = m->d_err;
            ba.n = 1;
            ba.kv_heads = d.kv_heads;
            ba.G = m->G;
            ba.S = kAttnSplits;
            ba.scale = d.attention_multiplier;
            if ((e = launch_battention_tc(ba, &m->kvmaps[2 * l], &m->kvmaps[2 * l + 1], s)) != cudaSuccess) return e;
        } else {
            aa.tma = m->attn_tma && !aa.cluster ? 1 : 0;
            aa.mma = m->attn_mma && !aa.kv_f32 && !aa.cluster && m->G <= 8 ? 1 : 0;
            if (spec && m->spec_mode == 3 && !aa.tma && !aa.mma && !aa.kv_f32 && !aa.cluster) {
                aa.spec_ids = m->spec_ids;
                aa.spec_k = d.k;
                aa.spec_E = d.experts;
                aa.spec_gu = L.gate_up;
                aa.spec_dn = L.down;
                aa.spec_gu_bytes = (unsigned long long)2 * d.inter * wrow_bytes(d.hidden, m->q8);
                aa.spec_dn_bytes = (unsigned long long)d.hidden * wrow_bytes(d.inter, m->q8);
            }
            if ((e = launch_attention(aa, s, pdl, aa.tma ? &m->kvboxmaps[2 * l] : nullptr,
                                      aa.tma ? &m->kvboxmaps[2 * l + 1] : nullptr)) != cudaSuccess)
                return e;
        }
        if ((e = mark(pe, s, KK_ATTN)) != cudaSuccess) return e;

        OprojArgs oa{};
        oa.att = m->att;
        oa.w = L.wo;
        oa.q8 = m->q8;
        oa.h = m->h;
        oa.resid = d.residual_multiplier;
        oa.H = d.hidden;
        oa.qd = m->qd;
        oa.route = 1;
        oa.wr_t = L.wr_t;
        oa.shares = m->op_partial;
        oa.E = d.experts;
        oa.smem_weights = m->oproj_smem && !(!m->attn_tc && m->attn_merge == 1) ? 1 : 0;
        oa.err = m->d_err;
        if (!m->attn_tc && m->attn_merge == 1) {  // the attention left its per-split partials
            oa.part_acc = m->part_acc;
            oa.part_ml = m->part_ml;
            oa.splits = aa.splits;
            oa.heads = d.heads;
        }
        if (spec && m->spec_mode == 2) {
            oa.spec = m->spec_logits;
            oa.spec_E = d.experts;
            oa.spec_k = d.k;
            oa.spec_gu = L.gate_up;
            oa.spec_dn = L.down;
            oa.spec_gu_bytes = (unsigned long long)2 * d.inter * wrow_bytes(d.hidden, m->q8);
            oa.spec_dn_bytes = (unsigned long long)d.hidden * wrow_bytes(d.inter, m->q8);
        }
        oa.trace = slot();
        if ((e = launch_oproj(oa, s, pdl)) != cudaSuccess) return e;
        if ((e = mark(pe, s, KK_OPROJ)) != cudaSuccess) return e;

        if (moe_on(m)) {
            MoeArgs ma{};
            ma.h = m->h;
            ma.ln = L.ln_moe;
            ma.rs.shares = m->op_partial;
            ma.rs.nb = oproj_grid(d.hidden);
            ma.rs.eps = d.eps;
            ma.rs.ids_out = m->route_ids + (size_t)l * d.k;
            ma.rs.weights_out = m->route_w + (size_t)l * d.k;
            ma.rs.logits_out = m->rlogits;
            ma.w_gu = L.gate_up;
            ma.w_dn = L.down;
            ma.q8 = m->q8;
            ma.a = m->a;
            ma.barrier = m->moe_barrier;
            ma.err = m->d_err;
            ma.resid = d.residual_multiplier;
            ma.H = d.hidden;
            ma.I = d.inter;
            ma.k = d.k;
            ma.E = d.experts;
            ma.stages = m->moe.stages;
            ma.stage_bytes = m->moe.stage_bytes;
            ma.gu_chunk = m->moe.gu_chunk;
            ma.slots_per_chunk = m->moe.slots_per_chunk;
            if (l + 1 < d.layers) {  // L2 hint: the next layer's q/k/v and output-projection rows
                const LayerDev& N = m->L[l + 1];
                ma.pf[0] = N.wqkv;
                ma.pf_bytes[0] = (unsigned long long)(m->qd + 2 * m->kvd) * wrow_bytes(d.hidden, m->q8);
                ma.pf[1] = N.wo;
                ma.pf_bytes[1] = (unsigned long long)d.hidden * wrow_bytes(m->qd, m->q8);
            }
            ma.trace = slot();
            if ((e = launch_moe(ma, m->moe, s, pdl)) != cudaSuccess) return e;
            if ((e = mark(pe, s, KK_MOE)) != cudaSuccess) return e;
            continue;
        }

        RouteShares rs{};
        rs.shares = m->op_partial;
        rs.nb = oproj_grid(d.hidden);
        rs.eps = d.eps;
        rs.ids_out = m->route_ids + (size_t)l * d.k;
        rs.weights_out = m->route_w + (size_t)l * d.k;
        rs.logits_out = m->rlogits;

        GateUpArgs ga{};
        ga.x = m->h;
        ga.ln = L.ln_moe;
        ga.rs = rs;
        ga.w = L.gate_up;
        ga.q8 = m->q8;
        ga.a = m->a;
        ga.err = m->d_err;
        ga.H = d.hidden;
        ga.I = d.inter;
        ga.k = d.k;
        ga.E = d.experts;
        ga.down_w = m->gu_prefetch_down ? L.down : nullptr;
        ga.down_row_bytes = wrow_bytes(d.inter, m->q8);
        ga.spec = spec && m->spec_mode == 1 ? m->spec_logits : nullptr;
        if (m->route_handoff) {
            ga.route_flag = m->route_flags + l;
            ga.step_ctr = m->step_ctr;
        }
        ga.trace = slot();
        if ((e = launch_gate_up(ga, s, pdl)) != cudaSuccess) return e;
        if ((e = mark(pe, s, KK_GATE_UP)) != cudaSuccess) return e;

        DownArgs da{};
        da.a = m->a;
        da.rs = rs;
        da.w = L.down;
        da.q8 = m->q8;
        da.out = m->h;
        da.resid = d.residual_multiplier;
        da.accumulate = 1;
        da.err = m->d_err;
        da.H = d.hidden;
        da.I = d.inter;
        da.k = d.k;
        da.E = d.experts;
        if (l + 1 < d.layers) {  // L2 hint: the next layer's q/k/v and output-projection rows (C3: +1 %)
            const LayerDev& N = m->L[l + 1];
            da.pf[0] = N.wqkv;
            da.pf_bytes[0] = (unsigned long long)(m->qd + 2 * m->kvd) * wrow_bytes(d.hidden, m->q8);
            da.pf[1] = N.wo;
            da.pf_bytes[1] = (unsigned long long)d.hidden * wrow_bytes(m->qd, m->q8);
        }
        if (m->route_handoff) {
            da.route_flag = m->route_flags + l;
            da.step_ctr = m->step_ctr;
        }
        da.trace = slot();
        if ((e = launch_down(da, s, pdl)) != cudaSuccess) return e;
        if ((e = mark(pe, s, KK_DOWN)) != cudaSuccess) return e;
    }
    HeadArgs ha{};
    ha.h = m->h;
    ha.ln = m->norm;
    ha.eps = d.eps;
    ha.w = m->embed;
    ha.logits_scaling = d.logits_scaling;
    ha.logits_out = m->logits;
    ha.partial = m->head_partial;
    ha.counter = m->head_counter;
    ha.token_out = m->d_token;
    ha.out_ids = m->d_out_ids;
    ha.out_cap = m->max_len + 1;
    ha.step = m->d_step;
    ha.pos = m->d_pos;
    ha.V = d.vocab;
    ha.H = d.hidden;
    ha.trace = slot();
    if ((e = launch_head(ha, s, pdl, nullptr)) != cudaSuccess) return e;
    return mark(pe, s, KK_HEAD);
}

// one step on the stream: graph replay (captured at first use) or direct launches
int run_step(lastro_model* m) {
    cudaStream_t s = m->ctx->stream;
    if (!m->use_graphs) {
        MTRY(enqueue_step(m, s), "step launch");
        return LASTRO_OK;
    }
    if (!m->graph) {
        cudaGraph_t g = nullptr;
        MTRY(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal), "begin capture");
        cudaError_t e = enqueue_step(m, s);
        cudaError_t e2 = cudaStreamEndCapture(s, &g);
        if (e == cudaSuccess) e = e2;
        if (e != cudaSuccess) {
            if (g) cudaGraphDestroy(g);
            return model_fail(m, e, "step capture");
        }
        e = cudaGraphInstantiate(&m->graph, g, 0);
        cudaGraphDestroy(g);
        if (e != cudaSuccess) {
            m->graph = nullptr;
            return model_fail(m, e, "graph instantiate");
        }
    }
    MTRY(cudaGraphLaunch(m->graph, s), "graph launch");
    return LASTRO_OK;
}

// synchronize the stream and report a bounded wait that gave up inside a kernel (poisons the model)
int finish(lastro_model* m, const char* what) {
    cudaStream_t s = m->ctx->stream;
    MTRY(cudaMemcpyAsync(m->h_err, m->d_err, sizeof(int), cudaMemcpyDeviceToHost, s), what);
    MTRY(cudaStreamSynchronize(s), what);
    if (*m->h_err) {
        m->poisoned = true;
        return set_err(m->ctx, LASTRO_E_CUDA, "%s: a kernel wait gave up (code %d); model poisoned", what, *m->h_err);
    }
    return LASTRO_OK;
}

int check_ready(lastro_model* m) {
    if (m->poisoned) return set_err(m->ctx, LASTRO_E_POISONED, "model unusable after an earlier error");
    int rc = missing_tensor(m);
    if (rc) return rc;
    bool any = false;
    for (LayerDev& L : m->L)
        if (L.fold_dirty) {
            MTRY(launch_router_fold(L.router, m->q8, L.ln_moe, L.wr_t, m->d.experts, m->d.hidden, m->ctx->stream),
                 "router fold");
            L.fold_dirty = false;
            any = true;
        }
    if (any) MTRY(cudaStreamSynchronize(m->ctx->stream), "router fold");
    return LASTRO_OK;
}

// host copy of the paged layout's identity page table
int init_page_table(lastro_model* m) {
    std::vector<int> pt(m->max_pages);
    for (int i = 0; i < m->max_pages; ++i) pt[i] = i;
    MTRY(cudaMemcpyAsync(m->page_table, pt.data(), sizeof(int) * pt.size(), cudaMemcpyHostToDevice, m->ctx->stream),
         "page table");
    MTRY(cudaStreamSynchronize(m->ctx->stream), "page table");
    return LASTRO_OK;
}

}  // namespace

int lastro_capi::model_check_ready(lastro_model* m) { return check_ready(m); }

extern "C" int lastro_model_create(lastro_ctx* ctx, const lastro_model_desc* desc, int32_t max_len, lastro_model** out) {
    if (!ctx || !desc || !out) return LASTRO_E_ARG;
    *out = nullptr;
    const lastro_model_desc& d = *desc;
    if (d.layers < 1 || d.heads < 1 || d.kv_heads < 1 || d.vocab < 2 || max_len < 1)
        return set_err(ctx, LASTRO_E_ARG, "bad model description");
    if (d.heads % d.kv_heads) return set_err(ctx, LASTRO_E_ARG, "heads %d not a multiple of kv_heads %d", d.heads, d.kv_heads);
    if (d.head_dim != kHeadDim) return set_err(ctx, LASTRO_E_UNSUPPORTED, "head_dim %d (kernels implement %d)", d.head_dim, kHeadDim);
    const int G = d.heads / d.kv_heads;
    if (!(G == 1 || G == 2 || G == 3 || G == 4 || G == 6 || G == 8))
        return set_err(ctx, LASTRO_E_UNSUPPORTED, "GQA group %d", G);
    int rc = check_block_shape(ctx, d.experts, d.hidden, d.inter, d.k);
    if (rc) return rc;
    if (d.heads * d.head_dim > kMaxHidden) return set_err(ctx, LASTRO_E_UNSUPPORTED, "heads*head_dim > %d", kMaxHidden);
    if (d.weight_dtype != LASTRO_DTYPE_BF16 && d.weight_dtype != LASTRO_DTYPE_Q8_0)
        return set_err(ctx, LASTRO_E_UNSUPPORTED, "weight dtype %d", d.weight_dtype);
    if (d.weight_dtype == LASTRO_DTYPE_Q8_0 && (d.hidden % 32 || d.inter % 32 || (d.heads * d.head_dim) % 32))
        return set_err(ctx, LASTRO_E_UNSUPPORTED, "Q8_0 needs hidden, inter and heads*head_dim multiples of 32");
    if (d.weight_dtype == LASTRO_DTYPE_Q8_0 &&
        (gate_up_smem(d.hidden, 1) > kMaxSmemBytes || down_smem(d.hidden, d.inter, d.k, 1) > kMaxSmemBytes))
        return set_err(ctx, LASTRO_E_UNSUPPORTED, "Q8_0 expert tiles exceed shared memory");
    if (d.kv_dtype != LASTRO_DTYPE_BF16 && d.kv_dtype != LASTRO_DTYPE_F32)
        return set_err(ctx, LASTRO_E_UNSUPPORTED, "kv dtype %d", d.kv_dtype);
    if (!(d.eps >= 0.0f) || !(d.logits_scaling != 0.0f) || !(d.rope_theta > 0.0f))
        return set_err(ctx, LASTRO_E_ARG, "bad eps / logits_scaling / rope_theta");
    if (attn_smem(max_len, d.kv_dtype == LASTRO_DTYPE_F32, kAttnSplits) > kMaxSmemBytes)
        return set_err(ctx, LASTRO_E_UNSUPPORTED, "max_len %d: the attention CTAs cannot stage their K/V share", max_len);

    cudaSetDevice(ctx->device);
    lastro_model* m = new lastro_model();
    m->ctx = ctx;
    m->d = d;
    m->max_len = max_len;
    m->qd = d.heads * d.head_dim;
    m->kvd = d.kv_heads * d.head_dim;
    m->G = G;
    m->q8 = d.weight_dtype == LASTRO_DTYPE_Q8_0;
    m->max_pages = (max_len + kPageSize - 1) / kPageSize;
    m->head_grid = head_grid(d.vocab);
    m->loaded.assign((size_t)(d.layers + 1) * K_COUNT, 0);
    m->L.resize(d.layers);
    const size_t H = d.hidden, I = d.inter, E = d.experts, V = d.vocab;
    const size_t kvpool = (size_t)m->max_pages * d.kv_heads * kPageSize * d.head_dim * kv_elem_bytes(m);
    Arena& A = m->arena;
    bool bad = A.alloc(&m->embed, V * H) || A.alloc(&m->norm, H);
    for (int l = 0; l < d.layers && !bad; ++l) {
        LayerDev& L = m->L[l];
        const size_t rbh = wrow_bytes((int)H, m->q8), rbq = wrow_bytes(m->qd, m->q8), rbi = wrow_bytes((int)I, m->q8);
        bad = A.alloc(&L.ln_attn, H) || A.alloc(&L.ln_moe, H) || A.alloc(&L.wqkv, (size_t)(m->qd + 2 * m->kvd) * rbh) ||
              A.alloc(&L.wo, H * rbq) || A.alloc(&L.router, E * rbh) || A.alloc(&L.gate_up, E * 2 * I * rbh) ||
              A.alloc(&L.down, E * H * rbi) || A.alloc(&L.k_pool, kvpool) || A.alloc(&L.v_pool, kvpool) ||
              A.alloc(&L.wr_t, E * H);
    }
    bad = bad || A.alloc(&m->rope_cs, (size_t)max_len * d.head_dim) || A.alloc(&m->page_table, m->max_pages) ||
          A.alloc(&m->h, H) || A.alloc(&m->q, m->qd) || A.alloc(&m->att, m->qd) || A.alloc(&m->rlogits, E) || A.alloc(&m->spec_logits, E) ||
          A.alloc(&m->part_acc, (size_t)d.heads * kAttnSplits * d.head_dim) ||
          A.alloc(&m->part_ml, (size_t)d.heads * kAttnSplits * 2) ||
          A.alloc(&m->route_w, (size_t)d.layers * d.k) || A.alloc(&m->route_ids, (size_t)d.layers * d.k) ||
          A.alloc(&m->rnorm, 1) || A.alloc(&m->a, (size_t)d.k * I) || A.alloc(&m->logits, V) ||
          A.alloc(&m->d_token, 2) || A.alloc(&m->d_pos, 1) || A.alloc(&m->d_step, 1) ||
          A.alloc(&m->d_out_ids, (size_t)max_len + 1) || A.alloc(&m->d_prompt, (size_t)max_len + 1) ||
          A.alloc(&m->router_counter, 1) || A.alloc(&m->head_counter, 1) || A.alloc(&m->attn_counters, d.kv_heads) ||
          A.alloc(&m->head_partial, m->head_grid) ||
          A.alloc(&m->op_partial, (size_t)oproj_grid(d.hidden) * (E + 1)) || A.alloc(&m->moe_barrier, 1) ||
          A.alloc(&m->step_ctr, 1) || A.alloc(&m->route_flags, (size_t)d.layers) ||
          A.alloc(&m->spec_ids, kMaxTopK) || A.alloc(&m->spec_ticket, 1);
    m->moe_ok = !bad && moe_plan(d.hidden, d.inter, d.k, m->q8, &m->moe);
    // the fused step: one CTA per SM, when the per-CTA shares of every phase fit in shared memory
    int n_sm = 0, coop = 0;
    if (cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, ctx->device) != cudaSuccess ||
        cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, ctx->device) != cudaSuccess) {
        cudaGetLastError();
        n_sm = 0;
    }
    if (!bad && n_sm > 0 && coop && !m->q8 &&
        fused_plan(d.hidden, d.inter, d.experts, d.k, m->qd, m->kvd, d.kv_heads, G, d.vocab,
                   d.kv_dtype == LASTRO_DTYPE_F32, n_sm, &m->flay)) {
        int per_sm = 0;
        if (fused_blocks_per_sm(d.hidden, m->qd, d.inter, d.kv_dtype == LASTRO_DTYPE_F32, m->flay.smem, &per_sm) !=
            cudaSuccess)
            cudaGetLastError();
        m->fused_ok = per_sm >= 1;
    }
    const size_t n_qkv = (size_t)m->qd + 2 * m->kvd, n_part = (size_t)d.heads * m->flay.max_splits * kPartStride,
                 n_share = (size_t)m->flay.nb * (E + 1);
    if (m->fused_ok)
        bad = bad || A.alloc(&m->f_layers, (size_t)d.layers) || A.alloc(&m->f_ticket, 1) || A.alloc(&m->f_epoch, 1) ||
              A.alloc(&m->f_count, (size_t)kExchangeKinds * kCountStride) ||
              A.alloc(&m->fx.h, H) || A.alloc(&m->fx.qkv, n_qkv) || A.alloc(&m->fx.part, n_part) ||
              A.alloc(&m->fx.att, (size_t)m->qd) || A.alloc(&m->fx.share, n_share) || A.alloc(&m->fx.act, (size_t)d.k * I) ||
              A.alloc(&m->f_best, (size_t)m->flay.nb);
    if (bad || cudaMallocHost(&m->h_token, 2 * sizeof(int)) != cudaSuccess) {
        cudaGetLastError();
        A.release();
        delete m;
        return set_err(ctx, LASTRO_E_NOMEM, "model allocation failed");
    }
    cudaStream_t s = ctx->stream;
    cudaError_t e = cudaSuccess;
    for (int l = 0; l < d.layers && !e; ++l) {
        e = cudaMemsetAsync(m->L[l].k_pool, 0, kvpool, s);
        if (!e) e = cudaMemsetAsync(m->L[l].v_pool, 0, kvpool, s);
    }
    // the token and the error word sit side by side on both sides: a step reads both back in one copy
    m->h_err = m->h_token + 1;
    m->d_err = m->d_token + 1;
    for (void* p : {(void*)m->router_counter, (void*)m->head_counter, (void*)m->d_pos, (void*)m->d_step,
                    (void*)m->d_token, (void*)m->d_err})
        if (!e) e = cudaMemsetAsync(p, 0, sizeof(int), s);
    if (!e) e = cudaMemsetAsync(m->attn_counters, 0, sizeof(unsigned) * d.kv_heads, s);
    if (!e) e = cudaMemsetAsync(m->moe_barrier, 0, sizeof(unsigned long long), s);
    if (!e) e = cudaMemsetAsync(m->step_ctr, 0, sizeof(unsigned int), s);
    if (!e) e = cudaMemsetAsync(m->spec_ticket, 0, sizeof(unsigned int), s);
    if (!e) e = cudaMemsetAsync(m->spec_ids, 0, sizeof(int) * kMaxTopK, s);
    if (!e) e = cudaMemsetAsync(m->route_flags, 0, sizeof(unsigned int) * (size_t)d.layers, s);
    std::vector<FusedLayer> fl;
    if (m->fused_ok) {
        // tag 0 is never written: zeroed exchange words never match a wait
        if (!e) e = cudaMemsetAsync(m->f_ticket, 0, sizeof(unsigned), s);
        if (!e) e = cudaMemsetAsync(m->f_count, 0, sizeof(unsigned) * kExchangeKinds * kCountStride, s);
        if (!e) e = cudaMemsetAsync(m->f_epoch, 0, sizeof(unsigned), s);
        const std::pair<unsigned long long*, size_t> words[] = {{m->fx.h, H}, {m->fx.qkv, n_qkv}, {m->fx.part, n_part},
                                                                {m->fx.att, (size_t)m->qd}, {m->fx.share, n_share},
                                                                {m->fx.act, (size_t)d.k * I}};
        for (const auto& w : words)
            if (!e) e = cudaMemsetAsync(w.first, 0, w.second * sizeof(unsigned long long), s);
        for (int l = 0; l < d.layers; ++l) {
            const LayerDev& L = m->L[l];
            fl.push_back(FusedLayer{L.ln_attn, L.ln_moe, L.wr_t, reinterpret_cast<const uint16_t*>(L.wqkv),
                                    reinterpret_cast<const uint16_t*>(L.wo), reinterpret_cast<const uint16_t*>(L.gate_up),
                                    reinterpret_cast<const uint16_t*>(L.down), L.k_pool, L.v_pool});
        }
        if (!e) e = cudaMemcpyAsync(m->f_layers, fl.data(), sizeof(FusedLayer) * fl.size(), cudaMemcpyHostToDevice, s);
    }
    if (!e) e = cudaMemsetAsync(m->route_ids, 0, sizeof(int) * d.layers * d.k, s);
    if (!e) e = cudaMemsetAsync(m->route_w, 0, sizeof(float) * d.layers * d.k, s);
    const std::vector<float> cs = rope_table(d, max_len);
    if (!e) e = cudaMemcpyAsync(m->rope_cs, cs.data(), sizeof(float) * cs.size(), cudaMemcpyHostToDevice, s);
    if (!e) e = cudaStreamSynchronize(s);
    if (e) {
        cudaGetLastError();
        A.release();
        cudaFreeHost(m->h_token);
        delete m;
        return set_err(ctx, LASTRO_E_CUDA, "model init: %s", cudaGetErrorString(e));
    }
    if (init_page_table(m)) {
        A.release();
        cudaFreeHost(m->h_token);
        delete m;
        return LASTRO_E_CUDA;
    }
    if (d.kv_dtype == LASTRO_DTYPE_BF16 && m->G <= 8) {  // TMA page maps for the tensor-core attention
        const uint64_t rows = (uint64_t)m->max_pages * d.kv_heads * kPageSize;
        m->kvmaps.resize((size_t)d.layers * 2);
        bool ok = true;
        for (int l = 0; l < d.layers && ok; ++l)
            ok = make_kv_map(&m->kvmaps[2 * l], m->L[l].k_pool, rows) == cudaSuccess &&
                 make_kv_map(&m->kvmaps[2 * l + 1], m->L[l].v_pool, rows) == cudaSuccess;
        if (!ok) {
            cudaGetLastError();
            m->kvmaps.clear();
        }
        m->kvboxmaps.resize((size_t)d.layers * 2);
        ok = kPageSize % 8 == 0 && d.head_dim == 64;
        for (int l = 0; l < d.layers && ok; ++l)
            ok = make_kv_box_map(&m->kvboxmaps[2 * l], m->L[l].k_pool, rows) == cudaSuccess &&
                 make_kv_box_map(&m->kvboxmaps[2 * l + 1], m->L[l].v_pool, rows) == cudaSuccess;
        if (!ok) {
            cudaGetLastError();
            m->kvboxmaps.clear();
        }
        m->attn_tma = false;  // the boxes measure slower than one bulk copy per page run on C3 (LASTRO_TUNE_ATTN_TMA)
        // off by default: at batch 1 (16 splits, one token) the CUDA-core kernel, whose split merge is one round of
        // loads and shuffles, measures faster on B200 (C3: 16.4 vs 13 us per launch)
        m->attn_tc = false;
    }
    m->spec_mode = 0;  // both forms measure even with the plain chain on C3 (gate_up gains what oproj/down lose)
    ctx_retain(ctx);
    *out = m;
    return LASTRO_OK;
}

extern "C" int lastro_model_load_tensor(lastro_model* m, const char* name, int32_t dtype, const int64_t* shape,
                                        int32_t ndim, const void* host) {
    if (!m) return LASTRO_E_ARG;
    lastro_ctx* ctx = m->ctx;
    if (m->poisoned) return set_err(ctx, LASTRO_E_POISONED, "model unusable after an earlier error");
    if (!name || !host || (!shape && ndim > 0)) return set_err(ctx, LASTRO_E_ARG, "null argument");
    const lastro_model_desc& d = m->d;
    const int64_t H = d.hidden, I = d.inter, E = d.experts, V = d.vocab, qd = m->qd, kvd = m->kvd;
    int layer = -1, kind = -1;
    const char* rest = nullptr;
    if (!strcmp(name, kind_name(K_EMBED)))
        kind = K_EMBED;
    else if (!strcmp(name, kind_name(K_NORM)))
        kind = K_NORM;
    else if (!strncmp(name, "model.layers.", 13)) {
        char* endp = nullptr;
        long l = strtol(name + 13, &endp, 10);
        if (endp == name + 13 || *endp != '.' || l < 0 || l >= d.layers)
            return set_err(ctx, LASTRO_E_ARG, "tensor %s: bad layer index", name);
        layer = (int)l;
        rest = endp + 1;
        for (int k = K_LN_ATTN; k < K_COUNT; ++k)
            if (!strcmp(rest, kind_name(k))) kind = k;
    }
    if (kind < 0) return set_err(ctx, LASTRO_E_ARG, "unknown tensor %s", name);
    std::vector<int64_t> want;
    void* dst = nullptr;
    bool is_norm = false;
    const LayerDev* L = layer >= 0 ? &m->L[layer] : nullptr;
    switch (kind) {
    case K_EMBED: want = {V, H}; dst = m->embed; break;
    case K_NORM: want = {H}; dst = m->norm; is_norm = true; break;
    case K_LN_ATTN: want = {H}; dst = L->ln_attn; is_norm = true; break;
    case K_LN_MOE: want = {H}; dst = L->ln_moe; is_norm = true; break;
    case K_Q: want = {qd, H}; dst = L->wqkv; break;
    case K_K: want = {kvd, H}; dst = L->wqkv + (size_t)qd * wrow_bytes((int)H, m->q8); break;
    case K_V: want = {kvd, H}; dst = L->wqkv + (size_t)(qd + kvd) * wrow_bytes((int)H, m->q8); break;
    case K_O: want = {H, qd}; dst = L->wo; break;
    case K_ROUTER: want = {E, H}; dst = L->router; break;
    case K_GATE_UP: want = {E, 2 * I, H}; dst = L->gate_up; break;
    case K_DOWN: want = {E, H, I}; dst = L->down; break;
    }
    bool shape_ok = ndim == (int32_t)want.size();
    for (int i = 0; shape_ok && i < ndim; ++i) shape_ok = shape[i] == want[i];
    if (!shape_ok) return set_err(ctx, LASTRO_E_ARG, "tensor %s: unexpected shape", name);
    size_t n = 1;
    for (int64_t v : want) n *= (size_t)v;
    cudaSetDevice(ctx->device);
    cudaStream_t s = ctx->stream;
    if (is_norm) {
        std::vector<float> f(n);
        if (dtype == LASTRO_DTYPE_BF16) {
            const uint16_t* b = static_cast<const uint16_t*>(host);
            for (size_t i = 0; i < n; ++i) {
                uint32_t u = (uint32_t)b[i] << 16;
                memcpy(&f[i], &u, 4);
            }
        } else if (dtype == LASTRO_DTYPE_F32) {
            memcpy(f.data(), host, n * 4);
        } else {
            return set_err(ctx, LASTRO_E_ARG, "tensor %s: dtype %d", name, dtype);
        }
        MTRY(cudaMemcpyAsync(dst, f.data(), n * 4, cudaMemcpyHostToDevice, s), "tensor upload");
        MTRY(cudaStreamSynchronize(s), "tensor upload");
    } else if (m->q8 && kind != K_EMBED) {
        // Q8_0 linear: host blocks of 34 bytes (fp16 scale, 32 int8 values) along each row, repacked into the device
        // row layout (the row's values, then its scales)
        if (dtype != LASTRO_DTYPE_Q8_0) return set_err(ctx, LASTRO_E_ARG, "tensor %s: dtype %d (Q8_0 expected)", name, dtype);
        const int cols = (int)want.back();
        const std::vector<unsigned char> buf = repack_q8_rows(static_cast<const unsigned char*>(host), n / (size_t)cols, cols);
        MTRY(cudaMemcpyAsync(dst, buf.data(), buf.size(), cudaMemcpyHostToDevice, s), "tensor upload");
        MTRY(cudaStreamSynchronize(s), "tensor upload");
    } else {
        if (dtype != LASTRO_DTYPE_BF16) return set_err(ctx, LASTRO_E_ARG, "tensor %s: dtype %d (bf16 expected)", name, dtype);
        MTRY(cudaMemcpyAsync(dst, host, n * 2, cudaMemcpyHostToDevice, s), "tensor upload");
        MTRY(cudaStreamSynchronize(s), "tensor upload");
    }
    loaded_flag(m, layer, kind) = 1;
    if (layer >= 0 && (kind == K_ROUTER || kind == K_LN_MOE)) m->L[layer].fold_dirty = true;
    return LASTRO_OK;
}

extern "C" int lastro_model_fill_synthetic(lastro_model* m, uint64_t seed, float sd, float norm_sd) {
    if (!m) return LASTRO_E_ARG;
    lastro_ctx* ctx = m->ctx;
    if (m->poisoned) return set_err(ctx, LASTRO_E_POISONED, "model unusable after an earlier error");
    cudaSetDevice(ctx->device);
    cudaStream_t s = ctx->stream;
    const lastro_model_desc& d = m->d;
    const size_t H = d.hidden, I = d.inter, E = d.experts, V = d.vocab, qd = m->qd, kvd = m->kvd;
    const float sc = synth_scale(sd), nsc = synth_scale(norm_sd);
    MTRY(launch_synth_bf16(m->embed, V * H, tensor_seed(seed, -1, K_EMBED), sc, 0.0f, s), "synth");
    MTRY(launch_synth_norm_f32(m->norm, H, tensor_seed(seed, -1, K_NORM), nsc, s), "synth");
    for (int l = 0; l < d.layers; ++l) {
        LayerDev& L = m->L[l];
        MTRY(launch_synth_norm_f32(L.ln_attn, H, tensor_seed(seed, l, K_LN_ATTN), nsc, s), "synth");
        MTRY(launch_synth_norm_f32(L.ln_moe, H, tensor_seed(seed, l, K_LN_MOE), nsc, s), "synth");
        if (m->q8) {
            // int8 ~U[-127, 127], fp16 scales ~U(1e-4, 4e-3), the oracle's generator
            const size_t rbh = wrow_bytes((int)H, 1);
            MTRY(launch_synth_q8_0(L.wqkv, qd, (int)H, tensor_seed(seed, l, K_Q), s), "synth");
            MTRY(launch_synth_q8_0(L.wqkv + qd * rbh, kvd, (int)H, tensor_seed(seed, l, K_K), s), "synth");
            MTRY(launch_synth_q8_0(L.wqkv + (qd + kvd) * rbh, kvd, (int)H, tensor_seed(seed, l, K_V), s), "synth");
            MTRY(launch_synth_q8_0(L.wo, H, (int)qd, tensor_seed(seed, l, K_O), s), "synth");
            MTRY(launch_synth_q8_0(L.router, E, (int)H, tensor_seed(seed, l, K_ROUTER), s), "synth");
            MTRY(launch_synth_q8_0(L.gate_up, E * 2 * I, (int)H, tensor_seed(seed, l, K_GATE_UP), s), "synth");
            MTRY(launch_synth_q8_0(L.down, E * H, (int)I, tensor_seed(seed, l, K_DOWN), s), "synth");
            continue;
        }
        uint16_t *wqkv = reinterpret_cast<uint16_t*>(L.wqkv), *wo = reinterpret_cast<uint16_t*>(L.wo);
        MTRY(launch_synth_bf16(wqkv, qd * H, tensor_seed(seed, l, K_Q), sc, 0.0f, s), "synth");
        MTRY(launch_synth_bf16(wqkv + qd * H, kvd * H, tensor_seed(seed, l, K_K), sc, 0.0f, s), "synth");
        MTRY(launch_synth_bf16(wqkv + (qd + kvd) * H, kvd * H, tensor_seed(seed, l, K_V), sc, 0.0f, s), "synth");
        MTRY(launch_synth_bf16(wo, H * qd, tensor_seed(seed, l, K_O), sc, 0.0f, s), "synth");
        MTRY(launch_synth_bf16(reinterpret_cast<uint16_t*>(L.router), E * H, tensor_seed(seed, l, K_ROUTER), sc, 0.0f, s),
             "synth");
        MTRY(launch_synth_bf16(reinterpret_cast<uint16_t*>(L.gate_up), E * 2 * I * H, tensor_seed(seed, l, K_GATE_UP), sc,
                               0.0f, s),
             "synth");
        MTRY(launch_synth_bf16(reinterpret_cast<uint16_t*>(L.down), E * H * I, tensor_seed(seed, l, K_DOWN), sc, 0.0f, s),
             "synth");
    }
    MTRY(cudaStreamSynchronize(s), "synth");
    std::fill(m->loaded.begin(), m->loaded.end(), 1);
    for (LayerDev& L : m->L) L.fold_dirty = true;
    return LASTRO_OK;
}

extern "C" int lastro_model_fill_kv_synthetic(lastro_model* m, int32_t n, uint64_t seed, float sd) {
    if (!m) return LASTRO_E_ARG;
    lastro_ctx* ctx = m->ctx;
    if (m->poisoned) return set_err(ctx, LASTRO_E_POISONED, "model unusable after an earlier error");
    if (n < 0 || n > m->max_len) return set_err(ctx, LASTRO_E_ARG, "fill_kv_synthetic: %d positions (max_len %d)", n, m->max_len);
    cudaSetDevice(ctx->device);
    cudaStream_t s = ctx->stream;
    const lastro_model_desc& d = m->d;
    const float sc = synth_scale(sd);
    const int f32 = d.kv_dtype == LASTRO_DTYPE_F32;
    // layer l's K and V streams are seeded mix64(seed + 2l) and mix64(seed + 2l + 1), as the CPU oracle's fill
    for (int l = 0; l < d.layers; ++l) {
        const uint64_t sk = mix64_host(seed + 2 * (uint64_t)l), sv = mix64_host(seed + 2 * (uint64_t)l + 1);
        MTRY(launch_synth_kv_pages(m->L[l].k_pool, f32, m->page_table, n, d.kv_heads, d.head_dim, kPageSize, sk, sc, s),
             "kv fill");
        MTRY(launch_synth_kv_pages(m->L[l].v_pool, f32, m->page_table, n, d.kv_heads, d.head_dim, kPageSize, sv, sc, s),
             "kv fill");
    }
    MTRY(cudaMemcpyAsync(m->d_pos, &n, sizeof(int), cudaMemcpyHostToDevice, s), "kv fill");
    MTRY(cudaMemsetAsync(m->d_step, 0, sizeof(int), s), "kv fill");
    MTRY(cudaStreamSynchronize(s), "kv fill");
    m->pos_host = n;
    return LASTRO_OK;
}

extern "C" int lastro_model_read_kv(lastro_model* m, int32_t layer, int32_t pos0, int32_t n, float* k_out, float* v_out) {
    if (!m) return LASTRO_E_ARG;
    lastro_ctx* ctx = m->ctx;
    if (m->poisoned) return set_err(ctx, LASTRO_E_POISONED, "model unusable after an earlier error");
    const lastro_model_desc& d = m->d;
    if (layer < 0 || layer >= d.layers || pos0 < 0 || n < 0 || (int64_t)pos0 + n > m->pos_host)
        return set_err(ctx, LASTRO_E_ARG, "read_kv: layer %d, positions [%d, %d) of %d", layer, pos0, pos0 + n,
                       m->pos_host);
    if (n == 0) return LASTRO_OK;
    cudaSetDevice(ctx->device);
    cudaStream_t s = ctx->stream;
    const int ps = kPageSize, dh = d.head_dim, kvh = d.kv_heads;
    const size_t eb = kv_elem_bytes(m), page_elems = (size_t)kvh * ps * dh;
    const int pg0 = pos0 / ps, pg1 = (pos0 + n - 1) / ps;
    std::vector<int> pt(pg1 + 1);
    MTRY(cudaMemcpyAsync(pt.data(), m->page_table, sizeof(int) * pt.size(), cudaMemcpyDeviceToHost, s), "read_kv");
    MTRY(cudaStreamSynchronize(s), "read_kv");
    std::vector<unsigned char> buf(page_elems * eb);
    for (int which = 0; which < 2; ++which) {
        float* out = which ? v_out : k_out;
        if (!out) continue;
        const unsigned char* pool = static_cast<const unsigned char*>(which ? m->L[layer].v_pool : m->L[layer].k_pool);
        for (int pg = pg0; pg <= pg1; ++pg) {
            MTRY(cudaMemcpyAsync(buf.data(), pool + (size_t)pt[pg] * page_elems * eb, buf.size(), cudaMemcpyDeviceToHost, s),
                 "read_kv");
            MTRY(cudaStreamSynchronize(s), "read_kv");
            for (int p = std::max(pos0, pg * ps); p < std::min(pos0 + n, (pg + 1) * ps); ++p)
                for (int h = 0; h < kvh; ++h)
                    for (int j = 0; j < dh; ++j) {
                        const size_t src = ((size_t)h * ps + (p - pg * ps)) * dh + j;
                        float v;
                        if (eb == 4) {
                            memcpy(&v, buf.data() + src * 4, 4);
                        } else {
                            uint16_t b;
                            memcpy(&b, buf.data() + src * 2, 2);
                            const uint32_t u = (uint32_t)b << 16;
                            memcpy(&v, &u, 4);
                        }
                        out[(size_t)(p - pos0) * kvh * dh + (size_t)h * dh + j] = v;
                    }
        }
    }
    return LASTRO_OK;
}

extern "C" int lastro_model_step(lastro_model* m, int32_t token, float* logits, int32_t* next_token, int32_t* route_ids,
                                 float* route_weights) {
    if (!m) return LASTRO_E_ARG;
    lastro_ctx* ctx = m->ctx;
    int rc = check_ready(m);
    if (rc) return rc;
    // gpu_model.rs:252-257: refused before any launch, the model stays usable
    if (m->pos_host >= m->max_len) return set_err(ctx, LASTRO_E_FULL, "KV cache full (%d positions)", m->max_len);
    if (token < 0 || token >= m->d.vocab) return set_err(ctx, LASTRO_E_ARG, "token %d outside the vocabulary (%d)", token, m->d.vocab);
    cudaSetDevice(ctx->device);
    cudaStream_t s = ctx->stream;
    *m->h_token = token;
    MTRY(cudaMemcpyAsync(m->d_token, m->h_token, sizeof(int), cudaMemcpyHostToDevice, s), "token upload");
    rc = run_step(m);
    if (rc) return rc;
    const lastro_model_desc& d = m->d;
    if (logits) MTRY(cudaMemcpyAsync(logits, m->logits, sizeof(float) * d.vocab, cudaMemcpyDeviceToHost, s), "logits");
    if (route_ids)
        MTRY(cudaMemcpyAsync(route_ids, m->route_ids, sizeof(int) * d.layers * d.k, cudaMemcpyDeviceToHost, s), "routes");
    if (route_weights)
        MTRY(cudaMemcpyAsync(route_weights, m->route_w, sizeof(float) * d.layers * d.k, cudaMemcpyDeviceToHost, s), "routes");
    // the next token and the error word in one copy into pinned memory (the token upload above read it first)
    MTRY(cudaMemcpyAsync(m->h_token, m->d_token, 2 * sizeof(int), cudaMemcpyDeviceToHost, s), "step");
    MTRY(cudaStreamSynchronize(s), "step");
    if (*m->h_err) {
        m->poisoned = true;
        return set_err(ctx, LASTRO_E_CUDA, "step: a kernel wait gave up (code %d); model poisoned", *m->h_err);
    }
    if (next_token) *next_token = m->h_token[0];
    m->pos_host += 1;
    return LASTRO_OK;
}

extern "C" int lastro_model_generate(lastro_model* m, const int32_t* prompt, int32_t n_prompt, int32_t n_new,
                                     int32_t* out_ids) {
    if (!m) return LASTRO_E_ARG;
    lastro_ctx* ctx = m->ctx;
    int rc = check_ready(m);
    if (rc) return rc;
    if (n_prompt < 1 || n_new < 0 || !prompt) return set_err(ctx, LASTRO_E_ARG, "generate needs a prompt");
    for (int i = 0; i < n_prompt; ++i)
        if (prompt[i] < 0 || prompt[i] >= m->d.vocab) return set_err(ctx, LASTRO_E_ARG, "prompt token %d out of range", prompt[i]);
    const int steps = n_prompt + (n_new > 0 ? n_new - 1 : 0);
    if (m->pos_host + steps > m->max_len) return set_err(ctx, LASTRO_E_FULL, "generate would overflow the KV cache");
    cudaSetDevice(ctx->device);
    cudaStream_t s = ctx->stream;
    MTRY(cudaMemcpyAsync(m->d_prompt, prompt, sizeof(int) * n_prompt, cudaMemcpyHostToDevice, s), "prompt upload");
    MTRY(cudaMemsetAsync(m->d_step, 0, sizeof(int), s), "step reset");
    for (int i = 0; i < n_prompt; ++i) {
        MTRY(cudaMemcpyAsync(m->d_token, m->d_prompt + i, sizeof(int), cudaMemcpyDeviceToDevice, s), "token");
        rc = run_step(m);
        if (rc) return rc;
    }
    for (int i = 1; i < n_new; ++i) {
        rc = run_step(m);
        if (rc) return rc;
    }
    if (out_ids && n_new > 0)
        MTRY(cudaMemcpyAsync(out_ids, m->d_out_ids + (n_prompt - 1), sizeof(int) * n_new, cudaMemcpyDeviceToHost, s),
             "ids download");
    rc = finish(m, "generate");
    if (rc) return rc;
    m->pos_host += steps;
    return LASTRO_OK;
}

extern "C" int lastro_model_generate_until(lastro_model* m, const int32_t* prompt, int32_t n_prompt, int32_t n_new,
                                           int32_t eos, int32_t* out_ids, int32_t* n_out) {
    if (!m) return LASTRO_E_ARG;
    lastro_ctx* ctx = m->ctx;
    int rc = check_ready(m);
    if (rc) return rc;
    if (n_prompt < 1 || n_new < 1 || !prompt || !out_ids || !n_out)
        return set_err(ctx, LASTRO_E_ARG, "generate_until needs a prompt, n_new >= 1 and both outputs");
    if (eos >= m->d.vocab) return set_err(ctx, LASTRO_E_ARG, "eos %d out of range", eos);
    for (int i = 0; i < n_prompt; ++i)
        if (prompt[i] < 0 || prompt[i] >= m->d.vocab) return set_err(ctx, LASTRO_E_ARG, "prompt token %d out of range", prompt[i]);
    if (m->pos_host + n_prompt + n_new - 1 > m->max_len)
        return set_err(ctx, LASTRO_E_FULL, "generate would overflow the KV cache");
    cudaSetDevice(ctx->device);
    cudaStream_t s = ctx->stream;
    const int start = m->pos_host;
    MTRY(cudaMemcpyAsync(m->d_prompt, prompt, sizeof(int) * n_prompt, cudaMemcpyHostToDevice, s), "prompt upload");
    MTRY(cudaMemsetAsync(m->d_step, 0, sizeof(int), s), "step reset");
    for (int i = 0; i < n_prompt; ++i) {
        MTRY(cudaMemcpyAsync(m->d_token, m->d_prompt + i, sizeof(int), cudaMemcpyDeviceToDevice, s), "token");
        rc = run_step(m);
        if (rc) return rc;
    }
    // generated token i sits at d_out_ids[n_prompt - 1 + i]; steps run in chunks, each chunk's ids read back once, so
    // the host sees an end of text at most kChunk - 1 steps late; the position is then rolled back to the reference's
    // (geracao_regra.rs:230-245: the end-of-text token is emitted, never fed)
    constexpr int kChunk = 16;
    int produced = 1, done = 0;  // the prompt's last step produced token 0
    while (true) {
        MTRY(cudaMemcpyAsync(out_ids + done, m->d_out_ids + (n_prompt - 1) + done, sizeof(int) * (produced - done),
                             cudaMemcpyDeviceToHost, s),
             "ids download");
        rc = finish(m, "generate");
        if (rc) return rc;
        int stop = -1;
        if (eos >= 0)
            for (int i = done; i < produced; ++i)
                if (out_ids[i] == eos) {
                    stop = i;
                    break;
                }
        if (stop >= 0 || produced == n_new) {
            const int n = stop >= 0 ? stop + 1 : produced;
            const int pos = start + n_prompt + n - 1;  // prompt and the generated tokens before the last one were fed
            *n_out = n;
            if (pos != start + n_prompt + produced - 1) {
                MTRY(cudaMemcpyAsync(m->d_pos, &pos, sizeof(int), cudaMemcpyHostToDevice, s), "position rollback");
                MTRY(cudaMemcpyAsync(m->d_token, out_ids + n - 1, sizeof(int), cudaMemcpyHostToDevice, s), "token");
                MTRY(cudaStreamSynchronize(s), "position rollback");
            }
            m->pos_host = pos;
            return LASTRO_OK;
        }
        done = produced;
        const int run = std::min(kChunk, n_new - produced);
        for (int i = 0; i < run; ++i) {
            rc = run_step(m);
            if (rc) return rc;
        }
        produced += run;
    }
}

extern "C" int lastro_model_decode(lastro_model* m, int32_t n) {
    if (!m) return LASTRO_E_ARG;
    lastro_ctx* ctx = m->ctx;
    int rc = check_ready(m);
    if (rc) return rc;
    if (n < 0) return set_err(ctx, LASTRO_E_ARG, "negative step count");
    if (m->pos_host + n > m->max_len) return set_err(ctx, LASTRO_E_FULL, "decode would overflow the KV cache");
    cudaSetDevice(ctx->device);
    MTRY(cudaMemsetAsync(m->d_step, 0, sizeof(int), ctx->stream), "step reset");
    for (int i = 0; i < n; ++i) {
        rc = run_step(m);
        if (rc) return rc;
    }
    rc = finish(m, "decode");
    if (rc) return rc;
    m->pos_host += n;
    return LASTRO_OK;
}

extern "C" int lastro_model_reset(lastro_model* m) {
    if (!m) return LASTRO_E_ARG;
    if (m->poisoned) return set_err(m->ctx, LASTRO_E_POISONED, "model unusable after an earlier error");
    cudaSetDevice(m->ctx->device);
    cudaStream_t s = m->ctx->stream;
    MTRY(cudaMemsetAsync(m->d_pos, 0, sizeof(int), s), "reset");
    MTRY(cudaMemsetAsync(m->d_step, 0, sizeof(int), s), "reset");
    MTRY(cudaStreamSynchronize(s), "reset");
    m->pos_host = 0;
    return init_page_table(m);
}

extern "C" int lastro_model_position(const lastro_model* m, int32_t* pos) {
    if (!m || !pos) return LASTRO_E_ARG;
    *pos = m->pos_host;
    return LASTRO_OK;
}

extern "C" int lastro_model_profile(lastro_model* m, int32_t steps, float* kernel_ms, int32_t n_kinds) {
    if (!m) return LASTRO_E_ARG;
    lastro_ctx* ctx = m->ctx;
    int rc = check_ready(m);
    if (rc) return rc;
    if (steps < 1 || !kernel_ms || n_kinds < KK_COUNT) return set_err(ctx, LASTRO_E_ARG, "profile arguments");
    if (m->pos_host + steps > m->max_len) return set_err(ctx, LASTRO_E_FULL, "profile would overflow the KV cache");
    cudaSetDevice(ctx->device);
    cudaStream_t s = ctx->stream;
    const int n_ev = 8 * m->d.layers + 2;
    std::vector<cudaEvent_t> ev(n_ev, nullptr);
    std::vector<int> kinds(n_ev, -1);
    for (auto& e : ev) MTRY(cudaEventCreate(&e), "event create");
    std::vector<double> acc(KK_COUNT, 0.0);
    int result = LASTRO_OK;
    for (int st = 0; st < steps && result == LASTRO_OK; ++st) {
        StepEvents pe;
        pe.ev = ev.data();
        pe.kind = kinds.data();
        cudaError_t e = enqueue_step(m, s, &pe);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) {
            result = model_fail(m, e, "profile step");
            break;
        }
        for (int i = 0; i + 1 < pe.next; ++i) {
            float ms = 0.0f;
            cudaEventElapsedTime(&ms, ev[i], ev[i + 1]);
            if (kinds[i] >= 0) acc[kinds[i]] += ms;
        }
        m->pos_host += 1;
    }
    for (auto& e : ev) cudaEventDestroy(e);
    for (int k = 0; k < KK_COUNT; ++k) kernel_ms[k] = (float)(acc[k] / steps);
    return result;
}

extern "C" int lastro_model_trace(lastro_model* m, int32_t steps, float* exposed_ms, float* span_ms, float* wait_ms,
                                  int32_t n_kinds, float* step_ms) {
    if (!m) return LASTRO_E_ARG;
    lastro_ctx* ctx = m->ctx;
    int rc = check_ready(m);
    if (rc) return rc;
    if (steps < 1 || !exposed_ms || !span_ms || !wait_ms || !step_ms || n_kinds < KK_COUNT)
        return set_err(ctx, LASTRO_E_ARG, "trace arguments");
    if (m->fused_ok && m->use_fused) return set_err(ctx, LASTRO_E_UNSUPPORTED, "trace: the fused step has no per-kernel launches");
    if (m->pos_host + steps > m->max_len) return set_err(ctx, LASTRO_E_FULL, "trace would overflow the KV cache");
    cudaSetDevice(ctx->device);
    cudaStream_t s = ctx->stream;
    const int per_layer = moe_on(m) ? 4 : 5;
    const int launches = per_layer * m->d.layers + 1;
    const size_t words = (size_t)launches * kTraceMaxCtas * kTraceWords;
    const size_t words_max = (size_t)(5 * m->d.layers + 1) * kTraceMaxCtas * kTraceWords;  // either chain fits
    if (!m->d_trace) MTRY(m->arena.alloc(&m->d_trace, words_max), "trace buffer");
    if (!m->trace_graph) {
        // the product step's kernels, launch for launch, with the stamps on; captured like the product graph
        cudaGraph_t g = nullptr;
        MTRY(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal), "begin capture");
        cudaError_t e = cudaMemsetAsync(m->d_trace, 0, words * sizeof(unsigned long long), s);
        if (e == cudaSuccess) e = enqueue_step(m, s, nullptr, m->d_trace);
        cudaError_t e2 = cudaStreamEndCapture(s, &g);
        if (e == cudaSuccess) e = e2;
        if (e == cudaSuccess) e = cudaGraphInstantiate(&m->trace_graph, g, 0);
        if (g) cudaGraphDestroy(g);
        if (e != cudaSuccess) {
            m->trace_graph = nullptr;
            return model_fail(m, e, "trace capture");
        }
    }
    std::vector<int> kind(launches);
    for (int l = 0; l < m->d.layers; ++l) {
        const int k5[5] = {KK_QKV, KK_ATTN, KK_OPROJ, KK_GATE_UP, KK_DOWN};
        for (int i = 0; i < per_layer; ++i) kind[per_layer * l + i] = (per_layer == 4 && i == 3) ? KK_MOE : k5[i];
    }
    kind[launches - 1] = KK_HEAD;
    std::vector<unsigned long long> h(words);
    std::vector<double> ex(KK_COUNT, 0.0), sp(KK_COUNT, 0.0), wt(KK_COUNT, 0.0);
    double step_acc = 0.0;
    MTRY(cudaMemsetAsync(m->d_step, 0, sizeof(int), s), "step reset");
    for (int st = 0; st < steps; ++st) {
        MTRY(cudaGraphLaunch(m->trace_graph, s), "trace launch");
        MTRY(cudaMemcpyAsync(h.data(), m->d_trace, words * sizeof(unsigned long long), cudaMemcpyDeviceToHost, s),
             "trace copy");
        MTRY(cudaStreamSynchronize(s), "trace");
        unsigned long long first = ~0ull, prev_end = 0, last = 0;
        for (int i = 0; i < launches; ++i) {
            unsigned long long t0 = ~0ull, rel = ~0ull, t1 = 0;
            for (int c = 0; c < kTraceMaxCtas; ++c) {
                const unsigned long long* w = &h[((size_t)i * kTraceMaxCtas + c) * kTraceWords];
                if (!w[0]) continue;
                t0 = std::min(t0, w[0]);
                if (w[1]) rel = std::min(rel, w[1]);
                t1 = std::max(t1, w[2]);
            }
            if (t0 == ~0ull) continue;  // a launch without stamps (tensor-core attention)
            if (rel == ~0ull) rel = t0;
            first = std::min(first, t0);
            last = std::max(last, t1);
            const unsigned long long from = prev_end ? prev_end : t0;  // a gap before the launch counts as its own
            ex[kind[i]] += t1 > from ? (double)(t1 - from) : 0.0;
            sp[kind[i]] += (double)(t1 - t0);
            wt[kind[i]] += prev_end && rel > prev_end ? (double)(rel - prev_end) : 0.0;  // hand-off latency
            prev_end = std::max(prev_end, t1);
        }
        if (last > first && first != ~0ull) step_acc += (double)(last - first);
    }
    rc = finish(m, "trace");
    if (rc) return rc;
    m->trace_host.assign(h.begin(), h.begin() + words);  // the last traced step, for lastro_model_trace_raw
    m->pos_host += steps;
    for (int k = 0; k < KK_COUNT; ++k) {
        exposed_ms[k] = (float)(ex[k] / steps * 1e-6);
        span_ms[k] = (float)(sp[k] / steps * 1e-6);
        wait_ms[k] = (float)(wt[k] / steps * 1e-6);
    }
    *step_ms = (float)(step_acc / steps * 1e-6);
    return LASTRO_OK;
}

extern "C" int lastro_model_trace_raw(const lastro_model* m, int32_t launch, unsigned long long* out, int32_t words) {
    if (!m || !out || launch < 0) return LASTRO_E_ARG;
    const size_t per = (size_t)kTraceMaxCtas * kTraceWords;
    if ((size_t)(launch + 1) * per > m->trace_host.size() || (size_t)words < per) return LASTRO_E_ARG;
    memcpy(out, m->trace_host.data() + (size_t)launch * per, per * sizeof(unsigned long long));
    return LASTRO_OK;
}

extern "C" int lastro_model_set_options(lastro_model* m, int32_t use_graphs, int32_t use_pdl, int32_t use_fused) {
    if (!m) return LASTRO_E_ARG;
    cudaSetDevice(m->ctx->device);
    cudaStreamSynchronize(m->ctx->stream);
    if (m->graph) {
        cudaGraphExecDestroy(m->graph);
        m->graph = nullptr;
    }
    if (m->trace_graph) {
        cudaGraphExecDestroy(m->trace_graph);
        m->trace_graph = nullptr;
    }
    m->use_graphs = use_graphs != 0;
    m->use_pdl = use_pdl != 0;
    m->use_fused = use_fused != 0;
    return LASTRO_OK;
}

extern "C" int lastro_model_set_moe(lastro_model* m, int32_t one_launch) {
    if (!m) return LASTRO_E_ARG;
    if (one_launch && !m->moe_ok)
        return set_err(m->ctx, LASTRO_E_UNSUPPORTED, "the one-launch MoE block does not fit these shapes");
    cudaSetDevice(m->ctx->device);
    cudaStreamSynchronize(m->ctx->stream);
    for (cudaGraphExec_t* g : {&m->graph, &m->trace_graph})
        if (*g) {
            cudaGraphExecDestroy(*g);
            *g = nullptr;
        }
    m->use_moe = one_launch != 0;
    return LASTRO_OK;
}

extern "C" int lastro_model_moe(const lastro_model* m) { return m && moe_on(m) ? 1 : 0; }

extern "C" int lastro_model_set_tuning(lastro_model* m, int32_t attn_splits, int32_t attn_merge, int32_t flags) {
    if (!m) return LASTRO_E_ARG;
    const int f32 = m->d.kv_dtype == LASTRO_DTYPE_F32;
    const int splits = attn_splits == 0 ? attn_splits_default(m->max_len, f32) : attn_splits;
    if (splits != 8 && splits != kAttnSplits) return set_err(m->ctx, LASTRO_E_ARG, "attention splits %d (8 or 16)", splits);
    if (attn_merge < 0 || attn_merge > 2)
        return set_err(m->ctx, LASTRO_E_ARG, "attention merge %d with %d splits", attn_merge, splits);
    if (attn_smem(m->max_len, f32, splits) > kMaxSmemBytes)
        return set_err(m->ctx, LASTRO_E_UNSUPPORTED, "%d attention splits do not fit max_len %d", splits, m->max_len);
    cudaSetDevice(m->ctx->device);
    cudaStreamSynchronize(m->ctx->stream);
    for (cudaGraphExec_t* g : {&m->graph, &m->trace_graph})
        if (*g) {
            cudaGraphExecDestroy(*g);
            *g = nullptr;
        }
    m->attn_splits = splits;
    m->attn_merge = attn_merge;
    m->oproj_smem = (flags & LASTRO_TUNE_OPROJ_SMEM) != 0;
    m->gu_prefetch_down = (flags & LASTRO_TUNE_PREFETCH_DOWN) != 0;
    if ((flags & LASTRO_TUNE_ATTN_TMA) && m->kvboxmaps.empty())
        return set_err(m->ctx, LASTRO_E_UNSUPPORTED, "TMA staging of the attention needs bf16 KV");
    if ((flags & LASTRO_TUNE_ATTN_MMA) && m->d.kv_dtype == LASTRO_DTYPE_F32)
        return set_err(m->ctx, LASTRO_E_UNSUPPORTED, "tensor-core attention needs bf16 KV");
    m->attn_tma = (flags & LASTRO_TUNE_ATTN_TMA) != 0;
    m->spec_mode = (flags & LASTRO_TUNE_SPEC_STAGE) ? 1 : (flags & LASTRO_TUNE_SPEC_L2) ? 2
                   : (flags & LASTRO_TUNE_SPEC_ATTN) ? 3 : 0;
    m->attn_mma = (flags & LASTRO_TUNE_ATTN_MMA) != 0;
    m->route_handoff = (flags & LASTRO_TUNE_DOWN_ROUTES) == 0;
    return LASTRO_OK;
}

extern "C" int lastro_model_fused(const lastro_model* m) { return m && m->fused_ok && m->use_fused ? 1 : 0; }

extern "C" int lastro_model_set_attention(lastro_model* m, int32_t tensor_cores) {
    if (!m) return LASTRO_E_ARG;
    if (tensor_cores && m->kvmaps.empty())
        return set_err(m->ctx, LASTRO_E_UNSUPPORTED, "tensor-core attention needs bf16 KV and TMA page maps");
    cudaSetDevice(m->ctx->device);
    cudaStreamSynchronize(m->ctx->stream);
    if (m->graph) {
        cudaGraphExecDestroy(m->graph);
        m->graph = nullptr;
    }
    if (m->trace_graph) {
        cudaGraphExecDestroy(m->trace_graph);
        m->trace_graph = nullptr;
    }
    m->attn_tc = tensor_cores != 0;
    return LASTRO_OK;
}

extern "C" void lastro_model_destroy(lastro_model* m) {
    if (!m) return;
    cudaSetDevice(m->ctx->device);
    cudaStreamSynchronize(m->ctx->stream);  // gpu_model.rs:448-455
    if (m->pbatch) lastro_batch_destroy(m->pbatch);  // aliases the model's KV cache: destroyed first
    if (m->graph) cudaGraphExecDestroy(m->graph);
    if (m->trace_graph) cudaGraphExecDestroy(m->trace_graph);
    m->arena.release();
    if (m->h_token) cudaFreeHost(m->h_token);
    lastro_ctx* ctx = m->ctx;
    delete m;
    ctx_release(ctx);
}
