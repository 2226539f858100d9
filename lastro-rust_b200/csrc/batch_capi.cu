// C ABI of the batched decode step: many independent sequences decoded together on the weights of one lastro_model,
// with the MoE experts partitioned over the ranks of an expert-parallel group (one process per GPU).
//
// The reference decodes one sequence at a time (gpu_model.rs GpuModel::step); a batched step has the reference's
// own multi-position contract: every sequence's results equal its single-sequence step up to summation order
// (cpu.rs:234-238).  A lastro_batch holds the sequences' paged KV caches and the step's scratch; the weights stay in
// the model.  Every rank of a group creates its batch with the same max_seqs and world, exchanges the handle of its
// exchange region (lastro_batch_exchange_handle) with the others, and connects (lastro_batch_connect); the ranks then
// call the step functions the same number of times, each for its own sequences.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <map>
#include <vector>

#include "batch.h"
#include "capi_internal.h"

using namespace lastro;
using namespace lastro_capi;

struct lastro_batch {
    lastro_model* m = nullptr;
    lastro_ctx* ctx = nullptr;
    int max_seqs = 0, max_len = 0, max_pages = 0, rank = 0, world = 1, epr = 0;
    int ks_qkv = 1, ks_o = 1, R = 0;
    int attn_S = 1, attn_cap = 1;  // attention splits per (token, KV head) and positions one split stages
    int n_sm = 148;
    bool poisoned = false, connected = false, use_graphs = true;
    unsigned long long wait_ns = 10ull * 1000 * 1000 * 1000;  // bound of the exchange's flag waits
    int gemm_mode = 2;  // 0 mma.sync, 1 tcgen05 (cp.async stages), 2 tcgen05 warp-specialised (TMA weight tiles)
    // TMA tensor maps of the weights (mode 2): per layer qkv, o, gate_up, down; then the embedding (lm_head)
    std::vector<CUtensorMap> wmaps;
    // bf16 KV: attention on tensor cores with TMA page loads (per layer: K map, V map); else the CUDA-core kernel
    std::vector<CUtensorMap> kvmaps;
    bool attn_tc = false;
    Arena arena;
    std::vector<void*> kpool, vpool;  // per layer: [max_seqs * max_pages pages][kv_heads][page][d]
    float* rope_cs = nullptr;
    int *page_table = nullptr, *d_pos = nullptr;
    std::vector<int> pos_host;
    int *d_seq = nullptr, *d_tok = nullptr, *d_next = nullptr, *d_hist = nullptr;
    int *h_seq = nullptr, *h_tok = nullptr, *h_err = nullptr;  // pinned
    float *h = nullptr, *qkv_part = nullptr, *q = nullptr, *att = nullptr, *part_acc = nullptr, *part_ml = nullptr;
    float *o_part = nullptr, *rw = nullptr, *logits = nullptr, *bias = nullptr;
    uint16_t *xa_hi = nullptr, *xa_lo = nullptr, *att_hi = nullptr, *att_lo = nullptr;
    uint16_t *a_hi = nullptr, *a_lo = nullptr;
    unsigned int *attn_counters = nullptr, *counters = nullptr, *epoch = nullptr;
    int *ids = nullptr, *route_hist = nullptr, *x_rows = nullptr, *src = nullptr, *g_off = nullptr, *g_cnt = nullptr;
    int *n_pos = nullptr, *d_err = nullptr;
    XLayout lay{};
    unsigned char* xreg = nullptr;
    unsigned char** d_peers = nullptr;
    // expert placement: owner rank and index among the owner's experts of every expert, this rank's experts
    int *d_owner = nullptr, *d_local = nullptr, *d_gexp = nullptr;
    std::vector<void*> opened;  // peer regions mapped from IPC handles
    std::map<int, cudaGraphExec_t> graphs;  // one per token count
    bool has_bias = false, want_hist = false;
    // multi-position steps of a model's own sequence (lastro_model_step_positions): the KV pools, page table, position
    // and RoPE table are the model's; token z of a step sits off[z] = z positions past the sequence's position
    bool alias = false;
    int* d_off = nullptr;
    // profiling: an event recorded after every launch of a direct (uncaptured) step, with the launch's kind
    std::vector<cudaEvent_t>* prof_ev = nullptr;
    std::vector<int>* prof_kind = nullptr;
    // in-graph timeline (lastro_batch_trace): every CTA's stamps of the last traced step
    unsigned long long* d_trace = nullptr;
    std::vector<unsigned long long> trace_host;
};

namespace {

int bfail(lastro_batch* b, cudaError_t e, const char* what) { return cuda_fail(b->ctx, &b->poisoned, e, what); }

// kernel kinds of the batched step, in launch order within a layer, then the head
enum { BK_NORM = 0, BK_QKV, BK_ROPE, BK_ATTN, BK_OPROJ, BK_ROUTER, BK_GROUP, BK_GATE_UP, BK_DOWN, BK_COMBINE,
       BK_LM_HEAD, BK_ARGMAX, BK_COUNT };

cudaError_t mark(lastro_batch* b, cudaStream_t s, int kind, cudaError_t e) {
    if (e != cudaSuccess || !b->prof_ev) return e;
    cudaEvent_t ev;
    if ((e = cudaEventCreate(&ev)) != cudaSuccess) return e;
    b->prof_ev->push_back(ev);
    b->prof_kind->push_back(kind);
    return cudaEventRecord(ev, s);
}

#define BTRY(expr, what)                                        \
    do {                                                        \
        cudaError_t e_ = (expr);                                \
        if (e_ != cudaSuccess) return bfail(b, e_, what);       \
    } while (0)

const CUtensorMap* wmap(const lastro_batch* b, int layer, int which) {
    const size_t i = (size_t)layer * 4 + which;
    return i < b->wmaps.size() ? &b->wmaps[i] : nullptr;
}

struct Placement {
    std::vector<int> owner, local, mine;
};

// local index of every expert among its owner's experts (ascending ids) and this rank's experts in that order, then
// the tables to the device (asynchronously on the batch's stream: `pl` must live until the stream passes the copies)
cudaError_t upload_placement(lastro_batch* b, Placement& pl) {
    const int E = (int)pl.owner.size();
    std::vector<int> seen(b->world, 0);
    pl.local.assign(E, 0);
    pl.mine.clear();
    for (int x = 0; x < E; ++x) {
        pl.local[x] = seen[pl.owner[x]]++;
        if (pl.owner[x] == b->rank) pl.mine.push_back(x);
    }
    cudaStream_t s = b->ctx->stream;
    cudaError_t e = cudaMemcpyAsync(b->d_owner, pl.owner.data(), sizeof(int) * E, cudaMemcpyHostToDevice, s);
    if (!e) e = cudaMemcpyAsync(b->d_local, pl.local.data(), sizeof(int) * E, cudaMemcpyHostToDevice, s);
    if (!e) e = cudaMemcpyAsync(b->d_gexp, pl.mine.data(), sizeof(int) * pl.mine.size(), cudaMemcpyHostToDevice, s);
    return e;
}

// split-K slices for a dense GEMM of `rows` x K: at most two CTAs per SM, slices of at least 256 columns (4 stages; on
// C5 slices of 128 measured the same kernel times with twice the partial-sum traffic)
int pick_ks(int rows, int K, int n_sm) {
    const int tiles = (rows + kBRows - 1) / kBRows, chunks = K / kBK;
    int best = 1;
    for (int d = 1; d <= chunks; ++d)
        if (chunks % d == 0 && K / d >= 256 && tiles * d <= 2 * n_sm && d <= 16) best = d;
    return best;
}

// launches of one step: the layer-0 norm, 8 per layer, the lm_head and the argmax
int bstep_launches(const lastro_batch* b) { return 8 * b->m->d.layers + 3; }

// `trace` (optional): kTraceMaxCtas * kTraceWords stamps per launch, in launch order
cudaError_t enqueue_bstep(lastro_batch* b, int n, cudaStream_t s, unsigned long long* trace = nullptr) {
    lastro_model* m = b->m;
    const lastro_model_desc& d = m->d;
    const int H = d.hidden, I = d.inter, E = d.experts, k = d.k, qd = m->qd, kvd = m->kvd, R = b->R;
    cudaError_t e = cudaSuccess;
    size_t launch = 0;
    auto tr = [&]() -> unsigned long long* {
        return trace ? trace + (launch++) * (size_t)kTraceMaxCtas * kTraceWords : nullptr;
    };
    BExchangeArgs xa{};
    xa.peers = b->d_peers;
    xa.lay = b->lay;
    xa.rank = b->rank;
    xa.world = b->world;
    xa.experts_per_rank = b->epr;
    xa.owner = b->d_owner;
    xa.local = b->d_local;
    xa.epoch_base = b->epoch;
    xa.err = b->d_err;
    xa.wait_ns = b->wait_ns;
    xa.n = n;
    xa.k = k;
    xa.H = H;
    xa.x_rows = b->x_rows;
    xa.src = b->src;
    xa.g_off = b->g_off;
    xa.g_cnt = b->g_cnt;
    xa.n_pos = b->n_pos;
    xa.h = b->h;
    xa.weights = b->rw;
    xa.resid = d.residual_multiplier;
    xa.eps = d.eps;
    xa.xn_hi = b->xa_hi;
    xa.xn_lo = b->xa_lo;
    const uint16_t* rx = reinterpret_cast<const uint16_t*>(b->xreg + b->lay.rx);
    // layer 0's attention norm on the embedding rows; every later norm (and the final one) comes out of the combine
    BNormArgs na{};
    na.h = b->h;
    na.embed = m->embed;
    na.tokens = b->d_tok;
    na.emb_mult = d.embedding_multiplier;
    na.ln = m->L[0].ln_attn;
    na.eps = d.eps;
    na.x_hi = b->xa_hi;
    na.x_lo = b->xa_lo;
    na.H = H;
    na.trace = tr();
    if ((e = mark(b, s, BK_NORM, launch_battn_norm(na, n, s)))) return e;
    for (int l = 0; l < d.layers && e == cudaSuccess; ++l) {
        const LayerDev& L = m->L[l];
        xa.layer = l;
        BGemmArgs ga{};
        ga.w = reinterpret_cast<const uint16_t*>(L.wqkv);
        ga.rows = R;
        ga.K = H;
        ga.k_split = H / b->ks_qkv;
        ga.x_hi = b->xa_hi;
        ga.x_lo = b->xa_lo;
        ga.ldx = H;
        ga.n = n;
        ga.y = b->qkv_part;
        ga.ldy = R;
        ga.z_stride = (long long)n * R;
        ga.div = 1.0f;
        ga.tc = b->gemm_mode;
        ga.trace = tr();
        if ((e = mark(b, s, BK_QKV, launch_bgemm(ga, BEPI_STORE, 1, s, wmap(b, l, 0))))) break;

        BRopeArgs ra{};
        ra.part = b->qkv_part;
        ra.ks = b->ks_qkv;
        ra.seq = b->d_seq;
        ra.pos = b->d_pos;
        ra.off = b->d_off;
        ra.rope_cs = b->rope_cs;
        ra.q = b->q;
        ra.k_pool = b->kpool[l];
        ra.v_pool = b->vpool[l];
        ra.page_table = b->page_table;
        ra.pt_stride = b->max_pages;
        ra.page_size = kPageSize;
        ra.kv_f32 = d.kv_dtype == LASTRO_DTYPE_F32;
        ra.n = n;
        ra.qd = qd;
        ra.kvd = kvd;
        ra.d = d.head_dim;
        ra.kv_heads = d.kv_heads;
        ra.trace = tr();
        if ((e = mark(b, s, BK_ROPE, launch_brope_kv(ra, s)))) break;

        BAttnArgs aa{};
        aa.q = b->q;
        aa.k_pool = b->kpool[l];
        aa.v_pool = b->vpool[l];
        aa.page_table = b->page_table;
        aa.pt_stride = b->max_pages;
        aa.page_size = kPageSize;
        aa.kv_f32 = ra.kv_f32;
        aa.seq = b->d_seq;
        aa.pos = b->d_pos;
        aa.off = b->d_off;
        aa.part_acc = b->part_acc;
        aa.part_ml = b->part_ml;
        aa.counters = b->attn_counters;
        aa.att_out = b->att;
        aa.att_hi = b->att_hi;
        aa.att_lo = b->att_lo;
        aa.err = b->d_err;
        aa.n = n;
        aa.kv_heads = d.kv_heads;
        aa.G = m->G;
        aa.S = b->attn_S;
        aa.cap = b->attn_cap;
        aa.scale = d.attention_multiplier;
        aa.trace = tr();
        if (b->attn_tc) {
            // context splits for few tokens: at most about 4 CTAs per SM in all (one split while the tokens alone
            // fill that), at most 16 splits, at least 2 pages each
            const int want = (4 * b->n_sm) / (n * d.kv_heads);
            aa.S = std::max(1, std::min({want, 16, b->max_pages / 2}));
            e = mark(b, s, BK_ATTN, launch_battention_tc(aa, &b->kvmaps[2 * l], &b->kvmaps[2 * l + 1], s));
        }
        else
            e = mark(b, s, BK_ATTN, launch_battention(aa, s));
        if (e) break;

        BGemmArgs oa{};
        oa.w = reinterpret_cast<const uint16_t*>(L.wo);
        oa.rows = H;
        oa.K = qd;
        oa.k_split = qd / b->ks_o;
        oa.x_hi = b->att_hi;
        oa.x_lo = b->att_lo;
        oa.ldx = qd;
        oa.n = n;
        oa.y = b->o_part;
        oa.ldy = H;
        oa.z_stride = (long long)n * H;
        oa.div = 1.0f;
        oa.tc = b->gemm_mode;
        oa.trace = tr();
        if ((e = mark(b, s, BK_OPROJ, launch_bgemm(oa, BEPI_STORE, 1, s, wmap(b, l, 1))))) break;

        BRouterArgs rta{};
        rta.h = b->h;
        rta.opart = b->o_part;
        rta.ks = b->ks_o;
        rta.resid = d.residual_multiplier;
        rta.ln = L.ln_moe;
        rta.eps = d.eps;
        rta.wr = reinterpret_cast<const uint16_t*>(L.router);
        rta.bias = b->has_bias ? b->bias + (size_t)l * E : nullptr;
        rta.x = xa;
        rta.x.counter = b->counters;
        rta.ids = b->ids;
        rta.weights = b->rw;
        rta.route_hist = b->want_hist ? b->route_hist : nullptr;
        rta.layer = l;
        rta.layers = d.layers;
        rta.n = n;
        rta.H = H;
        rta.E = E;
        rta.k = k;
        rta.trace = tr();
        if ((e = mark(b, s, BK_ROUTER, launch_brouter(rta, s)))) break;

        BGemmArgs gu{};
        gu.w = reinterpret_cast<const uint16_t*>(L.gate_up);
        gu.group_stride = (long long)2 * I * H;
        gu.group_expert = b->d_gexp;
        gu.rows = 2 * I;
        gu.K = H;
        gu.k_split = H;
        gu.x_hi = rx;
        gu.x_lo = rx + H;
        gu.ldx = 2 * H;
        gu.x_rows = b->x_rows;
        gu.g_off = b->g_off;
        gu.g_cnt = b->g_cnt;
        gu.a_hi = b->a_hi;
        gu.a_lo = b->a_lo;
        gu.I = I;
        gu.div = 1.0f;
        gu.tc = b->gemm_mode;
        gu.trace = tr();
        if ((e = mark(b, s, BK_GATE_UP, launch_bgemm(gu, BEPI_SWIGLU, b->epr, s, wmap(b, l, 2))))) break;

        BGemmArgs dn{};
        dn.w = reinterpret_cast<const uint16_t*>(L.down);
        dn.group_stride = (long long)H * I;
        dn.group_expert = b->d_gexp;
        dn.rows = H;
        dn.K = I;
        dn.k_split = I;
        dn.x_hi = b->a_hi;
        dn.x_lo = b->a_lo;
        dn.ldx = I;
        dn.g_off = b->g_off;
        dn.g_cnt = b->g_cnt;
        dn.div = 1.0f;
        dn.tc = b->gemm_mode;
        dn.x = xa;
        dn.x.counter = b->counters + 32;
        dn.trace = tr();
        if ((e = mark(b, s, BK_DOWN, launch_bgemm(dn, BEPI_RETURN, b->epr, s, wmap(b, l, 3))))) break;

        BExchangeArgs ca = xa;
        ca.ln_next = l + 1 < d.layers ? m->L[l + 1].ln_attn : m->norm;
        ca.trace = tr();
        if ((e = mark(b, s, BK_COMBINE, launch_ep_combine(ca, s)))) break;
    }
    if (e) return e;
    BGemmArgs ha{};
    ha.w = m->embed;
    ha.rows = d.vocab;
    ha.K = H;
    ha.k_split = H;
    ha.x_hi = b->xa_hi;
    ha.x_lo = b->xa_lo;
    ha.ldx = H;
    ha.n = n;
    ha.y = b->logits;
    ha.ldy = d.vocab;
    ha.div = d.logits_scaling;
    ha.tc = b->gemm_mode;
    ha.trace = tr();
    if ((e = mark(b, s, BK_LM_HEAD, launch_bgemm(ha, BEPI_STORE, 1, s, wmap(b, b->m->d.layers, 0))))) return e;
    BHeadArgs hd{};
    hd.logits = b->logits;
    hd.V = d.vocab;
    hd.n = n;
    hd.seq = b->d_seq;
    hd.pos = b->d_pos;
    hd.off = b->d_off;
    hd.next = b->d_next;
    hd.tokens = b->d_tok;
    hd.epoch_base = b->epoch;
    hd.layers = d.layers;
    hd.trace = tr();
    return mark(b, s, BK_ARGMAX, launch_bargmax(hd, s));
}

int run_bstep(lastro_batch* b, int n) {
    cudaStream_t s = b->ctx->stream;
    if (!b->use_graphs) {
        BTRY(enqueue_bstep(b, n, s), "batch step launch");
        return LASTRO_OK;
    }
    auto it = b->graphs.find(n);
    if (it == b->graphs.end()) {
        cudaGraph_t g = nullptr;
        BTRY(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal), "begin capture");
        cudaError_t e = enqueue_bstep(b, n, s);
        cudaError_t e2 = cudaStreamEndCapture(s, &g);
        if (e == cudaSuccess) e = e2;
        if (e != cudaSuccess) {
            if (g) cudaGraphDestroy(g);
            return bfail(b, e, "batch step capture");
        }
        cudaGraphExec_t x = nullptr;
        e = cudaGraphInstantiate(&x, g, 0);
        cudaGraphDestroy(g);
        if (e != cudaSuccess) return bfail(b, e, "batch graph instantiate");
        it = b->graphs.emplace(n, x).first;
    }
    BTRY(cudaGraphLaunch(it->second, s), "batch graph launch");
    return LASTRO_OK;
}

int bfinish(lastro_batch* b, const char* what) {
    cudaStream_t s = b->ctx->stream;
    BTRY(cudaMemcpyAsync(b->h_err, b->d_err, sizeof(int), cudaMemcpyDeviceToHost, s), what);
    BTRY(cudaStreamSynchronize(s), what);
    if (*b->h_err) {
        b->poisoned = true;
        return set_err(b->ctx, LASTRO_E_CUDA, "%s: a kernel wait gave up (code %d); batch poisoned", what, *b->h_err);
    }
    return LASTRO_OK;
}

int bready(lastro_batch* b) {
    if (b->poisoned) return set_err(b->ctx, LASTRO_E_POISONED, "batch unusable after an earlier error");
    if (!b->connected) return set_err(b->ctx, LASTRO_E_STATE, "batch not connected (lastro_batch_connect)");
    return model_check_ready(b->m);
}

// seq ids in range and distinct, tokens in range, room for `steps` more positions; copies them to the device
int bstage(lastro_batch* b, int n, const int32_t* seq, const int32_t* tok, int steps) {
    const lastro_model_desc& d = b->m->d;
    if (n < 1 || n > b->max_seqs || !seq || !tok) return set_err(b->ctx, LASTRO_E_ARG, "batch of %d sequences", n);
    std::vector<char> seen(b->max_seqs, 0);
    for (int i = 0; i < n; ++i) {
        if (seq[i] < 0 || seq[i] >= b->max_seqs || seen[seq[i]])
            return set_err(b->ctx, LASTRO_E_ARG, "sequence id %d out of range or repeated", seq[i]);
        seen[seq[i]] = 1;
        if (tok[i] < 0 || tok[i] >= d.vocab) return set_err(b->ctx, LASTRO_E_ARG, "token %d out of range", tok[i]);
        if (b->pos_host[seq[i]] + steps > b->max_len)
            return set_err(b->ctx, LASTRO_E_FULL, "sequence %d: KV cache full (max_len %d)", seq[i], b->max_len);
    }
    memcpy(b->h_seq, seq, sizeof(int) * n);
    memcpy(b->h_tok, tok, sizeof(int) * n);
    cudaStream_t s = b->ctx->stream;
    BTRY(cudaMemcpyAsync(b->d_seq, b->h_seq, sizeof(int) * n, cudaMemcpyHostToDevice, s), "stage");
    BTRY(cudaMemcpyAsync(b->d_tok, b->h_tok, sizeof(int) * n, cudaMemcpyHostToDevice, s), "stage");
    return LASTRO_OK;
}

}  // namespace

namespace {

// alias: a batch of up to max_seqs tokens of the model's own sequence (world 1), on the model's KV cache
int batch_create(lastro_model* m, int32_t max_seqs, int32_t max_len, int32_t rank, int32_t world, bool alias,
                 lastro_batch** out) {
    if (!m || !out) return LASTRO_E_ARG;
    *out = nullptr;
    lastro_ctx* ctx = m->ctx;
    const lastro_model_desc& d = m->d;
    if (max_seqs < 1 || max_len < 1 || world < 1 || world > kBMaxRanks || rank < 0 || rank >= world)
        return set_err(ctx, LASTRO_E_ARG, "batch: max_seqs %d, max_len %d, rank %d of %d", max_seqs, max_len, rank, world);
    if (m->q8) return set_err(ctx, LASTRO_E_UNSUPPORTED, "batched decode runs bf16 weights");
    if (d.experts % world) return set_err(ctx, LASTRO_E_UNSUPPORTED, "%d experts over %d ranks", d.experts, world);
    if (d.hidden % kBRows || m->qd % kBK || d.inter % 64 || d.hidden > 2048)
        return set_err(ctx, LASTRO_E_UNSUPPORTED, "batched GEMMs need hidden a multiple of 128, heads*head_dim and inter of 64");
    if (world * max_seqs * d.k > kBMaxSlots)
        return set_err(ctx, LASTRO_E_UNSUPPORTED, "world x max_seqs x k = %d pairs exceed %d", world * max_seqs * d.k, kBMaxSlots);
    const int attn_S = (max_len + kBAttnRows - 1) / kBAttnRows;
    if (attn_S > kBAttnMaxSplits)
        return set_err(ctx, LASTRO_E_UNSUPPORTED, "max_len %d beyond %d positions", max_len, kBAttnRows * kBAttnMaxSplits);
    cudaSetDevice(ctx->device);
    int n_sm = 148;
    cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, ctx->device);
    lastro_batch* b = new lastro_batch();
    b->m = m;
    b->ctx = ctx;
    b->max_seqs = max_seqs;
    b->max_len = max_len;
    b->max_pages = (max_len + kPageSize - 1) / kPageSize;
    b->rank = rank;
    b->world = world;
    b->epr = d.experts / world;
    b->R = m->qd + 2 * m->kvd;
    b->attn_S = attn_S;
    b->n_sm = n_sm;
    b->attn_cap = (max_len + attn_S - 1) / attn_S + 1;
    b->ks_qkv = pick_ks(b->R, d.hidden, n_sm);
    b->ks_o = pick_ks(d.hidden, m->qd, n_sm);
    b->pos_host.assign(max_seqs, 0);
    b->lay = x_layout(world, max_seqs, d.k, d.hidden);
    b->alias = alias;
    if (alias) b->max_pages = m->max_pages;
    const size_t H = d.hidden, I = d.inter, S = max_seqs, E = d.experts, k = d.k, V = d.vocab;
    const size_t pairs = (size_t)world * b->lay.cap;
    const size_t kv_elems = S * b->max_pages * kPageSize * (size_t)m->kvd;
    const size_t kv_bytes = kv_elems * (d.kv_dtype == LASTRO_DTYPE_F32 ? 4 : 2);
    Arena& A = b->arena;
    bool bad = false;
    b->kpool.assign(d.layers, nullptr);
    b->vpool.assign(d.layers, nullptr);
    for (int l = 0; l < d.layers && !bad; ++l) {
        if (alias) {
            b->kpool[l] = m->L[l].k_pool;
            b->vpool[l] = m->L[l].v_pool;
        } else {
            bad = A.alloc(&b->kpool[l], kv_bytes) || A.alloc(&b->vpool[l], kv_bytes);
        }
    }
    if (alias) {
        b->rope_cs = m->rope_cs;
        b->page_table = m->page_table;
        b->d_pos = m->d_pos;
        bad = bad || A.alloc(&b->d_off, S);
    } else {
        bad = bad || A.alloc(&b->rope_cs, (size_t)max_len * d.head_dim) || A.alloc(&b->page_table, S * b->max_pages) ||
              A.alloc(&b->d_pos, S);
    }
    bad = bad || A.alloc(&b->d_seq, S) || A.alloc(&b->d_tok, S) || A.alloc(&b->d_next, S) ||
          A.alloc(&b->d_hist, (size_t)max_len * S) || A.alloc(&b->h, S * H) || A.alloc(&b->xa_hi, S * H) ||
          A.alloc(&b->xa_lo, S * H) || A.alloc(&b->qkv_part, (size_t)b->ks_qkv * S * b->R) ||
          A.alloc(&b->q, S * m->qd) || A.alloc(&b->att, S * m->qd) || A.alloc(&b->att_hi, S * m->qd) ||
          A.alloc(&b->att_lo, S * m->qd) || A.alloc(&b->part_acc, S * d.heads * std::max(attn_S, 16) * d.head_dim) ||
          A.alloc(&b->part_ml, S * d.heads * std::max(attn_S, 16) * 2) || A.alloc(&b->attn_counters, S * d.kv_heads) ||
          A.alloc(&b->o_part, (size_t)b->ks_o * S * H) || A.alloc(&b->ids, S * k) || A.alloc(&b->rw, S * k) ||
          A.alloc(&b->bias, (size_t)d.layers * E) ||
          A.alloc(&b->x_rows, pairs) || A.alloc(&b->src, pairs) || A.alloc(&b->g_off, kMaxExperts) ||
          A.alloc(&b->g_cnt, kMaxExperts) || A.alloc(&b->n_pos, 1) || A.alloc(&b->a_hi, pairs * I) ||
          A.alloc(&b->a_lo, pairs * I) || A.alloc(&b->logits, S * V) ||
          A.alloc(&b->route_hist, S * d.layers * k) || A.alloc(&b->counters, 64) || A.alloc(&b->epoch, 1) ||
          A.alloc(&b->d_err, 1) || A.alloc(&b->xreg, b->lay.bytes) || A.alloc(&b->d_peers, (size_t)world) ||
          A.alloc(&b->d_owner, E) || A.alloc(&b->d_local, E) || A.alloc(&b->d_gexp, (size_t)b->epr);
    if (!bad) bad = cudaMallocHost(&b->h_seq, sizeof(int) * S) != cudaSuccess;
    if (!bad) bad = cudaMallocHost(&b->h_tok, sizeof(int) * S) != cudaSuccess;
    if (!bad) bad = cudaMallocHost(&b->h_err, sizeof(int)) != cudaSuccess;
    if (bad) {
        cudaGetLastError();
        if (b->h_seq) cudaFreeHost(b->h_seq);
        if (b->h_tok) cudaFreeHost(b->h_tok);
        if (b->h_err) cudaFreeHost(b->h_err);
        A.release();
        delete b;
        return set_err(ctx, LASTRO_E_NOMEM, "batch allocation failed");
    }
    *b->h_err = 0;
    cudaStream_t s = ctx->stream;
    std::vector<int> pt(S * b->max_pages);
    for (size_t i = 0; i < pt.size(); ++i) pt[i] = (int)i;  // sequence q owns pages [q * max_pages, (q+1) * max_pages)
    const std::vector<float> cs = rope_table(d, max_len);
    std::vector<int> offs(S);
    for (size_t i = 0; i < offs.size(); ++i) offs[i] = (int)i;
    cudaError_t e = cudaSuccess;
    if (alias) {
        e = cudaMemcpyAsync(b->d_off, offs.data(), sizeof(int) * S, cudaMemcpyHostToDevice, s);
        if (!e) e = cudaMemsetAsync(b->d_seq, 0, sizeof(int) * S, s);  // every token is the model's sequence
    } else {
        e = cudaMemcpyAsync(b->page_table, pt.data(), sizeof(int) * pt.size(), cudaMemcpyHostToDevice, s);
        if (!e) e = cudaMemcpyAsync(b->rope_cs, cs.data(), sizeof(float) * cs.size(), cudaMemcpyHostToDevice, s);
        if (!e) e = cudaMemsetAsync(b->d_pos, 0, sizeof(int) * S, s);
    }
    if (!e) e = cudaMemsetAsync(b->attn_counters, 0, sizeof(unsigned int) * S * d.kv_heads, s);
    if (!e) e = cudaMemsetAsync(b->counters, 0, sizeof(unsigned int) * 64, s);
    if (!e) e = cudaMemsetAsync(b->epoch, 0, sizeof(unsigned int), s);
    if (!e) e = cudaMemsetAsync(b->d_err, 0, sizeof(int), s);
    if (!e) e = cudaMemsetAsync(b->xreg, 0, b->lay.bytes, s);
    for (int l = 0; l < d.layers && !e && !alias; ++l) {  // finite values past every context (whole pages are read)
        e = cudaMemsetAsync(b->kpool[l], 0, kv_bytes, s);
        if (!e) e = cudaMemsetAsync(b->vpool[l], 0, kv_bytes, s);
    }
    if (!e) e = cudaMemsetAsync(b->route_hist, 0, sizeof(int) * S * d.layers * k, s);
    Placement pl;  // contiguous: experts [r * E / world, (r + 1) * E / world) on rank r
    for (int x = 0; x < (int)E; ++x) pl.owner.push_back(x / b->epr);
    if (!e) e = upload_placement(b, pl);
    if (!e) e = cudaStreamSynchronize(s);
    if (e) {
        cudaGetLastError();
        cudaFreeHost(b->h_seq);
        cudaFreeHost(b->h_tok);
        cudaFreeHost(b->h_err);
        A.release();
        delete b;
        return set_err(ctx, LASTRO_E_CUDA, "batch init: %s", cudaGetErrorString(e));
    }
    // tensor maps of the weight matrices for the warp-specialised GEMM; without them the GEMMs run mode 1
    b->wmaps.resize((size_t)d.layers * 4 + 1);
    bool maps_ok = true;
    for (int l = 0; l < d.layers && maps_ok; ++l) {
        const LayerDev& L = m->L[l];
        maps_ok = make_weight_map(&b->wmaps[l * 4 + 0], L.wqkv, b->R, H) == cudaSuccess &&
                  make_weight_map(&b->wmaps[l * 4 + 1], L.wo, H, m->qd) == cudaSuccess &&
                  make_weight_map(&b->wmaps[l * 4 + 2], L.gate_up, E * 2 * I, H) == cudaSuccess &&
                  make_weight_map(&b->wmaps[l * 4 + 3], L.down, E * H, I) == cudaSuccess;
    }
    maps_ok = maps_ok && make_weight_map(&b->wmaps[(size_t)d.layers * 4], m->embed, V, H) == cudaSuccess;
    if (!maps_ok) {
        cudaGetLastError();
        b->wmaps.clear();
        b->gemm_mode = 1;
    }
    if (d.kv_dtype == LASTRO_DTYPE_BF16 && m->G <= 8) {
        const uint64_t kv_rows = (uint64_t)(alias ? 1 : S) * b->max_pages * d.kv_heads * kPageSize;
        b->kvmaps.resize((size_t)d.layers * 2);
        bool kv_ok = true;
        for (int l = 0; l < d.layers && kv_ok; ++l)
            kv_ok = make_kv_map(&b->kvmaps[2 * l], b->kpool[l], kv_rows) == cudaSuccess &&
                    make_kv_map(&b->kvmaps[2 * l + 1], b->vpool[l], kv_rows) == cudaSuccess;
        if (!kv_ok) {
            cudaGetLastError();
            b->kvmaps.clear();
        }
        b->attn_tc = kv_ok;
    }
    ctx_retain(ctx);
    *out = b;
    return LASTRO_OK;
}

}  // namespace

extern "C" int lastro_batch_create(lastro_model* m, int32_t max_seqs, int32_t max_len, int32_t rank, int32_t world,
                                   lastro_batch** out) {
    return batch_create(m, max_seqs, max_len, rank, world, false, out);
}

extern "C" int lastro_model_step_positions(lastro_model* m, int32_t n, const int32_t* tokens, float* logits,
                                           int32_t* next) {
    if (!m) return LASTRO_E_ARG;
    lastro_ctx* ctx = m->ctx;
    int rc = model_check_ready(m);
    if (rc) return rc;
    const lastro_model_desc& d = m->d;
    if (n < 1 || n > kMaxStepPositions || !tokens)
        return set_err(ctx, LASTRO_E_ARG, "step of %d positions (1..%d)", n, kMaxStepPositions);
    for (int i = 0; i < n; ++i)
        if (tokens[i] < 0 || tokens[i] >= d.vocab) return set_err(ctx, LASTRO_E_ARG, "token %d out of range", tokens[i]);
    if (m->pos_host + n > m->max_len) return set_err(ctx, LASTRO_E_FULL, "KV cache full (max_len %d)", m->max_len);
    if (m->fused_ok && m->use_fused) return set_err(ctx, LASTRO_E_UNSUPPORTED, "multi-position steps run the kernel chain");
    cudaSetDevice(ctx->device);
    if (!m->pbatch) {
        lastro_batch* b = nullptr;
        rc = batch_create(m, kMaxStepPositions, m->max_len, 0, 1, true, &b);
        if (rc) return rc;
        rc = lastro_batch_connect(b, nullptr, (int32_t)sizeof(cudaIpcMemHandle_t));
        if (rc) {
            lastro_batch_destroy(b);
            return rc;
        }
        m->pbatch = b;
    }
    lastro_batch* b = m->pbatch;
    if (b->poisoned) {
        m->poisoned = true;
        return set_err(ctx, LASTRO_E_POISONED, "model unusable after an earlier error");
    }
    cudaStream_t s = ctx->stream;
    memcpy(b->h_tok, tokens, sizeof(int) * n);
    if (b->want_hist) {
        for (auto& g : b->graphs) cudaGraphExecDestroy(g.second);
        b->graphs.clear();
        b->want_hist = false;
    }
    rc = [&]() -> int {
        BTRY(cudaMemcpyAsync(b->d_tok, b->h_tok, sizeof(int) * n, cudaMemcpyHostToDevice, s), "stage");
        int r = run_bstep(b, n);
        if (r) return r;
        // the next single-position step (or device-side decode) continues from the last position's greedy id
        BTRY(cudaMemcpyAsync(m->d_token, b->d_next + (n - 1), sizeof(int), cudaMemcpyDeviceToDevice, s), "token");
        if (next) BTRY(cudaMemcpyAsync(next, b->d_next, sizeof(int) * n, cudaMemcpyDeviceToHost, s), "next download");
        if (logits)
            BTRY(cudaMemcpyAsync(logits, b->logits, sizeof(float) * n * d.vocab, cudaMemcpyDeviceToHost, s),
                 "logits download");
        return bfinish(b, "multi-position step");
    }();
    if (rc) {
        m->poisoned = true;
        return rc;
    }
    m->pos_host += n;
    return LASTRO_OK;
}

extern "C" int lastro_batch_exchange_handle(lastro_batch* b, void* handle, int32_t bytes) {
    if (!b || !handle || bytes < (int)sizeof(cudaIpcMemHandle_t)) return LASTRO_E_ARG;
    cudaSetDevice(b->ctx->device);
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, b->xreg);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return set_err(b->ctx, LASTRO_E_CUDA, "exchange handle: %s", cudaGetErrorString(e));
    }
    memcpy(handle, &h, sizeof h);
    return LASTRO_OK;
}

extern "C" int lastro_batch_connect(lastro_batch* b, const void* handles, int32_t bytes_each) {
    if (!b) return LASTRO_E_ARG;
    if (b->connected) return set_err(b->ctx, LASTRO_E_STATE, "batch already connected");
    if (b->world > 1 && (!handles || bytes_each < (int)sizeof(cudaIpcMemHandle_t)))
        return set_err(b->ctx, LASTRO_E_ARG, "connect: %d handles of %d bytes", b->world, bytes_each);
    cudaSetDevice(b->ctx->device);
    std::vector<unsigned char*> peers(b->world, nullptr);
    for (int q = 0; q < b->world; ++q) {
        if (q == b->rank) {
            peers[q] = b->xreg;
            continue;
        }
        cudaIpcMemHandle_t h;
        memcpy(&h, static_cast<const unsigned char*>(handles) + (size_t)q * bytes_each, sizeof h);
        void* p = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            cudaGetLastError();
            for (void* o : b->opened) cudaIpcCloseMemHandle(o);
            b->opened.clear();
            return set_err(b->ctx, LASTRO_E_CUDA, "connect to rank %d: %s", q, cudaGetErrorString(e));
        }
        b->opened.push_back(p);
        peers[q] = static_cast<unsigned char*>(p);
    }
    cudaError_t e = cudaMemcpyAsync(b->d_peers, peers.data(), sizeof(unsigned char*) * b->world, cudaMemcpyHostToDevice,
                                    b->ctx->stream);
    if (!e) e = cudaStreamSynchronize(b->ctx->stream);
    if (e) return bfail(b, e, "connect");
    b->connected = true;
    return LASTRO_OK;
}

extern "C" int lastro_batch_set_router_bias(lastro_batch* b, const float* bias) {
    if (!b) return LASTRO_E_ARG;
    if (b->poisoned) return set_err(b->ctx, LASTRO_E_POISONED, "batch unusable after an earlier error");
    cudaSetDevice(b->ctx->device);
    if (bias) {
        BTRY(cudaMemcpyAsync(b->bias, bias, sizeof(float) * b->m->d.layers * b->m->d.experts, cudaMemcpyHostToDevice,
                             b->ctx->stream),
             "bias upload");
        BTRY(cudaStreamSynchronize(b->ctx->stream), "bias upload");
    }
    if ((bias != nullptr) != b->has_bias) {  // the captured graphs read the flag at capture time
        for (auto& g : b->graphs) cudaGraphExecDestroy(g.second);
        b->graphs.clear();
    }
    b->has_bias = bias != nullptr;
    return LASTRO_OK;
}

extern "C" int lastro_batch_set_expert_placement(lastro_batch* b, const int32_t* owner, int32_t n_experts) {
    if (!b) return LASTRO_E_ARG;
    if (b->poisoned) return set_err(b->ctx, LASTRO_E_POISONED, "batch unusable after an earlier error");
    const int E = b->m->d.experts;
    if (!owner || n_experts != E)
        return set_err(b->ctx, LASTRO_E_ARG, "placement of %d experts, the model has %d", n_experts, E);
    std::vector<int> per(b->world, 0);
    for (int x = 0; x < E; ++x) {
        if (owner[x] < 0 || owner[x] >= b->world)
            return set_err(b->ctx, LASTRO_E_ARG, "expert %d placed on rank %d of %d", x, owner[x], b->world);
        ++per[owner[x]];
    }
    for (int r = 0; r < b->world; ++r)
        if (per[r] != b->epr)
            return set_err(b->ctx, LASTRO_E_ARG, "rank %d gets %d experts, every rank must get %d", r, per[r], b->epr);
    cudaSetDevice(b->ctx->device);
    Placement pl;
    pl.owner.assign(owner, owner + E);
    BTRY(cudaStreamSynchronize(b->ctx->stream), "placement");  // no step in flight reads the tables
    BTRY(upload_placement(b, pl), "placement upload");
    BTRY(cudaStreamSynchronize(b->ctx->stream), "placement upload");
    return LASTRO_OK;
}

extern "C" int lastro_batch_step(lastro_batch* b, int32_t n, const int32_t* seq_ids, const int32_t* tokens,
                                 int32_t* next, float* logits, int32_t* route_ids) {
    if (!b) return LASTRO_E_ARG;
    int rc = bready(b);
    if (rc) return rc;
    cudaSetDevice(b->ctx->device);
    if ((rc = bstage(b, n, seq_ids, tokens, 1))) return rc;
    const bool hist = route_ids != nullptr;
    if (hist != b->want_hist) {
        for (auto& g : b->graphs) cudaGraphExecDestroy(g.second);
        b->graphs.clear();
        b->want_hist = hist;
    }
    if ((rc = run_bstep(b, n))) return rc;
    cudaStream_t s = b->ctx->stream;
    const lastro_model_desc& d = b->m->d;
    if (next) BTRY(cudaMemcpyAsync(next, b->d_next, sizeof(int) * n, cudaMemcpyDeviceToHost, s), "next download");
    if (logits)
        BTRY(cudaMemcpyAsync(logits, b->logits, sizeof(float) * n * d.vocab, cudaMemcpyDeviceToHost, s), "logits download");
    if (route_ids)
        BTRY(cudaMemcpyAsync(route_ids, b->route_hist, sizeof(int) * n * d.layers * d.k, cudaMemcpyDeviceToHost, s),
             "routes download");
    if ((rc = bfinish(b, "batch step"))) return rc;
    for (int i = 0; i < n; ++i) b->pos_host[seq_ids[i]] += 1;
    return LASTRO_OK;
}

extern "C" int lastro_batch_decode(lastro_batch* b, int32_t n, const int32_t* seq_ids, const int32_t* tokens,
                                   int32_t steps, int32_t* out_ids) {
    if (!b) return LASTRO_E_ARG;
    int rc = bready(b);
    if (rc) return rc;
    if (steps < 0) return set_err(b->ctx, LASTRO_E_ARG, "steps %d", steps);
    cudaSetDevice(b->ctx->device);
    if ((rc = bstage(b, n, seq_ids, tokens, steps))) return rc;
    if (b->want_hist) {
        for (auto& g : b->graphs) cudaGraphExecDestroy(g.second);
        b->graphs.clear();
        b->want_hist = false;
    }
    cudaStream_t s = b->ctx->stream;
    for (int i = 0; i < steps; ++i) {
        if ((rc = run_bstep(b, n))) return rc;
        if (out_ids && i < b->max_len)
            BTRY(cudaMemcpyAsync(b->d_hist + (size_t)i * n, b->d_next, sizeof(int) * n, cudaMemcpyDeviceToDevice, s),
                 "history");
    }
    if (out_ids && steps > 0)
        BTRY(cudaMemcpyAsync(out_ids, b->d_hist, sizeof(int) * (size_t)steps * n, cudaMemcpyDeviceToHost, s), "ids");
    if ((rc = bfinish(b, "batch decode"))) return rc;
    for (int i = 0; i < n; ++i) b->pos_host[seq_ids[i]] += steps;
    return LASTRO_OK;
}

extern "C" int lastro_batch_fill_kv_synthetic(lastro_batch* b, int32_t seq, int32_t n, uint64_t seed, float sd) {
    if (!b) return LASTRO_E_ARG;
    if (b->poisoned) return set_err(b->ctx, LASTRO_E_POISONED, "batch unusable after an earlier error");
    if (seq < 0 || seq >= b->max_seqs || n < 0 || n > b->max_len)
        return set_err(b->ctx, LASTRO_E_ARG, "fill_kv_synthetic: sequence %d, %d positions", seq, n);
    cudaSetDevice(b->ctx->device);
    const lastro_model_desc& d = b->m->d;
    const size_t per_seq = (size_t)b->max_pages * kPageSize * b->m->kvd;  // elements of one sequence's pages
    const float sc = synth_scale(sd);
    cudaStream_t s = b->ctx->stream;
    for (int l = 0; l < d.layers; ++l) {
        const uint64_t sk = mix64_host(seed + 2 * (uint64_t)l + 1000003u * (uint64_t)seq);
        const uint64_t sv = mix64_host(seed + 2 * (uint64_t)l + 1 + 1000003u * (uint64_t)seq);
        const size_t elems = (size_t)((n + kPageSize - 1) / kPageSize) * kPageSize * b->m->kvd;
        if (d.kv_dtype == LASTRO_DTYPE_F32) {
            BTRY(launch_synth_f32(static_cast<float*>(b->kpool[l]) + seq * per_seq, elems, sk, sc, s), "kv fill");
            BTRY(launch_synth_f32(static_cast<float*>(b->vpool[l]) + seq * per_seq, elems, sv, sc, s), "kv fill");
        } else {
            BTRY(launch_synth_bf16(static_cast<uint16_t*>(b->kpool[l]) + seq * per_seq, elems, sk, sc, 0.0f, s), "kv fill");
            BTRY(launch_synth_bf16(static_cast<uint16_t*>(b->vpool[l]) + seq * per_seq, elems, sv, sc, 0.0f, s), "kv fill");
        }
    }
    BTRY(cudaMemcpyAsync(b->d_pos + seq, &n, sizeof(int), cudaMemcpyHostToDevice, s), "position");
    BTRY(cudaStreamSynchronize(s), "kv fill");
    b->pos_host[seq] = n;
    return LASTRO_OK;
}

extern "C" int lastro_batch_reset(lastro_batch* b, int32_t seq) {
    if (!b) return LASTRO_E_ARG;
    if (b->poisoned) return set_err(b->ctx, LASTRO_E_POISONED, "batch unusable after an earlier error");
    if (seq < 0 || seq >= b->max_seqs) return set_err(b->ctx, LASTRO_E_ARG, "sequence %d", seq);
    cudaSetDevice(b->ctx->device);
    const int zero = 0;
    BTRY(cudaMemcpyAsync(b->d_pos + seq, &zero, sizeof(int), cudaMemcpyHostToDevice, b->ctx->stream), "reset");
    BTRY(cudaStreamSynchronize(b->ctx->stream), "reset");
    b->pos_host[seq] = 0;
    return LASTRO_OK;
}

extern "C" int lastro_batch_position(const lastro_batch* b, int32_t seq, int32_t* pos) {
    if (!b || !pos || seq < 0 || seq >= b->max_seqs) return LASTRO_E_ARG;
    *pos = b->pos_host[seq];
    return LASTRO_OK;
}

extern "C" int lastro_batch_profile(lastro_batch* b, int32_t n, const int32_t* seq_ids, const int32_t* tokens,
                                    int32_t steps, float* kernel_ms, int32_t n_kinds) {
    if (!b || !kernel_ms || n_kinds < BK_COUNT || steps < 1) return LASTRO_E_ARG;
    int rc = bready(b);
    if (rc) return rc;
    cudaSetDevice(b->ctx->device);
    if ((rc = bstage(b, n, seq_ids, tokens, steps))) return rc;
    cudaStream_t s = b->ctx->stream;
    std::vector<cudaEvent_t> ev;
    std::vector<int> kind;
    cudaEvent_t start;
    BTRY(cudaEventCreate(&start), "profile");
    for (int k = 0; k < n_kinds; ++k) kernel_ms[k] = 0.0f;
    cudaError_t e = cudaSuccess;
    for (int i = 0; i < steps && e == cudaSuccess; ++i) {
        ev.clear();
        kind.clear();
        b->prof_ev = &ev;
        b->prof_kind = &kind;
        e = cudaEventRecord(start, s);
        if (e == cudaSuccess) e = enqueue_bstep(b, n, s);
        b->prof_ev = nullptr;
        b->prof_kind = nullptr;
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        cudaEvent_t prev = start;
        for (size_t j = 0; j < ev.size() && e == cudaSuccess; ++j) {
            float ms = 0.0f;
            e = cudaEventElapsedTime(&ms, prev, ev[j]);
            kernel_ms[kind[j]] += ms / (float)steps;
            prev = ev[j];
        }
        for (cudaEvent_t x : ev) cudaEventDestroy(x);
    }
    cudaEventDestroy(start);
    if (e) return bfail(b, e, "batch profile");
    if ((rc = bfinish(b, "batch profile"))) return rc;
    for (int i = 0; i < n; ++i) b->pos_host[seq_ids[i]] += steps;
    return LASTRO_OK;
}

extern "C" int lastro_batch_trace(lastro_batch* b, int32_t n, const int32_t* seq_ids, const int32_t* tokens,
                                  int32_t steps, float* exposed_ms, float* span_ms, float* wait_ms, int32_t n_kinds,
                                  float* step_ms) {
    if (!b || steps < 1 || !exposed_ms || !span_ms || !wait_ms || !step_ms || n_kinds < BK_COUNT) return LASTRO_E_ARG;
    int rc = bready(b);
    if (rc) return rc;
    cudaSetDevice(b->ctx->device);
    if ((rc = bstage(b, n, seq_ids, tokens, steps))) return rc;
    cudaStream_t s = b->ctx->stream;
    const int L = b->m->d.layers, launches = bstep_launches(b);
    const size_t words = (size_t)launches * kTraceMaxCtas * kTraceWords;
    if (!b->d_trace) BTRY(b->arena.alloc(&b->d_trace, words), "trace buffer");
    // the product step's launches with the stamps on, captured like the product graph (a fresh capture per call)
    cudaGraph_t g = nullptr;
    cudaGraphExec_t x = nullptr;
    BTRY(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal), "begin capture");
    cudaError_t e = cudaMemsetAsync(b->d_trace, 0, words * sizeof(unsigned long long), s);
    if (e == cudaSuccess) e = enqueue_bstep(b, n, s, b->d_trace);
    cudaError_t e2 = cudaStreamEndCapture(s, &g);
    if (e == cudaSuccess) e = e2;
    if (e == cudaSuccess) e = cudaGraphInstantiate(&x, g, 0);
    if (g) cudaGraphDestroy(g);
    if (e != cudaSuccess) return bfail(b, e, "batch trace capture");
    std::vector<int> kind(launches);
    kind[0] = BK_NORM;
    const int k8[8] = {BK_QKV, BK_ROPE, BK_ATTN, BK_OPROJ, BK_ROUTER, BK_GATE_UP, BK_DOWN, BK_COMBINE};
    for (int l = 0; l < L; ++l)
        for (int i = 0; i < 8; ++i) kind[1 + 8 * l + i] = k8[i];
    kind[launches - 2] = BK_LM_HEAD;
    kind[launches - 1] = BK_ARGMAX;
    std::vector<unsigned long long> h(words);
    std::vector<double> ex(BK_COUNT, 0.0), sp(BK_COUNT, 0.0), wt(BK_COUNT, 0.0);
    double step_acc = 0.0;
    for (int st = 0; st < steps && e == cudaSuccess; ++st) {
        e = cudaGraphLaunch(x, s);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(h.data(), b->d_trace, words * sizeof(unsigned long long), cudaMemcpyDeviceToHost, s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) break;
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
            if (t0 == ~0ull) continue;  // a launch without stamps (the non-default GEMM and attention forms)
            if (rel == ~0ull) rel = t0;
            first = std::min(first, t0);
            last = std::max(last, t1);
            const unsigned long long from = prev_end ? prev_end : t0;
            ex[kind[i]] += t1 > from ? (double)(t1 - from) : 0.0;
            sp[kind[i]] += (double)(t1 - t0);
            wt[kind[i]] += prev_end && rel > prev_end ? (double)(rel - prev_end) : 0.0;
            prev_end = std::max(prev_end, t1);
        }
        if (last > first && first != ~0ull) step_acc += (double)(last - first);
    }
    cudaGraphExecDestroy(x);
    if (e != cudaSuccess) return bfail(b, e, "batch trace");
    if ((rc = bfinish(b, "batch trace"))) return rc;
    b->trace_host.swap(h);
    for (int i = 0; i < n; ++i) b->pos_host[seq_ids[i]] += steps;
    for (int k = 0; k < n_kinds; ++k) exposed_ms[k] = span_ms[k] = wait_ms[k] = 0.0f;
    for (int k = 0; k < BK_COUNT; ++k) {
        exposed_ms[k] = (float)(ex[k] / steps * 1e-6);
        span_ms[k] = (float)(sp[k] / steps * 1e-6);
        wait_ms[k] = (float)(wt[k] / steps * 1e-6);
    }
    *step_ms = (float)(step_acc / steps * 1e-6);
    return LASTRO_OK;
}

extern "C" int lastro_batch_trace_raw(const lastro_batch* b, int32_t launch, unsigned long long* out, int32_t words) {
    if (!b || !out || launch < 0) return LASTRO_E_ARG;
    const size_t per = (size_t)kTraceMaxCtas * kTraceWords;
    if ((size_t)(launch + 1) * per > b->trace_host.size() || (size_t)words < per) return LASTRO_E_ARG;
    memcpy(out, b->trace_host.data() + (size_t)launch * per, per * sizeof(unsigned long long));
    return LASTRO_OK;
}

extern "C" int lastro_batch_set_options(lastro_batch* b, int32_t use_graphs, int32_t use_tcgen05, int32_t attn_tc) {
    if (!b) return LASTRO_E_ARG;
    if (attn_tc && b->kvmaps.empty())
        return set_err(b->ctx, LASTRO_E_UNSUPPORTED, "tensor-core attention needs bf16 KV and TMA page maps");
    if (use_tcgen05 < 0 || use_tcgen05 > 2) return set_err(b->ctx, LASTRO_E_ARG, "GEMM mode %d", use_tcgen05);
    if (use_tcgen05 == 2 && b->wmaps.empty())
        return set_err(b->ctx, LASTRO_E_UNSUPPORTED, "no weight tensor maps (TMA unavailable)");
    b->use_graphs = use_graphs != 0;
    if (use_tcgen05 != b->gemm_mode || (attn_tc != 0) != b->attn_tc) {  // the captured graphs hold the other kernels
        for (auto& g : b->graphs) cudaGraphExecDestroy(g.second);
        b->graphs.clear();
    }
    b->gemm_mode = use_tcgen05;
    b->attn_tc = attn_tc != 0;
    return LASTRO_OK;
}

extern "C" int lastro_batch_set_wait_limit(lastro_batch* b, uint64_t wait_ns) {
    if (!b) return LASTRO_E_ARG;
    if (wait_ns < 1000000ull || wait_ns > 600ull * 1000 * 1000 * 1000)
        return set_err(b->ctx, LASTRO_E_ARG, "wait limit %llu ns outside [1 ms, 600 s]", (unsigned long long)wait_ns);
    cudaSetDevice(b->ctx->device);
    cudaStreamSynchronize(b->ctx->stream);
    if (wait_ns != b->wait_ns) {  // the captured graphs hold the old limit in their kernel arguments
        for (auto& g : b->graphs) cudaGraphExecDestroy(g.second);
        b->graphs.clear();
    }
    b->wait_ns = wait_ns;
    return LASTRO_OK;
}

extern "C" void lastro_batch_destroy(lastro_batch* b) {
    if (!b) return;
    cudaSetDevice(b->ctx->device);
    cudaStreamSynchronize(b->ctx->stream);
    for (auto& g : b->graphs) cudaGraphExecDestroy(g.second);
    for (void* p : b->opened) cudaIpcCloseMemHandle(p);
    if (b->h_seq) cudaFreeHost(b->h_seq);
    if (b->h_tok) cudaFreeHost(b->h_tok);
    if (b->h_err) cudaFreeHost(b->h_err);
    b->arena.release();
    lastro_ctx* ctx = b->ctx;
    delete b;
    ctx_release(ctx);
}
