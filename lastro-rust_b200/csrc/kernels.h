// Kernel arguments and host-side launchers of the batch-1 Granite-MoE decode step.
//
// One decode step of layer l is six kernels, each a single pass over its weights:
//   qkv_rope     RMSNorm(h) -> [q;k;v] GEMV -> RoPE(q,k) -> K/V appended to the paged cache
//   attention    split-KV GQA decode attention; the last CTA of each KV head merges the splits
//   oproj        h += resid * (W_o . att)
//   router       RMSNorm(h) -> router GEMV -> top-k (lowest index on ties) -> softmax over k
//   gate_up      a[j] = silu(W_g x) * (W_u x) for the k chosen experts, grouped in one launch
//   down         h += resid * sum_j w_j (W_d[e_j] . a_j), experts summed in routing order
// and the step ends with
//   head         RMSNorm(h) -> tied-embedding GEMV / logits_scaling -> argmax (last max on ties)
// All activations are f32, weights bf16, accumulators f32.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace lastro {

// in-graph timeline: CTAs per launch that stamp their three words (CtaTrace in common.cuh)
constexpr int kTraceMaxCtas = 1024;
constexpr int kTraceMarks = 8;
constexpr int kTraceWords = 3 + kTraceMarks;  // per CTA: start, release, end, milestones

// Linear weights are bf16 ([rows, cols] row-major) or Q8_0.  A Q8_0 row on the device is its cols int8 values, then its
// cols/32 fp16 block scales, padded to a multiple of 16 bytes (so rows stay 16-byte aligned for bulk copies); weight =
// scale * value.  `q8` in the argument structs below selects the Q8_0 kernels.
__host__ __device__ inline size_t wrow_bytes(int cols, int q8) {
    return q8 ? (((size_t)cols + (size_t)cols / 16 + 15) & ~(size_t)15) : (size_t)cols * 2;
}

struct QkvArgs {
    const float* h;        // residual stream [H] (ignored when embed_mode)
    float* h_write;        // embed_mode: CTA 0 writes the embedding row x multiplier here
    const uint16_t* embed; // [V, H] bf16 (embed_mode)
    const int* token;      // device token id (embed_mode)
    float emb_mult;
    int embed_mode;
    const float* ln;       // [H]
    const void* w;         // [qd + 2 kvd, H] (bf16 or Q8_0 rows): q rows, k rows, v rows
    int q8;
    const float* rope_cs;  // [max_len, d]: cos(d/2) then sin(d/2) per position
    const int* pos;        // device position of the token
    float* q_out;          // [qd] roped q
    void* k_pool;          // [pages, kv_heads, page, d]
    void* v_pool;
    const int* page_table; // [max_pages]
    int page_size, kv_f32;
    int H, qd, kvd, d, kv_heads;
    float eps;
    unsigned long long* trace;  // in-graph timeline stamps of this launch (CtaTrace), or null
    // optional: the routing predicted from this layer's input, for the gate_up kernel's early staging: CTA c < spec_E
    // writes spec_out[c] = sum_i router[c][i] * ln_moe[i] * h[i] (the router logit of h itself; the MoE block's input
    // is h after this layer's attention, normalised by a positive factor that leaves the order of the logits as is)
    const uint16_t* spec_router;  // [E, H] bf16 router rows, or null
    const float* spec_ln;         // [H] MoE norm weight
    float* spec_out;              // [E]
    int spec_E;
    // optional: the step counter the routing hand-off of gate_up to down is stamped with (GateUpArgs route_flag);
    // the embedding launch (embed_mode, the first kernel of every step) advances it
    unsigned int* step_ctr;
    // optional (with spec_out): the last of the spec_E CTAs (ticket) also takes the top spec_k of the predicted
    // logits into spec_ids, for the attention kernel's L2 hints (AttnArgs spec_ids)
    int* spec_ids;
    unsigned int* spec_ticket;  // zero between launches
    int spec_k;
};

struct AttnArgs {
    const float* q;          // [heads*d]
    const void* k_pool;
    const void* v_pool;
    const int* page_table;
    int page_size, kv_f32;
    const int* pos;          // attends positions 0..pos
    float* part_acc;         // [heads, kAttnSplits, d]: per-split unnormalised outputs
    float* part_ml;          // [heads, kAttnSplits, 2]: per-split running max and sum of exponentials
    unsigned int* counters;  // [kv_heads], zero between launches
    float* att_out;          // [heads * d], merged by the last CTA of each KV head
    int* err;
    int kv_heads, G, d;
    int max_len, split_cap;  // split_cap = attn_split_cap(max_len, splits): K/V rows one CTA stages
    int splits;              // context splits (grid x): 8 or 16
    int merge;               // 1: the last CTA of each KV head merges the splits into att_out; 0: the partials are
                             // left for the output projection (OprojArgs part_acc)
    int cluster;             // 1: the splits of a KV head form a thread-block cluster that merges them in distributed
                             // shared memory (splits <= 8; batch-1 only)
    int mma;                 // 1: bf16 K/V scored and summed on tensor cores (mma.sync, q and p split into bf16 hi + lo),
                             // else on CUDA cores in f32
    // optional: the experts predicted for this layer (QkvArgs spec_ids, final when this kernel is released): every CTA
    // hints its share of their gate_up and down weights into L2 while the attention and the output projection run
    const int* spec_ids;
    int spec_k, spec_E;
    const void* spec_gu;  // [E, 2I, H] rows: spec_gu_bytes per expert
    const void* spec_dn;  // [E, H, I] rows: spec_dn_bytes per expert
    unsigned long long spec_gu_bytes, spec_dn_bytes;
    int tma;                 // 1: bf16 K/V staged by 8-row TMA boxes with the 128-byte swizzle (launch_attention's maps:
                             // make_kv_box_map over the layer's pools; page_size a multiple of 8), else bulk copies
    float scale;
    // batched decode (grid z = the launch's tokens, null seq = batch-1): token z reads q and writes att_out at
    // z * heads * d and its partials/counters at its own offsets, and attends the cache of sequence seq[z] (page-table
    // row seq[z] of pt_stride entries, position pos[seq[z]])
    const int* seq;
    int tokens, pt_stride;
    uint16_t* att_hi;  // optional: att_out split into bf16 hi + lo (the batched o-projection's operands)
    uint16_t* att_lo;
    unsigned long long* trace;  // in-graph timeline stamps of this launch (CtaTrace), or null
};

struct OprojArgs {
    const float* att;   // [qd]
    const void* w;      // [H, qd] (bf16 or Q8_0 rows)
    int q8;
    float* h;           // [H], updated in place
    float resid;
    int H, qd;
    // fused MoE router (route != 0): every CTA writes its rows' shares of the router logits and of sum h^2
    int route;
    const float* wr_t;      // [H, E]: router weight x MoE norm weight, transposed (launch_router_fold)
    float* shares;          // [oproj_grid(H), E + 1]
    int E;
    // optional: the attention's per-split partials (part_acc [heads, splits, d], part_ml [heads, splits, 2]), merged
    // into the attention output on load; null: att holds the merged output
    const float* part_acc;
    const float* part_ml;
    int splits, heads;
    int smem_weights;  // 1: the weight rows staged in shared memory, 256 threads (oproj_smem_kernel)
    int* err;          // error word of that kernel's bounded copy wait
    unsigned long long* trace;  // in-graph timeline stamps of this launch (CtaTrace), or null
    // optional: the predicted router logits (QkvArgs spec_out, final when this kernel starts): before
    // griddepcontrol.wait the CTAs take their top spec_k and hint the predicted experts' gate_up and down weights
    // into L2, each CTA its share, while the attention still runs
    const float* spec;
    int spec_E, spec_k;
    const void* spec_gu;  // [E, 2I, H] rows: spec_gu_bytes per expert
    const void* spec_dn;  // [E, H, I] rows: spec_dn_bytes per expert
    unsigned long long spec_gu_bytes, spec_dn_bytes;
};

// Routing of the fused path: the output projection's per-CTA shares, reduced by every CTA of the expert kernels in
// the same fixed order, so each CTA holds bitwise the same routing without another launch or cross-CTA exchange.
struct RouteShares {
    const float* shares;  // [nb, E + 1], or null when the routing comes from the router kernel (ids/weights)
    int nb;
    float eps;
    // published by CTA 0 of the gate_up kernel (the step's routing output)
    int* ids_out;
    float* weights_out;
    float* logits_out;
};

struct RouterArgs {
    const float* x;         // norm_mode: residual h; otherwise the block input
    const float* ln;        // norm weight (norm_mode)
    float eps;
    int norm_mode;
    const void* w;          // [E, H] (bf16 or Q8_0 rows)
    int q8;
    float* logits;          // [E]
    int* ids;               // [k]
    float* weights;         // [k]
    float* rnorm_out;       // norm_mode: 1/sqrt(mean(h^2)+eps) for the experts
    unsigned int* counter;  // zero between launches
    int E, H, k;
};

struct GateUpArgs {
    const float* x;       // rs.shares set: residual h (xn = ln * (h * r)); otherwise the block input
    const float* ln;      // MoE norm weight (with shares)
    const int* ids;       // [k] from the router kernel (without shares)
    RouteShares rs;
    const void* w;        // [E, 2I, H] (bf16 or Q8_0 rows)
    int q8;
    float* a;             // [k, I]
    int* err;             // error word: a bounded wait that gave up writes its code here
    int H, I, k, E;
    // optional (streaming kernel of the model step): the down weights [E, H, I], whose chosen slabs are hinted into L2
    const void* down_w;
    size_t down_row_bytes;
    int stream;  // the streaming kernel (one wave, all rows in flight): measured slower on C3, kept selectable
    unsigned long long* trace;  // in-graph timeline stamps of this launch (CtaTrace), or null
    // optional (with rs.shares): the predicted router logits (QkvArgs spec_out), final when this kernel starts.  Before
    // griddepcontrol.wait every CTA takes their top-k and stages the rows of its slot's predicted expert; after the
    // routing a CTA whose expert was predicted computes it where the routing put it, the others re-stage the experts
    // nobody predicted (the results do not depend on the prediction)
    const float* spec;
    // optional (with rs.shares): once CTA 0 has published the routing (rs.ids_out, rs.weights_out) it stamps this
    // layer's flag with the step counter, so the down kernel takes the routing instead of reducing the shares again
    unsigned int* route_flag;
    const unsigned int* step_ctr;
};

struct DownArgs {
    const float* a;        // [k, I]
    const int* ids;        // [k] from the router kernel (without shares)
    const float* weights;  // [k]
    RouteShares rs;
    const void* w;         // [E, H, I] (bf16 or Q8_0 rows)
    int q8;
    float* out;            // accumulate: h += resid*y ; else out = y
    float resid;
    int accumulate;
    int* err;
    int H, I, k, E;
    // optional: byte ranges prefetched into L2 for the kernels that follow (the next layer's dense weights)
    const void* pf[2];
    unsigned long long pf_bytes[2];
    unsigned long long* trace;  // in-graph timeline stamps of this launch (CtaTrace), or null
    // optional (with rs.shares): the routing gate_up's CTA 0 published (rs.ids_out, rs.weights_out), taken once
    // route_flag holds the step counter; a bounded wait, after which the CTA reduces the shares itself
    const unsigned int* route_flag;
    const unsigned int* step_ctr;
};

// The MoE block of the model step in one persistent launch (moe_kernel): routing from the output projection's shares,
// gate_up + SwiGLU, down + combine + residual, streamed through a ring of shared-memory stages.
struct MoeArgs {
    float* h;              // residual [H]: read for the MoE norm, updated in place (h += resid * y)
    const float* ln;       // MoE norm weight [H]
    RouteShares rs;
    const void* w_gu;      // [E, 2I, H] (bf16 or Q8_0 rows)
    const void* w_dn;      // [E, H, I]
    int q8;
    float* a;              // [k, I] SwiGLU activations (global: every CTA reads every slot's after the grid barrier)
    unsigned long long* barrier;  // grid barrier counter: zero at creation, grows by the grid size per launch
    int* err;
    float resid;
    int H, I, k, E;
    int stages, stage_bytes, gu_chunk, slots_per_chunk;  // ring geometry (moe_plan)
    const void* pf[2];                                   // optional: byte ranges hinted into L2 (the next layer's)
    unsigned long long pf_bytes[2];
    unsigned long long* trace;
};

struct MoePlan {
    int grid, stages, stage_bytes, gu_chunk, slots_per_chunk;
    size_t smem;
};
// ring geometry of moe_kernel for these shapes on the current device; false when the shapes do not fit it
bool moe_plan(int H, int I, int k, int q8, MoePlan* out);
cudaError_t launch_moe(const MoeArgs& a, const MoePlan& p, cudaStream_t s, bool pdl);

struct HeadArgs {
    const float* h;                 // [H]
    const float* ln;                // final norm [H]
    float eps;
    const uint16_t* w;              // [V, H] (tied embedding)
    float logits_scaling;
    float* logits_out;              // [V] or null
    unsigned long long* partial;    // [grid]
    unsigned int* counter;          // zero between launches
    int* token_out;                 // next token (device)
    int* out_ids;                   // history of generated ids (device) or null
    int out_cap;                    // entries of out_ids
    int* step;                      // index into out_ids
    int* pos;                       // incremented once per step
    int V, H;
    unsigned long long* trace;  // in-graph timeline stamps of this launch (CtaTrace), or null
};

// Launchers: `pdl` marks the launch as programmatic-dependent on the previous kernel of the stream.
cudaError_t launch_qkv_rope(const QkvArgs& a, cudaStream_t s, bool pdl);
cudaError_t launch_attention(const AttnArgs& a, cudaStream_t s, bool pdl, const CUtensorMap* kmap = nullptr,
                             const CUtensorMap* vmap = nullptr);
// bf16 K/V staged in 8-row boxes: a split's rows [p0, p1) with p1 - p0 < cap, widened to whole boxes, span at most
// cap + 13 rows; a multiple of 8 keeps the V rows 1024-byte aligned after the K rows
__host__ __device__ inline int attn_tma_rows(int cap) { return (cap + 20) / 8 * 8; }
cudaError_t launch_oproj(const OprojArgs& a, cudaStream_t s, bool pdl);
cudaError_t launch_router(const RouterArgs& a, cudaStream_t s, bool pdl);
int oproj_grid(int H);
cudaError_t launch_router_fold(const void* wr, int q8, const float* ln, float* wr_t, int E, int H, cudaStream_t s);
cudaError_t launch_gate_up(const GateUpArgs& a, cudaStream_t s, bool pdl);
cudaError_t launch_down(const DownArgs& a, cudaStream_t s, bool pdl);
cudaError_t launch_head(const HeadArgs& a, cudaStream_t s, bool pdl, int* grid_out);
int head_grid(int V);

// Synthetic fill (same integer formula as the CPU oracle): value(i) = (sum of four 16-bit chunks of
// mix64(seed + (i+1)*golden) - 131070) * scale (+ mean), rounded to bf16.
cudaError_t launch_synth_bf16(uint16_t* out, size_t n, uint64_t seed, float scale, float mean, cudaStream_t s);
cudaError_t launch_synth_f32(float* out, size_t n, uint64_t seed, float scale, cudaStream_t s);
// Q8_0 matrix [rows, cols] in the device row layout: int8 values uniform in [-127, 127] and fp16 block scales uniform in
// [1e-4, 4e-3) from the same integer hash as the CPU oracle's lo_synth_q8_0
cudaError_t launch_synth_q8_0(unsigned char* out, size_t rows, int cols, uint64_t seed, cudaStream_t s);
// norms: bf16(1 + value) widened to f32
cudaError_t launch_synth_norm_f32(float* out, size_t n, uint64_t seed, float scale, cudaStream_t s);
// positions [0, n) of a paged K or V pool, element for element the CPU oracle's synthetic context
cudaError_t launch_synth_kv_pages(void* pool, int kv_f32, const int* page_table, int n, int kv_heads, int d,
                                  int page_size, uint64_t seed, float scale, cudaStream_t s);

// ---- fused decode step: the whole step (every layer and the head) in one persistent cooperative launch -----------
// One CTA per SM.  Every value one CTA hands to another inside the step travels as a 64-bit word {f32 value, u32 tag}
// written with one relaxed store; the reader spins on the words themselves until every tag is the one it expects
// (the tag encodes step, layer and producing phase), so a dependency costs one round trip and no counter or flag.
// Every CTA streams the weights of its next phase into shared memory before it waits for the phase's inputs.
constexpr int kFusedThreads = 384;
constexpr int kPartStride = 66;  // attention partial per (head, split): acc[64], m, l
constexpr int kGuStages = 4;     // gate_up rows arrive in this many chunks, each on its own barrier
constexpr int kMaxHeadStages = 6;
constexpr int kExchangeKinds = 6;  // qkv, attention, merge, oproj, gate_up, down
constexpr int kCountStride = 32;   // u32 words per arrival counter (one 128-byte line each)

struct FusedLayer {
    const float* ln_attn;
    const float* ln_moe;
    const float* wr_t;  // [H, E] router weight x MoE norm weight, transposed
    const uint16_t* wqkv;
    const uint16_t* wo;
    const uint16_t* gate_up;
    const uint16_t* down;
    void* k_pool;
    void* v_pool;
};

// Work split maxima and shared-memory layout (bytes), computed on the host by fused_plan.
struct FusedLayout {
    int nb;                          // CTAs
    int qkv_pairs, rows, gu_pairs;   // per-CTA maxima: RoPE row pairs, output rows (oproj/down), gate_up pairs
    int max_splits, kv_cap;          // attention: splits per KV head (<= nb / kv_heads), K/V rows per staged chunk
    int head_rows, head_stages;      // lm_head rows per staged chunk, chunks in flight
    int off_qkv, off_kv, off_wo, off_gu, off_dn, off_head, off_f, off_own, smem;
};

// The exchange words ({value, tag}, see above) of one step, each written by one CTA and read by others.
struct FusedExchange {
    unsigned long long* h;      // [H] residual stream after the output projection and after the experts
    unsigned long long* qkv;    // [qd + 2 kvd] roped q, the new K row (as cached), the new V row
    unsigned long long* part;   // [heads, max_splits, kPartStride] attention partials
    unsigned long long* att;    // [qd] merged attention output
    unsigned long long* share;  // [nb, E + 1] router-logit shares and sum h^2 of each CTA's rows
    unsigned long long* act;    // [k, I] SwiGLU activations
};

struct FusedArgs {
    const FusedLayer* layers;  // [L] (device)
    int L;
    const uint16_t* embed;     // [V, H]
    const float* norm;         // final norm [H]
    const float* rope_cs;      // [max_len, d]
    const int* page_table;
    int page_size;
    int* pos;
    int* token;
    int* step;
    int* out_ids;
    int out_cap;
    FusedExchange x;
    float* logits;             // [V]
    int* route_ids;            // [L, k]
    float* route_w;            // [L, k]
    float* rlogits;            // [E] (last layer)
    unsigned long long* best;  // [nb]
    unsigned int* ticket;      // lm_head arrivals, monotonic
    unsigned int* count;       // [kExchangeKinds * kCountStride] arrivals per exchange kind, monotonic
    unsigned int* epoch;       // steps completed by this model's fused kernel
    int* err;
    int H, I, E, k, qd, kvd, kv_heads, G, V;
    float eps, emb_mult, resid, attn_scale, logits_scaling;
    FusedLayout lay;
};

// false when the shapes do not fit the fused kernel (the multi-kernel step is used instead); nb is the SM count
bool fused_plan(int H, int I, int E, int k, int qd, int kvd, int kv_heads, int G, int V, int kv_f32, int nb,
                FusedLayout* out);
cudaError_t launch_fused_step(const FusedArgs& a, int kv_f32, cudaStream_t s);
// CTAs of the fused kernel one SM holds with `smem` dynamic shared memory (the launch needs >= 1)
cudaError_t fused_blocks_per_sm(int H, int qd, int I, int kv_f32, int smem, int* blocks);

// limits enforced by the host before any launch
constexpr int kMaxHidden = 2048;   // H (and qd) <= 2048, multiple of 8
constexpr int kMaxInter = 2048;
constexpr int kMaxExperts = 64;
constexpr int kMaxTopK = 8;
constexpr int kHeadDim = 64;
constexpr int kMaxGroup = 8;
constexpr int kMaxHeads = kMaxHidden / kHeadDim;
constexpr size_t kMaxSmemBytes = 220 * 1024;  // dynamic shared memory one CTA may use (B200: 227 KB)

// attention: splits (CTAs) per KV head and the shared memory they stage K/V rows in
constexpr int kAttnSplits = 16;
int attn_split_cap(int max_len, int splits);
size_t attn_smem(int max_len, int kv_f32, int splits);
int attn_splits_default(int max_len, int kv_f32);

// shared memory the grouped expert kernels need (host-side checks)
size_t gate_up_smem(int H, int q8 = 0);
size_t down_smem(int H, int I, int k, int q8 = 0);
int gate_up_rows_per_cta();  // I must be a multiple
int down_rows_per_cta();     // H must be a multiple

}  // namespace lastro
