// Kernel arguments and launchers of the batched decode step (many independent sequences, one token each), with the
// MoE experts partitioned over the ranks of an expert-parallel group.
//
// Per layer, on every rank for its own tokens:
//   gemm         [q;k;v] partial sums over K slices (split-K)
//   rope_kv      slices summed in order -> RoPE -> q; K/V appended to each sequence's paged cache
//   attention    bf16 KV: streaming tensor-core kernel, CTA per (KV head, token) over TMA-loaded pages (context
//                splits with an in-order merge when a rank holds few tokens); f32 KV: CUDA-core split kernel;
//                writes att split into hi + lo
//   gemm         o-projection partial sums over K slices
//   router       h += resid * sum of the slices; RMSNorm(h) -> router GEMV (+ bias) -> top-k -> softmax; then the
//                token's xn row (hi + lo) is pushed once to the exchange region of every rank owning one of its experts;
//                the grid's last CTA then waits for every rank's dispatch and groups the received pairs by local
//                expert, in (sender, pair) order
//   gemm         gate_up of every local expert on its pairs, SwiGLU in the epilogue -> a hi + lo
//   gemm         down of every local expert; the epilogue writes each result row into the combine rows of the
//                pair's sender (peer memory)
//   combine      h += resid * sum_j w_j y_j, slots in routing order; then the next layer's attention norm (or the
//                final norm) -> xn hi + lo
// (layer 0's attention norm runs on the embedding rows first) and the step ends with the tied lm_head GEMM and a
// per-token argmax.
//
// The GEMMs run on the tensor cores with bf16 operands and f32 accumulators: tcgen05 with the accumulator in tensor
// memory (default: warp-specialised, TMA weight tiles) or mma.sync.  The weights are bf16 and each f32 activation x is
// split into hi = bf16(x) and lo = bf16(x - hi), both multiplied (x - hi - lo is below 2^-17 |x|), so the products
// carry f32-level accuracy rather than bf16 rounding of the activations.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace lastro {

constexpr int kBTok = 64;         // tokens of one GEMM tile (a CTA loops over tiles)
constexpr int kBRows = 128;       // weight rows of one GEMM CTA (SwiGLU: 64 gate rows + the 64 matching up rows)
constexpr int kBK = 64;           // K of one pipeline stage
constexpr int kBStages = 3;
constexpr size_t kBStageBytes = (size_t)kBRows * kBK * 2 + 2 * (size_t)kBTok * kBK * 2;  // 32 KB
constexpr size_t kBGemmSmem = kBStages * kBStageBytes;
constexpr int kBMaxSlots = 4096;  // pairs one rank may receive in one layer (world * tokens per rank * k)
constexpr int kBMaxRanks = 32;    // ranks of one expert-parallel group

// Exchange region of one rank (the same layout on every rank; every rank maps every other rank's region):
//   rx      [world][cap_tok] token rows, each bf16 hi [H] then lo [H] (written by the senders, once per owner)
//   rx_ids  [world][cap] expert of each pair                       (written by the senders)
//   rx_n    [world] tokens of each sender in this layer           (written by the senders)
//   cb      [cap] f32 [H] result rows of this rank's pairs        (written by the owners)
//   flags   [2][world] u32, 128 bytes apart: dispatch, return     (written with release stores by the peers)
struct XLayout {
    size_t rx, rx_ids, rx_n, cb, flags, bytes;
    int cap;      // pairs per sender: tokens per rank * k
    int cap_tok;  // tokens per sender
};

XLayout x_layout(int world, int tokens_per_rank, int k, int H);

struct BExchangeArgs {
    unsigned char* const* peers;  // [world] exchange region of every rank (this rank's own at [rank])
    XLayout lay;
    int rank, world;
    int experts_per_rank;
    const int* owner;             // [world * experts_per_rank] rank that computes each expert
    const int* local;             // [same] the expert's index among its owner's experts (ascending expert ids)
    const unsigned int* epoch_base;  // flags carry epoch_base + layer + 1
    int layer;
    int* err;
    unsigned long long wait_ns;   // bound of every flag wait (lastro_batch_set_wait_limit)
    unsigned int* counter;        // last-CTA election, zero between launches
    int n, k, H;
    // group (owner): outputs for the grouped GEMMs and the return
    int* x_rows;                  // [positions] -> rx token row (sender * cap_tok + token)
    int* src;                     // [positions] -> pair (sender * cap + pair), for the return
    int* g_off;                   // [experts_per_rank]
    int* g_cnt;
    int* n_pos;                   // [1]
    // combine (sender), then the next norm: xn = ln_next * (h * r) split into hi + lo (ln_next null: none)
    float* h;                     // [n, H]
    const float* weights;         // [n, k]
    float resid;
    const float* ln_next;
    float eps;
    uint16_t* xn_hi;
    uint16_t* xn_lo;
    unsigned long long* trace;    // optional: CtaTrace stamps of the combine launch (lastro_batch_trace)
};

enum BEpi { BEPI_STORE = 0, BEPI_SWIGLU = 1, BEPI_RETURN = 2 };

struct BGemmArgs {
    const uint16_t* w;        // bf16 [groups][rows][K]
    long long group_stride;   // elements between groups
    int group0;               // first group of this launch (no group_expert)
    const int* group_expert;  // optional [groups]: weight group of launch group g (null: group0 + g)
    int rows, K, k_split;     // k_split: K of one grid-z slice (multiple of kBK)
    const uint16_t* x_hi;     // activation rows, bf16 hi / lo, row stride ldx elements
    const uint16_t* x_lo;
    int ldx;
    const int* x_rows;        // optional: position -> activation row (null: the position itself)
    const int* g_off;         // optional (grouped): per group first position and count; null: positions 0..n-1
    const int* g_cnt;
    int n;
    // BEPI_STORE: y[z * z_stride + pos * ldy + row] = acc / div (div 1: acc as is)
    float* y;
    int ldy;
    long long z_stride;
    float div;
    // BEPI_SWIGLU: a[pos * I + r] = silu(gate_r) * up_r, split into hi + lo (gate rows r, up rows I + r)
    uint16_t* a_hi;
    uint16_t* a_lo;
    int I;
    // BEPI_RETURN: row block of position pos to the combine rows of its sender (x.src[pos]), then the grid's last
    // CTA publishes this rank's return flag on every rank
    BExchangeArgs x;
    // 0: mma.sync (register accumulators); 1: tcgen05, all threads load the stages with cp.async; 2: tcgen05,
    // warp-specialised: weight tiles by TMA (the launch's tensor map), activation tiles by two cp.async warps, one
    // thread issuing the MMAs
    int tc;
    unsigned long long* trace;    // optional: CtaTrace stamps of this launch (lastro_batch_trace)
};

struct BNormArgs {
    float* h;                  // [n, H] residual stream (written in embed mode)
    const uint16_t* embed;     // embed mode: [V, H] bf16, rows tokens[t]
    const int* tokens;
    float emb_mult;
    const float* ln;           // [H]
    float eps;
    uint16_t* x_hi;            // [n, H]
    uint16_t* x_lo;
    int H;
    unsigned long long* trace;    // optional: CtaTrace stamps of this launch (lastro_batch_trace)
};

struct BRopeArgs {
    const float* part;         // [ks][n][qd + 2 kvd] partial sums
    int ks;
    const int* seq;            // [n] sequence of each token
    const int* pos;            // [sequences] position of the current token
    const int* off;            // optional [n]: token z writes position pos[seq[z]] + off[z] (a multi-position step)
    const float* rope_cs;      // [max_len, d]
    float* q;                  // [n, qd]
    void* k_pool;              // [pages, kv_heads, page, d]
    void* v_pool;
    const int* page_table;     // [sequences, pt_stride]
    int pt_stride, page_size, kv_f32;
    int n, qd, kvd, d, kv_heads;
    unsigned long long* trace;    // optional: CtaTrace stamps of this launch (lastro_batch_trace)
};

struct BRouterArgs {
    float* h;                  // [n, H], updated: h += resid * sum_z opart[z]
    const float* opart;        // [ks][n][H]
    int ks;
    float resid;
    const float* ln;           // MoE norm [H]
    float eps;
    const uint16_t* wr;        // [E, H] bf16
    const float* bias;         // [E] or null
    BExchangeArgs x;           // dispatch of the MoE input rows
    int* ids;                  // [n, k]
    float* weights;            // [n, k]
    int* route_hist;           // optional [n][layers][k] history of the step
    int layer, layers;
    int n, H, E, k;
    unsigned long long* trace;    // optional: CtaTrace stamps of this launch (lastro_batch_trace)
};

struct BHeadArgs {
    const float* logits;          // [n, V]
    int V, n;
    const int* seq;
    int* pos;                     // incremented per token's sequence
    const int* off;               // optional [n] (a multi-position step: several tokens of one sequence)
    int* next;                    // [n] argmax (last maximum)
    int* tokens;                  // optional: next token fed back as the next step's input
    unsigned int* epoch_base;     // advanced by `layers` (CTA 0)
    int layers;
    unsigned long long* trace;    // optional: CtaTrace stamps of this launch (lastro_batch_trace)
};

// Batched decode attention: CTA per (split, KV head, token) over the token's sequence; splits of at most kBAttnRows
// positions (S = ceil(max_len / kBAttnRows) splits), staged to shared memory with bulk copies; the last CTA of each
// (token, KV head) merges the S partials.
constexpr int kBAttnRows = 128;
constexpr int kBAttnMaxSplits = 32;

struct BAttnArgs {
    const float* q;            // [n][heads * d] roped queries
    const void* k_pool;        // [pages][kv_heads][page][d]
    const void* v_pool;
    const int* page_table;     // [sequences][pt_stride]
    int pt_stride, page_size, kv_f32;
    const int* seq;            // [n] (null: one token, sequence 0)
    const int* pos;            // [sequences]: the token attends positions 0..pos (+ off[z])
    const int* off;            // optional [n]: token z sits off[z] positions past its sequence's position
    float* part_acc;           // [n][heads][S][d]
    float* part_ml;            // [n][heads][S][2]
    unsigned int* counters;    // [n][kv_heads], zero between launches
    float* att_out;            // [n][heads * d]
    uint16_t* att_hi;          // [n][heads * d] split of att_out (null: not written)
    uint16_t* att_lo;
    int* err;
    int n, kv_heads, G, S, cap;  // cap: positions one split stages (>= ceil(max_len / S))
    float scale;
    unsigned long long* trace;    // optional: CtaTrace stamps of this launch (lastro_batch_trace)
};

cudaError_t launch_battention(const BAttnArgs& a, cudaStream_t s);
// bf16 KV on tensor cores: CTA per (KV head, token) streaming the context's pages by TMA through `kmap` / `vmap`
// (make_kv_map over the layer's pools); positions past the context must hold finite values (zeroed pools)
cudaError_t launch_battention_tc(const BAttnArgs& a, const CUtensorMap* kmap, const CUtensorMap* vmap, cudaStream_t s);
cudaError_t make_kv_map(CUtensorMap* map, const void* pool, uint64_t rows);
size_t battn_smem(int cap, int kv_f32);

// `wmap` (mode 2): 2-D bf16 tensor map over the weight rows [groups * rows][K], box 64 columns x 64 rows, 128-byte
// swizzle (make_weight_map)
cudaError_t launch_bgemm(const BGemmArgs& a, int epi, int groups, cudaStream_t s, const CUtensorMap* wmap = nullptr);
// host: tensor map for launch_bgemm's mode 2 over a row-major bf16 matrix [rows][cols]
cudaError_t make_weight_map(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols);
// the same with boxes of box_rows rows (<= 256) x 64 columns
cudaError_t make_tile_map(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows);
// bf16 KV pool as rows of one head's position (64 columns) in boxes of 8 rows, 128-byte swizzle: the batch-1
// attention's staging (AttnArgs::tma)
cudaError_t make_kv_box_map(CUtensorMap* map, const void* pool, uint64_t rows);
cudaError_t launch_battn_norm(const BNormArgs& a, int n, cudaStream_t s);
cudaError_t launch_brope_kv(const BRopeArgs& a, cudaStream_t s);
cudaError_t launch_brouter(const BRouterArgs& a, cudaStream_t s);
cudaError_t launch_ep_combine(const BExchangeArgs& a, cudaStream_t s);
cudaError_t launch_bargmax(const BHeadArgs& a, cudaStream_t s);

}  // namespace lastro
