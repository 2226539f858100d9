// Fused batch-1 decode step: every layer and the lm_head in ONE persistent cooperative launch (sm_100a).
//
// Why: at batch 1 each layer moves ~55 MB (3B shape) and a kernel boundary costs about a microsecond of drain,
// launch and griddepcontrol latency on top of the ramp of the next kernel's loads; five boundaries per layer were
// most of the step.  Here one CTA per SM runs the whole step, and the phases of a layer hand their results to one
// another through exchange words: {f32 value, u32 tag} written with one 64-bit relaxed store, the tag naming the
// step (epoch), the layer and the producing phase.  A consumer spins on the words it needs until every tag is the
// expected one -- the wait and the data load are the same round trip, and no counter, flag or fence is needed
// (each word is self-validating).  A word is overwritten only by a later phase that cannot start before every
// reader of the word has produced its own output of the phase that read it (every CTA produces a share of every
// exchange: fused_plan caps the CTA count accordingly), so a reader never sees a newer tag than the one it waits for.
//
// Each CTA streams the weights of its next phase into shared memory with bulk async copies (TMA), issued by one
// producer thread, BEFORE it waits for the phase's inputs:
//
//   layer start    W_o rows (own output rows) and the router operand rows -> shared memory
//   qkv            RMSNorm(h) -> own RoPE row pairs of [q;k;v] (staged during the previous layer) -> q, new K/V row
//                  (exchange) and the K/V append to the paged cache (read by later steps)
//   attention      unit (KV head, split): own K/V rows (staged during the previous layer) + the new row; scores,
//                  online softmax and P.V across the whole CTA; partial (acc, m, l) per query head
//   merge          CTA h < heads merges the splits of query head h (flash-decoding)
//   oproj          h[own rows] += resid * W_o . att; the rows' shares of the router logits and of sum h^2
//   gate_up        routing reduced from all shares in a fixed order (bitwise the same in every CTA), then own
//                  (expert slot, row) pairs streamed in kGuStages chunks; the down rows are prefetched into L2
//   down           own output rows of the k chosen experts (staged after gate_up), h += resid * sum_j w_j d_j;
//                  meanwhile the next layer's qkv rows and K/V rows are staged
//   head           final norm, own vocabulary rows streamed through a ring of stages, argmax; the last CTA to
//                  finish (ticket) publishes the token and advances the position and the epoch
//
// Every wait is bounded (mbarrier waits and exchange polls); a wait that gives up records its code in the error
// word, drains the CTA's own copies in flight and returns; the other CTAs see the error word and return too.
//
// Reference behaviour restated (brenoperucchi/lastro-rust, rust/moe-rt/src): RMSNorm model.rs:141-145, RoPE
// rotate_half model.rs:147-158, attention model.rs:203-222, routing block.rs:79-89, SwiGLU cpu.rs:64-68, experts
// cpu.rs:115-150, step model.rs:181-243, argmax (last maximum) bin/m1b-gulosa.rs:22-24.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "ops.cuh"

namespace lastro {

namespace {

using u64 = unsigned long long;

constexpr int kFT = kFusedThreads;
constexpr int kFW = kFT / 32;
constexpr int kHalf = kHeadDim / 2;
constexpr int kProd = 32;     // the thread that arms barriers and issues the bulk copies (warp 1, lane 0)
constexpr int kPollMax = 17;  // router shares one thread polls at once (ceil(nb / (kFT / (E + 1))))

enum { B_QKV = 0, B_KV, B_WO, B_GU0, B_DN = B_GU0 + kGuStages, B_HD0, NBARS = B_HD0 + kMaxHeadStages };
enum { TG_QKV = 0, TG_ATTN, TG_MERGE, TG_OPROJ, TG_UP, TG_DOWN };

// error codes of the fused kernel's bounded waits
enum { ERR_POLL = 20, ERR_BAR = 21, ERR_DRAIN = 22 };

constexpr uint32_t kSpinLimit = 1u << 21;

// tag of the words phase `kind` of layer `l` writes in step `epoch` (never 0: fresh memory never matches)
LDEV uint32_t tag_of(uint32_t epoch, int L, int l, int kind) {
    return (epoch * (uint32_t)L + (uint32_t)l) * 8u + (uint32_t)kind + 1u;
}

LDEV void st_word(u64* p, float v, uint32_t tag) {
    const u64 w = ((u64)tag << 32) | (u64)__float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

LDEV u64 ld_word(const u64* p) {
    u64 w;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}

LDEV float word_val(u64 w) { return __uint_as_float((uint32_t)w); }
LDEV uint32_t word_tag(u64 w) { return (uint32_t)(w >> 32); }

LDEV float div_rn(float x, float y) { return __fdiv_rn(x, y); }
LDEV float sqrt_rn(float x) { return __fsqrt_rn(x); }
LDEV float exp_f(float x) { return expf(x); }

LDEV int ld_volatile_int(const int* p) { return *reinterpret_cast<const volatile int*>(p); }

LDEV unsigned ld_relaxed_u32(const unsigned* p) {
    unsigned v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Arrival counters in front of the exchange words.  Spinning on the words themselves (every CTA re-reading kilobytes
// of words per poll) floods the L2 lines they live on and stalls every CTA's memory pipeline; so a consumer spins on
// the exchange kind's counter (one word, one line) and then reads the words once.  The producer's increment is
// relaxed and unfenced: the words validate themselves by their tags, so a word that is not yet visible when the count
// is complete is simply polled again.
LDEV void arrive_count(unsigned* ctr) {
    __syncthreads();
    if (threadIdx.x == 0) atomicAdd(ctr, 1u);
}

// all threads call; every CTA arrives once per layer on every kind, so layer lp of step epoch is complete at
// (epoch * L + lp + 1) * nb arrivals
LDEV bool wait_count(const unsigned* ctr, unsigned target, int* err) {
    bool ok = true;
    if (threadIdx.x == 0) {
        for (uint32_t i = 0;; ++i) {
            if ((int)(ld_relaxed_u32(ctr) - target) >= 0) break;
            if (i >= kSpinLimit || ((i & 63u) == 63u && ld_volatile_int(err) != 0)) {
                ok = false;
                break;
            }
        }
        if (!ok) atomicCAS(err, 0, (int)ERR_POLL);
    }
    return __syncthreads_and(ok) != 0;
}

LDEV void prefetch_l2(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// shared memory last touched by ordinary loads/stores is about to be written by the async (TMA) proxy
LDEV void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

struct Range {
    int lo, hi;
};

LDEV Range split_range(int total, int c, int nb) {
    return {(int)((unsigned)(total * c) / (unsigned)nb), (int)((unsigned)(total * (c + 1)) / (unsigned)nb)};
}

__host__ __device__ __forceinline__ int round4(int n) { return (n + 3) & ~3; }

LDEV int attn_splits(int len, int max_splits) { return max(1, min(max_splits, (len + 31) / 32)); }

// CTA-uniform state: barrier parities and the barriers armed (copies issued, not yet waited on).
struct Flow {
    uint64_t* bars;
    uint32_t parity;
    uint32_t armed;
};

// all threads call with the same arguments; the producer thread arms the barrier for `bytes` (0 completes it)
LDEV void arm(Flow& f, int b, uint32_t bytes) {
    if (threadIdx.x == kProd) mbar_expect_tx(&f.bars[b], bytes);
    f.armed |= 1u << b;
}

LDEV bool bar_wait(Flow& f, int b, int* err) {
    const bool ok = mbar_wait(&f.bars[b], (f.parity >> b) & 1u, err, ERR_BAR);
    f.parity ^= 1u << b;
    f.armed &= ~(1u << b);
    return __syncthreads_and(ok) != 0;
}

// before returning on an error: wait (bounded) for every copy this CTA still has in flight
__device__ __noinline__ void drain(Flow f, int* err) {  // by value: f stays in registers
    for (int b = 0; b < NBARS; ++b)
        if (f.armed & (1u << b)) mbar_wait(&f.bars[b], (f.parity >> b) & 1u, err, ERR_DRAIN);
    f.armed = 0;
}

// Up to three segments of exchange words, concatenated: dst[i] = value of the i-th word once every word carries
// `tag`.  A thread polls PM words at a time (one round trip when n <= PM * kFT; longer exchanges are walked in
// chunks).  All threads call; false when the wait gave up (error word set).
struct Seg {
    const u64* src;
    int n;
};

template <int PM>
LDEV bool poll_words(Seg s0, Seg s1, Seg s2, uint32_t tag, float* dst, int* err) {
    const int n = s0.n + s1.n + s2.n;
    bool ok = true;
    for (int base = 0; base < n && ok; base += PM * kFT) {
        u64 w[PM];
        ok = false;
        for (uint32_t it = 0; it < kSpinLimit; ++it) {
#pragma unroll
            for (int k = 0; k < PM; ++k) {
                const int i = base + threadIdx.x + k * kFT;
                if (i < n) {
                    const u64* p = i < s0.n ? s0.src + i
                                            : (i < s0.n + s1.n ? s1.src + (i - s0.n) : s2.src + (i - s0.n - s1.n));
                    w[k] = ld_word(p);
                }
            }
            bool all = true;
#pragma unroll
            for (int k = 0; k < PM; ++k) {
                const int i = base + threadIdx.x + k * kFT;
                if (i < n && word_tag(w[k]) != tag) all = false;
            }
            if (all) {
                ok = true;
                break;
            }
            if ((it & 63u) == 63u && ld_volatile_int(err) != 0) break;
        }
        if (ok) {
#pragma unroll
            for (int k = 0; k < PM; ++k) {
                const int i = base + threadIdx.x + k * kFT;
                if (i < n) dst[i] = word_val(w[k]);
            }
        }
    }
    if (!ok) atomicCAS(err, 0, (int)ERR_POLL);
    return __syncthreads_and(ok) != 0;
}

template <int PM>
LDEV bool poll_words(Seg s0, uint32_t tag, float* dst, int* err) {
    return poll_words<PM>(s0, Seg{s0.src, 0}, Seg{s0.src, 0}, tag, dst, err);
}

// xs = ln * (v * r), r = 1/sqrt(mean(v^2) + eps), for H <= 4 * kFT; v is this thread's float4 of the vector
LDEV float norm_to_smem(float4 v, const float* ln, int H, float eps, float* xs, float* red) {
    float ss = 0.0f;
    ss = fmaf(v.x, v.x, ss);
    ss = fmaf(v.y, v.y, ss);
    ss = fmaf(v.z, v.z, ss);
    ss = fmaf(v.w, v.w, ss);
    const float tot = block_sum(ss, red);
    const float r = div_rn(1.0f, sqrt_rn(__fadd_rn(div_rn(tot, (float)H), eps)));
    if (4 * (int)threadIdx.x < H) {
        const float4 l4 = __ldg(reinterpret_cast<const float4*>(ln) + threadIdx.x);
        reinterpret_cast<float4*>(xs)[threadIdx.x] = ln_times(l4, v, r);
    }
    __syncthreads();
    return r;
}

LDEV float4 smem_f4(const float* p, int H) {
    return 4 * (int)threadIdx.x < H ? reinterpret_cast<const float4*>(p)[threadIdx.x] : make_float4(0.f, 0.f, 0.f, 0.f);
}

// ---- copies issued by the producer thread (callers arm the barrier with the same byte count first) ---------------

// RoPE row pairs [p0, p1) of wqkv: rows hh*d + j (the "A" half) and hh*d + j + d/2 ("B") per pair (hh, j); runs of
// pairs inside one head are contiguous in both halves.  A rows land at [0, np), B rows at [np_max, np_max + np).
LDEV uint32_t qkv_bytes(int p0, int p1, int H) { return (uint32_t)(2 * (p1 - p0)) * H * 2; }
__device__ __noinline__ void issue_qkv(const uint16_t* w, int p0, int p1, int np_max, int H, uint16_t* dst, uint64_t* bar) {
#pragma unroll 1
    for (int p = p0; p < p1;) {
        const int hh = p / kHalf, j = p - hh * kHalf;
        const int e = min(p1, (hh + 1) * kHalf), n = e - p;
        const size_t ra = (size_t)hh * kHeadDim + j;
        bulk_g2s(dst + (size_t)(p - p0) * H, w + ra * H, (uint32_t)n * H * 2, bar);
        bulk_g2s(dst + (size_t)(np_max + p - p0) * H, w + (ra + kHalf) * H, (uint32_t)n * H * 2, bar);
        p = e;
    }
}

// K/V rows [r0, r1) of KV head kvh (r1 <= pos: rows already final) into the K and V tiles, one copy per page run
template <int RB>
__device__ __noinline__ void issue_kv_rows(const void* k_pool, const void* v_pool, const int* page_table, int page_size, int kv_heads,
                        int kvh, int r0, int r1, unsigned char* kt, unsigned char* vt, uint64_t* bar) {
#pragma unroll 1
    for (int p = r0; p < r1;) {
        const int pg = p / page_size, e = min(r1, (pg + 1) * page_size);
        const int page = __ldcg(page_table + pg);
        const size_t off = (((size_t)page * kv_heads + kvh) * page_size + (p - pg * page_size)) * RB;
        bulk_g2s(kt + (size_t)(p - r0) * RB, static_cast<const unsigned char*>(k_pool) + off, (uint32_t)(e - p) * RB, bar);
        bulk_g2s(vt + (size_t)(p - r0) * RB, static_cast<const unsigned char*>(v_pool) + off, (uint32_t)(e - p) * RB, bar);
        p = e;
    }
}

// gate_up pairs [q0, q1) (pair q = slot * I + j: gate row j and up row I + j of expert sid[slot]); gate rows land
// at [q0 - base, ...), up rows at [gu_max + q0 - base, ...)
__device__ __noinline__ void issue_gu(const uint16_t* w, const int* sid, int E, int I, int H, int q0, int q1, int base, int gu_max,
                   uint16_t* dst, uint64_t* bar) {
#pragma unroll 1
    for (int q = q0; q < q1;) {
        const int slot = q / I, j = q - slot * I;
        const int e = min(q1, (slot + 1) * I), n = e - q;
        const int ex = min(max(sid[slot], 0), E - 1);
        const uint16_t* base_w = w + (size_t)ex * 2 * I * H;
        bulk_g2s(dst + (size_t)(q - base) * H, base_w + (size_t)j * H, (uint32_t)n * H * 2, bar);
        bulk_g2s(dst + (size_t)(gu_max + q - base) * H, base_w + (size_t)(I + j) * H, (uint32_t)n * H * 2, bar);
        q = e;
    }
}

LDEV int gu_chunk_pairs(int gu_max) { return (gu_max + kGuStages - 1) / kGuStages; }

struct CtaPlan {
    uint32_t epoch;
    int pos, len;
    int pq_lo, pq_hi, pr_lo, pr_hi, pg_lo, pg_hi, pv_lo, pv_hi;
    int S, has_unit, kvh, split, u0, u1, has_new, nrows, gcp, nhc;
};

// CTA plan fields, read from shared memory at every use (volatile: never cached in registers)
#define PL(field) (*reinterpret_cast<volatile const int*>(&plan_s.field))
#define PLU(field) (*reinterpret_cast<volatile const uint32_t*>(&plan_s.field))
// shared-memory regions of the layout (the offsets are kernel parameters)
#define CNT(kind) (a.count + (kind) * kCountStride)
#define CNT_TARGET(lp) ((PLU(epoch) * (unsigned)a.L + (unsigned)(lp) + 1u) * gridDim.x)
#define WAIT_COUNT(kind, lp)                                           \
    do {                                                               \
        if (!wait_count(CNT(kind), CNT_TARGET(lp), a.err)) {           \
            drain(f, a.err);                                           \
            return;                                                    \
        }                                                              \
    } while (0)
#define SM_QKV reinterpret_cast<uint16_t*>(sm + a.lay.off_qkv)
#define SM_KT (sm + a.lay.off_kv)
#define SM_VT (sm + a.lay.off_kv + (size_t)a.lay.kv_cap * RB)
#define SM_WO reinterpret_cast<uint16_t*>(sm + a.lay.off_wo)
#define SM_GU reinterpret_cast<uint16_t*>(sm + a.lay.off_gu)
#define SM_DN reinterpret_cast<uint16_t*>(sm + a.lay.off_dn)
#define SM_HD reinterpret_cast<uint16_t*>(sm + a.lay.off_head)
#define SM_F reinterpret_cast<float*>(sm + a.lay.off_f)
#define SM_OWN reinterpret_cast<float*>(sm + a.lay.off_own)                      // h of this CTA's rows
#define SM_WRT (reinterpret_cast<float*>(sm + a.lay.off_own) + round4(a.lay.rows))  // [rows][E] router operand rows

template <int NCH, int NCI, bool KV_F32>
__global__ void __launch_bounds__(kFT, 1) fused_step_kernel(const FusedArgs a) {
    constexpr int ESZ = KV_F32 ? 4 : 2;
    constexpr int RB = kHeadDim * ESZ;  // bytes per K/V row of one head
    constexpr int CHK = RB / 16;        // 16-byte chunks per K/V row
    extern __shared__ __align__(128) unsigned char sm[];
    __shared__ __align__(8) uint64_t bars[NBARS];
    __shared__ float red[kFT];
    __shared__ int sid[kMaxTopK];
    __shared__ float sval[kMaxTopK], sw[kMaxTopK], s_r;
    __shared__ float s_m[kMaxGroup], s_l[kMaxGroup], s_alpha[kMaxGroup];
    __shared__ unsigned long long wbest[kFW];
    __shared__ bool s_flag;

    // Everything constant for the CTA lives in shared memory (read where used) or in the kernel parameters: a
    // persistent kernel that kept it in registers across the layer loop would spill its working sets.
    __shared__ CtaPlan plan_s;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) {
        CtaPlan p;
        const int c = blockIdx.x, nb = gridDim.x;
        p.epoch = __ldcg(a.epoch);
        p.pos = __ldcg(a.pos);
        p.len = p.pos + 1;
        const Range pq = split_range((a.qd + 2 * a.kvd) / 2, c, nb), pr = split_range(a.H, c, nb);
        const Range pg = split_range(a.k * a.I, c, nb), pv = split_range(a.V, c, nb);
        p.pq_lo = pq.lo;
        p.pq_hi = pq.hi;
        p.pr_lo = pr.lo;
        p.pr_hi = pr.hi;
        p.pg_lo = pg.lo;
        p.pg_hi = pg.hi;
        p.pv_lo = pv.lo;
        p.pv_hi = pv.hi;
        p.S = attn_splits(p.len, a.lay.max_splits);
        p.has_unit = c < a.kv_heads * p.S;
        p.kvh = p.has_unit ? c / p.S : 0;
        p.split = p.has_unit ? c - p.kvh * p.S : 0;
        p.u0 = p.has_unit ? (int)((unsigned)(p.len * p.split) / (unsigned)p.S) : 0;
        p.u1 = p.has_unit ? (int)((unsigned)(p.len * (p.split + 1)) / (unsigned)p.S) : 0;
        p.has_new = p.has_unit && p.pos >= p.u0 && p.pos < p.u1;
        p.nrows = pr.hi - pr.lo;
        p.gcp = gu_chunk_pairs(a.lay.gu_pairs);
        p.nhc = (pv.hi - pv.lo + a.lay.head_rows - 1) / a.lay.head_rows;
        plan_s = p;
        #pragma unroll 1
        for (int b = 0; b < NBARS; ++b) mbar_init(&bars[b], 1);
    }
    __syncthreads();
    Flow f{bars, 0u, 0u};

    // ---- staging helpers (uniform: every thread calls them; the producer thread issues the copies) -----------------
    auto stage_qkv_kv = [&](int l) {
        const FusedLayer& Ly = a.layers[l];
        arm(f, B_QKV, qkv_bytes(PL(pq_lo), PL(pq_hi), a.H));
        if (threadIdx.x == kProd) issue_qkv(Ly.wqkv, PL(pq_lo), PL(pq_hi), a.lay.qkv_pairs, a.H, SM_QKV, &bars[B_QKV]);
        const int old_hi = min(min(PL(u1), PL(u0) + a.lay.kv_cap), PL(pos));
        const int n_old = PL(has_unit) ? max(0, old_hi - PL(u0)) : 0;
        arm(f, B_KV, (uint32_t)n_old * RB * 2);
        if (threadIdx.x == kProd && n_old > 0)
            issue_kv_rows<RB>(Ly.k_pool, Ly.v_pool, a.page_table, a.page_size, a.kv_heads, PL(kvh), PL(u0), old_hi, SM_KT, SM_VT,
                              &bars[B_KV]);
    };
    auto stage_wo = [&](int l) {
        const FusedLayer& Ly = a.layers[l];
        const uint32_t bytes = (uint32_t)PL(nrows) * a.qd * 2;
        arm(f, B_WO, bytes);
        if (threadIdx.x == kProd && bytes) bulk_g2s(SM_WO, Ly.wo + (size_t)PL(pr_lo) * a.qd, bytes, &bars[B_WO]);
        const int n_wrt = PL(nrows) * a.E;
        const float* wsrc = Ly.wr_t + (size_t)PL(pr_lo) * a.E;
        #pragma unroll 1
        for (int t = threadIdx.x; t < n_wrt; t += kFT) SM_WRT[t] = __ldg(wsrc + t);
    };
    auto head_chunk_rows = [&](int ch) { return min(a.lay.head_rows, (PL(pv_hi) - PL(pv_lo)) - ch * a.lay.head_rows); };
    auto stage_head = [&](int st, int ch) {
        const int n = max(0, head_chunk_rows(ch));
        arm(f, B_HD0 + st, (uint32_t)n * a.H * 2);
        if (threadIdx.x == kProd && n > 0)
            bulk_g2s(SM_HD + (size_t)st * a.lay.head_rows * a.H, a.embed + (size_t)(PL(pv_lo) + ch * a.lay.head_rows) * a.H,
                     (uint32_t)n * a.H * 2, &bars[B_HD0 + st]);
    };

    // the step's first layer: nothing is staged yet
    stage_qkv_kv(0);
    stage_wo(0);

    #pragma unroll 1
    for (int l = 0; l < a.L; ++l) {
        const FusedLayer& Ly = a.layers[l];

        // ================= qkv =================
        {
            float* xs = SM_F;
            float* rowout = SM_F + a.H;
            float4 v;
            if (l == 0) {
                // model.rs:134-138: embedding row x embedding_multiplier is the residual stream of layer 0
                const int tok = __ldcg(a.token);
                const uint16_t* er = a.embed + (size_t)tok * a.H;
                v = make_float4(0.f, 0.f, 0.f, 0.f);
                if (4 * (int)threadIdx.x < a.H) {
                    const uint2 u = __ldg(reinterpret_cast<const uint2*>(er) + threadIdx.x);
                    v = make_float4(__fmul_rn(bf_lo(u.x), a.emb_mult), __fmul_rn(bf_hi(u.x), a.emb_mult),
                                    __fmul_rn(bf_lo(u.y), a.emb_mult), __fmul_rn(bf_hi(u.y), a.emb_mult));
                }
                const int nr = PL(nrows), r0 = PL(pr_lo);
                #pragma unroll 1
                for (int i = threadIdx.x; i < nr; i += kFT)
                    SM_OWN[i] = __fmul_rn(__uint_as_float((uint32_t)__ldg(er + r0 + i) << 16), a.emb_mult);
            } else {
                WAIT_COUNT(TG_DOWN, l - 1);
                if (!poll_words<4>(Seg{a.x.h, a.H}, tag_of(PLU(epoch), a.L, l - 1, TG_DOWN), xs, a.err)) {
                    drain(f, a.err);
                    return;
                }
                v = smem_f4(xs, a.H);
            }
            norm_to_smem(v, Ly.ln_attn, a.H, a.eps, xs, red);
            float4 xa[NCH], xb[NCH];
            x_to_regs<NCH>(xs, a.H, lane, xa, xb);
            if (!bar_wait(f, B_QKV, a.err)) {
                drain(f, a.err);
                return;
            }
            const int np = PL(pq_hi) - PL(pq_lo);
            #pragma unroll 1
            for (int ri = warp; ri < 2 * np; ri += kFW) {
                const uint16_t* row = SM_QKV + ((size_t)((ri & 1) ? a.lay.qkv_pairs : 0) + (ri >> 1)) * a.H;
                const float d = warp_sum(smem_row_dot<NCH>(row, xa, xb, a.H, lane));
                if (lane == 0) rowout[ri] = d;
            }
            __syncthreads();
            const uint32_t tq = tag_of(PLU(epoch), a.L, l, TG_QKV);
            #pragma unroll 1
            for (int t = threadIdx.x; t < np; t += kFT) {
                const int p = PL(pq_lo) + t;
                const int hh = p / kHalf, j = p - hh * kHalf;
                const int ra = hh * kHeadDim + j, rb = ra + kHalf;
                const float x1 = rowout[2 * t], x2 = rowout[2 * t + 1];
                const float* cs = a.rope_cs + (size_t)PL(pos) * kHeadDim;
                const float cc = __ldg(cs + j), sn = __ldg(cs + kHalf + j);
                // model.rs:153-155: x1*(int)blockIdx.x - x2*s, x2*(int)blockIdx.x + x1*s (no contraction)
                const float ro0 = __fsub_rn(__fmul_rn(x1, cc), __fmul_rn(x2, sn));
                const float ro1 = __fadd_rn(__fmul_rn(x2, cc), __fmul_rn(x1, sn));
                if (ra < a.qd) {
                    st_word(a.x.qkv + ra, ro0, tq);
                    st_word(a.x.qkv + rb, ro1, tq);
                    continue;
                }
                int rr = ra - a.qd;
                const bool is_k = rr < a.kvd;
                if (!is_k) rr -= a.kvd;
                const int kh = rr / kHeadDim;
                float v0 = is_k ? ro0 : x1, v1 = is_k ? ro1 : x2;
                const int page = __ldcg(a.page_table + PL(pos) / a.page_size), slot = PL(pos) % a.page_size;
                const size_t base = (((size_t)page * a.kv_heads + kh) * a.page_size + slot) * kHeadDim;
                void* pool = is_k ? Ly.k_pool : Ly.v_pool;
                if (KV_F32) {
                    float* pp = static_cast<float*>(pool) + base;
                    pp[j] = v0;
                    pp[j + kHalf] = v1;
                } else {
                    uint16_t* pp = static_cast<uint16_t*>(pool) + base;
                    const uint16_t b0 = f32_to_bf16_rne(v0), b1 = f32_to_bf16_rne(v1);
                    pp[j] = b0;
                    pp[j + kHalf] = b1;
                    v0 = __uint_as_float((uint32_t)b0 << 16);  // this step attends to the row as cached
                    v1 = __uint_as_float((uint32_t)b1 << 16);
                }
                st_word(a.x.qkv + ra, v0, tq);
                st_word(a.x.qkv + rb, v1, tq);
            }
        }

        arrive_count(CNT(TG_QKV));

        // ================= attention =================
        {
            // scratch: sq [a.G][64], newk [64], newv [64], sc [kv_cap][a.G], accp [RG][a.G][64]
            float* sq = SM_F;
            float* newk = sq + a.G * kHeadDim;
            float* newv = newk + kHeadDim;
            float* sc = newv + kHeadDim;
            float* accp = sc + a.lay.kv_cap * a.G;
            const int RG = kFT / (32 * a.G);
            const bool pv_active = (int)threadIdx.x < a.G * 32 * RG;
            const int pv_g = threadIdx.x / (32 * RG), pv_rg = (threadIdx.x / 32) % RG, pv_dp = lane;
            float acc0 = 0.0f, acc1 = 0.0f;
            __syncthreads();  // the qkv phase's scratch is read
            if (PL(has_unit)) {
                const uint32_t tq = tag_of(PLU(epoch), a.L, l, TG_QKV);
                const Seg qs{a.x.qkv + (size_t)PL(kvh) * a.G * kHeadDim, a.G * kHeadDim};
                const Seg ks{a.x.qkv + a.qd + (size_t)PL(kvh) * kHeadDim, PL(has_new) ? kHeadDim : 0};
                const Seg vs{a.x.qkv + a.qd + a.kvd + (size_t)PL(kvh) * kHeadDim, PL(has_new) ? kHeadDim : 0};
                // sq, newk and newv are contiguous: one poll fills them
                WAIT_COUNT(TG_QKV, l);
                if (!poll_words<2>(qs, ks, vs, tq, sq, a.err)) {
                    drain(f, a.err);
                    return;
                }
                if (threadIdx.x < a.G) {
                    s_m[threadIdx.x] = -INFINITY;
                    s_l[threadIdx.x] = 0.0f;
                }
            }
            bool ok = true;
            // every CTA waits on the first chunk's barrier (armed with 0 bytes when it has no unit)
            const int u0 = PL(u0), u1 = PL(u1);
            #pragma unroll 1
            for (int cb = u0, first = 1; first || cb < u1; cb += a.lay.kv_cap, first = 0) {
                const int ce = min(PL(u1), cb + a.lay.kv_cap), nrow = max(0, ce - cb);
                if (!first) {
                    __syncthreads();  // every read of the previous chunk is done
                    const int old_hi = min(ce, PL(pos));
                    const int n_old = max(0, old_hi - cb);
                    if (threadIdx.x == kProd) fence_async_smem();
                    arm(f, B_KV, (uint32_t)n_old * RB * 2);
                    if (threadIdx.x == kProd && n_old > 0)
                        issue_kv_rows<RB>(Ly.k_pool, Ly.v_pool, a.page_table, a.page_size, a.kv_heads, PL(kvh), cb, old_hi,
                                          SM_KT, SM_VT, &bars[B_KV]);
                }
                if (PL(has_new) && PL(pos) >= cb && PL(pos) < ce && (int)threadIdx.x < 2 * kHeadDim) {
                    // the row this layer's qkv phase just produced, as the cache holds it
                    const bool is_v = threadIdx.x >= kHeadDim;
                    const int dim = threadIdx.x - (is_v ? kHeadDim : 0);
                    const float val = (is_v ? newv : newk)[dim];
                    unsigned char* rowp = (is_v ? SM_VT : SM_KT) + (size_t)(PL(pos) - cb) * RB;
                    if (KV_F32)
                        reinterpret_cast<float*>(rowp)[dim] = val;
                    else
                        reinterpret_cast<uint16_t*>(rowp)[dim] = (uint16_t)(__float_as_uint(val) >> 16);
                }
                if (!bar_wait(f, B_KV, a.err)) {  // includes a __syncthreads
                    ok = false;
                    break;
                }
                if (!PL(has_unit)) break;
                // scores: thread (row, g); a.k chunks read in a row-rotated order so 8 consecutive rows hit distinct banks
                #pragma unroll 1
                for (int i = threadIdx.x; i < nrow * a.G; i += kFT) {
                    const int row = i / a.G, g = i - row * a.G;
                    const uint4* kr = reinterpret_cast<const uint4*>(SM_KT + (size_t)row * RB);
                    const float* qg = sq + g * kHeadDim;
                    float s = 0.0f;
#pragma unroll
                    for (int cc = 0; cc < CHK; ++cc) {
                        const int ch = (cc + row) & (CHK - 1);
                        const uint4 kc = kr[ch];
                        if (KV_F32) {
                            const float4 q4 = *reinterpret_cast<const float4*>(qg + ch * 4);
                            s = fmaf(q4.x, __uint_as_float(kc.x), s);
                            s = fmaf(q4.y, __uint_as_float(kc.y), s);
                            s = fmaf(q4.z, __uint_as_float(kc.z), s);
                            s = fmaf(q4.w, __uint_as_float(kc.w), s);
                        } else {
                            const float4 qa = *reinterpret_cast<const float4*>(qg + ch * 8);
                            const float4 qb = *reinterpret_cast<const float4*>(qg + ch * 8 + 4);
                            s = dot8(kc, qa, qb, s);
                        }
                    }
                    sc[i] = __fmul_rn(s, a.attn_scale);
                }
                __syncthreads();
                // online softmax per query head: warp g
                if (warp < a.G) {
                    const int g = warp;
                    float mx = -INFINITY;
                    #pragma unroll 1
                    for (int row = lane; row < nrow; row += 32) mx = fmaxf(mx, sc[row * a.G + g]);
                    mx = warp_max(mx);
                    const float m_old = s_m[g];
                    const float mn = fmaxf(m_old, mx);
                    float ls = 0.0f;
                    #pragma unroll 1
                    for (int row = lane; row < nrow; row += 32) {
                        const float p = exp_f(sc[row * a.G + g] - mn);
                        sc[row * a.G + g] = p;
                        ls += p;
                    }
                    ls = warp_sum(ls);
                    if (lane == 0) {
                        const float alpha = (m_old == -INFINITY) ? 0.0f : exp_f(m_old - mn);
                        s_l[g] = s_l[g] * alpha + ls;
                        s_m[g] = mn;
                        s_alpha[g] = alpha;
                    }
                }
                __syncthreads();
                if (pv_active) {
                    const float al = s_alpha[pv_g];
                    acc0 *= al;
                    acc1 *= al;
                    int row = pv_rg;
                    // four rows per iteration: their loads are independent
                    #pragma unroll 1
                    for (; row + 3 * RG < nrow; row += 4 * RG) {
                        float p[4], v0[4], v1[4];
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            const int rr = row + u * RG;
                            p[u] = sc[rr * a.G + pv_g];
                            if (KV_F32) {
                                const float2 t = reinterpret_cast<const float2*>(SM_VT + (size_t)rr * RB)[pv_dp];
                                v0[u] = t.x;
                                v1[u] = t.y;
                            } else {
                                const uint32_t t = reinterpret_cast<const uint32_t*>(SM_VT + (size_t)rr * RB)[pv_dp];
                                v0[u] = bf_lo(t);
                                v1[u] = bf_hi(t);
                            }
                        }
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            acc0 = fmaf(p[u], v0[u], acc0);
                            acc1 = fmaf(p[u], v1[u], acc1);
                        }
                    }
                    #pragma unroll 1
                    for (; row < nrow; row += RG) {
                        const float p = sc[row * a.G + pv_g];
                        float v0, v1;
                        if (KV_F32) {
                            const float2 t = reinterpret_cast<const float2*>(SM_VT + (size_t)row * RB)[pv_dp];
                            v0 = t.x;
                            v1 = t.y;
                        } else {
                            const uint32_t t = reinterpret_cast<const uint32_t*>(SM_VT + (size_t)row * RB)[pv_dp];
                            v0 = bf_lo(t);
                            v1 = bf_hi(t);
                        }
                        acc0 = fmaf(p, v0, acc0);
                        acc1 = fmaf(p, v1, acc1);
                    }
                }
            }
            if (!ok) {
                drain(f, a.err);
                return;
            }
            if (PL(has_unit)) {
                if (pv_active) {
                    accp[((size_t)pv_rg * a.G + pv_g) * kHeadDim + 2 * pv_dp] = acc0;
                    accp[((size_t)pv_rg * a.G + pv_g) * kHeadDim + 2 * pv_dp + 1] = acc1;
                }
                __syncthreads();
                const uint32_t ta = tag_of(PLU(epoch), a.L, l, TG_ATTN);
                #pragma unroll 1
                for (int t = threadIdx.x; t < a.G * kPartStride; t += kFT) {
                    const int g = t / kPartStride, j = t - g * kPartStride;
                    float v;
                    if (j < kHeadDim) {
                        v = 0.0f;
                        #pragma unroll 1
                        for (int rg = 0; rg < RG; ++rg) v += accp[((size_t)rg * a.G + g) * kHeadDim + j];
                    } else {
                        v = j == kHeadDim ? s_m[g] : s_l[g];
                    }
                    st_word(a.x.part + ((size_t)(PL(kvh) * a.G + g) * a.lay.max_splits + PL(split)) * kPartStride + j, v, ta);
                }
            }
        }

        arrive_count(CNT(TG_ATTN));

        // ================= merge (CTA hd < heads: query head hd) =================
        if ((int)blockIdx.x < (a.kv_heads * a.G)) {
            float* pbuf = SM_F;  // [PL(S)][kPartStride]
            __syncthreads();    // the attention scratch is read
            WAIT_COUNT(TG_ATTN, l);
            if (!poll_words<4>(Seg{a.x.part + (size_t)(int)blockIdx.x * a.lay.max_splits * kPartStride, PL(S) * kPartStride},
                            tag_of(PLU(epoch), a.L, l, TG_ATTN), pbuf, a.err)) {
                drain(f, a.err);
                return;
            }
            if ((int)threadIdx.x < kHeadDim) {
                const int dim = threadIdx.x, S = PL(S);
                float M = -INFINITY;
                #pragma unroll 1
                for (int sp = 0; sp < S; ++sp) M = fmaxf(M, pbuf[sp * kPartStride + kHeadDim]);
                float den = 0.0f, num = 0.0f;
                #pragma unroll 1
                for (int sp = 0; sp < S; ++sp) {
                    const float mv = pbuf[sp * kPartStride + kHeadDim];
                    const float e = mv == -INFINITY ? 0.0f : exp_f(mv - M);
                    den = fmaf(pbuf[sp * kPartStride + kHeadDim + 1], e, den);
                    num = fmaf(pbuf[sp * kPartStride + dim], e, num);
                }
                st_word(a.x.att + (size_t)(int)blockIdx.x * kHeadDim + dim, div_rn(num, den), tag_of(PLU(epoch), a.L, l, TG_MERGE));
            }
        }

        arrive_count(CNT(TG_MERGE));

        // ================= output projection + router shares =================
        {
            float* att = SM_F;
            __syncthreads();  // the merge scratch is read
            WAIT_COUNT(TG_MERGE, l);
            if (!poll_words<4>(Seg{a.x.att, a.qd}, tag_of(PLU(epoch), a.L, l, TG_MERGE), att, a.err)) {
                drain(f, a.err);
                return;
            }
            float4 xa[NCH], xb[NCH];
            x_to_regs<NCH>(att, a.qd, lane, xa, xb);
            if (!bar_wait(f, B_WO, a.err)) {
                drain(f, a.err);
                return;
            }
            const uint32_t to = tag_of(PLU(epoch), a.L, l, TG_OPROJ);
            const int nr = PL(nrows), r0 = PL(pr_lo);
            #pragma unroll 1
            for (int ri = warp; ri < nr; ri += kFW) {
                const float o = warp_sum(smem_row_dot<NCH>(SM_WO + (size_t)ri * a.qd, xa, xb, a.qd, lane));
                if (lane == 0) {
                    const float hn = __fadd_rn(SM_OWN[ri], __fmul_rn(a.resid, o));  // model.rs:223-227
                    SM_OWN[ri] = hn;
                    st_word(a.x.h + r0 + ri, hn, to);
                }
            }
            __syncthreads();
            const int E1 = a.E + 1;
            if ((int)threadIdx.x < a.E) {
                float p = 0.0f;
                #pragma unroll 1
                for (int i = 0; i < nr; ++i) p = fmaf(SM_WRT[i * a.E + threadIdx.x], SM_OWN[i], p);
                st_word(a.x.share + (size_t)(int)blockIdx.x * E1 + threadIdx.x, p, to);
            } else if ((int)threadIdx.x == a.E) {
                float ss = 0.0f;
                #pragma unroll 1
                for (int i = 0; i < nr; ++i) ss = fmaf(SM_OWN[i], SM_OWN[i], ss);
                st_word(a.x.share + (size_t)(int)blockIdx.x * E1 + a.E, ss, to);
            }
        }

        arrive_count(CNT(TG_OPROJ));

        // ================= routing + gate_up =================
        {
            const uint32_t to = tag_of(PLU(epoch), a.L, l, TG_OPROJ);
            float* xs = SM_F;
            float* guout = SM_F + a.H;
            // routing: thread (gi, e) sums the shares of CTAs gi, gi + groups, ... in that order (the same order in
            // every CTA); its loads and the thread's float4 of h are polled together
            const int E1 = a.E + 1, groups = kFT / E1;
            const bool rthread = (int)threadIdx.x < groups * E1;
            const int re = threadIdx.x % E1, rgi = threadIdx.x / E1;
            const int nsh = rthread ? ((int)gridDim.x - rgi + groups - 1) / groups : 0;  // <= kPollMax
            const bool hthread = 4 * (int)threadIdx.x < a.H;
            float acc = 0.0f;
            float4 hv = make_float4(0.f, 0.f, 0.f, 0.f);
            WAIT_COUNT(TG_OPROJ, l);
            {
                u64 w[kPollMax], hw[4];
                bool ok = false;
                #pragma unroll 1
                for (uint32_t it = 0; it < kSpinLimit; ++it) {
#pragma unroll
                    for (int q = 0; q < kPollMax; ++q)
                        if (q < nsh) w[q] = ld_word(a.x.share + (size_t)(rgi + q * groups) * E1 + re);
                    if (hthread) {
#pragma unroll
                        for (int q = 0; q < 4; ++q) hw[q] = ld_word(a.x.h + 4 * threadIdx.x + q);
                    }
                    bool all = true;
#pragma unroll
                    for (int q = 0; q < kPollMax; ++q)
                        if (q < nsh && word_tag(w[q]) != to) all = false;
                    if (hthread) {
#pragma unroll
                        for (int q = 0; q < 4; ++q)
                            if (word_tag(hw[q]) != to) all = false;
                    }
                    if (all) {
                        ok = true;
                        break;
                    }
                    if ((it & 63u) == 63u && ld_volatile_int(a.err) != 0) break;
                }
                if (ok) {
#pragma unroll
                    for (int q = 0; q < kPollMax; ++q)
                        if (q < nsh) acc = __fadd_rn(acc, word_val(w[q]));
                    if (hthread) hv = make_float4(word_val(hw[0]), word_val(hw[1]), word_val(hw[2]), word_val(hw[3]));
                } else {
                    atomicCAS(a.err, 0, (int)ERR_POLL);
                }
                if (!__syncthreads_and(ok)) {
                    drain(f, a.err);
                    return;
                }
            }
            red[threadIdx.x] = acc;
            __syncthreads();
            if (warp == 0) {
                float v[3];
#pragma unroll
                for (int q = 0; q < 3; ++q) {
                    const int e = lane + 32 * q;
                    float t = 0.0f;
                    if (e < E1)
                        #pragma unroll 1
                        for (int gi = 0; gi < groups; ++gi) t = __fadd_rn(t, red[gi * E1 + e]);
                    v[q] = t;
                }
                const float ssum = __shfl_sync(0xffffffffu, a.E < 32 ? v[0] : (a.E < 64 ? v[1] : v[2]), a.E & 31);
                const float r = div_rn(1.0f, sqrt_rn(__fadd_rn(div_rn(ssum, (float)a.H), a.eps)));
                const float l0 = lane < a.E ? __fmul_rn(v[0], r) : 0.0f;
                const float l1 = lane + 32 < a.E ? __fmul_rn(v[1], r) : 0.0f;
                route_topk_warp(l0, l1, a.E, a.k, sid, sval, sw);
                if (lane == 0) s_r = r;
                if ((int)blockIdx.x == 0) {
                    if (lane < a.E) a.rlogits[lane] = l0;
                    if (lane + 32 < a.E) a.rlogits[lane + 32] = l1;
                    if (lane < a.k) {
                        a.route_ids[(size_t)l * a.k + lane] = sid[lane];
                        a.route_w[(size_t)l * a.k + lane] = sw[lane];
                    }
                }
            }
            __syncthreads();
            const float r = s_r;
            // expert rows of this CTA: gate_up in kGuStages chunks (the gate_up region was last read by ordinary
            // loads: the staged rows of earlier phases)
            if (threadIdx.x == kProd) fence_async_smem();
            #pragma unroll 1
            for (int ci = 0; ci < kGuStages; ++ci) {
                const int q0 = min(PL(pg_hi), PL(pg_lo) + ci * PL(gcp)), q1 = min(PL(pg_hi), q0 + PL(gcp));
                arm(f, B_GU0 + ci, (uint32_t)(q1 - q0) * a.H * 4);
                if (threadIdx.x == kProd && q1 > q0)
                    issue_gu(Ly.gate_up, sid, a.E, a.I, a.H, q0, q1, PL(pg_lo), a.lay.gu_pairs, SM_GU, &bars[B_GU0 + ci]);
            }
            if (hthread) {
                const float4 l4 = __ldg(reinterpret_cast<const float4*>(Ly.ln_moe) + threadIdx.x);
                reinterpret_cast<float4*>(xs)[threadIdx.x] = ln_times(l4, hv, r);  // model.rs:141-145
            }
            __syncthreads();
            float4 xa[NCH], xb[NCH];
            x_to_regs<NCH>(xs, a.H, lane, xa, xb);
            bool ok = true;
            const int pgl = PL(pg_lo), pgh = PL(pg_hi), gcp = PL(gcp);
            #pragma unroll 1
            for (int ci = 0; ci < kGuStages; ++ci) {
                const int q0 = min(pgh, pgl + ci * gcp), q1 = min(pgh, q0 + gcp);
                if (!bar_wait(f, B_GU0 + ci, a.err)) {
                    ok = false;
                    break;
                }
                if (ci == kGuStages - 1 && threadIdx.x == kProd && PL(nrows) > 0)
                    // every gate_up byte has landed: the down rows stream into L2 while the last chunk is reduced
                    #pragma unroll 1
                    for (int j = 0; j < a.k; ++j) {
                        const int ex = min(max(sid[j], 0), a.E - 1);
                        prefetch_l2(Ly.down + ((size_t)ex * a.H + PL(pr_lo)) * a.I, (uint32_t)PL(nrows) * a.I * 2);
                    }
                #pragma unroll 1
                for (int ri = warp; ri < 2 * (q1 - q0); ri += kFW) {
                    const int pi = q0 - pgl + (ri >> 1), up = ri & 1;
                    const uint16_t* row = SM_GU + ((size_t)(up ? a.lay.gu_pairs : 0) + pi) * a.H;
                    const float d = warp_sum(smem_row_dot<NCH>(row, xa, xb, a.H, lane));
                    if (lane == 0) guout[2 * pi + up] = d;
                }
            }
            if (!ok) {
                drain(f, a.err);
                return;
            }
            __syncthreads();
            const uint32_t tu = tag_of(PLU(epoch), a.L, l, TG_UP);
            const int npg = PL(pg_hi) - PL(pg_lo), g0 = PL(pg_lo);
            #pragma unroll 1
            for (int t = threadIdx.x; t < npg; t += kFT) {
                const float g = guout[2 * t], u = guout[2 * t + 1];
                st_word(a.x.act + g0 + t, __fmul_rn(div_rn(g, __fadd_rn(1.0f, exp_f(-g))), u), tu);  // cpu.rs:64-68
            }
            // arrive (synchronises the CTA: every read of the gate_up rows is done before the region is refilled)
            arrive_count(CNT(TG_UP));
            if (threadIdx.x == kProd) fence_async_smem();
            const uint32_t dbytes = (uint32_t)PL(nrows) * a.I * 2;
            arm(f, B_DN, dbytes * a.k);
            if (threadIdx.x == kProd && dbytes)
                #pragma unroll 1
                for (int j = 0; j < a.k; ++j) {
                    const int ex = min(max(sid[j], 0), a.E - 1);
                    bulk_g2s(SM_DN + (size_t)j * a.lay.rows * a.I, Ly.down + ((size_t)ex * a.H + PL(pr_lo)) * a.I, dbytes, &bars[B_DN]);
                }
            if (l + 1 < a.L) {
                stage_qkv_kv(l + 1);
            } else {
                #pragma unroll 1
                for (int st = 0; st < a.lay.head_stages; ++st) stage_head(st, st);
            }
        }

        // ================= down =================
        {
            float* dpart = SM_F;  // [k][rows]
            const int wps = kFW / a.k;
            const int j = warp / wps, wi = warp - (warp / wps) * wps;
            const bool active = j < a.k;
            float4 xa[NCI], xb[NCI];
            WAIT_COUNT(TG_UP, l);
            {
                // the warp's expert activations a_j, polled straight into the x-in-registers layout
                const uint32_t tu = tag_of(PLU(epoch), a.L, l, TG_UP);
                const u64* src = a.x.act + (size_t)(active ? j : 0) * a.I;
                bool ok = false;
                #pragma unroll 1
                for (uint32_t it = 0; it < kSpinLimit; ++it) {
                    u64 w[NCI][8];
#pragma unroll
                    for (int cc = 0; cc < NCI; ++cc) {
                        const int col = (cc * 32 + lane) * 8;
#pragma unroll
                        for (int e = 0; e < 8; ++e) w[cc][e] = (active && col < a.I) ? ld_word(src + col + e) : ((u64)tu << 32);
                    }
                    bool all = true;
#pragma unroll
                    for (int cc = 0; cc < NCI; ++cc)
#pragma unroll
                        for (int e = 0; e < 8; ++e)
                            if (word_tag(w[cc][e]) != tu) all = false;
                    if (__all_sync(0xffffffffu, all)) {
#pragma unroll
                        for (int cc = 0; cc < NCI; ++cc) {
                            xa[cc] = make_float4(word_val(w[cc][0]), word_val(w[cc][1]), word_val(w[cc][2]), word_val(w[cc][3]));
                            xb[cc] = make_float4(word_val(w[cc][4]), word_val(w[cc][5]), word_val(w[cc][6]), word_val(w[cc][7]));
                        }
                        ok = true;
                        break;
                    }
                    if ((it & 63u) == 63u && ld_volatile_int(a.err) != 0) break;
                }
                if (!ok) atomicCAS(a.err, 0, (int)ERR_POLL);
                if (!__syncthreads_and(ok)) {
                    drain(f, a.err);
                    return;
                }
            }
            if (!bar_wait(f, B_DN, a.err)) {
                drain(f, a.err);
                return;
            }
            const int nr = PL(nrows), r0 = PL(pr_lo);
            if (active)
                #pragma unroll 1
                for (int i = wi; i < nr; i += wps) {
                    const float d =
                        warp_sum(smem_row_dot<NCI>(SM_DN + ((size_t)j * a.lay.rows + i) * a.I, xa, xb, a.I, lane));
                    if (lane == 0) dpart[j * a.lay.rows + i] = d;
                }
            __syncthreads();
            const uint32_t td = tag_of(PLU(epoch), a.L, l, TG_DOWN);
            #pragma unroll 1
            for (int t = threadIdx.x; t < nr; t += kFT) {
                float acc = 0.0f;
                #pragma unroll 1
                for (int jj = 0; jj < a.k; ++jj) acc = __fadd_rn(acc, __fmul_rn(sw[jj], dpart[jj * a.lay.rows + t]));
                const float hn = __fadd_rn(SM_OWN[t], __fmul_rn(a.resid, acc));  // cpu.rs:141-148, model.rs:230
                SM_OWN[t] = hn;
                st_word(a.x.h + r0 + t, hn, td);
            }
            arrive_count(CNT(TG_DOWN));  // synchronises the CTA: every read of the down rows is done
            if (l + 1 < a.L) {
                if (threadIdx.x == kProd) fence_async_smem();
                stage_wo(l + 1);
            }
        }
    }

    // ================= lm_head =================
    {
        float* xs = SM_F;
        WAIT_COUNT(TG_DOWN, a.L - 1);
        if (!poll_words<4>(Seg{a.x.h, a.H}, tag_of(PLU(epoch), a.L, a.L - 1, TG_DOWN), xs, a.err)) {
            drain(f, a.err);
            return;
        }
        norm_to_smem(smem_f4(xs, a.H), a.norm, a.H, a.eps, xs, red);
        float4 xa[NCH], xb[NCH];
        x_to_regs<NCH>(xs, a.H, lane, xa, xb);
        unsigned long long best = 0ull;
        const int nhc = PL(nhc), v0 = PL(pv_lo);
        #pragma unroll 1
        for (int ch = 0; ch < nhc; ++ch) {
            const int st = ch % a.lay.head_stages;
            if (!bar_wait(f, B_HD0 + st, a.err)) {
                drain(f, a.err);
                return;
            }
            const int n = head_chunk_rows(ch);
            #pragma unroll 1
            for (int ri = warp; ri < n; ri += kFW) {
                const int row = v0 + ch * a.lay.head_rows + ri;
                const float d = warp_sum(smem_row_dot<NCH>(SM_HD + ((size_t)st * a.lay.head_rows + ri) * a.H, xa, xb, a.H, lane));
                const float lg = div_rn(d, a.logits_scaling);
                if (lane == 0) a.logits[row] = lg;
                const unsigned long long kk = arg_key(lg, row);
                best = kk > best ? kk : best;
            }
            if (ch + a.lay.head_stages < PL(nhc)) {
                __syncthreads();  // stage st is read
                if (threadIdx.x == kProd) fence_async_smem();
                stage_head(st, ch + a.lay.head_stages);
            }
        }
        // barriers of stages that were armed but never needed (fewer chunks than stages) are complete already
        #pragma unroll 1
        for (int ch = nhc; ch < a.lay.head_stages; ++ch) {
            if (!bar_wait(f, B_HD0 + ch, a.err)) {
                drain(f, a.err);
                return;
            }
        }
        if (lane == 0) wbest[warp] = best;
        __syncthreads();
        const unsigned tgt = (PLU(epoch) + 1u) * (unsigned)(int)gridDim.x;
        if (threadIdx.x == 0) {
            unsigned long long b = 0ull;
            #pragma unroll 1
            for (int i = 0; i < kFW; ++i) b = wbest[i] > b ? wbest[i] : b;
            a.best[(int)blockIdx.x] = b;
            __threadfence();
            const unsigned t = atomicAdd(a.ticket, 1u);
            s_flag = (t == tgt - 1u);
        }
        __syncthreads();
        if (!s_flag) return;
        __threadfence();
        unsigned long long b = 0ull;
        #pragma unroll 1
        for (int i = threadIdx.x; i < (int)gridDim.x; i += kFT) {
            const unsigned long long t = __ldcg(a.best + i);
            b = t > b ? t : b;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long t = shfl_xor_u64(b, o);
            b = t > b ? t : b;
        }
        if (lane == 0) wbest[warp] = b;
        __syncthreads();
        if (threadIdx.x == 0) {
            unsigned long long mx = 0ull;
            #pragma unroll 1
            for (int i = 0; i < kFW; ++i) mx = wbest[i] > mx ? wbest[i] : mx;
            const int tok = (int)(uint32_t)mx;
            *a.token = tok;
            if (a.out_ids) {
                const int st = __ldcg(a.step);
                if (st >= 0 && st < a.out_cap) a.out_ids[st] = tok;
                *a.step = st + 1;
            }
            *a.pos = PL(pos) + 1;
            __threadfence();
            *a.epoch = PLU(epoch) + 1u;
        }
    }
}

using FusedKern = void (*)(const FusedArgs);

template <int NCH, int NCI>
FusedKern pick(int kv_f32) {
    return kv_f32 ? fused_step_kernel<NCH, NCI, true> : fused_step_kernel<NCH, NCI, false>;
}

FusedKern fused_kernel_for(int H, int qd, int I, int kv_f32) {
    const int nch = (std::max(H, qd) + 255) / 256, nci = (I + 255) / 256;
    if (nch == 1 && nci == 1) return pick<1, 1>(kv_f32);
    if (nch == 3 && nci == 1) return pick<3, 1>(kv_f32);
    if (nch == 4 && nci == 2) return pick<4, 2>(kv_f32);
    if (nch == 6 && nci == 2) return pick<6, 2>(kv_f32);
    return pick<8, 8>(kv_f32);
}

size_t align128(size_t v) { return (v + 127) & ~(size_t)127; }

}  // namespace

bool fused_plan(int H, int I, int E, int k, int qd, int kvd, int kv_heads, int G, int V, int kv_f32, int n_sm,
                FusedLayout* out) {
    if (n_sm < 1 || H > 4 * kFT || qd > 4 * kFT || H % 8 || I % 8 || G > kMaxGroup || k > kFW || E > 64) return false;
    const int npair = (qd + 2 * kvd) / 2, nh = kv_heads * G;
    // every CTA must produce a share of every exchange (see the kernel's header comment)
    const int nb = std::min(std::min(n_sm, npair), std::min(H, k * I));
    if (nb < nh || nb < kv_heads) return false;
    // the routing poll: ceil(nb / groups) shares per thread
    const int groups = kFT / (E + 1);
    if (groups < 1 || (nb + groups - 1) / groups > kPollMax) return false;
    FusedLayout L{};
    L.nb = nb;
    L.qkv_pairs = (npair + nb - 1) / nb;
    L.rows = (H + nb - 1) / nb;
    L.gu_pairs = (k * I + nb - 1) / nb;
    L.max_splits = std::max(1, nb / kv_heads);
    const int RB = kHeadDim * (kv_f32 ? 4 : 2);
    L.kv_cap = kv_f32 ? 64 : 128;
    const size_t qkv = (size_t)2 * L.qkv_pairs * H * 2;
    const size_t kv = (size_t)2 * L.kv_cap * RB;
    const size_t wo = (size_t)L.rows * qd * 2;
    const size_t dn = (size_t)k * L.rows * I * 2;
    const size_t gu = (size_t)2 * L.gu_pairs * H * 2;
    L.off_dn = 0;
    L.off_wo = 0;
    L.off_gu = 0;
    L.off_qkv = (int)align128(std::max(dn, wo));
    L.off_kv = (int)align128(L.off_qkv + qkv);
    L.off_head = (int)align128(dn);
    const size_t base_end = std::max(align128(L.off_kv + kv), align128(gu));
    // phase scratch (floats)
    const int RG = kFT / (32 * G);
    size_t fl = (size_t)H + 2 * L.qkv_pairs;                                                               // qkv
    fl = std::max(fl, (size_t)G * kHeadDim + 2 * kHeadDim + (size_t)L.kv_cap * G + (size_t)RG * G * kHeadDim);  // attention
    fl = std::max(fl, (size_t)L.max_splits * kPartStride);                                                 // merge
    fl = std::max(fl, (size_t)qd);                                                                         // oproj
    fl = std::max(fl, (size_t)H + 2 * L.gu_pairs);                                                         // gate_up
    fl = std::max(fl, (size_t)k * L.rows);                                                                 // down
    const size_t fbytes = align128(fl * 4);
    const size_t own = align128((size_t)(round4(L.rows) + L.rows * E) * 4);
    // lm_head ring in what is left: rows per stage x stages
    L.head_rows = 0;
    for (int hr : {16, 8, 4}) {
        for (int st = kMaxHeadStages; st >= 2 && !L.head_rows; --st) {
            const size_t ring_end = L.off_head + (size_t)st * hr * H * 2;
            const size_t total = std::max(base_end, align128(ring_end)) + fbytes + own;
            if (total <= kMaxSmemBytes && (size_t)st * hr >= 32) {
                L.head_rows = hr;
                L.head_stages = st;
            }
        }
        if (L.head_rows) break;
    }
    if (!L.head_rows) return false;
    const size_t ring_end = L.off_head + (size_t)L.head_stages * L.head_rows * H * 2;
    L.off_f = (int)std::max(base_end, align128(ring_end));
    L.off_own = (int)(L.off_f + fbytes);
    L.smem = (int)(L.off_own + own);
    if ((size_t)L.smem > kMaxSmemBytes) return false;
    *out = L;
    return true;
}

cudaError_t launch_fused_step(const FusedArgs& a, int kv_f32, cudaStream_t s) {
    FusedKern kern = fused_kernel_for(a.H, a.qd, a.I, kv_f32);
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, a.lay.smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.lay.nb);
    cfg.blockDim = dim3(kFT);
    cfg.dynamicSmemBytes = a.lay.smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // all CTAs co-resident: the exchange polls cannot starve a CTA
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, a);
}

cudaError_t fused_blocks_per_sm(int H, int qd, int I, int kv_f32, int smem, int* blocks) {
    FusedKern kern = fused_kernel_for(H, qd, I, kv_f32);
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks, kern, kFT, smem);
}

}  // namespace lastro
