// Batch-1 Granite-MoE decode kernels for sm_100a.
//
// Design (B200): every kernel is one streaming pass over bf16 weights with 16-byte non-coherent loads, a warp per
// output row (or row pair), f32 activations staged in shared memory and warp-shuffle reductions.  At batch 1 each
// kernel is short (a few microseconds), so the design goal is memory-level parallelism on the critical path: every
// thread issues all of its loads before it consumes any of them (no load -> use -> load chains), and loads that do
// not depend on the previous kernel (weights, norm weights, expert ids two kernels back) are issued before
// griddepcontrol.wait, so with programmatic dependent launch a kernel's HBM traffic overlaps the tail of its
// predecessor.  Cross-CTA reductions (router top-k, attention split merge, lm_head argmax) use a last-CTA ticket
// instead of a second launch.
//
// Reference behaviour restated (brenoperucchi/lastro-rust, rust/moe-rt/src):
//   RMSNorm  model.rs:141-145   RoPE rotate_half model.rs:147-158   attention model.rs:203-222
//   routing  block.rs:79-89     SwiGLU cpu.rs:64-68               experts cpu.rs:115-150
//   step     model.rs:181-243   argmax (last maximum) bin/m1b-gulosa.rs:22-24
#include <cooperative_groups.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "ops.cuh"

namespace lastro {

namespace {

template <typename Kern, typename... Args>
cudaError_t launch_ex(Kern kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// the same with thread-block clusters of `cluster_x` CTAs along x
template <typename Kern, typename... Args>
cudaError_t launch_cluster_ex(Kern kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl, int cluster_x,
                              Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)cluster_x;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// ------------------------------------------------------------------------------------------------------------------
// qkv_rope: one warp per row pair (j, j + d/2) of a head, so RoPE's rotate_half partner is in the same warp.
// ------------------------------------------------------------------------------------------------------------------
template <int NCH, bool KV_F32, bool Q8, bool SPEC = false>
__global__ void __launch_bounds__(128) qkv_rope_kernel(QkvArgs a) {
    const CtaTrace trace_(a.trace);
    constexpr int BLOCK = 128;
    constexpr int NV = Vec<NCH, BLOCK>::NV;
    extern __shared__ __align__(16) float smem[];
    float* xs = smem;
    float* red = smem + a.H;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int half = a.d >> 1;
    const int npairs = (a.qd + 2 * a.kvd) >> 1;
    const int pair = blockIdx.x * (BLOCK >> 5) + warp;
    const bool active = pair < npairs;
    const int head = pair / half, j = pair - (pair / half) * half;
    const int r0 = head * a.d + j, r1 = r0 + half;

    const unsigned char* wb = static_cast<const unsigned char*>(a.w);
    const size_t rbh = wrow_bytes(a.H, Q8);
    WRow<NCH, Q8> w0, w1;
    w0.load(wb + (size_t)r0 * rbh, a.H, lane, active);
    w1.load(wb + (size_t)r1 * rbh, a.H, lane, active);
    float4 ln[NV];
    vec_load_ldg<BLOCK, NV>(a.ln, a.H, ln);
    // predicted routing: this CTA's router row times the MoE norm weight, in the layout of v
    const bool spec = SPEC && (int)blockIdx.x < a.spec_E;  // a separate instantiation: its registers cost the chain
    float4 sw4[NV];
    if (spec) {
        const uint2* rr = reinterpret_cast<const uint2*>(a.spec_router + (size_t)blockIdx.x * a.H);  // 4 bf16 per uint2
#pragma unroll
        for (int k = 0; k < NV; ++k) {
            const int i = threadIdx.x + k * BLOCK;
            if (4 * i < a.H) {
                const uint2 u = __ldg(rr + i);
                const float4 l4 = __ldg(reinterpret_cast<const float4*>(a.spec_ln) + i);
                sw4[k] = make_float4(bf_lo(u.x) * l4.x, bf_hi(u.x) * l4.y, bf_lo(u.y) * l4.z, bf_hi(u.y) * l4.w);
            } else {
                sw4[k] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
    }
    // The position changes only in the previous step's head kernel, which completed before this step's first kernel
    // started (that launch is not programmatic): so the position, its RoPE row and the K/V page of this token are
    // final before the wait, and their loads leave the critical path.
    const int pos = __ldcg(a.pos);
    float rc = 1.0f, rs = 0.0f;
    int page = 0;
    if (active && lane == 0) {
        rc = __ldg(a.rope_cs + (size_t)pos * a.d + j);
        rs = __ldg(a.rope_cs + (size_t)pos * a.d + half + j);
        if (r0 >= a.qd) page = __ldcg(a.page_table + pos / a.page_size);
    }

    pdl_wait();
    pdl_launch();
    trace_.released();

    float4 v[NV];
    if (a.embed_mode) {
        if (a.step_ctr && blockIdx.x == 0 && threadIdx.x == 0) *a.step_ctr += 1;  // read only by later kernels
        // model.rs:134-138: embedding row x embedding_multiplier is the residual stream of layer 0
        const int tok = __ldcg(a.token);
        const uint2* er = reinterpret_cast<const uint2*>(a.embed + (size_t)tok * a.H);  // 4 bf16 per uint2
#pragma unroll
        for (int k = 0; k < NV; ++k) {
            const int i = threadIdx.x + k * BLOCK;
            if (4 * i < a.H) {
                const uint2 u = __ldg(er + i);
                v[k] = make_float4(__fmul_rn(bf_lo(u.x), a.emb_mult), __fmul_rn(bf_hi(u.x), a.emb_mult),
                                   __fmul_rn(bf_lo(u.y), a.emb_mult), __fmul_rn(bf_hi(u.y), a.emb_mult));
                if (blockIdx.x == 0) reinterpret_cast<float4*>(a.h_write)[i] = v[k];
            } else {
                v[k] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
    } else {
        vec_load_cg<BLOCK, NV>(a.h, a.H, v);
    }
    norm_regs<BLOCK, NV>(v, ln, a.H, a.eps, xs, red);
    if (spec) {
        float p = 0.0f;
#pragma unroll
        for (int k = 0; k < NV; ++k) {
            p = fmaf(sw4[k].x, v[k].x, p);
            p = fmaf(sw4[k].y, v[k].y, p);
            p = fmaf(sw4[k].z, v[k].z, p);
            p = fmaf(sw4[k].w, v[k].w, p);
        }
        p = block_sum(p, red);
        if (threadIdx.x == 0) a.spec_out[blockIdx.x] = p;
        if (a.spec_ids) {
            // the last of the spec_E CTAs takes the predicted top-k (block.rs:81-89's order)
            __shared__ bool s_last;
            __shared__ int s_id[kMaxTopK];
            __shared__ float s_val[kMaxTopK], s_w[kMaxTopK];
            if (last_block_arrives(a.spec_ticket, (unsigned int)a.spec_E, &s_last) && warp == 0) {
                const float v0 = lane < a.spec_E ? __ldcg(a.spec_out + lane) : 0.0f;
                const float v1 = lane + 32 < a.spec_E ? __ldcg(a.spec_out + lane + 32) : 0.0f;
                route_topk_warp(v0, v1, a.spec_E, a.spec_k, s_id, s_val, s_w);
                if (lane < a.spec_k) a.spec_ids[lane] = s_id[lane];
            }
        }
    }
    trace_.mark(0);
    if (!active) return;

    const float x1 = warp_sum(w0.dot(xs, a.H, lane));
    const float x2 = warp_sum(w1.dot(xs, a.H, lane));
    if (lane != 0) return;
    // model.rs:153-155: x1*c - x2*s, x2*c + x1*s (no contraction)
    const float ro0 = __fsub_rn(__fmul_rn(x1, rc), __fmul_rn(x2, rs));
    const float ro1 = __fadd_rn(__fmul_rn(x2, rc), __fmul_rn(x1, rs));
    if (r0 < a.qd) {
        a.q_out[r0] = ro0;
        a.q_out[r1] = ro1;
        return;
    }
    int rr = r0 - a.qd;
    const bool is_k = rr < a.kvd;
    if (!is_k) rr -= a.kvd;
    const int kvh = rr / a.d;
    const float v0 = is_k ? ro0 : x1, v1 = is_k ? ro1 : x2;
    const int slot = pos % a.page_size;
    const size_t base = (((size_t)page * a.kv_heads + kvh) * a.page_size + slot) * a.d;
    void* pool = is_k ? a.k_pool : a.v_pool;
    if (KV_F32) {
        float* p = static_cast<float*>(pool) + base;
        p[j] = v0;
        p[j + half] = v1;
    } else {
        uint16_t* p = static_cast<uint16_t*>(pool) + base;
        p[j] = f32_to_bf16_rne(v0);
        p[j + half] = f32_to_bf16_rne(v1);
    }
}

// ------------------------------------------------------------------------------------------------------------------
// attention: CTA (split s, KV head).  Split s owns the positions [len*s/NS, len*(s+1)/NS).  K/V rows before `pos` do
// not change during a decode step (only the new row `pos` is written, by this layer's qkv kernel), so before
// griddepcontrol.wait the CTA streams its K and V rows out of the paged cache into shared memory with bulk async
// copies (one thread per page run); after it the CTA reads q and the new row.  Each lane scores one position against
// the G query heads of the group (GQA: K/V read once for all G heads), warps keep online-softmax partials and merge
// them in shared memory, and the CTA writes its partial (m, l, acc) per query head; the output-projection kernel
// merges the splits as it loads the attention output (flash-decoding), or the last CTA of each KV head merges them
// (lastro_model_set_tuning).  Positions past `len` are never read.
// ------------------------------------------------------------------------------------------------------------------
constexpr int kAttnWarps = 8;

// this CTA's share (cta of ctas) of the k predicted experts' gate_up and down weights, k x (gu + dn) bytes in expert
// order, hinted into L2; one thread
LDEV void spec_prefetch_share(const int* ids, int k, int E, const void* gu_w, unsigned long long gu_bytes,
                              const void* dn_w, unsigned long long dn_bytes, int cta, int ctas) {
    const unsigned long long per = gu_bytes + dn_bytes, all = per * k;
    const unsigned long long share = ((all + ctas - 1) / ctas + 15) & ~15ull;
    unsigned long long o = share * cta;
    const unsigned long long o1 = min(all, o + share);
    while (o < o1) {
        const int sl = (int)(o / per);
        const unsigned long long in = o - (unsigned long long)sl * per;
        const int e = min(max(ids[sl], 0), E - 1);
        const bool gu = in < gu_bytes;
        const unsigned long long part = gu ? gu_bytes : dn_bytes, at = gu ? in : in - gu_bytes;
        const unsigned long long n = min(o1 - o, part - at);
        bulk_prefetch_l2(static_cast<const unsigned char*>(gu ? gu_w : dn_w) + (size_t)e * part + at, (uint32_t)n);
        o += n;
    }
}

// One warp's share of a split on tensor cores (bf16 K/V): the warp takes the split's rows in groups of 16 (positions
// p0 + g0 .. g0 + 15 at staged row g0 + roff; K/V rows of 128 bytes, 128-byte swizzled when `swizzled`).  Per group
// S = Q K^T with the G query heads as the MMA's 16 rows (padded with zeros) and q split into bf16 hi + lo, the online
// softmax per head across the quad of lanes that holds it, and O += P V with P split into hi + lo from the S
// fragments and V through ldmatrix.trans.  Rows past the split re-read its last row (finite) and get P = 0.  Writes
// the warp's (m, l, acc) for the G heads.
template <int G>
LDEV void attention_rows_mma(const AttnArgs& a, const unsigned char* kt, const unsigned char* vt,
                             const float (*sq)[kHeadDim], int roff, bool swizzled, int nrow, float* wm, float* wl,
                             float (*wacc)[kHeadDim]) {
    constexpr int NW = kAttnWarps;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, gq = lane >> 2, tq = lane & 3;
    const int mi = lane >> 3, r8 = lane & 7;
    uint32_t qh[4][2], ql[4][2];
#pragma unroll
    for (int kk = 0; kk < 4; ++kk)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
            float2 v = make_float2(0.f, 0.f);
            if (gq < G) v = *reinterpret_cast<const float2*>(&sq[gq][16 * kk + 8 * hf + 2 * tq]);
            uint16_t h0, l0, h1, l1;
            split_bf16(v.x, h0, l0);
            split_bf16(v.y, h1, l1);
            qh[kk][hf] = pack_bf16(h0, h1);
            ql[kk][hf] = pack_bf16(l0, l1);
        }
    const uint32_t sK = smem_addr(kt), sV = smem_addr(vt);
    const int last = roff + nrow - 1;  // staged row of the split's last position
    auto row_addr = [&](uint32_t base, int row, int chunk) {
        row = min(row, last);
        return base + (swizzled ? swz(row, chunk) : (uint32_t)(row * 128 + (chunk << 4)));
    };
    float mr = -INFINITY, lr = 0.0f;
    float o[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int c = 0; c < 4; ++c) o[j][c] = 0.0f;
    for (int g0 = warp * 16; g0 < nrow; g0 += NW * 16) {
        const int ib = g0 + roff;
        float sf[2][4];
#pragma unroll
        for (int q = 0; q < 2; ++q)
#pragma unroll
            for (int c = 0; c < 4; ++c) sf[q][c] = 0.0f;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            uint32_t b[4];
            ldsm_x4(row_addr(sK, ib + (mi >> 1) * 8 + r8, kk * 2 + (mi & 1)), b);
            const uint32_t ah[4] = {qh[kk][0], 0u, qh[kk][1], 0u}, al[4] = {ql[kk][0], 0u, ql[kk][1], 0u};
            mma_bf16(sf[0], ah, b[0], b[1]);
            mma_bf16(sf[1], ah, b[2], b[3]);
            mma_bf16(sf[0], al, b[0], b[1]);
            mma_bf16(sf[1], al, b[2], b[3]);
        }
        const int rr[4] = {g0 + 2 * tq, g0 + 2 * tq + 1, g0 + 8 + 2 * tq, g0 + 9 + 2 * tq};
        const float raw[4] = {sf[0][0], sf[0][1], sf[1][0], sf[1][1]};
        float sc[4], cmax = -INFINITY;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            sc[i] = rr[i] < nrow ? __fmul_rn(raw[i], a.scale) : -INFINITY;
            cmax = fmaxf(cmax, sc[i]);
        }
        cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, 1));
        cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, 2));
        const float mn = fmaxf(mr, cmax);
        const float alpha = mr == -INFINITY ? 0.0f : expf(mr - mn);
        float pv[4], ps = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            pv[i] = rr[i] < nrow ? expf(sc[i] - mn) : 0.0f;
            ps += pv[i];
        }
        ps += __shfl_xor_sync(0xffffffffu, ps, 1);
        ps += __shfl_xor_sync(0xffffffffu, ps, 2);
        lr = lr * alpha + ps;
        mr = mn;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            o[j][0] *= alpha;
            o[j][1] *= alpha;
        }
        uint16_t h[4], l[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) split_bf16(pv[i], h[i], l[i]);
        const uint32_t ph[4] = {pack_bf16(h[0], h[1]), 0u, pack_bf16(h[2], h[3]), 0u};
        const uint32_t pl[4] = {pack_bf16(l[0], l[1]), 0u, pack_bf16(l[2], l[3]), 0u};
#pragma unroll
        for (int jp = 0; jp < 4; ++jp) {
            uint32_t b[4];
            ldsm_x4_trans(row_addr(sV, ib + (mi & 1) * 8 + r8, 2 * jp + (mi >> 1)), b);
            mma_bf16(o[2 * jp], ph, b[0], b[1]);
            mma_bf16(o[2 * jp + 1], ph, b[2], b[3]);
            mma_bf16(o[2 * jp], pl, b[0], b[1]);
            mma_bf16(o[2 * jp + 1], pl, b[2], b[3]);
        }
    }
    if (gq < G) {
        if (tq == 0) {
            wm[gq] = mr;
            wl[gq] = lr;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            wacc[gq][8 * j + 2 * tq] = o[j][0];
            wacc[gq][8 * j + 2 * tq + 1] = o[j][1];
        }
    }
}

// MODE (bf16 K/V only; 0 with f32 K/V): bit 0 stages K/V as 8-row TMA boxes with the 128-byte swizzle (AttnArgs tma),
// bit 1 scores and sums on tensor cores (AttnArgs mma); mode 0 is the default chain's form
template <bool KV_F32, int G, bool CL, int MODE = 0>
__global__ void __launch_bounds__(32 * kAttnWarps) attention_kernel(const __grid_constant__ CUtensorMap kmap,
                                                                    const __grid_constant__ CUtensorMap vmap, AttnArgs a) {
    const CtaTrace trace_(a.trace);
    constexpr int D = kHeadDim;
    constexpr int NW = kAttnWarps;
    constexpr int ESZ = KV_F32 ? 4 : 2;
    constexpr int RB = D * ESZ;  // bytes per K/V row of one head
    constexpr int CH = RB / 16;  // 16-byte chunks per row
    static_assert(KV_F32 || RB == 128, "swizzled boxes hold 128-byte rows");
    extern __shared__ __align__(128) unsigned char smem_raw[];
    // tma: K/V staged as 8-row boxes (TMA, 128-byte swizzle) from position p0 rounded down to a multiple of 8, each
    // box 1024-byte aligned; else one bulk copy per page run from position p0, unswizzled
    constexpr bool tma = !KV_F32 && (MODE & 1);
    const int cap = tma ? attn_tma_rows(a.split_cap) : a.split_cap;
    unsigned char* kt = tma ? reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023)
                            : smem_raw;  // [cap, RB]
    unsigned char* vt = kt + (size_t)cap * RB;  // [cap, RB]
    __shared__ __align__(16) float sq[G][D];
    __shared__ float wm[NW][G], wl[NW][G];
    __shared__ __align__(16) float wacc[NW][G][D];
    __shared__ __align__(8) uint64_t bar;
    __shared__ float cw[kAttnSplits][G], cden[G];
    __shared__ bool is_last;
    __shared__ float cM[G], cL[G];            // CL: this CTA's partial, read by the other CTAs of its cluster
    __shared__ __align__(16) float cA[G][D];
    const int NS = gridDim.x, s = blockIdx.x, kvh = blockIdx.y, z = blockIdx.z;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int HD = a.kv_heads * G * D;  // q / output floats of one token
    const int seq_id = a.seq ? __ldg(a.seq + z) : 0;
    const int* page_table = a.page_table + (size_t)seq_id * a.pt_stride;
    float* part_acc = a.part_acc + (size_t)z * HD * NS;
    float* part_ml = a.part_ml + (size_t)z * a.kv_heads * G * NS * 2;
    float* att_out = a.att_out + (size_t)z * HD;

    // the position is written only by the previous step's head kernel: constant for the whole step
    const int pos = __ldcg(a.pos + seq_id);
    const int len = pos + 1;
    const int p0 = (int)(((long long)len * s) / NS), p1 = (int)(((long long)len * (s + 1)) / NS);
    const int pb = min(p1, pos);  // rows [p0, pb) are final already
    const int r_base = tma ? (p0 & ~7) : p0;  // position of staged row 0
    const int roff = p0 - r_base;
    constexpr int swz = tma ? 7 : 0;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        uint32_t tx = 0u;
        if (pb > p0) tx = tma ? (uint32_t)(((pb - 1) >> 3) - (p0 >> 3) + 1) * 2u * 8u * RB : (uint32_t)(pb - p0) * RB * 2;
        mbar_expect_tx(&bar, tx);
    }
    __syncthreads();
    if (pb > p0 && tma) {
        // one thread per 8-row box (a box never crosses a page: page_size is a multiple of 8); rows of the box outside
        // [p0, pb) are in the same page and are never read
        const int g0 = p0 >> 3, ng = ((pb - 1) >> 3) - g0 + 1;
        for (int t = threadIdx.x; t < ng; t += blockDim.x) {
            const int row = (g0 + t) << 3, pg = row / a.page_size, slot = row - pg * a.page_size;
            const int y = (__ldcg(page_table + pg) * a.kv_heads + kvh) * a.page_size + slot;
            tma_load_2d(kt + (size_t)(row - r_base) * RB, &kmap, 0, y, &bar);
            tma_load_2d(vt + (size_t)(row - r_base) * RB, &vmap, 0, y, &bar);
        }
    } else if (pb > p0) {
        // one thread per page run: page-table reads and copies all in flight together
        const int pg0 = p0 / a.page_size, pg1 = (pb - 1) / a.page_size;
        for (int t = threadIdx.x; t <= pg1 - pg0; t += blockDim.x) {
            const int pg = pg0 + t;
            const int lo = max(p0, pg * a.page_size), hi = min(pb, (pg + 1) * a.page_size);
            const int page = __ldcg(page_table + pg);
            const size_t off = (((size_t)page * a.kv_heads + kvh) * a.page_size + (lo - pg * a.page_size)) * RB;
            bulk_g2s(kt + (size_t)(lo - p0) * RB, static_cast<const unsigned char*>(a.k_pool) + off, (uint32_t)(hi - lo) * RB, &bar);
            bulk_g2s(vt + (size_t)(lo - p0) * RB, static_cast<const unsigned char*>(a.v_pool) + off, (uint32_t)(hi - lo) * RB, &bar);
        }
    }

    pdl_wait();
    pdl_launch();
    trace_.released();

    if constexpr ((MODE & 4) != 0) {
        // this CTA's share of the predicted experts' weights into L2 (the routing of this layer is ~10 us away)
        if (threadIdx.x == 32) {
            int ids[kMaxTopK];
#pragma unroll
            for (int j = 0; j < kMaxTopK; ++j) ids[j] = j < a.spec_k ? __ldcg(a.spec_ids + j) : 0;
            spec_prefetch_share(ids, a.spec_k, a.spec_E, a.spec_gu, a.spec_gu_bytes, a.spec_dn, a.spec_dn_bytes,
                                blockIdx.x + gridDim.x * blockIdx.y, gridDim.x * gridDim.y);
        }
    }
    for (int i = threadIdx.x; i < G * D / 4; i += blockDim.x)
        reinterpret_cast<float4*>(&sq[0][0])[i] = __ldcg(reinterpret_cast<const float4*>(a.q + (size_t)z * HD + (size_t)kvh * G * D) + i);
    // with boxes, the box that holds the new row's slot carries its stale copy: the row is written after they land
    bool ok = tma ? mbar_wait(&bar, 0, a.err, 3) : true;
    if (pos >= p0 && pos < p1 && threadIdx.x < 2 * CH) {
        // the row this layer's qkv kernel just appended
        const int pg = pos / a.page_size, slot = pos - pg * a.page_size;
        const size_t off = (((size_t)__ldcg(page_table + pg) * a.kv_heads + kvh) * a.page_size + slot) * RB;
        const int c = threadIdx.x % CH, i = pos - r_base;
        const bool is_v = threadIdx.x >= CH;
        const uint4* src = reinterpret_cast<const uint4*>(static_cast<const unsigned char*>(is_v ? a.v_pool : a.k_pool) + off);
        reinterpret_cast<uint4*>((is_v ? vt : kt) + (size_t)i * RB)[c ^ (i & swz)] = __ldcg(src + c);
    }
    __syncthreads();
    if (!tma) ok = mbar_wait(&bar, 0, a.err, 3);
    trace_.mark(0);

    float m[G], l[G], acc0[G], acc1[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.0f;
        acc0[g] = 0.0f;
        acc1[g] = 0.0f;
    }
    const int nrow = ok ? p1 - p0 : 0;
    if constexpr (!KV_F32 && (MODE & 2)) {
        attention_rows_mma<G>(a, kt, vt, sq, roff, tma, nrow, wm[warp], wl[warp], wacc[warp]);
    } else {
    for (int base = warp * 32; base < nrow; base += NW * 32) {
        const int r = base + lane;
        const bool valid = r < nrow;
        float sc[G];
#pragma unroll
        for (int g = 0; g < G; ++g) sc[g] = 0.0f;
        if (valid) {
            // staged row of position p0 + r, and its 16-byte chunks' swizzle (lanes read rows of one 8-row box:
            // chunk c of eight consecutive rows lands in eight different bank groups)
            const int i = r + roff, sw = i & swz;
            const uint4* kr = reinterpret_cast<const uint4*>(kt + (size_t)i * RB);
#pragma unroll
            for (int c = 0; c < CH; ++c) {
                const uint4 kc = kr[c ^ sw];
                // the row's elements are unpacked once and used for all G heads
                float kf[8];
                if (KV_F32) {
                    kf[0] = __uint_as_float(kc.x);
                    kf[1] = __uint_as_float(kc.y);
                    kf[2] = __uint_as_float(kc.z);
                    kf[3] = __uint_as_float(kc.w);
                } else {
                    kf[0] = bf_lo(kc.x);
                    kf[1] = bf_hi(kc.x);
                    kf[2] = bf_lo(kc.y);
                    kf[3] = bf_hi(kc.y);
                    kf[4] = bf_lo(kc.z);
                    kf[5] = bf_hi(kc.z);
                    kf[6] = bf_lo(kc.w);
                    kf[7] = bf_hi(kc.w);
                }
                constexpr int EPC = KV_F32 ? 4 : 8;
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    const float* qg = &sq[g][c * EPC];
#pragma unroll
                    for (int e = 0; e < EPC; ++e) sc[g] = fmaf(qg[e], kf[e], sc[g]);
                }
            }
        }
        float pr[G];
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const float scv = valid ? __fmul_rn(sc[g], a.scale) : -INFINITY;
            const float mn = fmaxf(m[g], warp_max(scv));
            pr[g] = valid ? expf(scv - mn) : 0.0f;
            const float alpha = (m[g] == -INFINITY) ? 0.0f : expf(m[g] - mn);
            l[g] = l[g] * alpha + warp_sum(pr[g]);
            acc0[g] *= alpha;
            acc1[g] *= alpha;
            m[g] = mn;
        }
        const int nj = min(32, nrow - base);
        for (int jj = 0; jj < nj; ++jj) {
            const int i = base + jj + roff;
            float v0, v1;
            if (KV_F32) {
                const float2 t = reinterpret_cast<const float2*>(vt + (size_t)i * RB)[lane];
                v0 = t.x;
                v1 = t.y;
            } else {
                // lane's word (elements 2 lane, 2 lane + 1) sits in chunk lane / 4, swizzled like the K rows
                const uint32_t t =
                    reinterpret_cast<const uint32_t*>(vt + (size_t)i * RB)[(((lane >> 2) ^ (i & swz)) << 2) | (lane & 3)];
                v0 = bf_lo(t);
                v1 = bf_hi(t);
            }
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const float pj = __shfl_sync(0xffffffffu, pr[g], jj);
                acc0[g] = fmaf(pj, v0, acc0[g]);
                acc1[g] = fmaf(pj, v1, acc1[g]);
            }
        }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
        if (lane == 0) {
            wm[warp][g] = m[g];
            wl[warp][g] = l[g];
        }
        wacc[warp][g][2 * lane] = acc0[g];
        wacc[warp][g][2 * lane + 1] = acc1[g];
    }
    }
    trace_.mark(3);
    __syncthreads();
    trace_.mark(4);
    // this CTA's partial: warps merged; layout [head][split][...] so the consumer reads each head's splits together
    for (int t = threadIdx.x; t < G * D; t += blockDim.x) {
        const int g = t / D, dim = t - (t / D) * D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < NW; ++w) M = fmaxf(M, wm[w][g]);
        float L = 0.0f, A = 0.0f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < NW; ++w) {
                if (wm[w][g] == -INFINITY) continue;
                const float e = expf(wm[w][g] - M);
                L = fmaf(wl[w][g], e, L);
                A = fmaf(wacc[w][g][dim], e, A);
            }
        }
        if (CL) {
            cA[g][dim] = A;
            if (dim == 0) {
                cM[g] = M;
                cL[g] = L;
            }
        } else {
            const size_t hs = (size_t)(kvh * G + g) * NS + s;
            part_acc[hs * D + dim] = A;
            if (dim == 0) {
                part_ml[hs * 2] = M;
                part_ml[hs * 2 + 1] = L;
            }
        }
    }
    trace_.mark(1);
    if (CL) {
        // the NS splits of this KV head are one thread-block cluster: after a cluster barrier each CTA merges its
        // share of the G*D outputs from every CTA's partial in distributed shared memory (splits in order); a second
        // barrier keeps every CTA's shared memory alive until the others have read it
        namespace cg = cooperative_groups;
        cg::cluster_group cl = cg::this_cluster();
        cl.sync();
        const int per = (G * D + NS - 1) / NS;
        for (int t = threadIdx.x; t < per; t += blockDim.x) {
            const int o = s * per + t;
            if (o >= G * D) break;
            const int g = o / D, dim = o - (o / D) * D;
            float mq[kAttnSplits];
            float M = -INFINITY;
#pragma unroll
            for (int q = 0; q < kAttnSplits; ++q) {
                mq[q] = q < NS ? *cl.map_shared_rank(&cM[g], q) : -INFINITY;
                M = fmaxf(M, mq[q]);
            }
            float dn = 0.0f, num = 0.0f;
#pragma unroll
            for (int q = 0; q < kAttnSplits; ++q) {
                if (q >= NS || mq[q] == -INFINITY) continue;
                const float e = expf(mq[q] - M);
                dn = fmaf(*cl.map_shared_rank(&cL[g], q), e, dn);
                num = fmaf(*cl.map_shared_rank(&cA[g][dim], q), e, num);
            }
            att_out[((size_t)kvh * G + g) * D + dim] = num / dn;
        }
        cl.sync();
        trace_.mark(2);
        return;
    }
    if (!a.merge) return;  // the output projection merges the partials as it loads them
    // else the last CTA of this KV head merges the NS (<= 16) splits of its G heads: every load (each thread's NS
    // partial outputs, and one (m, l) pair per (head, split)) in one round, the per-head max and denominator by
    // 16-lane shuffles over the splits (padded with empty ones)
    if (!last_block_arrives(a.counters + (size_t)z * a.kv_heads + kvh, (unsigned int)NS, &is_last)) return;
    constexpr int NT = 32 * kAttnWarps, KO = (G * D + NT - 1) / NT;
    const float* pa = part_acc + (size_t)kvh * G * NS * D;
    float v[KO][kAttnSplits];
#pragma unroll
    for (int k = 0; k < KO; ++k) {
        const int t = threadIdx.x + k * NT;
        const int g = t / D, dim = t - (t / D) * D;
#pragma unroll
        for (int sp = 0; sp < kAttnSplits; ++sp)
            v[k][sp] = (t < G * D && sp < NS) ? __ldcg(pa + ((size_t)g * NS + sp) * D + dim) : 0.0f;
    }
    const int i = threadIdx.x, ig = i / kAttnSplits, isp = i - ig * kAttnSplits;
    const float2 mlv = (ig < G && isp < NS)
                           ? __ldcg(reinterpret_cast<const float2*>(part_ml) + (size_t)(kvh * G + ig) * NS + isp)
                           : make_float2(-INFINITY, 0.0f);
    if (i < ((G * kAttnSplits + 31) & ~31)) {  // whole warps
        float M = mlv.x;
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o, 16));
        const float e = mlv.x == -INFINITY ? 0.0f : expf(mlv.x - M);
        float dn = mlv.y * e;
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) dn += __shfl_xor_sync(0xffffffffu, dn, o, 16);
        if (i < G * kAttnSplits) {
            cw[isp][ig] = e;
            if (isp == 0) cden[ig] = dn;
        }
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < KO; ++k) {
        const int t = threadIdx.x + k * NT;
        if (t >= G * D) break;
        const int g = t / D, dim = t - (t / D) * D;
        float num = 0.0f;
#pragma unroll
        for (int sp = 0; sp < kAttnSplits; ++sp) num = fmaf(v[k][sp], cw[sp][g], num);
        att_out[((size_t)kvh * G + g) * D + dim] = num / cden[g];
    }
    trace_.mark(2);
}

template <int NCH, bool Q8>
__global__ void __launch_bounds__(128) router_kernel(RouterArgs a) {
    constexpr int BLOCK = 128;
    constexpr int NV = Vec<NCH, BLOCK>::NV;
    extern __shared__ __align__(16) float smem[];
    float* xs = smem;
    float* red = smem + a.H;
    __shared__ bool is_last;
    __shared__ int sid[kMaxTopK];
    __shared__ float sval[kMaxTopK], sw[kMaxTopK];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int e = blockIdx.x * (BLOCK >> 5) + warp;
    const bool active = e < a.E;
    WRow<NCH, Q8> w;
    w.load(static_cast<const unsigned char*>(a.w) + (size_t)e * wrow_bytes(a.H, Q8), a.H, lane, active);
    float4 ln[NV];
    if (a.norm_mode) vec_load_ldg<BLOCK, NV>(a.ln, a.H, ln);
    pdl_wait();
    pdl_launch();
    if (a.norm_mode) {
        float4 v[NV];
        vec_load_cg<BLOCK, NV>(a.x, a.H, v);
        const float r = norm_regs<BLOCK, NV>(v, ln, a.H, a.eps, xs, red);
        if (blockIdx.x == 0 && threadIdx.x == 0) *a.rnorm_out = r;
    } else {
        copy_to_smem<BLOCK>(a.x, a.H, xs);
    }
    if (active) {
        const float lg = warp_sum(w.dot(xs, a.H, lane));
        if (lane == 0) a.logits[e] = lg;
    }
    if (!last_block_arrives(a.counter, gridDim.x, &is_last)) return;
    if (warp != 0) return;
    const float v0 = lane < a.E ? __ldcg(a.logits + lane) : 0.0f;
    const float v1 = lane + 32 < a.E ? __ldcg(a.logits + lane + 32) : 0.0f;
    route_topk_warp(v0, v1, a.E, a.k, sid, sval, sw);
    if (lane < a.k) {
        a.ids[lane] = sid[lane];
        a.weights[lane] = sw[lane];
    }
}

// ------------------------------------------------------------------------------------------------------------------
// oproj (+ router): warp w of CTA b computes rows r = 32b + 2w, 2w+1: h[r] += resid * (W_o[r] . att)
// (model.rs:223-227).  With `route` set the MoE router is folded in: RMSNorm(h) . W_r^T equals
// r_norm * sum_c (W_r[e,c] * ln[c]) * h[c], so each CTA adds its 32 rows' share of every logit (from W_r^T scaled by
// ln, [H, E], prepared once per layer) and of sum h^2; the last CTA sums the shares in a fixed order, applies r_norm,
// and takes the top-k with block.rs:81-89's order and softmax.  The experts kernel reads r_norm.
// ------------------------------------------------------------------------------------------------------------------
// 48 CTAs for the 3B shape: more, smaller CTAs (192 x 8 rows measured 0.25 us faster here) make every gate_up and
// down CTA reduce 4x the router shares, and those few kilobytes, read by ~450 CTAs at once, cost gate_up's routing
// 1.1 us (C3: 1.066 vs 1.060 ms per step)
constexpr int kOpWarps = 16;
constexpr int kOpRows = 2 * kOpWarps;

// The attention output from the attention kernel's per-split partials (flash-decoding): for head h,
// att[h] = sum_s acc[h][s] * e_s / sum_s l[h][s] * e_s with e_s = exp(m[h][s] - max_s m[h][s]), splits in order.  Every
// partial is loaded at once into shared memory (one round of L2 latency), then weighted.  xs receives [heads * D].
template <int BLOCK>
LDEV void merge_attention(const OprojArgs& a, float* xs, float* pacc, float* pml, float* pw) {
    constexpr int D = kHeadDim;
    const int S = a.splits, HS = a.heads * S;
    const int n4 = HS * D / 4;
    const float4* src = reinterpret_cast<const float4*>(a.part_acc);
    for (int i = threadIdx.x; i < n4; i += BLOCK) reinterpret_cast<float4*>(pacc)[i] = __ldcg(src + i);
    for (int i = threadIdx.x; i < HS; i += BLOCK)
        reinterpret_cast<float2*>(pml)[i] = __ldcg(reinterpret_cast<const float2*>(a.part_ml) + i);
    __syncthreads();
    for (int h = threadIdx.x; h < a.heads; h += BLOCK) {
        float M = -INFINITY;
        for (int sp = 0; sp < S; ++sp) M = fmaxf(M, pml[2 * (h * S + sp)]);
        float L = 0.0f;
        for (int sp = 0; sp < S; ++sp) {
            const float m = pml[2 * (h * S + sp)];
            const float e = m == -INFINITY ? 0.0f : expf(m - M);
            pw[h * S + sp] = e;
            L = fmaf(pml[2 * (h * S + sp) + 1], e, L);
        }
        pw[HS + h] = L;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < a.heads * D; i += BLOCK) {
        const int h = i / D, dim = i - h * D;
        float num = 0.0f;
        for (int sp = 0; sp < S; ++sp) num = fmaf(pacc[(h * S + sp) * D + dim], pw[h * S + sp], num);
        xs[i] = num / pw[HS + h];
    }
    __syncthreads();
}

// The predicted top-k (OprojArgs spec) ranked like the routing, then this CTA's share of the k experts' gate_up and
// down weights (k x (gu + dn) bytes in expert order) hinted into L2 by thread 0.  Every thread of the block calls it.
LDEV void spec_prefetch_l2(const OprojArgs& a) {
    __shared__ unsigned long long key[kMaxExperts];
    __shared__ int pid[kMaxTopK];
    if ((int)threadIdx.x < a.spec_E) key[threadIdx.x] = route_key(__ldcg(a.spec + threadIdx.x), threadIdx.x);
    __syncthreads();
    if ((int)threadIdx.x < a.spec_E) {
        const unsigned long long me = key[threadIdx.x];
        int rank = 0;
        for (int j = 0; j < a.spec_E; ++j) rank += (int)(key[j] > me);
        if (rank < a.spec_k) pid[rank] = threadIdx.x;
    }
    __syncthreads();
    if (threadIdx.x != 0) return;
    spec_prefetch_share(pid, a.spec_k, a.spec_E, a.spec_gu, a.spec_gu_bytes, a.spec_dn, a.spec_dn_bytes, blockIdx.x,
                        gridDim.x);
}

template <int NCH, bool Q8, bool SPEC = false>
__global__ void __launch_bounds__(512) oproj_kernel(OprojArgs a) {
    const CtaTrace trace_(a.trace);
    constexpr int BLOCK = 32 * kOpWarps;
    extern __shared__ __align__(16) float smem[];
    float* xs = smem;          // [qd]
    float* wrs = smem + a.qd;  // [kOpRows, E]
    __shared__ float hs[kOpRows];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int r0 = blockIdx.x * kOpRows;
    const int ra = r0 + 2 * warp, rb = ra + 1;
    const unsigned char* wbase = static_cast<const unsigned char*>(a.w);
    const size_t rbq = wrow_bytes(a.qd, Q8);
    WRow<NCH, Q8> wa, wb;
    wa.load(wbase + (size_t)ra * rbq, a.qd, lane, ra < a.H);
    wb.load(wbase + (size_t)rb * rbq, a.qd, lane, rb < a.H);
    if (a.route) {
        const int n = kOpRows * a.E;
        for (int t = threadIdx.x; t < n; t += BLOCK) wrs[t] = (r0 + t / a.E < a.H) ? __ldg(a.wr_t + (size_t)r0 * a.E + t) : 0.0f;
    }
    if (SPEC) spec_prefetch_l2(a);  // a separate instantiation: the default one carries none of it
    pdl_wait();
    pdl_launch();
    trace_.released();
    const float ha = (lane == 0 && ra < a.H) ? __ldcg(a.h + ra) : 0.0f;
    const float hb = (lane == 0 && rb < a.H) ? __ldcg(a.h + rb) : 0.0f;
    if (a.part_acc) {
        // after xs and the router operand: the partials [heads*S*D], their (m, l) [heads*S*2], weights and sums
        float* pacc = wrs + (a.route ? (size_t)kOpRows * a.E : 0);
        float* pml = pacc + (size_t)a.heads * a.splits * kHeadDim;
        float* pw = pml + (size_t)a.heads * a.splits * 2;
        merge_attention<BLOCK>(a, xs, pacc, pml, pw);
    } else {
        copy_to_smem<BLOCK>(a.att, a.qd, xs);
    }
    trace_.mark(0);
    float4 xa[NCH], xb[NCH];
    x_to_regs<NCH>(xs, a.qd, lane, xa, xb);
    const float oa = warp_sum(wa.dot_regs(xa, xb, a.qd, lane));
    const float ob = warp_sum(wb.dot_regs(xa, xb, a.qd, lane));
    if (lane == 0) {
        const float na = __fadd_rn(ha, __fmul_rn(a.resid, oa)), nb = __fadd_rn(hb, __fmul_rn(a.resid, ob));
        if (ra < a.H) a.h[ra] = na;
        if (rb < a.H) a.h[rb] = nb;
        hs[2 * warp] = ra < a.H ? na : 0.0f;
        hs[2 * warp + 1] = rb < a.H ? nb : 0.0f;
    }
    trace_.mark(1);
    if (!a.route) return;
    __syncthreads();
    const int E1 = a.E + 1;
    if (threadIdx.x < a.E) {
        float p = 0.0f;
#pragma unroll 8
        for (int i = 0; i < kOpRows; ++i) p = fmaf(wrs[i * a.E + threadIdx.x], hs[i], p);
        a.shares[(size_t)blockIdx.x * E1 + threadIdx.x] = p;
    } else if (threadIdx.x == a.E) {
        float ss = 0.0f;
#pragma unroll 8
        for (int i = 0; i < kOpRows; ++i) ss = fmaf(hs[i], hs[i], ss);
        a.shares[(size_t)blockIdx.x * E1 + a.E] = ss;
    }
}

// The same output projection with its 32 weight rows staged in shared memory by one bulk copy issued before
// griddepcontrol.wait, and 256 threads (8 warps x 4 rows): about a third of the registers of the register-resident
// form, so its CTAs fit on the SMs beside the attention kernel's and their weights land while the attention still
// runs.  Every row's dot runs in the same order as oproj_kernel's: bitwise the same results.
template <int NCH, bool Q8>
__global__ void __launch_bounds__(256) oproj_smem_kernel(OprojArgs a) {
    const CtaTrace trace_(a.trace);
    constexpr int BLOCK = 256, NW = BLOCK / 32, RPW = kOpRows / NW;
    extern __shared__ __align__(128) unsigned char smem_raw[];
    const size_t rbq = wrow_bytes(a.qd, Q8);
    unsigned char* wrows = smem_raw;                                   // [kOpRows][rbq]
    float* xs = reinterpret_cast<float*>(wrows + (size_t)kOpRows * rbq);  // [qd]
    float* wrs = xs + a.qd;                                             // [kOpRows, E]
    __shared__ __align__(8) uint64_t bar;
    __shared__ float orow[kOpRows], hs[kOpRows];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int r0 = blockIdx.x * kOpRows, nrows = min(kOpRows, a.H - r0);
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        mbar_expect_tx(&bar, (uint32_t)(nrows * rbq));
        bulk_g2s(wrows, static_cast<const unsigned char*>(a.w) + (size_t)r0 * rbq, (uint32_t)(nrows * rbq), &bar);
    }
    if (a.route) {
        const int n = kOpRows * a.E;
        for (int t = threadIdx.x; t < n; t += BLOCK) wrs[t] = (r0 + t / a.E < a.H) ? __ldg(a.wr_t + (size_t)r0 * a.E + t) : 0.0f;
    }
    if (a.spec) spec_prefetch_l2(a);
    pdl_wait();
    pdl_launch();
    trace_.released();
    const float hv = threadIdx.x < nrows ? __ldcg(a.h + r0 + threadIdx.x) : 0.0f;
    copy_to_smem<BLOCK>(a.att, a.qd, xs);  // ends with __syncthreads: the barrier's initialisation is visible too
    trace_.mark(0);
    float4 xa[NCH], xb[NCH];
    x_to_regs<NCH>(xs, a.qd, lane, xa, xb);
    const bool ok = mbar_wait(&bar, 0, a.err, 5);  // on a give-up the CTA still meets its barriers, then leaves
#pragma unroll
    for (int i = 0; i < RPW; ++i) {
        const int row = warp * RPW + i;
        if (ok && row < nrows) {
            const float o = warp_sum(smem_row_dot_w<NCH, Q8>(wrows + (size_t)row * rbq, xa, xb, a.qd, lane));
            if (lane == 0) orow[row] = o;
        }
    }
    __syncthreads();
    if (!ok) return;
    if (threadIdx.x < kOpRows) {
        const float nh = threadIdx.x < nrows ? __fadd_rn(hv, __fmul_rn(a.resid, orow[threadIdx.x])) : 0.0f;
        if (threadIdx.x < nrows) a.h[r0 + threadIdx.x] = nh;
        hs[threadIdx.x] = nh;
    }
    trace_.mark(1);
    if (!a.route) return;
    __syncthreads();
    const int E1 = a.E + 1;
    if (threadIdx.x < a.E) {
        float p = 0.0f;
#pragma unroll 8
        for (int i = 0; i < kOpRows; ++i) p = fmaf(wrs[i * a.E + threadIdx.x], hs[i], p);
        a.shares[(size_t)blockIdx.x * E1 + threadIdx.x] = p;
    } else if (threadIdx.x == a.E) {
        float ss = 0.0f;
#pragma unroll 8
        for (int i = 0; i < kOpRows; ++i) ss = fmaf(hs[i], hs[i], ss);
        a.shares[(size_t)blockIdx.x * E1 + a.E] = ss;
    }
}

// W_r^T scaled by the MoE norm weight, [H, E] f32: the fused router's operand, prepared once per layer (a Q8_0 router
// weight is scale * value, exact in f32)
template <bool Q8>
__global__ void router_fold_kernel(const void* wr, const float* ln, float* wr_t, int E, int H) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= E * H) return;
    const int c = i / E, e = i - (i / E) * E;
    float w;
    if (Q8) {
        const unsigned char* row = static_cast<const unsigned char*>(wr) + (size_t)e * wrow_bytes(H, 1);
        const float sc = f16_to_f32(reinterpret_cast<const unsigned short*>(row + H)[c >> 5]);
        w = __fmul_rn(sc, (float)reinterpret_cast<const signed char*>(row)[c]);
    } else {
        w = __uint_as_float((uint32_t)static_cast<const uint16_t*>(wr)[(size_t)e * H + c] << 16);
    }
    wr_t[i] = __fmul_rn(w, ln[c]);
}

// ------------------------------------------------------------------------------------------------------------------
// gate_up: CTA per (expert slot, block of kGuPairs intermediate rows).  Thread 0 streams the block's gate rows and up
// rows into shared memory with bulk async copies, in two stages (the first half of the rows completes on its own
// barrier, so warps start on it while the second half is in flight); meanwhile the CTA builds xn = ln * (h * r).
// Warp w then computes rows j0+w and j0+w+8: g = W[e][j] . xn, u = W[e][I+j] . xn, a = silu(g) * u
// (cpu.rs:64-68, gpu.rs:45-74).  All k experts in one grid; every byte is requested at the start.
// ------------------------------------------------------------------------------------------------------------------
constexpr int kGuPairs = 16;

// the rows j0 .. j0 + 2 half of expert e (gate rows into wg, up rows into wu) in two stages completing on bar[0] and
// bar[1]; thread 0
LDEV void gu_stage(const GateUpArgs& a, int e, int j0, size_t rbh, int half, unsigned char* wg, unsigned char* wu,
                   uint64_t* bar) {
    e = min(max(e, 0), a.E - 1);  // clamped so that a stale id can never address outside the weights
    const unsigned char* base = static_cast<const unsigned char*>(a.w) + (size_t)e * 2 * a.I * rbh;
    const uint32_t bytes = (uint32_t)(half * rbh);
#pragma unroll
    for (int st = 0; st < 2; ++st) {
        mbar_expect_tx(&bar[st], 2 * bytes);
        bulk_g2s(wg + (size_t)st * half * rbh, base + (size_t)(j0 + st * half) * rbh, bytes, &bar[st]);
        bulk_g2s(wu + (size_t)st * half * rbh, base + (size_t)(a.I + j0 + st * half) * rbh, bytes, &bar[st]);
    }
}

// this CTA's share of the k experts' down slabs (k slabs of H rows) hinted into L2; thread 0
LDEV void gu_prefetch_down(const GateUpArgs& a, const int* ids) {
    const unsigned long long slab = (unsigned long long)a.H * a.down_row_bytes, all = slab * a.k;
    const unsigned long long share = ((all + gridDim.x - 1) / gridDim.x + 15) & ~15ull;
    unsigned long long o0 = share * blockIdx.x;
    const unsigned long long o1 = min(all, o0 + share);
    while (o0 < o1) {
        const int sl = (int)(o0 / slab);
        const unsigned long long in = o0 - (unsigned long long)sl * slab;
        const unsigned long long n = min(o1 - o0, slab - in);
        const int ex = min(max(ids[sl], 0), a.E - 1);
        bulk_prefetch_l2(static_cast<const unsigned char*>(a.down_w) + (size_t)ex * slab + in, (uint32_t)n);
        o0 += n;
    }
}

template <int NCH, bool Q8, bool SPEC = false>
__global__ void __launch_bounds__(256) gate_up_kernel(GateUpArgs a) {
    const CtaTrace trace_(a.trace);
    constexpr int BLOCK = 256, R = kGuPairs, HALF = R / 2;
    constexpr int NV = Vec<NCH, BLOCK>::NV;
    static_assert(HALF == BLOCK / 32, "one row pair per warp per stage");
    extern __shared__ __align__(128) unsigned char smem_raw[];
    const size_t rbh = wrow_bytes(a.H, Q8);  // bytes per weight row
    unsigned char* wg = smem_raw;             // [R] gate rows
    unsigned char* wu = wg + (size_t)R * rbh;  // [R] up rows
    float* xs = reinterpret_cast<float*>(wu + (size_t)R * rbh);
    __shared__ __align__(8) uint64_t bar[2];
    __shared__ float red[BLOCK];
    __shared__ int sid[kMaxTopK];
    __shared__ float sval[kMaxTopK], sw[kMaxTopK], s_r;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int per_slot = a.I / R;
    const int slot = blockIdx.x / per_slot, j0 = (blockIdx.x - slot * per_slot) * R;
    const bool fused = a.rs.shares != nullptr;
    const bool spec = SPEC && fused;  // a separate instantiation: the default one carries none of it
    __shared__ int spid[SPEC ? kMaxTopK : 1];                      // spec: the predicted experts by rank
    __shared__ unsigned long long spkey[SPEC ? kMaxExperts : 1];
    if (threadIdx.x == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
    }
    if (spec) {
        // the predicted top-k (the logits of the layer's input, final before this kernel started), ranked like the
        // routing; then this CTA's rows of its slot's predicted expert start streaming
        float lg = 0.0f;
        if (threadIdx.x < a.E) {
            lg = __ldcg(a.spec + threadIdx.x);
            spkey[threadIdx.x] = route_key(lg, threadIdx.x);
        }
        __syncthreads();
        if (threadIdx.x < a.E) {
            const unsigned long long me = spkey[threadIdx.x];
            int rank = 0;
            for (int j = 0; j < a.E; ++j) rank += (int)(spkey[j] > me);
            if (rank < a.k) spid[rank] = threadIdx.x;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            gu_stage(a, spid[slot], j0, rbh, HALF, wg, wu, bar);
            if (a.down_w) gu_prefetch_down(a, spid);
        }
    }
    float4 ln[NV];
    if (fused) vec_load_ldg<BLOCK, NV>(a.ln, a.H, ln);

    pdl_wait();
    pdl_launch();
    trace_.released();

    float4 v[NV];
    float r = 0.0f;
    if (fused) {
        vec_load_cg<BLOCK, NV>(a.x, a.H, v);  // in flight while the routing is reduced
        // every CTA reduces the shares (CTA 0 alone reducing them and the others waiting for its published routing
        // measured 1.4 us slower per layer: the flag's round trip outweighs the contention it saves)
        r = route_from_shares<BLOCK>(a.rs, a.E, a.k, a.H, red, sid, sval, sw, &s_r, blockIdx.x == 0, &trace_);
        // the routing warp's published stores are ordered before the flag by the block barrier above and this
        // thread's release (cumulative)
        if (a.route_flag && blockIdx.x == 0 && threadIdx.x == 0) st_release_gpu(a.route_flag, __ldcg(a.step_ctr));
    } else {
        __syncthreads();  // barrier init visible to every waiting thread
    }
    trace_.mark(0);
    int out_slot = slot;  // the routing slot whose rows j0.. this CTA computes
    uint32_t parity = 0;
    if (spec) {
        // predicted expert of this CTA's slot taken by the routing: computed where the routing put it.  Otherwise the
        // m-th such miss in slot order takes the m-th routed expert nobody predicted (as many of one as of the other)
        const int ep = spid[slot];
        int hit = -1, m = 0;
        for (int q = 0; q < a.k; ++q) hit = sid[q] == ep ? q : hit;
        if (hit >= 0) {
            out_slot = hit;
        } else {
            for (int q = 0; q < slot; ++q) {
                bool routed = false;
                for (int t = 0; t < a.k; ++t) routed |= sid[t] == spid[q];
                m += routed ? 0 : 1;
            }
            for (int q = 0; q < a.k; ++q) {
                bool predicted = false;
                for (int t = 0; t < a.k; ++t) predicted |= spid[t] == sid[q];
                if (!predicted && m-- == 0) {
                    out_slot = q;
                    break;
                }
            }
            // the predicted rows must have landed before the routed ones overwrite them
            bool ok = mbar_wait(&bar[0], 0, a.err, 1);
            ok = mbar_wait(&bar[1], 0, a.err, 1) && ok;
            if (!__syncthreads_and(ok)) return;
            if (threadIdx.x == 0) gu_stage(a, sid[out_slot], j0, rbh, HALF, wg, wu, bar);
            parity = 1;
            trace_.mark(6);  // timeline: this CTA re-staged after a misprediction
        }
    } else if (threadIdx.x == 0) {
        gu_stage(a, fused ? sid[slot] : __ldcg(a.ids + slot), j0, rbh, HALF, wg, wu, bar);
        // optional: the chosen experts' down rows hinted into L2, so the down kernel's CTAs, which find room on the
        // SMs only as these leave, read their rows from L2
        if (fused && a.down_w) gu_prefetch_down(a, sid);
    }
    if (fused) {
        // xn = ln * (h * r) (model.rs:141-145)
#pragma unroll
        for (int k = 0; k < NV; ++k) {
            const int i = threadIdx.x + k * BLOCK;
            if (4 * i < a.H) reinterpret_cast<float4*>(xs)[i] = ln_times(ln[k], v[k], r);
        }
        __syncthreads();
    } else {
        copy_to_smem<BLOCK>(a.x, a.H, xs);
    }
    float4 xa[NCH], xb[NCH];
    x_to_regs<NCH>(xs, a.H, lane, xa, xb);
#pragma unroll
    for (int st = 0; st < 2; ++st) {
        if (!mbar_wait(&bar[st], parity, a.err, 1)) return;
        trace_.mark(1 + st);
        const int pr = st * HALF + warp;
        const float g = warp_sum(smem_row_dot_w<NCH, Q8>(wg + (size_t)pr * rbh, xa, xb, a.H, lane));
        const float u = warp_sum(smem_row_dot_w<NCH, Q8>(wu + (size_t)pr * rbh, xa, xb, a.H, lane));
        if (lane == 0) a.a[(size_t)out_slot * a.I + j0 + pr] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
    }
}

// ------------------------------------------------------------------------------------------------------------------
// gate_up, streaming form (the model step): one wave of CTAs, about one per SM.  The k experts' (gate row j, up row j)
// pairs, slot-major (pair p = slot * I + j), are split into equal contiguous ranges, one per CTA.  Right after the
// routing is known every CTA requests ALL of its rows at once (a few hundred KB per SM at most, so the whole 25 MB of
// the 3B model's experts is in flight together), in kGsGroups groups that complete on their own barriers so warps
// start on the first group while the rest stream; then it hints into L2 its share of the chosen experts' down
// weights, which the down kernel reads next.  Warp w computes pairs w, w + 8, ...: a = silu(g) * u (cpu.rs:64-68).
// ------------------------------------------------------------------------------------------------------------------
constexpr int kGsGroups = 8;
constexpr int kGsThreads = 256;
constexpr int kGsMaxH = 2048;  // x staged in static shared memory

template <int NCH, bool Q8>
__global__ void __launch_bounds__(kGsThreads, 1) gate_up_stream_kernel(GateUpArgs a) {
    const CtaTrace trace_(a.trace);
    constexpr int BLOCK = kGsThreads, NW = BLOCK / 32;
    constexpr int NV = Vec<NCH, BLOCK>::NV;
    extern __shared__ __align__(128) unsigned char smem_raw[];
    const size_t rbh = wrow_bytes(a.H, Q8);
    unsigned char* wrows = smem_raw;  // [np][2][rbh]: gate row then up row of each pair
    __shared__ __align__(8) uint64_t bar[kGsGroups];
    __shared__ float red[BLOCK];
    __shared__ int sid[kMaxTopK];
    __shared__ float sval[kMaxTopK], sw[kMaxTopK], s_r;
    __shared__ __align__(16) float xs[kGsMaxH];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int total = a.k * a.I;
    const int p0 = (int)((long long)total * blockIdx.x / gridDim.x);
    const int np = (int)((long long)total * (blockIdx.x + 1) / gridDim.x) - p0;
    const int gsz = (np + kGsGroups - 1) / kGsGroups;  // pairs per barrier group
    if (threadIdx.x == 0)
        for (int g = 0; g < kGsGroups; ++g) mbar_init(&bar[g], 1);
    float4 ln[NV];
    vec_load_ldg<BLOCK, NV>(a.ln, a.H, ln);

    pdl_wait();
    pdl_launch();
    trace_.released();

    float4 v[NV];
    vec_load_cg<BLOCK, NV>(a.x, a.H, v);  // in flight while the routing is reduced
    // every CTA reduces the same shares in the same order: bitwise the same routing (CTA 0 publishes it); the
    // reduction's __syncthreads also makes the barrier initialisation visible
    const float r = route_from_shares<BLOCK>(a.rs, a.E, a.k, a.H, red, sid, sval, sw, &s_r, blockIdx.x == 0);
    if (threadIdx.x == 0) {
        const unsigned char* w = static_cast<const unsigned char*>(a.w);
        for (int g = 0; g * gsz < np; ++g) {
            const int q0 = g * gsz, q1 = min(np, q0 + gsz);
            mbar_expect_tx(&bar[g], (uint32_t)((q1 - q0) * 2 * rbh));
            for (int q = q0; q < q1; ++q) {
                const int p = p0 + q, slot = p / a.I, j = p - slot * a.I;
                // expert id clamped so that a stale id can never address outside the weights
                const int e = min(max(sid[slot], 0), a.E - 1);
                const unsigned char* base = w + (size_t)e * 2 * a.I * rbh;
                bulk_g2s(wrows + (size_t)(2 * q) * rbh, base + (size_t)j * rbh, (uint32_t)rbh, &bar[g]);
                bulk_g2s(wrows + (size_t)(2 * q + 1) * rbh, base + (size_t)(a.I + j) * rbh, (uint32_t)rbh, &bar[g]);
            }
        }
        // this CTA's share of the chosen experts' down slabs (k slabs of H rows), hinted into L2
        if (a.down_w) {
            const unsigned long long slab = (unsigned long long)a.H * a.down_row_bytes, all = slab * a.k;
            const unsigned long long share = ((all + gridDim.x - 1) / gridDim.x + 15) & ~15ull;
            unsigned long long o0 = share * blockIdx.x;
            const unsigned long long o1 = min(all, o0 + share);
            while (o0 < o1) {
                const int slot = (int)(o0 / slab);
                const unsigned long long in = o0 - (unsigned long long)slot * slab;
                const unsigned long long n = min(o1 - o0, slab - in);
                const int e = min(max(sid[slot], 0), a.E - 1);
                bulk_prefetch_l2(static_cast<const unsigned char*>(a.down_w) + (size_t)e * slab + in, (uint32_t)n);
                o0 += n;
            }
        }
    }
    // xn = ln * (h * r) (model.rs:141-145)
#pragma unroll
    for (int k = 0; k < NV; ++k) {
        const int i = threadIdx.x + k * BLOCK;
        if (4 * i < a.H) reinterpret_cast<float4*>(xs)[i] = ln_times(ln[k], v[k], r);
    }
    __syncthreads();
    float4 xa[NCH], xb[NCH];
    x_to_regs<NCH>(xs, a.H, lane, xa, xb);
    for (int q = warp; q < np; q += NW) {
        if (!mbar_wait(&bar[q / gsz], 0, a.err, 1)) return;
        const float g = warp_sum(smem_row_dot_w<NCH, Q8>(wrows + (size_t)(2 * q) * rbh, xa, xb, a.H, lane));
        const float u = warp_sum(smem_row_dot_w<NCH, Q8>(wrows + (size_t)(2 * q + 1) * rbh, xa, xb, a.H, lane));
        if (lane == 0) a.a[p0 + q] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
    }
}

// ------------------------------------------------------------------------------------------------------------------
// moe: the whole MoE block of the model step (routing, gate_up + SwiGLU, down + weighted combine + residual) as one
// persistent launch of one CTA per SM: 8 consumer warps and a producer warp.  The routing is reduced from the output
// projection's shares (bitwise the same in every CTA).  Then the producer's lane 0 streams, through a ring of shared
// memory stages (TMA bulk copies completing on `full` barriers, recycled through `empty` barriers), first this CTA's
// range of (gate row, up row) pairs of the k chosen experts, then -- as soon as stages free up -- the CTA's rows of
// the k experts' down matrices: the down weights stream while the gate_up pairs are still being computed, so HBM
// stays busy across the whole block.  Consumers compute a = silu(g) * u (cpu.rs:64-68) into global memory, meet at a
// grid barrier (every CTA is resident: one per SM), then each warp takes one routing slot j, holds a_j in registers
// and computes d_j = W_d[e_j] . a_j for the CTA's rows; the rows' y = sum_j w_j d_j is summed in routing order
// (cpu.rs:141-148) and h += resid * y (model.rs:230-232).  Every wait is bounded and reports through the error word.
// ------------------------------------------------------------------------------------------------------------------
constexpr int kMoeWarps = 8;
constexpr int kMoeThreads = 32 * (kMoeWarps + 1);
constexpr int kMoeMaxStages = 8;
constexpr int kMoeMaxRows = 32;  // down rows of one CTA (H / grid)
constexpr uint64_t kMoeBarrierNs = 2000000000ull;  // bound of the grid barrier: 2 s

LDEV void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

LDEV void consumers_sync() { asm volatile("bar.sync 1, %0;" ::"r"(32 * kMoeWarps) : "memory"); }

LDEV unsigned long long ld_acquire_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

template <int NCH, int NCI, bool Q8>
__global__ void __launch_bounds__(kMoeThreads, 1) moe_kernel(MoeArgs a) {
    const CtaTrace trace_(a.trace);
    constexpr int BLOCK = kMoeThreads, NW = kMoeWarps;
    constexpr int NV = Vec<NCH, BLOCK>::NV;
    extern __shared__ __align__(128) unsigned char ring[];  // [stages][stage_bytes]
    __shared__ __align__(8) uint64_t full[kMoeMaxStages], empty[kMoeMaxStages];
    __shared__ float red[BLOCK];
    __shared__ int sid[kMaxTopK];
    __shared__ float sval[kMaxTopK], sw[kMaxTopK], s_r;
    __shared__ __align__(16) float xs[kGsMaxH];
    __shared__ float part[kMaxTopK][kMoeMaxRows];
    __shared__ int s_ok;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int G = gridDim.x, c = blockIdx.x;
    const size_t rbh = wrow_bytes(a.H, Q8), rbi = wrow_bytes(a.I, Q8);
    const int total = a.k * a.I;
    const int p0 = (int)((long long)total * c / G), np = (int)((long long)total * (c + 1) / G) - p0;
    const int r0 = (int)((long long)a.H * c / G), nr = (int)((long long)a.H * (c + 1) / G) - r0;
    const int S = a.stages, CP = a.gu_chunk, SPC = a.slots_per_chunk;
    const int n1 = (np + CP - 1) / CP, n2 = (a.k + SPC - 1) / SPC;
    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], NW);
        }
        s_ok = 1;
    }
    float4 ln[NV];
    vec_load_ldg<BLOCK, NV>(a.ln, a.H, ln);

    pdl_wait();
    pdl_launch();
    trace_.released();

    float4 v[NV];
    vec_load_cg<BLOCK, NV>(a.h, a.H, v);  // in flight while the routing is reduced
    const float r = route_from_shares<BLOCK>(a.rs, a.E, a.k, a.H, red, sid, sval, sw, &s_r, c == 0);
    trace_.mark(0);

    // producer: one chunk of the ring; chunks [0, n1) are gate_up pairs, [n1, n1 + n2) down rows
    const unsigned char* wgu = static_cast<const unsigned char*>(a.w_gu);
    const unsigned char* wdn = static_cast<const unsigned char*>(a.w_dn);
    auto issue = [&](int i) {
        const int st = i % S;
        unsigned char* dst = ring + (size_t)st * a.stage_bytes;
        if (i < n1) {
            // pairs [q0, q1) of this CTA's range: gate rows at dst, up rows after them, in runs within one slot
            const int q0 = i * CP, q1 = min(np, q0 + CP), cnt = q1 - q0;
            mbar_expect_tx(&full[st], (uint32_t)(2 * cnt * rbh));
            for (int qa = q0; qa < q1;) {
                const int p = p0 + qa, slot = p / a.I, j = p - slot * a.I;
                const int qb = min(q1, qa + (a.I - j));  // the run stays inside one slot
                const int e = min(max(sid[slot], 0), a.E - 1);
                const unsigned char* base = wgu + (size_t)e * 2 * a.I * rbh;
                const uint32_t bytes = (uint32_t)((qb - qa) * rbh);
                bulk_g2s(dst + (size_t)(qa - q0) * rbh, base + (size_t)j * rbh, bytes, &full[st]);
                bulk_g2s(dst + (size_t)(cnt + qa - q0) * rbh, base + (size_t)(a.I + j) * rbh, bytes, &full[st]);
                qa = qb;
            }
        } else {
            // slots [j0, j1): rows [r0, r0 + nr) of each chosen expert's down matrix
            const int j0 = (i - n1) * SPC, j1 = min(a.k, j0 + SPC);
            mbar_expect_tx(&full[st], (uint32_t)((j1 - j0) * nr * rbi));
            for (int j = j0; j < j1 && nr > 0; ++j) {
                const int e = min(max(sid[j], 0), a.E - 1);
                bulk_g2s(dst + (size_t)(j - j0) * nr * rbi, wdn + ((size_t)e * a.H + r0) * rbi, (uint32_t)(nr * rbi),
                         &full[st]);
            }
        }
    };
    // the first S chunks go out at once (fresh stages, nothing to wait for)
    const int n_all = n1 + n2, first = min(S, n_all);
    if (warp == NW && lane == 0)
        for (int i = 0; i < first; ++i) issue(i);
    // xn = ln * (h * r) (model.rs:141-145), every thread its share
#pragma unroll
    for (int k = 0; k < NV; ++k) {
        const int i = threadIdx.x + k * BLOCK;
        if (4 * i < a.H) reinterpret_cast<float4*>(xs)[i] = ln_times(ln[k], v[k], r);
    }
    __syncthreads();
    if (warp == NW) {
        // the rest of the chunks, each into a stage the consumers have released
        if (lane != 0) return;
        for (int i = first; i < n_all; ++i) {
            if (!mbar_wait(&empty[i % S], (uint32_t)((i / S - 1) & 1), a.err, 21)) return;
            issue(i);
        }
        // the next layer's dense weights into L2 while this block computes (qkv_rope then reads them from L2)
        prefetch_share_l2(a.pf[0], a.pf_bytes[0], c, G);
        prefetch_share_l2(a.pf[1], a.pf_bytes[1], c, G);
        return;
    }

    // ---- consumers ---------------------------------------------------------------------------------------------
    bool ok = true;
    {
        float4 xa[NCH], xb[NCH];
        x_to_regs<NCH>(xs, a.H, lane, xa, xb);
        for (int i = 0; i < n1 && ok; ++i) {
            const int st = i % S;
            ok = mbar_wait(&full[st], (uint32_t)((i / S) & 1), a.err, 22);
            if (!ok) break;
            const unsigned char* src = ring + (size_t)st * a.stage_bytes;
            const int q0 = i * CP, cnt = min(np, q0 + CP) - q0;
            for (int q = warp; q < cnt; q += NW) {
                const float g = warp_sum(smem_row_dot_w<NCH, Q8>(src + (size_t)q * rbh, xa, xb, a.H, lane));
                const float u = warp_sum(smem_row_dot_w<NCH, Q8>(src + (size_t)(cnt + q) * rbh, xa, xb, a.H, lane));
                if (lane == 0) a.a[p0 + q0 + q] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[st]);
        }
    }
    trace_.mark(1);
    if (!ok) atomicExch(&s_ok, 0);
    // grid barrier: every CTA's activations written before any CTA reads them
    __threadfence();
    consumers_sync();
    if (threadIdx.x == 0 && s_ok) {
        const unsigned long long old = atomicAdd(a.barrier, 1ull);
        const unsigned long long target = (old / (unsigned long long)G + 1ull) * (unsigned long long)G;
        const uint64_t t0 = global_ns();
        while (ld_acquire_u64(a.barrier) < target) {
            if (*reinterpret_cast<volatile int*>(a.err) || global_ns() - t0 > kMoeBarrierNs) {
                atomicCAS(a.err, 0, 23);
                s_ok = 0;
                break;
            }
            __nanosleep(32);
        }
    }
    consumers_sync();
    trace_.mark(2);
    if (!s_ok) return;
    // down: warp w takes slot j = w: a_j in registers, its rows from the ring
    for (int j = warp; j < a.k; j += NW) {
        const int i = n1 + j / SPC, st = i % S;
        if (!mbar_wait(&full[st], (uint32_t)((i / S) & 1), a.err, 24)) {
            atomicExch(&s_ok, 0);
            break;
        }
        float4 xa[NCI], xb[NCI];
        x_to_regs_global<NCI>(a.a + (size_t)j * a.I, a.I, lane, xa, xb);
        const unsigned char* src = ring + (size_t)st * a.stage_bytes + (size_t)(j - (j / SPC) * SPC) * nr * rbi;
        for (int rr = 0; rr < nr; ++rr) {
            const float d = warp_sum(smem_row_dot_w<NCI, Q8>(src + (size_t)rr * rbi, xa, xb, a.I, lane));
            if (lane == 0) part[j][rr] = d;
        }
    }
    consumers_sync();
    trace_.mark(3);
    if (!s_ok || threadIdx.x >= nr) return;
    float acc = 0.0f;
#pragma unroll
    for (int j = 0; j < kMaxTopK; ++j)
        if (j < a.k) acc = __fadd_rn(acc, __fmul_rn(sw[j], part[j][threadIdx.x]));
    float* hp = a.h + r0 + threadIdx.x;
    *hp = __fadd_rn(__ldcg(hp), __fmul_rn(a.resid, acc));
}

// ------------------------------------------------------------------------------------------------------------------
// down: CTA per block of kDnRows output rows; warp j takes expert slot j for all rows of the block, so a_j is read
// once into registers.  Expert ids and weights come from the router, two kernels back, so before
// griddepcontrol.wait thread 0 already streams the k contiguous [kDnRows, I] slabs W_d[e_j][r0 .. r0+R] into
// shared memory.  Per row the k expert dots are then summed in routing order, y = sum_j w_j * d_j (cpu.rs:141-148),
// and h[r] += resid * y (model.rs:230-232) or out[r] = y (block forward).
// ------------------------------------------------------------------------------------------------------------------
constexpr int kDnRows = 8;
constexpr int kRouteWaitPolls = 1024;  // ~100 us at most; then the CTA reduces the shares itself

template <int NCI, bool Q8>
__global__ void __launch_bounds__(256) down_kernel(DownArgs a) {
    const CtaTrace trace_(a.trace);
    constexpr int BLOCK = 256, R = kDnRows;
    extern __shared__ __align__(128) unsigned char smem_raw[];
    const size_t rbi = wrow_bytes(a.I, Q8);                              // bytes per weight row
    unsigned char* wd = smem_raw;                                        // [k, R] rows of I weights
    float* part = reinterpret_cast<float*>(wd + (size_t)a.k * R * rbi);  // [k, R]
    __shared__ __align__(8) uint64_t bar;
    __shared__ float red[BLOCK];
    __shared__ int sid[kMaxTopK];
    __shared__ float sval[kMaxTopK], sw[kMaxTopK], s_r;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int r0 = blockIdx.x * R;
    const bool fused = a.rs.shares != nullptr;
    // the routing: gate_up's CTA 0 publishes it while this kernel's CTAs start (take it once its flag carries this
    // step's counter), or reduce the output projection's shares here, like gate_up (two kernels back: final already)
    __shared__ bool s_have;
    bool have = false;
    if (fused && a.route_flag) {
        if (threadIdx.x == 0) {
            const unsigned int want = __ldcg(a.step_ctr);
            bool got = false;
            for (int i = 0; i < kRouteWaitPolls && !got; ++i) {
                got = ld_acquire_gpu(a.route_flag) == want;
                if (!got) __nanosleep(64);
            }
            s_have = got;
        }
        __syncthreads();
        have = s_have;
        if (have && threadIdx.x < a.k) {
            sid[threadIdx.x] = __ldcg(a.rs.ids_out + threadIdx.x);
            sw[threadIdx.x] = __ldcg(a.rs.weights_out + threadIdx.x);
        }
    }
    if (fused && !have) route_from_shares<BLOCK>(a.rs, a.E, a.k, a.H, red, sid, sval, sw, &s_r, false);
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        const uint32_t bytes = (uint32_t)(R * rbi);
        mbar_expect_tx(&bar, bytes * a.k);
        for (int j = 0; j < a.k; ++j) {
            const int e = min(max(fused ? sid[j] : __ldcg(a.ids + j), 0), a.E - 1);
            bulk_g2s(wd + (size_t)j * R * rbi, static_cast<const unsigned char*>(a.w) + ((size_t)e * a.H + r0) * rbi, bytes,
                     &bar);
        }
        // the next layer's dense weights into L2 while this layer's MoE runs (qkv_rope then reads them from L2)
        prefetch_share_l2(a.pf[0], a.pf_bytes[0], blockIdx.x, gridDim.x);
        prefetch_share_l2(a.pf[1], a.pf_bytes[1], blockIdx.x, gridDim.x);
    }
    __syncthreads();  // the barrier is initialized before any thread waits on it
    float gw[kMaxTopK];
#pragma unroll
    for (int j = 0; j < kMaxTopK; ++j) gw[j] = j < a.k ? (fused ? sw[j] : __ldcg(a.weights + j)) : 0.0f;
    pdl_wait();
    pdl_launch();
    trace_.released();
    const float hr = (threadIdx.x < R && a.accumulate) ? __ldcg(a.out + r0 + threadIdx.x) : 0.0f;
    float4 xa[NCI], xb[NCI];
    if (warp < a.k) x_to_regs_global<NCI>(a.a + (size_t)warp * a.I, a.I, lane, xa, xb);
    const bool ok = mbar_wait(&bar, 0, a.err, 2);
    trace_.mark(0);
    if (ok && warp < a.k) {
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const float d = warp_sum(smem_row_dot_w<NCI, Q8>(wd + ((size_t)warp * R + r) * rbi, xa, xb, a.I, lane));
            if (lane == 0) part[warp * R + r] = d;
        }
    }
    __syncthreads();
    if (!ok || threadIdx.x >= R) return;
    float acc = 0.0f;
#pragma unroll
    for (int j = 0; j < kMaxTopK; ++j)
        if (j < a.k) acc = __fadd_rn(acc, __fmul_rn(gw[j], part[j * R + threadIdx.x]));
    a.out[r0 + threadIdx.x] = a.accumulate ? __fadd_rn(hr, __fmul_rn(a.resid, acc)) : acc;
}

// ------------------------------------------------------------------------------------------------------------------
// head: final RMSNorm, logits = (E . xn) / logits_scaling over the tied embedding, argmax keeping the last maximum
// (Iterator::max_by with total_cmp).  A fixed grid of CTAs walks the vocabulary two rows per warp at a time with the
// next pair's weights already in flight; the last CTA publishes the token, appends it to the history and advances
// the position.
// ------------------------------------------------------------------------------------------------------------------
constexpr int kHeadWarps = 8;
constexpr int kHeadCtas = 148 * 2;  // 128 registers x 256 threads: two CTAs per SM


template <int NCH>
LDEV void head_rows(const uint4 (&w)[2][NCH], int row, const HeadArgs& a, const float* xs, int lane,
                    unsigned long long& best) {
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const float d = warp_sum(row_dot<NCH>(w[r], xs, a.H, lane));
        if (row + r < a.V) {
            const float lg = __fdiv_rn(d, a.logits_scaling);
            if (lane == 0 && a.logits_out) a.logits_out[row + r] = lg;
            const unsigned long long k = arg_key(lg, row + r);
            best = k > best ? k : best;
        }
    }
}

template <int NCH>
LDEV void head_load(uint4 (&w)[2][NCH], int row, const HeadArgs& a, int lane) {
#pragma unroll
    for (int r = 0; r < 2; ++r) load_row<NCH>(w[r], a.w + (size_t)(row + r) * a.H, a.H, lane, row + r < a.V);
}

template <int NCH>
__global__ void __launch_bounds__(256) head_kernel(HeadArgs a) {
    const CtaTrace trace_(a.trace);
    constexpr int BLOCK = 32 * kHeadWarps;
    constexpr int NV = Vec<NCH, BLOCK>::NV;
    extern __shared__ __align__(16) float smem[];
    float* xs = smem;
    float* red = smem + a.H;
    __shared__ unsigned long long wbest[kHeadWarps];
    __shared__ bool is_last;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int stride = gridDim.x * kHeadWarps * 2;
    int row = (blockIdx.x * kHeadWarps + warp) * 2;
    uint4 wa[2][NCH], wb[2][NCH];
    head_load<NCH>(wa, row, a, lane);
    float4 ln[NV];
    vec_load_ldg<BLOCK, NV>(a.ln, a.H, ln);
    pdl_wait();
    pdl_launch();
    trace_.released();
    {
        float4 v[NV];
        vec_load_cg<BLOCK, NV>(a.h, a.H, v);
        norm_regs<BLOCK, NV>(v, ln, a.H, a.eps, xs, red);
    }
    unsigned long long best = 0ull;
    // two row pairs per iteration: the loads of one pair are in flight while the other is reduced
    for (; row < a.V; row += 2 * stride) {
        head_load<NCH>(wb, row + stride, a, lane);
        head_rows<NCH>(wa, row, a, xs, lane, best);
        if (row + stride >= a.V) break;
        head_load<NCH>(wa, row + 2 * stride, a, lane);
        head_rows<NCH>(wb, row + stride, a, xs, lane, best);
    }
    if (lane == 0) wbest[warp] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long b = 0ull;
        for (int i = 0; i < kHeadWarps; ++i) b = wbest[i] > b ? wbest[i] : b;
        a.partial[blockIdx.x] = b;
    }
    if (!last_block_arrives(a.counter, gridDim.x, &is_last)) return;
    unsigned long long b = 0ull;
    for (int i = threadIdx.x; i < (int)gridDim.x; i += blockDim.x) {
        const unsigned long long t = __ldcg(a.partial + i);
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
        for (int i = 0; i < kHeadWarps; ++i) mx = wbest[i] > mx ? wbest[i] : mx;
        const int tok = (int)(uint32_t)mx;
        *a.token_out = tok;
        if (a.out_ids) {
            const int st = __ldcg(a.step);
            if (st >= 0 && st < a.out_cap) a.out_ids[st] = tok;
            *a.step = st + 1;
        }
        *a.pos = __ldcg(a.pos) + 1;
    }
}

// ------------------------------------------------------------------------------------------------------------------
// synthetic fill
// ------------------------------------------------------------------------------------------------------------------
LDEV uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

LDEV float synth_value(uint64_t seed, uint64_t idx, float scale) {
    const uint64_t h = mix64(seed + (idx + 1ull) * 0x9E3779B97F4A7C15ull);
    const int s = (int)(h & 0xffffu) + (int)((h >> 16) & 0xffffu) + (int)((h >> 32) & 0xffffu) + (int)(h >> 48);
    return __fmul_rn((float)(s - 131070), scale);
}

__global__ void synth_bf16_kernel(uint16_t* out, size_t n, uint64_t seed, float scale, float mean) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        float v = synth_value(seed, i, scale);
        if (mean != 0.0f) v = __fadd_rn(v, mean);
        out[i] = f32_to_bf16_rne(v);
    }
}

__global__ void synth_f32_kernel(float* out, size_t n, uint64_t seed, float scale) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        out[i] = synth_value(seed, i, scale);
}

// Synthetic K/V context in the paged layout [page][kv_head][slot][d]: logical element i = pos * kvd + head * d + j of
// positions [0, n) gets the generator's value i (the CPU oracle's lo_session_fill_kv, element for element), rounded to
// bf16 when the pool is bf16.
template <bool F32>
__global__ void synth_kv_pages_kernel(void* pool, const int* page_table, int n, int kv_heads, int d, int page_size,
                                      uint64_t seed, float scale) {
    const size_t kvd = (size_t)kv_heads * d, total = (size_t)n * kvd;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int p = (int)(i / kvd);
        const int r = (int)(i - (size_t)p * kvd), h = r / d, j = r - h * d;
        const size_t dst = (((size_t)__ldg(page_table + p / page_size) * kv_heads + h) * page_size + p % page_size) * d + j;
        const float v = synth_value(seed, i, scale);
        if (F32)
            static_cast<float*>(pool)[dst] = v;
        else
            static_cast<uint16_t*>(pool)[dst] = f32_to_bf16_rne(v);
    }
}

__global__ void synth_norm_kernel(float* out, size_t n, uint64_t seed, float scale) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const float v = __fadd_rn(synth_value(seed, i, scale), 1.0f);
        out[i] = __uint_as_float((uint32_t)f32_to_bf16_rne(v) << 16);
    }
}

// Q8_0 synthetic fill (the CPU oracle's lo_synth_q8_0, same integer hash): value of element idx of the row-major
// matrix uniform in [-127, 127]; block b's fp16 scale = 1e-4 + u * 3.9e-3 with u from 24 hash bits, rounded to nearest
// even by the same integer routine as the oracle's lo_f32_to_f16
LDEV uint16_t f32_to_f16_rne(float f) {
    const uint32_t u = __float_as_uint(f);
    const uint32_t sign = (u >> 16) & 0x8000u, a = u & 0x7fffffffu;
    if (a >= 0x47800000u) return (uint16_t)(sign | 0x7c00u);
    if (a < 0x38800000u) {
        if (a < 0x33000000u) return (uint16_t)sign;
        const uint32_t m = (a & 0x7fffffu) | 0x800000u;
        const int sh = 126 - (int)(a >> 23);
        uint32_t q = m >> sh;
        const uint32_t rem = m & ((1u << sh) - 1u), half = 1u << (sh - 1);
        if (rem > half || (rem == half && (q & 1u))) ++q;
        return (uint16_t)(sign | q);
    }
    const uint32_t r = a - 0x38000000u;
    uint32_t q = r >> 13;
    const uint32_t rem = r & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) ++q;
    return (uint16_t)(sign | q);
}

__global__ void synth_q8_values_kernel(unsigned char* out, size_t rows, int cols, uint64_t seed) {
    const size_t n = rows * (size_t)cols, rb = wrow_bytes(cols, 1);
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const size_t r = i / cols, c = i - r * cols;
        const int v = (int)(mix64(seed + (i + 1ull) * 0x9E3779B97F4A7C15ull) % 255ull) - 127;
        out[r * rb + c] = (unsigned char)(signed char)v;
    }
}

__global__ void synth_q8_scales_kernel(unsigned char* out, size_t rows, int cols, uint64_t seed) {
    const size_t nb = (size_t)cols / 32, n = rows * nb, rb = wrow_bytes(cols, 1);
    for (size_t b = blockIdx.x * (size_t)blockDim.x + threadIdx.x; b < n; b += (size_t)gridDim.x * blockDim.x) {
        const uint64_t h = mix64((seed ^ 0xA5A5A5A5A5A5A5A5ull) + (b + 1ull) * 0x9E3779B97F4A7C15ull);
        const float u = __fmul_rn((float)(h >> 40), 1.0f / 16777216.0f);
        const size_t r = b / nb, j = b - r * nb;
        reinterpret_cast<uint16_t*>(out + r * rb + cols)[j] = f32_to_f16_rne(__fadd_rn(1e-4f, __fmul_rn(u, 3.9e-3f)));
    }
}

int chunks_for(int n) { return (n + 255) / 256; }

}  // namespace

// ---------------------------------------------------------------------------------------------------------------------
// launchers
// ---------------------------------------------------------------------------------------------------------------------
// Dynamic shared memory beyond the default must be opted into; the default leaves 48 KB minus the kernel's static
// shared memory, so any sizeable request sets the attribute.
template <typename Kern>
cudaError_t allow_smem(Kern k, size_t bytes) {
    if (bytes <= 16 * 1024) return cudaSuccess;
    return cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

#define LASTRO_NCH_SWITCH(nch, KERNEL_EXPR)                     \
    switch (nch) {                                              \
    case 1: { constexpr int N = 1; return KERNEL_EXPR; }        \
    case 2: { constexpr int N = 2; return KERNEL_EXPR; }        \
    case 3: { constexpr int N = 3; return KERNEL_EXPR; }        \
    case 4: { constexpr int N = 4; return KERNEL_EXPR; }        \
    case 5: { constexpr int N = 5; return KERNEL_EXPR; }        \
    case 6: { constexpr int N = 6; return KERNEL_EXPR; }        \
    case 7: { constexpr int N = 7; return KERNEL_EXPR; }        \
    case 8: { constexpr int N = 8; return KERNEL_EXPR; }        \
    default: return cudaErrorInvalidValue;                      \
    }

cudaError_t launch_qkv_rope(const QkvArgs& a, cudaStream_t s, bool pdl) {
    const int npairs = (a.qd + 2 * a.kvd) / 2;
    const dim3 grid((npairs + 3) / 4), block(128);
    const size_t smem = sizeof(float) * (a.H + 32);
    if (a.q8) {
        if (a.kv_f32) {
            LASTRO_NCH_SWITCH(chunks_for(a.H), launch_ex(qkv_rope_kernel<N, true, true>, grid, block, smem, s, pdl, a));
        }
        LASTRO_NCH_SWITCH(chunks_for(a.H), launch_ex(qkv_rope_kernel<N, false, true>, grid, block, smem, s, pdl, a));
    }
    if (a.spec_out) {
        if (a.kv_f32) {
            LASTRO_NCH_SWITCH(chunks_for(a.H), launch_ex(qkv_rope_kernel<N, true, false, true>, grid, block, smem, s, pdl, a));
        }
        LASTRO_NCH_SWITCH(chunks_for(a.H), launch_ex(qkv_rope_kernel<N, false, false, true>, grid, block, smem, s, pdl, a));
    }
    if (a.kv_f32) {
        LASTRO_NCH_SWITCH(chunks_for(a.H), launch_ex(qkv_rope_kernel<N, true, false>, grid, block, smem, s, pdl, a));
    }
    LASTRO_NCH_SWITCH(chunks_for(a.H), launch_ex(qkv_rope_kernel<N, false, false>, grid, block, smem, s, pdl, a));
}

int attn_split_cap(int max_len, int splits) { return (max_len + splits - 1) / splits + 1; }

// shared memory of the staged K/V rows: contiguous rows from p0, or (tma) whole 8-row boxes, 1024-byte aligned
static size_t attn_smem_staging(int max_len, int kv_f32, int splits, bool tma) {
    const int cap = attn_split_cap(max_len, splits);
    if (kv_f32 || !tma) return (size_t)2 * cap * kHeadDim * (kv_f32 ? 4 : 2);
    return (size_t)2 * attn_tma_rows(cap) * kHeadDim * 2 + 1024;
}

size_t attn_smem(int max_len, int kv_f32, int splits) {
    return std::max(attn_smem_staging(max_len, kv_f32, splits, false), attn_smem_staging(max_len, kv_f32, splits, true));
}

// context splits of the batch-1 attention: 8 while a split's rows fit about one pass of the CTA's 8 warps (256
// positions each at max_len 2048) and its staging fits shared memory, else 16
int attn_splits_default(int max_len, int kv_f32) {
    return (max_len <= 8 * 32 * kAttnWarps + 512 && attn_smem(max_len, kv_f32, 8) <= kMaxSmemBytes) ? 8 : kAttnSplits;
}

cudaError_t launch_attention(const AttnArgs& a, cudaStream_t s, bool pdl, const CUtensorMap* kmap, const CUtensorMap* vmap) {
    if (a.d != kHeadDim || a.splits < 1 || a.splits > kAttnSplits || a.split_cap != attn_split_cap(a.max_len, a.splits))
        return cudaErrorInvalidValue;
    if (a.tma && (a.kv_f32 || !kmap || !vmap || a.page_size % 8)) return cudaErrorInvalidValue;
    static const CUtensorMap none{};  // unused by launches that stage with plain bulk copies
    const CUtensorMap& km = a.tma ? *kmap : none;
    const CUtensorMap& vm = a.tma ? *vmap : none;
    if (a.cluster && a.seq) return cudaErrorInvalidValue;  // batch-1 only (16 splits: a non-portable cluster size)
    if (a.mma && a.kv_f32) return cudaErrorInvalidValue;
    if (a.cluster && (a.tma || a.mma)) return cudaErrorInvalidValue;  // the cluster merge runs the default form only
    const size_t smem = attn_smem_staging(a.max_len, a.kv_f32, a.splits, a.tma != 0);
    if (smem > kMaxSmemBytes) return cudaErrorInvalidValue;
    const dim3 grid(a.splits, a.kv_heads, a.seq ? a.tokens : 1), block(32 * kAttnWarps);
    if (a.spec_ids && (a.tma || a.mma || a.kv_f32 || a.seq)) return cudaErrorInvalidValue;  // bf16, batch 1, bulk form
    const int mode = a.spec_ids ? 4 : (a.tma ? 1 : 0) | (a.mma ? 2 : 0);
#define LASTRO_ATTN_G(GV)                                                                                  \
    case GV: {                                                                                             \
        if (a.cluster) {                                                                                   \
            auto k = a.kv_f32 ? attention_kernel<true, GV, true> : attention_kernel<false, GV, true>;      \
            cudaError_t e = allow_smem(k, smem);                                                           \
            if (e == cudaSuccess && a.splits > 8)                                                          \
                e = cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);            \
            return e != cudaSuccess ? e : launch_cluster_ex(k, grid, block, smem, s, pdl, a.splits, km, vm, a); \
        }                                                                                                  \
        auto k = a.kv_f32 ? attention_kernel<true, GV, false>                                              \
                 : mode == 1 ? attention_kernel<false, GV, false, 1>                                       \
                 : mode == 2 ? attention_kernel<false, GV, false, 2>                                       \
                 : mode == 3 ? attention_kernel<false, GV, false, 3>                                       \
                 : mode == 4 ? attention_kernel<false, GV, false, 4>                                       \
                             : attention_kernel<false, GV, false, 0>;                                      \
        cudaError_t e = allow_smem(k, smem);                                                               \
        return e != cudaSuccess ? e : launch_ex(k, grid, block, smem, s, pdl, km, vm, a);                  \
    }
    switch (a.G) {
        LASTRO_ATTN_G(1)
        LASTRO_ATTN_G(2)
        LASTRO_ATTN_G(3)
        LASTRO_ATTN_G(4)
        LASTRO_ATTN_G(6)
        LASTRO_ATTN_G(8)
    default: return cudaErrorInvalidValue;
    }
#undef LASTRO_ATTN_G
}

int oproj_grid(int H) { return (H + kOpRows - 1) / kOpRows; }

cudaError_t launch_oproj_smem(const OprojArgs& a, cudaStream_t s, bool pdl) {
    const dim3 grid(oproj_grid(a.H)), block(256);
    if (a.route && a.E > kMaxExperts) return cudaErrorInvalidValue;
    const size_t smem = (size_t)kOpRows * wrow_bytes(a.qd, a.q8) +
                        sizeof(float) * (a.qd + (a.route ? (size_t)kOpRows * a.E : 0));
    if (smem > kMaxSmemBytes || a.part_acc) return cudaErrorInvalidValue;
#define LASTRO_OPS(N)                                                                 \
    {                                                                                 \
        auto k = a.q8 ? oproj_smem_kernel<N, true> : oproj_smem_kernel<N, false>;     \
        cudaError_t e = allow_smem(k, smem);                                          \
        return e != cudaSuccess ? e : launch_ex(k, grid, block, smem, s, pdl, a);     \
    }
    switch (chunks_for(a.qd)) {
    case 1: LASTRO_OPS(1)
    case 2: LASTRO_OPS(2)
    case 3: LASTRO_OPS(3)
    case 4: LASTRO_OPS(4)
    case 5: LASTRO_OPS(5)
    case 6: LASTRO_OPS(6)
    case 7: LASTRO_OPS(7)
    case 8: LASTRO_OPS(8)
    default: return cudaErrorInvalidValue;
    }
#undef LASTRO_OPS
}

cudaError_t launch_oproj(const OprojArgs& a, cudaStream_t s, bool pdl) {
    if (a.smem_weights) return launch_oproj_smem(a, s, pdl);
    const dim3 grid(oproj_grid(a.H)), block(32 * kOpWarps);
    if (a.route && a.E > kMaxExperts) return cudaErrorInvalidValue;
    if (a.part_acc && (a.heads * kHeadDim != a.qd || a.splits < 1)) return cudaErrorInvalidValue;
    const size_t merge = a.part_acc ? (size_t)a.heads * a.splits * (kHeadDim + 3) + a.heads : 0;
    const size_t smem = sizeof(float) * (a.qd + (a.route ? (size_t)kOpRows * a.E : 0) + merge);
    if (smem > kMaxSmemBytes) return cudaErrorInvalidValue;
#define LASTRO_OP(N)                                                                  \
    {                                                                                 \
        auto k = a.q8 ? oproj_kernel<N, true> : a.spec ? oproj_kernel<N, false, true> : oproj_kernel<N, false>; \
        cudaError_t e = allow_smem(k, smem);                                          \
        return e != cudaSuccess ? e : launch_ex(k, grid, block, smem, s, pdl, a);     \
    }
    switch (chunks_for(a.qd)) {
    case 1: LASTRO_OP(1)
    case 2: LASTRO_OP(2)
    case 3: LASTRO_OP(3)
    case 4: LASTRO_OP(4)
    case 5: LASTRO_OP(5)
    case 6: LASTRO_OP(6)
    case 7: LASTRO_OP(7)
    case 8: LASTRO_OP(8)
    default: return cudaErrorInvalidValue;
    }
#undef LASTRO_OP
}

cudaError_t launch_router_fold(const void* wr, int q8, const float* ln, float* wr_t, int E, int H, cudaStream_t s) {
    const int n = E * H;
    if (q8)
        router_fold_kernel<true><<<(n + 255) / 256, 256, 0, s>>>(wr, ln, wr_t, E, H);
    else
        router_fold_kernel<false><<<(n + 255) / 256, 256, 0, s>>>(wr, ln, wr_t, E, H);
    return cudaGetLastError();
}

cudaError_t launch_router(const RouterArgs& a, cudaStream_t s, bool pdl) {
    const dim3 grid((a.E + 3) / 4), block(128);
    const size_t smem = sizeof(float) * (a.H + 32);
    LASTRO_NCH_SWITCH(chunks_for(a.H),
                      launch_ex(a.q8 ? router_kernel<N, true> : router_kernel<N, false>, grid, block, smem, s, pdl, a));
}

size_t gate_up_smem(int H, int q8) { return (size_t)2 * kGuPairs * wrow_bytes(H, q8) + (size_t)H * 4; }
size_t down_smem(int H, int I, int k, int q8) {
    (void)H;
    return (size_t)k * kDnRows * wrow_bytes(I, q8) + (size_t)k * kDnRows * 4;
}
int gate_up_rows_per_cta() { return kGuPairs; }
int down_rows_per_cta() { return kDnRows; }

// SMs of the current device (the streaming kernels launch about one CTA per SM)
int sm_count() {
    static int cached[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (!cached[dev]) {
        int n = 0;
        cached[dev] = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && n > 0 ? n : 148;
    }
    return cached[dev];
}

cudaError_t launch_gate_up_stream(const GateUpArgs& a, cudaStream_t s, bool pdl) {
    if (a.H > kGsMaxH || a.H % 8) return cudaErrorInvalidValue;
    const size_t pair_bytes = 2 * wrow_bytes(a.H, a.q8);
    const size_t budget = kMaxSmemBytes - 12 * 1024;  // the kernel's static shared memory stays below 12 KB
    const int total = a.k * a.I;
    const int cap = (int)(budget / pair_bytes);  // pairs one CTA can stage
    if (cap < 1) return cudaErrorInvalidValue;
    int grid = sm_count();
    if ((total + grid - 1) / grid > cap) grid = (total + cap - 1) / cap;
    if (grid > total) grid = total;
    const size_t smem = (size_t)((total + grid - 1) / grid) * pair_bytes;
#define LASTRO_GS(N)                                                                                   \
    {                                                                                                  \
        auto k = a.q8 ? gate_up_stream_kernel<N, true> : gate_up_stream_kernel<N, false>;             \
        cudaError_t e = allow_smem(k, smem);                                                           \
        return e != cudaSuccess ? e : launch_ex(k, dim3(grid), dim3(kGsThreads), smem, s, pdl, a);     \
    }
    switch (chunks_for(a.H)) {
    case 1: LASTRO_GS(1)
    case 2: LASTRO_GS(2)
    case 3: LASTRO_GS(3)
    case 4: LASTRO_GS(4)
    case 5: LASTRO_GS(5)
    case 6: LASTRO_GS(6)
    case 7: LASTRO_GS(7)
    case 8: LASTRO_GS(8)
    default: return cudaErrorInvalidValue;
    }
#undef LASTRO_GS
}

cudaError_t launch_gate_up(const GateUpArgs& a, cudaStream_t s, bool pdl) {
    if (a.rs.shares && a.stream) return launch_gate_up_stream(a, s, pdl);
    if (a.I % kGuPairs) return cudaErrorInvalidValue;
    const dim3 grid(a.k * (a.I / kGuPairs)), block(256);
    const size_t smem = gate_up_smem(a.H, a.q8);
    if (smem > kMaxSmemBytes) return cudaErrorInvalidValue;
#define LASTRO_GU(N)                                                                  \
    {                                                                                 \
        auto k = a.q8 ? gate_up_kernel<N, true> : a.spec ? gate_up_kernel<N, false, true> : gate_up_kernel<N, false>; \
        cudaError_t e = allow_smem(k, smem);                                          \
        return e != cudaSuccess ? e : launch_ex(k, grid, block, smem, s, pdl, a);     \
    }
    switch (chunks_for(a.H)) {
    case 1: LASTRO_GU(1)
    case 2: LASTRO_GU(2)
    case 3: LASTRO_GU(3)
    case 4: LASTRO_GU(4)
    case 5: LASTRO_GU(5)
    case 6: LASTRO_GU(6)
    case 7: LASTRO_GU(7)
    case 8: LASTRO_GU(8)
    default: return cudaErrorInvalidValue;
    }
#undef LASTRO_GU
}

bool moe_plan(int H, int I, int k, int q8, MoePlan* out) {
    if (H > kGsMaxH || H % 8 || I % 8 || k < 1 || k > kMaxTopK || chunks_for(H) > 8 || chunks_for(I) > 2) return false;
    const int total = k * I;
    int grid = sm_count();
    grid = std::min(grid, std::min(total, H));
    const size_t rbh = wrow_bytes(H, q8), rbi = wrow_bytes(I, q8);
    const int nr_max = (H + grid - 1) / grid;
    if (nr_max > kMoeMaxRows) return false;
    int cp = 8;  // pairs per gate_up chunk: one per consumer warp
    while (cp > 1 && (size_t)cp * 2 * rbh > 64 * 1024) --cp;
    size_t stage = std::max((size_t)cp * 2 * rbh, (size_t)nr_max * rbi);
    stage = (stage + 127) & ~(size_t)127;
    const size_t budget = kMaxSmemBytes - 16 * 1024;  // the kernel's static shared memory stays below 16 KB
    const int stages = (int)std::min<size_t>(kMoeMaxStages, budget / stage);
    const int spc = (int)std::min<size_t>((size_t)k, stage / ((size_t)nr_max * rbi));
    const int n2 = (k + spc - 1) / spc;
    if (stages < 2 || spc < 1 || n2 > stages) return false;  // every down chunk must reuse a gate_up chunk's stage
    out->grid = grid;
    out->stages = stages;
    out->stage_bytes = (int)stage;
    out->gu_chunk = cp;
    out->slots_per_chunk = spc;
    out->smem = (size_t)stages * stage;
    return true;
}

cudaError_t launch_moe(const MoeArgs& a, const MoePlan& p, cudaStream_t s, bool pdl) {
    if (a.stages != p.stages || a.stage_bytes != p.stage_bytes || !a.barrier) return cudaErrorInvalidValue;
#define LASTRO_MOE(N, NI)                                                                                    \
    {                                                                                                        \
        auto k = a.q8 ? moe_kernel<N, NI, true> : moe_kernel<N, NI, false>;                                  \
        cudaError_t e = allow_smem(k, p.smem);                                                               \
        return e != cudaSuccess ? e : launch_ex(k, dim3(p.grid), dim3(kMoeThreads), p.smem, s, pdl, a);      \
    }
#define LASTRO_MOE_I(N)                                                                                      \
    if (chunks_for(a.I) == 1) LASTRO_MOE(N, 1) else LASTRO_MOE(N, 2)
    switch (chunks_for(a.H)) {
    case 1: LASTRO_MOE_I(1)
    case 2: LASTRO_MOE_I(2)
    case 3: LASTRO_MOE_I(3)
    case 4: LASTRO_MOE_I(4)
    case 5: LASTRO_MOE_I(5)
    case 6: LASTRO_MOE_I(6)
    case 7: LASTRO_MOE_I(7)
    case 8: LASTRO_MOE_I(8)
    default: return cudaErrorInvalidValue;
    }
#undef LASTRO_MOE_I
#undef LASTRO_MOE
}

cudaError_t launch_down(const DownArgs& a, cudaStream_t s, bool pdl) {
    if (a.H % kDnRows) return cudaErrorInvalidValue;
    const dim3 grid(a.H / kDnRows), block(256);
    const size_t smem = down_smem(a.H, a.I, a.k, a.q8);
    if (smem > kMaxSmemBytes) return cudaErrorInvalidValue;
#define LASTRO_DN(N)                                                                  \
    {                                                                                 \
        auto k = a.q8 ? down_kernel<N, true> : down_kernel<N, false>;                 \
        cudaError_t e = allow_smem(k, smem);                                          \
        return e != cudaSuccess ? e : launch_ex(k, grid, block, smem, s, pdl, a);     \
    }
    switch (chunks_for(a.I)) {
    case 1: LASTRO_DN(1)
    case 2: LASTRO_DN(2)
    case 3: LASTRO_DN(3)
    case 4: LASTRO_DN(4)
    case 5: LASTRO_DN(5)
    case 6: LASTRO_DN(6)
    case 7: LASTRO_DN(7)
    case 8: LASTRO_DN(8)
    default: return cudaErrorInvalidValue;
    }
#undef LASTRO_DN
}

int head_grid(int V) {
    const int pairs = (V + 1) / 2;
    const int ctas = (pairs + kHeadWarps - 1) / kHeadWarps;
    return ctas < kHeadCtas ? ctas : kHeadCtas;
}

cudaError_t launch_head(const HeadArgs& a, cudaStream_t s, bool pdl, int* grid_out) {
    const dim3 grid(head_grid(a.V)), block(32 * kHeadWarps);
    if (grid_out) *grid_out = (int)grid.x;
    const size_t smem = sizeof(float) * (a.H + 32);
    LASTRO_NCH_SWITCH(chunks_for(a.H), launch_ex(head_kernel<N>, grid, block, smem, s, pdl, a));
}

cudaError_t launch_synth_q8_0(unsigned char* out, size_t rows, int cols, uint64_t seed, cudaStream_t s) {
    if (rows == 0 || cols % 32) return cols % 32 ? cudaErrorInvalidValue : cudaSuccess;
    synth_q8_values_kernel<<<148 * 16, 256, 0, s>>>(out, rows, cols, seed);
    synth_q8_scales_kernel<<<148 * 4, 256, 0, s>>>(out, rows, cols, seed);
    return cudaGetLastError();
}

cudaError_t launch_synth_bf16(uint16_t* out, size_t n, uint64_t seed, float scale, float mean, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    size_t blocks = (n + 255) / 256;
    if (blocks > 148 * 64) blocks = 148 * 64;
    synth_bf16_kernel<<<(unsigned)blocks, 256, 0, s>>>(out, n, seed, scale, mean);
    return cudaGetLastError();
}

cudaError_t launch_synth_f32(float* out, size_t n, uint64_t seed, float scale, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    size_t blocks = (n + 255) / 256;
    if (blocks > 148 * 64) blocks = 148 * 64;
    synth_f32_kernel<<<(unsigned)blocks, 256, 0, s>>>(out, n, seed, scale);
    return cudaGetLastError();
}

cudaError_t launch_synth_kv_pages(void* pool, int kv_f32, const int* page_table, int n, int kv_heads, int d,
                                  int page_size, uint64_t seed, float scale, cudaStream_t s) {
    if (n <= 0) return cudaSuccess;
    const size_t total = (size_t)n * kv_heads * d;
    size_t blocks = (total + 255) / 256;
    if (blocks > 148 * 64) blocks = 148 * 64;
    if (kv_f32)
        synth_kv_pages_kernel<true><<<(unsigned)blocks, 256, 0, s>>>(pool, page_table, n, kv_heads, d, page_size, seed, scale);
    else
        synth_kv_pages_kernel<false><<<(unsigned)blocks, 256, 0, s>>>(pool, page_table, n, kv_heads, d, page_size, seed, scale);
    return cudaGetLastError();
}

cudaError_t launch_synth_norm_f32(float* out, size_t n, uint64_t seed, float scale, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    size_t blocks = (n + 255) / 256;
    if (blocks > 148 * 64) blocks = 148 * 64;
    synth_norm_kernel<<<(unsigned)blocks, 256, 0, s>>>(out, n, seed, scale);
    return cudaGetLastError();
}

}  // namespace lastro
