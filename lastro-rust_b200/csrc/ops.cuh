// Device helpers shared by the decode kernels (kernels.cu) and the fused decode step (fused_step.cu):
// vectors of H floats, bf16 row dots with x in registers or shared memory, the router's top-k and the routing
// reduced from the output projection's shares.
#pragma once

#include <cuda_fp16.h>

#include "common.cuh"
#include "kernels.h"

namespace lastro {
namespace {

// ---- vectors of H floats, NV float4 per thread (H <= 4 * NV * BLOCK, H a multiple of 4) ---------------------------

template <int BLOCK, int NV>
LDEV void vec_load_cg(const float* p, int n, float4 (&r)[NV]) {
#pragma unroll
    for (int k = 0; k < NV; ++k) {
        const int i = threadIdx.x + k * BLOCK;
        r[k] = (4 * i < n) ? __ldcg(reinterpret_cast<const float4*>(p) + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
}

template <int BLOCK, int NV>
LDEV void vec_load_ldg(const float* p, int n, float4 (&r)[NV]) {
#pragma unroll
    for (int k = 0; k < NV; ++k) {
        const int i = threadIdx.x + k * BLOCK;
        r[k] = (4 * i < n) ? __ldg(reinterpret_cast<const float4*>(p) + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
}

LDEV float4 ln_times(float4 ln, float4 v, float r) {
    // model.rs:144: g * (v * r)
    return make_float4(__fmul_rn(ln.x, __fmul_rn(v.x, r)), __fmul_rn(ln.y, __fmul_rn(v.y, r)),
                       __fmul_rn(ln.z, __fmul_rn(v.z, r)), __fmul_rn(ln.w, __fmul_rn(v.w, r)));
}

// xs = ln * (v * r), r = 1/sqrt(mean(v^2) + eps) (model.rs:141-145; the sum of squares is a parallel reduction
// here).  v and ln are already in registers.  Returns r.
template <int BLOCK, int NV>
LDEV float norm_regs(const float4 (&v)[NV], const float4 (&ln)[NV], int H, float eps, float* xs, float* red) {
    float ss = 0.0f;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
        ss = fmaf(v[k].x, v[k].x, ss);
        ss = fmaf(v[k].y, v[k].y, ss);
        ss = fmaf(v[k].z, v[k].z, ss);
        ss = fmaf(v[k].w, v[k].w, ss);
    }
    const float tot = block_sum(ss, red);
    const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)H), eps)));
#pragma unroll
    for (int k = 0; k < NV; ++k) {
        const int i = threadIdx.x + k * BLOCK;
        if (4 * i < H) reinterpret_cast<float4*>(xs)[i] = ln_times(ln[k], v[k], r);
    }
    __syncthreads();
    return r;
}

// n floats (n a multiple of 4) to shared memory, eight independent 16-byte loads in flight per thread
template <int BLOCK>
LDEV void copy_to_smem(const float* src, int n, float* dst) {
    const float4* s4 = reinterpret_cast<const float4*>(src);
    float4* d4 = reinterpret_cast<float4*>(dst);
    const int n4 = n >> 2;
    for (int base = 0; base < n4; base += 8 * BLOCK) {
        float4 t[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int i = base + threadIdx.x + k * BLOCK;
            if (i < n4) t[k] = __ldcg(s4 + i);
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int i = base + threadIdx.x + k * BLOCK;
            if (i < n4) d4[i] = t[k];
        }
    }
    __syncthreads();
}

// dot of a bf16 row held as NCH 16-byte chunks per lane (chunk c covers columns (c*32+lane)*8 .. +8) with xs.
template <int NCH>
LDEV float row_dot(const uint4 (&w)[NCH], const float* xs, int H, int lane) {
    float acc = 0.0f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
        const int col = (c * 32 + lane) * 8;
        if (col < H) {
            const float4 xa = *reinterpret_cast<const float4*>(xs + col);
            const float4 xb = *reinterpret_cast<const float4*>(xs + col + 4);
            acc = dot8(w[c], xa, xb, acc);
        }
    }
    return acc;
}

template <int NCH>
LDEV void load_row(uint4 (&w)[NCH], const uint16_t* row, int H, int lane, bool active) {
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
        const int col = (c * 32 + lane) * 8;
        if (active && col < H)
            w[c] = ld_weight(row + col);
        else
            w[c] = make_uint4(0u, 0u, 0u, 0u);
    }
}

// dot of a bf16 row held in registers (NCH 16-byte chunks per lane) with x held in registers
template <int NCH>
LDEV float row_dot_regs(const uint4 (&w)[NCH], const float4 (&xa)[NCH], const float4 (&xb)[NCH], int H, int lane) {
    float acc = 0.0f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
        const int col = (c * 32 + lane) * 8;
        if (col < H) acc = dot8(w[c], xa[c], xb[c], acc);
    }
    return acc;
}

// ---- Q8_0 rows (device layout: cols int8 values, then cols/32 fp16 scales) -------------------------------------------
// A lane's chunk c covers the same 8 columns as a bf16 chunk, (c*32 + lane)*8 .. +8: 8 int8 values (8 bytes) and the
// scale of their block of 32.  dot: the 8 products summed, then scaled (one multiply per 8 weights).
struct Q8Chunk {
    uint2 q;
    float s;
};

LDEV float f16_to_f32(uint16_t h) { return __half2float(__ushort_as_half(h)); }

LDEV uint2 ld_weight8(const void* p) {
    uint2 r;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
    return r;
}

LDEV float dot8_q8(uint2 q, float s, float4 xa, float4 xb, float acc) {
    float p = 0.0f;
    p = fmaf((float)((int)(q.x << 24) >> 24), xa.x, p);
    p = fmaf((float)((int)(q.x << 16) >> 24), xa.y, p);
    p = fmaf((float)((int)(q.x << 8) >> 24), xa.z, p);
    p = fmaf((float)((int)q.x >> 24), xa.w, p);
    p = fmaf((float)((int)(q.y << 24) >> 24), xb.x, p);
    p = fmaf((float)((int)(q.y << 16) >> 24), xb.y, p);
    p = fmaf((float)((int)(q.y << 8) >> 24), xb.z, p);
    p = fmaf((float)((int)q.y >> 24), xb.w, p);
    return fmaf(s, p, acc);
}

template <int NCH>
LDEV void load_row_q8(Q8Chunk (&w)[NCH], const unsigned char* row, int H, int lane, bool active) {
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
        const int col = (c * 32 + lane) * 8;
        if (active && col < H) {
            w[c].q = ld_weight8(row + col);
            w[c].s = f16_to_f32(__ldg(reinterpret_cast<const unsigned short*>(row + H) + (col >> 5)));
        } else {
            w[c].q = make_uint2(0u, 0u);
            w[c].s = 0.0f;
        }
    }
}

template <int NCH>
LDEV float row_dot_regs_q8(const Q8Chunk (&w)[NCH], const float4 (&xa)[NCH], const float4 (&xb)[NCH], int H, int lane) {
    float acc = 0.0f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
        const int col = (c * 32 + lane) * 8;
        if (col < H) acc = dot8_q8(w[c].q, w[c].s, xa[c], xb[c], acc);
    }
    return acc;
}

template <int NCH>
LDEV float row_dot_q8(const Q8Chunk (&w)[NCH], const float* xs, int H, int lane) {
    float acc = 0.0f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
        const int col = (c * 32 + lane) * 8;
        if (col < H) {
            const float4 xa = *reinterpret_cast<const float4*>(xs + col);
            const float4 xb = *reinterpret_cast<const float4*>(xs + col + 4);
            acc = dot8_q8(w[c].q, w[c].s, xa, xb, acc);
        }
    }
    return acc;
}

// bf16 or Q8_0 row staged in shared memory, x in registers
template <int NCH, bool Q8>
LDEV float smem_row_dot_w(const unsigned char* row, const float4 (&xa)[NCH], const float4 (&xb)[NCH], int H, int lane) {
    float acc = 0.0f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
        const int col = (c * 32 + lane) * 8;
        if (col < H) {
            if (Q8) {
                const uint2 q = *reinterpret_cast<const uint2*>(row + col);
                const float sc = f16_to_f32(reinterpret_cast<const unsigned short*>(row + H)[col >> 5]);
                acc = dot8_q8(q, sc, xa[c], xb[c], acc);
            } else {
                acc = dot8(*reinterpret_cast<const uint4*>(row + 2 * col), xa[c], xb[c], acc);
            }
        }
    }
    return acc;
}

// A weight row held in registers (lane chunks as above), bf16 or Q8_0: load from its first byte, dot with x in shared
// memory or in registers.
template <int NCH, bool Q8>
struct WRow;

template <int NCH>
struct WRow<NCH, false> {
    uint4 w[NCH];
    LDEV void load(const unsigned char* row, int H, int lane, bool active) {
        load_row<NCH>(w, reinterpret_cast<const uint16_t*>(row), H, lane, active);
    }
    LDEV float dot(const float* xs, int H, int lane) const { return row_dot<NCH>(w, xs, H, lane); }
    LDEV float dot_regs(const float4 (&xa)[NCH], const float4 (&xb)[NCH], int H, int lane) const {
        return row_dot_regs<NCH>(w, xa, xb, H, lane);
    }
};

template <int NCH>
struct WRow<NCH, true> {
    Q8Chunk w[NCH];
    LDEV void load(const unsigned char* row, int H, int lane, bool active) { load_row_q8<NCH>(w, row, H, lane, active); }
    LDEV float dot(const float* xs, int H, int lane) const { return row_dot_q8<NCH>(w, xs, H, lane); }
    LDEV float dot_regs(const float4 (&xa)[NCH], const float4 (&xb)[NCH], int H, int lane) const {
        return row_dot_regs_q8<NCH>(w, xa, xb, H, lane);
    }
};

// float4 per thread for a vector of NCH*256 floats over BLOCK threads
template <int NCH, int BLOCK>
struct Vec {
    static constexpr int NV = (NCH * 64 + BLOCK - 1) / BLOCK;
};

// ------------------------------------------------------------------------------------------------------------------
// x held in registers: lane l owns columns (c*32 + l)*8 .. +8 of every row it multiplies, so a warp that computes
// several rows reads x once (shared memory bandwidth is the limit otherwise: a bf16 weight read from shared memory
// next to its f32 activation is 3x the weight bytes).
// ------------------------------------------------------------------------------------------------------------------
template <int NCH>
LDEV void x_to_regs(const float* xs, int H, int lane, float4 (&xa)[NCH], float4 (&xb)[NCH]) {
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
        const int col = (c * 32 + lane) * 8;
        if (col < H) {
            xa[c] = *reinterpret_cast<const float4*>(xs + col);
            xb[c] = *reinterpret_cast<const float4*>(xs + col + 4);
        } else {
            xa[c] = make_float4(0.f, 0.f, 0.f, 0.f);
            xb[c] = xa[c];
        }
    }
}

template <int NCH>
LDEV void x_to_regs_global(const float* x, int H, int lane, float4 (&xa)[NCH], float4 (&xb)[NCH]) {
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
        const int col = (c * 32 + lane) * 8;
        if (col < H) {
            xa[c] = __ldcg(reinterpret_cast<const float4*>(x + col));
            xb[c] = __ldcg(reinterpret_cast<const float4*>(x + col + 4));
        } else {
            xa[c] = make_float4(0.f, 0.f, 0.f, 0.f);
            xb[c] = xa[c];
        }
    }
}

// dot of a bf16 row in shared memory with x in registers
template <int NCH>
LDEV float smem_row_dot(const uint16_t* row, const float4 (&xa)[NCH], const float4 (&xb)[NCH], int H, int lane) {
    float acc = 0.0f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
        const int col = (c * 32 + lane) * 8;
        if (col < H) acc = dot8(*reinterpret_cast<const uint4*>(row + col), xa[c], xb[c], acc);
    }
    return acc;
}


// ------------------------------------------------------------------------------------------------------------------
// router: logits = W_r . xn (one warp per expert), then the last CTA takes the top-k with block.rs:81-89's order
// (total_cmp descending, lower index first on ties) and the softmax over the k.
// ------------------------------------------------------------------------------------------------------------------
LDEV unsigned long long route_key(float v, int idx) {
    // larger is better: value by total order, then lower index
    return ((unsigned long long)((uint32_t)total_key(v) ^ 0x80000000u) << 32) | (uint32_t)(~(uint32_t)idx);
}

LDEV unsigned long long shfl_u64(unsigned long long v, int src) {
    uint32_t lo = (uint32_t)v, hi = (uint32_t)(v >> 32);
    lo = __shfl_sync(0xffffffffu, lo, src);
    hi = __shfl_sync(0xffffffffu, hi, src);
    return ((unsigned long long)hi << 32) | lo;
}

LDEV unsigned long long shfl_xor_u64(unsigned long long v, int o) {
    uint32_t lo = (uint32_t)v, hi = (uint32_t)(v >> 32);
    lo = __shfl_xor_sync(0xffffffffu, lo, o);
    hi = __shfl_xor_sync(0xffffffffu, hi, o);
    return ((unsigned long long)hi << 32) | lo;
}

// Warp-wide top-k of E <= 64 logits (lane holds experts lane and lane + 32) in block.rs:81-89's order -- total_cmp
// descending, lower index first on ties -- then the softmax over the k (exp(v - v0), summed in order, divided).
// Every expert's rank is counted against all E keys at once (independent shuffles, no select-max chain); the k
// winners land at their rank in sid/sval, the softmax weights in sw (shared, kMaxTopK entries each).
LDEV void route_topk_warp(float v0, float v1, int E, int k, int* sid, float* sval, float* sw) {
    const int lane = threadIdx.x & 31;
    const unsigned long long k0 = lane < E ? route_key(v0, lane) : 0ull;
    const unsigned long long k1 = lane + 32 < E ? route_key(v1, lane + 32) : 0ull;
    int r0 = 0, r1 = 0;  // keys are distinct (the index is part of the key), so ranks are a permutation
#pragma unroll 8
    for (int src = 0; src < 32; ++src) {
        const unsigned long long a = shfl_u64(k0, src), b = shfl_u64(k1, src);
        r0 += (int)(a > k0) + (int)(b > k0);
        r1 += (int)(a > k1) + (int)(b > k1);
    }
    if (lane < E && r0 < k) {
        sid[r0] = lane;
        sval[r0] = v0;
    }
    if (lane + 32 < E && r1 < k) {
        sid[r1] = lane + 32;
        sval[r1] = v1;
    }
    __syncwarp();
    const float ex = lane < k ? expf(__fsub_rn(sval[lane], sval[0])) : 0.0f;
    float sum = 0.0f;
    for (int j = 0; j < k; ++j) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, ex, j));
    if (lane < k) sw[lane] = __fdiv_rn(ex, sum);
    __syncwarp();
}

// route_topk_warp's top-k computed by the whole block (every thread calls it; blockDim >= E; lg in shared memory):
// each expert's rank by counting the larger keys, then the softmax over the k by threads j < k.  Bitwise the same ids,
// values and weights as route_topk_warp: the same keys and comparisons, the same exponentials, the sum in the same
// order.  __syncthreads inside.
LDEV void route_topk_block(const float* lg, int E, int k, unsigned long long* keys, float* ex, int* sid, float* sval,
                           float* sw) {
    const int t = threadIdx.x;
    if (t < E) keys[t] = route_key(lg[t], t);
    __syncthreads();
    if (t < E) {
        const unsigned long long me = keys[t];
        int r = 0;
        for (int j = 0; j < E; ++j) r += (int)(keys[j] > me);
        if (r < k) {
            sid[r] = t;
            sval[r] = lg[t];
        }
    }
    __syncthreads();
    if (t < k) ex[t] = expf(__fsub_rn(sval[t], sval[0]));
    __syncthreads();
    if (t < k) {
        float sum = 0.0f;
        for (int j = 0; j < k; ++j) sum = __fadd_rn(sum, ex[j]);
        sw[t] = __fdiv_rn(ex[t], sum);
    }
    __syncthreads();
}

// Routing from the output projection's shares (RouteShares): the shares of CTA c go to thread (c % groups) * E1 + e,
// each thread loads its shares in batches of independent loads and sums them in order, the groups are summed in
// order, then r = 1/sqrt(sum h^2 / H + eps) (model.rs:141-145), logits = r * share-sums, the top-k by rank counting in
// block.rs:81-89's order and the softmax over the k.  Every CTA that calls this computes bitwise the same routing.
// Uses __syncthreads (every thread of the block calls it; blockDim >= E + 1); results in sid/sw (shared), returns r.
// (Spreading the steps after the share loads over the whole block, one step per barrier, measured slower on C3 than
// this single warp: gate_up gained 0.3 us, the down kernel lost 0.6 us, 1.034 vs 1.027 ms per step.)
template <int BLOCK>
LDEV float route_from_shares(const RouteShares& rs, int E, int k, int H, float* red, int* sid, float* sval, float* sw,
                             float* s_r, bool publish, const CtaTrace* tr = nullptr) {
    constexpr int kBatch = 8;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    // groups of share loads: fixed by a 256-thread block whatever BLOCK is, so every kernel that reduces the shares
    // (256 or 288 threads) sums them in the same order and gets bitwise the same routing
    const int E1 = E + 1, groups = (BLOCK < 256 ? BLOCK : 256) / E1;
    float acc = 0.0f;
    if (threadIdx.x < groups * E1) {
        const int e = threadIdx.x % E1, gi = threadIdx.x / E1;
        for (int c0 = gi; c0 < rs.nb; c0 += groups * kBatch) {
            float sh[kBatch];
#pragma unroll
            for (int q = 0; q < kBatch; ++q) {
                const int c = c0 + q * groups;
                sh[q] = c < rs.nb ? __ldcg(rs.shares + (size_t)c * E1 + e) : 0.0f;
            }
#pragma unroll
            for (int q = 0; q < kBatch; ++q)
                if (c0 + q * groups < rs.nb) acc = __fadd_rn(acc, sh[q]);
        }
    }
    red[threadIdx.x] = acc;
    __syncthreads();
    if (tr) tr->mark(3);
    if (warp == 0) {
        float v[2];
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            const int e = lane + 32 * q;
            float t = 0.0f;
            if (e < E1)
                for (int gi = 0; gi < groups; ++gi) t = __fadd_rn(t, red[gi * E1 + e]);
            v[q] = t;
        }
        const float ss = __shfl_sync(0xffffffffu, v[E >> 5], E & 31);  // entry E is the sum of squares
        const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)H), rs.eps)));
        const float l0 = lane < E ? __fmul_rn(v[0], r) : 0.0f;
        const float l1 = lane + 32 < E ? __fmul_rn(v[1], r) : 0.0f;
        if (tr) tr->mark(4);
        route_topk_warp(l0, l1, E, k, sid, sval, sw);
        if (lane == 0) *s_r = r;
        if (publish) {
            if (lane < E) rs.logits_out[lane] = l0;
            if (lane + 32 < E) rs.logits_out[lane + 32] = l1;
            if (lane < k) {
                rs.ids_out[lane] = sid[lane];
                rs.weights_out[lane] = sw[lane];
            }
        }
    }
    __syncthreads();
    return *s_r;
}


LDEV unsigned long long arg_key(float v, int idx) {
    // larger is better: value by total order, then the larger index (last maximum)
    return ((unsigned long long)((uint32_t)total_key(v) ^ 0x80000000u) << 32) | (uint32_t)idx;
}

}  // namespace
}  // namespace lastro
