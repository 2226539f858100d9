// Batched decode step kernels (see batch.h for the step's order and the exchange region).
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include "batch.h"
#include "common.cuh"
#include "kernels.h"
#include "ops.cuh"

namespace lastro {

namespace {

// ---- tensor-core GEMM helpers ----------------------------------------------------------------------------------
// 16-byte global -> shared copy; `valid` false fills the 16 bytes with zeros (nothing is read)
LDEV void cp_async16(uint32_t dst, const void* src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0) : "memory");
}
LDEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
LDEV void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// ---- bounded waits on flags written by other GPUs (global_ns: common.cuh) -----------------------------------------
LDEV unsigned int ld_acquire_sys(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
LDEV void st_release_sys(unsigned int* p, unsigned int v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
LDEV unsigned int ld_acquire_gpu(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
LDEV void st_release_gpu(unsigned int* p, unsigned int v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// the exchange's flags: system scope when the group spans GPUs, GPU scope for a group of one
LDEV unsigned int ld_acquire_x(const unsigned int* p, bool sys) { return sys ? ld_acquire_sys(p) : ld_acquire_gpu(p); }
LDEV void st_release_x(unsigned int* p, unsigned int v, bool sys) {
    if (sys)
        st_release_sys(p, v);
    else
        st_release_gpu(p, v);
}
// Waits until *flag reaches `want` (epochs only grow), at most `limit_ns`; on time-out records `code` in the error word
// and fails.  A wait that finds the error word already set (an earlier wait of this step gave up) fails at once, so a
// dead peer costs one limit per step, not one per layer.
LDEV bool wait_flag(const unsigned int* flag, unsigned int want, int* err, int code, bool sys, uint64_t limit_ns) {
    const uint64_t t0 = global_ns();
    for (uint32_t i = 0; (int)(ld_acquire_x(flag, sys) - want) < 0; ++i) {
        if ((i & 63) == 0 && *reinterpret_cast<volatile int*>(err)) return false;
        if (global_ns() - t0 > limit_ns) {
            atomicCAS(err, 0, code);
            return false;
        }
        __nanosleep(64);
    }
    return true;
}

// Last-CTA election across a grid whose CTAs wrote to other GPUs.  Each CTA orders its writes before its arrival with
// a GPU-scope fence; the last CTA, which has observed every arrival, then issues one system-scope fence before it
// publishes the flag with a system-scope release store: every CTA's peer writes precede the flag in causality order,
// without a system-scope fence in each of the grid's CTAs.  A group of one GPU (sys false) stays at GPU scope.
LDEV bool last_block_arrives_sys(unsigned int* counter, unsigned int total, bool* flag_smem, bool sys) {
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned int t = atomicAdd(counter, 1u);
        const bool last = (t == total - 1);
        if (last) atomicExch(counter, 0u);
        *flag_smem = last;
    }
    __syncthreads();
    const bool last = *flag_smem;
    if (last && sys) __threadfence_system();
    return last;
}

LDEV unsigned int* flag_ptr(unsigned char* region, const XLayout& L, int kind, int who) {
    return reinterpret_cast<unsigned int*>(region + L.flags + ((size_t)kind * 64 + who) * 128);
}

// weight group (expert) of a launch's group g
LDEV int weight_group(const BGemmArgs& a, int g) { return a.group_expert ? __ldg(a.group_expert + g) : a.group0 + g; }

}  // namespace

XLayout x_layout(int world, int tokens_per_rank, int k, int H) {
    auto up = [](size_t v) { return (v + 255) & ~(size_t)255; };
    XLayout L{};
    L.cap = tokens_per_rank * k;
    L.cap_tok = tokens_per_rank;
    size_t o = 0;
    L.rx = o;
    o = up(o + (size_t)world * L.cap_tok * H * 4);
    L.rx_ids = o;
    o = up(o + (size_t)world * L.cap * 4);
    L.rx_n = o;
    o = up(o + (size_t)world * 4);
    L.cb = o;
    o = up(o + (size_t)L.cap * H * 4);
    L.flags = o;
    o = up(o + (size_t)2 * 64 * 128);
    L.bytes = o;
    return L;
}

// ------------------------------------------------------------------------------------------------------------------
// GEMM: y[pos][row] = sum_k W[row][k] * x[pos][k] for the weight rows of one CTA (128, or 64 gate + 64 up rows) and
// all tokens of its group, tiles of 64 tokens at a time.  4 warps; warp w owns rows {16w..16w+15} of each 64-row half
// (m-tiles mt = 0, 1), so a SwiGLU thread holds gate and up of the same (row, token).  K streams through a 3-stage
// cp.async pipeline in chunks of 64; per 16-wide K step a warp loads its A fragments (ldmatrix.x4) once and issues
// 2 m-tiles x 8 token n-tiles x {hi, lo} mma.sync.
// ------------------------------------------------------------------------------------------------------------------
template <int EPI>
__global__ void __launch_bounds__(128) bgemm_kernel(BGemmArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = blockIdx.y, bx = blockIdx.x;
    pdl_wait();
    pdl_launch();
    __shared__ bool is_last;
    int p0 = 0, ntot = a.n;
    if (a.g_cnt) {
        p0 = __ldcg(a.g_off + g);
        ntot = __ldcg(a.g_cnt + g);
    }
    const uint16_t* W = a.w + (size_t)weight_group(a, g) * a.group_stride;
    const int kbeg = blockIdx.z * a.k_split;
    const int nk = min(a.k_split, a.K - kbeg) / kBK;
    if (nk <= 0) ntot = 0;
    if (EPI != BEPI_RETURN && ntot <= 0) return;  // (a RETURN CTA still votes below)
    const int ch = tid & 7;
    // this thread's 8 weight rows in the tile (fixed for the CTA)
    auto grow_of = [&](int sr) -> int {
        if (EPI == BEPI_SWIGLU) return sr < 64 ? bx * 64 + sr : a.I + bx * 64 + (sr - 64);
        return bx * kBRows + sr;
    };

    for (int t0 = 0; t0 < ntot; t0 += kBTok) {
        const int n = min(kBTok, ntot - t0);
        int xrow[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int tok = (tid >> 3) + 16 * i;
            const int p = p0 + t0 + tok;
            xrow[i] = tok < n ? (a.x_rows ? __ldcg(a.x_rows + p) : p) : 0;
        }
        auto load_stage = [&](int slot, int kt) {
            unsigned char* st = smem + (size_t)slot * kBStageBytes;
            const int k0 = kbeg + kt * kBK + ch * 8;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int sr = (tid >> 3) + 16 * i;
                const int gr = grow_of(sr);
                const bool v = gr < a.rows;
                cp_async16(smem_addr(st) + swz(sr, ch), W + (size_t)(v ? gr : 0) * a.K + k0, v);
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int tok = (tid >> 3) + 16 * i;
                const bool v = tok < n;
                const size_t xo = (size_t)xrow[i] * a.ldx + k0;
                const uint32_t d = swz(tok, ch);
                cp_async16(smem_addr(st + kBRows * 128) + d, a.x_hi + xo, v);
                cp_async16(smem_addr(st + kBRows * 128 + kBTok * 128) + d, a.x_lo + xo, v);
            }
        };

        float acc[2][8][4];
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
            for (int j = 0; j < 8; ++j)
#pragma unroll
                for (int c = 0; c < 4; ++c) acc[mt][j][c] = 0.0f;
        const int ntp = (n + 15) >> 4;  // active pairs of 8-token n-tiles

        if (t0 > 0) __syncthreads();  // the previous tile's last stage reads are done
#pragma unroll
        for (int s = 0; s < kBStages - 1; ++s) {
            if (s < nk) load_stage(s, s);
            cp_async_commit();
        }
        for (int kt = 0; kt < nk; ++kt) {
            cp_async_wait<kBStages - 2>();
            __syncthreads();
            const int pf = kt + kBStages - 1;
            if (pf < nk) load_stage(pf % kBStages, pf);
            cp_async_commit();
            const uint32_t sW = smem_addr(smem + (size_t)(kt % kBStages) * kBStageBytes);
            const uint32_t sXh = sW + kBRows * 128, sXl = sXh + kBTok * 128;
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk) {
                const int mi = lane >> 3, r8 = lane & 7;
                uint32_t af[2][4];
#pragma unroll
                for (int mt = 0; mt < 2; ++mt) {
                    const int sr = mt * 64 + warp * 16 + (mi & 1) * 8 + r8;
                    ldsm_x4(sW + swz(sr, kk * 2 + (mi >> 1)), af[mt]);
                }
#pragma unroll
                for (int jp = 0; jp < 4; ++jp) {
                    if (jp < ntp) {
                        const int tok = (2 * jp + (mi >> 1)) * 8 + r8;
                        const uint32_t off = swz(tok, kk * 2 + (mi & 1));
                        uint32_t bh[4], bl[4];
                        ldsm_x4(sXh + off, bh);
                        ldsm_x4(sXl + off, bl);
                        // the four hi products first, then the four lo products: an accumulator's two updates are
                        // three independent MMAs apart
#pragma unroll
                        for (int mt = 0; mt < 2; ++mt) {
                            mma_bf16(acc[mt][2 * jp], af[mt], bh[0], bh[1]);
                            mma_bf16(acc[mt][2 * jp + 1], af[mt], bh[2], bh[3]);
                        }
#pragma unroll
                        for (int mt = 0; mt < 2; ++mt) {
                            mma_bf16(acc[mt][2 * jp], af[mt], bl[0], bl[1]);
                            mma_bf16(acc[mt][2 * jp + 1], af[mt], bl[2], bl[3]);
                        }
                    }
                }
            }
        }
        cp_async_wait<0>();

        if (EPI == BEPI_RETURN) {
            // the tile through shared memory ([token][128 rows] f32), then one 512-byte row block per token to the
            // combine rows of the pair's sender
            __syncthreads();
            float* stile = reinterpret_cast<float*>(smem);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                if (j * 8 >= n) break;
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const int tok = j * 8 + (lane & 3) * 2 + (c & 1);
                    const int rr = warp * 16 + (lane >> 2) + ((c >> 1) << 3);
                    if (tok < n) {
                        stile[tok * kBRows + rr] = acc[0][j][c];
                        stile[tok * kBRows + 64 + rr] = acc[1][j][c];
                    }
                }
            }
            __syncthreads();
            const XLayout& L = a.x.lay;
            for (int tok = warp; tok < n; tok += 4) {
                const int i = __ldcg(a.x.src + p0 + t0 + tok);
                const int sender = i / L.cap, pair = i - sender * L.cap;
                float4* dst = reinterpret_cast<float4*>(a.x.peers[sender] + L.cb +
                                                        ((size_t)pair * a.rows + (size_t)bx * kBRows) * 4);
                dst[lane] = reinterpret_cast<const float4*>(stile + tok * kBRows)[lane];
            }
            __syncthreads();
            continue;
        }

        // epilogue: acc[mt][j][c] is (tile row mt*64 + 16 warp + lane/4 + 8 (c >= 2), token 8 j + 2 (lane % 4) + c % 2)
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            if (j * 8 >= n) break;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int tok = j * 8 + (lane & 3) * 2 + (c & 1);
                if (tok >= n) continue;
                const int rr = warp * 16 + (lane >> 2) + ((c >> 1) << 3);  // row within a 64-row half
                const size_t p = (size_t)(p0 + t0 + tok);
                if (EPI == BEPI_SWIGLU) {
                    const float gv = acc[0][j][c], uv = acc[1][j][c];
                    const float v = __fmul_rn(__fdiv_rn(gv, __fadd_rn(1.0f, expf(-gv))), uv);
                    uint16_t hi, lo;
                    split_bf16(v, hi, lo);
                    const size_t o = p * a.I + bx * 64 + rr;
                    a.a_hi[o] = hi;
                    a.a_lo[o] = lo;
                } else {
#pragma unroll
                    for (int mt = 0; mt < 2; ++mt) {
                        const int gr = bx * kBRows + mt * 64 + rr;
                        if (gr < a.rows)
                            a.y[blockIdx.z * a.z_stride + p * a.ldy + gr] = a.div == 1.0f ? acc[mt][j][c]
                                                                                            : __fdiv_rn(acc[mt][j][c], a.div);
                    }
                }
            }
        }
    }
    if (EPI == BEPI_RETURN) {
        if (!last_block_arrives_sys(a.x.counter, gridDim.x * gridDim.y * gridDim.z, &is_last, a.x.world > 1)) return;
        if (tid < a.x.world) {
            const unsigned int epoch = __ldcg(a.x.epoch_base) + a.x.layer + 1;
            st_release_x(flag_ptr(a.x.peers[tid], a.x.lay, 1, a.x.rank), epoch, a.x.world > 1);
        }
    }
}

// ------------------------------------------------------------------------------------------------------------------
// attention norm: h = embedding row x multiplier (layer 0) or the residual stream; xn = ln * (h * r) split hi + lo
// ------------------------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) battn_norm_kernel(BNormArgs a) {
    const CtaTrace trace_(a.trace);
    constexpr int BLOCK = 256, NV = 2;  // H <= 2048
    __shared__ float red[BLOCK / 32];
    const int t = blockIdx.x;
    float* h = a.h + (size_t)t * a.H;
    pdl_wait();
    pdl_launch();
    trace_.released();
    float4 v[NV];
#pragma unroll
    for (int k = 0; k < NV; ++k) {
        const int i = threadIdx.x + k * BLOCK;
        v[k] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (4 * i >= a.H) continue;
        if (a.embed) {
            const int tok = __ldg(a.tokens + t);
            const uint2 u = __ldg(reinterpret_cast<const uint2*>(a.embed + (size_t)tok * a.H) + i);
            v[k] = make_float4(__fmul_rn(bf_lo(u.x), a.emb_mult), __fmul_rn(bf_hi(u.x), a.emb_mult),
                               __fmul_rn(bf_lo(u.y), a.emb_mult), __fmul_rn(bf_hi(u.y), a.emb_mult));
            reinterpret_cast<float4*>(h)[i] = v[k];
        } else {
            v[k] = __ldcg(reinterpret_cast<const float4*>(h) + i);
        }
    }
    float ss = 0.0f;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
        ss = fmaf(v[k].x, v[k].x, ss);
        ss = fmaf(v[k].y, v[k].y, ss);
        ss = fmaf(v[k].z, v[k].z, ss);
        ss = fmaf(v[k].w, v[k].w, ss);
    }
    const float tot = block_sum(ss, red);
    const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)a.H), a.eps)));
#pragma unroll
    for (int k = 0; k < NV; ++k) {
        const int i = threadIdx.x + k * BLOCK;
        if (4 * i >= a.H) continue;
        const float4 ln = __ldg(reinterpret_cast<const float4*>(a.ln) + i);
        const float4 x = ln_times(ln, v[k], r);
        ushort4 hi, lo;
        split_bf16(x.x, hi.x, lo.x);
        split_bf16(x.y, hi.y, lo.y);
        split_bf16(x.z, hi.z, lo.z);
        split_bf16(x.w, hi.w, lo.w);
        reinterpret_cast<ushort4*>(a.x_hi + (size_t)t * a.H)[i] = hi;
        reinterpret_cast<ushort4*>(a.x_lo + (size_t)t * a.H)[i] = lo;
    }
}

// ------------------------------------------------------------------------------------------------------------------
// RoPE + KV append: the q/k/v partial slices summed in slice order, then per RoPE pair (j, j + d/2) of each head
// x1*c - x2*s, x2*c + x1*s (model.rs:153-155); q to its buffer, K (roped) and V to the token's sequence page.
// ------------------------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(128) brope_kv_kernel(BRopeArgs a) {
    const CtaTrace trace_(a.trace);
    constexpr int kMaxKs = 16;
    const int t = blockIdx.x;
    const int R = a.qd + 2 * a.kvd, half = a.d >> 1;
    const int pi = blockIdx.y * blockDim.x + threadIdx.x;  // RoPE pair of this thread
    pdl_wait();
    pdl_launch();
    trace_.released();
    if (pi >= R / 2) return;
    const int sq = __ldg(a.seq + t);
    const int pos = __ldcg(a.pos + sq) + (a.off ? __ldg(a.off + t) : 0);
    const float* cs = a.rope_cs + (size_t)pos * a.d;
    const int head = pi / half, j = pi - head * half;
    const int r0 = head * a.d + j, r1 = r0 + half;
    // every slice's two values in flight at once, then summed in slice order
    float v1[kMaxKs], v2[kMaxKs];
#pragma unroll
    for (int z = 0; z < kMaxKs; ++z) {
        if (z < a.ks) {
            const float* pz = a.part + ((size_t)z * a.n + t) * R;
            v1[z] = __ldcg(pz + r0);
            v2[z] = __ldcg(pz + r1);
        }
    }
    float x1 = 0.0f, x2 = 0.0f;
#pragma unroll
    for (int z = 0; z < kMaxKs; ++z) {
        if (z < a.ks) {
            x1 = __fadd_rn(x1, v1[z]);
            x2 = __fadd_rn(x2, v2[z]);
        }
    }
    const float c = __ldg(cs + j), s = __ldg(cs + half + j);
    const float ro0 = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
    const float ro1 = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
    if (r0 < a.qd) {
        a.q[(size_t)t * a.qd + r0] = ro0;
        a.q[(size_t)t * a.qd + r1] = ro1;
        return;
    }
    const int page = __ldg(a.page_table + (size_t)sq * a.pt_stride + pos / a.page_size), slot = pos % a.page_size;
    int rr = r0 - a.qd;
    const bool is_k = rr < a.kvd;
    if (!is_k) rr -= a.kvd;
    const int kvh = rr / a.d;
    const float w0 = is_k ? ro0 : x1, w1 = is_k ? ro1 : x2;
    const size_t base = (((size_t)page * a.kv_heads + kvh) * a.page_size + slot) * a.d;
    void* pool = is_k ? a.k_pool : a.v_pool;
    if (a.kv_f32) {
        float* p = static_cast<float*>(pool) + base;
        p[j] = w0;
        p[j + half] = w1;
    } else {
        uint16_t* p = static_cast<uint16_t*>(pool) + base;
        p[j] = f32_to_bf16_rne(w0);
        p[j + half] = f32_to_bf16_rne(w1);
    }
}

// ------------------------------------------------------------------------------------------------------------------
// batched attention: CTA (split s, KV head, token z), 4 warps.  The split's K/V rows (at most cap) arrive in shared
// memory by bulk copies (one thread per page run); lane l of warp w scores row 32 w + l (+ 128 ...) against the G query
// heads, reading the row's 16-byte chunks in the order (c + l) mod 8 so that the 8 lanes of a shared-memory phase hit
// 8 different chunks (no bank conflicts on K, nor on q); each warp keeps its online-softmax partial, P.V with lane l
// owning dims 2l, 2l+1; the warps merge in shared memory and the CTA writes its partial.  The last CTA of (token, KV
// head) merges the S partials in split order.
// ------------------------------------------------------------------------------------------------------------------
template <bool KV_F32, int G>
__global__ void __launch_bounds__(128) battn_kernel(BAttnArgs a) {
    constexpr int D = kHeadDim, NW = 4;
    constexpr int ESZ = KV_F32 ? 4 : 2;
    constexpr int RB = D * ESZ;  // bytes per K/V row of one head
    constexpr int CH = RB / 16;  // 16-byte chunks per row
    constexpr int EPC = 16 / ESZ;
    extern __shared__ __align__(128) unsigned char smem_raw[];
    unsigned char* kt = smem_raw;
    unsigned char* vt = smem_raw + (size_t)a.cap * RB;
    __shared__ __align__(16) float sq[G][D];
    __shared__ float wm[NW][G], wl[NW][G];
    __shared__ __align__(16) float wacc[NW][G][D];
    __shared__ __align__(8) uint64_t bar;
    __shared__ bool is_last;
    const int S = gridDim.x, s = blockIdx.x, kvh = blockIdx.y, z = blockIdx.z;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int HD = a.kv_heads * G * D;
    pdl_wait();
    pdl_launch();
    const int sqid = __ldg(a.seq + z);
    const int* page_table = a.page_table + (size_t)sqid * a.pt_stride;
    const int len = __ldcg(a.pos + sqid) + (a.off ? __ldg(a.off + z) : 0) + 1;  // causal within a multi-position step
    const int p0 = (int)(((long long)len * s) / S), p1 = (int)(((long long)len * (s + 1)) / S);
    const int nrow = min(p1 - p0, a.cap);
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        mbar_expect_tx(&bar, nrow > 0 ? (uint32_t)nrow * RB * 2 : 0u);
    }
    __syncthreads();
    if (nrow > 0) {
        const int pe = p0 + nrow;
        const int pg0 = p0 / a.page_size, pg1 = (pe - 1) / a.page_size;
        for (int t = threadIdx.x; t <= pg1 - pg0; t += blockDim.x) {
            const int pg = pg0 + t;
            const int lo = max(p0, pg * a.page_size), hi = min(pe, (pg + 1) * a.page_size);
            const int page = __ldcg(page_table + pg);
            const size_t off = (((size_t)page * a.kv_heads + kvh) * a.page_size + (lo - pg * a.page_size)) * RB;
            bulk_g2s(kt + (size_t)(lo - p0) * RB, static_cast<const unsigned char*>(a.k_pool) + off, (uint32_t)(hi - lo) * RB, &bar);
            bulk_g2s(vt + (size_t)(lo - p0) * RB, static_cast<const unsigned char*>(a.v_pool) + off, (uint32_t)(hi - lo) * RB, &bar);
        }
    }
    for (int i = threadIdx.x; i < G * D / 4; i += blockDim.x)
        reinterpret_cast<float4*>(&sq[0][0])[i] = __ldcg(reinterpret_cast<const float4*>(a.q + (size_t)z * HD + (size_t)kvh * G * D) + i);
    __syncthreads();
    const bool ok = mbar_wait(&bar, 0, a.err, 4);

    float m[G], l[G], acc0[G], acc1[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.0f;
        acc0[g] = 0.0f;
        acc1[g] = 0.0f;
    }
    const int nr = ok ? nrow : 0;
    for (int base = warp * 32; base < nr; base += NW * 32) {
        const int r = base + lane;
        const bool valid = r < nr;
        float sc[G];
#pragma unroll
        for (int g = 0; g < G; ++g) sc[g] = 0.0f;
        if (valid) {
            const uint4* kr = reinterpret_cast<const uint4*>(kt + (size_t)r * RB);
#pragma unroll
            for (int c0 = 0; c0 < CH; ++c0) {
                const int c = (c0 + lane) & (CH - 1);
                const uint4 kc = kr[c];
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
        const int nj = min(32, nr - base);
        for (int jj = 0; jj < nj; ++jj) {
            float v0, v1;
            if (KV_F32) {
                const float2 t = reinterpret_cast<const float2*>(vt + (size_t)(base + jj) * RB)[lane];
                v0 = t.x;
                v1 = t.y;
            } else {
                const uint32_t t = reinterpret_cast<const uint32_t*>(vt + (size_t)(base + jj) * RB)[lane];
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
    __syncthreads();
    float* part_acc = a.part_acc + (size_t)z * HD * S;
    float* part_ml = a.part_ml + (size_t)z * a.kv_heads * G * S * 2;
    for (int t = threadIdx.x; t < G * D; t += blockDim.x) {
        const int g = t / D, dim = t - g * D;
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
        const size_t hs = (size_t)(kvh * G + g) * S + s;
        part_acc[hs * D + dim] = A;
        if (dim == 0) {
            part_ml[hs * 2] = M;
            part_ml[hs * 2 + 1] = L;
        }
    }
    if (!last_block_arrives(a.counters + (size_t)z * a.kv_heads + kvh, (unsigned int)S, &is_last)) return;
    // merge the S splits of the G heads, in split order
    for (int t = threadIdx.x; t < G * D; t += blockDim.x) {
        const int g = t / D, dim = t - g * D;
        const size_t h0 = (size_t)(kvh * G + g) * S;
        float M = -INFINITY;
        for (int sp = 0; sp < S; ++sp) M = fmaxf(M, __ldcg(part_ml + (h0 + sp) * 2));
        float den = 0.0f, num = 0.0f;
        for (int sp = 0; sp < S; ++sp) {
            const float ms = __ldcg(part_ml + (h0 + sp) * 2);
            if (ms == -INFINITY) continue;
            const float e = expf(ms - M);
            den = fmaf(__ldcg(part_ml + (h0 + sp) * 2 + 1), e, den);
            num = fmaf(__ldcg(part_acc + (h0 + sp) * D + dim), e, num);
        }
        const float o = num / den;
        const size_t oi = (size_t)z * HD + ((size_t)kvh * G + g) * D + dim;
        a.att_out[oi] = o;
        uint16_t hi, lo;
        split_bf16(o, hi, lo);
        a.att_hi[oi] = hi;
        a.att_lo[oi] = lo;
    }
}

// ------------------------------------------------------------------------------------------------------------------
// group (owner, run by the router grid's last CTA): after every sender's dispatch flag, the received pairs whose
// expert is local are ordered by (local expert, sender, pair): per expert offsets and counts for the grouped GEMMs,
// and per position its rx token row and pair.
// ------------------------------------------------------------------------------------------------------------------
LDEV void group_pairs(const BExchangeArgs& a) {
    __shared__ short le[kBMaxSlots];
    __shared__ int cnt[kMaxExperts], off[kMaxExperts];
    __shared__ int ok_all;
    __shared__ int pairs[kBMaxRanks];  // pairs each sender dispatched in this layer
    const XLayout& L = a.lay;
    unsigned char* me = a.peers[a.rank];
    const unsigned int epoch = __ldcg(a.epoch_base) + a.layer + 1;
    if (threadIdx.x == 0) ok_all = 1;
    if (threadIdx.x < kMaxExperts) cnt[threadIdx.x] = 0;
    __syncthreads();
    if (threadIdx.x < a.world) {
        if (wait_flag(flag_ptr(me, L, 0, threadIdx.x), epoch, a.err, 10 + threadIdx.x, a.world > 1, a.wait_ns))
            pairs[threadIdx.x] =
                (int)ld_acquire_x(reinterpret_cast<const unsigned int*>(me + L.rx_n) + threadIdx.x, a.world > 1) * a.k;
        else
            atomicExch(&ok_all, 0);
    }
    __syncthreads();
    const int slots = a.world * L.cap;
    const int n_experts = a.world * a.experts_per_rank;
    const int* rx_ids = reinterpret_cast<const int*>(me + L.rx_ids);
    for (int i = threadIdx.x; i < slots; i += blockDim.x) {
        const int s = i / L.cap, p = i - s * L.cap;
        int x = -1;
        if (ok_all && p < pairs[s]) {
            const int id = __ldcg(rx_ids + i);
            if (id >= 0 && id < n_experts && __ldg(a.owner + id) == a.rank) {
                x = __ldg(a.local + id);
                atomicAdd(&cnt[x], 1);
            }
        }
        le[i] = (short)x;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int o = 0;
        for (int e = 0; e < a.experts_per_rank; ++e) {
            off[e] = o;
            o += cnt[e];
            a.g_off[e] = off[e];
            a.g_cnt[e] = cnt[e];
        }
        *a.n_pos = o;
    }
    __syncthreads();
    // position of slot i = off[e] + (slots of expert e before i): per chunk of 1024 slots, the rank within the warp
    // from __match_any_sync, the warps' counts per expert prefixed in warp order, plus the earlier chunks' counts
    __shared__ int wcnt[32][kMaxExperts];
    __shared__ int run[kMaxExperts];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (threadIdx.x < kMaxExperts) run[threadIdx.x] = 0;
    for (int c0 = 0; c0 < slots; c0 += blockDim.x) {
        const int i = c0 + threadIdx.x;
        const int e = i < slots ? le[i] : -1;
        wcnt[warp][lane] = 0;
        wcnt[warp][lane + 32] = 0;
        __syncwarp();
        const unsigned int same = __match_any_sync(0xffffffffu, e);
        const int rk = __popc(same & ((1u << lane) - 1u));
        if (e >= 0 && rk == 0) wcnt[warp][e] = __popc(same);
        __syncthreads();
        if (threadIdx.x < a.experts_per_rank) {
            int acc = run[threadIdx.x];
            for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
                const int c = wcnt[w][threadIdx.x];
                wcnt[w][threadIdx.x] = acc;
                acc += c;
            }
            run[threadIdx.x] = acc;
        }
        __syncthreads();
        if (e >= 0) {
            const int pos = off[e] + wcnt[warp][e] + rk;
            const int sender = i / L.cap, pair = i - sender * L.cap;
            a.x_rows[pos] = sender * L.cap_tok + pair / a.k;
            a.src[pos] = i;
        }
        __syncthreads();
    }
}

// ------------------------------------------------------------------------------------------------------------------
// router: h += resid * (o-projection slices summed in order); xn = RMSNorm(h) (f32, kept for the router, split hi + lo
// for the experts); logits_e = W_r[e] . xn (+ bias_e), one warp per expert; top-k in block.rs:81-89's order, softmax.
// ------------------------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) brouter_kernel(BRouterArgs a) {
    const CtaTrace trace_(a.trace);
    constexpr int BLOCK = 256, NV = 2;
    extern __shared__ __align__(16) float xs[];  // [H]
    __shared__ float red[BLOCK / 32];
    __shared__ float lg[kMaxExperts];
    __shared__ int sid[kMaxTopK];
    __shared__ float sval[kMaxTopK], sw[kMaxTopK], ex[kMaxTopK];
    __shared__ unsigned long long keys[kMaxExperts];
    __shared__ bool is_last;
    const int t = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float* h = a.h + (size_t)t * a.H;
    pdl_wait();
    pdl_launch();
    trace_.released();
    float4 v[NV];
#pragma unroll
    for (int k = 0; k < NV; ++k) {
        const int i = threadIdx.x + k * BLOCK;
        v[k] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (4 * i >= a.H) continue;
        float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
        float4 pz[16];  // every slice in flight at once (ks <= 16), summed in slice order
#pragma unroll
        for (int z = 0; z < 16; ++z)
            if (z < a.ks) pz[z] = __ldcg(reinterpret_cast<const float4*>(a.opart + ((size_t)z * a.n + t) * a.H) + i);
#pragma unroll
        for (int z = 0; z < 16; ++z) {
            if (z < a.ks) {
                o.x = __fadd_rn(o.x, pz[z].x);
                o.y = __fadd_rn(o.y, pz[z].y);
                o.z = __fadd_rn(o.z, pz[z].z);
                o.w = __fadd_rn(o.w, pz[z].w);
            }
        }
        const float4 hv = __ldcg(reinterpret_cast<const float4*>(h) + i);
        v[k] = make_float4(__fadd_rn(hv.x, __fmul_rn(a.resid, o.x)), __fadd_rn(hv.y, __fmul_rn(a.resid, o.y)),
                           __fadd_rn(hv.z, __fmul_rn(a.resid, o.z)), __fadd_rn(hv.w, __fmul_rn(a.resid, o.w)));
        reinterpret_cast<float4*>(h)[i] = v[k];
    }
    float ss = 0.0f;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
        ss = fmaf(v[k].x, v[k].x, ss);
        ss = fmaf(v[k].y, v[k].y, ss);
        ss = fmaf(v[k].z, v[k].z, ss);
        ss = fmaf(v[k].w, v[k].w, ss);
    }
    const float tot = block_sum(ss, red);
    const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)a.H), a.eps)));
#pragma unroll
    for (int k = 0; k < NV; ++k) {
        const int i = threadIdx.x + k * BLOCK;
        if (4 * i >= a.H) continue;
        reinterpret_cast<float4*>(xs)[i] = ln_times(__ldg(reinterpret_cast<const float4*>(a.ln) + i), v[k], r);
    }
    __syncthreads();
    trace_.mark_after(5, xs[threadIdx.x]);
    for (int e = warp; e < a.E; e += BLOCK / 32) {
        // the row's chunks (H <= 2048: at most 8 per lane) all loaded before the first product
        const uint16_t* row = a.wr + (size_t)e * a.H;
        uint4 w[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const int c = lane * 8 + q * 256;
            w[q] = c < a.H ? ld_weight(row + c) : make_uint4(0u, 0u, 0u, 0u);
        }
        float acc = 0.0f;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const int c = lane * 8 + q * 256;
            if (c < a.H)
                acc = dot8(w[q], *reinterpret_cast<const float4*>(xs + c), *reinterpret_cast<const float4*>(xs + c + 4), acc);
        }
        acc = warp_sum(acc);
        if (lane == 0) lg[e] = a.bias ? __fadd_rn(acc, __ldg(a.bias + e)) : acc;
    }
    __syncthreads();
    trace_.mark_after(0, lg[threadIdx.x & 31]);
    // the top-k over the whole block (one warp exchanging the keys by shuffles while the other seven waited at the
    // barrier measured 17.6 us per layer with the trace stamps on; this form 1.0 us, and bitwise the same routing)
    route_topk_block(lg, a.E, a.k, keys, ex, sid, sval, sw);
    if (threadIdx.x < a.k) {
        a.ids[(size_t)t * a.k + threadIdx.x] = sid[threadIdx.x];
        a.weights[(size_t)t * a.k + threadIdx.x] = sw[threadIdx.x];
        if (a.route_hist) a.route_hist[((size_t)t * a.layers + a.layer) * a.k + threadIdx.x] = sid[threadIdx.x];
    }
    trace_.mark_after(3, sw[0]);
    // dispatch: the token's MoE input row (hi then lo) once to every rank that owns one of its experts, its k expert
    // ids to every rank; the last CTA publishes this rank's dispatch flag on every rank
    const BExchangeArgs& x = a.x;
    const XLayout& L = x.lay;
    for (int j = 0; j < a.k; ++j) {
        const int o = __ldg(x.owner + sid[j]);
        bool seen = false;
        for (int jj = 0; jj < j; ++jj) seen |= __ldg(x.owner + sid[jj]) == o;
        if (seen) continue;  // the same for every thread (sid is shared)
        unsigned char* dst = x.peers[o] + L.rx + ((size_t)x.rank * L.cap_tok + t) * (size_t)a.H * 4;
        for (int i = threadIdx.x; i < a.H / 4; i += BLOCK) {
            const float4 v4 = reinterpret_cast<const float4*>(xs)[i];
            ushort4 hi, lo;
            split_bf16(v4.x, hi.x, lo.x);
            split_bf16(v4.y, hi.y, lo.y);
            split_bf16(v4.z, hi.z, lo.z);
            split_bf16(v4.w, hi.w, lo.w);
            reinterpret_cast<ushort4*>(dst)[i] = hi;
            reinterpret_cast<ushort4*>(dst + (size_t)a.H * 2)[i] = lo;
        }
    }
    trace_.mark(4);
    for (int i = threadIdx.x; i < x.world * a.k; i += BLOCK) {
        const int q = i / a.k, j = i - q * a.k;
        reinterpret_cast<int*>(x.peers[q] + L.rx_ids)[(size_t)x.rank * L.cap + (size_t)t * a.k + j] = sid[j];
    }
    if (t == 0 && threadIdx.x < x.world) reinterpret_cast<int*>(x.peers[threadIdx.x] + L.rx_n)[x.rank] = a.n;
    trace_.mark(1);
    if (!last_block_arrives_sys(x.counter, gridDim.x, &is_last, x.world > 1)) return;
    if (threadIdx.x < x.world) {
        const unsigned int epoch = __ldcg(x.epoch_base) + x.layer + 1;
        st_release_x(flag_ptr(x.peers[threadIdx.x], L, 0, x.rank), epoch, x.world > 1);
    }
    trace_.mark(2);
    // the same CTA then waits for every rank's dispatch and groups the pairs this rank's experts received
    __syncthreads();
    group_pairs(x);
}

// ------------------------------------------------------------------------------------------------------------------
// combine (sender): CTA per token, after every owner's return flag: h += resid * sum_j w_j y_j, slots in routing
// order (cpu.rs:141-148).
// ------------------------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) ep_combine_kernel(BExchangeArgs a) {
    const CtaTrace trace_(a.trace);
    constexpr int BLOCK = 256, NV = 8;  // H <= 2048
    __shared__ int ok_all;
    __shared__ float red[BLOCK / 32];
    const XLayout& L = a.lay;
    unsigned char* me = a.peers[a.rank];
    const int t = blockIdx.x;
    pdl_wait();
    pdl_launch();
    trace_.released();
    const unsigned int epoch = __ldcg(a.epoch_base) + a.layer + 1;
    if (threadIdx.x == 0) ok_all = 1;
    __syncthreads();
    if (threadIdx.x < a.world &&
        !wait_flag(flag_ptr(me, L, 1, threadIdx.x), epoch, a.err, 30 + threadIdx.x, a.world > 1, a.wait_ns))
        atomicExch(&ok_all, 0);
    __syncthreads();
    trace_.mark(0);
    if (!ok_all) return;
    float w[kMaxTopK];
#pragma unroll
    for (int j = 0; j < kMaxTopK; ++j) w[j] = j < a.k ? __ldcg(a.weights + (size_t)t * a.k + j) : 0.0f;
    const float* cb = reinterpret_cast<const float*>(me + L.cb) + (size_t)t * a.k * a.H;
    float* h = a.h + (size_t)t * a.H;
    // every load of the thread first (the stores to h below would otherwise keep the compiler from hoisting them)
    float hv[NV], yv[NV][kMaxTopK];
#pragma unroll
    for (int q = 0; q < NV; ++q) {
        const int i = threadIdx.x + q * BLOCK;
        hv[q] = i < a.H ? __ldcg(h + i) : 0.0f;
#pragma unroll
        for (int j = 0; j < kMaxTopK; ++j) yv[q][j] = (i < a.H && j < a.k) ? __ldcg(cb + (size_t)j * a.H + i) : 0.0f;
    }
    float ss = 0.0f;
#pragma unroll
    for (int q = 0; q < NV; ++q) {
        const int i = threadIdx.x + q * BLOCK;
        if (i >= a.H) continue;
        float acc = 0.0f;
#pragma unroll
        for (int j = 0; j < kMaxTopK; ++j)
            if (j < a.k) acc = __fadd_rn(acc, __fmul_rn(w[j], yv[q][j]));
        hv[q] = __fadd_rn(hv[q], __fmul_rn(a.resid, acc));
        h[i] = hv[q];
        ss = fmaf(hv[q], hv[q], ss);
    }
    if (!a.ln_next) return;
    // the next RMSNorm (model.rs:141-145): xn = ln * (h * r), split into hi + lo
    const float tot = block_sum(ss, red);
    const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)a.H), a.eps)));
#pragma unroll
    for (int q = 0; q < NV; ++q) {
        const int i = threadIdx.x + q * BLOCK;
        if (i >= a.H) continue;
        uint16_t hi, lo;
        split_bf16(__fmul_rn(__ldg(a.ln_next + i), __fmul_rn(hv[q], r)), hi, lo);
        a.xn_hi[(size_t)t * a.H + i] = hi;
        a.xn_lo[(size_t)t * a.H + i] = lo;
    }
}

// ------------------------------------------------------------------------------------------------------------------
// argmax per token (the last maximum, bin/m1b-gulosa.rs:22-24), position advanced, next token fed back
// ------------------------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) bargmax_kernel(BHeadArgs a) {
    const CtaTrace trace_(a.trace);
    __shared__ unsigned long long best[32];
    const int t = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const float* lg = a.logits + (size_t)t * a.V;
    pdl_wait();
    pdl_launch();
    trace_.released();
    // four independent running maxima per thread (keys order by value, then by index: the last maximum wins)
    unsigned long long b0 = 0ull, b1 = 0ull, b2 = 0ull, b3 = 0ull;
    const int stride = 4 * blockDim.x;
    for (int v = threadIdx.x; v < a.V; v += stride) {
        const int v1 = v + blockDim.x, v2 = v + 2 * blockDim.x, v3 = v + 3 * blockDim.x;
        const unsigned long long k0 = arg_key(__ldcg(lg + v), v);
        const unsigned long long k1 = v1 < a.V ? arg_key(__ldcg(lg + v1), v1) : 0ull;
        const unsigned long long k2 = v2 < a.V ? arg_key(__ldcg(lg + v2), v2) : 0ull;
        const unsigned long long k3 = v3 < a.V ? arg_key(__ldcg(lg + v3), v3) : 0ull;
        b0 = k0 > b0 ? k0 : b0;
        b1 = k1 > b1 ? k1 : b1;
        b2 = k2 > b2 ? k2 : b2;
        b3 = k3 > b3 ? k3 : b3;
    }
    unsigned long long b = b0 > b1 ? b0 : b1;
    b = b2 > b ? b2 : b;
    b = b3 > b ? b3 : b;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long x = shfl_xor_u64(b, o);
        b = x > b ? x : b;
    }
    if (lane == 0) best[warp] = b;
    __syncthreads();
    if (threadIdx.x != 0) return;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) b = best[w] > b ? best[w] : b;
    const int id = (int)(uint32_t)b;
    a.next[t] = id;
    if (a.tokens) a.tokens[t] = id;
    atomicAdd(a.pos + __ldg(a.seq + t), 1);  // a multi-position step has several tokens of one sequence
    if (t == 0) *a.epoch_base += (unsigned int)a.layers;
}

// ------------------------------------------------------------------------------------------------------------------
// The same GEMM on the 5th-generation tensor cores.  The shared-memory tiles are those of bgemm_kernel (rows of 128 bytes,
// 16-byte chunk c of row r at c ^ (r & 7): the 128-byte swizzle of the K-major canonical layout, atoms of 8 rows = 1024
// bytes), loaded by all threads with cp.async; thread 0 issues, per 16-wide K step, tcgen05.mma kind::f16 (bf16 A = 128
// weight rows, bf16 B = the N token rows, N = n rounded up to 16) twice -- x hi, then x lo -- into one f32 accumulator of
// 128 lanes x N columns in tensor memory, and commits each stage to an mbarrier that frees the stage for the next load.
// The epilogue reads the accumulator with tcgen05.ld (warp w: lanes 32w..32w+31 = weight rows, one register per token).
// ------------------------------------------------------------------------------------------------------------------
namespace {

LDEV uint64_t smem_desc_sw128(uint32_t addr) {
    // start address >> 4 [0,14), leading byte offset 16 B >> 4 [16,30), stride byte offset 1024 B >> 4 [32,46),
    // descriptor version 1 [46,48), base offset 0, 128-byte swizzle (2) [61,64)
    return (uint64_t)((addr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) |
           ((uint64_t)2 << 61);
}

// kind::f16 instruction descriptor: f32 accumulator (bits 4-5 = 1), bf16 A and B (bits 7-9, 10-12 = 1), both K-major,
// N >> 3 at bits 17-22, M >> 4 at bits 24-28
LDEV uint32_t idesc_bf16_f32(int M, int N) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

LDEV void tc_mma(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, bool accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"((uint32_t)accumulate)
        : "memory");
}

LDEV void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

LDEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
LDEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

LDEV void tc_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

constexpr int kTmemCols = 64;  // accumulator columns (tokens of one tile)

}  // namespace

template <int EPI>
__global__ void __launch_bounds__(128) bgemm_tc_kernel(BGemmArgs a) {
    extern __shared__ unsigned char smem_dyn[];
    // tiles on a 1024-byte boundary (the swizzle atom); the launch reserves the slack
    unsigned char* smem = smem_dyn + ((1024 - (smem_addr(smem_dyn) & 1023)) & 1023);
    __shared__ __align__(8) uint64_t bar[kBStages];
    __shared__ uint32_t tmem_base;
    __shared__ bool is_last;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = blockIdx.y, bx = blockIdx.x;
    pdl_wait();
    pdl_launch();
    int p0 = 0, ntot = a.n;
    if (a.g_cnt) {
        p0 = __ldcg(a.g_off + g);
        ntot = __ldcg(a.g_cnt + g);
    }
    const uint16_t* W = a.w + (size_t)weight_group(a, g) * a.group_stride;
    const int kbeg = blockIdx.z * a.k_split;
    const int nk = min(a.k_split, a.K - kbeg) / kBK;
    if (nk <= 0) ntot = 0;
    if (EPI != BEPI_RETURN && ntot <= 0) return;  // (a RETURN CTA still votes below)
    const int ch = tid & 7;
    auto grow_of = [&](int sr) -> int {
        if (EPI == BEPI_SWIGLU) return sr < 64 ? bx * 64 + sr : a.I + bx * 64 + (sr - 64);
        return bx * kBRows + sr;
    };
    if (ntot > 0) {
        if (warp == 0) {
            asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&tmem_base)),
                         "r"(kTmemCols)
                         : "memory");
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        }
        if (tid == 0)
            for (int i = 0; i < kBStages; ++i) mbar_init(&bar[i], 1);
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
    }
    const uint32_t tmem = tmem_base;
    // per stage barrier: bit s of `used` once a commit has targeted it, bit s of `par` the parity of its commit count
    // (every thread tracks them alike); the wait for the latest commit of stage s is on phase parity par_s ^ 1
    uint32_t used = 0, par = 0;
    bool ok = true;

    for (int t0 = 0; t0 < ntot && ok; t0 += kBTok) {
        const int n = min(kBTok, ntot - t0);
        const int N = (n + 15) & ~15;
        const uint32_t idesc = idesc_bf16_f32(128, N);
        int xrow[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int tok = (tid >> 3) + 16 * i;
            const int p = p0 + t0 + tok;
            xrow[i] = tok < n ? (a.x_rows ? __ldcg(a.x_rows + p) : p) : 0;
        }
        auto load_stage = [&](int slot, int kt) {
            unsigned char* st = smem + (size_t)slot * kBStageBytes;
            const int k0 = kbeg + kt * kBK + ch * 8;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int sr = (tid >> 3) + 16 * i;
                const int gr = grow_of(sr);
                const bool v = gr < a.rows;
                cp_async16(smem_addr(st) + swz(sr, ch), W + (size_t)(v ? gr : 0) * a.K + k0, v);
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int tok = (tid >> 3) + 16 * i;
                const bool v = tok < n;
                const size_t xo = (size_t)xrow[i] * a.ldx + k0;
                const uint32_t d = swz(tok, ch);
                cp_async16(smem_addr(st + kBRows * 128) + d, a.x_hi + xo, v);
                cp_async16(smem_addr(st + kBRows * 128 + kBTok * 128) + d, a.x_lo + xo, v);
            }
        };
        // wait until the MMAs that read `slot` last have completed (bounded)
        auto stage_free = [&](int slot) -> bool {
            if (!((used >> slot) & 1)) return true;
            return mbar_wait(&bar[slot], ((par >> slot) & 1) ^ 1, a.x.err, 5);
        };
#pragma unroll
        for (int s = 0; s < kBStages - 1; ++s) {
            if (s < nk) {
                ok = ok && stage_free(s);
                load_stage(s, s);
            }
            cp_async_commit();
        }
        for (int kt = 0; kt < nk; ++kt) {
            const int slot = kt % kBStages;
            cp_async_wait<kBStages - 2>();
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // cp.async data visible to the tensor core
            __syncthreads();
            if (tid == 0) {
                tc_fence_after();
                const uint32_t sW = smem_addr(smem + (size_t)slot * kBStageBytes);
                const uint32_t sXh = sW + kBRows * 128, sXl = sXh + kBTok * 128;
#pragma unroll
                for (int kk = 0; kk < kBK / 16; ++kk) {
                    const uint64_t ad = smem_desc_sw128(sW + kk * 32);
                    tc_mma(tmem, ad, smem_desc_sw128(sXh + kk * 32), idesc, kt > 0 || kk > 0);
                    tc_mma(tmem, ad, smem_desc_sw128(sXl + kk * 32), idesc, true);
                }
                tc_commit(&bar[slot]);
            }
            used |= 1u << slot;
            par ^= 1u << slot;
            const int pf = kt + kBStages - 1;
            if (pf < nk) {
                const int ps = pf % kBStages;
                ok = ok && stage_free(ps);
                load_stage(ps, pf);
            }
            cp_async_commit();
        }
        cp_async_wait<0>();
        // every MMA of this tile done: the last stage's barrier (commits track all earlier MMAs of the thread)
        const int last = (nk - 1) % kBStages;
        ok = ok && mbar_wait(&bar[last], ((par >> last) & 1) ^ 1, a.x.err, 6);
        tc_fence_after();
        if (!ok) break;

        // epilogue: thread (warp w, lane) holds tile row 32w + lane, columns = tokens
        const int row = warp * 32 + lane;
        const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
        if (EPI == BEPI_STORE) {
            const int gr = bx * kBRows + row;
            for (int c0 = 0; c0 < N; c0 += 16) {
                float v[16];
                tc_ld16(trow + c0, v);
#pragma unroll
                for (int c = 0; c < 16; ++c) {
                    const int tok = c0 + c;
                    if (tok < n && gr < a.rows)
                        a.y[blockIdx.z * a.z_stride + (size_t)(p0 + t0 + tok) * a.ldy + gr] =
                            a.div == 1.0f ? v[c] : __fdiv_rn(v[c], a.div);
                }
            }
        } else {
            // stage the tile as [token][128 rows] f32 in shared memory (the pipeline buffers are free now)
            __syncthreads();
            float* stile = reinterpret_cast<float*>(smem);
            for (int c0 = 0; c0 < N; c0 += 16) {
                float v[16];
                tc_ld16(trow + c0, v);
#pragma unroll
                for (int c = 0; c < 16; ++c) stile[(c0 + c) * kBRows + row] = v[c];
            }
            __syncthreads();
            if (EPI == BEPI_SWIGLU) {
                for (int i = tid; i < n * 64; i += 128) {
                    const int tok = i >> 6, r = i & 63;
                    const float gv = stile[tok * kBRows + r], uv = stile[tok * kBRows + 64 + r];
                    const float v = __fmul_rn(__fdiv_rn(gv, __fadd_rn(1.0f, expf(-gv))), uv);
                    uint16_t hi, lo;
                    split_bf16(v, hi, lo);
                    const size_t o = (size_t)(p0 + t0 + tok) * a.I + bx * 64 + r;
                    a.a_hi[o] = hi;
                    a.a_lo[o] = lo;
                }
            } else {
                const XLayout& L = a.x.lay;
                for (int tok = warp; tok < n; tok += 4) {
                    const int i = __ldcg(a.x.src + p0 + t0 + tok);
                    const int sender = i / L.cap, pair = i - sender * L.cap;
                    float4* dst = reinterpret_cast<float4*>(a.x.peers[sender] + L.cb +
                                                            ((size_t)pair * a.rows + (size_t)bx * kBRows) * 4);
                    dst[lane] = reinterpret_cast<const float4*>(stile + tok * kBRows)[lane];
                }
            }
            __syncthreads();
        }
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
    }
    if (ntot > 0) {
        tc_fence_before();
        __syncthreads();
        if (warp == 0)
            asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
    if (EPI == BEPI_RETURN) {
        if (!last_block_arrives_sys(a.x.counter, gridDim.x * gridDim.y * gridDim.z, &is_last, a.x.world > 1)) return;
        if (tid < a.x.world) {
            const unsigned int epoch = __ldcg(a.x.epoch_base) + a.x.layer + 1;
            st_release_x(flag_ptr(a.x.peers[tid], a.x.lay, 1, a.x.rank), epoch, a.x.world > 1);
        }
    }
}

// bgemm_ws setup (all threads): the accumulator's tensor-memory columns, the stage barriers (full: the TMA thread's
// expect_tx arrival + 64 cp.async arrivals; empty: one MMA commit), the tile's done barrier
LDEV void bgemm_ws_setup(uint32_t* tmem_base, uint64_t* full, uint64_t* empty, uint64_t* done, int stages,
                         const CUtensorMap* wmap, int tid, int warp) {
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_base)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
        for (int i = 0; i < stages; ++i) {
            mbar_init(&full[i], 1 + 64);
            mbar_init(&empty[i], 1);
        }
        mbar_init(done, 1);
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(wmap)) : "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
}

// ------------------------------------------------------------------------------------------------------------------
// Warp-specialised tcgen05 GEMM (mode 2).  Per stage: 16 KB of weight rows by TMA (two boxes of 64 rows x 64 columns,
// 128-byte swizzle, issued by lane 0 of warp 0) and the token rows' hi and lo (cp.async by warps 2-3, 16 each per
// thread, arriving on the stage's full barrier when they land); lane 0 of warp 1 waits for the full barrier, issues
// the 8 MMAs of the stage and commits them to the stage's empty barrier, which the producers wait on before they
// refill it.  No block-wide barrier inside the K loop.  The epilogue (all 4 warps) follows the final commit.
// ------------------------------------------------------------------------------------------------------------------
namespace {

LDEV void cp_async_arrive_noinc(uint64_t* bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_addr(bar)) : "memory");
}

}  // namespace

template <int EPI, int TOK>
__global__ void __launch_bounds__(128) bgemm_ws_kernel(const __grid_constant__ CUtensorMap wmap, BGemmArgs a) {
    // TOK tokens per tile: 64 with 3 stages of 32 KB (2 CTAs per SM), or 32 with 2 stages of 24 KB (4 CTAs per SM).
    // Measured on the C5 step (1 B200): 64/3 for every GEMM 5.05 ms, 32/4 for the expert groups 5.15 ms, 32/2 5.21 ms;
    // the launches use 64.
    const CtaTrace trace_(a.trace);
    static_assert(TOK == 32 || TOK == 64, "token tile");
    constexpr int S = TOK == 64 ? 3 : 2;
    constexpr size_t STAGE = (size_t)kBRows * 128 + 2 * (size_t)TOK * 128;
    static_assert(S * STAGE <= kBGemmSmem, "stages fit the launch's shared memory");
    extern __shared__ unsigned char smem_dyn[];
    unsigned char* smem = smem_dyn + ((1024 - (smem_addr(smem_dyn) & 1023)) & 1023);
    __shared__ __align__(8) uint64_t full[S], empty[S], done;
    __shared__ uint32_t tmem_base;
    __shared__ bool is_last;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = blockIdx.y, bx = blockIdx.x;
    const int kbeg = blockIdx.z * a.k_split;
    const int nk = min(a.k_split, a.K - kbeg) / kBK;
    // weight rows of the tile's two 64-row boxes (row coordinates in the tensor map)
    const int wg = weight_group(a, g);
    const int wrow0 = wg * a.rows + (EPI == BEPI_SWIGLU ? bx * 64 : bx * kBRows);
    const int wrow1 = wg * a.rows + (EPI == BEPI_SWIGLU ? a.I + bx * 64 : bx * kBRows + 64);
    // a dense launch (no groups) knows its tokens and weights before the previous kernel ends: its setup and the
    // weight tiles of the first S stages are issued before griddepcontrol.wait
    const int pre = (!a.g_cnt && a.n > 0 && nk > 0) ? min(S, nk) : 0;
    if (pre > 0) {
        bgemm_ws_setup(&tmem_base, full, empty, &done, S, &wmap, tid, warp);
        if (tid == 0) {
            for (int kt = 0; kt < pre; ++kt) {
                unsigned char* st = smem + (size_t)kt * STAGE;
                mbar_expect_tx(&full[kt], kBRows * 128);
                tma_load_2d(st, &wmap, kbeg + kt * kBK, wrow0, &full[kt]);
                tma_load_2d(st + 64 * 128, &wmap, kbeg + kt * kBK, wrow1, &full[kt]);
            }
        }
    }
    pdl_wait();
    pdl_launch();
    trace_.released();
    int p0 = 0, ntot = a.n;
    if (a.g_cnt) {
        p0 = __ldcg(a.g_off + g);
        ntot = __ldcg(a.g_cnt + g);
    }
    if (nk <= 0) ntot = 0;
    if (EPI != BEPI_RETURN && ntot <= 0) return;  // (a RETURN CTA still votes below)
    if (ntot > 0 && pre == 0) bgemm_ws_setup(&tmem_base, full, empty, &done, S, &wmap, tid, warp);
    trace_.mark(0);
    const uint32_t tmem = tmem_base;
    bool ok = true;
    int it = 0;  // global stage counter over the CTA's tiles (stage it % S, round it / S)
    int tile = 0;
    for (int t0 = 0; t0 < ntot; t0 += TOK, ++tile) {
        const int n = min(TOK, ntot - t0);
        const int N = (n + 15) & ~15;
        // (the whole of warps 0 and 1 runs their loops, lane 0 doing the work, so that the idle lanes wait at
        // __syncwarp instead of spinning on a barrier in the lanes' own divergent path)
        if (warp == 0) {
            bool go = true;
            for (int kt = 0; kt < nk && go; ++kt) {
                if (lane == 0 && it + kt >= pre) {
                    const int s = (it + kt) % S, r = (it + kt) / S;
                    if (r > 0 && !mbar_wait(&empty[s], (r - 1) & 1, a.x.err, 7)) {
                        go = false;
                    } else {
                        unsigned char* st = smem + (size_t)s * STAGE;
                        mbar_expect_tx(&full[s], kBRows * 128);
                        const int x = kbeg + kt * kBK;
                        tma_load_2d(st, &wmap, x, wrow0, &full[s]);
                        tma_load_2d(st + 64 * 128, &wmap, x, wrow1, &full[s]);
                    }
                }
                go = __shfl_sync(0xffffffffu, go, 0);
            }
        } else if (warp == 1) {
            const uint32_t idesc = idesc_bf16_f32(128, N);
            bool go = true;
            for (int kt = 0; kt < nk && go; ++kt) {
                if (lane == 0) {
                    const int s = (it + kt) % S, r = (it + kt) / S;
                    if (!mbar_wait(&full[s], r & 1, a.x.err, 8)) {
                        go = false;
                    } else {
                        if (tile == 0 && kt == 0) trace_.mark(1, 32);
                        if (tile == 0 && kt == 1) trace_.mark(4, 32);
                        if (tile == 0 && kt == nk / 2) trace_.mark(5, 32);
                        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // the cp.async rows, for the MMA
                        tc_fence_after();
                        const uint32_t sW = smem_addr(smem + (size_t)s * STAGE);
                        const uint32_t sXh = sW + kBRows * 128, sXl = sXh + TOK * 128;
#pragma unroll
                        for (int kk = 0; kk < kBK / 16; ++kk) {
                            const uint64_t ad = smem_desc_sw128(sW + kk * 32);
                            tc_mma(tmem, ad, smem_desc_sw128(sXh + kk * 32), idesc, kt > 0 || kk > 0);
                            tc_mma(tmem, ad, smem_desc_sw128(sXl + kk * 32), idesc, true);
                        }
                        tc_commit(&empty[s]);
                    }
                }
                go = __shfl_sync(0xffffffffu, go, 0);
            }
            if (!go) ok = false;
            if (tile == 0) trace_.mark(2, 32);
            if (lane == 0) tc_commit(&done);  // all MMAs of the tile
            __syncwarp();
        } else {
            // warps 2-3: the token rows of every stage, 16 cp.async per thread, then an arrival when they land
            const int pt = tid - 64;  // 0..63
            const int ch = pt & 7;
            int xrow[TOK / 8];
#pragma unroll
            for (int i = 0; i < TOK / 8; ++i) {
                const int tok = (pt >> 3) + 8 * i;
                const int p = p0 + t0 + tok;
                xrow[i] = tok < n ? (a.x_rows ? __ldcg(a.x_rows + p) : p) : 0;
            }
            for (int kt = 0; kt < nk; ++kt) {
                const int s = (it + kt) % S, r = (it + kt) / S;
                if (r > 0 && !mbar_wait(&empty[s], (r - 1) & 1, a.x.err, 9)) break;
                unsigned char* st = smem + (size_t)s * STAGE;
                const int k0 = kbeg + kt * kBK + ch * 8;
#pragma unroll
                for (int i = 0; i < TOK / 8; ++i) {
                    const int tok = (pt >> 3) + 8 * i;
                    const bool v = tok < n;
                    const size_t xo = (size_t)xrow[i] * a.ldx + k0;
                    const uint32_t d = swz(tok, ch);
                    cp_async16(smem_addr(st + kBRows * 128) + d, a.x_hi + xo, v);
                    cp_async16(smem_addr(st + kBRows * 128 + TOK * 128) + d, a.x_lo + xo, v);
                }
                cp_async_arrive_noinc(&full[s]);
            }
        }
        it += nk;
        // epilogue (all warps): after the tile's final commit
        ok = mbar_wait(&done, tile & 1, a.x.err, 10) && ok;
        tc_fence_after();
        if (tile == 0) trace_.mark(3);
        if (!ok) break;
        const int row = warp * 32 + lane;
        const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
        if (EPI == BEPI_STORE) {
            const int gr = bx * kBRows + row;
            for (int c0 = 0; c0 < N; c0 += 16) {
                float v[16];
                tc_ld16(trow + c0, v);
#pragma unroll
                for (int c = 0; c < 16; ++c) {
                    const int tok = c0 + c;
                    if (tok < n && gr < a.rows)
                        a.y[blockIdx.z * a.z_stride + (size_t)(p0 + t0 + tok) * a.ldy + gr] =
                            a.div == 1.0f ? v[c] : __fdiv_rn(v[c], a.div);
                }
            }
        } else {
            // the pipeline buffers are idle: the tile goes through shared memory as [token][128 rows] f32
            float* stile = reinterpret_cast<float*>(smem);
            for (int c0 = 0; c0 < N; c0 += 16) {
                float v[16];
                tc_ld16(trow + c0, v);
#pragma unroll
                for (int c = 0; c < 16; ++c) stile[(c0 + c) * kBRows + row] = v[c];
            }
            __syncthreads();
            if (EPI == BEPI_SWIGLU) {
                for (int i = tid; i < n * 64; i += 128) {
                    const int tok = i >> 6, r = i & 63;
                    const float gv = stile[tok * kBRows + r], uv = stile[tok * kBRows + 64 + r];
                    const float v = __fmul_rn(__fdiv_rn(gv, __fadd_rn(1.0f, expf(-gv))), uv);
                    uint16_t hi, lo;
                    split_bf16(v, hi, lo);
                    const size_t o = (size_t)(p0 + t0 + tok) * a.I + bx * 64 + r;
                    a.a_hi[o] = hi;
                    a.a_lo[o] = lo;
                }
            } else {
                const XLayout& L = a.x.lay;
                for (int tok = warp; tok < n; tok += 4) {
                    const int i = __ldcg(a.x.src + p0 + t0 + tok);
                    const int sender = i / L.cap, pair = i - sender * L.cap;
                    float4* dst = reinterpret_cast<float4*>(a.x.peers[sender] + L.cb +
                                                            ((size_t)pair * a.rows + (size_t)bx * kBRows) * 4);
                    dst[lane] = reinterpret_cast<const float4*>(stile + tok * kBRows)[lane];
                }
            }
        }
        // the next tile's loads and MMAs reuse shared memory and the accumulator
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
    }
    if (ntot > 0) {
        tc_fence_before();
        __syncthreads();
        if (warp == 0)
            asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
    if (EPI == BEPI_RETURN) {
        if (!last_block_arrives_sys(a.x.counter, gridDim.x * gridDim.y * gridDim.z, &is_last, a.x.world > 1)) return;
        if (tid < a.x.world) {
            const unsigned int epoch = __ldcg(a.x.epoch_base) + a.x.layer + 1;
            st_release_x(flag_ptr(a.x.peers[tid], a.x.lay, 1, a.x.rank), epoch, a.x.world > 1);
        }
    }
}

cudaError_t make_weight_map(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols) {
    return make_tile_map(map, base, rows, cols, 64);
}

cudaError_t make_tile_map(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
    static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    if (!encode) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
        if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn) return e != cudaSuccess ? e : cudaErrorNotSupported;
        encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    if ((reinterpret_cast<uintptr_t>(base) & 15) || (cols * 2) % 16 || rows >= (1ull << 31) || box_rows < 1 || box_rows > 256)
        return cudaErrorInvalidValue;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols * 2};
    const cuuint32_t box[2] = {64, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// ------------------------------------------------------------------------------------------------------------------
// Batched attention on tensor cores (bf16 KV), streaming.  CTA per (KV head, token), 4 warps, walking the token's
// context one 64-position page at a time through a 3-stage TMA pipeline (K and V page per stage, 128-byte swizzle):
// warp w owns rows 16w..16w+15 of every page.  Per page: S = Q K^T with the G query heads as the M = 16 rows (padded
// with zeros) and q split into bf16 hi + lo (mma.sync m16n8k16, f32 accumulators), online softmax per head across
// the quad of lanes that holds it, O += P V with P (split hi + lo) taken straight from the S accumulators as the A
// operand and V through ldmatrix.trans.  Positions past the context carry finite values (the pools are zeroed at
// creation and only ever hold model outputs) and get P = 0.  The 4 warps merge in shared memory at the end.  With
// few tokens (expert parallelism leaves a rank 64/N of them) the context is split over gridDim.x CTAs of consecutive
// pages, each writing a partial (m, l, acc); the last CTA of (token, KV head) merges them in split order.
// ------------------------------------------------------------------------------------------------------------------
namespace {
LDEV void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
constexpr int kAttnStages = 3;
constexpr int kPageBytes = 64 * 128;  // one KV head's 64 positions, bf16
}  // namespace

template <int G>
__global__ void __launch_bounds__(128) battn_tc_kernel(const __grid_constant__ CUtensorMap kmap,
                                                       const __grid_constant__ CUtensorMap vmap, BAttnArgs a) {
    const CtaTrace trace_(a.trace);
    constexpr int D = kHeadDim, NW = 4, P = kAttnStages;
    static_assert(G <= 8, "heads of a group padded to the MMA's 16 rows");
    extern __shared__ unsigned char smem_dyn[];
    unsigned char* st0 = smem_dyn + ((1024 - (smem_addr(smem_dyn) & 1023)) & 1023);  // [P][K page, V page]
    __shared__ __align__(8) uint64_t full[P], empty[P];
    __shared__ float wm[NW][G], wl[NW][G];
    __shared__ __align__(16) float wacc[NW][G][D];
    __shared__ bool is_last;
    const int S = gridDim.x, sp = blockIdx.x, kvh = blockIdx.y, z = blockIdx.z;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, gq = lane >> 2, tq = lane & 3;
    const int HD = a.kv_heads * G * D;
    // The sequence, its page table and position were written two or more kernels back (the host's copy, the previous
    // step's argmax): read before griddepcontrol.wait.  Pages wholly below the current position hold K/V of earlier
    // steps: their TMA loads start before the wait too, overlapping the previous kernel's tail; the page of the
    // current position (written by the previous kernel) is loaded after it.
    const int sqid = a.seq ? __ldg(a.seq + z) : 0;
    const int* page_table = a.page_table + (size_t)sqid * a.pt_stride;
    const int base = __ldcg(a.pos + sqid);  // this step's first new position (of the sequence)
    const int len = base + (a.off ? __ldg(a.off + z) : 0) + 1;  // causal within a multi-position step
    const int ntot = (len + 63) / 64;
    const int per = (ntot + S - 1) / S;
    const int pbeg = min(ntot, sp * per), npages = min(ntot, pbeg + per) - pbeg;  // this split's pages
    const int fresh = base / 64;  // first page holding a row the previous kernel wrote
    auto issue = [&](int i) {  // thread 0: the split's i-th page into stage i % P
        const int pg = pbeg + i;
        const int st = i % P;
        const int y = (__ldcg(page_table + pg) * a.kv_heads + kvh) * 64;
        mbar_expect_tx(&full[st], 2 * kPageBytes);
        tma_load_2d(st0 + (size_t)st * 2 * kPageBytes, &kmap, 0, y, &full[st]);
        tma_load_2d(st0 + (size_t)st * 2 * kPageBytes + kPageBytes, &vmap, 0, y, &full[st]);
    };
    const int pre = min(P, npages);
    if (threadIdx.x == 0) {
        for (int i = 0; i < P; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], NW);
        }
        for (int i = 0; i < pre; ++i)
            if (pbeg + i < fresh) issue(i);
    }
    pdl_wait();
    pdl_launch();
    trace_.released();
    if (threadIdx.x == 0)
        for (int i = 0; i < pre; ++i)
            if (pbeg + i >= fresh) issue(i);
    // q fragments: a0 = (head gq, dims 16kk + 2tq, +1), a2 = (head gq, dims 16kk + 8 + 2tq, +1); heads >= G are zero
    uint32_t qh[4][2], ql[4][2];
#pragma unroll
    for (int kk = 0; kk < 4; ++kk)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
            float2 v = make_float2(0.f, 0.f);
            if (gq < G) v = __ldcg(reinterpret_cast<const float2*>(a.q + (size_t)z * HD + ((size_t)kvh * G + gq) * D +
                                                                   16 * kk + 8 * hf + 2 * tq));
            uint16_t h0, l0, h1, l1;
            split_bf16(v.x, h0, l0);
            split_bf16(v.y, h1, l1);
            qh[kk][hf] = pack_bf16(h0, h1);
            ql[kk][hf] = pack_bf16(l0, l1);
        }
    __syncthreads();  // barriers initialised

    float m_run = -INFINITY, l_run = 0.0f;
    float o[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int c = 0; c < 4; ++c) o[j][c] = 0.0f;
    const int mi = lane >> 3, r8 = lane & 7;
    bool ok = true;
    for (int pg = 0; pg < npages && ok; ++pg) {
        const int st = pg % P;
        ok = mbar_wait(&full[st], (pg / P) & 1, a.err, 4);
        if (!ok) break;
        const uint32_t sK = smem_addr(st0 + (size_t)st * 2 * kPageBytes), sV = sK + kPageBytes;
        const int r0 = warp * 16;                        // rows of this warp in the page
        const int nrow = min(64, len - (pbeg + pg) * 64);  // valid rows of the page
        if (r0 < nrow) {
            float sf[2][4];
#pragma unroll
            for (int q = 0; q < 2; ++q)
#pragma unroll
                for (int c = 0; c < 4; ++c) sf[q][c] = 0.0f;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                uint32_t b[4];
                ldsm_x4(sK + swz(r0 + (mi >> 1) * 8 + r8, kk * 2 + (mi & 1)), b);
                const uint32_t ah[4] = {qh[kk][0], 0u, qh[kk][1], 0u}, al[4] = {ql[kk][0], 0u, ql[kk][1], 0u};
                mma_bf16(sf[0], ah, b[0], b[1]);
                mma_bf16(sf[1], ah, b[2], b[3]);
                mma_bf16(sf[0], al, b[0], b[1]);
                mma_bf16(sf[1], al, b[2], b[3]);
            }
            const int rr[4] = {r0 + 2 * tq, r0 + 2 * tq + 1, r0 + 8 + 2 * tq, r0 + 9 + 2 * tq};
            const float raw[4] = {sf[0][0], sf[0][1], sf[1][0], sf[1][1]};
            float sc[4], cmax = -INFINITY;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                sc[i] = rr[i] < nrow ? __fmul_rn(raw[i], a.scale) : -INFINITY;
                cmax = fmaxf(cmax, sc[i]);
            }
            cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, 1));
            cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, 2));
            const float mn = fmaxf(m_run, cmax);
            const float alpha = m_run == -INFINITY ? 0.0f : expf(m_run - mn);
            float pv[4], ps = 0.0f;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                pv[i] = rr[i] < nrow ? expf(sc[i] - mn) : 0.0f;
                ps += pv[i];
            }
            ps += __shfl_xor_sync(0xffffffffu, ps, 1);
            ps += __shfl_xor_sync(0xffffffffu, ps, 2);
            l_run = l_run * alpha + ps;
            m_run = mn;
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
                ldsm_x4_trans(sV + swz(r0 + (mi & 1) * 8 + r8, 2 * jp + (mi >> 1)), b);
                mma_bf16(o[2 * jp], ph, b[0], b[1]);
                mma_bf16(o[2 * jp + 1], ph, b[2], b[3]);
                mma_bf16(o[2 * jp], pl, b[0], b[1]);
                mma_bf16(o[2 * jp + 1], pl, b[2], b[3]);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
        // thread 0 refills the stage with page pg + P once all 4 warps have released it
        if (threadIdx.x == 0 && pg + P < npages) {
            ok = mbar_wait(&empty[st], (pg / P) & 1, a.err, 11);
            if (ok) issue(pg + P);
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
    }
    if (gq < G) {
        if (tq == 0) {
            wm[warp][gq] = m_run;
            wl[warp][gq] = l_run;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            wacc[warp][gq][8 * j + 2 * tq] = o[j][0];
            wacc[warp][gq][8 * j + 2 * tq + 1] = o[j][1];
        }
    }
    __syncthreads();
    float* part_acc = a.part_acc + (size_t)z * HD * S;
    float* part_ml = a.part_ml + (size_t)z * a.kv_heads * G * S * 2;
    for (int t = threadIdx.x; t < G * D; t += blockDim.x) {
        const int g = t / D, dim = t - g * D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < NW; ++w) M = fmaxf(M, wm[w][g]);
        float L = 0.0f, A = 0.0f;
#pragma unroll
        for (int w = 0; w < NW; ++w) {
            if (wm[w][g] == -INFINITY) continue;
            const float e = expf(wm[w][g] - M);
            L = fmaf(wl[w][g], e, L);
            A = fmaf(wacc[w][g][dim], e, A);
        }
        if (S == 1) {
            const float ov = A / L;
            const size_t oi = (size_t)z * HD + ((size_t)kvh * G + g) * D + dim;
            a.att_out[oi] = ov;
            if (a.att_hi) {
                uint16_t hi, lo;
                split_bf16(ov, hi, lo);
                a.att_hi[oi] = hi;
                a.att_lo[oi] = lo;
            }
        } else {
            const size_t hs = (size_t)(kvh * G + g) * S + sp;
            part_acc[hs * D + dim] = A;
            if (dim == 0) {
                part_ml[hs * 2] = M;
                part_ml[hs * 2 + 1] = L;
            }
        }
    }
    if (S == 1) return;
    if (!last_block_arrives(a.counters + (size_t)z * a.kv_heads + kvh, (unsigned int)S, &is_last)) return;
    for (int t = threadIdx.x; t < G * D; t += blockDim.x) {
        const int g = t / D, dim = t - g * D;
        const size_t h0 = (size_t)(kvh * G + g) * S;
        float M = -INFINITY;
        for (int q = 0; q < S; ++q) M = fmaxf(M, __ldcg(part_ml + (h0 + q) * 2));
        float den = 0.0f, num = 0.0f;
        for (int q = 0; q < S; ++q) {
            const float ms = __ldcg(part_ml + (h0 + q) * 2);
            if (ms == -INFINITY) continue;
            const float e = expf(ms - M);
            den = fmaf(__ldcg(part_ml + (h0 + q) * 2 + 1), e, den);
            num = fmaf(__ldcg(part_acc + (h0 + q) * D + dim), e, num);
        }
        const float ov = num / den;
        const size_t oi = (size_t)z * HD + ((size_t)kvh * G + g) * D + dim;
        a.att_out[oi] = ov;
        if (a.att_hi) {
            uint16_t hi, lo;
            split_bf16(ov, hi, lo);
            a.att_hi[oi] = hi;
            a.att_lo[oi] = lo;
        }
    }
}

// ---- launchers: every batched kernel waits for its predecessor with griddepcontrol.wait first, so all launch with
// programmatic dependent launch (the next kernel's launch overlaps the tail of the current one) -------------------
template <typename Kern>
cudaError_t set_smem(Kern k, size_t bytes) {
    return cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

template <typename Kern, typename... Args>
cudaError_t launch_pdl(Kern kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

cudaError_t make_kv_box_map(CUtensorMap* map, const void* pool, uint64_t rows) {
    return make_tile_map(map, pool, rows, kHeadDim, 8);
}

cudaError_t make_kv_map(CUtensorMap* map, const void* pool, uint64_t rows) {
    // K or V pool of one layer as [pages * kv_heads * 64 rows][64 dims] bf16: the same 64 x 64 box as the weights
    return make_weight_map(map, pool, rows, kHeadDim);
}

cudaError_t launch_battention_tc(const BAttnArgs& a, const CUtensorMap* kmap, const CUtensorMap* vmap, cudaStream_t s) {
    if (a.kv_f32 || a.n < 1 || !kmap || !vmap || a.S < 1 || a.S > kBAttnMaxSplits) return cudaErrorInvalidValue;
    const size_t smem = (size_t)kAttnStages * 2 * kPageBytes + 1024;
    const dim3 grid(a.S, a.kv_heads, a.n), block(128);
#define LASTRO_BATTN_TC(GV)                                                                    \
    case GV: {                                                                                 \
        cudaError_t e = set_smem(battn_tc_kernel<GV>, smem);                                   \
        return e != cudaSuccess ? e : launch_pdl(battn_tc_kernel<GV>, grid, block, smem, s, *kmap, *vmap, a); \
    }
    switch (a.G) {
        LASTRO_BATTN_TC(1)
        LASTRO_BATTN_TC(2)
        LASTRO_BATTN_TC(3)
        LASTRO_BATTN_TC(4)
        LASTRO_BATTN_TC(6)
        LASTRO_BATTN_TC(8)
    default: return cudaErrorInvalidValue;
    }
#undef LASTRO_BATTN_TC
}

cudaError_t launch_bgemm(const BGemmArgs& a, int epi, int groups, cudaStream_t s, const CUtensorMap* wmap) {
    if (a.K % kBK || a.k_split % kBK || a.k_split <= 0 || a.ldx % 8 || groups < 1) return cudaErrorInvalidValue;
    const int ks = (a.K + a.k_split - 1) / a.k_split;
    cudaError_t e;
    if (a.tc == 2) {
        if (!wmap) return cudaErrorInvalidValue;
        const size_t smem = kBGemmSmem + 1024;                                       // token tiles of 64, 3 stages
        const dim3 block(128);
        if (epi == BEPI_SWIGLU) {
            if (a.I % 64 || a.rows != 2 * a.I || ks != 1) return cudaErrorInvalidValue;
            if ((e = set_smem(bgemm_ws_kernel<BEPI_SWIGLU, 64>, smem)) != cudaSuccess) return e;
            return launch_pdl(bgemm_ws_kernel<BEPI_SWIGLU, 64>, dim3(a.I / 64, groups, 1), block, smem, s, *wmap, a);
        }
        if (epi == BEPI_RETURN) {
            if (a.rows % kBRows || ks != 1 || a.x.world > 32) return cudaErrorInvalidValue;
            if ((e = set_smem(bgemm_ws_kernel<BEPI_RETURN, 64>, smem)) != cudaSuccess) return e;
            return launch_pdl(bgemm_ws_kernel<BEPI_RETURN, 64>, dim3(a.rows / kBRows, groups, 1), block, smem, s, *wmap, a);
        }
        if ((e = set_smem(bgemm_ws_kernel<BEPI_STORE, 64>, smem)) != cudaSuccess) return e;
        return launch_pdl(bgemm_ws_kernel<BEPI_STORE, 64>, dim3((a.rows + kBRows - 1) / kBRows, groups, ks), block, smem,
                          s, *wmap, a);
    }
    if (a.tc) {
        const size_t smem = kBGemmSmem + 1024;
        const dim3 block(128);
        if (epi == BEPI_SWIGLU) {
            if (a.I % 64 || a.rows != 2 * a.I || ks != 1) return cudaErrorInvalidValue;
            if ((e = set_smem(bgemm_tc_kernel<BEPI_SWIGLU>, smem)) != cudaSuccess) return e;
            return launch_pdl(bgemm_tc_kernel<BEPI_SWIGLU>, dim3(a.I / 64, groups, 1), block, smem, s, a);
        }
        if (epi == BEPI_RETURN) {
            if (a.rows % kBRows || ks != 1 || a.x.world > 32) return cudaErrorInvalidValue;
            if ((e = set_smem(bgemm_tc_kernel<BEPI_RETURN>, smem)) != cudaSuccess) return e;
            return launch_pdl(bgemm_tc_kernel<BEPI_RETURN>, dim3(a.rows / kBRows, groups, 1), block, smem, s, a);
        }
        if ((e = set_smem(bgemm_tc_kernel<BEPI_STORE>, smem)) != cudaSuccess) return e;
        return launch_pdl(bgemm_tc_kernel<BEPI_STORE>, dim3((a.rows + kBRows - 1) / kBRows, groups, ks), block, smem, s,
                          a);
    }
    if (epi == BEPI_SWIGLU) {
        if (a.I % 64 || a.rows != 2 * a.I || ks != 1) return cudaErrorInvalidValue;
        e = set_smem(bgemm_kernel<BEPI_SWIGLU>, kBGemmSmem);
        if (e != cudaSuccess) return e;
        e = launch_pdl(bgemm_kernel<BEPI_SWIGLU>, dim3(a.I / 64, groups, 1), dim3(128), kBGemmSmem, s, a);
        if (e != cudaSuccess) return e;
    } else if (epi == BEPI_RETURN) {
        if (a.rows % kBRows || ks != 1 || a.x.world > 32) return cudaErrorInvalidValue;
        e = set_smem(bgemm_kernel<BEPI_RETURN>, kBGemmSmem);
        if (e != cudaSuccess) return e;
        e = launch_pdl(bgemm_kernel<BEPI_RETURN>, dim3(a.rows / kBRows, groups, 1), dim3(128), kBGemmSmem, s, a);
        if (e != cudaSuccess) return e;
    } else {
        e = set_smem(bgemm_kernel<BEPI_STORE>, kBGemmSmem);
        if (e != cudaSuccess) return e;
        e = launch_pdl(bgemm_kernel<BEPI_STORE>, dim3((a.rows + kBRows - 1) / kBRows, groups, ks), dim3(128), kBGemmSmem,
                       s, a);
        if (e != cudaSuccess) return e;
    }
    return cudaGetLastError();
}

size_t battn_smem(int cap, int kv_f32) { return (size_t)2 * cap * kHeadDim * (kv_f32 ? 4 : 2); }

cudaError_t launch_battention(const BAttnArgs& a, cudaStream_t s) {
    if (a.S < 1 || a.S > kBAttnMaxSplits || a.cap < 1 || a.n < 1) return cudaErrorInvalidValue;
    const size_t smem = battn_smem(a.cap, a.kv_f32);
    if (smem > kMaxSmemBytes) return cudaErrorInvalidValue;
    const dim3 grid(a.S, a.kv_heads, a.n), block(128);
#define LASTRO_BATTN_G(GV)                                                                     \
    case GV: {                                                                                 \
        auto k = a.kv_f32 ? battn_kernel<true, GV> : battn_kernel<false, GV>;                  \
        cudaError_t e = set_smem(k, smem);                                                     \
        return e != cudaSuccess ? e : launch_pdl(k, grid, block, smem, s, a);                  \
    }
    switch (a.G) {
        LASTRO_BATTN_G(1)
        LASTRO_BATTN_G(2)
        LASTRO_BATTN_G(3)
        LASTRO_BATTN_G(4)
        LASTRO_BATTN_G(6)
        LASTRO_BATTN_G(8)
    default: return cudaErrorInvalidValue;
    }
#undef LASTRO_BATTN_G
}

cudaError_t launch_battn_norm(const BNormArgs& a, int n, cudaStream_t s) {
    if (a.H % 4 || a.H > 2048 || n < 1) return cudaErrorInvalidValue;
    return launch_pdl(battn_norm_kernel, dim3(n), dim3(256), 0, s, a);
}

cudaError_t launch_brope_kv(const BRopeArgs& a, cudaStream_t s) {
    if (a.n < 1 || a.ks > 16) return cudaErrorInvalidValue;
    return launch_pdl(brope_kv_kernel, dim3(a.n, (a.qd + 2 * a.kvd + 255) / 256), dim3(128), 0, s, a);
}

cudaError_t launch_brouter(const BRouterArgs& a, cudaStream_t s) {
    if (a.x.world * a.x.lay.cap > kBMaxSlots || a.x.experts_per_rank > kMaxExperts) return cudaErrorInvalidValue;
    if (a.ks > 16 || a.H % 8 || a.H > 2048 || a.E > kMaxExperts || a.k > kMaxTopK || a.n < 1) return cudaErrorInvalidValue;
    return launch_pdl(brouter_kernel, dim3(a.n), dim3(256), sizeof(float) * a.H, s, a);
}

cudaError_t launch_ep_combine(const BExchangeArgs& a, cudaStream_t s) {
    if (a.H > 2048) return cudaErrorInvalidValue;
    return launch_pdl(ep_combine_kernel, dim3(a.n), dim3(256), 0, s, a);
}

cudaError_t launch_bargmax(const BHeadArgs& a, cudaStream_t s) {
    return launch_pdl(bargmax_kernel, dim3(a.n), dim3(1024), 0, s, a);
}

}  // namespace lastro
