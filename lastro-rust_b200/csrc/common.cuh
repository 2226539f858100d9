// Shared device helpers of the lastro-b200 kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "kernels.h"  // kTraceMaxCtas

#define LDEV __device__ __forceinline__

namespace lastro {

constexpr int kWarp = 32;

// ---- programmatic dependent launch (PDL) -----------------------------------------------------------------------
// Every kernel of the decode chain reads only immutable weights before pdl_wait(); activations written by the
// previous kernel are read, and any buffer is written, only after it.  griddepcontrol.wait returns once the
// preceding grid has completed and its memory is visible; launch_dependents lets the next kernel of the stream be
// scheduled early so that its weight loads overlap this kernel.
LDEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
LDEV void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---- in-graph timeline (lastro_model_trace) -----------------------------------------------------------------------
// With a non-null trace base, every CTA of a launch stamps the global timer (ns) into its own kTraceWords words: [0]
// when thread 0 starts, [1] when thread 0 passes griddepcontrol.wait, [2] the latest exit of any warp (atomicMax by
// lane 0 of each warp; the destructor runs on every return path), [3..] the kernel's own milestones (mark).  The host
// reduces over CTAs: min start, min release, max end.  A null base (the product path) costs one predicated branch per
// stamp.  The stamps are kept this lean on purpose: a memory clobber on the timer read (which pins a stamp between
// the loads and stores around it) and stamps of the SM id and clock cost the product path 0.9 % on C3 through the
// code they leave in every kernel; a stamp may therefore land a little before or after the work around it.
LDEV unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

struct CtaTrace {
    unsigned long long* p;
    LDEV explicit CtaTrace(unsigned long long* base) : p(nullptr) {
        const unsigned cta = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
        if (base && cta < (unsigned)kTraceMaxCtas) p = base + kTraceWords * (size_t)cta;
        if (p && threadIdx.x == 0) p[0] = global_ns();
    }
    LDEV void released() const {
        if (p && threadIdx.x == 0) p[1] = global_ns();
    }
    // a kernel's own milestone i (< kTraceMarks) as thread `tid` reaches it (diagnostics of the phases inside a launch)
    LDEV void mark(int i, unsigned tid = 0) const {
        if (p && threadIdx.x == tid) p[3 + i] = global_ns();
    }
    // the same, stamped only once `v` (a value the phase produced) is available: the branch on it orders the timer
    // read after the load or arithmetic that yields v
    LDEV void mark_after(int i, float v, unsigned tid = 0) const {
        if (p && threadIdx.x == tid && __float_as_uint(v) != 0xffffffffu) p[3 + i] = global_ns();
    }
    LDEV ~CtaTrace() {
        if (p && (threadIdx.x & 31) == 0) atomicMax(p + 2, global_ns());
    }
};

// ---- loads ------------------------------------------------------------------------------------------------------
// 16-byte weight load, read once per step: non-coherent path, no L1 allocation.
LDEV uint4 ld_weight(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

// Load of data written by another CTA of the same grid (after a fence/ticket): bypass L1.
LDEV float ld_cg(const float* p) { return __ldcg(p); }
LDEV int ld_cg(const int* p) { return __ldcg(p); }

// ---- bf16 -------------------------------------------------------------------------------------------------------
LDEV float bf_lo(uint32_t u) { return __uint_as_float(u << 16); }
LDEV float bf_hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }

// sum_{i<8} w[i] * x[i] for 8 bf16 weights packed in a uint4 and 8 f32 activations
LDEV float dot8(uint4 w, float4 xa, float4 xb, float acc) {
    acc = fmaf(bf_lo(w.x), xa.x, acc);
    acc = fmaf(bf_hi(w.x), xa.y, acc);
    acc = fmaf(bf_lo(w.y), xa.z, acc);
    acc = fmaf(bf_hi(w.y), xa.w, acc);
    acc = fmaf(bf_lo(w.z), xb.x, acc);
    acc = fmaf(bf_hi(w.z), xb.y, acc);
    acc = fmaf(bf_lo(w.w), xb.z, acc);
    acc = fmaf(bf_hi(w.w), xb.w, acc);
    return acc;
}

LDEV uint16_t f32_to_bf16_rne(float f) {
    uint32_t u = __float_as_uint(f);
    if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x7fffffu)) return (uint16_t)((u >> 16) | 0x40);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

// ---- reductions ---------------------------------------------------------------------------------------------------
LDEV float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

LDEV float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Key that orders floats like Rust's f32::total_cmp when compared as signed integers.
LDEV int32_t total_key(float f) {
    int32_t x = __float_as_int(f);
    return x ^ (int32_t)(((uint32_t)(x >> 31)) >> 1);
}

// Block-wide sum; `red` holds >= blockDim.x/32 floats.  All threads get the result.
LDEV float block_sum(float v, float* red) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[wid] = v;
    __syncthreads();
    float t = 0.0f;
    for (int i = 0; i < nw; ++i) t += red[i];
    return t;
}

// Last-CTA election: every CTA calls this once after writing its results; returns true in exactly one CTA (the
// last to arrive), which may then read every other CTA's results.  The counter is reset for the next launch.
LDEV bool last_block_arrives(unsigned int* counter, unsigned int total, bool* flag_smem) {
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned int t = atomicAdd(counter, 1u);
        bool last = (t == total - 1);
        if (last) atomicExch(counter, 0u);
        *flag_smem = last;
    }
    __syncthreads();
    bool last = *flag_smem;
    if (last) __threadfence();
    return last;
}

// ---- warp-level tensor-core tiles (mma.sync m16n8k16, bf16 operands, f32 accumulators) ------------------------
LDEV void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
LDEV void ldsm_x4_trans(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
// d += a (16x16, row) * b (16x8, col), bf16 operands, f32 accumulators
LDEV void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// shared tiles are rows of 64 bf16 (128 bytes = 8 chunks of 16 bytes); chunk c of row r sits at c ^ (r & 7) so that
// the 8 rows one ldmatrix phase reads fall in 8 different bank groups (the 128-byte TMA swizzle of 1024-byte
// aligned boxes)
LDEV uint32_t swz(int row, int chunk) { return (uint32_t)(row * 128 + ((chunk ^ (row & 7)) << 4)); }
LDEV uint32_t pack_bf16(uint16_t lo, uint16_t hi) { return (uint32_t)lo | ((uint32_t)hi << 16); }
// v = hi + lo with both bf16: an f32 operand of a bf16 product kept to a relative 2^-17
LDEV void split_bf16(float v, uint16_t& hi, uint16_t& lo) {
    hi = f32_to_bf16_rne(v);
    lo = f32_to_bf16_rne(__fsub_rn(v, __uint_as_float((uint32_t)hi << 16)));
}

// ---- flags written by another CTA of this GPU --------------------------------------------------------------------
LDEV unsigned int ld_acquire_gpu(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
LDEV void st_release_gpu(unsigned int* p, unsigned int v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// ---- bulk (TMA) copies global -> shared, completed on an mbarrier ----------------------------------------------
LDEV uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// thread 0 only, before any copy targets the barrier; the CTA synchronizes before other threads wait on it
LDEV void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

LDEV void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}

// one box of a 2-D tensor map (x innermost, a multiple of 16 bytes) into shared memory, completing on `bar`
LDEV void tma_load_2d(void* dst, const void* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

// `bytes` and both addresses must be multiples of 16
LDEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_addr(dst)),
                 "l"(src), "r"(bytes), "r"(smem_addr(bar))
                 : "memory");
}

// hint: bring [src, src + bytes) into L2 (16-byte aligned address, size a multiple of 16); no completion to wait for
LDEV void bulk_prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// this CTA's share (of `ctas`, in 16-byte multiples) of an L2 prefetch of [base, base + bytes)
LDEV void prefetch_share_l2(const void* base, unsigned long long bytes, int cta, int ctas) {
    if (!base || bytes == 0) return;
    const unsigned long long share = ((bytes + ctas - 1) / ctas + 15) & ~15ull;
    const unsigned long long off = (unsigned long long)cta * share;
    if (off >= bytes) return;
    const unsigned long long n = min(share, bytes - off);
    bulk_prefetch_l2(static_cast<const unsigned char*>(base) + off, (uint32_t)n);
}

LDEV bool mbar_try_wait(uint64_t* bar, uint32_t phase) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(phase)
        : "memory");
    return ok != 0;
}

// Bounded wait: each try_wait suspends for a hardware-chosen interval; after the iteration limit the wait gives up,
// records `code` in the error word (the host reports it and poisons the object) and returns false.
constexpr uint32_t kWaitLimit = 1u << 22;
LDEV bool mbar_wait(uint64_t* bar, uint32_t phase, int* err, int code) {
    for (uint32_t i = 0; i < kWaitLimit; ++i)
        if (mbar_try_wait(bar, phase)) return true;
    if (err) atomicExch(err, code);
    return false;
}

}  // namespace lastro
