// Allocation-free MoE block forward: lastro_moe_block_forward_noalloc.
//
// Some callers cannot call cudaMalloc: a host runtime whose device memory is owned by another allocator (a Rust
// runtime handing out borrowed buffers, an inference server with a pooled arena), code that runs inside a stream
// capture, or a latency-critical path where cudaMalloc's implicit synchronisation is not acceptable.  They pass
// every input and output buffer themselves; the only other memory this entry point touches is the scratch below, a
// file-scope __device__ array that every GPU loading the library holds until the process exits.
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/lastro_b200.h"
#include "kernels.h"

using namespace lastro;

namespace {

constexpr int kNoAllocMaxExperts = 64;
constexpr int kNoAllocMaxActivations = 16384;  // k * I floats: 64 KB

// Scratch of one call: router logits, the router's last-CTA ticket, the bounded-wait error word and the SwiGLU
// activations between the two expert kernels.  About 66 KB per device.
struct NoAllocScratch {
    float logits[kNoAllocMaxExperts];
    unsigned int counter;  // cleared by every call
    int err;               // cleared by every call
    int pad[14];
    alignas(16) float a[kNoAllocMaxActivations];
};

static __device__ __align__(256) NoAllocScratch g_noalloc_scratch;

// The host name g_noalloc_scratch is only a stand-in for the symbol, not a device address: the address is looked
// up with the device current and cached per device, together with the CUDA context it was looked up in.  A device
// reset (or a primary context torn down and re-created) loads the module again at another address; the context
// changes with it, so the next call looks the address up again instead of using a stale one.
constexpr int kMaxDevices = 64;
struct ScratchAddr {
    NoAllocScratch* p = nullptr;
    CUcontext ctx = nullptr;
};
ScratchAddr g_scratch_addr[kMaxDevices];
std::mutex g_scratch_mu;

// cuCtxGetCurrent through the runtime's driver entry point (the library links only the runtime)
CUcontext current_context() {
    using GetCurrent = CUresult (*)(CUcontext*);
    static GetCurrent fn = nullptr;
    if (!fn) {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess || !f) {
            cudaGetLastError();
            return nullptr;
        }
        fn = reinterpret_cast<GetCurrent>(f);
    }
    CUcontext c = nullptr;
    return fn(&c) == CUDA_SUCCESS ? c : nullptr;
}

int scratch_for_current_device(NoAllocScratch** out) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        cudaGetLastError();
        return LASTRO_E_CUDA;
    }
    const CUcontext ctx = current_context();
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    ScratchAddr& a = g_scratch_addr[dev];
    if (!a.p || !ctx || a.ctx != ctx) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) {
            cudaGetLastError();
            return LASTRO_E_CUDA;
        }
        a.p = static_cast<NoAllocScratch*>(p);
        a.ctx = current_context();  // the runtime may only now have made the primary context current
    }
    *out = a.p;
    return LASTRO_OK;
}

int launch_failed() {
    cudaGetLastError();  // clear a non-sticky launch error so the caller's next CUDA call does not inherit it
    return LASTRO_E_CUDA;
}

}  // namespace

extern "C" int lastro_moe_block_forward_noalloc(const float* x, const uint16_t* router, const uint16_t* gate_up,
                                                const uint16_t* down, int32_t experts, int32_t hidden, int32_t inter,
                                                int32_t k, float* y, int32_t* ids, float* weights, void* stream) {
    if (!x || !router || !gate_up || !down || !y || !ids || !weights) return LASTRO_E_ARG;
    if (experts < 1 || hidden < 8 || inter < 8 || k < 1 || k > experts) return LASTRO_E_ARG;
    if (hidden % 8 || inter % 8 || hidden > kMaxHidden || inter > kMaxInter || experts > kNoAllocMaxExperts ||
        k > kMaxTopK || (int64_t)k * inter > kNoAllocMaxActivations || inter % gate_up_rows_per_cta() ||
        hidden % down_rows_per_cta() || down_smem(hidden, inter, k) > kMaxSmemBytes ||
        gate_up_smem(hidden) > kMaxSmemBytes)
        return LASTRO_E_UNSUPPORTED;
    NoAllocScratch* sc = nullptr;
    int rc = scratch_for_current_device(&sc);
    if (rc) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // the ticket and the error word must start at zero; the rest is fully overwritten
    if (cudaMemsetAsync(&sc->counter, 0, 2 * sizeof(int), s) != cudaSuccess) return launch_failed();

    RouterArgs ra{};
    ra.x = x;
    ra.w = router;
    ra.logits = sc->logits;
    ra.ids = ids;
    ra.weights = weights;
    ra.counter = &sc->counter;
    ra.E = experts;
    ra.H = hidden;
    ra.k = k;
    if (launch_router(ra, s, false) != cudaSuccess) return launch_failed();

    GateUpArgs ga{};
    ga.x = x;
    ga.ids = ids;
    ga.w = gate_up;
    ga.a = sc->a;
    ga.err = &sc->err;
    ga.H = hidden;
    ga.I = inter;
    ga.k = k;
    ga.E = experts;
    if (launch_gate_up(ga, s, true) != cudaSuccess) return launch_failed();

    DownArgs da{};
    da.a = sc->a;
    da.ids = ids;
    da.weights = weights;
    da.w = down;
    da.out = y;
    da.accumulate = 0;
    da.err = &sc->err;
    da.H = hidden;
    da.I = inter;
    da.k = k;
    da.E = experts;
    if (launch_down(da, s, true) != cudaSuccess) return launch_failed();
    return LASTRO_OK;
}

extern "C" int lastro_moe_block_noalloc_status(int32_t* status, void* stream) {
    if (!status) return LASTRO_E_ARG;
    NoAllocScratch* sc = nullptr;
    int rc = scratch_for_current_device(&sc);
    if (rc) return rc;
    // enqueued after the caller's blocks on the same stream: the word the last of them left (0 = every wait completed)
    if (cudaMemcpyAsync(status, &sc->err, sizeof(int), cudaMemcpyDefault, static_cast<cudaStream_t>(stream)) !=
        cudaSuccess)
        return launch_failed();
    return LASTRO_OK;
}
