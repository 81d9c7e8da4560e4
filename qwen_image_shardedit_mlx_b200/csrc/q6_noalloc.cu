// q6_mlp_bf16_noalloc: the image feed-forward MLP for callers that cannot
// allocate device memory.
//
// q6_mlp_bf16 needs a caller-provided workspace for the bf16 hidden
// activations between fc1 and fc2.  Some callers have no way to obtain one:
// plugin hosts and FFI bindings that only receive raw input/output pointers
// and own no allocator, serving loops that forbid cudaMalloc because it can
// synchronise the device, and runtimes whose memory is fully carved up by
// their own pool.  This entry point keeps the hidden activations in a
// library-owned, file-scope device array instead, so the call itself never
// allocates.
//
// The array is a fixed 32 MiB per GPU (static, so every GPU that loads the
// library holds it until the process exits).  It fits M * H * 2 bytes of bf16
// hidden activations: up to 1365 tokens at H = 12288.  Larger problems are
// rejected with Q6_ERR_WORKSPACE before anything is launched.
//
// All calls on a device share the one array and it keeps the previous call's
// contents; nothing in it has to start at zero because fc1 overwrites every
// hidden element the call later reads.  Two calls whose GPU work overlaps (on
// different streams, or from different host threads without ordering) race on
// the array and produce wrong results; order them on one stream.
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

#include "q6_b200.h"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;

// Device-side storage.  In host code this name is only a handle for
// cudaGetSymbolAddress, never a device address.
static __device__ __align__(256) unsigned char g_noalloc_hidden[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_hidden_addr[kMaxDevices] = {};
void* g_hidden_ctx[kMaxDevices] = {};  // the context the cached address belongs to

using CtxGetCurrentFn = CUresult (*)(CUcontext*);

CtxGetCurrentFn ctx_get_current() {
    static CtxGetCurrentFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<CtxGetCurrentFn>(ptr);
    });
    return fn;
}

// Device address of g_noalloc_hidden on the current device.  It is looked up
// once per device and context with cudaGetSymbolAddress (the first call on a
// device does this set-up; make that first call before any stream capture)
// and looked up again when the device's context changes (after a
// cudaDeviceReset the module, and with it the array, is loaded anew).
int hidden_address(void** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return Q6_ERR_CUDA;
    if (dev < 0 || dev >= kMaxDevices) return Q6_ERR_UNSUPPORTED;
    // Binding the (already current) device again makes the runtime initialise
    // its primary context on this thread, so that the driver reports it as current.
    if (cudaSetDevice(dev) != cudaSuccess) return Q6_ERR_CUDA;
    CUcontext ctx = nullptr;
    const CtxGetCurrentFn get = ctx_get_current();
    if (!get || get(&ctx) != CUDA_SUCCESS) return Q6_ERR_CUDA;
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_hidden_addr[dev] == nullptr || g_hidden_ctx[dev] != static_cast<void*>(ctx)) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_hidden) != cudaSuccess || p == nullptr) return Q6_ERR_CUDA;
        g_hidden_addr[dev] = p;
        g_hidden_ctx[dev] = static_cast<void*>(ctx);
    }
    *out = g_hidden_addr[dev];
    return Q6_OK;
}

}  // namespace

extern "C" int q6_mlp_bf16_noalloc(const uint16_t* x, const uint32_t* w1, const uint16_t* scales1,
                                   const uint16_t* qbiases1, const uint16_t* bias1, const uint32_t* w2,
                                   const uint16_t* scales2, const uint16_t* qbiases2, const uint16_t* bias2,
                                   const uint16_t* residual, const uint16_t* gate, uint16_t* y, int64_t M,
                                   int64_t D, int64_t H, int group_size, q6_stream_t stream) {
    if (M <= 0 || H <= 0 || D <= 0) return Q6_ERR_INVALID_ARGUMENT;
    if (static_cast<double>(M) * static_cast<double>(H) * 2.0 > static_cast<double>(kNoAllocScratchBytes))
        return Q6_ERR_WORKSPACE;
    void* hidden = nullptr;
    const int st = hidden_address(&hidden);
    if (st != Q6_OK) return st;
    return q6_mlp_bf16(x, w1, scales1, qbiases1, bias1, w2, scales2, qbiases2, bias2, residual, gate, y, M, D, H,
                       group_size, hidden, kNoAllocScratchBytes, stream);
}
