// LoRA pre-pass xa = x @ A for the fused LoRA delta of the q6 linear.
//
// The reference's LoRA-additive linear computes y = q6(x) + s * ((x @ A) @ B)
// (dense_img_ff_window.py:48-60).  The tensor-core q6 kernel accumulates
// s * (xa @ B) into its own tile; this kernel produces xa = x @ A, a bf16
// [M, K] x [K, r] product with fp32 accumulation and one bf16 rounding, r a
// multiple of 32 up to 256.  With r far below the ridge point (r FLOP per
// byte of x) the product is bound by reading x once from HBM, so it is a
// plain warp-level MMA kernel (mma.sync m16n8k16) built for memory-level
// parallelism: each CTA owns 16 token rows (one MMA row tile) and every rank
// column, its four warps split the rank columns (r / 4 each), and K streams
// through a cp.async ring of 64-wide chunks about 150 KB deep (12 stages at
// rank 64, 4 at rank 256), so that a CTA keeps over 100 KB in flight: each
// CTA re-reads all of A (K x r, 384 KB at K = 3072, r = 64) from L2 besides
// its 96 KB of x, and with one CTA per SM the ring depth sets its bandwidth
// (M = 3456 runs 216 CTAs).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>

#include "q6_internal.h"
#include "q6_ptx.cuh"

namespace q6 {
namespace {

constexpr int kRowsPerCta = 16;
constexpr int kBK = 64;                    // K per chunk: four K = 16 MMA steps
constexpr int kXStride = kBK + 8;          // bf16 per shared x row (16 bytes of padding: no bank conflicts)
constexpr int kThreads = 128;
constexpr int kRingBytes = 150 * 1024;     // target ring depth in bytes

template <int R>
struct LoraCfg {
    static constexpr int kAStride = R + 8;  // bf16 per shared A row (16 bytes of padding)
    static constexpr int kXBytes = kRowsPerCta * kXStride * 2;
    static constexpr int kABytes = kBK * kAStride * 2;
    static constexpr int kStageBytes = kXBytes + kABytes;
    static constexpr int kStages =
        kRingBytes / kStageBytes < 3 ? 3 : (kRingBytes / kStageBytes > 12 ? 12 : kRingBytes / kStageBytes);
    static constexpr int kSmemBytes = kStages * kStageBytes;
    static_assert(kXBytes % 16 == 0 && kStageBytes % 16 == 0, "16-byte aligned stage slices");
    static_assert(kSmemBytes <= 227 * 1024, "shared memory");
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
    const int n = valid ? 16 : 0;  // zero-fill rows past M and columns past K
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x2_trans(uint32_t addr, uint32_t (&r)[2]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0, %1}, [%2];"
                 : "=r"(r[0]), "=r"(r[1])
                 : "r"(addr));
}
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// R = rank (compile-time, multiple of 32, <= 256).
template <int R>
__global__ void __launch_bounds__(kThreads) lora_xa_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ a,
                                                          uint16_t* __restrict__ xa, int64_t M, int64_t K) {
    using C = LoraCfg<R>;
    constexpr int kCols = R / 4;           // columns per warp
    constexpr int kTiles = kCols / 8;      // n8 tiles per warp
    extern __shared__ __align__(16) uint8_t lora_smem[];

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int64_t m0 = static_cast<int64_t>(blockIdx.x) * kRowsPerCta;
    const int chunks = static_cast<int>((K + kBK - 1) / kBK);
    auto xs = [&](int s) { return reinterpret_cast<uint16_t*>(lora_smem + s * C::kStageBytes); };
    auto as = [&](int s) { return reinterpret_cast<uint16_t*>(lora_smem + s * C::kStageBytes + C::kXBytes); };

    pdl_launch_dependents();
    pdl_wait();  // x may be the previous kernel's output

    constexpr int kStages = C::kStages;
    auto load_chunk = [&](int c) {
        const int s = c % kStages;
        const int64_t k0 = static_cast<int64_t>(c) * kBK;
        // x: 16 rows x 64 bf16 = 8 x 16-byte pieces per row
        for (int i = tid; i < kRowsPerCta * 8; i += kThreads) {
            const int row = i >> 3, piece = i & 7;
            const int64_t gm = m0 + row, gk = k0 + piece * 8;
            const bool ok = gm < M && gk < K;
            cp_async16(smem_u32(xs(s) + row * kXStride + piece * 8), ok ? x + gm * K + gk : x, ok);
        }
        // A: 64 rows of K x R bf16 = R / 8 pieces per row
        for (int i = tid; i < kBK * (R / 8); i += kThreads) {
            const int row = i / (R / 8), piece = i % (R / 8);
            const int64_t gk = k0 + row;
            const bool ok = gk < K;
            cp_async16(smem_u32(as(s) + row * C::kAStride + piece * 8), ok ? a + gk * R + piece * 8 : a, ok);
        }
    };

    float acc[kTiles][4];
#pragma unroll
    for (int t = 0; t < kTiles; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.0f;

    // Prologue: chunks 0 .. kStages - 2 in flight (one commit group each; a
    // group past the last chunk is empty, which keeps the wait counts uniform).
    for (int c = 0; c < kStages - 1; ++c) {
        if (c < chunks) load_chunk(c);
        cp_async_commit();
    }
    for (int c = 0; c < chunks; ++c) {
        cp_async_wait<kStages - 2>();  // this thread's copies of chunk c have landed
        __syncthreads();               // ... and everyone's; the slot of chunk c - 1 is free again
        if (c + kStages - 1 < chunks) load_chunk(c + kStages - 1);
        cp_async_commit();
        const uint16_t* xt = xs(c % kStages);
        const uint16_t* at = as(c % kStages);
#pragma unroll
        for (int ks = 0; ks < kBK / 16; ++ks) {
            // A operand: the 16 rows, K columns 16 ks .. +15 of the x chunk.
            uint32_t af[4];
            ldmatrix_x4(smem_u32(xt + (lane & 15) * kXStride + 16 * ks + 8 * (lane >> 4)), af);
#pragma unroll
            for (int t = 0; t < kTiles; ++t) {
                // B operand: K rows 16 ks .. +15 (row-major [k][n] in shared memory,
                // transposed by ldmatrix), n columns warp r/4 + 8 t .. +7.
                uint32_t bf[2];
                ldmatrix_x2_trans(smem_u32(at + (16 * ks + (lane & 15)) * C::kAStride + kCols * warp + 8 * t), bf);
                mma_bf16_16816(acc[t], af, bf);
            }
        }
    }
    cp_async_wait<0>();

    // Accumulator layout: thread holds rows g, g + 8 (g = lane / 4) and
    // columns 2 (lane % 4), +1 of each n8 tile.
    const int g = lane >> 2;
    const int cq = 2 * (lane & 3);
#pragma unroll
    for (int t = 0; t < kTiles; ++t) {
        const int col = kCols * warp + 8 * t + cq;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int64_t row = m0 + g + 8 * h;
            if (row < M) {
                const __nv_bfloat162 v = __floats2bfloat162_rn(acc[t][2 * h], acc[t][2 * h + 1]);
                *reinterpret_cast<__nv_bfloat162*>(xa + row * R + col) = v;
            }
        }
    }
}

template <int R>
int launch_r(const uint16_t* x, const uint16_t* a, uint16_t* xa, int64_t M, int64_t K, cudaStream_t stream) {
    using C = LoraCfg<R>;
    static std::atomic<bool> attr_set_for_device[kMaxDevices];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return Q6_ERR_CUDA;
    if (dev < 0 || dev >= kMaxDevices) return Q6_ERR_UNSUPPORTED;
    if (!attr_set_for_device[dev].load(std::memory_order_acquire)) {
        if (cudaFuncSetAttribute(lora_xa_kernel<R>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes) !=
            cudaSuccess)
            return Q6_ERR_CUDA;
        attr_set_for_device[dev].store(true, std::memory_order_release);
    }
    const int64_t blocks = (M + kRowsPerCta - 1) / kRowsPerCta;
    if (blocks > 0x7fffffff) return Q6_ERR_UNSUPPORTED;
    const cudaError_t e = launch_pdl(lora_xa_kernel<R>, dim3(static_cast<unsigned>(blocks)), dim3(kThreads),
                                     C::kSmemBytes, stream, x, a, xa, M, K);
    return e == cudaSuccess ? Q6_OK : Q6_ERR_CUDA;
}

}  // namespace

int launch_lora_xa(const uint16_t* x, const uint16_t* a, uint16_t* xa, int64_t M, int64_t K, int r,
                   cudaStream_t stream) {
    switch (r) {
        case 32: return launch_r<32>(x, a, xa, M, K, stream);
        case 64: return launch_r<64>(x, a, xa, M, K, stream);
        case 96: return launch_r<96>(x, a, xa, M, K, stream);
        case 128: return launch_r<128>(x, a, xa, M, K, stream);
        case 160: return launch_r<160>(x, a, xa, M, K, stream);
        case 192: return launch_r<192>(x, a, xa, M, K, stream);
        case 224: return launch_r<224>(x, a, xa, M, K, stream);
        case 256: return launch_r<256>(x, a, xa, M, K, stream);
        default: return Q6_ERR_SHAPE;
    }
}

}  // namespace q6
