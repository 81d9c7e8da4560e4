// LoRA pre-pass xa = x @ A for the fused LoRA delta of the q6 linear.
//
// The reference's LoRA-additive linear computes y = q6(x) + s * ((x @ A) @ B)
// (dense_img_ff_window.py:48-60).  The tensor-core q6 kernel accumulates
// s * (xa @ B) into its own tile; this kernel produces xa = x @ A, a bf16
// [M, K] x [K, r] product with fp32 accumulation and one bf16 rounding, r a
// multiple of 32 up to 256.  With r far below the ridge point (r FLOP per
// byte of x) the product is bound by moving bytes, so it is a plain
// warp-level MMA kernel (mma.sync m16n8k16) built around its data movement
// and its latencies.  Each CTA owns 32 token rows (two MMA row tiles) and
// every rank column.  K streams in 64-wide chunks through a ring of TMA stages
// (one CTA per SM, up to 16 stages in flight): one [32 rows x 64] box of x and
// r / 64 [64 x 64] boxes of A with the 128-byte swizzle (a rank that is an odd
// multiple of 32 adds one [64 x 32] box with the 64-byte swizzle), which
// keeps the ldmatrix reads conflict-free.  The eight warps split the chunks,
// not the output: warp (K group kg, column group cg) takes the chunks
// c = kg, kg + G, ... (G K groups) for all 32 rows and its r / (8 / G) rank
// columns, so a warp waits on one chunk in G and keeps 2 x (its n8 tiles)
// independent MMA chains (16 at r = 64).  With every warp on every chunk, a
// chunk cost each warp ~100 dependent instructions at ~10 cycles each, and the
// kernel took chunks x 0.55 us whatever its grid.  At the end the K groups'
// partial sums meet in the drained ring and are added in K-group order.  The
// last warp to release a ring slot refills it, and each CTA starts its K loop
// at a different chunk; every sum runs in a fixed order per CTA.  Every wait
// is bounded.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <mutex>

#include "q6_internal.h"
#include "q6_ptx.cuh"

namespace q6 {
namespace {

constexpr int kRowsPerCta = 32;
constexpr int kRowTiles = kRowsPerCta / 16;    // MMA row tiles per CTA
constexpr int kBK = 64;                        // K per chunk: four K = 16 MMA steps
constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kXBoxBytes = kRowsPerCta * 128;  // [32 rows x 64 bf16], 128-byte swizzled
constexpr int kABoxBytes = kBK * 128;          // [64 k x 64 rank columns], 128-byte swizzled
constexpr int kATailBytes = kBK * 64;          // [64 k x 32 rank columns], 64-byte swizzled
constexpr int kRingBytes = 200 * 1024;         // one CTA per SM

template <int R>
struct LoraCfg {
    static constexpr int kABoxes = R / 64;          // full 64-column boxes
    static constexpr bool kTail = R % 64 != 0;      // one 32-column box
    static constexpr int kStageBytes = kXBoxBytes + kABoxes * kABoxBytes + (kTail ? kATailBytes : 0);
    static constexpr int kStages = kRingBytes / kStageBytes < 2 ? 2 : (kRingBytes / kStageBytes > 16 ? 16
                                                                                                  : kRingBytes / kStageBytes);
    static constexpr int kSmemBytes = kStages * kStageBytes + 1024 /* alignment */;
    // Column groups: the fewest (1, 2 or 4) that leave a warp at most eight n8 tiles.
    static constexpr int kColGroups = R / 8 <= 8 ? 1 : (R / 8 <= 16 ? 2 : 4);
    static constexpr int kKGroups = kWarps / kColGroups;
    static constexpr int kTilesW = R / 8 / kColGroups;  // n8 tiles per warp
    static constexpr int kFrag = kRowTiles * kTilesW * 4;  // accumulator floats per lane
    static_assert((R / 8) % kColGroups == 0, "column groups must split the n8 tiles evenly");
    static_assert(kStageBytes % 1024 == 0, "swizzled boxes need 1024-byte alignment");
    static_assert(kSmemBytes <= 227 * 1024, "shared memory");
    static_assert(kWarps * kFrag * 32 * 4 <= kStages * kStageBytes, "partial sums fit the drained ring");
};

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

// Byte offset of 16-byte chunk c of row `row` in a 128-byte-swizzled box
// (128-byte rows: chunk bits 4-6 XOR address bits 7-9) and in a
// 64-byte-swizzled box (64-byte rows: chunk bits 4-5 XOR address bits 7-8).
__device__ __forceinline__ uint32_t swz(int row, int c) { return static_cast<uint32_t>(row * 128 + ((c ^ (row & 7)) << 4)); }
__device__ __forceinline__ uint32_t swz64(int row, int c) {
    return static_cast<uint32_t>(row * 64 + ((c ^ ((row >> 1) & 3)) << 4));
}

// R = rank (compile-time, multiple of 32, <= 256).
template <int R>
__global__ void __launch_bounds__(kThreads) lora_xa_kernel(const __grid_constant__ CUtensorMap tmap_x,
                                                          const __grid_constant__ CUtensorMap tmap_a,
                                                          const __grid_constant__ CUtensorMap tmap_a_tail,
                                                          uint16_t* __restrict__ xa, int64_t M, int64_t K,
                                                          uint32_t x_box_bytes) {
    using C = LoraCfg<R>;
    constexpr int kStages = C::kStages;
    constexpr int kTilesW = C::kTilesW;
    constexpr int kKGroups = C::kKGroups;
    constexpr int kColGroups = C::kColGroups;
    extern __shared__ uint8_t lora_raw[];
    uint8_t* ring = smem_align_up<1024>(lora_raw);
    __shared__ __align__(8) uint64_t full[kStages];
    __shared__ uint32_t released[kStages];
    __shared__ int abort_flag;
    __shared__ int issued_total;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int kg = warp / kColGroups;  // this warp's K group: chunks kg, kg + kKGroups, ...
    const int cg = warp % kColGroups;  // and its rank columns [cg R / kColGroups, +R / kColGroups)
    const int m0 = static_cast<int>(blockIdx.x) * kRowsPerCta;
    const int chunks = static_cast<int>((K + kBK - 1) / kBK);
    const uint32_t tx = x_box_bytes + C::kABoxes * kABoxBytes + (C::kTail ? kATailBytes : 0);
    // Ring position c holds K chunk (c + k_first) mod chunks: the CTAs start at
    // different chunks, so they do not all read the same few kilobytes of A
    // from the same L2 slices at the same moment.
    const int k_first = static_cast<int>((blockIdx.x * 7u) % static_cast<unsigned>(chunks));
    auto kchunk = [&](int c) { return (c + k_first) % chunks; };

    auto issue_a = [&](int c) {  // A: a weight, never written by a kernel
        const int s = c % kStages;
        uint8_t* st = ring + s * C::kStageBytes;
        const uint32_t bar = smem_u32(&full[s]);
        mbar_arrive_expect_tx(bar, tx);
#pragma unroll
        for (int b = 0; b < C::kABoxes; ++b)
            tma_load_2d(smem_u32(st + kXBoxBytes + b * kABoxBytes), &tmap_a, bar, 64 * b, kchunk(c) * kBK);
        if constexpr (C::kTail)
            tma_load_2d(smem_u32(st + kXBoxBytes + C::kABoxes * kABoxBytes), &tmap_a_tail, bar, 64 * C::kABoxes,
                        kchunk(c) * kBK);
    };
    auto issue_x = [&](int c) {
        const int s = c % kStages;
        tma_load_2d(smem_u32(ring + s * C::kStageBytes), &tmap_x, smem_u32(&full[s]), kchunk(c) * kBK, m0);
    };

    const int pre = chunks < kStages ? chunks : kStages;
    if (threadIdx.x == 0) {
        abort_flag = 0;
        issued_total = pre;
        for (int s = 0; s < kStages; ++s) {
            mbar_init(smem_u32(&full[s]), 1);
            released[s] = 0;
        }
        fence_mbar_init();
        for (int c = 0; c < pre; ++c) issue_a(c);
    }
    pdl_launch_dependents();
    pdl_wait();  // x may be the previous kernel's output
    if (threadIdx.x == 0)
        for (int c = 0; c < pre; ++c) issue_x(c);
    __syncthreads();

    // acc[rt][t]: row tile rt, n8 tile t (rank columns cg R / kColGroups + 8 t .. +7)
    float acc[kRowTiles][kTilesW][4];
#pragma unroll
    for (int i = 0; i < kRowTiles; ++i)
#pragma unroll
        for (int t = 0; t < kTilesW; ++t) acc[i][t][0] = acc[i][t][1] = acc[i][t][2] = acc[i][t][3] = 0.0f;
    bool ok = true;
    for (int c = kg; c < chunks; c += kKGroups) {
        const int s = c % kStages;
        const uint8_t* st = ring + s * C::kStageBytes;
        if (ok && !__all_sync(0xffffffffu, mbar_wait(smem_u32(&full[s]), static_cast<uint32_t>((c / kStages) & 1),
                                                     &abort_flag, Q6_SITE_GEMM_MAX)))
            ok = false;
        if (ok) {
            const uint32_t xs = smem_u32(st);
            const uint32_t as = smem_u32(st + kXBoxBytes);
#pragma unroll
            for (int ks = 0; ks < kBK / 16; ++ks) {
                // A operands: both row tiles' 16 rows, K columns 16 ks .. +15 of the x chunk
                uint32_t af[kRowTiles][4];
#pragma unroll
                for (int i = 0; i < kRowTiles; ++i) ldmatrix_x4(xs + swz(16 * i + (lane & 15), 2 * ks + (lane >> 4)), af[i]);
#pragma unroll
                for (int t = 0; t < kTilesW; ++t) {
                    // B operand: K rows 16 ks .. +15 of A, 8 rank columns
                    const int col = (R / kColGroups) * cg + 8 * t;
                    const int krow = 16 * ks + (lane & 15);
                    uint32_t bf[2];
                    if (col / 64 < C::kABoxes)
                        ldmatrix_x2_trans(as + (col / 64) * kABoxBytes + swz(krow, (col % 64) / 8), bf);
                    else
                        ldmatrix_x2_trans(as + C::kABoxes * kABoxBytes + swz64(krow, (col % 64) / 8), bf);
#pragma unroll
                    for (int i = 0; i < kRowTiles; ++i) mma_bf16_16816(acc[i][t], af[i], bf);
                }
            }
        }
        // Release the slot; the last of the chunk's kColGroups warps refills it with chunk c + kStages.
        __syncwarp();
        if (lane == 0) {
            uint32_t prev;
            asm volatile("atom.acq_rel.cta.shared::cta.add.u32 %0, [%1], 1;"
                         : "=r"(prev)
                         : "r"(smem_u32(&released[s]))
                         : "memory");
            if (prev == kColGroups - 1) {
                released[s] = 0;
                const int cn = c + kStages;
                if (cn < chunks && !abort_flag) {
                    fence_proxy_async_smem();  // the generic reads of the slot before the copies into it
                    issue_a(cn);
                    issue_x(cn);
                    atomicMax(&issued_total, cn + 1);
                }
            }
        }
    }

    // Copies in flight land before the ring holds the partial sums (bounded;
    // with every chunk consumed there are none).
    __syncthreads();
    if (threadIdx.x == 0) {
        const int issued = issued_total;
        for (int c = issued > kStages ? issued - kStages : 0; c < issued; ++c)
            mbar_wait_drain(smem_u32(&full[c % kStages]), static_cast<uint32_t>((c / kStages) & 1));
    }
    __syncthreads();
    // K groups 1.. store their partial sums (fragment order, lane-contiguous);
    // K group 0 adds them in K-group order and stores bf16.
    float* part = reinterpret_cast<float*>(ring);
    if (kg > 0) {
        float* mine = part + warp * (C::kFrag * 32) + lane;
#pragma unroll
        for (int i = 0; i < kRowTiles; ++i)
#pragma unroll
            for (int t = 0; t < kTilesW; ++t)
#pragma unroll
                for (int e = 0; e < 4; ++e) mine[((i * kTilesW + t) * 4 + e) * 32] = acc[i][t][e];
    }
    __syncthreads();
    if (kg == 0 && ok && !abort_flag) {
        // Accumulator layout: thread holds rows g, g + 8 (g = lane / 4) of each
        // row tile and columns 2 (lane % 4), +1 of each n8 tile.
        const int g = lane >> 2;
        const int cq = 2 * (lane & 3);
#pragma unroll
        for (int i = 0; i < kRowTiles; ++i)
#pragma unroll
            for (int t = 0; t < kTilesW; ++t) {
                float v[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    v[e] = acc[i][t][e];
                    for (int q = 1; q < kKGroups; ++q)
                        v[e] += part[(q * kColGroups + cg) * (C::kFrag * 32) + ((i * kTilesW + t) * 4 + e) * 32 + lane];
                }
                const int col = (R / kColGroups) * cg + 8 * t + cq;
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int64_t row = m0 + 16 * i + g + 8 * h;
                    if (row < M)
                        *reinterpret_cast<__nv_bfloat162*>(xa + row * R + col) = __floats2bfloat162_rn(v[2 * h], v[2 * h + 1]);
                }
            }
    }
}

PFN_cuTensorMapEncodeTiled_v12000 lora_encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult qr{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &qr) == cudaSuccess &&
            qr == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    });
    return fn;
}

// 2-D bf16 tensor map [outer][inner] with a [box_outer][box_inner] box
// (box_inner 64 with the 128-byte swizzle, 32 with the 64-byte swizzle).
bool lora_map(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint32_t box_inner,
              uint32_t box_outer) {
    auto fn = lora_encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {inner * 2};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    const CUtensorMapSwizzle sw = box_inner == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
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
    if (blocks > 0x7fffffff || M > 0x7fffffff) return Q6_ERR_UNSUPPORTED;
    // boxes no larger than the tensor: x rows past M stay unwritten (their
    // products land in accumulator rows that are never stored)
    const uint32_t x_rows = static_cast<uint32_t>(M < kRowsPerCta ? M : kRowsPerCta);
    CUtensorMap tx, ta, tt;
    if (!lora_map(&tx, x, static_cast<uint64_t>(K), static_cast<uint64_t>(M), 64, x_rows) ||
        (C::kABoxes > 0 && !lora_map(&ta, a, static_cast<uint64_t>(R), static_cast<uint64_t>(K), 64, kBK)) ||
        (C::kTail && !lora_map(&tt, a, static_cast<uint64_t>(R), static_cast<uint64_t>(K), 32, kBK)))
        return Q6_ERR_CUDA;
    if (C::kABoxes == 0) ta = tt;
    if (!C::kTail) tt = ta;
    const cudaError_t e = launch_pdl(lora_xa_kernel<R>, dim3(static_cast<unsigned>(blocks)), dim3(kThreads),
                                     C::kSmemBytes, stream, tx, ta, tt, xa, M, K, x_rows * 128u);
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
