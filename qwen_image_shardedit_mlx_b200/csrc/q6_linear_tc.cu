// tcgen05 q6 linear: dequantisation in the main loop, weights as the TMEM operand.
//
// Problem: y[m, n] = epi(sum_k x[m, k] * W[n, k]),  W = dequant(codes, scales, qbiases)
// (shardedit_mlx/q6_metal_mlp.py:58-83 computes the same function one output
// per thread).  Here the MMA computes the transpose D[n, m] = W[n, :] . x[m, :]:
//
//   * operand A (M = 128 weight rows) lives in tensor memory.  Dequant warps
//     read packed codes (TMA-staged in shared memory), expand them to bf16 in
//     registers and write them straight into TMEM with tcgen05.st, so the
//     dequantised tile never touches shared memory;
//   * operand B (N = NT tokens) is the activation tile, TMA-loaded with
//     128-byte swizzling into shared memory (K-major);
//   * the fp32 accumulator D (128 lanes x NT columns) sits in TMEM; epilogue
//     warps read it with tcgen05.ld, add bias, apply GELU / residual gate and
//     store bf16 rows of y.
//
// Warp roles (384 threads): warp 0 TMA producer, warp 1 MMA issuer, warp 2
// TMEM allocator, warp 3 idle, warps 4-7 epilogue, warps 8-11 dequant.  The
// CTA is persistent over (token tile, weight tile) pairs; accumulators are
// double buffered when NT <= 192 so the epilogue of one tile overlaps the main
// loop of the next.  Every mbarrier wait is bounded (q6_ptx.cuh).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "q6_dequant.cuh"
#include "q6_internal.h"
#include "q6_ptx.cuh"

namespace q6 {
namespace {

constexpr int kRows = 128;                       // weight rows per tile (MMA M)
constexpr int kBK = 64;                          // K per pipeline stage
constexpr int kCodeRowBytes = kBK * 6 / 8;       // 48 bytes of codes per row per stage
constexpr int kCodeStageBytes = kRows * kCodeRowBytes;  // 6144
constexpr int kCodeWordsPerStage = kBK * 6 / 32;        // 12
constexpr int kAStages = 4;                      // TMEM ring of dequantised A tiles
constexpr int kAColsPerStage = kBK / 2;          // bf16x2 per 32-bit column
constexpr int kThreads = 384;
constexpr int kSmemBudget = 227 * 1024;

constexpr int pow2_at_least(int v) {
    int p = 32;
    while (p < v) p <<= 1;
    return p;
}

template <int NT>
struct Cfg {
    static_assert(NT % 16 == 0 && NT >= 16 && NT <= 256, "MMA N must be a multiple of 16 in [16, 256]");
    static constexpr int kNAcc = (2 * NT + kAStages * kAColsPerStage <= 512) ? 2 : 1;
    static constexpr int kXStageBytes = NT * 128;  // NT rows of 64 bf16
    static constexpr int kStageBytes = kXStageBytes + kCodeStageBytes;
    static constexpr int kBarrierBytes = 256;
    static constexpr int kStagesFit = (kSmemBudget - 1024 - kBarrierBytes) / kStageBytes;
    static constexpr int kStages = kStagesFit > 8 ? 8 : kStagesFit;
    static constexpr int kSmemBytes = 1024 + kStages * kStageBytes + kBarrierBytes;
    static constexpr int kAccCols = kNAcc * NT;
    static constexpr int kTmemCols = pow2_at_least(kAccCols + kAStages * kAColsPerStage);
    static constexpr uint32_t kIdesc = idesc_bf16_f32(kRows, NT);
    static_assert(kStages >= 2, "need at least two pipeline stages");
    static_assert(kTmemCols <= 512, "TMEM budget");
    static_assert(kXStageBytes % 1024 == 0, "stage bases must stay 1024-byte aligned");
};

struct TcParams {
    const uint16_t* scales;
    const uint16_t* qbiases;
    const uint16_t* bias;
    const uint16_t* residual;
    const uint16_t* gate;
    uint16_t* y;
    int M, N, K, gs, groups, flags;
    int tiles_n, num_tiles, k_stages;
};

__device__ __forceinline__ float bf16f(uint16_t v) { return __uint_as_float(static_cast<uint32_t>(v) << 16); }

// Warp-uniform bounded wait: every lane polls, the warp proceeds only if all succeeded.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, int site) {
    const bool ok = mbar_wait(bar, parity, abort_flag, site);
    return __all_sync(0xffffffffu, ok);
}

template <int NT>
__global__ void __launch_bounds__(kThreads, 1)
    q6_linear_tc_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                        const TcParams p) {
    using C = Cfg<NT>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* x_smem = smem;
    uint8_t* c_smem = smem + C::kStages * C::kXStageBytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(c_smem + C::kStages * kCodeStageBytes);
    uint64_t* full = bars;
    uint64_t* empty = full + C::kStages;
    uint64_t* a_full = empty + C::kStages;
    uint64_t* a_empty = a_full + kAStages;
    uint64_t* acc_full = a_empty + kAStages;
    uint64_t* acc_empty = acc_full + C::kNAcc;
    uint64_t* drain = acc_empty + C::kNAcc;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::kStages; ++s) {
            mbar_init(smem_u32(full + s), 1);
            mbar_init(smem_u32(empty + s), 1 + 4);  // MMA commit + 4 dequant warps
        }
        for (int s = 0; s < kAStages; ++s) {
            mbar_init(smem_u32(a_full + s), 4);
            mbar_init(smem_u32(a_empty + s), 1);
        }
        for (int s = 0; s < C::kNAcc; ++s) {
            mbar_init(smem_u32(acc_full + s), 1);
            mbar_init(smem_u32(acc_empty + s), 4);
        }
        mbar_init(smem_u32(drain), 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 2) {
        tmem_alloc(smem_u32(tmem_slot), C::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        if (lane == 0) {
            tma_prefetch_map(&tmap_x);
            tma_prefetch_map(&tmap_w);
            int stage = 0;
            uint32_t phase = 0;
            long issued = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
                const int mb = tile / p.tiles_n;
                const int nb = tile - mb * p.tiles_n;
                for (int ks = 0; ks < p.k_stages; ++ks) {
                    if (!mbar_wait(smem_u32(empty + stage), phase ^ 1u, abort_flag, 1)) {
                        ok = false;
                        break;
                    }
                    const uint32_t fb = smem_u32(full + stage);
                    mbar_arrive_expect_tx(fb, C::kStageBytes);
                    tma_load_2d(smem_u32(x_smem + stage * C::kXStageBytes), &tmap_x, fb, ks * kBK, mb * NT);
                    tma_load_2d(smem_u32(c_smem + stage * kCodeStageBytes), &tmap_w, fb,
                                ks * kCodeWordsPerStage, nb * kRows);
                    ++issued;
                    if (++stage == C::kStages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            // Every issued copy must land before this CTA may exit.
            const long tail = issued < C::kStages ? issued : C::kStages;
            for (long i = 0; i < tail; ++i) {
                const long L = issued - 1 - i;
                mbar_wait_drain(smem_u32(full + (L % C::kStages)), static_cast<uint32_t>((L / C::kStages) & 1));
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            int stage = 0, astage = 0, acc = 0;
            uint32_t phase = 0, aphase = 0, accphase = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
                if (!mbar_wait(smem_u32(acc_empty + acc), accphase ^ 1u, abort_flag, 2)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * NT);
                for (int ks = 0; ks < p.k_stages; ++ks) {
                    if (!mbar_wait(smem_u32(full + stage), phase, abort_flag, 3) ||
                        !mbar_wait(smem_u32(a_full + astage), aphase, abort_flag, 4)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_tmem = tmem_base + static_cast<uint32_t>(C::kAccCols + astage * kAColsPerStage);
                    const uint64_t bdesc = sdesc_kmajor_sw128(smem_u32(x_smem + stage * C::kXStageBytes));
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; ++kk) {
                        mma_bf16_ts(d_tmem, a_tmem + kk * 8, bdesc + static_cast<uint64_t>(kk * 2), C::kIdesc,
                                    (ks | kk) != 0 ? 1u : 0u);
                    }
                    tc_commit(smem_u32(empty + stage));
                    tc_commit(smem_u32(a_empty + astage));
                    if (++stage == C::kStages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                    if (++astage == kAStages) {
                        astage = 0;
                        aphase ^= 1u;
                    }
                }
                if (!ok) break;
                tc_commit(smem_u32(acc_full + acc));
                if (++acc == C::kNAcc) {
                    acc = 0;
                    accphase ^= 1u;
                }
            }
            // All issued MMAs complete before TMEM may be released.
            tc_commit(smem_u32(drain));
            mbar_wait_drain(smem_u32(drain), 0);
        }
    } else if (warp >= 4 && warp < 8) {
        // ------------------------------------------------ epilogue
        constexpr int kChunk = NT >= 32 ? 32 : 16;  // accumulator columns per tcgen05.ld
        static_assert(NT % kChunk == 0, "token tile must be a multiple of the load width");
        const int q = warp & 3;
        const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
        int acc = 0;
        uint32_t accphase = 0;
        for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
            const int mb = tile / p.tiles_n;
            const int nb = tile - mb * p.tiles_n;
            const int n = nb * kRows + q * 32 + lane;
            const bool n_ok = n < p.N;
            const float bias_n = (n_ok && p.bias) ? bf16f(p.bias[n]) : 0.0f;
            const float gate_n = (n_ok && p.gate) ? bf16f(p.gate[n]) : 1.0f;
            if (!warp_wait(smem_u32(acc_full + acc), accphase, abort_flag, 5)) break;
            tc_fence_after();
#pragma unroll 1
            for (int c = 0; c < NT / kChunk; ++c) {
                uint32_t v[kChunk];
                const uint32_t taddr = tmem_base + lane_base + static_cast<uint32_t>(acc * NT + c * kChunk);
                if constexpr (kChunk == 32) {
                    tmem_ld_32x32b_x32(taddr, v);
                } else {
                    tmem_ld_32x32b_x16(taddr, v);
                }
                tmem_wait_ld();
                const int m0 = mb * NT + c * kChunk;
                if (n_ok) {
#pragma unroll
                    for (int j = 0; j < kChunk; ++j) {
                        const int m = m0 + j;
                        if (m < p.M) {
                            float val = __uint_as_float(v[j]) + bias_n;
                            if (p.flags & Q6_EPI_GELU) val = gelu_tanh(val);
                            if (p.gate) val *= gate_n;
                            const size_t off = static_cast<size_t>(m) * p.N + n;
                            if (p.residual) val += bf16f(p.residual[off]);
                            __nv_bfloat16 h = __float2bfloat16_rn(val);
                            p.y[off] = *reinterpret_cast<uint16_t*>(&h);
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(acc_empty + acc));
            if (++acc == C::kNAcc) {
                acc = 0;
                accphase ^= 1u;
            }
        }
    } else if (warp >= 8) {
        // ------------------------------------------------ dequant -> TMEM
        const int q = warp & 3;
        const int r = q * 32 + lane;
        const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
        int stage = 0, astage = 0;
        uint32_t phase = 0, aphase = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
            const int mb = tile / p.tiles_n;
            const int nb = tile - mb * p.tiles_n;
            const int n = nb * kRows + r;
            const bool n_ok = n < p.N;
            const uint16_t* srow = p.scales + static_cast<size_t>(n_ok ? n : 0) * p.groups;
            const uint16_t* brow = p.qbiases + static_cast<size_t>(n_ok ? n : 0) * p.groups;
            for (int ks = 0; ks < p.k_stages; ++ks) {
                const int k0 = ks * kBK;
                const int g0 = k0 / p.gs;
                const int g1 = (k0 + kBK / 2) / p.gs;
                float s0 = 0.f, b0 = 0.f, s1 = 0.f, b1 = 0.f;
                if (n_ok) {
                    s0 = bf16f(__ldg(srow + g0));
                    b0 = bf16f(__ldg(brow + g0));
                    s1 = bf16f(__ldg(srow + g1));
                    b1 = bf16f(__ldg(brow + g1));
                }
                if (!warp_wait(smem_u32(full + stage), phase, abort_flag, 6)) {
                    ok = false;
                    break;
                }
                const uint4* src = reinterpret_cast<const uint4*>(c_smem + stage * kCodeStageBytes + r * kCodeRowBytes);
                const uint4 c0 = src[0], c1 = src[1], c2 = src[2];
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(empty + stage));
                uint32_t a[32];
                dequant16_bf16x2(c0.x, c0.y, c0.z, s0, b0, a);
                dequant16_bf16x2(c0.w, c1.x, c1.y, s0, b0, a + 8);
                dequant16_bf16x2(c1.z, c1.w, c2.x, s1, b1, a + 16);
                dequant16_bf16x2(c2.y, c2.z, c2.w, s1, b1, a + 24);
                if (!warp_wait(smem_u32(a_empty + astage), aphase ^ 1u, abort_flag, 7)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                tmem_st_32x32b_x32(tmem_base + lane_base + static_cast<uint32_t>(C::kAccCols + astage * kAColsPerStage), a);
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(a_full + astage));
                if (++stage == C::kStages) {
                    stage = 0;
                    phase ^= 1u;
                }
                if (++astage == kAStages) {
                    astage = 0;
                    aphase ^= 1u;
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc(tmem_base, C::kTmemCols);
    }
}

// ------------------------------------------------------------- host side

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess) {
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
        }
    });
    return fn;
}

bool make_map_2d(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes, const void* base, uint64_t inner,
                 uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                 CUtensorMapSwizzle swizzle) {
    auto fn = encode_fn();
    if (!fn) return false;
    (void)elem_bytes;
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

template <int NT>
int launch_tc(const LinearArgs& a, cudaStream_t stream) {
    using C = Cfg<NT>;
    static int attr_set_for_device[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return Q6_ERR_CUDA;
    if (dev >= 0 && dev < 64 && !attr_set_for_device[dev]) {
        if (cudaFuncSetAttribute(q6_linear_tc_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 C::kSmemBytes) != cudaSuccess)
            return Q6_ERR_CUDA;
        attr_set_for_device[dev] = 1;
    }
    CUtensorMap tmap_x, tmap_w;
    if (!make_map_2d(&tmap_x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.x, a.K, a.M, a.K * 2, kBK, NT,
                     CU_TENSOR_MAP_SWIZZLE_128B))
        return Q6_ERR_CUDA;
    const uint64_t words = static_cast<uint64_t>(a.K) * 6 / 32;
    if (!make_map_2d(&tmap_w, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, a.w, words, a.N, words * 4, kCodeWordsPerStage,
                     kRows, CU_TENSOR_MAP_SWIZZLE_NONE))
        return Q6_ERR_CUDA;
    TcParams p;
    p.scales = a.scales;
    p.qbiases = a.qbiases;
    p.bias = a.bias;
    p.residual = a.residual;
    p.gate = a.gate;
    p.y = static_cast<uint16_t*>(a.y);
    p.M = static_cast<int>(a.M);
    p.N = static_cast<int>(a.N);
    p.K = static_cast<int>(a.K);
    p.gs = a.group_size;
    p.groups = static_cast<int>(a.K / a.group_size);
    p.flags = a.flags;
    p.tiles_n = static_cast<int>((a.N + kRows - 1) / kRows);
    const int tiles_m = static_cast<int>((a.M + NT - 1) / NT);
    p.num_tiles = tiles_m * p.tiles_n;
    p.k_stages = static_cast<int>(a.K / kBK);
    const int grid = std::min(p.num_tiles, device_sm_count());
    q6_linear_tc_kernel<NT><<<grid, kThreads, C::kSmemBytes, stream>>>(tmap_x, tmap_w, p);
    return cudaGetLastError() == cudaSuccess ? Q6_OK : Q6_ERR_CUDA;
}

}  // namespace

int error_word_tc(bool clear) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)) != cudaSuccess) return -1;
    if (clear && v != 0) {
        const int zero = 0;
        if (cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int)) != cudaSuccess) return -1;
    }
    return v;
}

bool tc_supported(const LinearArgs& a) {
    if (a.K % kBK != 0) return false;
    if (a.M > (int64_t(1) << 30) || a.N > (int64_t(1) << 30) || a.K > (int64_t(1) << 24)) return false;
    if (reinterpret_cast<uintptr_t>(a.x) % 16 != 0) return false;
    if (reinterpret_cast<uintptr_t>(a.w) % 16 != 0) return false;
    return true;
}

int choose_token_tile(int64_t M, int64_t N) {
    static const int kTiles[] = {256, 192, 128, 64, 32, 16};
    const int64_t sms = device_sm_count();
    const int64_t tiles_n = (N + kRows - 1) / kRows;
    int best = 16;
    int64_t best_cost = -1;
    for (int nt : kTiles) {
        const int64_t tiles = ((M + nt - 1) / nt) * tiles_n;
        const int64_t waves = (tiles + sms - 1) / sms;
        const int64_t cost = waves * (nt + 32);  // per-tile fixed overhead ~ 32 token-columns
        if (best_cost < 0 || cost < best_cost) {
            best_cost = cost;
            best = nt;
        }
    }
    return best;
}

int launch_linear_tc(const LinearArgs& a, int token_tile, cudaStream_t stream) {
    switch (token_tile) {
        case 256: return launch_tc<256>(a, stream);
        case 192: return launch_tc<192>(a, stream);
        case 128: return launch_tc<128>(a, stream);
        case 64: return launch_tc<64>(a, stream);
        case 32: return launch_tc<32>(a, stream);
        case 16: return launch_tc<16>(a, stream);
        default: return Q6_ERR_UNSUPPORTED;
    }
}

}  // namespace q6
