// q6 linear for a few token rows (M <= 32): warp-level MMA on the raw codes.
//
// With a handful of token rows the linear is bound by reading the packed
// weights (0.8125 bytes per weight at group size 64), so the arithmetic per
// code must stay a few instructions and the memory pipeline must stay full.
// The reference's sum_k x_k (scale * code_k + qbias) (shardedit_mlx/
// q6_metal_mlp.py:42-83) is evaluated per scale group g as
//
//     scale_g * sum_{k in g} x_k (128 + code_k) + (qbias_g - 128 scale_g) * sum_{k in g} x_k
//
// where 128 + code is exact in bf16 (exponent 2^7, the code in the low
// mantissa bits), so the two sums are exact-product bf16 MMAs with fp32
// accumulation (mma.sync m16n8k16): A = the token rows (one or two tiles of
// 16, zero past M), B = 128 + code for 8 weight rows, and a second B of ones
// gives the per-token sums of x.  The weights keep the reference kernel's
// fp32 semantics (no bf16 rounding of scale * code + qbias), like the
// CUDA-core paths.
//
// Layout of the MMA K dimension.  Each lane (g = lane / 4, q = lane % 4)
// owns the 16-code unit q (three packed words) of every 64-code block of its
// two weight rows g and 8 + g, and MMA K step s of the block takes codes
// 4s .. 4s + 3 of every lane's unit.  The K order inside the block is
// permuted, which the sum does not see, and the matching x values of a lane
// are x[16q + 4s .. 16q + 4s + 3]: eight contiguous bytes, so x fragments
// are plain 16-byte loads.  A code pair becomes one bf16x2 word with two
// shifts (one when a code sits on a byte boundary), a byte permute and one
// logic instruction that masks the codes and sets the exponent bits (a
// runtime word, so it stays one instruction).
//
// Data movement: each warp streams its 16 weight rows through a private
// two-slot ring in shared memory; its lane 0 loads a stage (16 rows x
// 8 * group_size codes with their 8 scale and bias groups) with three 2-D
// TMA copies while the warp works on the other slot.  A CTA of four warps
// covers 64 / splits rows; `splits` warps share a row block and split its
// K range, their partial sums meeting in shared memory (fixed order:
// bitwise reproducible) before one warp applies the epilogue (bias, GELU,
// gate, residual) and stores bf16.  Every barrier wait is bounded.
//
// Requirements (else another path runs): bf16 activations and output,
// 1 <= M <= 32, group size 64 or 128, K a multiple of 8 * group_size,
// 16-byte aligned x, codes, scales and biases, no LoRA delta.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <mutex>
#include <type_traits>

#include "q6_dequant.cuh"
#include "q6_internal.h"
#include "q6_ptx.cuh"

namespace q6 {
namespace {

constexpr int kWarps = 4;         // warps per CTA
constexpr int kRowsPerWarp = 16;  // weight rows of one warp (two n8 MMA tiles)
constexpr int kSlots = 2;         // ring slots per warp
constexpr int kSbGroups = 8;      // scale groups per stage (the 16-byte TMA box minimum)

template <int GS>
struct SkCfg {
    static constexpr int kStageCodes = kSbGroups * GS;                      // per row
    static constexpr int kStageWords = kStageCodes * 6 / 32;                // per row
    static constexpr int kCodeBytes = kRowsPerWarp * kStageWords * 4;       // 6144 (gs64) / 12288 (gs128)
    static constexpr int kSbBytes = kRowsPerWarp * kSbGroups * 2;           // 256: one array
    static constexpr int kStageBytes = ((kCodeBytes + 2 * kSbBytes) + 127) & ~127;
    static constexpr int kSmemBytes = kWarps * kSlots * kStageBytes + kWarps * kSlots * 8 + 128;
    static_assert(kStageWords <= 256, "TMA box inner extent");
};

struct SkParams {
    const uint16_t* x;
    const uint16_t* bias;
    const uint16_t* gate;
    const uint16_t* residual;
    uint16_t* y;
    int M, N, K, flags;
    int splits;             // warps per row block (K split), 1, 2 or 4
    int stages_per_split;   // stages of 8 * gs codes each warp runs
    uint32_t exp_pair;      // 0x43004300: bf16 exponent of 2^7 in both halves
};

__device__ __forceinline__ float bf16f(uint16_t v) { return __uint_as_float(static_cast<uint32_t>(v) << 16); }

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// bf16x2 (128 + code_lo, 128 + code_hi) from a word whose low byte pair holds
// code_lo at bit 0 and whose high byte pair holds code_hi at bit 16.
__device__ __forceinline__ uint32_t code_pair(uint32_t lo_src, uint32_t hi_src, uint32_t sel, uint32_t exp_pair) {
    return (__byte_perm(lo_src, hi_src, sel) & 0x003F003Fu) | exp_pair;
}

// B fragments (b0, b1) of MMA K step S for a unit (w0, w1, w2): pairs
// (4S, 4S + 1) and (4S + 2, 4S + 3).  Byte-permute selectors: 0x7610 takes
// bytes 0, 1 of the first word and 2, 3 of the second; 0x7613 / 0x7612 /
// 0x7611 take byte 3 / 2 / 1 of the first word into byte 0.
template <int S>
__device__ __forceinline__ void unit_pairs(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t e, uint32_t& b0,
                                           uint32_t& b1) {
    if constexpr (S == 0) {  // codes 0, 1 at w0 bits 0, 6; codes 2, 3 at 12, 18
        b0 = code_pair(w0, w0 << 10, 0x7610, e);
        b1 = code_pair(w0 >> 12, w0 >> 2, 0x7610, e);
    } else if constexpr (S == 1) {  // code 4 at w0 bit 24, code 5 at w0 30 .. w1 3; codes 6, 7 at w1 4, 10
        b0 = code_pair(w0, __funnelshift_r(w0, w1, 14), 0x7613, e);
        b1 = code_pair(w1 >> 4, w1 << 6, 0x7610, e);
    } else if constexpr (S == 2) {  // codes 8, 9 at w1 16, 22; code 10 at w1 28 .. w2 1, code 11 at w2 2
        b0 = code_pair(w1, w1 >> 6, 0x7612, e);
        b1 = code_pair(__funnelshift_r(w1, w2, 28), w2 << 14, 0x7610, e);
    } else {  // codes 12, 13 at w2 8, 14; codes 14, 15 at w2 20, 26
        b0 = code_pair(w2, w2 << 2, 0x7611, e);
        b1 = code_pair(w2 >> 20, w2 >> 10, 0x7610, e);
    }
}

template <int MTI, int GS>
__global__ void __launch_bounds__(kWarps * 32) skinny_kernel(const __grid_constant__ CUtensorMap tmap_w,
                                                            const __grid_constant__ CUtensorMap tmap_s,
                                                            const __grid_constant__ CUtensorMap tmap_b,
                                                            const SkParams p) {
    using C = SkCfg<GS>;
    extern __shared__ __align__(128) uint8_t sk_smem[];
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int g = lane >> 2;
    const int q = lane & 3;
    const int rb_per_cta = kWarps / p.splits;
    const int rb_local = warp / p.splits;
    const int split = warp - rb_local * p.splits;
    const int n0 = (blockIdx.x * rb_per_cta + rb_local) * kRowsPerWarp;
    const bool active = n0 < p.N;  // the same for every warp of a row block
    uint8_t* ring = sk_smem + warp * kSlots * C::kStageBytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(sk_smem + kWarps * kSlots * C::kStageBytes) + warp * kSlots;
    const int st0 = split * p.stages_per_split;
    const int nst = active ? p.stages_per_split : 0;

    auto issue = [&](int t) {  // lane 0: stage t of this warp into slot t % kSlots
        const uint32_t slot = smem_u32(ring + (t % kSlots) * C::kStageBytes);
        const uint32_t bar = smem_u32(full + (t % kSlots));
        mbar_arrive_expect_tx(bar, C::kCodeBytes + 2 * C::kSbBytes);
        const int st = st0 + t;
        tma_load_2d(slot, &tmap_w, bar, st * C::kStageWords, n0);
        tma_load_2d(slot + C::kCodeBytes, &tmap_s, bar, st * kSbGroups, n0);
        tma_load_2d(slot + C::kCodeBytes + C::kSbBytes, &tmap_b, bar, st * kSbGroups, n0);
    };

    if (lane == 0) {
        for (int s = 0; s < kSlots; ++s) mbar_init(smem_u32(full + s), 1);
        fence_mbar_init();
        tma_prefetch_map(&tmap_w);
        for (int t = 0; t < kSlots && t < nst; ++t) issue(t);  // weights: before the dependency wait
    }
    __syncwarp();
    pdl_launch_dependents();
    pdl_wait();  // x, the epilogue operands and y may belong to the previous kernel

    float acc[MTI][2][4];
#pragma unroll
    for (int i = 0; i < MTI; ++i)
#pragma unroll
        for (int j = 0; j < 2; ++j) acc[i][j][0] = acc[i][j][1] = acc[i][j][2] = acc[i][j][3] = 0.0f;

    const uint32_t e = p.exp_pair;
    const uint32_t ones = 0x3F803F80u;  // bf16 (1, 1)
    volatile int no_abort = 0;          // the ring is private to the warp
    const uint16_t* xg = p.x;
    // token rows of this lane: 16 i + g and 16 i + g + 8
    bool tok_ok[MTI][2];
#pragma unroll
    for (int i = 0; i < MTI; ++i) {
        tok_ok[i][0] = 16 * i + g < p.M;
        tok_ok[i][1] = 16 * i + g + 8 < p.M;
    }

    int consumed = 0;  // stages whose copies this warp has waited for
    for (int t = 0; t < nst; ++t) {
        const uint8_t* slot = ring + (t % kSlots) * C::kStageBytes;
        if (!__all_sync(0xffffffffu, mbar_wait(smem_u32(full + (t % kSlots)), static_cast<uint32_t>((t / kSlots) & 1),
                                               &no_abort, 12)))
            break;
        consumed = t + 1;
        const uint32_t* codes = reinterpret_cast<const uint32_t*>(slot);
        const uint16_t* scl = reinterpret_cast<const uint16_t*>(slot + C::kCodeBytes);
        const uint16_t* bia = reinterpret_cast<const uint16_t*>(slot + C::kCodeBytes + C::kSbBytes);
        const int k_stage = (st0 + t) * C::kStageCodes;
#pragma unroll 1
        for (int gi = 0; gi < kSbGroups; ++gi) {
            // scale and folded bias (qbias - 128 scale) of the accumulator rows 8 j + 2 q + c
            float2 sv[2], bv[2];
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const int r = 8 * j + 2 * q;
                const float s0 = bf16f(scl[r * kSbGroups + gi]), s1 = bf16f(scl[(r + 1) * kSbGroups + gi]);
                const float c0 = bf16f(bia[r * kSbGroups + gi]), c1 = bf16f(bia[(r + 1) * kSbGroups + gi]);
                sv[j] = make_float2(s0, s1);
                bv[j] = make_float2(fmaf(-128.0f, s0, c0), fmaf(-128.0f, s1, c1));
            }
            float D[MTI][2][4], X[MTI][4];
#pragma unroll
            for (int i = 0; i < MTI; ++i) {
                X[i][0] = X[i][1] = X[i][2] = X[i][3] = 0.0f;
#pragma unroll
                for (int j = 0; j < 2; ++j) D[i][j][0] = D[i][j][1] = D[i][j][2] = D[i][j][3] = 0.0f;
            }
#pragma unroll
            for (int blk = 0; blk < GS / 64; ++blk) {
                const int kb = gi * GS + blk * 64;            // stage-local K of the 64-code block
                const int uo = (kb >> 4) * 3 + 3 * q;          // this lane's unit: word offset in a stage row
                const uint32_t* r0 = codes + g * C::kStageWords + uo;
                const uint32_t* r1 = codes + (8 + g) * C::kStageWords + uo;
                const uint32_t u00 = r0[0], u01 = r0[1], u02 = r0[2];
                const uint32_t u10 = r1[0], u11 = r1[1], u12 = r1[2];
                // x values of this lane's codes: 16 bf16 per token row = 2 x 16 bytes
                uint4 xa[MTI][2][2];
#pragma unroll
                for (int i = 0; i < MTI; ++i)
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        if (tok_ok[i][h]) {
                            const uint4* src = reinterpret_cast<const uint4*>(
                                xg + static_cast<size_t>(16 * i + g + 8 * h) * p.K + k_stage + kb + 16 * q);
                            xa[i][h][0] = __ldg(src);
                            xa[i][h][1] = __ldg(src + 1);
                        } else {
                            xa[i][h][0] = xa[i][h][1] = make_uint4(0, 0, 0, 0);
                        }
                    }
                auto step = [&](auto S_, uint32_t p0a, uint32_t p0b, uint32_t p1a, uint32_t p1b) {
                    constexpr int S = decltype(S_)::value;
#pragma unroll
                    for (int i = 0; i < MTI; ++i) {
                        // x words 2S, 2S + 1 of each token row: codes 4S .. 4S + 3 of the lane's unit
                        const uint32_t* lo = reinterpret_cast<const uint32_t*>(&xa[i][0][S / 2]);
                        const uint32_t* hi = reinterpret_cast<const uint32_t*>(&xa[i][1][S / 2]);
                        const uint32_t a0 = lo[2 * (S % 2)], a2 = lo[2 * (S % 2) + 1];
                        const uint32_t a1 = hi[2 * (S % 2)], a3 = hi[2 * (S % 2) + 1];
                        mma_bf16_16816(D[i][0], a0, a1, a2, a3, p0a, p0b);
                        mma_bf16_16816(D[i][1], a0, a1, a2, a3, p1a, p1b);
                        mma_bf16_16816(X[i], a0, a1, a2, a3, ones, ones);
                    }
                };
                uint32_t b00, b01, b10, b11;
                unit_pairs<0>(u00, u01, u02, e, b00, b01);
                unit_pairs<0>(u10, u11, u12, e, b10, b11);
                step(std::integral_constant<int, 0>{}, b00, b01, b10, b11);
                unit_pairs<1>(u00, u01, u02, e, b00, b01);
                unit_pairs<1>(u10, u11, u12, e, b10, b11);
                step(std::integral_constant<int, 1>{}, b00, b01, b10, b11);
                unit_pairs<2>(u00, u01, u02, e, b00, b01);
                unit_pairs<2>(u10, u11, u12, e, b10, b11);
                step(std::integral_constant<int, 2>{}, b00, b01, b10, b11);
                unit_pairs<3>(u00, u01, u02, e, b00, b01);
                unit_pairs<3>(u10, u11, u12, e, b10, b11);
                step(std::integral_constant<int, 3>{}, b00, b01, b10, b11);
            }
            // acc += scale * sum x (128 + code) + (qbias - 128 scale) * sum x, per (token, row) pair
#pragma unroll
            for (int i = 0; i < MTI; ++i)
#pragma unroll
                for (int j = 0; j < 2; ++j)
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        float2 a = make_float2(acc[i][j][2 * h], acc[i][j][2 * h + 1]);
                        a = __ffma2_rn(sv[j], make_float2(D[i][j][2 * h], D[i][j][2 * h + 1]), a);
                        a = __ffma2_rn(bv[j], make_float2(X[i][2 * h], X[i][2 * h + 1]), a);
                        acc[i][j][2 * h] = a.x;
                        acc[i][j][2 * h + 1] = a.y;
                    }
        }
        // hand the slot back to this warp's producer lane for stage t + kSlots
        __syncwarp();
        if (lane == 0 && t + kSlots < nst) {
            fence_proxy_async_smem();
            issue(t + kSlots);
        }
    }
    // After a wait that gave up, copies issued for later stages may still be in
    // flight: wait for them (bounded) before the ring is reused or the CTA exits.
    if (lane == 0) {
        const int issued = nst < consumed + kSlots ? nst : consumed + kSlots;
        for (int u = consumed; u < issued; ++u)
            mbar_wait_drain(smem_u32(full + (u % kSlots)), static_cast<uint32_t>((u / kSlots) & 1));
    }
    __syncwarp();
    if (!active) return;  // every warp of an inactive row block leaves together

    // K split: the partial sums of warps 1 .. splits - 1 of a row block meet
    // in shared memory (each warp's own idle ring), summed in split order.
    if (p.splits > 1) {
        float* mine = reinterpret_cast<float*>(ring);
        if (split != 0) {
#pragma unroll
            for (int i = 0; i < MTI; ++i)
#pragma unroll
                for (int j = 0; j < 2; ++j)
#pragma unroll
                    for (int c = 0; c < 4; ++c) mine[((i * 2 + j) * 4 + c) * 32 + lane] = acc[i][j][c];
        }
        asm volatile("bar.sync %0, %1;" ::"r"(1 + rb_local), "r"(32 * p.splits) : "memory");
        if (split != 0) return;
        for (int sp = 1; sp < p.splits; ++sp) {
            const float* other = reinterpret_cast<const float*>(sk_smem + (warp + sp) * kSlots * C::kStageBytes);
#pragma unroll
            for (int i = 0; i < MTI; ++i)
#pragma unroll
                for (int j = 0; j < 2; ++j)
#pragma unroll
                    for (int c = 0; c < 4; ++c) acc[i][j][c] += other[((i * 2 + j) * 4 + c) * 32 + lane];
        }
    }

    // Epilogue: lane holds tokens 16 i + g (+ 8) x rows n0 + 8 j + 2 q (+ 1).
    const bool gelu = (p.flags & (Q6_EPI_GELU | Q6_EPI_GELU_PRECISE)) != 0;
    const bool precise = (p.flags & Q6_EPI_GELU_PRECISE) != 0;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        const int n = n0 + 8 * j + 2 * q;
        const bool ok0 = n < p.N, ok1 = n + 1 < p.N;
        const float b0 = (ok0 && p.bias) ? bf16f(p.bias[n]) : 0.0f;
        const float b1 = (ok1 && p.bias) ? bf16f(p.bias[n + 1]) : 0.0f;
        const float g0 = (ok0 && p.gate) ? bf16f(p.gate[n]) : 1.0f;
        const float g1 = (ok1 && p.gate) ? bf16f(p.gate[n + 1]) : 1.0f;
#pragma unroll
        for (int i = 0; i < MTI; ++i)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int m = 16 * i + g + 8 * h;
                if (m >= p.M) continue;
                float v0 = acc[i][j][2 * h] + b0, v1 = acc[i][j][2 * h + 1] + b1;
                if (gelu) {
                    v0 = gelu_select(v0, precise);
                    v1 = gelu_select(v1, precise);
                }
                v0 *= g0;
                v1 *= g1;
                const size_t off = static_cast<size_t>(m) * p.N + n;
                if (p.residual) {
                    if (ok0) v0 += bf16f(p.residual[off]);
                    if (ok1) v1 += bf16f(p.residual[off + 1]);
                }
                const uint32_t w = pack_bf16x2(v0, v1);
                if (ok1 && (reinterpret_cast<uintptr_t>(p.y + off) & 3) == 0) {
                    *reinterpret_cast<uint32_t*>(p.y + off) = w;
                } else {
                    if (ok0) p.y[off] = static_cast<uint16_t>(w & 0xFFFFu);
                    if (ok1) p.y[off + 1] = static_cast<uint16_t>(w >> 16);
                }
            }
    }
}

PFN_cuTensorMapEncodeTiled_v12000 sk_encode_fn() {
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

bool sk_map(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner, uint64_t outer,
            uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer) {
    auto fn = sk_encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    return fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Warps per row block (K split) for an (N, K) problem: the split whose CTAs,
// four warps each, best fill the GPU at the resident CTAs per SM that the
// shared memory allows, fewer splits on a tie.  Q6_SKINNY_SPLITS overrides.
int plan_splits(int64_t N, int stages, int ctas_per_sm) {
    if (const char* v = std::getenv("Q6_SKINNY_SPLITS")) {
        const int s = std::atoi(v);
        if ((s == 1 || s == 2 || s == 4) && stages % s == 0) return s;
    }
    const int64_t sms = device_sm_count();
    const int64_t row_blocks = (N + kRowsPerWarp - 1) / kRowsPerWarp;
    int best = 1;
    int64_t best_cost = -1;
    for (int s : {1, 2, 4}) {
        if (stages % s) continue;
        const int64_t ctas = (row_blocks + kWarps / s - 1) / (kWarps / s);
        const int64_t per_sm = (ctas + sms - 1) / sms;                  // CTAs on the busiest SM
        const int64_t waves = (per_sm + ctas_per_sm - 1) / ctas_per_sm;  // rounds of resident CTAs there
        const int64_t spw = stages / s;                                  // stages per warp
        // Busiest SM: its warps' stages over four schedulers at ~0.8 of issue,
        // but no faster than one warp alone (~0.4 of issue) per round.
        const int64_t cost = std::max<int64_t>(per_sm * kWarps * spw * 5, waves * spw * 10) * 4 + s;
        if (best_cost < 0 || cost < best_cost) {
            best_cost = cost;
            best = s;
        }
    }
    return best;
}

template <int MTI, int GS>
int launch_skinny_t(const LinearArgs& a, cudaStream_t stream) {
    using C = SkCfg<GS>;
    static std::atomic<bool> attr_set_for_device[kMaxDevices];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return Q6_ERR_CUDA;
    if (dev < 0 || dev >= kMaxDevices) return Q6_ERR_UNSUPPORTED;
    if (!attr_set_for_device[dev].load(std::memory_order_acquire)) {
        if (cudaFuncSetAttribute(skinny_kernel<MTI, GS>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes) !=
            cudaSuccess)
            return Q6_ERR_CUDA;
        attr_set_for_device[dev].store(true, std::memory_order_release);
    }
    const uint64_t words = static_cast<uint64_t>(a.K) * 6 / 32;
    const uint64_t groups = static_cast<uint64_t>(a.K / GS);
    CUtensorMap tw, ts, tb;
    if (!sk_map(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT32, a.w, words, a.N, words * 4, C::kStageWords, kRowsPerWarp) ||
        !sk_map(&ts, CU_TENSOR_MAP_DATA_TYPE_UINT16, a.scales, groups, a.N, groups * 2, kSbGroups, kRowsPerWarp) ||
        !sk_map(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT16, a.qbiases, groups, a.N, groups * 2, kSbGroups, kRowsPerWarp))
        return Q6_ERR_CUDA;
    const int stages = static_cast<int>(a.K / C::kStageCodes);
    const int ctas_per_sm = std::max(1, (227 * 1024) / (C::kSmemBytes + 1024));
    SkParams p;
    p.x = static_cast<const uint16_t*>(a.x);
    p.bias = a.bias;
    p.gate = a.gate;
    p.residual = a.residual;
    p.y = static_cast<uint16_t*>(a.y);
    p.M = static_cast<int>(a.M);
    p.N = static_cast<int>(a.N);
    p.K = static_cast<int>(a.K);
    p.flags = a.flags;
    p.splits = plan_splits(a.N, stages, ctas_per_sm);
    p.stages_per_split = stages / p.splits;
    p.exp_pair = 0x43004300u;
    const int64_t row_blocks = (a.N + kRowsPerWarp - 1) / kRowsPerWarp;
    const int rb_per_cta = kWarps / p.splits;
    const int64_t ctas = (row_blocks + rb_per_cta - 1) / rb_per_cta;
    const cudaError_t err = launch_pdl(skinny_kernel<MTI, GS>, dim3(static_cast<unsigned>(ctas)), dim3(kWarps * 32),
                                       C::kSmemBytes, stream, tw, ts, tb, p);
    return err == cudaSuccess ? Q6_OK : Q6_ERR_CUDA;
}

}  // namespace

bool skinny_supported(const LinearArgs& a) {
    if (a.M < 1 || a.M > 32 || a.lora_rank != 0) return false;
    if (a.group_size != 64 && a.group_size != 128) return false;
    if (a.K % (kSbGroups * a.group_size) != 0 || a.K > (int64_t(1) << 24) || a.N > (int64_t(1) << 30)) return false;
    const uintptr_t al = reinterpret_cast<uintptr_t>(a.x) | reinterpret_cast<uintptr_t>(a.w) |
                         reinterpret_cast<uintptr_t>(a.scales) | reinterpret_cast<uintptr_t>(a.qbiases);
    return al % 16 == 0;
}

int launch_skinny(const LinearArgs& a, cudaStream_t stream) {
    const bool two = a.M > 16;
    if (a.group_size == 64) return two ? launch_skinny_t<2, 64>(a, stream) : launch_skinny_t<1, 64>(a, stream);
    return two ? launch_skinny_t<2, 128>(a, stream) : launch_skinny_t<1, 128>(a, stream);
}

int error_word_skinny(bool clear) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)) != cudaSuccess) return -1;
    if (clear && v != 0) {
        const int zero = 0;
        if (cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int)) != cudaSuccess) return -1;
    }
    return v;
}

}  // namespace q6
