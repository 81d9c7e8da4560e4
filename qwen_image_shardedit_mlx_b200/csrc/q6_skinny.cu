// q6 linear for a few token rows (M <= 16): warp-level MMA on the raw codes,
// K streamed in CTA-wide stages.
//
// With a handful of token rows the linear is bound by reading the packed
// weights (0.8125 bytes per weight at group size 64), so the arithmetic per
// code must stay a few instructions and HBM must stay busy.  The reference's
// sum_k x_k (scale * code_k + qbias) (shardedit_mlx/q6_metal_mlp.py:42-83) is
// evaluated per 64-code block of one scale group g as
//
//     scale_g * sum_k x_k (128 + code_k) + (qbias_g - 128 scale_g) * sum_k x_k
//
// where 128 + code is exact in bf16 (exponent 2^7, the code in the low
// mantissa bits), so both sums are exact-product bf16 MMAs with fp32
// accumulation (mma.sync m16n8k16): A = the token rows (one tile of 16, zero
// past M), B = 128 + code for 8 weight rows, and a B of ones gives the sums
// of x.  The weights keep the reference kernel's fp32 semantics (no bf16
// rounding of scale * code + qbias), like the CUDA-core paths.
//
// Layout of the MMA K dimension.  Lane (g = lane / 4, q = lane % 4) owns the
// 16-code unit q (three packed words) of every 64-code block of weight row g
// of a tile, and MMA K step s of the block takes codes 4s .. 4s + 3 of every
// lane's unit.  The K order inside the block is permuted, which the sum does
// not see; the matching activations of a lane are x[16q + 4s .. 16q + 4s + 3]
// of its token rows, eight contiguous bytes.  A code pair becomes one bf16x2
// word with a shift or two, a byte permute and one logic instruction.
//
// Work and data movement.  A CTA owns a block of 8 T weight rows (T n8 tiles,
// T even, at most 16) and streams all of K through a ring of CTA-wide stages
// of 512 codes.  Each stage arrives by TMA (one [rows x 100 words] code box,
// 4 words more than the stage's 96 so that the 400-byte shared rows put the
// eight rows a warp reads in different banks; eight [tokens x 64] activation
// boxes with the 128-byte swizzle; the stage's scale and bias groups), and the
// last of the sixteen MMA warps to release a ring slot refills it, so no warp
// waits to produce.  The warps consume a stage as follows: warp (block b, half h) takes the 64-code block b of the
// stage for tile half h, so the activations of a block are loaded once per
// warp and serve all of its tiles.  At the end of a row block the eight block
// warps of each half hold partial sums over K; they meet in shared memory and
// are summed in block order (bitwise reproducible) before the epilogue
// (bias, GELU, gate, residual) stores bf16.  A CTA walks row blocks
// b, b + gridDim.x, ... with the stage ring running on across them.  Every
// barrier wait is bounded.
//
// Requirements (else another path runs): bf16 activations and output,
// 1 <= M <= 16, K a multiple of 512, group size 32, 64 or 128 with
// K / group_size a multiple of 8, 16-byte aligned x, codes, scales and
// biases, no LoRA delta.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <mutex>

#include "q6_dequant.cuh"
#include "q6_internal.h"
#include "q6_ptx.cuh"

namespace q6 {
namespace {

constexpr int kBlocks = 8;                  // 64-code blocks per stage
constexpr int kChunk = 64 * kBlocks;        // codes per row per stage
constexpr int kHalves = 2;                  // MMA warps per block (tile halves)
constexpr int kMmaWarps = kBlocks * kHalves;
constexpr int kThreads = kMmaWarps * 32;
constexpr int kMaxTiles = 16;               // n8 tiles per row block
constexpr int kTok = 16;                    // token rows of the A tile
constexpr int kXBoxStride = kTok * 128;     // shared-memory slot of one [tokens x 64] bf16 activation box
constexpr int kMaxStages = 4;
constexpr int kCodeRowWords = 100;         // words per shared code row: the stage's 96 and 4 of padding
constexpr int kSmemBudget = 227 * 1024 - 1024;  // dynamic shared memory (the kernel's statics stay below 1 KB)

struct SkGeom {
    int tiles;          // n8 tiles per row block (even)
    int rows;           // 8 * tiles
    int sb_groups;      // scale groups per stage box (>= 8)
    int code_bytes;     // per stage: rows x 400 bytes
    int sb_bytes;       // per stage, one of scales / biases
    int stage_bytes;    // activation boxes first (1024-byte aligned for the swizzle)
    int scratch_bytes;  // per-warp partial sums of a row block
    int stages;
    int smem_bytes;
};

inline int align_up(int v, int a) { return (v + a - 1) / a * a; }

inline SkGeom sk_geometry(int tiles, int gs) {
    SkGeom g;
    g.tiles = tiles;
    g.rows = 8 * tiles;
    g.sb_groups = std::max(8, kChunk / gs);
    g.code_bytes = g.rows * kCodeRowWords * 4;
    g.sb_bytes = g.rows * g.sb_groups * 2;
    g.stage_bytes = align_up(kBlocks * kXBoxStride + g.code_bytes + 2 * g.sb_bytes, 1024);
    g.scratch_bytes = kMmaWarps * (tiles / kHalves) * 4 * 32 * 4;
    const int fixed = g.scratch_bytes + 1024 /* alignment */ + kMaxStages * 8 /* barriers */;
    g.stages = std::min(kMaxStages, (kSmemBudget - fixed) / g.stage_bytes);
    g.smem_bytes = g.stages * g.stage_bytes + fixed;
    return g;
}

struct SkParams {
    const uint16_t* bias;
    const uint16_t* gate;
    const uint16_t* residual;
    uint16_t* y;
    int M, N, K, flags;
    int gs_shift;
    int rows, sb_groups, code_bytes, sb_bytes, stage_bytes, stages;
    int row_blocks;
    uint32_t x_box_bytes;  // M rows x 128 bytes
    uint32_t exp_pair;     // 0x43004300: bf16 exponent of 2^7 in both halves
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

// A fragment words of K step S (activation pairs 4S, 4S + 1 and 4S + 2, 4S + 3
// of the lane's unit) from the lane's 16 activations of a token row.
template <int S>
__device__ __forceinline__ void a_words(const uint4 (&r)[2], uint32_t& lo, uint32_t& hi) {
    const uint4 v = r[S / 2];
    if constexpr (S % 2 == 0) {
        lo = v.x;
        hi = v.y;
    } else {
        lo = v.z;
        hi = v.w;
    }
}

// Refill of ring slot s with stage t (one thread): the weights part (codes,
// scales, biases: never written by a kernel) and the activations part.
struct SkIssue {
    const CUtensorMap* tx;
    const CUtensorMap* tw;
    const CUtensorMap* ts;
    const CUtensorMap* tb;
    uint8_t* ring;
    uint64_t* full;
    int stages, stage_bytes, chunks, rows, code_bytes, sb_bytes, groups_per_chunk;
    uint32_t tx_bytes;

    __device__ __forceinline__ void weights(int t, int rb) const {
        const int s = t % stages;
        uint8_t* codes = ring + s * stage_bytes + kBlocks * kXBoxStride;
        const uint32_t bar = smem_u32(full + s);
        const int c = t % chunks;
        const int r0 = rb * rows;
        mbar_arrive_expect_tx(bar, tx_bytes);
        tma_load_2d(smem_u32(codes), tw, bar, c * (kChunk * 6 / 32), r0);
        const int gbox = (c * groups_per_chunk) & ~7;  // 16-byte aligned box start
        tma_load_2d(smem_u32(codes + code_bytes), ts, bar, gbox, r0);
        tma_load_2d(smem_u32(codes + code_bytes + sb_bytes), tb, bar, gbox, r0);
    }
    __device__ __forceinline__ void activations(int t) const {
        const int s = t % stages;
        uint8_t* st = ring + s * stage_bytes;
        const uint32_t bar = smem_u32(full + s);
        const int c = t % chunks;
#pragma unroll 1
        for (int b = 0; b < kBlocks; ++b)
            tma_load_2d(smem_u32(st + b * kXBoxStride), tx, bar, c * kChunk + b * 64, 0);
    }
};

// GS: group size; TPW: n8 tiles per warp (the row block holds 2 TPW tiles).
template <int GS, int TPW>
__global__ void __launch_bounds__(kThreads, 1) skinny_kernel(const __grid_constant__ CUtensorMap tmap_x,
                                                            const __grid_constant__ CUtensorMap tmap_w,
                                                            const __grid_constant__ CUtensorMap tmap_s,
                                                            const __grid_constant__ CUtensorMap tmap_b,
                                                            const SkParams p) {
    extern __shared__ uint8_t sk_raw[];
    uint8_t* ring = smem_align_up<1024>(sk_raw);
    float* scratch = reinterpret_cast<float*>(ring + p.stages * p.stage_bytes);
    uint64_t* full = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(scratch) +
                                                 kMmaWarps * TPW * 4 * 32 * 4);
    __shared__ int abort_flag;
    __shared__ uint32_t released[kMaxStages];  // warps done with the slot's current stage
    __shared__ int issued_total;               // stages whose copies were issued

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int chunks = p.K / kChunk;
    const int my_blocks =
        static_cast<int>(blockIdx.x) < p.row_blocks ? (p.row_blocks - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
    const int total = my_blocks * chunks;  // stages of this CTA
    const int code_off = kBlocks * kXBoxStride;
    SkIssue io;
    io.tx = &tmap_x;
    io.tw = &tmap_w;
    io.ts = &tmap_s;
    io.tb = &tmap_b;
    io.ring = ring;
    io.full = full;
    io.stages = p.stages;
    io.stage_bytes = p.stage_bytes;
    io.chunks = chunks;
    io.rows = p.rows;
    io.code_bytes = p.code_bytes;
    io.sb_bytes = p.sb_bytes;
    io.groups_per_chunk = kChunk / GS;
    io.tx_bytes = kBlocks * p.x_box_bytes + p.code_bytes + 2 * p.sb_bytes;
    auto block_of = [&](int t) { return static_cast<int>(blockIdx.x) + (t / chunks) * static_cast<int>(gridDim.x); };

    const int pre = total < p.stages ? total : p.stages;
    if (threadIdx.x == 0) {
        abort_flag = 0;
        issued_total = pre;
        for (int s = 0; s < kMaxStages; ++s) released[s] = 0;
        for (int s = 0; s < p.stages; ++s) mbar_init(smem_u32(full + s), 1);
        fence_mbar_init();
        tma_prefetch_map(&tmap_w);
        tma_prefetch_map(&tmap_x);
        for (int t = 0; t < pre; ++t) io.weights(t, block_of(t));  // before the dependency wait
    }
    pdl_launch_dependents();
    pdl_wait();  // x, the epilogue operands and y may belong to the previous kernel
    if (threadIdx.x == 0)
        for (int t = 0; t < pre; ++t) io.activations(t);
    __syncthreads();

    const int blk = warp >> 1;         // 64-code block of each stage
    const int half = warp & 1;         // tile half
    const int g = lane >> 2;
    const int q = lane & 3;
    const int tile0 = half * TPW;      // first tile of this warp in the row block
    const uint32_t e = p.exp_pair;
    const uint32_t ones = 0x3F803F80u;  // bf16 (1, 1)
    const bool row_lo = g < p.M, row_hi = g + 8 < p.M;
    const int swz = g & 7;              // 128-byte swizzle of token rows g and g + 8
    const uint32_t mask0 = (GS == 32 && q >= 2) ? 0u : 0xFFFFFFFFu;  // group size 32: lanes of group 0
    bool ok = true;

    for (int rbi = 0; rbi < my_blocks; ++rbi) {
        const int rb = blockIdx.x + rbi * gridDim.x;
        float2 acc[TPW][2];  // (token g: rows 2q, 2q + 1), (token g + 8: rows 2q, 2q + 1)
#pragma unroll
        for (int j = 0; j < TPW; ++j) acc[j][0] = acc[j][1] = make_float2(0.0f, 0.0f);

        for (int c = 0; c < chunks; ++c) {
            const int t = rbi * chunks + c;
            const int s = t % p.stages;
            const uint8_t* st = ring + s * p.stage_bytes;
            if (ok && !__all_sync(0xffffffffu, mbar_wait(smem_u32(full + s), static_cast<uint32_t>((t / p.stages) & 1),
                                                         &abort_flag, Q6_SITE_GEMM_MAX)))
                ok = false;
            if (ok) {
                // activations of this block: token rows g and g + 8, logical 16-byte chunks 2q and 2q + 1
                uint4 xr[2][2];
                const uint8_t* xb = st + blk * kXBoxStride;
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const bool live = h ? row_hi : row_lo;
                    const uint8_t* row = xb + (g + 8 * h) * 128;
                    const uint4 z = make_uint4(0u, 0u, 0u, 0u);
                    xr[h][0] = live ? *reinterpret_cast<const uint4*>(row + 16 * ((2 * q) ^ swz)) : z;
                    xr[h][1] = live ? *reinterpret_cast<const uint4*>(row + 16 * ((2 * q + 1) ^ swz)) : z;
                }
                uint32_t a[4][4];  // A fragments of the four K steps
                a_words<0>(xr[0], a[0][0], a[0][2]);
                a_words<0>(xr[1], a[0][1], a[0][3]);
                a_words<1>(xr[0], a[1][0], a[1][2]);
                a_words<1>(xr[1], a[1][1], a[1][3]);
                a_words<2>(xr[0], a[2][0], a[2][2]);
                a_words<2>(xr[1], a[2][1], a[2][3]);
                a_words<3>(xr[0], a[3][0], a[3][2]);
                a_words<3>(xr[1], a[3][1], a[3][3]);
                // Sums of x over the block.  Group size 32: codes 0-31 of the block are
                // the units of lanes q = 0, 1 and codes 32-63 those of q = 2, 3, so each
                // group's sums take B operands zeroed in the other group's lanes.
                float X0[4] = {0.0f, 0.0f, 0.0f, 0.0f}, X1[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
                for (int ks = 0; ks < 4; ++ks) {
                    mma_bf16_16816(X0, a[ks][0], a[ks][1], a[ks][2], a[ks][3], ones & mask0, ones & mask0);
                    if constexpr (GS == 32)
                        mma_bf16_16816(X1, a[ks][0], a[ks][1], a[ks][2], a[ks][3], ones & ~mask0, ones & ~mask0);
                }
                const uint32_t* codes = reinterpret_cast<const uint32_t*>(st + code_off) +
                                        (8 * tile0 + g) * kCodeRowWords + blk * 12 + 3 * q;
                const uint16_t* scl = reinterpret_cast<const uint16_t*>(st + code_off + p.code_bytes);
                const uint16_t* bia = scl + p.sb_bytes / 2;
                // scale group of this block within the stage's scale box; rows 2q, 2q + 1 of tile 0
                const int gin = (((c * kChunk) >> p.gs_shift) & 7) + ((blk * 64) >> p.gs_shift);
                const uint16_t* scl0 = scl + (8 * tile0 + 2 * q) * p.sb_groups + gin;
                const uint16_t* bia0 = bia + (8 * tile0 + 2 * q) * p.sb_groups + gin;
                const int tile_sb = 8 * p.sb_groups;  // scale entries per tile
#pragma unroll
                for (int j = 0; j < TPW; ++j) {
                    const uint32_t* u = codes + j * 8 * kCodeRowWords;
                    const uint32_t w0 = u[0], w1 = u[1], w2 = u[2];
                    float D0[4] = {0.0f, 0.0f, 0.0f, 0.0f}, D1[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                    uint32_t b[4][2];
                    unit_pairs<0>(w0, w1, w2, e, b[0][0], b[0][1]);
                    unit_pairs<1>(w0, w1, w2, e, b[1][0], b[1][1]);
                    unit_pairs<2>(w0, w1, w2, e, b[2][0], b[2][1]);
                    unit_pairs<3>(w0, w1, w2, e, b[3][0], b[3][1]);
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks) {
                        mma_bf16_16816(D0, a[ks][0], a[ks][1], a[ks][2], a[ks][3], b[ks][0] & mask0, b[ks][1] & mask0);
                        if constexpr (GS == 32)
                            mma_bf16_16816(D1, a[ks][0], a[ks][1], a[ks][2], a[ks][3], b[ks][0] & ~mask0,
                                           b[ks][1] & ~mask0);
                    }
                    // acc += scale * sum x (128 + code) + (qbias - 128 scale) * sum x, rows 2q and 2q + 1
                    auto fold = [&](const float (&D)[4], const float (&X)[4], int gi) {
                        const uint16_t* sp = scl0 + j * tile_sb + gi;
                        const uint16_t* bp = bia0 + j * tile_sb + gi;
                        const float2 sv = make_float2(bf16f(sp[0]), bf16f(sp[p.sb_groups]));
                        const float2 bv = make_float2(bf16f(bp[0]), bf16f(bp[p.sb_groups]));
                        const float2 cv = __ffma2_rn(make_float2(-128.0f, -128.0f), sv, bv);
                        acc[j][0] = __ffma2_rn(sv, make_float2(D[0], D[1]), acc[j][0]);
                        acc[j][0] = __ffma2_rn(cv, make_float2(X[0], X[1]), acc[j][0]);
                        acc[j][1] = __ffma2_rn(sv, make_float2(D[2], D[3]), acc[j][1]);
                        acc[j][1] = __ffma2_rn(cv, make_float2(X[2], X[3]), acc[j][1]);
                    };
                    fold(D0, X0, 0);
                    if constexpr (GS == 32) fold(D1, X1, 1);
                }
            }
            // Release the slot; the last warp to release it refills it with stage t + stages.
            __syncwarp();
            if (lane == 0) {
                uint32_t prev;
                asm volatile("atom.acq_rel.cta.shared::cta.add.u32 %0, [%1], 1;"
                             : "=r"(prev)
                             : "r"(smem_u32(&released[s]))
                             : "memory");
                if (prev == kMmaWarps - 1) {
                    released[s] = 0;
                    const int tn = t + p.stages;
                    if (tn < total && !abort_flag) {
                        fence_proxy_async_smem();  // the generic reads of the slot before the copies into it
                        io.weights(tn, block_of(tn));
                        io.activations(tn);
                        atomicMax(&issued_total, tn + 1);
                    }
                }
            }
        }

        // The eight block warps of each half meet in shared memory; warp w sums
        // tile w of the row block over them in block order.
        float* mine = scratch + warp * (TPW * 4 * 32);
#pragma unroll
        for (int j = 0; j < TPW; ++j) {
            mine[(j * 4 + 0) * 32 + lane] = acc[j][0].x;
            mine[(j * 4 + 1) * 32 + lane] = acc[j][0].y;
            mine[(j * 4 + 2) * 32 + lane] = acc[j][1].x;
            mine[(j * 4 + 3) * 32 + lane] = acc[j][1].y;
        }
        __syncthreads();
        const int tile = warp;  // 2 TPW <= 16 tiles per row block: at most one per warp
        if (ok && tile < 2 * TPW) {
            const int h = tile / TPW, jl = tile - h * TPW;
            float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            for (int b = 0; b < kBlocks; ++b) {
                const float* src = scratch + (b * kHalves + h) * (TPW * 4 * 32) + jl * 4 * 32 + lane;
#pragma unroll
                for (int k = 0; k < 4; ++k) v[k] += src[k * 32];
            }
            // epilogue: tokens g and g + 8 x rows n and n + 1
            const int n = rb * p.rows + 8 * tile + 2 * q;
            const bool ok0 = n < p.N, ok1 = n + 1 < p.N;
            const float bi0 = (ok0 && p.bias) ? bf16f(p.bias[n]) : 0.0f;
            const float bi1 = (ok1 && p.bias) ? bf16f(p.bias[n + 1]) : 0.0f;
            const float g0 = (ok0 && p.gate) ? bf16f(p.gate[n]) : 1.0f;
            const float g1 = (ok1 && p.gate) ? bf16f(p.gate[n + 1]) : 1.0f;
            const bool gelu = (p.flags & (Q6_EPI_GELU | Q6_EPI_GELU_PRECISE)) != 0;
            const bool precise = (p.flags & Q6_EPI_GELU_PRECISE) != 0;
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                const int m = g + 8 * hh;
                if (m >= p.M || !ok0) continue;
                float v0 = v[2 * hh] + bi0, v1 = v[2 * hh + 1] + bi1;
                if (gelu) {
                    v0 = gelu_select(v0, precise);
                    v1 = gelu_select(v1, precise);
                }
                v0 *= g0;
                v1 *= g1;
                const size_t off = static_cast<size_t>(m) * p.N + n;
                if (p.residual) {
                    v0 += bf16f(p.residual[off]);
                    if (ok1) v1 += bf16f(p.residual[off + 1]);
                }
                const uint32_t w = pack_bf16x2(v0, v1);
                if (ok1 && (reinterpret_cast<uintptr_t>(p.y + off) & 3) == 0) {
                    *reinterpret_cast<uint32_t*>(p.y + off) = w;
                } else {
                    p.y[off] = static_cast<uint16_t>(w & 0xFFFFu);
                    if (ok1) p.y[off + 1] = static_cast<uint16_t>(w >> 16);
                }
            }
        }
        __syncthreads();  // the scratch is free again
    }
    // Copies in flight land before the CTA exits (bounded).
    if (threadIdx.x == 0) {
        const int issued = issued_total;
        for (int t = issued > p.stages ? issued - p.stages : 0; t < issued; ++t)
            mbar_wait_drain(smem_u32(full + t % p.stages), static_cast<uint32_t>((t / p.stages) & 1));
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
            uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle) {
    auto fn = sk_encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    return fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// n8 tiles per row block, one of 2, 4, 8, 12, 16 (1, 2, 4, 6, 8 per warp):
// the smallest that spreads the rows over the SMs in one round, 16 at most.
// Q6_SKINNY_TILES (one of those counts) overrides.
int plan_tiles(int64_t N) {
    static const int kChoices[] = {2, 4, 8, 12, 16};
    if (const char* v = std::getenv("Q6_SKINNY_TILES")) {
        const int t = std::atoi(v);
        for (int c : kChoices)
            if (t == c) return t;
    }
    const int64_t sms = device_sm_count();
    const int64_t per = ((N + 7) / 8 + sms - 1) / sms;  // tiles per SM for one round
    for (int c : kChoices)
        if (c >= per) return c;
    return kMaxTiles;
}

template <int GS, int TPW>
int launch_skinny_t(const LinearArgs& a, cudaStream_t stream) {
    const SkGeom geo = sk_geometry(2 * TPW, GS);
    if (geo.stages < 2) return Q6_ERR_UNSUPPORTED;
    static std::atomic<bool> attr_set_for_device[kMaxDevices];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return Q6_ERR_CUDA;
    if (dev < 0 || dev >= kMaxDevices) return Q6_ERR_UNSUPPORTED;
    if (!attr_set_for_device[dev].load(std::memory_order_acquire)) {
        if (cudaFuncSetAttribute(skinny_kernel<GS, TPW>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBudget) !=
            cudaSuccess)
            return Q6_ERR_CUDA;
        attr_set_for_device[dev].store(true, std::memory_order_release);
    }
    const uint64_t words = static_cast<uint64_t>(a.K) * 6 / 32;
    const uint64_t groups = static_cast<uint64_t>(a.K / GS);
    const uint32_t m = static_cast<uint32_t>(a.M);
    CUtensorMap tx, tw, ts, tb;
    if (!sk_map(&tx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.x, a.K, a.M, a.K * 2, 64, m, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !sk_map(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT32, a.w, words, a.N, words * 4, kCodeRowWords, geo.rows,
                CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !sk_map(&ts, CU_TENSOR_MAP_DATA_TYPE_UINT16, a.scales, groups, a.N, groups * 2, geo.sb_groups, geo.rows,
                CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !sk_map(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT16, a.qbiases, groups, a.N, groups * 2, geo.sb_groups, geo.rows,
                CU_TENSOR_MAP_SWIZZLE_NONE))
        return Q6_ERR_CUDA;
    SkParams p;
    p.bias = a.bias;
    p.gate = a.gate;
    p.residual = a.residual;
    p.y = static_cast<uint16_t*>(a.y);
    p.M = static_cast<int>(a.M);
    p.N = static_cast<int>(a.N);
    p.K = static_cast<int>(a.K);
    p.flags = a.flags;
    p.gs_shift = GS == 32 ? 5 : (GS == 64 ? 6 : 7);
    p.rows = geo.rows;
    p.sb_groups = geo.sb_groups;
    p.code_bytes = geo.code_bytes;
    p.sb_bytes = geo.sb_bytes;
    p.stage_bytes = geo.stage_bytes;
    p.stages = geo.stages;
    p.row_blocks = static_cast<int>((a.N + geo.rows - 1) / geo.rows);
    p.x_box_bytes = m * 128u;
    p.exp_pair = 0x43004300u;
    const int grid = std::min(p.row_blocks, device_sm_count());
    const cudaError_t err = launch_pdl(skinny_kernel<GS, TPW>, dim3(static_cast<unsigned>(grid)), dim3(kThreads),
                                       geo.smem_bytes, stream, tx, tw, ts, tb, p);
    return err == cudaSuccess ? Q6_OK : Q6_ERR_CUDA;
}

template <int GS>
int launch_skinny_gs(const LinearArgs& a, cudaStream_t stream) {
    switch (plan_tiles(a.N)) {
        case 2: return launch_skinny_t<GS, 1>(a, stream);
        case 4: return launch_skinny_t<GS, 2>(a, stream);
        case 8: return launch_skinny_t<GS, 4>(a, stream);
        case 12: return launch_skinny_t<GS, 6>(a, stream);
        default: return launch_skinny_t<GS, 8>(a, stream);
    }
}

}  // namespace

bool skinny_supported(const LinearArgs& a) {
    if (a.M < 1 || a.M > kTok || a.lora_rank != 0) return false;
    if (a.group_size != 32 && a.group_size != 64 && a.group_size != 128) return false;
    if (a.K % kChunk != 0 || (a.K / a.group_size) % 8 != 0) return false;
    if (a.K > (int64_t(1) << 24) || a.N > (int64_t(1) << 30)) return false;
    const uintptr_t al = reinterpret_cast<uintptr_t>(a.x) | reinterpret_cast<uintptr_t>(a.w) |
                         reinterpret_cast<uintptr_t>(a.scales) | reinterpret_cast<uintptr_t>(a.qbiases);
    return al % 16 == 0;
}

int launch_skinny(const LinearArgs& a, cudaStream_t stream) {
    switch (a.group_size) {
        case 32: return launch_skinny_gs<32>(a, stream);
        case 64: return launch_skinny_gs<64>(a, stream);
        default: return launch_skinny_gs<128>(a, stream);
    }
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
