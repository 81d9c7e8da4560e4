// q6 linear for a few token rows (M <= 16): warp-level MMA on the raw codes,
// K streamed in CTA-wide stages and split over the CTAs of a cluster.
//
// With a handful of token rows the linear is bound by reading the packed
// weights (0.8125 bytes per weight at group size 64), so the arithmetic per
// code must stay a few instructions, every SM must stream the same number of
// bytes, and HBM must stay busy.  The reference's
// sum_k x_k (scale * code_k + qbias) (shardedit_mlx/q6_metal_mlp.py:42-83) is
// evaluated per 64-code block of one scale group g as
//
//     scale_g * sum_k x_k (128 + code_k) + (qbias_g - 128 scale_g) * sum_k x_k
//
// where 128 + code is exact in bf16 (exponent 2^7, the code in the low
// mantissa bits), so both sums are exact-product bf16 MMAs with fp32
// accumulation (mma.sync m16n8k16): A = 128 + code for 16 weight rows, B =
// the token rows (one n8 tile for up to 8 tokens, two for 9-16, zero past M),
// and an A of ones gives the sums of x.  The weights keep the reference
// kernel's fp32 semantics (no bf16 rounding of scale * code + qbias), like the
// CUDA-core paths.
//
// Layout of the MMA K dimension.  Lane (g = lane / 4, q = lane % 4) owns the
// 16-code unit q (three packed words) of the block in weight rows g and g + 8
// of a tile.  The unit's codes pair up as (0,4) (1,5) (2,6) (3,7) (8,12)
// (9,13) (10,14) (11,15): a byte permute gathers two 4-code groups of the unit
// into one word, so a pair is a shift and one logic instruction (18
// instructions per 16 codes).  MMA K step s takes pairs 2s and 2s + 1; the K
// order inside the block is permuted, which the sum does not see, and the
// lane's activations are paired the same way with one byte permute each.
//
// Work and data movement.  A CTA owns a row block of 32 TPW weight rows
// (2 TPW tiles of 16) and a contiguous share of K: the S CTAs of a cluster
// split K between them, so that about one CTA per SM streams the same number
// of bytes (12288 x 3072: 96 row blocks of 128 rows over 48 clusters of 3;
// 3072 x 12288: 48 row blocks of 64 rows over 48 clusters of 3).  K streams
// through a ring of CTA-wide stages of 512 codes: one padded TMA code box
// ([rows x 100 words], 400-byte shared rows that put the rows a warp reads in
// different banks), eight 128-byte-swizzled activation boxes, the stage's
// scale and bias groups.  Warp (block b, group h) takes the 64-code block b of
// every stage for the tiles of group h, so each block's activations are
// loaded once per warp; the last of the sixteen warps to release a ring slot
// refills it.  At the end of a row block the warps' sums meet in the ring slot
// of the block's last stage (held back from its refill meanwhile) and are
// added in block order, the CTAs of the cluster add their partial sums in
// rank order through distributed shared memory, and the epilogue (bias,
// GELU, gate, residual) stores bf16.  Every sum runs in a fixed order, so
// the result does not depend on the row-block size or the cluster count.
// Every barrier wait is bounded.
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
#include <cstdio>
#include <mutex>

#include "q6_dequant.cuh"
#include "q6_internal.h"
#include "q6_ptx.cuh"

namespace q6 {
namespace {

constexpr int kBlocks = 8;                  // 64-code blocks per stage
constexpr int kChunk = 64 * kBlocks;        // codes per row per stage
constexpr int kGroups = 2;                  // warps per block, each with half of the row block's tiles
constexpr int kWarps = kBlocks * kGroups;
constexpr int kThreads = kWarps * 32;
constexpr int kTok = 16;                    // token rows at most (two n8 MMA tiles)
constexpr int kMaxSplit = 4;                // CTAs per cluster (K splits)
constexpr int kMaxStages = 4;
constexpr int kCodeRowWords = 100;          // words per shared code row: the stage's 96 and 4 of padding
constexpr int kSmemBudget = 227 * 1024 - 1024;  // dynamic shared memory (the kernel's statics stay below 1 KB)

struct SkGeom {
    int tpw;            // 16-row tiles per warp
    int nt;             // n8 token tiles
    int rows;           // weight rows per row block: 2 tpw tiles of 16
    int x_slot;         // shared bytes of one [tokens x 64] activation box
    int sb_groups;      // scale groups per stage box (>= 8)
    int code_bytes;     // per stage: rows x 400 bytes
    int sb_bytes;       // per stage, one of scales / biases
    int stage_bytes;    // activation boxes first (1024-byte aligned for the swizzle)
    int scratch_bytes;  // the warps' sums at the end of a row block (inside a ring slot)
    int part_stride;    // floats per token row of the CTA's partial sums
    int part_bytes;
    int stages;
    int smem_bytes;
};

__host__ __device__ constexpr int align_up(int v, int a) { return (v + a - 1) / a * a; }

__host__ __device__ constexpr SkGeom sk_geometry(int tpw, int gs, int nt) {
    SkGeom g{};
    g.tpw = tpw;
    g.nt = nt;
    g.rows = 16 * kGroups * tpw;
    g.x_slot = nt * 8 * 128;
    g.sb_groups = kChunk / gs > 8 ? kChunk / gs : 8;
    g.code_bytes = g.rows * kCodeRowWords * 4;
    g.sb_bytes = g.rows * g.sb_groups * 2;
    g.stage_bytes = align_up(kBlocks * g.x_slot + g.code_bytes + 2 * g.sb_bytes, 1024);
    g.scratch_bytes = kWarps * (4 * tpw * nt) * 32 * 4;
    g.part_stride = g.rows + 4;  // token rows 4 banks apart: conflict-free fragment stores
    g.part_bytes = 8 * nt * g.part_stride * 4;
    const int fixed = g.part_bytes + 1024 /* alignment */ + kMaxStages * 8 /* barriers */;
    g.stages = (kSmemBudget - fixed) / g.stage_bytes < kMaxStages ? (kSmemBudget - fixed) / g.stage_bytes : kMaxStages;
    g.smem_bytes = g.stages * g.stage_bytes + fixed;
    return g;
}

struct SkParams {
    const uint16_t* bias;
    const uint16_t* gate;
    const uint16_t* residual;
    uint16_t* y;
    int M, N, K, flags;
    int row_blocks;
    int split;             // CTAs per cluster, each with a contiguous share of the K stages
    uint32_t x_box_bytes;  // M rows x 128 bytes
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

__device__ __forceinline__ float ld_cluster_f32(uint32_t cluster_addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(cluster_addr) : "memory");
    return v;
}

// One 16-code unit (three packed words, 12 bytes) -> eight bf16x2 words
// (128 + code) holding the code pairs (0,4) (1,5) (2,6) (3,7) (8,12) (9,13)
// (10,14) (11,15).  Bytes 0-2, 3-5, 6-8, 9-11 each hold four codes at bits
// 0, 6, 12, 18; a byte permute puts bytes (0, 1) of one group and of the
// next into the two halves of a word, so codes 4j and 4j + 1 of both groups
// sit at bits 0 / 16 and 6 / 22, and bytes (1, 2) give codes 4j + 2, 4j + 3
// at bits 4 / 20 and 10 / 26.
__device__ __forceinline__ void unit_pairs(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t (&u)[8]) {
    constexpr uint32_t kMask = 0x003F003Fu;
    constexpr uint32_t kExp = 0x43004300u;  // bf16 2^7 in both halves
    const uint32_t r1 = __byte_perm(w0, w1, 0x4310);  // unit bytes 0, 1, 3, 4
    const uint32_t r2 = __byte_perm(w0, w1, 0x5421);  // unit bytes 1, 2, 4, 5
    const uint32_t r3 = __byte_perm(w1, w2, 0x6532);  // unit bytes 6, 7, 9, 10
    const uint32_t r4 = __byte_perm(w1, w2, 0x7643);  // unit bytes 7, 8, 10, 11
    u[0] = (r1 & kMask) | kExp;
    u[1] = ((r1 >> 6) & kMask) | kExp;
    u[2] = ((r2 >> 4) & kMask) | kExp;
    u[3] = ((r2 >> 10) & kMask) | kExp;
    u[4] = (r3 & kMask) | kExp;
    u[5] = ((r3 >> 6) & kMask) | kExp;
    u[6] = ((r4 >> 4) & kMask) | kExp;
    u[7] = ((r4 >> 10) & kMask) | kExp;
}

// The activations of a unit (x0..x7 in lo, x8..x15 in hi, bf16 pairs) paired
// like its codes: b[s] = the B fragment words of MMA K step s.
__device__ __forceinline__ void x_pairs(const uint4& lo, const uint4& hi, uint32_t (&b)[4][2]) {
    b[0][0] = __byte_perm(lo.x, lo.z, 0x5410);  // x0, x4
    b[0][1] = __byte_perm(lo.x, lo.z, 0x7632);  // x1, x5
    b[1][0] = __byte_perm(lo.y, lo.w, 0x5410);  // x2, x6
    b[1][1] = __byte_perm(lo.y, lo.w, 0x7632);  // x3, x7
    b[2][0] = __byte_perm(hi.x, hi.z, 0x5410);  // x8, x12
    b[2][1] = __byte_perm(hi.x, hi.z, 0x7632);  // x9, x13
    b[3][0] = __byte_perm(hi.y, hi.w, 0x5410);  // x10, x14
    b[3][1] = __byte_perm(hi.y, hi.w, 0x7632);  // x11, x15
}

// Refill of ring slot t % stages with stage t (one thread): the weights part
// (codes, scales, biases: never written by a kernel) and the activations part.
struct SkIssue {
    const CUtensorMap* tx;
    const CUtensorMap* tw;
    const CUtensorMap* ts;
    const CUtensorMap* tb;
    uint8_t* ring;
    uint64_t* full;
    int stages, stage_bytes, rows, code_bytes, sb_bytes, x_slot, groups_per_chunk;
    uint32_t tx_bytes;

    __device__ __forceinline__ void weights(int t, int rb, int c) const {
        const int s = t % stages;
        uint8_t* codes = ring + s * stage_bytes + kBlocks * x_slot;
        const uint32_t bar = smem_u32(full + s);
        const int r0 = rb * rows;
        mbar_arrive_expect_tx(bar, tx_bytes);
        tma_load_2d(smem_u32(codes), tw, bar, c * (kChunk * 6 / 32), r0);
        const int gbox = (c * groups_per_chunk) & ~7;  // 16-byte aligned box start
        tma_load_2d(smem_u32(codes + code_bytes), ts, bar, gbox, r0);
        tma_load_2d(smem_u32(codes + code_bytes + sb_bytes), tb, bar, gbox, r0);
    }
    __device__ __forceinline__ void activations(int t, int c) const {
        const int s = t % stages;
        uint8_t* st = ring + s * stage_bytes;
        const uint32_t bar = smem_u32(full + s);
#pragma unroll 1
        for (int b = 0; b < kBlocks; ++b) tma_load_2d(smem_u32(st + b * x_slot), tx, bar, c * kChunk + b * 64, 0);
    }
};

// GS: group size; TPW: 16-row tiles per warp (the row block holds 2 TPW);
// NT: n8 token tiles (1: M <= 8, 2: M <= 16).
template <int GS, int TPW, int NT>
__global__ void __launch_bounds__(kThreads, 1) skinny_kernel(const __grid_constant__ CUtensorMap tmap_x,
                                                            const __grid_constant__ CUtensorMap tmap_w,
                                                            const __grid_constant__ CUtensorMap tmap_s,
                                                            const __grid_constant__ CUtensorMap tmap_b,
                                                            const SkParams p) {
    constexpr int kE = 4 * TPW * NT;  // sums per lane: tiles x token tiles x (row g, row g + 8) x (token pair)
    constexpr int kGroupsPerBlock = GS == 32 ? 2 : 1;
    constexpr SkGeom G = sk_geometry(TPW, GS, NT);
    constexpr int kGsShift = GS == 32 ? 5 : (GS == 64 ? 6 : 7);
    static_assert(G.stages >= 2 && G.scratch_bytes <= G.stage_bytes, "ring too shallow");
    extern __shared__ uint8_t sk_raw[];
    uint8_t* ring = smem_align_up<1024>(sk_raw);
    float* part = reinterpret_cast<float*>(ring + G.stages * G.stage_bytes);
    uint64_t* full = reinterpret_cast<uint64_t*>(part + 8 * NT * G.part_stride);
    __shared__ int abort_flag;
    __shared__ uint32_t released[kMaxStages];  // warps done with the slot's current stage
    __shared__ int issued_total;               // stages whose copies were issued

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int S = p.split;
    const int rank = S > 1 ? static_cast<int>(cluster_ctarank()) : 0;
    const int cluster = static_cast<int>(blockIdx.x) / S;
    const int clusters = static_cast<int>(gridDim.x) / S;
    const int chunks = p.K / kChunk;
    const int k0 = rank * chunks / S;
    const int kc = (rank + 1) * chunks / S - k0;  // this CTA's stages per row block (>= 1)
    const int my_blocks = cluster < p.row_blocks ? (p.row_blocks - cluster + clusters - 1) / clusters : 0;
    const int total = my_blocks * kc;  // stages of this CTA
    SkIssue io;
    io.tx = &tmap_x;
    io.tw = &tmap_w;
    io.ts = &tmap_s;
    io.tb = &tmap_b;
    io.ring = ring;
    io.full = full;
    io.stages = G.stages;
    io.stage_bytes = G.stage_bytes;
    io.rows = G.rows;
    io.code_bytes = G.code_bytes;
    io.sb_bytes = G.sb_bytes;
    io.x_slot = G.x_slot;
    io.groups_per_chunk = kChunk / GS;
    io.tx_bytes = kBlocks * p.x_box_bytes + G.code_bytes + 2 * G.sb_bytes;
    auto block_of = [&](int t) { return cluster + (t / kc) * clusters; };
    auto chunk_of = [&](int t) { return k0 + t % kc; };
    // Stage t + stages refills the slot of stage t, except after the last
    // stage of a row block, whose slot holds the reduction first.
    auto refill_after = [&](int t) { return (t % kc) != kc - 1; };

    const int pre = total < G.stages ? total : G.stages;
    if (threadIdx.x == 0) {
        abort_flag = 0;
        issued_total = pre;
        for (int s = 0; s < kMaxStages; ++s) released[s] = 0;
        for (int s = 0; s < G.stages; ++s) mbar_init(smem_u32(full + s), 1);
        fence_mbar_init();
        tma_prefetch_map(&tmap_w);
        tma_prefetch_map(&tmap_x);
        for (int t = 0; t < pre; ++t) io.weights(t, block_of(t), chunk_of(t));  // before the dependency wait
    }
    pdl_launch_dependents();
    pdl_wait();  // x, the epilogue operands and y may belong to the previous kernel
    if (threadIdx.x == 0)
        for (int t = 0; t < pre; ++t) io.activations(t, chunk_of(t));
    __syncthreads();

    const int blk = warp % kBlocks;   // 64-code block of each stage
    const int grp = warp / kBlocks;   // tile group
    const int g = lane >> 2;
    const int q = lane & 3;
    const int tile0 = grp * TPW;      // first tile of this warp in the row block
    const uint32_t ones = 0x3F803F80u;  // bf16 (1, 1)
    const uint32_t mask0 = (GS == 32 && q >= 2) ? 0u : 0xFFFFFFFFu;  // group size 32: lanes of group 0
    const int ps = G.part_stride;
    bool ok = true;

    for (int rbi = 0; rbi < my_blocks; ++rbi) {
        const int rb = cluster + rbi * clusters;
        float2 acc[TPW][NT][2];  // [tile][token tile][row g, row g + 8]: tokens (2q, 2q + 1)
#pragma unroll
        for (int i = 0; i < TPW; ++i)
#pragma unroll
            for (int j = 0; j < NT; ++j) acc[i][j][0] = acc[i][j][1] = make_float2(0.0f, 0.0f);

        for (int c = 0; c < kc; ++c) {
            const int t = rbi * kc + c;
            const int s = t % G.stages;
            const uint8_t* st = ring + s * G.stage_bytes;
            if (ok && !__all_sync(0xffffffffu, mbar_wait(smem_u32(full + s), static_cast<uint32_t>((t / G.stages) & 1),
                                                         &abort_flag, Q6_SITE_GEMM_MAX)))
                ok = false;
            if (ok) {
                // B fragments of this block: token 8 j + g, the lane's unit q, paired like the codes
                uint32_t bx[NT][4][2];
                const uint8_t* xb = st + blk * G.x_slot;
#pragma unroll
                for (int j = 0; j < NT; ++j) {
                    const int tok = 8 * j + g;
                    const int sw = tok & 7;  // 128-byte swizzle of the token row
                    const uint8_t* row = xb + tok * 128;
                    const bool live = tok < p.M;
                    const uint4 z = make_uint4(0u, 0u, 0u, 0u);
                    const uint4 lo = live ? *reinterpret_cast<const uint4*>(row + 16 * ((2 * q) ^ sw)) : z;
                    const uint4 hi = live ? *reinterpret_cast<const uint4*>(row + 16 * ((2 * q + 1) ^ sw)) : z;
                    x_pairs(lo, hi, bx[j]);
                }
                // Sums of x over the block per token.  Group size 32: codes 0-31 of the
                // block are the units of lanes q = 0, 1 and codes 32-63 those of q = 2, 3,
                // so each group's sums take A operands zeroed in the other group's lanes.
                float X[NT][kGroupsPerBlock][4];
#pragma unroll
                for (int j = 0; j < NT; ++j) {
#pragma unroll
                    for (int gi = 0; gi < kGroupsPerBlock; ++gi) {
                        const uint32_t a = gi == 0 ? (ones & mask0) : (ones & ~mask0);
                        X[j][gi][0] = X[j][gi][1] = X[j][gi][2] = X[j][gi][3] = 0.0f;
#pragma unroll
                        for (int ks = 0; ks < 4; ++ks) mma_bf16_16816(X[j][gi], a, a, a, a, bx[j][ks][0], bx[j][ks][1]);
                    }
                }
                const uint32_t* codes = reinterpret_cast<const uint32_t*>(st + kBlocks * G.x_slot) +
                                        (16 * tile0 + g) * kCodeRowWords + blk * 12 + 3 * q;
                const uint16_t* scl = reinterpret_cast<const uint16_t*>(st + kBlocks * G.x_slot + G.code_bytes);
                const uint16_t* bia = scl + G.sb_bytes / 2;
                // scale group of this block within the stage's scale box; row g of tile 0
                const int cc = k0 + c;
                const int gin = (((cc * kChunk) >> kGsShift) & 7) + ((blk * 64) >> kGsShift);
                const uint16_t* scl0 = scl + (16 * tile0 + g) * G.sb_groups + gin;
                const uint16_t* bia0 = bia + (16 * tile0 + g) * G.sb_groups + gin;
#pragma unroll
                for (int i = 0; i < TPW; ++i) {
                    const uint32_t* u0 = codes + i * 16 * kCodeRowWords;  // row g of tile i
                    const uint32_t* u1 = u0 + 8 * kCodeRowWords;          // row g + 8
                    uint32_t lo[8], hi[8];
                    unit_pairs(u0[0], u0[1], u0[2], lo);
                    unit_pairs(u1[0], u1[1], u1[2], hi);
#pragma unroll
                    for (int gi = 0; gi < kGroupsPerBlock; ++gi) {
                        const uint32_t m = gi == 0 ? mask0 : ~mask0;
                        float D[NT][4];
#pragma unroll
                        for (int j = 0; j < NT; ++j) {
                            D[j][0] = D[j][1] = D[j][2] = D[j][3] = 0.0f;
#pragma unroll
                            for (int ks = 0; ks < 4; ++ks) {
                                if constexpr (GS == 32)
                                    mma_bf16_16816(D[j], lo[2 * ks] & m, hi[2 * ks] & m, lo[2 * ks + 1] & m,
                                                   hi[2 * ks + 1] & m, bx[j][ks][0], bx[j][ks][1]);
                                else
                                    mma_bf16_16816(D[j], lo[2 * ks], hi[2 * ks], lo[2 * ks + 1], hi[2 * ks + 1],
                                                   bx[j][ks][0], bx[j][ks][1]);
                            }
                        }
                        // acc += scale * sum x (128 + code) + (qbias - 128 scale) * sum x
                        const uint16_t* sp = scl0 + i * 16 * G.sb_groups + gi;
                        const uint16_t* bp = bia0 + i * 16 * G.sb_groups + gi;
                        const float2 sv = make_float2(bf16f(sp[0]), bf16f(sp[8 * G.sb_groups]));  // rows g, g + 8
                        const float2 bv = make_float2(bf16f(bp[0]), bf16f(bp[8 * G.sb_groups]));
                        const float2 cv = __ffma2_rn(make_float2(-128.0f, -128.0f), sv, bv);
#pragma unroll
                        for (int j = 0; j < NT; ++j) {
                            const float2 xs = make_float2(X[j][gi][0], X[j][gi][1]);
                            acc[i][j][0] = __ffma2_rn(make_float2(sv.x, sv.x), make_float2(D[j][0], D[j][1]),
                                                      acc[i][j][0]);
                            acc[i][j][0] = __ffma2_rn(make_float2(cv.x, cv.x), xs, acc[i][j][0]);
                            acc[i][j][1] = __ffma2_rn(make_float2(sv.y, sv.y), make_float2(D[j][2], D[j][3]),
                                                      acc[i][j][1]);
                            acc[i][j][1] = __ffma2_rn(make_float2(cv.y, cv.y), xs, acc[i][j][1]);
                        }
                    }
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
                if (prev == kWarps - 1) {
                    released[s] = 0;
                    const int tn = t + G.stages;
                    if (refill_after(t) && tn < total && !abort_flag) {
                        fence_proxy_async_smem();  // the generic reads of the slot before the copies into it
                        io.weights(tn, block_of(tn), chunk_of(tn));
                        io.activations(tn, chunk_of(tn));
                        atomicMax(&issued_total, tn + 1);
                    }
                }
            }
        }

        // The warps' sums meet in the ring slot of this row block's last stage
        // (every warp is done with it, and it is not refilled yet).
        const int t_last = rbi * kc + kc - 1;
        float* scratch = reinterpret_cast<float*>(ring + (t_last % G.stages) * G.stage_bytes);
        __syncthreads();
        {
            float* mine = scratch + warp * (kE * 32) + lane;
#pragma unroll
            for (int i = 0; i < TPW; ++i)
#pragma unroll
                for (int j = 0; j < NT; ++j)
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int e = ((i * NT + j) * 2 + h) * 2;
                        mine[e * 32] = acc[i][j][h].x;
                        mine[(e + 1) * 32] = acc[i][j][h].y;
                    }
        }
        __syncthreads();
        // CTA partial sums: the eight block warps of a tile group in block order,
        // into part[token][row].
        for (int idx = threadIdx.x; idx < kGroups * kE * 32; idx += kThreads) {
            const int gr = idx / (kE * 32);
            const int e = (idx / 32) % kE;
            const int l = idx % 32;
            float v = 0.0f;
#pragma unroll
            for (int b = 0; b < kBlocks; ++b) v += scratch[((gr * kBlocks + b) * kE + e) * 32 + l];
            const int comp = e & 1, h = (e >> 1) & 1, ij = e >> 2;
            const int i = ij / NT, j = ij % NT;
            const int row = 16 * (gr * TPW + i) + (l >> 2) + 8 * h;
            const int tok = 8 * j + 2 * (l & 3) + comp;
            part[tok * ps + row] = v;
        }
        __syncthreads();
        // The slot is free again: stage t_last + stages goes into it.
        if (threadIdx.x == 0) {
            const int tn = t_last + G.stages;
            if (tn < total && !abort_flag) {
                fence_proxy_async_smem();
                io.weights(tn, block_of(tn), chunk_of(tn));
                io.activations(tn, chunk_of(tn));
                atomicMax(&issued_total, tn + 1);
            }
        }
        if (S > 1) cluster_sync();  // every CTA's partial sums are written and visible
        // This CTA's share of the row block's outputs: the cluster's partial sums
        // in rank order, then the epilogue.  Token-major, so the stores coalesce.
        {
            const int tot = G.rows * p.M;
            const int lo = rank * tot / S, hi = (rank + 1) * tot / S;
            const bool gelu = (p.flags & (Q6_EPI_GELU | Q6_EPI_GELU_PRECISE)) != 0;
            const bool precise = (p.flags & Q6_EPI_GELU_PRECISE) != 0;
            for (int idx = lo + static_cast<int>(threadIdx.x); idx < hi; idx += kThreads) {
                const int tok = idx / G.rows;
                const int row = idx - tok * G.rows;
                const int n = rb * G.rows + row;
                if (n >= p.N) continue;
                const float* src = part + tok * ps + row;
                float v = 0.0f;
                for (int k = 0; k < S; ++k) v += k == rank ? *src : ld_cluster_f32(mapa_shared(smem_u32(src), k));
                if (!ok) continue;
                if (p.bias) v += bf16f(p.bias[n]);
                if (gelu) v = gelu_select(v, precise);
                if (p.gate) v *= bf16f(p.gate[n]);
                const size_t off = static_cast<size_t>(tok) * p.N + n;
                if (p.residual) v += bf16f(p.residual[off]);
                p.y[off] = static_cast<uint16_t>(pack_bf16x2(v, 0.0f) & 0xFFFFu);
            }
        }
        if (S > 1)
            cluster_sync();  // the peers are done reading this CTA's partial sums
        else
            __syncthreads();
    }
    // Copies in flight land before the CTA exits (bounded).
    if (threadIdx.x == 0) {
        const int issued = issued_total;
        for (int t = issued > G.stages ? issued - G.stages : 0; t < issued; ++t)
            mbar_wait_drain(smem_u32(full + t % G.stages), static_cast<uint32_t>((t / G.stages) & 1));
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

// Shared-memory attribute of one kernel instance, set once per device.
template <int GS, int TPW, int NT>
bool sk_prepare(int dev) {
    static std::atomic<bool> done[kMaxDevices];
    if (dev < 0 || dev >= kMaxDevices) return false;
    if (done[dev].load(std::memory_order_acquire)) return true;
    if (cudaFuncSetAttribute(skinny_kernel<GS, TPW, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBudget) !=
        cudaSuccess)
        return false;
    done[dev].store(true, std::memory_order_release);
    return true;
}

// Clusters of `split` CTAs that can be resident at once (cached per device).
template <int GS, int TPW, int NT>
int sk_cluster_capacity(int dev, int split, int smem) {
    static std::atomic<int> cache[kMaxDevices][kMaxSplit + 1];
    static std::atomic<bool> init[kMaxDevices][kMaxSplit + 1];
    if (init[dev][split].load(std::memory_order_acquire)) return cache[dev][split].load(std::memory_order_relaxed);
    int n = 0;
    if (split == 1) {
        int per_sm = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, skinny_kernel<GS, TPW, NT>, kThreads, smem) !=
            cudaSuccess)
            per_sm = 0;
        n = per_sm * device_sm_count();
    } else {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(static_cast<unsigned>(split * device_sm_count()));
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = static_cast<size_t>(smem);
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = static_cast<unsigned>(split);
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        if (cudaOccupancyMaxActiveClusters(&n, skinny_kernel<GS, TPW, NT>, &cfg) != cudaSuccess) {
            (void)cudaGetLastError();
            n = 0;
        }
    }
    cache[dev][split].store(n, std::memory_order_relaxed);
    init[dev][split].store(true, std::memory_order_release);
    return n;
}

struct SkPlan {
    int tpw = 0;
    int split = 1;
    int clusters = 0;
    double cost = 0.0;
};

// Estimated time of a (tpw, split) plan, in row-stages (128 rows x 512 codes
// take about 1.1 us of the kernel's issue-bound decode at 1.97 GHz): row blocks
// per cluster x rows x the CTA's stages, with the per-tile activation work of
// small tiles, the row block's reduction (more with a cluster's exchange) and
// the CTAs that share an SM counted on top.  Fitted to measured plans on B200
// (3072 -> 12288 and 12288 -> 3072, 1 and 16 rows).
inline double sk_cost(int64_t N, int chunks, int tpw, int split, int capacity, int* clusters_out) {
    const int rows = 32 * tpw;
    const int64_t rb = (N + rows - 1) / rows;
    const int64_t clusters = std::min<int64_t>(rb, capacity);
    if (clusters < 1) return -1.0;
    const int64_t per = (rb + clusters - 1) / clusters;
    const int kc = (chunks + split - 1) / split;
    const int64_t sms = std::max(1, device_sm_count());
    const double per_sm = std::max<double>(1.0, static_cast<double>((clusters * split + sms - 1) / sms));
    *clusters_out = static_cast<int>(clusters);
    return static_cast<double>(per) * rows * (kc * (1.0 + 0.25 / tpw) + (split > 1 ? 1.5 : 0.5)) * per_sm;
}

template <int GS, int TPW, int NT>
int launch_plan(const LinearArgs& a, int split, int clusters, cudaStream_t stream) {
    const SkGeom geo = sk_geometry(TPW, GS, NT);
    if (geo.stages < 2 || geo.scratch_bytes > geo.stage_bytes) return Q6_ERR_UNSUPPORTED;
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
    p.row_blocks = static_cast<int>((a.N + geo.rows - 1) / geo.rows);
    p.split = split;
    p.x_box_bytes = m * 128u;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(clusters * split));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = static_cast<size_t>(geo.smem_bytes);
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    int na = 0;
    if (split > 1) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = static_cast<unsigned>(split);
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = 1;
        ++na;
    }
    if (pdl_enabled()) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    cfg.attrs = attr;
    cfg.numAttrs = static_cast<unsigned>(na);
    const cudaError_t err = cudaLaunchKernelEx(&cfg, skinny_kernel<GS, TPW, NT>, tx, tw, ts, tb, p);
    return err == cudaSuccess ? Q6_OK : Q6_ERR_CUDA;
}

// Plan override: Q6_SKINNY_PLAN="tpw,split" (tpw 1-4; split 1-4).
bool sk_plan_override(int* tpw, int* split) {
    const char* v = std::getenv("Q6_SKINNY_PLAN");
    if (!v) return false;
    int t = 0, s = 0;
    if (std::sscanf(v, "%d,%d", &t, &s) != 2) return false;
    if (t < 1 || t > 4 || s < 1 || s > kMaxSplit) return false;
    *tpw = t;
    *split = s;
    return true;
}

template <int GS, int NT>
int sk_capacity(int dev, int tpw, int split) {
    const int smem = sk_geometry(tpw, GS, NT).smem_bytes;
    switch (tpw) {
        case 1: return sk_cluster_capacity<GS, 1, NT>(dev, split, smem);
        case 2: return sk_cluster_capacity<GS, 2, NT>(dev, split, smem);
        case 3: return sk_cluster_capacity<GS, 3, NT>(dev, split, smem);
        default: return sk_cluster_capacity<GS, 4, NT>(dev, split, smem);
    }
}

// The plan for a shape: Q6_SKINNY_PLAN if set, else the (tpw, split) of least
// estimated work per CTA over the clusters that fit at once.
template <int GS, int NT>
int sk_choose(const LinearArgs& a, int dev, SkPlan* best) {
    if (!sk_prepare<GS, 1, NT>(dev) || !sk_prepare<GS, 2, NT>(dev) || !sk_prepare<GS, 3, NT>(dev) ||
        !sk_prepare<GS, 4, NT>(dev))
        return Q6_ERR_CUDA;
    const int chunks = static_cast<int>(a.K / kChunk);
    *best = SkPlan{};
    int ot = 0, os = 0;
    if (sk_plan_override(&ot, &os)) {
        os = std::min(os, chunks);
        int cl = 0;
        if (sk_cost(a.N, chunks, ot, os, sk_capacity<GS, NT>(dev, ot, os), &cl) < 0.0) return Q6_ERR_UNSUPPORTED;
        best->tpw = ot;
        best->split = os;
        best->clusters = cl;
        return Q6_OK;
    }
    for (int tpw : {4, 3, 2, 1}) {
        const SkGeom geo = sk_geometry(tpw, GS, NT);
        if (geo.stages < 2 || geo.scratch_bytes > geo.stage_bytes) continue;
        for (int split = 1; split <= kMaxSplit && split <= chunks; ++split) {
            int cl = 0;
            const double cost = sk_cost(a.N, chunks, tpw, split, sk_capacity<GS, NT>(dev, tpw, split), &cl);
            if (cost < 0.0) continue;
            if (best->tpw == 0 || cost < best->cost * 0.999) {
                best->tpw = tpw;
                best->split = split;
                best->clusters = cl;
                best->cost = cost;
            }
        }
    }
    return best->tpw == 0 ? Q6_ERR_UNSUPPORTED : Q6_OK;
}

template <int GS, int NT>
int launch_skinny_nt(const LinearArgs& a, cudaStream_t stream) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return Q6_ERR_CUDA;
    if (dev < 0 || dev >= kMaxDevices) return Q6_ERR_UNSUPPORTED;
    SkPlan best;
    const int st = sk_choose<GS, NT>(a, dev, &best);
    if (st != Q6_OK) return st;
    auto go = [&](int split, int clusters) {
        switch (best.tpw) {
            case 1: return launch_plan<GS, 1, NT>(a, split, clusters, stream);
            case 2: return launch_plan<GS, 2, NT>(a, split, clusters, stream);
            case 3: return launch_plan<GS, 3, NT>(a, split, clusters, stream);
            default: return launch_plan<GS, 4, NT>(a, split, clusters, stream);
        }
    };
    int rc = go(best.split, best.clusters);
    if (rc == Q6_ERR_CUDA && best.split > 1) {
        // A cluster launch the device refused: one CTA per row block instead.
        (void)cudaGetLastError();
        const int rows = 32 * best.tpw;
        const int rb = static_cast<int>((a.N + rows - 1) / rows);
        rc = go(1, std::min(rb, std::max(1, sk_capacity<GS, NT>(dev, best.tpw, 1))));
    }
    return rc;
}

template <int GS>
int launch_skinny_gs(const LinearArgs& a, cudaStream_t stream) {
    return a.M <= 8 ? launch_skinny_nt<GS, 1>(a, stream) : launch_skinny_nt<GS, 2>(a, stream);
}

template <int GS>
int plan_gs(const LinearArgs& a, int* tpw, int* split, int* clusters) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return Q6_ERR_CUDA;
    if (dev < 0 || dev >= kMaxDevices) return Q6_ERR_UNSUPPORTED;
    SkPlan best;
    const int st = a.M <= 8 ? sk_choose<GS, 1>(a, dev, &best) : sk_choose<GS, 2>(a, dev, &best);
    if (st != Q6_OK) return st;
    *tpw = best.tpw;
    *split = best.split;
    *clusters = best.clusters;
    return Q6_OK;
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

int skinny_plan(const LinearArgs& a, int* tpw, int* split, int* clusters) {
    switch (a.group_size) {
        case 32: return plan_gs<32>(a, tpw, split, clusters);
        case 64: return plan_gs<64>(a, tpw, split, clusters);
        default: return plan_gs<128>(a, tpw, split, clusters);
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
