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
//     128-byte swizzling into shared memory (K-major, two 64-wide boxes per
//     stage);
//   * the fp32 accumulator D (128 lanes x NT columns) sits in TMEM; epilogue
//     warps read it with tcgen05.ld, add bias, apply GELU / residual gate and
//     store bf16 rows of y.
//
// One pipeline stage covers K = 128 (eight K=16 MMAs).  The single thread that
// issues the MMAs is on the critical path (each tcgen05.mma and
// tcgen05.commit holds it for tens of cycles), so a stage costs it exactly one
// barrier wait ("ready": activations landed and the A tile is in TMEM) and one
// commit ("done": releases the activation slot and the TMEM A slot).
//
// Three TMA rings feed the stage: activations (one producer thread), packed
// codes (a second producer thread, deeper ring since codes are small), and
// scales / biases in chunks of 8 groups (issued by the code producer; each
// chunk serves 2 to 8 stages).  Shapes whose scale rows are not 16-byte
// aligned read scales with per-lane global loads instead.
//
// Warp roles: warp 0 activation producer, warp 1 MMA issuer, warp 2 TMEM
// allocator, warp 3 code + scale producer, warps 4-7 epilogue, warps 8-23
// dequant (two sets of eight warps; set s takes the stages g % 2 == s and is
// the only writer of TMEM A slot s and of the code slots of that parity - a
// layout in which three sets rotating over two A slots showed rare corrupted
// tiles at K = 12288, while one owner per slot never did).  The CTA is
// persistent over (token tile, weight tile) pairs; accumulators are double
// buffered when NT <= 192 so the epilogue of one tile overlaps the main loop of
// the next.  Every mbarrier wait is bounded (q6_ptx.cuh).
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

constexpr int kRows = 128;                               // weight rows per tile (MMA M)
constexpr int kBK = 128;                                 // K per pipeline stage
constexpr int kBoxK = 64;                                // K per activation TMA box (128-byte swizzle span)
constexpr int kCodeRowBytes = kBK * 6 / 8;               // 96 bytes of codes per row per stage
constexpr int kCodeStageBytes = kRows * kCodeRowBytes;   // 12288
constexpr int kCodeWordsPerStage = kBK * 6 / 32;         // 24
// Stage g is announced to the MMA issuer by one barrier, ready[g % kRing]
// (the activation TMA bytes plus one arrival per dequant warp of the stage),
// and handed back by one MMA commit, done[g % kRing], which frees both its
// activation slot (g % kXStages) and its TMEM A slot (g % kAStages).  Every
// agent that waits on done for stage g - d (d <= kRing) has already seen
// stage g - d - 1 or earlier complete, and every agent that arrives on
// ready for stage g has seen done(g - kRing) or later, so no wait or arrival
// can be taken by a phase kRing stages away.
constexpr int kRing = 8;
constexpr int kAColsPerStage = kBK / 2;                  // bf16x2 per 32-bit column
constexpr int kControlThreads = 256;                     // warps 0-3 control, warps 4-7 epilogue
constexpr int kSmemBudget = 227 * 1024;
constexpr int kBarrierBytes = 512;

constexpr int kDqWarpsPerSet = 8;                      // two warps per TMEM lane quarter
constexpr int kDqSets = 2;                              // set s dequantises the stages g % 2 == s
constexpr int kDqWarps = kDqWarpsPerSet * kDqSets;

// Scales and biases reach shared memory as TMA boxes of 8 groups (16 bytes,
// the smallest TMA row) x 128 weight rows, one box each per chunk of 8
// groups (2, 4 or 8 stages for group sizes 32, 64, 128), in a ring of two
// chunk slots.
constexpr int kSbGroups = 8;
constexpr int kSbBoxBytes = kRows * kSbGroups * 2;     // 2048
constexpr int kSbSlotBytes = 2 * kSbBoxBytes;          // scales box + biases box
constexpr int kSbSlots = 2;

__host__ __device__ constexpr int tc_threads(int dq_sets) { return kControlThreads + 32 * kDqWarpsPerSet * dq_sets; }

constexpr int pow2_at_least(int v) {
    int p = 32;
    while (p < v) p <<= 1;
    return p;
}

constexpr int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

// kPair: a cluster of two CTAs shares each cta_group::2 MMA (M = 256 weight
// rows, 128 per CTA); each CTA stages only its half of the NT activation rows.
template <int NT, bool kPair = false>
struct Cfg {
    static_assert(NT % 16 == 0 && NT >= 16 && NT <= 256, "MMA N must be a multiple of 16 in [16, 256]");
    static constexpr int kAStages = 2;  // TMEM ring of dequantised A tiles, one slot per dequant set
    static constexpr int kNAcc = (2 * NT + kAStages * kAColsPerStage <= 512) ? 2 : 1;
    static constexpr int kXRows = kPair ? NT / 2 : NT;  // activation rows this CTA stages
    static constexpr int kXBoxBytes = kXRows * 128;     // kXRows rows of 64 bf16
    static constexpr int kXStageBytes = 2 * kXBoxBytes;
    static constexpr int kUsable = kSmemBudget - 1024 - kBarrierBytes;
    static constexpr int kXStages = clampi((kUsable * 2 / 3) / kXStageBytes, 2, 8);
    // even, so that with two dequant sets every code slot belongs to one set
    static constexpr int kCStages =
        clampi((kUsable - kXStages * kXStageBytes - kSbSlots * kSbSlotBytes) / kCodeStageBytes, 2, 12) & ~1;
    static constexpr int kSmemBytes = 1024 + kXStages * kXStageBytes + kCStages * kCodeStageBytes +
                                      kSbSlots * kSbSlotBytes + kBarrierBytes;
    static constexpr int kAccCols = kNAcc * NT;
    static constexpr int kTmemCols = pow2_at_least(kAccCols + kAStages * kAColsPerStage);
    static constexpr uint32_t kIdesc = idesc_bf16_f32(kPair ? 2 * kRows : kRows, NT);
    static_assert(kSmemBytes <= kSmemBudget, "shared memory budget");
    static_assert(kXStages <= kRing && kRing % kAStages == 0, "stage barrier ring");
    static_assert(kTmemCols <= 512, "TMEM budget");
    static_assert(kXBoxBytes % 1024 == 0, "activation boxes must stay 1024-byte aligned");
};

// Epilogue variants, chosen on the host so that the per-element loop carries
// no flag tests: bias only, bias + GELU, and the general form (optional
// GELU, gate and residual).
constexpr int kEpiPlain = 0;
constexpr int kEpiGelu = 1;
constexpr int kEpiGeneral = 2;

struct TcParams {
    const uint16_t* scales;
    const uint16_t* qbiases;
    const uint16_t* bias;
    const uint16_t* residual;
    const uint16_t* gate;
    uint16_t* y;
    int M, N, K, gs, gs_shift, groups, flags;
    int sb_shift;  // log2(stages per 8-group chunk) when scales are TMA-staged
    int tiles_n, num_tiles, k_stages, last_ksteps;
    // LoRA delta s * (xa @ B) (xa = x @ A, bf16 [M, r]; B bf16 [r, N]): two
    // extra stages per tile after the q6 stages, each covering r / 2 of the
    // rank (lora_ksteps = r / 32 MMAs of K = 16, r <= 256 so a stage fits
    // the two 64-wide activation boxes), with A(TMEM)[n, j] =
    // bf16(s * B[j, n]) and the activation boxes loaded from xa.  0 stages
    // without LoRA.  Two stages keep every stage's parity, so each dequant
    // set still owns the code slots of its parity.
    const uint16_t* lora_b;
    float lora_scale;
    int lora_rank, lora_stages, lora_ksteps;
    int lora_b_nmajor;  // lora_b is [N, r]: 16-byte loads of an output row's rank values
    SpliceExp3 sexp;  // splice exponent words, runtime values so each splice is one instruction
    // Split-K: work item it covers tile it / ksplit and the q6 stages
    // [s * ks_per, min((s + 1) * ks_per, k_stages)) of split s = it % ksplit
    // (ks_per a multiple of the stages per staged scale chunk, so chunks never
    // straddle splits).  With
    // ksplit > 1 the epilogue stores fp32 partials [ksplit][M][N] and a second
    // kernel sums them in split order and applies the epilogue.
    int ksplit, ks_per, num_items;
    float* partial;
};

struct Item {
    int mb, nb, split, ks0, ks1, lora;
    __device__ __forceinline__ int stages() const { return ks1 - ks0 + lora; }
    // q6 stage of local index l, or k_stages + (LoRA stage index) past ks1
    __device__ __forceinline__ int ks_of(int l, int k_stages) const {
        return l < ks1 - ks0 ? ks0 + l : k_stages + (l - (ks1 - ks0));
    }
};

__device__ __forceinline__ Item item_at(const TcParams& p, int it) {
    Item I;
    const int tile = it / p.ksplit;
    I.split = it - tile * p.ksplit;
    I.mb = tile / p.tiles_n;
    I.nb = tile - I.mb * p.tiles_n;
    I.ks0 = I.split * p.ks_per;
    I.ks1 = I.ks0 + p.ks_per < p.k_stages ? I.ks0 + p.ks_per : p.k_stages;
    I.lora = I.split == p.ksplit - 1 ? p.lora_stages : 0;  // the LoRA delta once per tile
    return I;
}

__device__ __forceinline__ float bf16f(uint16_t v) { return __uint_as_float(static_cast<uint32_t>(v) << 16); }

// Warp-uniform bounded wait: every lane polls, the warp proceeds only if all succeeded.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, int site) {
    const bool ok = mbar_wait(bar, parity, abort_flag, site);
    return __all_sync(0xffffffffu, ok);
}

template <int NT, bool kSbTma, int kEpi, bool kPair>
__global__ void __launch_bounds__(tc_threads(kDqSets), 1)
    q6_linear_tc_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                        const __grid_constant__ CUtensorMap tmap_s, const __grid_constant__ CUtensorMap tmap_b,
                        const __grid_constant__ CUtensorMap tmap_xa, const TcParams p) {
    using C = Cfg<NT, kPair>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_align_up<1024>(smem_raw);
    uint8_t* x_smem = smem;
    uint8_t* c_smem = smem + C::kXStages * C::kXStageBytes;
    uint8_t* sb_smem = c_smem + C::kCStages * kCodeStageBytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sb_smem + kSbSlots * kSbSlotBytes);
    uint64_t* ready = bars;            // [kRing] activations landed + A tile in TMEM
    uint64_t* done = ready + kRing;    // [kRing] MMAs of the stage retired
    uint64_t* c_full = done + kRing;
    uint64_t* c_empty = c_full + C::kCStages;
    uint64_t* s_full = c_empty + C::kCStages;  // [kSbSlots] scale chunk landed
    uint64_t* s_empty = s_full + kSbSlots;     // [kSbSlots] every dequant warp is done with it
    uint64_t* acc_full = s_empty + kSbSlots;
    uint64_t* acc_empty = acc_full + C::kNAcc;
    uint64_t* drain = acc_empty + C::kNAcc;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // CTA pairs: rank 0 issues the MMAs of both; work items are per pair, and
    // this CTA's weight rows are the (rank)th 128 of the pair's 256.
    const uint32_t rank = kPair ? cluster_ctarank() : 0u;
    const bool leader = rank == 0;
    const int it0 = kPair ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
    const int istep = kPair ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);
    constexpr int kTileRows = kPair ? 2 * kRows : kRows;
    const int row0 = static_cast<int>(rank) * kRows;
    constexpr int kPeers = kPair ? 2 : 1;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kRing; ++s) {
            mbar_init(smem_u32(ready + s), 1 + kPeers * kDqWarpsPerSet);  // activation producer + dequant sets
            mbar_init(smem_u32(done + s), 1);                    // MMA commit
        }
        for (int s = 0; s < C::kCStages; ++s) {
            mbar_init(smem_u32(c_full + s), 1);
            mbar_init(smem_u32(c_empty + s), kDqWarpsPerSet);  // the warps of the dequant set that read it
        }
        for (int s = 0; s < kSbSlots; ++s) {
            mbar_init(smem_u32(s_full + s), 1);
            mbar_init(smem_u32(s_empty + s), kDqWarps);
        }
        for (int s = 0; s < C::kNAcc; ++s) {
            mbar_init(smem_u32(acc_full + s), 1);
            mbar_init(smem_u32(acc_empty + s), 4 * kPeers);
        }
        mbar_init(smem_u32(drain), 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 2) {
        if constexpr (kPair) {
            tmem_alloc_pair(smem_u32(tmem_slot), C::kTmemCols);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(smem_u32(tmem_slot), C::kTmemCols);
            tmem_relinquish();
        }
    }
    tc_fence_before();
    __syncthreads();
    if constexpr (kPair) cluster_sync();  // both CTAs' barriers exist before any cross-CTA arrival
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    pdl_launch_dependents();

    if (warp == 0) {
        // ------------------------------------------------ activation producer
        if (lane == 0) {
            tma_prefetch_map(&tmap_x);
            if (p.lora_stages) tma_prefetch_map(&tmap_xa);
            pdl_wait();  // the activations may come from the previous kernel
            uint32_t g = 0;  // stage counter over all tiles of this CTA
            int s = 0;       // g % kXStages
            bool ok = true;
            for (int it = it0; it < p.num_items && ok; it += istep) {
                const Item I = item_at(p, it);
                const int mb = I.mb;
                for (int l = 0; l < I.stages(); ++l, ++g) {
                    const int ks = I.ks_of(l, p.k_stages);
                    // x slot s was last read by the MMAs of stage g - kXStages.
                    if (g >= static_cast<uint32_t>(C::kXStages)) {
                        const uint32_t prev = g - C::kXStages;
                        if (!mbar_wait(smem_u32(done + prev % kRing), (prev / kRing) & 1u, abort_flag, 1)) {
                            ok = false;
                            break;
                        }
                    }
                    const uint32_t fb = smem_u32(ready + g % kRing);
                    const uint32_t dst = smem_u32(x_smem + s * C::kXStageBytes);
                    if constexpr (kPair) {
                        // Each CTA loads its half of the token rows; both halves count
                        // on the leader's barrier, which expects the pair's bytes.
                        const uint32_t fbc = mapa_shared(fb, 0);
                        const int y0 = mb * NT + static_cast<int>(rank) * C::kXRows;
                        if (ks < p.k_stages) {
                            if (leader) mbar_arrive_expect_tx(fb, 2u * C::kXStageBytes);
                            tma_load_2d_pair(dst, &tmap_x, fbc, ks * kBK, y0);
                            tma_load_2d_pair(dst + C::kXBoxBytes, &tmap_x, fbc, ks * kBK + kBoxK, y0);
                        } else {
                            const int x0 = (ks - p.k_stages) * (p.lora_rank / 2);
                            const bool two = p.lora_rank > 2 * kBoxK;
                            if (leader) mbar_arrive_expect_tx(fb, 2u * (two ? C::kXStageBytes : C::kXBoxBytes));
                            tma_load_2d_pair(dst, &tmap_xa, fbc, x0, y0);
                            if (two) tma_load_2d_pair(dst + C::kXBoxBytes, &tmap_xa, fbc, x0 + kBoxK, y0);
                        }
                    } else if (ks < p.k_stages) {
                        mbar_arrive_expect_tx(fb, C::kXStageBytes);
                        tma_load_2d(dst, &tmap_x, fb, ks * kBK, mb * NT);
                        tma_load_2d(dst + C::kXBoxBytes, &tmap_x, fb, ks * kBK + kBoxK, mb * NT);
                    } else {  // LoRA stage l: xa columns [l r/2, (l + 1) r/2), one box per 64
                        const int x0 = (ks - p.k_stages) * (p.lora_rank / 2);
                        const bool two = p.lora_rank > 2 * kBoxK;
                        mbar_arrive_expect_tx(fb, two ? C::kXStageBytes : C::kXBoxBytes);
                        tma_load_2d(dst, &tmap_xa, fb, x0, mb * NT);
                        if (two) tma_load_2d(dst + C::kXBoxBytes, &tmap_xa, fb, x0 + kBoxK, mb * NT);
                    }
                    if (++s == C::kXStages) s = 0;
                }
            }
            // Every issued copy must land before this CTA may exit: wait until
            // the MMAs of the last stages retired (they read those copies).
            const uint32_t tail = g < static_cast<uint32_t>(C::kXStages) ? g : C::kXStages;
            for (uint32_t i = 0; i < tail; ++i) {
                const uint32_t L = g - 1 - i;
                mbar_wait_drain(smem_u32(done + L % kRing), (L / kRing) & 1u);
            }
        }
    } else if (warp == 3) {
        // ------------------------------------------------ code producer
        if (lane == 0) {
            tma_prefetch_map(&tmap_w);
            if constexpr (kSbTma) {
                tma_prefetch_map(&tmap_s);
                tma_prefetch_map(&tmap_b);
            }
            int s = 0;
            uint32_t ph = 0;
            long issued = 0;
            int ss = 0;
            uint32_t sph = 0;
            long s_issued = 0;
            bool ok = true;
            for (int it = it0; it < p.num_items && ok; it += istep) {
                const Item I = item_at(p, it);
                const int nb = I.nb;
                for (int ks = I.ks0; ks < I.ks1; ++ks) {
                    if (kSbTma && (ks & ((1 << p.sb_shift) - 1)) == 0) {
                        // first stage of a chunk: its scales and biases
                        if (!mbar_wait(smem_u32(s_empty + ss), sph ^ 1u, abort_flag, 9)) {
                            ok = false;
                            break;
                        }
                        const uint32_t fb = smem_u32(s_full + ss);
                        const uint32_t dst = smem_u32(sb_smem + ss * kSbSlotBytes);
                        const int gx = (ks >> p.sb_shift) * kSbGroups;
                        mbar_arrive_expect_tx(fb, kSbSlotBytes);
                        tma_load_2d(dst, &tmap_s, fb, gx, nb * kTileRows + row0);
                        tma_load_2d(dst + kSbBoxBytes, &tmap_b, fb, gx, nb * kTileRows + row0);
                        ++s_issued;
                        if (++ss == kSbSlots) {
                            ss = 0;
                            sph ^= 1u;
                        }
                    }
                    if (!mbar_wait(smem_u32(c_empty + s), ph ^ 1u, abort_flag, 8)) {
                        ok = false;
                        break;
                    }
                    const uint32_t fb = smem_u32(c_full + s);
                    mbar_arrive_expect_tx(fb, kCodeStageBytes);
                    tma_load_2d(smem_u32(c_smem + s * kCodeStageBytes), &tmap_w, fb, ks * kCodeWordsPerStage,
                                nb * kTileRows + row0);
                    ++issued;
                    if (++s == C::kCStages) {
                        s = 0;
                        ph ^= 1u;
                    }
                }
            }
            const long tail = issued < C::kCStages ? issued : C::kCStages;
            for (long i = 0; i < tail; ++i) {
                const long L = issued - 1 - i;
                mbar_wait_drain(smem_u32(c_full + (L % C::kCStages)), static_cast<uint32_t>((L / C::kCStages) & 1));
            }
            const long s_tail = s_issued < kSbSlots ? s_issued : kSbSlots;
            for (long i = 0; i < s_tail; ++i) {
                const long L = s_issued - 1 - i;
                mbar_wait_drain(smem_u32(s_full + (L % kSbSlots)), static_cast<uint32_t>((L / kSbSlots) & 1));
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        // The whole warp runs the loop, so every operand is warp-uniform and
        // stays in uniform registers; one elected lane (the same one each time,
        // which its commits require) issues each stage's tcgen05.mma and commit.  With
        // the loop on lane 0 alone, each MMA cost ~100 cycles of issue and each
        // stage ~380 cycles between its commit and the next stage's first MMA,
        // whatever the MMA's size.
        if (leader) {
            const uint64_t desc_base = sdesc_kmajor_sw128(smem_u32(x_smem));
            const uint32_t desc_lo = static_cast<uint32_t>(desc_base);
            const uint32_t desc_hi = static_cast<uint32_t>(desc_base >> 32);
            const uint32_t a_base = tmem_base + static_cast<uint32_t>(C::kAccCols);
            uint32_t g = 0;  // stage counter over all tiles of this CTA
            int xs = 0, acc = 0;
            uint32_t accph = 0;
            bool ok = true;
            for (int it = it0; it < p.num_items && ok; it += istep) {
                const Item I = item_at(p, it);
                if (!warp_wait(smem_u32(acc_empty + acc), accph ^ 1u, abort_flag, 2)) break;
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * NT);
                for (int l = 0; l < I.stages(); ++l, ++g) {
                    const int ks = I.ks_of(l, p.k_stages);
                    const uint32_t rs = g % kRing;
                    if (!warp_wait(smem_u32(ready + rs), (g / kRing) & 1u, abort_flag, 3)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t lo = desc_lo + static_cast<uint32_t>(xs * (C::kXStageBytes >> 4));
                    const uint32_t a_tmem = a_base + (rs % C::kAStages) * kAColsPerStage;
                    const uint32_t first = l != 0 ? 1u : 0u;
                    // K step kk reads activation box kk / 4 at 32-byte offset kk % 4
                    // and TMEM A columns 8 kk .. 8 kk + 7.
                    auto issue = [&](int kk) {
                        const uint32_t off = static_cast<uint32_t>((kk / 4) * (C::kXBoxBytes >> 4) + (kk % 4) * 2);
                        if constexpr (kPair)
                            mma_bf16_ts_pair(d_tmem, a_tmem + kk * 8, make_desc(lo + off, desc_hi), C::kIdesc,
                                             kk == 0 ? first : 1u);
                        else
                            mma_bf16_ts(d_tmem, a_tmem + kk * 8, make_desc(lo + off, desc_hi), C::kIdesc,
                                        kk == 0 ? first : 1u);
                    };
                    if (elect_one()) {  // one lane issues the stage's MMAs and its commit
                        if (ks + 1 < p.k_stages || (ks + 1 == p.k_stages && p.last_ksteps == kBK / 16)) {
#pragma unroll
                            for (int kk = 0; kk < kBK / 16; ++kk) issue(kk);
                        } else if (ks < p.k_stages) {  // K % 128 == 64 tail: the first box only
#pragma unroll
                            for (int kk = 0; kk < kBK / 32; ++kk) issue(kk);
                        } else {  // LoRA stage: r / 32 K-steps (the second box once r > 128)
                            for (int kk = 0; kk < p.lora_ksteps; ++kk) issue(kk);
                        }
                        if constexpr (kPair)
                            tc_commit_pair(smem_u32(done + rs), 3);
                        else
                            tc_commit(smem_u32(done + rs));
                    }
                    __syncwarp();
                    if (++xs == C::kXStages) xs = 0;
                }
                if (!ok) break;
                if (elect_one()) {
                    if constexpr (kPair)
                        tc_commit_pair(smem_u32(acc_full + acc), 3);
                    else
                        tc_commit(smem_u32(acc_full + acc));
                }
                __syncwarp();
                if (++acc == C::kNAcc) {
                    acc = 0;
                    accph ^= 1u;
                }
            }
            // All issued MMAs complete before TMEM may be released.
            if (elect_one()) {
                if constexpr (kPair)
                    tc_commit_pair(smem_u32(drain), 1);
                else
                    tc_commit(smem_u32(drain));
                mbar_wait_drain(smem_u32(drain), 0);
            }
            __syncwarp();
        }
    } else if (warp >= 4 && warp < 8) {
        // ------------------------------------------------ epilogue
        constexpr int kChunk = 16;  // accumulator columns per tcgen05.ld (16 keeps the epilogue within registers)
        static_assert(NT % kChunk == 0, "token tile must be a multiple of the load width");
        const int q = warp & 3;
        const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
        const bool gelu = kEpi == kEpiGelu || (kEpi == kEpiGeneral && (p.flags & Q6_EPI_GELU) != 0);
        const bool precise = kEpi == kEpiGeneral && (p.flags & Q6_EPI_GELU_PRECISE) != 0;
        // Paired stores: lanes 2i and 2i+1 swap one value so that each writes a
        // 32-bit word holding two adjacent output columns (even lane: token j,
        // odd lane: token j+1).  Needs an even row length and 4-byte aligned y.
        const bool paired = (p.N % 2 == 0) && ((reinterpret_cast<uintptr_t>(p.y) & 3) == 0) &&
                            ((reinterpret_cast<uintptr_t>(p.residual) & 3) == 0);
        const bool odd = (lane & 1) != 0;
        pdl_wait();  // y, the residual, the gate and the partials may be the previous kernel's
        int acc = 0;
        uint32_t accph = 0;
        for (int it = it0; it < p.num_items; it += istep) {
            const Item I = item_at(p, it);
            const int mb = I.mb;
            const int nb = I.nb;
            const int n = nb * kTileRows + row0 + q * 32 + lane;
            const bool n_ok = n < p.N;
            const float bias_n = (n_ok && p.bias) ? bf16f(p.bias[n]) : 0.0f;
            const float gate_n = (n_ok && p.gate) ? bf16f(p.gate[n]) : 1.0f;
            // the gate of the two columns of this lane's paired word (n & ~1, n | 1)
            const int ne = n & ~1;
            const float2 gate_w = (n_ok && p.gate) ? make_float2(bf16f(p.gate[ne]), bf16f(p.gate[ne + 1]))
                                                   : make_float2(1.0f, 1.0f);
            if (!warp_wait(smem_u32(acc_full + acc), accph, abort_flag, 5)) break;
            tc_fence_after();
#pragma unroll 1
            for (int c = 0; c < NT / kChunk; ++c) {
                uint32_t v[kChunk];
                const uint32_t taddr = tmem_base + lane_base + static_cast<uint32_t>(acc * NT + c * kChunk);
                tmem_ld_32x32b_x16(taddr, v);
                tmem_wait_ld();
                const int m0 = mb * NT + c * kChunk;
                if (p.ksplit > 1) {
                    // split-K partial: fp32, epilogue applied after the sum
                    float* dst = p.partial + (static_cast<size_t>(I.split) * p.M + m0) * p.N + n;
#pragma unroll
                    for (int j = 0; j < kChunk; ++j)
                        if (n_ok && m0 + j < p.M) dst[static_cast<size_t>(j) * p.N] = __uint_as_float(v[j]);
                    continue;
                }
                if (kEpi != kEpiGeneral && paired && m0 + kChunk <= p.M) {
                    // Whole chunk inside the token range: one paired 32-bit store
                    // per token pair, the row pointer advanced by two rows each time.
                    uint32_t* yp = reinterpret_cast<uint32_t*>(p.y + static_cast<size_t>(m0 + (odd ? 1 : 0)) * p.N +
                                                               (n & ~1));
                    const size_t step = static_cast<size_t>(p.N);  // two rows in 32-bit words
#pragma unroll
                    for (int j = 0; j < kChunk; j += 2) {
                        float2 val = __fadd2_rn(make_float2(__uint_as_float(v[j]), __uint_as_float(v[j + 1])),
                                                make_float2(bias_n, bias_n));
                        if constexpr (kEpi == kEpiGelu) val = gelu_tanh2(val);
                        const float send = odd ? val.x : val.y;
                        const float recv = __shfl_xor_sync(0xffffffffu, send, 1);
                        const uint32_t word = pack_bf16x2(odd ? recv : val.x, odd ? val.y : recv);
                        if (n_ok) *yp = word;
                        yp += step;
                    }
                    continue;
                }
                if (kEpi == kEpiGeneral && paired) {
                    // Paired words as above; the gate and the residual act on the
                    // word's two columns: one 32-bit residual load per store.  All
                    // the chunk's residual words are loaded before its first store
                    // (y may alias the residual, so loads after a store would wait
                    // for it: one memory round trip per chunk instead of per word).
                    uint32_t rw[kChunk / 2];
#pragma unroll
                    for (int j = 0; j < kChunk; j += 2) {
                        const int row = m0 + j + (odd ? 1 : 0);
                        rw[j / 2] = (p.residual && n_ok && row < p.M)
                                        ? *reinterpret_cast<const uint32_t*>(p.residual + static_cast<size_t>(row) * p.N + ne)
                                        : 0u;
                    }
#pragma unroll
                    for (int j = 0; j < kChunk; j += 2) {
                        float2 val = make_float2(__uint_as_float(v[j]) + bias_n, __uint_as_float(v[j + 1]) + bias_n);
                        if (gelu) val = gelu_tanh2_select(val, precise);
                        const float send = odd ? val.x : val.y;
                        const float recv = __shfl_xor_sync(0xffffffffu, send, 1);
                        const int row = m0 + j + (odd ? 1 : 0);
                        float2 w2 = odd ? make_float2(recv, val.y) : make_float2(val.x, recv);
                        if (p.gate) w2 = __fmul2_rn(w2, gate_w);
                        if (p.residual) {
                            const uint32_t r = rw[j / 2];
                            w2 = __fadd2_rn(w2, make_float2(__uint_as_float(r << 16), __uint_as_float(r & 0xFFFF0000u)));
                        }
                        if (n_ok && row < p.M)
                            *reinterpret_cast<uint32_t*>(p.y + static_cast<size_t>(row) * p.N + ne) =
                                pack_bf16x2(w2.x, w2.y);
                    }
                    continue;
                }
#pragma unroll
                for (int j = 0; j < kChunk; j += 2) {
                    // tokens m0 + j (x) and m0 + j + 1 (y) of this lane's column n
                    float2 val = make_float2(__uint_as_float(v[j]) + bias_n, __uint_as_float(v[j + 1]) + bias_n);
                    if (gelu) val = gelu_tanh2_select(val, precise);
                    if (kEpi == kEpiGeneral && p.gate) val = __fmul2_rn(val, make_float2(gate_n, gate_n));
                    if (kEpi == kEpiGeneral && p.residual && n_ok) {
                        const size_t off = static_cast<size_t>(m0 + j) * p.N + n;
                        if (m0 + j < p.M) val.x += bf16f(p.residual[off]);
                        if (m0 + j + 1 < p.M) val.y += bf16f(p.residual[off + p.N]);
                    }
                    if (paired) {
                        const float send = odd ? val.x : val.y;
                        const float recv = __shfl_xor_sync(0xffffffffu, send, 1);
                        const int row = m0 + j + (odd ? 1 : 0);
                        const uint32_t word = odd ? pack_bf16x2(recv, val.y) : pack_bf16x2(val.x, recv);
                        if (n_ok && row < p.M)
                            *reinterpret_cast<uint32_t*>(p.y + static_cast<size_t>(row) * p.N + (n & ~1)) = word;
                    } else if (n_ok) {
                        const size_t off = static_cast<size_t>(m0 + j) * p.N + n;
                        const uint32_t word = pack_bf16x2(val.x, val.y);
                        if (m0 + j < p.M) p.y[off] = static_cast<uint16_t>(word & 0xFFFFu);
                        if (m0 + j + 1 < p.M) p.y[off + p.N] = static_cast<uint16_t>(word >> 16);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if constexpr (kPair)
                    mbar_arrive_cluster(mapa_shared(smem_u32(acc_empty + acc), 0));
                else
                    mbar_arrive(smem_u32(acc_empty + acc));
            }
            if (++acc == C::kNAcc) {
                acc = 0;
                accph ^= 1u;
            }
        }
    } else if (warp >= 8) {
        // ------------------------------------------------ dequant -> TMEM
        // Two sets of eight warps.  Set s takes the stages g with g % 2 == s,
        // so it alone writes A slot s and code slots of its parity.  Within a
        // set, warp (half h, lane quarter q) expands K half h of the stage
        // (64 codes, TMEM columns 32h..32h+31) for the 32 weight rows of q.
        const int dw = warp - 8;
        const int set = dw >> 3;
        const int half = (dw >> 2) & 1;
        const int q = warp & 3;
        const int r = q * 32 + lane;
        const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
        uint32_t gstage = 0;  // stage counter over all tiles of this CTA
        uint32_t gqstage = 0; // q6 (code-carrying) stage counter: the code ring's index
        uint32_t gchunk = 0;  // scale chunk counter over all tiles of this CTA
        bool ok = true;
        for (int it = it0; it < p.num_items && ok; it += istep) {
            const Item I = item_at(p, it);
            const int nb = I.nb;
            const int n = nb * kTileRows + row0 + r;
            const bool n_ok = n < p.N;
            const uint16_t* srow = p.scales + static_cast<size_t>(n_ok ? n : 0) * p.groups;
            const uint16_t* brow = p.qbiases + static_cast<size_t>(n_ok ? n : 0) * p.groups;
            // Scale and bias of the two 32-code quarters of this warp's K half
            // of stage ks: one group for group sizes 64 and 128, two adjacent
            // groups for 32.  A half beyond K (a K % 128 == 64 tail) gets 0.
            // Staged path: group gi of the current chunk slot; otherwise a
            // global load per lane, issued one stage of this set ahead.
            auto load_sb = [&](int ks, const uint8_t* slot, float (&sb)[4]) {
                const int k = ks * kBK + half * 64;
                const bool in = n_ok && k < p.K;
                const int g = in ? (k >> p.gs_shift) : 0;
                if constexpr (kSbTma) {
                    const int gi = g & (kSbGroups - 1);
                    const uint16_t* srow_s = reinterpret_cast<const uint16_t*>(slot) + r * kSbGroups;
                    const uint16_t* brow_s = srow_s + kSbBoxBytes / 2;
                    sb[0] = in ? bf16f(srow_s[gi]) : 0.0f;
                    sb[1] = in ? bf16f(brow_s[gi]) : 0.0f;
                    if (p.gs == 32) {
                        sb[2] = in ? bf16f(srow_s[gi + 1]) : 0.0f;
                        sb[3] = in ? bf16f(brow_s[gi + 1]) : 0.0f;
                    } else {
                        sb[2] = sb[0];
                        sb[3] = sb[1];
                    }
                } else {
                    (void)slot;
                    sb[0] = in ? bf16f(__ldg(srow + g)) : 0.0f;
                    sb[1] = in ? bf16f(__ldg(brow + g)) : 0.0f;
                    if (p.gs == 32) {
                        sb[2] = in ? bf16f(__ldg(srow + g + 1)) : 0.0f;
                        sb[3] = in ? bf16f(__ldg(brow + g + 1)) : 0.0f;
                    } else {
                        sb[2] = sb[0];
                        sb[3] = sb[1];
                    }
                }
            };
            const uint32_t g_base = gstage;
            const uint32_t gq_base = gqstage;
            gstage += static_cast<uint32_t>(I.stages());
            gqstage += static_cast<uint32_t>(I.ks1 - I.ks0);
            int ks = I.ks0 + static_cast<int>((static_cast<uint32_t>(set) + kDqSets - g_base % kDqSets) % kDqSets);
            float sb_next[4];
            if (!kSbTma && ks < I.ks1) load_sb(ks, nullptr, sb_next);
            // Chunks of 8 scale groups (the whole tile when scales are not staged).
            // Every dequant warp takes every chunk slot and hands it back, also a
            // chunk that holds none of its stages, so that each s_empty phase
            // counts exactly one arrival per warp.
            const int chunk_len = kSbTma ? (1 << p.sb_shift) : p.k_stages;
            const int c_first = kSbTma ? (I.ks0 >> p.sb_shift) : 0;
            const int c_last = kSbTma ? (I.ks1 + chunk_len - 1) >> p.sb_shift : 1;
            for (int j = c_first; j < c_last && ok; ++j, ++gchunk) {
                const int ks_end = kSbTma ? ((j + 1) * chunk_len < I.ks1 ? (j + 1) * chunk_len : I.ks1) : I.ks1;
                const uint8_t* slot = sb_smem + (gchunk % kSbSlots) * kSbSlotBytes;
                if constexpr (kSbTma) {
                    if (!warp_wait(smem_u32(s_full + gchunk % kSbSlots), (gchunk / kSbSlots) & 1u, abort_flag, 10)) {
                        ok = false;
                        break;
                    }
                }
                for (; ks < ks_end; ks += kDqSets) {
                    const uint32_t g = g_base + static_cast<uint32_t>(ks - I.ks0);
                    const uint32_t gq = gq_base + static_cast<uint32_t>(ks - I.ks0);
                    const int cs = static_cast<int>(gq % C::kCStages);
                    const uint32_t cph = (gq / C::kCStages) & 1u;
                    const int as = static_cast<int>(g % C::kAStages);
                    const uint32_t rs = g % kRing;
                    float sb[4];
                    if constexpr (kSbTma) {
                        load_sb(ks, slot, sb);
                    } else {
#pragma unroll
                        for (int i = 0; i < 4; ++i) sb[i] = sb_next[i];
                        if (ks + kDqSets < I.ks1) load_sb(ks + kDqSets, nullptr, sb_next);
                    }
                    if (!warp_wait(smem_u32(c_full + cs), cph, abort_flag, 6)) {
                        ok = false;
                        break;
                    }
                    const uint4* src =
                        reinterpret_cast<const uint4*>(c_smem + cs * kCodeStageBytes + r * kCodeRowBytes) + half * 3;
                    const uint4 c0 = src[0], c1 = src[1], c2 = src[2];
                    __syncwarp();
                    if (lane == 0) mbar_arrive(smem_u32(c_empty + cs));
                    uint32_t a[32];
                    // Folded-offset dequant unless a lane's group needs the exact path.
                    const FoldedBias f0 = fold_bias(sb[0], sb[1]);
                    const FoldedBias f1 = fold_bias(sb[2], sb[3]);
                    if (__all_sync(0xffffffffu, f0.exact && f1.exact)) {
                        dequant16_bf16x2_fold(c0.x, c0.y, c0.z, sb[0], f0.b, p.sexp, a);
                        dequant16_bf16x2_fold(c0.w, c1.x, c1.y, sb[0], f0.b, p.sexp, a + 8);
                        dequant16_bf16x2_fold(c1.z, c1.w, c2.x, sb[2], f1.b, p.sexp, a + 16);
                        dequant16_bf16x2_fold(c2.y, c2.z, c2.w, sb[2], f1.b, p.sexp, a + 24);
                    } else {
                        dequant16_bf16x2_e3(c0.x, c0.y, c0.z, sb[0], sb[1], p.sexp, a);
                        dequant16_bf16x2_e3(c0.w, c1.x, c1.y, sb[0], sb[1], p.sexp, a + 8);
                        dequant16_bf16x2_e3(c1.z, c1.w, c2.x, sb[2], sb[3], p.sexp, a + 16);
                        dequant16_bf16x2_e3(c2.y, c2.z, c2.w, sb[2], sb[3], p.sexp, a + 24);
                    }
                    // A slot `as` was last read by the MMAs of stage g - C::kAStages.
                    if (g >= static_cast<uint32_t>(C::kAStages)) {
                        const uint32_t prev = g - C::kAStages;
                        if (!warp_wait(smem_u32(done + prev % kRing), (prev / kRing) & 1u, abort_flag, 7)) {
                            ok = false;
                            break;
                        }
                    }
                    tc_fence_after();
                    tmem_st_32x32b_x32(
                        tmem_base + lane_base + static_cast<uint32_t>(C::kAccCols + as * kAColsPerStage + half * 32),
                        a);
                    tmem_wait_st();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) {
                    if constexpr (kPair)
                        mbar_arrive_cluster(mapa_shared(smem_u32(ready + rs), 0));
                    else
                        mbar_arrive(smem_u32(ready + rs));
                }
                }
                if constexpr (kSbTma) {
                    __syncwarp();
                    if (lane == 0) mbar_arrive(smem_u32(s_empty + gchunk % kSbSlots));
                }
            }
            // LoRA stages: A[n, k] = bf16(s * B[l r/2 + k, n]) for the r / 2 rank
            // columns of stage l (zero beyond), one coalesced row of B per k.
            for (; ok && ks < I.ks1 + I.lora; ks += kDqSets) {
                const uint32_t g = g_base + static_cast<uint32_t>(ks - I.ks0);
                const int as = static_cast<int>(g % C::kAStages);
                const uint32_t rs = g % kRing;
                const int half_r = p.lora_rank / 2;
                const int j0 = (ks - I.ks1) * half_r;
                if (g >= static_cast<uint32_t>(C::kAStages)) {
                    const uint32_t prev = g - C::kAStages;
                    if (!warp_wait(smem_u32(done + prev % kRing), (prev / kRing) & 1u, abort_flag, 7)) {
                        ok = false;
                        break;
                    }
                }
                tc_fence_after();
                // 16 columns (32 rank values) at a time: a register budget the
                // q6 stages of the same kernel can afford (one array of 32 here
                // made every variant spill in its dequant loop)
#pragma unroll 1
                for (int hh = 0; hh < 2; ++hh) {
                    uint32_t a[16];
                    if (p.lora_b_nmajor) {
                        // B^T row n: the 32 rank values of this slice are contiguous (four
                        // 16-byte loads); half_r is a multiple of 16, so an 8-value chunk
                        // lies wholly inside or outside the stage's rank range
                        const uint16_t* src =
                            p.lora_b + static_cast<size_t>(n_ok ? n : 0) * p.lora_rank + j0 + half * 64 + hh * 32;
#pragma unroll
                        for (int c8 = 0; c8 < 4; ++c8) {
                            const int k = half * 64 + hh * 32 + 8 * c8;
                            uint4 v = make_uint4(0u, 0u, 0u, 0u);
                            if (n_ok && k < half_r) v = __ldg(reinterpret_cast<const uint4*>(src + 8 * c8));
                            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                            for (int i = 0; i < 4; ++i)
                                a[4 * c8 + i] = pack_bf16x2(p.lora_scale * bf16f(static_cast<uint16_t>(w[i] & 0xFFFFu)),
                                                            p.lora_scale * bf16f(static_cast<uint16_t>(w[i] >> 16)));
                        }
                    } else {
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            const int k = half * 64 + hh * 32 + 2 * i;  // stage-local K of the pair
                            float v0 = 0.0f, v1 = 0.0f;
                            if (n_ok && k < half_r)
                                v0 = p.lora_scale * bf16f(p.lora_b[static_cast<size_t>(j0 + k) * p.N + n]);
                            if (n_ok && k + 1 < half_r)
                                v1 = p.lora_scale * bf16f(p.lora_b[static_cast<size_t>(j0 + k + 1) * p.N + n]);
                            a[i] = pack_bf16x2(v0, v1);
                        }
                    }
                    tmem_st_32x32b_x16(tmem_base + lane_base +
                                           static_cast<uint32_t>(C::kAccCols + as * kAColsPerStage + half * 32 + hh * 16),
                                       a);
                }
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    if constexpr (kPair)
                        mbar_arrive_cluster(mapa_shared(smem_u32(ready + rs), 0));
                    else
                        mbar_arrive(smem_u32(ready + rs));
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if constexpr (kPair) cluster_sync();  // the leader's MMAs into this CTA's tensor memory have retired
    if (warp == 2) {
        tc_fence_after();
        if constexpr (kPair)
            tmem_dealloc_pair(tmem_base, C::kTmemCols);
        else
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

bool make_map_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner, uint64_t outer,
                 uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle) {
    auto fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// Scales and biases can be TMA-staged when every row of them starts on a
// 16-byte boundary (groups a multiple of 8, 16-byte aligned bases).
bool sb_tma_ok(const LinearArgs& a) {
    const int64_t groups = a.K / a.group_size;
    return groups % kSbGroups == 0 && reinterpret_cast<uintptr_t>(a.scales) % 16 == 0 &&
           reinterpret_cast<uintptr_t>(a.qbiases) % 16 == 0;
}

// Split-K plan: how many K splits the tensor-core path uses at token tile
// NT, with stages per split a multiple of `align` (the stages one staged scale
// chunk covers: 2, 4 or 8 for group sizes 32, 64, 128; 1 without staging).
// One split when the tiles already fill half the GPU; otherwise the count that
// minimises waves x (stages per split + a fixed per-item cost of about 8
// stages), plus the reduce pass.  Q6_TC_KSPLIT (1..16) overrides the choice.
struct KSplit {
    int splits, stages_per_split;
};

KSplit plan_ksplit(int64_t M, int64_t N, int64_t K, int NT, int align) {
    const int64_t sms = device_sm_count();
    const int64_t tiles = ((M + NT - 1) / NT) * ((N + kRows - 1) / kRows);
    const int64_t k_stages = (K + kBK - 1) / kBK;
    auto per_split = [&](int64_t s) { return ((k_stages + s - 1) / s + align - 1) / align * align; };
    int want = 0;
    if (const char* v = std::getenv("Q6_TC_KSPLIT")) want = std::atoi(v);
    if (want >= 1 && want <= 16) {
        const int64_t ps = per_split(want);
        return KSplit{static_cast<int>((k_stages + ps - 1) / ps), static_cast<int>(ps)};
    }
    KSplit best{1, static_cast<int>(k_stages)};
    if (tiles * 2 > sms) return best;
    int64_t best_cost = ((tiles + sms - 1) / sms) * (k_stages + 8);
    for (int64_t s = 2; s <= 16; ++s) {
        const int64_t ps = per_split(s);
        const int64_t splits = (k_stages + ps - 1) / ps;
        if (splits != s) continue;
        const int64_t cost = ((tiles * s + sms - 1) / sms) * (ps + 8) + 4;
        if (cost < best_cost) {
            best_cost = cost;
            best = KSplit{static_cast<int>(s), static_cast<int>(ps)};
        }
    }
    return best;
}

// Sums the split-K partials [splits][M][N] in split order and applies the
// epilogue of the tensor-core kernel: + bias, GELU, * gate, + residual, bf16.
__global__ void __launch_bounds__(256) splitk_reduce_kernel(const float* __restrict__ partial, int splits, int64_t M,
                                                           int64_t N, const uint16_t* bias, const uint16_t* gate,
                                                           const uint16_t* residual, int flags, uint16_t* y) {
    pdl_launch_dependents();
    pdl_wait();  // the partials of the kernel before
    const int64_t total = M * N;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t n = i % N;
        float v = 0.0f;
        for (int s = 0; s < splits; ++s) v += partial[s * total + i];
        if (bias) v += bf16f(bias[n]);
        if (flags & Q6_EPI_GELU) v = gelu_select(v, (flags & Q6_EPI_GELU_PRECISE) != 0);
        if (gate) v *= bf16f(gate[n]);
        if (residual) v += bf16f(residual[i]);
        y[i] = static_cast<uint16_t>(pack_bf16x2(v, 0.0f) & 0xFFFFu);
    }
}

// The same sum and epilogue, eight consecutive outputs per thread: 16-byte
// loads of the partials, bias, gate and residual and one 16-byte store
// (N % 8 == 0, every operand 16-byte aligned).  Each output is summed in split
// order exactly as above, so the results are bitwise those of the scalar kernel.
__device__ __forceinline__ void bf16x8_to_f32(uint4 w, float (&f)[8]) {
    const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        f[2 * j] = __uint_as_float(u[j] << 16);
        f[2 * j + 1] = __uint_as_float(u[j] & 0xFFFF0000u);
    }
}

__global__ void __launch_bounds__(256) splitk_reduce8_kernel(const float* __restrict__ partial, int splits, int64_t M,
                                                            int64_t N, const uint16_t* bias, const uint16_t* gate,
                                                            const uint16_t* residual, int flags, uint16_t* y) {
    pdl_launch_dependents();
    pdl_wait();  // the partials of the kernel before
    const int64_t total = M * N;
    const int64_t groups = total / 8;
    for (int64_t gi = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; gi < groups;
         gi += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t i = gi * 8;
        const int64_t n = i % N;
        float v[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
        for (int s = 0; s < splits; ++s) {
            const float4* src = reinterpret_cast<const float4*>(partial + s * total + i);
            const float4 a = src[0], b = src[1];
            v[0] += a.x; v[1] += a.y; v[2] += a.z; v[3] += a.w;
            v[4] += b.x; v[5] += b.y; v[6] += b.z; v[7] += b.w;
        }
        float t[8];
        if (bias) {
            bf16x8_to_f32(*reinterpret_cast<const uint4*>(bias + n), t);
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] += t[j];
        }
        if (flags & Q6_EPI_GELU) {
            const bool precise = (flags & Q6_EPI_GELU_PRECISE) != 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = gelu_select(v[j], precise);
        }
        if (gate) {
            bf16x8_to_f32(*reinterpret_cast<const uint4*>(gate + n), t);
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] *= t[j];
        }
        if (residual) {
            bf16x8_to_f32(*reinterpret_cast<const uint4*>(residual + i), t);
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] += t[j];
        }
        *reinterpret_cast<uint4*>(y + i) = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]),
                                                      pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
    }
}

// Launches a CTA-pair grid: clusters of two along x, with programmatic
// dependent launch when it is enabled.
template <typename... KArgs, typename... Args>
cudaError_t launch_pair_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                            Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Status of a CTA-pair launch that the device refused before anything ran
// (cluster size or co-scheduling not available); the caller falls back to
// one CTA per tile.
constexpr int kPairRefused = -1;

bool pair_launch_refused(cudaError_t e) {
    return e == cudaErrorInvalidClusterSize || e == cudaErrorLaunchOutOfResources || e == cudaErrorNotSupported;
}

std::atomic<long> g_pair_fallbacks{0};

template <int NT, bool kSbTma, int kEpi, bool kPair>
int launch_tc(const LinearArgs& a, cudaStream_t stream) {
    using C = Cfg<NT, kPair>;
    // Opt-in shared memory size, set once per device (idempotent, so two
    // threads racing to set it both succeed).
    static std::atomic<bool> attr_set_for_device[kMaxDevices];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return Q6_ERR_CUDA;
    if (dev < 0 || dev >= kMaxDevices) return Q6_ERR_UNSUPPORTED;
    if (!attr_set_for_device[dev].load(std::memory_order_acquire)) {
        if (cudaFuncSetAttribute(q6_linear_tc_kernel<NT, kSbTma, kEpi, kPair>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes) != cudaSuccess)
            return Q6_ERR_CUDA;
        attr_set_for_device[dev].store(true, std::memory_order_release);
    }
    CUtensorMap tmap_x, tmap_w, tmap_s, tmap_b, tmap_xa;
    if (!make_map_2d(&tmap_x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.x, a.K, a.M, a.K * 2, kBoxK, C::kXRows,
                     CU_TENSOR_MAP_SWIZZLE_128B))
        return Q6_ERR_CUDA;
    const uint64_t words = static_cast<uint64_t>(a.K) * 6 / 32;
    if (!make_map_2d(&tmap_w, CU_TENSOR_MAP_DATA_TYPE_UINT32, a.w, words, a.N, words * 4, kCodeWordsPerStage, kRows,
                     CU_TENSOR_MAP_SWIZZLE_NONE))
        return Q6_ERR_CUDA;
    const uint64_t groups = static_cast<uint64_t>(a.K / a.group_size);
    if constexpr (kSbTma) {
        if (!make_map_2d(&tmap_s, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.scales, groups, a.N, groups * 2, kSbGroups,
                         kRows, CU_TENSOR_MAP_SWIZZLE_NONE) ||
            !make_map_2d(&tmap_b, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.qbiases, groups, a.N, groups * 2, kSbGroups,
                         kRows, CU_TENSOR_MAP_SWIZZLE_NONE))
            return Q6_ERR_CUDA;
    } else {
        tmap_s = tmap_w;  // unused
        tmap_b = tmap_w;
    }
    if (a.lora_rank > 0) {
        if (!make_map_2d(&tmap_xa, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.lora_xa, a.lora_rank, a.M,
                         static_cast<uint64_t>(a.lora_rank) * 2, kBoxK, C::kXRows, CU_TENSOR_MAP_SWIZZLE_128B))
            return Q6_ERR_CUDA;
    } else {
        tmap_xa = tmap_x;  // unused
    }
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
    p.gs_shift = a.group_size == 32 ? 5 : (a.group_size == 64 ? 6 : 7);
    p.sb_shift = p.gs_shift - 4;  // 8 groups of gs codes = gs / 16 stages of 128
    p.groups = static_cast<int>(groups);
    p.flags = a.flags;
    constexpr int kTileRows = kPair ? 2 * kRows : kRows;  // weight rows per work item
    p.tiles_n = static_cast<int>((a.N + kTileRows - 1) / kTileRows);
    const int tiles_m = static_cast<int>((a.M + NT - 1) / NT);
    p.num_tiles = tiles_m * p.tiles_n;
    p.k_stages = static_cast<int>((a.K + kBK - 1) / kBK);
    p.last_ksteps = static_cast<int>((a.K - static_cast<int64_t>(p.k_stages - 1) * kBK) / 16);
    p.lora_b = a.lora_b;
    p.lora_scale = a.lora_scale;
    p.lora_rank = a.lora_rank;
    p.lora_stages = a.lora_rank > 0 ? 2 : 0;
    p.lora_ksteps = a.lora_rank / 32;
    p.lora_b_nmajor = (a.flags & Q6_LORA_B_NMAJOR) ? 1 : 0;
    p.sexp = splice_exp3_host();
    const KSplit ksp = kPair ? KSplit{1, p.k_stages} : plan_ksplit(a.M, a.N, a.K, NT, kSbTma ? (1 << p.sb_shift) : 1);
    const size_t need = static_cast<size_t>(ksp.splits) * a.M * a.N * sizeof(float);
    const bool split = ksp.splits > 1 && a.workspace && a.workspace_bytes >= need &&
                       reinterpret_cast<uintptr_t>(a.workspace) % 16 == 0;
    p.ksplit = split ? ksp.splits : 1;
    p.ks_per = split ? ksp.stages_per_split : p.k_stages;
    p.num_items = p.num_tiles * p.ksplit;
    p.partial = split ? static_cast<float*>(a.workspace) : nullptr;
    if constexpr (kPair) {
        const int pairs = std::min(p.num_items, device_sm_count() / 2);
        const cudaError_t e = launch_pair_pdl(q6_linear_tc_kernel<NT, kSbTma, kEpi, true>, dim3(2 * pairs),
                                              dim3(tc_threads(kDqSets)), C::kSmemBytes, stream, tmap_x, tmap_w,
                                              tmap_s, tmap_b, tmap_xa, p);
        if (e != cudaSuccess) return pair_launch_refused(e) ? kPairRefused : Q6_ERR_CUDA;
    } else {
        const int grid = std::min(p.num_items, device_sm_count());
        if (launch_pdl(q6_linear_tc_kernel<NT, kSbTma, kEpi, false>, dim3(grid), dim3(tc_threads(kDqSets)),
                       C::kSmemBytes, stream, tmap_x, tmap_w, tmap_s, tmap_b, tmap_xa, p) != cudaSuccess)
            return Q6_ERR_CUDA;
    }
    if (split) {
        const int64_t total = a.M * a.N;
        const uintptr_t al = reinterpret_cast<uintptr_t>(a.y) | reinterpret_cast<uintptr_t>(a.bias) |
                             reinterpret_cast<uintptr_t>(a.gate) | reinterpret_cast<uintptr_t>(a.residual);
        if (a.N % 8 == 0 && al % 16 == 0) {
            const int blocks =
                static_cast<int>(std::min<int64_t>((total / 8 + 255) / 256, int64_t(device_sm_count()) * 8));
            if (launch_pdl(splitk_reduce8_kernel, dim3(blocks), dim3(256), 0, stream,
                           static_cast<const float*>(p.partial), p.ksplit, a.M, a.N, a.bias, a.gate, a.residual,
                           a.flags, static_cast<uint16_t*>(a.y)) != cudaSuccess)
                return Q6_ERR_CUDA;
            return Q6_OK;
        }
        const int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, int64_t(device_sm_count()) * 8));
        if (launch_pdl(splitk_reduce_kernel, dim3(blocks), dim3(256), 0, stream,
                       static_cast<const float*>(p.partial), p.ksplit, a.M, a.N, a.bias, a.gate, a.residual, a.flags,
                       static_cast<uint16_t*>(a.y)) != cudaSuccess)
            return Q6_ERR_CUDA;
    }
    return Q6_OK;
}

// Staged scales with a specialised epilogue for the MLP's two shapes
// (bias + GELU, bias only); everything else takes the general epilogue.
template <int NT, bool kPair = false>
int launch_tc_sb(const LinearArgs& a, cudaStream_t stream) {
    if (!sb_tma_ok(a)) return launch_tc<NT, false, kEpiGeneral, kPair>(a, stream);
    if (a.residual || a.gate || (a.flags & Q6_EPI_GELU_PRECISE)) return launch_tc<NT, true, kEpiGeneral, kPair>(a, stream);
    if (a.flags & Q6_EPI_GELU) return launch_tc<NT, true, kEpiGelu, kPair>(a, stream);
    return launch_tc<NT, true, kEpiPlain, kPair>(a, stream);
}

// CTA pairs (one cta_group::2 MMA over 256 weight rows) for token tiles of
// 128 and more when the pairs' tiles fill every SM pair at least once (so no
// split-K plan is given up).  Q6_TC_PAIR=0 turns them off, =1 forces them.
bool pair_mode(const LinearArgs& a, int token_tile) {
    if (token_tile < 128) return false;
    const char* v = std::getenv("Q6_TC_PAIR");
    if (v && v[0] == '0') return false;
    if (v && v[0] == '1') return true;
    const int64_t pair_tiles = ((a.M + token_tile - 1) / token_tile) * ((a.N + 2 * kRows - 1) / (2 * kRows));
    return pair_tiles >= device_sm_count() / 2;
}

}  // namespace

long pair_fallbacks() { return g_pair_fallbacks.load(std::memory_order_relaxed); }

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
    if (a.K % kBoxK != 0) return false;
    if (a.lora_rank != 0) {
        // two LoRA stages of r / 2 rank columns each, within the stage's two 64-wide boxes
        if (a.lora_rank < 32 || a.lora_rank > 256 || a.lora_rank % 32 != 0) return false;
        if (!a.lora_xa || !a.lora_b || reinterpret_cast<uintptr_t>(a.lora_xa) % 16 != 0) return false;
    }
    if (a.M > (int64_t(1) << 30) || a.N > (int64_t(1) << 30) || a.K > (int64_t(1) << 24)) return false;
    if (reinterpret_cast<uintptr_t>(a.x) % 16 != 0) return false;
    if (reinterpret_cast<uintptr_t>(a.w) % 16 != 0) return false;
    return true;
}

size_t tc_workspace_bytes(int64_t M, int64_t N, int64_t K) {
    if (M <= 0 || N <= 0 || K <= 0) return 0;
    // the largest plan any group size (scale-chunk alignment) can choose
    size_t need = 0;
    for (int align : {1, 2, 4, 8}) {
        const KSplit ksp = plan_ksplit(M, N, K, choose_token_tile(M, N), align);
        if (ksp.splits > 1) need = std::max(need, static_cast<size_t>(ksp.splits) * M * N * sizeof(float));
    }
    return need;
}

int choose_token_tile(int64_t M, int64_t N) {
    if (const char* v = std::getenv("Q6_TC_TOKEN_TILE")) {
        const int t = std::atoi(v);
        if (t == 16 || t == 32 || t == 64 || t == 128 || t == 192 || t == 256) return t;
    }
    static const int kTiles[] = {256, 192, 128, 64, 32, 16};
    const int64_t sms = device_sm_count();
    const int64_t tiles_n = (N + kRows - 1) / kRows;
    // A tile costs about max(nt, floor) + 32 token-columns per K stage: below
    // ~128 tokens the dequantisation of its 128 weight rows, not the MMA, sets
    // the pace, so narrower tiles only multiply the dequantisation work (the
    // floor stops at M itself for a few token rows).
    const int64_t floor = std::min<int64_t>(128, (M + 15) / 16 * 16);
    int best = 16;
    int64_t best_cost = -1;
    for (int nt : kTiles) {
        const int64_t tiles = ((M + nt - 1) / nt) * tiles_n;
        const int64_t waves = (tiles + sms - 1) / sms;
        const int64_t cost = waves * (std::max<int64_t>(nt, floor) + 32);
        if (best_cost < 0 || cost < best_cost) {
            best_cost = cost;
            best = nt;
        }
    }
    return best;
}

int launch_linear_tc(const LinearArgs& a, int token_tile, cudaStream_t stream) {
    if (pair_mode(a, token_tile)) {
        int st = Q6_ERR_UNSUPPORTED;
        switch (token_tile) {
            case 256: st = launch_tc_sb<256, true>(a, stream); break;
            case 192: st = launch_tc_sb<192, true>(a, stream); break;
            case 128: st = launch_tc_sb<128, true>(a, stream); break;
            default: break;
        }
        if (st != kPairRefused) return st;
        // A device or context that cannot co-schedule two-CTA clusters refuses
        // the launch itself (nothing ran): clear that launch error, count the
        // fallback (q6_pair_fallbacks) and run one CTA per tile.  Any other
        // launch failure is returned as it is.
        (void)cudaGetLastError();
        g_pair_fallbacks.fetch_add(1, std::memory_order_relaxed);
    }
    switch (token_tile) {
        case 256: return launch_tc_sb<256>(a, stream);
        case 192: return launch_tc_sb<192>(a, stream);
        case 128: return launch_tc_sb<128>(a, stream);
        case 64: return launch_tc_sb<64>(a, stream);
        case 32: return launch_tc_sb<32>(a, stream);
        case 16: return launch_tc_sb<16>(a, stream);
        default: return Q6_ERR_UNSUPPORTED;
    }
}

}  // namespace q6
