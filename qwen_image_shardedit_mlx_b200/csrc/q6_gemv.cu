// q6 linear for a few token rows (M <= 4): a memory-streaming GEMV.
//
// With one to four activation rows the linear is bound by reading the packed
// weights (0.8125 bytes per weight with scales and biases).  The kernel keeps
// HBM busy by decoupling loads from arithmetic:
//
//   * every warp works through pairs of weight rows (rows 2p, 2p+1), in
//     K chunks of up to 4096 codes; a stage is one (pair, chunk): both rows'
//     codes, scales and biases;
//   * each warp owns a two-slot ring in shared memory (three slots when the
//     shared memory holds one CTA per SM either way); its lane 0 fetches the
//     next stages with 1-D bulk copies (completing on the slot's mbarrier)
//     while the warp computes the current one, so one or two stages per warp
//     are always in flight;
//   * within a stage, lane l takes the 16-code units j = l, l + 32, ... of
//     both rows (K = 3072: six units per lane, an even split);
//   * the reference kernel's sum_k x_k (scale * code_k + qbias)
//     (shardedit_mlx/q6_metal_mlp.py:42-83) is evaluated per 16-code unit
//     (within one scale group) as scale * sum_k x_k code_k + qbias * sum_k x_k.
//     One shift per code pair puts the pair at bits 11 and 17, where a splice
//     reads 4096 + code (even) and 64 + code (odd); packed FFMA2s accumulate
//     sum_k x_k (offset_k + code_k) in (even, odd) halves, and the offsets
//     leave again once per unit through the per-unit sums of x over even and
//     odd codes (computed once per CTA, with the plain x sum).  Relative to
//     the exact integer dot this costs about 1e-5 of the unit's magnitude.
//     The activations sit in shared memory as fp32 with an XOR swizzle that
//     keeps the unit-per-lane reads free of bank conflicts.
//
// Requirements (else the CUDA-core linear_simt_kernel runs): bf16 activations
// and output, K % 64 == 0, K / group_size % 8 == 0 (16-byte aligned scale
// rows), K <= 4096 or K % 4096 == 0, 16-byte aligned x, codes, scales and
// biases, and the fp32 activations within the shared-memory budget.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdlib>

#include "q6_dequant.cuh"
#include "q6_internal.h"
#include "q6_ptx.cuh"

namespace q6 {
namespace {

constexpr int kWarps = 8;          // warps per CTA, each with its own ring
constexpr int kMinSlots = 2;       // ring slots per warp: 2, or 3 when that keeps the CTAs per SM
constexpr int kMaxSlots = 3;
constexpr int kMaxChunk = 4096;    // codes per row per stage
constexpr int kSmemCap = 220 * 1024;

__device__ __forceinline__ float bf16f(uint16_t v) { return __uint_as_float(static_cast<uint32_t>(v) << 16); }

__device__ __forceinline__ float gelu_ref(float x) {
    const float x3 = x * x * x;
    return 0.5f * x * (1.0f + tanhf(0.7978845608028654f * (x + 0.044715f * x3)));
}

// Physical float4 slot of logical float4 F of an activation row: F ^ ((F >> 3) & 7).
// Lanes read float4 e of consecutive 16-code units j (F = 4j + e); eight such
// lanes, starting at a multiple of 8, land in eight different 16-byte bank groups.
__device__ __forceinline__ int xswz(int F) { return F ^ ((F >> 3) & 7); }

struct GemvLayout {
    int chunk;        // codes per row per stage
    int code_bytes;   // per row per stage
    int sb_bytes;     // scales (or biases) bytes per row per stage
    int stage_bytes;  // two rows: codes, scales, biases (128-byte multiple)
};

__host__ __device__ inline GemvLayout gemv_layout(int K, int gs, int max_chunk) {
    GemvLayout L;
    L.chunk = K < max_chunk ? K : max_chunk;
    L.code_bytes = L.chunk * 6 / 8;
    L.sb_bytes = (L.chunk / gs) * 2;
    L.stage_bytes = (2 * L.code_bytes + 4 * L.sb_bytes + 127) & ~127;
    return L;
}

// UPL = 16-code units per lane per stage (chunk / 512) when it is a compile-
// time constant (every K that is a multiple of 512), which unrolls the unit
// loop so that all shared-memory addresses are a per-lane base plus an
// immediate; UPL = 0 is the generic loop.
template <int MT, int UPL>
__global__ void __launch_bounds__(kWarps * 32, MT == 1 ? 3 : 2) gemv_stream_kernel(const LinearArgs a, int gs_shift,
                                                                                const SpliceExp3 sx, int max_chunk,
                                                                                int slots) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int K = static_cast<int>(a.K);
    const int N = static_cast<int>(a.N);
    const int M = static_cast<int>(a.M);
    const GemvLayout L = gemv_layout(K, 1 << gs_shift, max_chunk);
    const int nchunks = K / L.chunk;
    const int K4 = K / 4;
    const int U16 = K / 16;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    uint8_t* ring = smem + warp * slots * L.stage_bytes;
    float4* xs4 = reinterpret_cast<float4*>(smem + kWarps * slots * L.stage_bytes);  // [MT][K/4]
    float2* xsum = reinterpret_cast<float2*>(xs4 + MT * K4);  // [MT][K/16]: x sums over a unit's even, odd codes
    uint64_t* full = reinterpret_cast<uint64_t*>(xsum + MT * U16) + warp * slots;

    const int npairs = (N + 1) / 2;
    const int gw = blockIdx.x * kWarps + warp;
    const int total_warps = gridDim.x * kWarps;
    const int words_per_row = K * 6 / 32;
    const int groups = K >> gs_shift;
    // This warp's stages t = 0, 1, ...: pair gw + (t / nchunks) * total_warps, chunk t % nchunks.
    const int my_pairs = gw < npairs ? (npairs - gw + total_warps - 1) / total_warps : 0;
    const int my_stages = my_pairs * nchunks;

    auto issue = [&](int t) {  // lane 0 only
        const int p = gw + (t / nchunks) * total_warps;
        const int c = t - (t / nchunks) * nchunks;
        const int n0 = 2 * p;
        const bool two = n0 + 1 < N;
        const uint32_t slot = smem_u32(ring + (t % slots) * L.stage_bytes);
        const uint32_t bar = smem_u32(full + (t % slots));
        const uint32_t cb = L.code_bytes, sbb = L.sb_bytes;
        mbar_arrive_expect_tx(bar, (two ? 2u : 1u) * (cb + 2 * sbb));
        const uint8_t* wrow = reinterpret_cast<const uint8_t*>(a.w + static_cast<size_t>(n0) * words_per_row) +
                              static_cast<size_t>(c) * cb;
        const uint8_t* srow = reinterpret_cast<const uint8_t*>(a.scales + static_cast<size_t>(n0) * groups) +
                              static_cast<size_t>(c) * sbb;
        const uint8_t* brow = reinterpret_cast<const uint8_t*>(a.qbiases + static_cast<size_t>(n0) * groups) +
                              static_cast<size_t>(c) * sbb;
        const size_t wstride = static_cast<size_t>(words_per_row) * 4, sstride = static_cast<size_t>(groups) * 2;
        bulk_load(slot, wrow, cb, bar);
        bulk_load(slot + 2 * cb, srow, sbb, bar);
        bulk_load(slot + 2 * cb + 2 * sbb, brow, sbb, bar);
        if (two) {
            bulk_load(slot + cb, wrow + wstride, cb, bar);
            bulk_load(slot + 2 * cb + sbb, srow + sstride, sbb, bar);
            bulk_load(slot + 2 * cb + 3 * sbb, brow + sstride, sbb, bar);
        }
    };

    pdl_launch_dependents();
    if (lane == 0) {
        for (int s = 0; s < slots; ++s) mbar_init(smem_u32(full + s), 1);
        fence_mbar_init();
        for (int t = 0; t < slots && t < my_stages; ++t) issue(t);  // weights: before the dependency wait
    }
    __syncwarp();
    pdl_wait();  // x, y and the epilogue operands may come from the previous kernel

    // Stage the activations (bf16 -> fp32, swizzled; rows M..MT-1 zero), then
    // the per-unit sums.  The first weight stages are already in flight.
    const uint16_t* x = static_cast<const uint16_t*>(a.x);
    for (int i = threadIdx.x; i < MT * K / 8; i += blockDim.x) {
        const uint4 v = i < M * K / 8 ? __ldg(reinterpret_cast<const uint4*>(x) + i) : make_uint4(0, 0, 0, 0);
        const int m = (2 * i) / K4;
        const int F = 2 * i - m * K4;
        float4* row = xs4 + m * K4;
        row[xswz(F)] = make_float4(__uint_as_float(v.x << 16), __uint_as_float(v.x & 0xFFFF0000u),
                                   __uint_as_float(v.y << 16), __uint_as_float(v.y & 0xFFFF0000u));
        row[xswz(F + 1)] = make_float4(__uint_as_float(v.z << 16), __uint_as_float(v.z & 0xFFFF0000u),
                                       __uint_as_float(v.w << 16), __uint_as_float(v.w & 0xFFFF0000u));
    }
    __syncthreads();
    for (int i = threadIdx.x; i < MT * U16; i += blockDim.x) {
        const int m = i / U16;
        const int J = i - m * U16;
        const float4* row = xs4 + m * K4;
        float ev = 0.0f, od = 0.0f;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float4 v = row[xswz(4 * J + e)];
            ev += v.x + v.z;
            od += v.y + v.w;
        }
        xsum[i] = make_float2(ev, od);
    }
    __syncthreads();

    volatile int no_abort = 0;  // the ring is private to the warp: no CTA-wide abort
    float acc0[MT], acc1[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) acc0[m] = acc1[m] = 0.0f;
    for (int t = 0; t < my_stages; ++t) {
        const int c = t % nchunks;
        const int p = gw + (t / nchunks) * total_warps;
        const int n0 = 2 * p;
        const int si = t % slots;
        const uint8_t* slot = ring + si * L.stage_bytes;
        if (!__all_sync(0xffffffffu, mbar_wait(smem_u32(full + si), static_cast<uint32_t>((t / slots) & 1),
                                               &no_abort, 11)))
            break;
        const uint8_t* codes0 = slot;
        const uint8_t* codes1 = slot + L.code_bytes;
        const uint16_t* sc0 = reinterpret_cast<const uint16_t*>(slot + 2 * L.code_bytes);
        const uint16_t* sc1 = sc0 + L.sb_bytes / 2;
        const uint16_t* bi0 = sc0 + L.sb_bytes;
        const uint16_t* bi1 = bi0 + L.sb_bytes / 2;
        const int units = L.chunk / 16;
        auto unit = [&](int j, int J, int gl, int xslot_base, int e_slots[4]) {
            const uint32_t* wa = reinterpret_cast<const uint32_t*>(codes0 + 12 * j);
            const uint32_t* wb = reinterpret_cast<const uint32_t*>(codes1 + 12 * j);
            // Code pairs (2i, 2i+1) of each row at bits 11 and 17 of va[i] / vb[i]
            // (stale slot bytes for an odd last row: never stored).
            uint32_t va[8], vb[8];
            pair_words16(wa[0], wa[1], wa[2], va);
            pair_words16(wb[0], wb[1], wb[2], vb);
            const float s0 = bf16f(sc0[gl]), b0 = bf16f(bi0[gl]);
            const float s1 = bf16f(sc1[gl]), b1 = bf16f(bi1[gl]);
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                const float4* xrow = xs4 + m * K4 + xslot_base;
                // (even, odd) code halves of the dot, each code carrying its splice
                // offset (4096 even, 64 odd): sum_k x_k (offset_k + q_k)
                float2 d0 = make_float2(0.0f, 0.0f), d1 = make_float2(0.0f, 0.0f);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float4 xv = xrow[e_slots[e]];
                    const float2 xlo = make_float2(xv.x, xv.y), xhi = make_float2(xv.z, xv.w);
                    d0 = __ffma2_rn(xlo, pair_at11_17(va[2 * e], sx), d0);
                    d0 = __ffma2_rn(xhi, pair_at11_17(va[2 * e + 1], sx), d0);
                    d1 = __ffma2_rn(xlo, pair_at11_17(vb[2 * e], sx), d1);
                    d1 = __ffma2_rn(xhi, pair_at11_17(vb[2 * e + 1], sx), d1);
                }
                const float2 xs = xsum[m * U16 + J];
                // remove the offsets: sum_k x_k q_k = d.x - 4096 xs.x + d.y - 64 xs.y
                const float2 off = make_float2(-4096.0f, -64.0f);
                const float2 t0 = __ffma2_rn(off, xs, d0), t1 = __ffma2_rn(off, xs, d1);
                const float xt = xs.x + xs.y;
                acc0[m] = fmaf(s0, t0.x + t0.y, fmaf(b0, xt, acc0[m]));
                acc1[m] = fmaf(s1, t1.x + t1.y, fmaf(b1, xt, acc1[m]));
            }
        };
        // Two adjacent units (one scale group for every group size) per lane:
        // units jA = 2 lane + 64 i and jA + 1.  Their 24 code bytes per row are
        // 8-byte aligned, their eight activation float4s sit at slots
        // 4 JA + (e ^ (lane & 7)) (the swizzle term (JA >> 1) & 7 is lane & 7
        // because the chunk's unit count is a multiple of 16), and the affine
        // map is applied once per pair.
        auto unit_pair = [&](int i) {
            const int jA = 2 * lane + 64 * i;
            const int JA = c * units + jA;
            const int gl = (16 * jA) >> gs_shift;
            const uint2* pa = reinterpret_cast<const uint2*>(codes0) + 3 * (lane + 32 * i);
            const uint2* pb = reinterpret_cast<const uint2*>(codes1) + 3 * (lane + 32 * i);
            const uint2 a0 = pa[0], a1 = pa[1], a2 = pa[2];
            const uint2 b0w = pb[0], b1w = pb[1], b2w = pb[2];
            uint32_t va[16], vb[16];
            pair_words16(a0.x, a0.y, a1.x, *reinterpret_cast<uint32_t(*)[8]>(va));
            pair_words16(a1.y, a2.x, a2.y, *reinterpret_cast<uint32_t(*)[8]>(va + 8));
            pair_words16(b0w.x, b0w.y, b1w.x, *reinterpret_cast<uint32_t(*)[8]>(vb));
            pair_words16(b1w.y, b2w.x, b2w.y, *reinterpret_cast<uint32_t(*)[8]>(vb + 8));
            const float s0 = bf16f(sc0[gl]), b0 = bf16f(bi0[gl]);
            const float s1 = bf16f(sc1[gl]), b1 = bf16f(bi1[gl]);
            const int sw = lane & 7;
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                const float4* xrow = xs4 + m * K4 + 4 * JA;
                float2 dA0 = make_float2(0.0f, 0.0f), dB0 = dA0, dA1 = dA0, dB1 = dA0;
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float4 xa = xrow[e ^ sw];
                    const float4 xb = xrow[(e + 4) ^ sw];
                    dA0 = __ffma2_rn(make_float2(xa.x, xa.y), pair_at11_17(va[2 * e], sx), dA0);
                    dA0 = __ffma2_rn(make_float2(xa.z, xa.w), pair_at11_17(va[2 * e + 1], sx), dA0);
                    dB0 = __ffma2_rn(make_float2(xb.x, xb.y), pair_at11_17(va[8 + 2 * e], sx), dB0);
                    dB0 = __ffma2_rn(make_float2(xb.z, xb.w), pair_at11_17(va[8 + 2 * e + 1], sx), dB0);
                    dA1 = __ffma2_rn(make_float2(xa.x, xa.y), pair_at11_17(vb[2 * e], sx), dA1);
                    dA1 = __ffma2_rn(make_float2(xa.z, xa.w), pair_at11_17(vb[2 * e + 1], sx), dA1);
                    dB1 = __ffma2_rn(make_float2(xb.x, xb.y), pair_at11_17(vb[8 + 2 * e], sx), dB1);
                    dB1 = __ffma2_rn(make_float2(xb.z, xb.w), pair_at11_17(vb[8 + 2 * e + 1], sx), dB1);
                }
                const float4 xq = *reinterpret_cast<const float4*>(xsum + m * U16 + JA);  // units JA, JA + 1
                const float2 xs = __fadd2_rn(make_float2(xq.x, xq.y), make_float2(xq.z, xq.w));
                const float2 off = make_float2(-4096.0f, -64.0f);
                const float2 t0 = __ffma2_rn(off, xs, __fadd2_rn(dA0, dB0));
                const float2 t1 = __ffma2_rn(off, xs, __fadd2_rn(dA1, dB1));
                const float xt = xs.x + xs.y;
                acc0[m] = fmaf(s0, t0.x + t0.y, fmaf(b0, xt, acc0[m]));
                acc1[m] = fmaf(s1, t1.x + t1.y, fmaf(b1, xt, acc1[m]));
            }
        };
        if constexpr (UPL > 0 && UPL % 2 == 0 && MT <= 2) {  // four token rows: the unit path fits 128 registers
#pragma unroll
            for (int i = 0; i < UPL / 2; ++i) unit_pair(i);
        } else if constexpr (UPL > 0) {
            // units j = lane + 32 i: the x swizzle term (J >> 1) & 7 = (lane >> 1) & 7
            // is the same for every i, so the four float4 slots of a unit are
            // per-lane constants plus 128 i.
            const int h = (lane >> 1) & 7;
            int e_slots[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) e_slots[e] = (4 * lane + e) ^ h;
            const int gstep = 512 >> gs_shift;  // groups per 32 units
#pragma unroll
            for (int i = 0; i < UPL; ++i) {
                const int j = lane + 32 * i;
                unit(j, c * units + j, ((16 * lane) >> gs_shift) + i * gstep, 4 * (c * units + 32 * i), e_slots);
            }
        } else {
            for (int j = lane; j < units; j += 32) {
                const int J = c * units + j;
                int e_slots[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) e_slots[e] = xswz(4 * J + e) - 4 * J;
                unit(j, J, (16 * j) >> gs_shift, 4 * J, e_slots);
            }
        }
        // Hand the slot back to this warp's producer lane for stage t + slots.
        __syncwarp();
        if (lane == 0 && t + slots < my_stages) {
            fence_proxy_async_smem();
            issue(t + slots);
        }
        if (c == nchunks - 1) {
#pragma unroll
            for (int m = 0; m < MT; ++m) {
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) {
                    acc0[m] += __shfl_xor_sync(0xffffffffu, acc0[m], off);
                    acc1[m] += __shfl_xor_sync(0xffffffffu, acc1[m], off);
                }
            }
            // Lane 2m + r writes token m of row n0 + r.
            if (lane < 2 * MT) {
                const int m = lane >> 1;
                const int r = lane & 1;
                float v = 0.0f;
#pragma unroll
                for (int mm = 0; mm < MT; ++mm)
                    if (mm == m) v = r ? acc1[mm] : acc0[mm];
                const int n = n0 + r;
                if (m < M && n < N) {
                    if (a.bias) v += bf16f(a.bias[n]);
                    if (a.flags & (Q6_EPI_GELU | Q6_EPI_GELU_PRECISE)) v = gelu_ref(v);
                    if (a.gate) v *= bf16f(a.gate[n]);
                    if (a.residual) v += bf16f(a.residual[static_cast<size_t>(m) * N + n]);
                    __nv_bfloat16 h = __float2bfloat16_rn(v);
                    static_cast<uint16_t*>(a.y)[static_cast<size_t>(m) * N + n] = *reinterpret_cast<uint16_t*>(&h);
                }
            }
#pragma unroll
            for (int m = 0; m < MT; ++m) acc0[m] = acc1[m] = 0.0f;
        }
    }
}

// Codes per row per stage: Q6_GEMV_CHUNK (a multiple of 512 up to 4096)
// overrides the default of 4096.
int gemv_max_chunk() {
    if (const char* v = std::getenv("Q6_GEMV_CHUNK")) {
        const int c = std::atoi(v);
        if (c >= 512 && c <= kMaxChunk && c % 512 == 0) return c;
    }
    return kMaxChunk;
}

size_t gemv_smem_bytes(int64_t K, int gs, int mt, int slots) {
    const GemvLayout L = gemv_layout(static_cast<int>(K), gs, gemv_max_chunk());
    return static_cast<size_t>(kWarps) * slots * L.stage_bytes + static_cast<size_t>(mt) * K * 4 +
           static_cast<size_t>(mt) * (K / 16) * 8 + kWarps * slots * 8;
}

// Ring depth: a third slot (two stages in flight per warp) when it costs no
// CTA per SM, i.e. when shared memory already holds only one CTA (long K:
// the fp32 activations take 48 KB at K = 12288).
int gemv_slots(int64_t K, int gs, int mt) {
    const size_t two = gemv_smem_bytes(K, gs, mt, kMinSlots), three = gemv_smem_bytes(K, gs, mt, kMaxSlots);
    if (three > static_cast<size_t>(kSmemCap)) return kMinSlots;
    const size_t per_sm = 228 * 1024;  // shared memory per SM (each CTA also reserves 1 KB)
    return (per_sm / (three + 1024)) >= (per_sm / (two + 1024)) ? kMaxSlots : kMinSlots;
}

template <int MT, int UPL>
int launch_gemv_mt(const LinearArgs& a, cudaStream_t stream) {
    const int slots = gemv_slots(a.K, a.group_size, MT);
    const size_t smem = gemv_smem_bytes(a.K, a.group_size, MT, slots);
    static std::atomic<bool> attr_set_for_device[kMaxDevices];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return Q6_ERR_CUDA;
    if (dev < 0 || dev >= kMaxDevices) return Q6_ERR_UNSUPPORTED;
    if (!attr_set_for_device[dev].load(std::memory_order_acquire)) {
        if (cudaFuncSetAttribute(gemv_stream_kernel<MT, UPL>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemCap) !=
            cudaSuccess)
            return Q6_ERR_CUDA;
        attr_set_for_device[dev].store(true, std::memory_order_release);
    }
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gemv_stream_kernel<MT, UPL>, kWarps * 32, smem) !=
            cudaSuccess ||
        per_sm <= 0)
        return Q6_ERR_CUDA;
    const int64_t pairs = (a.N + 1) / 2;
    const int64_t want = (pairs + kWarps - 1) / kWarps;
    const int blocks = static_cast<int>(std::min<int64_t>(want, static_cast<int64_t>(device_sm_count()) * per_sm));
    const int gs_shift = a.group_size == 32 ? 5 : (a.group_size == 64 ? 6 : 7);
    const cudaError_t err = launch_pdl(gemv_stream_kernel<MT, UPL>, dim3(blocks), dim3(kWarps * 32), smem, stream, a,
                                       gs_shift, splice_exp3_host(), gemv_max_chunk(), slots);
    return err == cudaSuccess ? Q6_OK : Q6_ERR_CUDA;
}

}  // namespace

int error_word_gemv(bool clear) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)) != cudaSuccess) return -1;
    if (clear && v != 0) {
        const int zero = 0;
        if (cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int)) != cudaSuccess) return -1;
    }
    return v;
}

bool gemv_supported(const LinearArgs& a) {
    if (a.M < 1 || a.M > 4 || a.K % 64 != 0) return false;
    if (a.K > (int64_t(1) << 20) || a.N > (int64_t(1) << 30)) return false;
    if ((a.K / a.group_size) % 8 != 0) return false;
    const int chunk = gemv_max_chunk();
    if (a.K > chunk && a.K % chunk != 0) return false;
    const uintptr_t align = reinterpret_cast<uintptr_t>(a.x) | reinterpret_cast<uintptr_t>(a.w) |
                            reinterpret_cast<uintptr_t>(a.scales) | reinterpret_cast<uintptr_t>(a.qbiases);
    if (align % 16 != 0) return false;
    const int mt = a.M == 3 ? 4 : static_cast<int>(a.M);  // token rows of the kernel instantiation
    return gemv_smem_bytes(a.K, a.group_size, mt, kMinSlots) <= static_cast<size_t>(kSmemCap);
}

template <int MT>
int launch_gemv_upl(const LinearArgs& a, cudaStream_t stream) {
    const int64_t chunk = a.K < gemv_max_chunk() ? a.K : gemv_max_chunk();
    const int upl = chunk % 512 == 0 ? static_cast<int>(chunk / 512) : 0;
    switch (upl) {
        case 1: return launch_gemv_mt<MT, 1>(a, stream);
        case 2: return launch_gemv_mt<MT, 2>(a, stream);
        case 3: return launch_gemv_mt<MT, 3>(a, stream);
        case 4: return launch_gemv_mt<MT, 4>(a, stream);
        case 5: return launch_gemv_mt<MT, 5>(a, stream);
        case 6: return launch_gemv_mt<MT, 6>(a, stream);
        case 7: return launch_gemv_mt<MT, 7>(a, stream);
        case 8: return launch_gemv_mt<MT, 8>(a, stream);
        default: return launch_gemv_mt<MT, 0>(a, stream);
    }
}

int launch_gemv(const LinearArgs& a, cudaStream_t stream) {
    switch (a.M) {
        case 1: return launch_gemv_upl<1>(a, stream);
        case 2: return launch_gemv_upl<2>(a, stream);
        default: return launch_gemv_upl<4>(a, stream);  // M = 3 or 4
    }
}

}  // namespace q6
