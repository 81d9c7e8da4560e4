// Sequence-parallel collectives of the tensor-parallel block, fused with the
// row work between its GEMMs, over peer (NVLink) memory.
//
// The tensor-parallel MMDiT block keeps the joint rows [B S, D] sharded
// between its GEMMs: rank r owns rows [r R, (r + 1) R).  Each half of the
// block ends in a row-parallel GEMM whose partial sums P_r [B S, D] must be
// reduced onto the owner of each row, and the next half starts with a
// column-parallel GEMM that needs every row.  Instead of a reduce-scatter
// and an all-gather around the residual add and adaLN modulate, one kernel
// per half does all of it:
//
//   h   = x + sum_r P_r[rows of this rank]     (peer loads, rank order, fp32 sum, one bf16 rounding)
//   y   = LayerNorm(h) * (1 + scale[v]) + shift[v]
//   Z_r[rows of this rank] = y  for every rank r  (peer stores)
//
// reading the partials of every rank and writing the modulated rows into every
// rank's gather buffer, all of which live in memory every rank can address
// (CUDA peer mappings of symmetric buffers).  Between the phases a barrier
// kernel orders the ranks: each rank releases a flag into every peer's signal
// slots (system scope) and waits, bounded, for every peer's flag.  The
// barrier's epoch comes from a counter in device memory that the barrier
// itself advances, so a CUDA graph of a whole step replays correctly.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "q6_internal.h"
#include "q6_ptx.cuh"

namespace q6 {
namespace {

constexpr int kMaxRanks = 8;
constexpr int kSpWarps = 4;  // rows per CTA

struct PeerIn {
    const uint4* p[kMaxRanks];
};
struct PeerOut {
    uint4* p[kMaxRanks];
};
struct PeerSignals {
    uint32_t* p[kMaxRanks];
};

__device__ __forceinline__ float lo_f(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float hi_f(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// One warp per local row; NV uint4 (8 bf16) per lane, D = 256 NV.
template <int NV, bool kParts>
__global__ void __launch_bounds__(kSpWarps * 32) sp_add_ln_gather_kernel(
    const uint4* __restrict__ x, const PeerIn parts, uint4* h_out, const uint4* __restrict__ shift,
    const uint4* __restrict__ scale, int64_t vstride8, const PeerOut dst, int world, int64_t R, int64_t row0,
    int64_t seq_len, int64_t text_len, float eps) {
    pdl_launch_dependents();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int64_t row = static_cast<int64_t>(blockIdx.x) * kSpWarps + (threadIdx.x >> 5);
    if (row >= R) return;
    constexpr int D8 = 32 * NV;  // uint4 per row
    const int64_t grow = row0 + row;
    float h[NV][8];
    {
        const uint4* xr = x + row * D8;
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            const uint4 v = xr[lane + 32 * j];
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                h[j][2 * i] = lo_f(w[i]);
                h[j][2 * i + 1] = hi_f(w[i]);
            }
        }
    }
    if constexpr (kParts) {
        // x plus the partial sums of every rank for this row, in rank order (fp32)
        for (int r = 0; r < world; ++r) {
            const uint4* pr = parts.p[r] + grow * D8;
            uint4 v[NV];
#pragma unroll
            for (int j = 0; j < NV; ++j) v[j] = pr[lane + 32 * j];
#pragma unroll
            for (int j = 0; j < NV; ++j) {
                const uint32_t w[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    h[j][2 * i] += lo_f(w[i]);
                    h[j][2 * i + 1] += hi_f(w[i]);
                }
            }
        }
        // h rounded to bf16 once; the LayerNorm reads the rounded row
        uint4* hr = h_out ? h_out + row * D8 : nullptr;
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            uint32_t w[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                w[i] = pack2(h[j][2 * i], h[j][2 * i + 1]);
                h[j][2 * i] = lo_f(w[i]);
                h[j][2 * i + 1] = hi_f(w[i]);
            }
            if (hr) hr[lane + 32 * j] = make_uint4(w[0], w[1], w[2], w[3]);
        }
        if (dst.p[0] == nullptr) return;  // the reduction alone (a stack's last block)
    }
    float sum = 0.0f;
#pragma unroll
    for (int j = 0; j < NV; ++j)
#pragma unroll
        for (int i = 0; i < 8; ++i) sum += h[j][i];
    const float mean = warp_sum(sum) * (1.0f / (256 * NV));
    float sq = 0.0f;
#pragma unroll
    for (int j = 0; j < NV; ++j)
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float d = h[j][i] - mean;
            sq = fmaf(d, d, sq);
        }
    const float rstd = rsqrtf(warp_sum(sq) * (1.0f / (256 * NV)) + eps);
    int64_t vec = 0;
    if (seq_len > 0) vec = (grow / seq_len) * 2 + ((grow % seq_len) >= text_len ? 1 : 0);
    const uint4* sh = shift + vec * vstride8;
    const uint4* sc = scale + vec * vstride8;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
        const uint4 a = __ldg(sh + lane + 32 * j), b = __ldg(sc + lane + 32 * j);
        const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, bw[4] = {b.x, b.y, b.z, b.w};
        uint32_t o[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float v0 = (h[j][2 * i] - mean) * rstd, v1 = (h[j][2 * i + 1] - mean) * rstd;
            o[i] = pack2(fmaf(v0, 1.0f + lo_f(bw[i]), lo_f(aw[i])), fmaf(v1, 1.0f + hi_f(bw[i]), hi_f(aw[i])));
        }
        const uint4 out = make_uint4(o[0], o[1], o[2], o[3]);
        for (int r = 0; r < world; ++r) dst.p[r][grow * D8 + lane + 32 * j] = out;
    }
    // No fence here: the peer stores are complete when this grid is, and the
    // q6_sp_barrier launch that follows on the stream (never a programmatic
    // dependent) releases them to the peers at system scope.
}

// Barrier across `world` ranks: thread t releases the new epoch into slot
// `rank` of peer t's signal array and waits (bounded) until peer t has done
// the same into slot t of ours.
__global__ void __launch_bounds__(32) sp_barrier_kernel(const PeerSignals sig, uint32_t* epoch_ctr, int world,
                                                        int rank, uint64_t timeout_ns) {
    __shared__ uint32_t ep;
    if (threadIdx.x == 0) {
        ep = *epoch_ctr + 1u;
        *epoch_ctr = ep;
    }
    __syncthreads();
    const int t = threadIdx.x;
    if (t < world) {
        const uint32_t e = ep;
        uint32_t* remote = sig.p[t] + rank;
        asm volatile("fence.acq_rel.sys;\n\tst.release.sys.global.u32 [%0], %1;" ::"l"(remote), "r"(e) : "memory");
        const uint32_t* mine = sig.p[rank] + t;
        const uint64_t t0 = global_timer_ns();
        for (uint32_t i = 0;; ++i) {
            uint32_t v;
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
            if (static_cast<int32_t>(v - e) >= 0) break;
            if ((i & 63u) == 63u && global_timer_ns() - t0 > timeout_ns) {
                record_error(Q6_SITE_PEER_BARRIER);
                break;
            }
        }
    }
    __syncthreads();
}

template <int NV>
int launch_sp(const uint4* x, const PeerIn& parts, bool has_parts, uint4* h_out, const uint4* shift,
              const uint4* scale, int64_t vstride8, const PeerOut& dst, int world, int64_t R, int64_t row0,
              int64_t seq_len, int64_t text_len, float eps, cudaStream_t stream) {
    const int64_t blocks = (R + kSpWarps - 1) / kSpWarps;
    cudaError_t e;
    if (has_parts)
        e = launch_pdl(sp_add_ln_gather_kernel<NV, true>, dim3(static_cast<unsigned>(blocks)), dim3(kSpWarps * 32), 0,
                       stream, x, parts, h_out, shift, scale, vstride8, dst, world, R, row0, seq_len, text_len,
                       eps);
    else
        e = launch_pdl(sp_add_ln_gather_kernel<NV, false>, dim3(static_cast<unsigned>(blocks)), dim3(kSpWarps * 32), 0,
                       stream, x, parts, h_out, shift, scale, vstride8, dst, world, R, row0, seq_len, text_len,
                       eps);
    return e == cudaSuccess ? Q6_OK : Q6_ERR_CUDA;
}

}  // namespace

int error_word_sp(bool clear) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)) != cudaSuccess) return -1;
    if (clear && v != 0) {
        const int zero = 0;
        if (cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int)) != cudaSuccess) return -1;
    }
    return v;
}

}  // namespace q6

extern "C" {

Q6_API int q6_sp_add_layernorm_gather_bf16(const uint16_t* x_local, const uint16_t* const* partials,
                                           uint16_t* h_out, const uint16_t* shift, const uint16_t* scale,
                                           int64_t vec_stride, uint16_t* const* gathered, int world, int rank,
                                           int64_t R, int64_t D, int64_t seq_len, int64_t text_len, float eps,
                                           q6_stream_t stream) {
    if (!x_local || R <= 0 || D <= 0 || !(eps >= 0.0f)) return Q6_ERR_INVALID_ARGUMENT;
    if (world < 1 || world > q6::kMaxRanks || rank < 0 || rank >= world) return Q6_ERR_INVALID_ARGUMENT;
    if (h_out && !partials) return Q6_ERR_INVALID_ARGUMENT;
    if (gathered ? (!shift || !scale) : (!partials || !h_out)) return Q6_ERR_INVALID_ARGUMENT;
    if (seq_len < 0 || text_len < 0 || text_len > seq_len) return Q6_ERR_INVALID_ARGUMENT;
    if (D % 256 != 0) return Q6_ERR_SHAPE;
    if (vec_stride == 0) vec_stride = D;
    if (vec_stride < D) return Q6_ERR_INVALID_ARGUMENT;
    if (vec_stride % 8 != 0) return Q6_ERR_ALIGNMENT;
    uintptr_t al = reinterpret_cast<uintptr_t>(x_local) | reinterpret_cast<uintptr_t>(shift) |
                   reinterpret_cast<uintptr_t>(scale) | reinterpret_cast<uintptr_t>(h_out);
    q6::PeerIn parts{};
    q6::PeerOut dst{};
    for (int r = 0; r < world; ++r) {
        if ((gathered && !gathered[r]) || (partials && !partials[r])) return Q6_ERR_INVALID_ARGUMENT;
        if (gathered) {
            dst.p[r] = reinterpret_cast<uint4*>(gathered[r]);
            al |= reinterpret_cast<uintptr_t>(gathered[r]);
        }
        if (partials) {
            parts.p[r] = reinterpret_cast<const uint4*>(partials[r]);
            al |= reinterpret_cast<uintptr_t>(partials[r]);
        }
    }
    if (al % 16 != 0) return Q6_ERR_ALIGNMENT;
    const uint4* x = reinterpret_cast<const uint4*>(x_local);
    const uint4* sh = reinterpret_cast<const uint4*>(shift);
    const uint4* sc = reinterpret_cast<const uint4*>(scale);
    uint4* h = reinterpret_cast<uint4*>(h_out);
    const int64_t row0 = static_cast<int64_t>(rank) * R;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const bool hp = partials != nullptr;
    const int64_t vs8 = vec_stride / 8;
    switch (D / 256) {
        case 1: return q6::launch_sp<1>(x, parts, hp, h, sh, sc, vs8, dst, world, R, row0, seq_len, text_len, eps, s);
        case 2: return q6::launch_sp<2>(x, parts, hp, h, sh, sc, vs8, dst, world, R, row0, seq_len, text_len, eps, s);
        case 4: return q6::launch_sp<4>(x, parts, hp, h, sh, sc, vs8, dst, world, R, row0, seq_len, text_len, eps, s);
        case 12: return q6::launch_sp<12>(x, parts, hp, h, sh, sc, vs8, dst, world, R, row0, seq_len, text_len, eps, s);
        default: return Q6_ERR_UNSUPPORTED;
    }
}

Q6_API int q6_sp_barrier(uint32_t* const* signals, uint32_t* epoch, int world, int rank, int64_t timeout_ns,
                         q6_stream_t stream) {
    if (!signals || !epoch || world < 1 || world > q6::kMaxRanks || rank < 0 || rank >= world)
        return Q6_ERR_INVALID_ARGUMENT;
    if (timeout_ns < 1000 || timeout_ns > 60000000000ll) return Q6_ERR_INVALID_ARGUMENT;
    q6::PeerSignals sig{};
    for (int r = 0; r < world; ++r) {
        if (!signals[r] || reinterpret_cast<uintptr_t>(signals[r]) % 4 != 0) return Q6_ERR_INVALID_ARGUMENT;
        sig.p[r] = signals[r];
    }
    q6::sp_barrier_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        sig, epoch, world, rank, static_cast<uint64_t>(timeout_ns));
    return cudaGetLastError() == cudaSuccess ? Q6_OK : Q6_ERR_CUDA;
}

}  // extern "C"
