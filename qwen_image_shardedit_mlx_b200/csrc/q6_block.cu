// The MMDiT block's memory-bound steps around the q6 linears:
//
//   * q6_layernorm_modulate_bf16: y = LayerNorm(x) * (1 + scale) + shift, the
//     adaLN `_modulate(norm(x), mod)` of the Qwen-Image block
//     (benchmarks/profile_qwen_block.py:172-181 and :262-263: LayerNorm
//     without affine parameters, eps 1e-6, then shift / scale from the
//     modulation linear).  One warp per row, the row held in registers, mean
//     and variance in fp32 (two passes over the registers), one bf16 rounding
//     at the output.
//   * q6_qk_rmsnorm_rope_bf16: per head of 128, x <- rope(rmsnorm(x) * w), in
//     place (profile_qwen_block.py:203-217: norm_q / norm_k, then
//     _apply_rope_qwen).  The rotation acts on interleaved pairs
//     (x[2i], x[2i+1]) with the per-token angle tables cos / sin [M, 64] (the
//     complex form of the Qwen-Image rotary embedding).  One warp per token,
//     two heads per step (eight values per lane, a half-warp reduction for
//     the mean square), the weight and angle factors folded once per token.
//
// Both read and write each element once: HBM-bound, ~12 bytes per element
// for the modulate (x in, y out, shift/scale from L1) and 4 for the in-place
// rope (+ 2 floats of table per pair, shared by the heads of a token).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "q6_internal.h"
#include "q6_ptx.cuh"

namespace q6 {
namespace {

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

constexpr int kLnWarps = 4;  // rows per CTA

// NV uint4 (8 bf16) per lane: D = 256 NV.  kAdd: the row is first formed as
// h = bf16(x + add) (stored to h_out when given).  Row g = row0 + m of the
// joint batched sequence takes modulation vector
// v = (g / seq_len) * 2 + (g % seq_len >= text_len) (0 when seq_len == 0),
// vectors vstride8 uint4 apart.
template <int NV, bool kAdd>
__global__ void __launch_bounds__(kLnWarps * 32) layernorm_modulate_kernel(
    const uint4* __restrict__ x, const uint4* __restrict__ add, uint4* h_out, const uint4* __restrict__ shift,
    const uint4* __restrict__ scale, int64_t vstride8, uint4* y, int64_t M, int64_t row0, int64_t seq_len,
    int64_t text_len, float eps) {
    pdl_launch_dependents();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int64_t row = static_cast<int64_t>(blockIdx.x) * kLnWarps + (threadIdx.x >> 5);
    if (row >= M) return;
    constexpr int D = 256 * NV;
    const uint4* xr = x + row * (D / 8);
    uint4 v[NV];
#pragma unroll
    for (int j = 0; j < NV; ++j) v[j] = xr[lane + 32 * j];
    if constexpr (kAdd) {
        const uint4* ar = add + row * (D / 8);
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            const uint4 b = ar[lane + 32 * j];
            v[j] = make_uint4(pack2(lo_f(v[j].x) + lo_f(b.x), hi_f(v[j].x) + hi_f(b.x)),
                              pack2(lo_f(v[j].y) + lo_f(b.y), hi_f(v[j].y) + hi_f(b.y)),
                              pack2(lo_f(v[j].z) + lo_f(b.z), hi_f(v[j].z) + hi_f(b.z)),
                              pack2(lo_f(v[j].w) + lo_f(b.w), hi_f(v[j].w) + hi_f(b.w)));
        }
        if (h_out) {
            uint4* hr = h_out + row * (D / 8);
#pragma unroll
            for (int j = 0; j < NV; ++j) hr[lane + 32 * j] = v[j];
        }
    }
    int64_t vec = 0;
    if (seq_len > 0) {
        const int64_t g = row0 + row;
        vec = (g / seq_len) * 2 + ((g % seq_len) >= text_len ? 1 : 0);
    }
    shift += vec * vstride8;
    scale += vec * vstride8;
    float s = 0.0f;
#pragma unroll
    for (int j = 0; j < NV; ++j)
        s += (lo_f(v[j].x) + hi_f(v[j].x)) + (lo_f(v[j].y) + hi_f(v[j].y)) + (lo_f(v[j].z) + hi_f(v[j].z)) +
             (lo_f(v[j].w) + hi_f(v[j].w));
    const float mean = warp_sum(s) * (1.0f / D);
    float q = 0.0f;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
        const uint32_t w[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float a = lo_f(w[i]) - mean, b = hi_f(w[i]) - mean;
            q = fmaf(a, a, fmaf(b, b, q));
        }
    }
    const float rstd = rsqrtf(warp_sum(q) * (1.0f / D) + eps);
    uint4* yr = y + row * (D / 8);
#pragma unroll
    for (int j = 0; j < NV; ++j) {
        const uint4 sh = __ldg(shift + lane + 32 * j), sc = __ldg(scale + lane + 32 * j);
        const uint32_t w[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
        const uint32_t shw[4] = {sh.x, sh.y, sh.z, sh.w}, scw[4] = {sc.x, sc.y, sc.z, sc.w};
        uint32_t o[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float a = (lo_f(w[i]) - mean) * rstd, b = (hi_f(w[i]) - mean) * rstd;
            o[i] = pack2(fmaf(a, 1.0f + lo_f(scw[i]), lo_f(shw[i])), fmaf(b, 1.0f + hi_f(scw[i]), hi_f(shw[i])));
        }
        yr[lane + 32 * j] = make_uint4(o[0], o[1], o[2], o[3]);
    }
}

struct LnArgs {
    const void* x;
    const void* add;
    void* h_out;
    const void* shift;
    const void* scale;
    int64_t vstride8;
    void* y;
    int64_t M, row0, seq_len, text_len;
    float eps;
};

template <int NV>
int launch_ln(const LnArgs& a, cudaStream_t stream) {
    const int64_t blocks = (a.M + kLnWarps - 1) / kLnWarps;
    auto go = [&](auto kernel) {
        return launch_pdl(kernel, dim3(static_cast<unsigned>(blocks)), dim3(kLnWarps * 32), 0, stream,
                          static_cast<const uint4*>(a.x), static_cast<const uint4*>(a.add),
                          static_cast<uint4*>(a.h_out), static_cast<const uint4*>(a.shift),
                          static_cast<const uint4*>(a.scale), a.vstride8, static_cast<uint4*>(a.y), a.M, a.row0,
                          a.seq_len, a.text_len, a.eps);
    };
    const cudaError_t e = a.add ? go(layernorm_modulate_kernel<NV, true>) : go(layernorm_modulate_kernel<NV, false>);
    return e == cudaSuccess ? Q6_OK : Q6_ERR_CUDA;
}

int dispatch_ln(const LnArgs& a, int64_t D, cudaStream_t s) {
    switch (D / 256) {
        case 1: return launch_ln<1>(a, s);
        case 2: return launch_ln<2>(a, s);
        case 3: return launch_ln<3>(a, s);
        case 4: return launch_ln<4>(a, s);
        case 6: return launch_ln<6>(a, s);
        case 8: return launch_ln<8>(a, s);
        case 12: return launch_ln<12>(a, s);
        case 16: return launch_ln<16>(a, s);
        default: return Q6_ERR_UNSUPPORTED;
    }
}

constexpr int kRopeWarps = 8;  // rows per CTA
constexpr int kRopeUnroll = 4;  // head pairs loaded before any is processed

// One warp per row; each half-warp takes one head of 128 per step (lane l
// holds elements 8 (l % 16) .. 8 (l % 16) + 7, i.e. rotary pairs
// 4 (l % 16) .. 4 (l % 16) + 3), so a step covers two heads and the mean
// square reduces over 16 lanes.  Row m is row g = row0 + m of sequences of
// seq_len rows (seq_len 0: g = m, one sequence): it takes angle-table row
// g % seq_len and the first weight vector for the first text_len rows of a
// sequence, the second for the rest.  The weight and angles of a lane are
// the same for every head of the row, so they are folded once per row into
// four coefficients per pair:
//   o_even = r (x_even (w_even cos) - x_odd (w_odd sin))
//   o_odd  = r (x_even (w_even sin) + x_odd (w_odd cos))
// with r = rsqrt(mean(x^2) + eps) of the head.
__global__ void __launch_bounds__(kRopeWarps * 32) qk_rmsnorm_rope_kernel(uint4* __restrict__ qk, int64_t row_stride16,
                                                                         int64_t M, int H,
                                                                         const uint4* __restrict__ w_text,
                                                                         const uint4* __restrict__ w_image,
                                                                         const float4* __restrict__ cs,
                                                                         const float4* __restrict__ sn, int64_t row0,
                                                                         int64_t seq_len, int64_t text_len, float eps) {
    pdl_launch_dependents();
    const int lane = threadIdx.x & 31;
    const int half = lane >> 4, hl = lane & 15;
    const int64_t row = static_cast<int64_t>(blockIdx.x) * kRopeWarps + (threadIdx.x >> 5);
    if (row >= M) return;
    const int64_t trow = seq_len > 0 ? (row0 + row) % seq_len : row;
    pdl_wait();
    const uint4 w = __ldg((trow < text_len ? w_text : w_image) + hl);
    const float4 c = __ldg(cs + trow * 16 + hl), s = __ldg(sn + trow * 16 + hl);
    const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
    const float cc[4] = {c.x, c.y, c.z, c.w}, ss[4] = {s.x, s.y, s.z, s.w};
    float ka[4], kb[4], kc[4], kd[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float we = lo_f(ww[i]), wo = hi_f(ww[i]);
        ka[i] = we * cc[i];
        kb[i] = wo * ss[i];
        kc[i] = we * ss[i];
        kd[i] = wo * cc[i];
    }
    uint4* p = qk + row * row_stride16 + hl;  // 128 bf16 = 16 uint4 per head
    const int pairs = (H + 1) >> 1;
    for (int h0 = 0; h0 < pairs; h0 += kRopeUnroll) {
        uint4 v[kRopeUnroll];
#pragma unroll
        for (int u = 0; u < kRopeUnroll; ++u) {
            const int head = 2 * (h0 + u) + half;
            v[u] = make_uint4(0u, 0u, 0u, 0u);
            if (h0 + u < pairs && head < H) v[u] = p[head * 16];
        }
#pragma unroll
        for (int u = 0; u < kRopeUnroll; ++u) {
            const int head = 2 * (h0 + u) + half;
            if (h0 + u >= pairs) break;  // warp-uniform
            const uint32_t x[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
            float q = 0.0f;
#pragma unroll
            for (int i = 0; i < 4; ++i) q = fmaf(lo_f(x[i]), lo_f(x[i]), fmaf(hi_f(x[i]), hi_f(x[i]), q));
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
            const float r = rsqrtf(q * (1.0f / 128.0f) + eps);
            uint32_t out[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float xe = lo_f(x[i]) * r, xo = hi_f(x[i]) * r;
                out[i] = pack2(fmaf(xe, ka[i], -xo * kb[i]), fmaf(xe, kc[i], xo * kd[i]));
            }
            if (head < H) p[head * 16] = make_uint4(out[0], out[1], out[2], out[3]);
        }
    }
}

}  // namespace
}  // namespace q6

extern "C" {

Q6_API int q6_layernorm_modulate_bf16(const uint16_t* x, const uint16_t* shift, const uint16_t* scale, uint16_t* y,
                                      int64_t M, int64_t D, float eps, q6_stream_t stream) {
    return q6_add_layernorm_modulate_bf16(x, nullptr, nullptr, shift, scale, 0, y, M, D, 0, 0, 0, eps, stream);
}

Q6_API int q6_add_layernorm_modulate_bf16(const uint16_t* x, const uint16_t* add, uint16_t* h_out,
                                          const uint16_t* shift, const uint16_t* scale, int64_t vec_stride,
                                          uint16_t* y, int64_t M, int64_t D, int64_t row0, int64_t seq_len,
                                          int64_t text_len, float eps, q6_stream_t stream) {
    if (!x || !shift || !scale || !y || M <= 0 || D <= 0 || !(eps >= 0.0f)) return Q6_ERR_INVALID_ARGUMENT;
    if (h_out && !add) return Q6_ERR_INVALID_ARGUMENT;
    if (row0 < 0 || seq_len < 0 || text_len < 0 || text_len > seq_len) return Q6_ERR_INVALID_ARGUMENT;
    if (D % 256 != 0) return Q6_ERR_SHAPE;
    if (vec_stride == 0) vec_stride = D;
    if (vec_stride < D) return Q6_ERR_INVALID_ARGUMENT;
    if (vec_stride % 8 != 0) return Q6_ERR_ALIGNMENT;
    const uintptr_t al = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(shift) |
                         reinterpret_cast<uintptr_t>(scale) | reinterpret_cast<uintptr_t>(y) |
                         reinterpret_cast<uintptr_t>(add) | reinterpret_cast<uintptr_t>(h_out);
    if (al % 16 != 0) return Q6_ERR_ALIGNMENT;
    const q6::LnArgs a{x, add, h_out, shift, scale, vec_stride / 8, y, M, row0, seq_len, text_len, eps};
    return q6::dispatch_ln(a, D, reinterpret_cast<cudaStream_t>(stream));
}

Q6_API int q6_qk_rmsnorm_rope_bf16(uint16_t* qk, int64_t row_stride, int64_t M, int heads, int head_dim,
                                   const uint16_t* weight, const float* cos, const float* sin, float eps,
                                   q6_stream_t stream) {
    return q6_qk_rmsnorm_rope_joint_bf16(qk, row_stride, M, heads, head_dim, weight, weight, cos, sin, 0, 0, 0, eps,
                                         stream);
}

Q6_API int q6_qk_rmsnorm_rope_joint_bf16(uint16_t* qk, int64_t row_stride, int64_t M, int heads, int head_dim,
                                         const uint16_t* weight_text, const uint16_t* weight_image, const float* cos,
                                         const float* sin, int64_t row0, int64_t seq_len, int64_t text_len, float eps,
                                         q6_stream_t stream) {
    if (!qk || !weight_text || !weight_image || !cos || !sin || M <= 0 || heads <= 0 || !(eps >= 0.0f))
        return Q6_ERR_INVALID_ARGUMENT;
    if (row0 < 0 || seq_len < 0 || text_len < 0 || text_len > seq_len) return Q6_ERR_INVALID_ARGUMENT;
    if (head_dim != 128 || row_stride < static_cast<int64_t>(heads) * head_dim) return Q6_ERR_SHAPE;
    const uintptr_t al = reinterpret_cast<uintptr_t>(qk) | reinterpret_cast<uintptr_t>(weight_text) |
                         reinterpret_cast<uintptr_t>(weight_image) | reinterpret_cast<uintptr_t>(cos) |
                         reinterpret_cast<uintptr_t>(sin);
    if (al % 16 != 0 || row_stride % 8 != 0) return Q6_ERR_ALIGNMENT;
    const int64_t blocks = (M + q6::kRopeWarps - 1) / q6::kRopeWarps;
    const cudaError_t e = q6::launch_pdl(
        q6::qk_rmsnorm_rope_kernel, dim3(static_cast<unsigned>(blocks)), dim3(q6::kRopeWarps * 32), 0,
        reinterpret_cast<cudaStream_t>(stream), reinterpret_cast<uint4*>(qk), row_stride / 8, M, heads,
        reinterpret_cast<const uint4*>(weight_text), reinterpret_cast<const uint4*>(weight_image),
        reinterpret_cast<const float4*>(cos), reinterpret_cast<const float4*>(sin), row0, seq_len, text_len, eps);
    return e == cudaSuccess ? Q6_OK : Q6_ERR_CUDA;
}

}  // extern "C"
