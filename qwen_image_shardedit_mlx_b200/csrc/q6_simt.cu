// CUDA-core q6 kernels: dense dequantisation and a warp-per-output-row linear.
//
// The linear here keeps fp32 dequantised weights, exactly like the reference
// kernel's `scale * float(code) + qbias` (shardedit_mlx/q6_metal_mlp.py:42-83),
// so it also serves fp32 activations (the reference's dtype=float32 tests) and
// shapes the tensor-core path does not take (K % 64 != 0, M of a few rows).
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

__device__ __forceinline__ float bf16f(uint16_t v) { return __uint_as_float(static_cast<uint32_t>(v) << 16); }

// ---------------------------------------------------------------- dequant

// One thread per 16 codes: three words in, sixteen bf16 (two 16-byte stores) out.
__global__ void __launch_bounds__(256) dequantize_kernel(const uint32_t* __restrict__ w,
                                                         const uint16_t* __restrict__ scales,
                                                         const uint16_t* __restrict__ qbiases,
                                                         uint4* __restrict__ out, int64_t N,
                                                         int64_t K, int gs) {
    const int64_t units_per_row = K / 16;
    const int64_t words_per_row = K * 6 / 32;
    const int64_t groups = K / gs;
    const int64_t total = N * units_per_row;
    for (int64_t u = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; u < total;
         u += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t n = u / units_per_row;
        const int64_t j = u - n * units_per_row;
        const uint32_t* src = w + n * words_per_row + j * 3;
        const int64_t g = n * groups + (j * 16) / gs;
        const float s = bf16f(__ldg(scales + g));
        const float b = bf16f(__ldg(qbiases + g));
        uint32_t o[8];
        dequant16_bf16x2(__ldg(src), __ldg(src + 1), __ldg(src + 2), s, b, o);
        uint4* dst = out + u * 2;
        dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
        dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
    }
}

// ------------------------------------------------------------------ linear

__device__ __forceinline__ float gelu_precise(float x) {
    const float x3 = x * x * x;
    return 0.5f * x * (1.0f + tanhf(0.7978845608028654f * (x + 0.044715f * x3)));
}

template <bool kF32>
__device__ __forceinline__ void load_x16(const void* x, int64_t row, int64_t K, int64_t j, float (&v)[16]) {
    if constexpr (kF32) {
        const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(x) + row * K + j * 16);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float4 t = __ldg(p + i);
            v[4 * i] = t.x; v[4 * i + 1] = t.y; v[4 * i + 2] = t.z; v[4 * i + 3] = t.w;
        }
    } else {
        const uint4* p = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(x) + row * K + j * 16);
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const uint4 t = __ldg(p + i);
            const uint32_t words[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                v[8 * i + 2 * q] = __uint_as_float(words[q] << 16);
                v[8 * i + 2 * q + 1] = __uint_as_float(words[q] & 0xFFFF0000u);
            }
        }
    }
}

// One warp per (output row n, chunk of MT tokens); lanes stride over 16-code units.
template <bool kF32, int MT>
__global__ void __launch_bounds__(256) linear_simt_kernel(const LinearArgs a) {
    const int lane = threadIdx.x & 31;
    const int64_t warp = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
    const int64_t num_warps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    const int64_t units = a.K / 16;
    const int64_t words_per_row = a.K * 6 / 32;
    const int64_t groups = a.K / a.group_size;
    const int64_t chunks = (a.M + MT - 1) / MT;
    const int64_t work = a.N * chunks;
    for (int64_t t = warp; t < work; t += num_warps) {
        const int64_t n = t % a.N;
        const int64_t m0 = (t / a.N) * MT;
        const int mt = static_cast<int>(a.M - m0 < MT ? a.M - m0 : MT);
        float acc[MT];
#pragma unroll
        for (int i = 0; i < MT; ++i) acc[i] = 0.0f;
        const uint32_t* wrow = a.w + n * words_per_row;
        for (int64_t j = lane; j < units; j += 32) {
            const int64_t g = n * groups + (j * 16) / a.group_size;
            float wv[16];
            dequant16_f32(__ldg(wrow + 3 * j), __ldg(wrow + 3 * j + 1), __ldg(wrow + 3 * j + 2),
                          bf16f(__ldg(a.scales + g)), bf16f(__ldg(a.qbiases + g)), wv);
#pragma unroll
            for (int i = 0; i < MT; ++i) {
                if (i < mt) {
                    float xv[16];
                    load_x16<kF32>(a.x, m0 + i, a.K, j, xv);
                    float s = acc[i];
#pragma unroll
                    for (int e = 0; e < 16; ++e) s = fmaf(xv[e], wv[e], s);
                    acc[i] = s;
                }
            }
        }
#pragma unroll
        for (int i = 0; i < MT; ++i) {
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], off);
        }
        if (lane < mt) {
            float v = acc[0];
#pragma unroll
            for (int i = 1; i < MT; ++i)
                if (lane == i) v = acc[i];
            const int64_t m = m0 + lane;
            if (a.bias) v += bf16f(a.bias[n]);
            if (a.flags & (Q6_EPI_GELU | Q6_EPI_GELU_PRECISE)) v = gelu_precise(v);
            if (a.gate) v *= bf16f(a.gate[n]);
            if (a.residual) v += bf16f(a.residual[m * a.N + n]);
            if constexpr (kF32) {
                static_cast<float*>(a.y)[m * a.N + n] = v;
            } else {
                __nv_bfloat16 h = __float2bfloat16_rn(v);
                static_cast<uint16_t*>(a.y)[m * a.N + n] = *reinterpret_cast<uint16_t*>(&h);
            }
        }
    }
}

// ------------------------------------------------------------ self-test

// One thread waits on an mbarrier that nothing arrives at, through the same
// bounded wait the GEMM pipeline uses, so the wait runs out after limit_ns,
// records Q6_SITE_SELFTEST in the device error word and returns.  No copy is
// in flight and no tensor memory is held when it gives up.
__global__ void __launch_bounds__(32) selftest_wait_kernel(uint64_t limit_ns) {
    __shared__ __align__(8) uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        mbar_init(smem_u32(&bar), 1);
        abort_flag = 0;
        fence_mbar_init();
    }
    __syncwarp();
    if (threadIdx.x == 0) {
        // phase 0 of a barrier expecting one arrival that never comes
        (void)mbar_wait_limit(smem_u32(&bar), 0u, &abort_flag, Q6_SITE_SELFTEST, limit_ns, 1000u);
    }
}

}  // namespace

int launch_selftest_wait(uint64_t limit_ns, cudaStream_t stream) {
    selftest_wait_kernel<<<1, 32, 0, stream>>>(limit_ns);
    return cudaGetLastError() == cudaSuccess ? Q6_OK : Q6_ERR_CUDA;
}

int error_word_simt(bool clear) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)) != cudaSuccess) return -1;
    if (clear && v != 0) {
        const int zero = 0;
        if (cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int)) != cudaSuccess) return -1;
    }
    return v;
}

bool pdl_enabled() {
    static std::atomic<int> v{-1};  // every thread computes the same value
    int cur = v.load(std::memory_order_relaxed);
    if (cur < 0) {
        const char* e = std::getenv("Q6_PDL");
        cur = (e && e[0] == '0') ? 0 : 1;
        v.store(cur, std::memory_order_relaxed);
    }
    return cur == 1;
}

int device_sm_count() {
    static std::atomic<int> cached[kMaxDevices];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (dev < 0 || dev >= kMaxDevices) return 148;
    int n = cached[dev].load(std::memory_order_relaxed);
    if (n == 0) {
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cached[dev].store(n, std::memory_order_relaxed);
    }
    return n;
}

int launch_dequantize(const uint32_t* w, const uint16_t* scales, const uint16_t* qbiases,
                      uint16_t* out, int64_t N, int64_t K, int group_size, cudaStream_t stream) {
    const int64_t total = N * (K / 16);
    const int threads = 256;
    const int64_t want = (total + threads - 1) / threads;
    const int blocks = static_cast<int>(std::min<int64_t>(want, static_cast<int64_t>(device_sm_count()) * 32));
    dequantize_kernel<<<blocks, threads, 0, stream>>>(w, scales, qbiases, reinterpret_cast<uint4*>(out),
                                                      N, K, group_size);
    return cudaGetLastError() == cudaSuccess ? Q6_OK : Q6_ERR_CUDA;
}

int launch_linear_simt(const LinearArgs& a, bool f32_io, cudaStream_t stream) {
    constexpr int kMT = 4;
    const int64_t chunks = (a.M + kMT - 1) / kMT;
    const int64_t warps = a.N * chunks;
    const int threads = 256;
    const int64_t want = (warps * 32 + threads - 1) / threads;
    const int blocks = static_cast<int>(std::min<int64_t>(want, static_cast<int64_t>(device_sm_count()) * 16));
    if (f32_io) {
        linear_simt_kernel<true, kMT><<<blocks, threads, 0, stream>>>(a);
    } else {
        linear_simt_kernel<false, kMT><<<blocks, threads, 0, stream>>>(a);
    }
    return cudaGetLastError() == cudaSuccess ? Q6_OK : Q6_ERR_CUDA;
}

}  // namespace q6
