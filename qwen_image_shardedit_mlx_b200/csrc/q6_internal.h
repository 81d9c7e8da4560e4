// Host-side interfaces between the C ABI (q6_capi.cu) and the kernel launchers.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "q6_b200.h"

namespace q6 {

// Device ordinals the per-device host caches cover; calls on a higher ordinal
// return Q6_ERR_UNSUPPORTED.
constexpr int kMaxDevices = 64;

// Operands of one q6 linear, y = epilogue(x @ dequant(W)^T).
struct LinearArgs {
    const void* x;          // [M, K] bf16 (or fp32 for the fp32 path), row-major
    const uint32_t* w;      // [N, K*6/32] packed codes
    const uint16_t* scales; // [N, K/gs] bf16
    const uint16_t* qbiases;// [N, K/gs] bf16
    const uint16_t* bias;   // [N] bf16 or null
    const uint16_t* residual;  // [M, N] bf16 or null
    const uint16_t* gate;      // [N] bf16 or null
    void* y;                // [M, N] bf16 (fp32 for the fp32 path)
    int64_t M, N, K;
    int group_size;
    int flags;              // Q6_EPI_* bits
    // Optional LoRA delta lora_scale * (lora_xa @ lora_b): xa = x @ A bf16 [M, r]
    // (computed by the caller), B bf16 [r, N].  Tensor-core path only.
    const uint16_t* lora_xa = nullptr;
    const uint16_t* lora_b = nullptr;
    float lora_scale = 0.0f;
    int lora_rank = 0;
    // Caller workspace (device memory).  The tensor-core path splits K across
    // CTAs when the tiles alone would leave SMs idle and this holds
    // tc_workspace_bytes(M, N, K) bytes; otherwise it is not touched.
    void* workspace = nullptr;
    size_t workspace_bytes = 0;
};

// Path selection recorded for tests and benchmarks.
enum class Path : int { kNone = 0, kSimt = 1, kTensor = 2 };

int launch_dequantize(const uint32_t* w, const uint16_t* scales, const uint16_t* qbiases,
                      uint16_t* out, int64_t N, int64_t K, int group_size, cudaStream_t stream);

// CUDA-core path: any shape the format allows, bf16 or fp32 activations,
// fp32 (un-rounded) dequantised weights.
int launch_linear_simt(const LinearArgs& a, bool f32_io, cudaStream_t stream);

// Streaming GEMV for M <= 4 bf16 rows (fp32 dequantised weights, like the
// CUDA-core path) when K % 64 == 0, K / group_size % 8 == 0, K <= 4096 or
// K % 4096 == 0, the operands are 16-byte aligned and the fp32 activations fit
// in shared memory.
bool gemv_supported(const LinearArgs& a);
int launch_gemv(const LinearArgs& a, cudaStream_t stream);

// Warp-level MMA path for 1 <= M <= 16 bf16 rows on the raw codes (fp32
// weight semantics): group size 32, 64 or 128, K % 512 == 0,
// (K / group_size) % 8 == 0, 16-byte aligned x, codes, scales and biases,
// no LoRA.  K is split over the CTAs of a cluster where that balances the SMs.
bool skinny_supported(const LinearArgs& a);
int launch_skinny(const LinearArgs& a, cudaStream_t stream);
// The few-row path's plan for a shape (tiles per warp, K split, clusters).
int skinny_plan(const LinearArgs& a, int* tpw, int* split, int* clusters);

// tcgen05 path: bf16 activations, bf16-dequantised weights, fp32 accumulate.
// Requires K % 64 == 0 and 16-byte aligned x / w rows.
int launch_linear_tc(const LinearArgs& a, int token_tile, cudaStream_t stream);

// Token tile the tensor-core path picks for an (M, N) problem.
int choose_token_tile(int64_t M, int64_t N);

// Workspace bytes the tensor-core path's split-K uses for (M, N, K) (0: no split).
size_t tc_workspace_bytes(int64_t M, int64_t N, int64_t K);

bool tc_supported(const LinearArgs& a);

int device_sm_count();

// Programmatic dependent launch for the kernels that execute pdl_wait before
// their dependent reads and writes (Q6_PDL=0 turns the attribute off).
bool pdl_enabled();

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Times a CTA-pair GEMM launch was refused by the device and ran one CTA per
// tile instead (process-wide).
long pair_fallbacks();

// Bounded-wait self-test kernel (q6_selftest_bounded_wait).
int launch_selftest_wait(uint64_t limit_ns, cudaStream_t stream);

// LoRA pre-pass xa = x @ A (q6_lora_xa_bf16).
int launch_lora_xa(const uint16_t* x, const uint16_t* a, uint16_t* xa, int64_t M, int64_t K, int r,
                   cudaStream_t stream);

// Per-translation-unit device error words (value, optionally cleared; -1 on
// a failed copy).
int error_word_simt(bool clear);
int error_word_tc(bool clear);
int error_word_gemv(bool clear);
int error_word_skinny(bool clear);
int error_word_sp(bool clear);

}  // namespace q6
