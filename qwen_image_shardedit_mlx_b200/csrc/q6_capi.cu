// extern "C" entry points of libq6b200.so (declared in include/q6_b200.h).
//
// Each entry point validates its arguments the way the reference's Python
// surface does (rank/width checks and bits/group-size checks at
// shardedit_mlx/q6_metal_mlp.py:114-134 and :166-173 raise ValueError; here
// they return a q6_status code before any launch), then dispatches to a
// kernel path.  No entry point allocates device memory or synchronises.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdlib>

#include "q6_b200.h"
#include "q6_internal.h"

namespace {

thread_local int g_last_path = Q6_PATH_AUTO;

constexpr int kEpiFlags = Q6_EPI_GELU | Q6_EPI_GELU_PRECISE;

bool valid_group_size(int gs) { return gs == 32 || gs == 64 || gs == 128; }

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

int check_weights(const uint32_t* w, const uint16_t* scales, const uint16_t* qbiases, int64_t N, int64_t K,
                  int group_size) {
    if (!w || !scales || !qbiases) return Q6_ERR_INVALID_ARGUMENT;
    if (N <= 0 || K <= 0) return Q6_ERR_INVALID_ARGUMENT;
    if (!valid_group_size(group_size)) return Q6_ERR_GROUP_SIZE;
    if (K % group_size != 0 || K % 16 != 0) return Q6_ERR_SHAPE;
    if (!aligned(w, 4) || !aligned(scales, 2) || !aligned(qbiases, 2)) return Q6_ERR_ALIGNMENT;
    return Q6_OK;
}

// The SIMT path loads activations 16 at a time with 16-byte vector loads.
bool simt_aligned(const void* x, int64_t K, int elem_bytes) {
    return aligned(x, 16) && ((K * elem_bytes) % 16 == 0);
}

// Few-row policy of the auto path, from B200 measurements with rotating weights
// larger than 4x L2 (3072 <-> 12288, 3072 -> 18432 / 36864, group sizes
// 32 / 64 / 128): the warp-MMA kernel for 2..16 token rows when the weights hold
// at least 2^24 codes (3072 -> 12288: 12.1-14.2 us against the tensor path's
// 16.8 us; 3072 -> 36864 at 2 rows: 26.1 us against the GEMV's 32.9 us), except
// group size 32 past 8 rows; the streaming GEMV for one row (10.4 us against
// 12.1 us) and for small weights.  Q6_SKINNY=1 takes the warp-MMA kernel for
// every 1..16-row shape it supports, Q6_SKINNY=0 never (read once per process).
bool skinny_auto(const q6::LinearArgs& a) {
    static const int mode = [] {
        const char* v = std::getenv("Q6_SKINNY");
        if (!v || !v[0]) return -1;
        return v[0] == '1' ? 1 : 0;
    }();
    if (mode == 0 || a.lora_rank > 0 || !q6::skinny_supported(a)) return false;
    if (mode == 1) return true;
    return a.M >= 2 && a.N * a.K >= (int64_t(1) << 24) && (a.group_size != 32 || a.M <= 8);
}

int run_linear(const q6::LinearArgs& a, int path, cudaStream_t stream) {
    const bool tc_ok = q6::tc_supported(a);
    int chosen = path;
    if (chosen == Q6_PATH_AUTO) {
        if (skinny_auto(a))
            chosen = Q6_PATH_SKINNY;
        else
            // The streaming GEMV at 1-2 rows; from 3 rows the tensor-core path
            // (at 4 rows 3072 -> 3072: 6.5 us against 7.9 us).
            chosen = (tc_ok && (a.M > 2 || a.lora_rank > 0)) ? Q6_PATH_TENSOR : Q6_PATH_SIMT;
    }
    if (chosen == Q6_PATH_SKINNY) {
        if (a.lora_rank > 0 || !q6::skinny_supported(a)) return Q6_ERR_UNSUPPORTED;
        g_last_path = Q6_PATH_SKINNY;
        return q6::launch_skinny(a, stream);
    }
    if (chosen == Q6_PATH_TENSOR) {
        if (!tc_ok) return Q6_ERR_UNSUPPORTED;
        g_last_path = Q6_PATH_TENSOR;
        return q6::launch_linear_tc(a, q6::choose_token_tile(a.M, a.N), stream);
    }
    if (chosen == Q6_PATH_SIMT) {
        if (a.lora_rank > 0) return Q6_ERR_UNSUPPORTED;  // the LoRA delta is fused on the tensor-core path
        if (!simt_aligned(a.x, a.K, 2)) return Q6_ERR_ALIGNMENT;
        g_last_path = Q6_PATH_SIMT;
        if (q6::gemv_supported(a)) return q6::launch_gemv(a, stream);
        return q6::launch_linear_simt(a, false, stream);
    }
    return Q6_ERR_INVALID_ARGUMENT;
}

}  // namespace

extern "C" {

int q6_abi_version(void) { return 2; }

const char* q6_status_string(int status) {
    switch (status) {
        case Q6_OK: return "ok";
        case Q6_ERR_INVALID_ARGUMENT: return "invalid argument (null pointer or non-positive size)";
        case Q6_ERR_SHAPE: return "K must be a multiple of 16 and of group_size";
        case Q6_ERR_GROUP_SIZE: return "group_size must be 32, 64 or 128";
        case Q6_ERR_ALIGNMENT: return "pointer alignment not supported by this path";
        case Q6_ERR_UNSUPPORTED: return "the requested path cannot run this problem";
        case Q6_ERR_CUDA: return "a CUDA runtime call failed";
        case Q6_ERR_DEVICE: return "a kernel reported a device-side error";
        case Q6_ERR_WORKSPACE: return "workspace missing or too small";
        default: return "unknown status";
    }
}

int q6_dequantize_bf16(const uint32_t* w, const uint16_t* scales, const uint16_t* qbiases, uint16_t* out,
                       int64_t N, int64_t K, int group_size, q6_stream_t stream) {
    int st = check_weights(w, scales, qbiases, N, K, group_size);
    if (st != Q6_OK) return st;
    if (!out) return Q6_ERR_INVALID_ARGUMENT;
    if (!aligned(out, 16)) return Q6_ERR_ALIGNMENT;
    return q6::launch_dequantize(w, scales, qbiases, out, N, K, group_size, reinterpret_cast<cudaStream_t>(stream));
}

size_t q6_linear_tc_workspace_bytes(int64_t M, int64_t N, int64_t K) { return q6::tc_workspace_bytes(M, N, K); }

int q6_linear_bf16(const uint16_t* x, const uint32_t* w, const uint16_t* scales, const uint16_t* qbiases,
                   const uint16_t* bias, const uint16_t* residual, const uint16_t* gate, const uint16_t* lora_xa,
                   const uint16_t* lora_b, float lora_scale, int lora_rank, uint16_t* y, int64_t M, int64_t N,
                   int64_t K, int group_size, int flags, int path, void* workspace, size_t workspace_bytes,
                   q6_stream_t stream) {
    int st = check_weights(w, scales, qbiases, N, K, group_size);
    if (st != Q6_OK) return st;
    if (!x || !y || M <= 0) return Q6_ERR_INVALID_ARGUMENT;
    if ((flags & ~(kEpiFlags | Q6_LORA_B_NMAJOR)) != 0) return Q6_ERR_INVALID_ARGUMENT;
    if (flags & Q6_EPI_GELU_PRECISE) flags |= Q6_EPI_GELU;  // the precise flag implies GELU
    if ((lora_xa == nullptr) != (lora_b == nullptr)) return Q6_ERR_INVALID_ARGUMENT;
    if (lora_xa && lora_rank <= 0) return Q6_ERR_INVALID_ARGUMENT;
    if ((flags & Q6_LORA_B_NMAJOR) && (!lora_b || !aligned(lora_b, 16))) return Q6_ERR_INVALID_ARGUMENT;
    q6::LinearArgs a{x, w, scales, qbiases, bias, residual, gate, y, M, N, K, group_size, flags};
    if (lora_xa) {
        a.lora_xa = lora_xa;
        a.lora_b = lora_b;
        a.lora_scale = lora_scale;
        a.lora_rank = lora_rank;
    }
    a.workspace = workspace;
    a.workspace_bytes = workspace ? workspace_bytes : 0;
    return run_linear(a, path, reinterpret_cast<cudaStream_t>(stream));
}

int q6_linear_f32(const float* x, const uint32_t* w, const uint16_t* scales, const uint16_t* qbiases,
                  const uint16_t* bias, float* y, int64_t M, int64_t N, int64_t K, int group_size, int flags,
                  q6_stream_t stream) {
    int st = check_weights(w, scales, qbiases, N, K, group_size);
    if (st != Q6_OK) return st;
    if (!x || !y || M <= 0) return Q6_ERR_INVALID_ARGUMENT;
    if ((flags & ~kEpiFlags) != 0) return Q6_ERR_INVALID_ARGUMENT;
    if (flags & Q6_EPI_GELU_PRECISE) flags |= Q6_EPI_GELU;
    if (!simt_aligned(x, K, 4)) return Q6_ERR_ALIGNMENT;
    q6::LinearArgs a{x, w, scales, qbiases, bias, nullptr, nullptr, y, M, N, K, group_size, flags};
    g_last_path = Q6_PATH_SIMT;
    return q6::launch_linear_simt(a, true, reinterpret_cast<cudaStream_t>(stream));
}

size_t q6_mlp_workspace_bytes(int64_t M, int64_t H) {
    if (M <= 0 || H <= 0) return 0;
    return static_cast<size_t>(M) * static_cast<size_t>(H) * 2;
}

int q6_mlp_bf16(const uint16_t* x, const uint32_t* w1, const uint16_t* scales1, const uint16_t* qbiases1,
                const uint16_t* bias1, const uint32_t* w2, const uint16_t* scales2, const uint16_t* qbiases2,
                const uint16_t* bias2, const uint16_t* residual, const uint16_t* gate, uint16_t* y, int64_t M,
                int64_t D, int64_t H, int group_size, void* workspace, size_t workspace_bytes,
                q6_stream_t stream) {
    int st = check_weights(w1, scales1, qbiases1, H, D, group_size);
    if (st != Q6_OK) return st;
    st = check_weights(w2, scales2, qbiases2, D, H, group_size);
    if (st != Q6_OK) return st;
    if (!x || !y || M <= 0) return Q6_ERR_INVALID_ARGUMENT;
    if (!workspace || workspace_bytes < q6_mlp_workspace_bytes(M, H)) return Q6_ERR_WORKSPACE;
    if (!aligned(workspace, 16)) return Q6_ERR_ALIGNMENT;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    uint16_t* hidden = static_cast<uint16_t*>(workspace);
    // Workspace past the hidden activations (from a 256-byte boundary) is the
    // linears' split-K space: with q6_linear_tc_workspace_bytes of a linear
    // there, a few-hundred-token fc2 (K = H) splits K instead of leaving SMs idle.
    const size_t split_off = (q6_mlp_workspace_bytes(M, H) + 255) & ~size_t(255);
    void* split_ws = workspace_bytes > split_off ? static_cast<char*>(workspace) + split_off : nullptr;
    const size_t split_bytes = workspace_bytes > split_off ? workspace_bytes - split_off : 0;
    q6::LinearArgs a1{x, w1, scales1, qbiases1, bias1, nullptr, nullptr, hidden, M, H, D, group_size, Q6_EPI_GELU};
    a1.workspace = split_ws;
    a1.workspace_bytes = split_bytes;
    st = run_linear(a1, Q6_PATH_AUTO, s);
    if (st != Q6_OK) return st;
    q6::LinearArgs a2{hidden, w2, scales2, qbiases2, bias2, residual, gate, y, M, D, H, group_size, Q6_EPI_NONE};
    a2.workspace = split_ws;
    a2.workspace_bytes = split_bytes;
    return run_linear(a2, Q6_PATH_AUTO, s);
}

int q6_get_device_error(int* code) {
    if (!code) return Q6_ERR_INVALID_ARGUMENT;
    if (cudaDeviceSynchronize() != cudaSuccess) return Q6_ERR_CUDA;
    const int words[5] = {q6::error_word_simt(false), q6::error_word_tc(false), q6::error_word_gemv(false),
                          q6::error_word_skinny(false), q6::error_word_sp(false)};
    *code = 0;
    for (int w : words) {
        if (w < 0) return Q6_ERR_CUDA;
        if (*code == 0) *code = w;
    }
    return Q6_OK;
}

int q6_clear_device_error(void) {
    if (cudaDeviceSynchronize() != cudaSuccess) return Q6_ERR_CUDA;
    if (q6::error_word_simt(true) < 0 || q6::error_word_tc(true) < 0 || q6::error_word_gemv(true) < 0 ||
        q6::error_word_skinny(true) < 0 || q6::error_word_sp(true) < 0)
        return Q6_ERR_CUDA;
    return Q6_OK;
}

int q6_last_path(void) { return g_last_path; }

int64_t q6_pair_fallback_count(void) { return static_cast<int64_t>(q6::pair_fallbacks()); }

int q6_selftest_bounded_wait(int64_t limit_ns, q6_stream_t stream) {
    if (limit_ns < 1000 || limit_ns > 1000000000) return Q6_ERR_INVALID_ARGUMENT;
    return q6::launch_selftest_wait(static_cast<uint64_t>(limit_ns), reinterpret_cast<cudaStream_t>(stream));
}

int q6_lora_xa_bf16(const uint16_t* x, const uint16_t* a, uint16_t* xa, int64_t M, int64_t K, int r,
                    q6_stream_t stream) {
    if (!x || !a || !xa || M <= 0 || K <= 0) return Q6_ERR_INVALID_ARGUMENT;
    if (r < 32 || r > 256 || r % 32 != 0 || K % 16 != 0) return Q6_ERR_SHAPE;
    const uintptr_t al = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(a) |
                         reinterpret_cast<uintptr_t>(xa);
    if (al % 16 != 0) return Q6_ERR_ALIGNMENT;
    return q6::launch_lora_xa(x, a, xa, M, K, r, reinterpret_cast<cudaStream_t>(stream));
}

int q6_tensor_token_tile(int64_t M, int64_t N) {
    if (M <= 0 || N <= 0) return 0;
    return q6::choose_token_tile(M, N);
}

int q6_skinny_plan(int64_t M, int64_t N, int64_t K, int group_size, int* tpw, int* split, int* clusters) {
    if (!tpw || !split || !clusters) return Q6_ERR_INVALID_ARGUMENT;
    q6::LinearArgs a{};
    a.M = M;
    a.N = N;
    a.K = K;
    a.group_size = group_size;
    if (M <= 0 || N <= 0 || K <= 0 || !q6::skinny_supported(a)) return Q6_ERR_UNSUPPORTED;
    return q6::skinny_plan(a, tpw, split, clusters);
}

}  // extern "C"
