/*
 * q6_b200.h - C ABI of the B200 (sm_100a) q6 affine linear / image-FF MLP library.
 *
 * Weight format (MLX affine, bits = 6): for a linear with N outputs and K
 * inputs,
 *   w       uint32 [N, K*6/32]  6-bit codes, code k of row n in bits [6k, 6k+6)
 *                               of the row's little-endian word stream
 *   scales  bf16   [N, K/gs]    per-group scale
 *   qbiases bf16   [N, K/gs]    per-group bias, so  W[n,k] = scale*q + qbias
 *   bias    bf16   [N]          optional output bias
 * bf16 tensors are passed as uint16_t bit patterns.  All pointers are device
 * pointers, rows are dense (row stride = row length).  Calls are
 * stream-ordered on `stream` (a cudaStream_t; 0 = legacy default stream),
 * never synchronise, allocate no device memory, and are safe to issue from
 * several host threads on different streams.
 *
 * Every entry point returns 0 (Q6_OK) or a q6_status code; argument checks
 * happen before anything is launched.
 */
#ifndef Q6_B200_H
#define Q6_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define Q6_API __attribute__((visibility("default")))
#else
#define Q6_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* q6_stream_t; /* identical to cudaStream_t */

enum q6_status {
    Q6_OK = 0,
    Q6_ERR_INVALID_ARGUMENT = 1, /* null pointer or non-positive size        */
    Q6_ERR_SHAPE = 2,            /* K not a multiple of 16 or of group_size   */
    Q6_ERR_GROUP_SIZE = 3,       /* group_size not in {32, 64, 128}           */
    Q6_ERR_ALIGNMENT = 4,        /* pointer not aligned as the path requires  */
    Q6_ERR_UNSUPPORTED = 5,      /* requested path cannot run this problem    */
    Q6_ERR_CUDA = 6,             /* a CUDA runtime call failed                */
    Q6_ERR_DEVICE = 7,           /* a kernel raised the device error word     */
    Q6_ERR_WORKSPACE = 8         /* workspace missing or too small            */
};

/* Epilogue and operand flags (bit set). */
enum q6_epilogue {
    Q6_EPI_NONE = 0,
    Q6_EPI_GELU = 1,         /* GELU-tanh after the bias (mlx nn.gelu_approx), hardware tanh.approx */
    Q6_EPI_GELU_PRECISE = 2, /* the same GELU with the IEEE-accurate tanhf the reference kernel
                                calls (metal::precise::tanh, q6_metal_mlp.py:21-26); implies GELU */
    Q6_LORA_B_NMAJOR = 4     /* q6_linear_bf16 only: lora_b is laid out [N, r] (B transposed, each
                                output row's r values contiguous, 16-byte aligned), which the
                                fused LoRA stages read with 16-byte loads */
};

/* Site codes a kernel writes into the device error word when one of its
   bounded waits gives up (q6_get_device_error). */
enum q6_error_site {
    Q6_SITE_GEMM_MIN = 1,       /* 1..12: GEMM, GEMV and few-row MMA pipeline barriers */
    Q6_SITE_GEMM_MAX = 12,
    Q6_SITE_PEER_BARRIER = 13,  /* q6_sp_barrier: a peer's flag did not arrive in time */
    Q6_SITE_SELFTEST = 64       /* q6_selftest_bounded_wait */
};

/* Kernel path for q6_linear_bf16 (Q6_PATH_AUTO picks one). */
enum q6_path {
    Q6_PATH_AUTO = 0,
    Q6_PATH_SIMT = 1,   /* CUDA-core kernel, fp32 dequantised weights   */
    Q6_PATH_TENSOR = 2, /* tcgen05 kernel, bf16 dequantised weights     */
    Q6_PATH_SKINNY = 3  /* warp-MMA kernel for 1..16 token rows on the raw codes,
                           fp32 weight semantics, K a multiple of 512, group size
                           32 / 64 / 128; K split over a thread-block cluster */
};

/*
 * Dense bf16 weights from packed q6: out[n,k] = bf16_rn(fp32(scale)*q + fp32(qbias)).
 * Replaces `dequantize_linear` / mx.dequantize(mode="affine")
 * (shardedit_mlx/q6_metal_mlp.py:143-154).  out: uint16 [N, K].
 */
Q6_API int q6_dequantize_bf16(const uint32_t* w, const uint16_t* scales, const uint16_t* qbiases,
                       uint16_t* out, int64_t N, int64_t K, int group_size, q6_stream_t stream);

/*
 * y = epi(x @ dequant(W)^T)      x bf16 [M, K], y bf16 [M, N]
 * epi: + bias[n] (if bias), GELU (if flags & Q6_EPI_GELU, or with an accurate tanh if
 *      flags & Q6_EPI_GELU_PRECISE), then
 *      y = residual[m,n] + gate[n] * value  (each term only if its pointer is non-null).
 * LoRA (lora_xa bf16 [M, r] = x @ A computed by the caller, lora_b bf16 [r, N], or
 *      [N, r] with flags & Q6_LORA_B_NMAJOR, both non-null, r a multiple of 32 in
 *      [32, 256]): the value gains
 *      lora_scale * (lora_xa @ lora_b) before the bias, accumulated in the same
 *      fp32 tile as the q6 product (tensor-core path; Q6_PATH_SIMT returns
 *      Q6_ERR_UNSUPPORTED).
 * Replaces `affine_q6_qmm_t` (shardedit_mlx/q6_metal_mlp.py:157-204), its tiled
 * and simdgroup twins (q6_steel_mlp.py:163-220, q6_simdgroup_mlp.py:133-181),
 * the stock `mx.quantized_matmul(x, w, scales, biases, transpose=True,
 * group_size, bits=6)` + bias call (benchmarks/benchmark_qwen_gemm.py:188-200),
 * the LoRA-additive linear (dense_img_ff_window.py:48-60) and the block's
 * residual gate `x + gate * ff(x)` (benchmarks/profile_qwen_block.py:294-301).
 */
Q6_API int q6_linear_bf16(const uint16_t* x, const uint32_t* w, const uint16_t* scales,
                   const uint16_t* qbiases, const uint16_t* bias, const uint16_t* residual,
                   const uint16_t* gate, const uint16_t* lora_xa, const uint16_t* lora_b,
                   float lora_scale, int lora_rank, uint16_t* y, int64_t M, int64_t N, int64_t K,
                   int group_size, int flags, int path, void* workspace, size_t workspace_bytes,
                   q6_stream_t stream);

/*
 * LoRA pre-pass xa = x @ A (bf16 in, fp32 accumulation, bf16 out) for the
 * fused LoRA delta of q6_linear_bf16:  x bf16 [M, K], A bf16 [K, r] (row-major,
 * the adapter's down projection as the reference stores it), xa bf16 [M, r].
 * r a multiple of 32 in [32, 256], K a multiple of 16, 16-byte aligned
 * pointers.  Replaces the `x @ lora_A` half of the LoRA-additive linear
 * (dense_img_ff_window.py:48-60).  HBM-bound: each x row is read once.
 */
Q6_API int q6_lora_xa_bf16(const uint16_t* x, const uint16_t* a, uint16_t* xa, int64_t M, int64_t K, int r,
                           q6_stream_t stream);

/*
 * Workspace bytes with which q6_linear_bf16's tensor-core path splits K across
 * CTAs for an (M, N, K) problem whose tiles alone would leave SMs idle (few
 * tokens, or few output rows: 12288 -> 3072 at M <= 256).  0 when it would not
 * split.  Given at least this much 16-byte aligned workspace, the call writes
 * fp32 partial sums there and reduces them in a second kernel on the same
 * stream; with less (or none) it runs unsplit.  The split has no counterpart
 * in the reference, whose Metal kernels compute one output per thread.
 */
Q6_API size_t q6_linear_tc_workspace_bytes(int64_t M, int64_t N, int64_t K);

/*
 * fp32 activations in and out, fp32 dequantised weights (no bf16 rounding):
 * the dtype=float32 use of `affine_q6_qmm_t` (q6_metal_mlp.py:157-204) that the
 * reference's fp32 tests check against a dense fp32 matmul.
 * Bias / residual / gate stay bf16 as in the weight files.
 */
Q6_API int q6_linear_f32(const float* x, const uint32_t* w, const uint16_t* scales,
                  const uint16_t* qbiases, const uint16_t* bias, float* y, int64_t M, int64_t N,
                  int64_t K, int group_size, int flags, q6_stream_t stream);

/*
 * Image feed-forward MLP  y = fc2(gelu(fc1(x)))  [+ residual/gate epilogue]:
 *   x bf16 [M, D]; fc1: D -> H (+ bias, GELU); fc2: H -> D (+ bias); y bf16 [M, D].
 * The bf16 hidden [M, H] lives in the caller's workspace
 * (q6_mlp_workspace_bytes(M, H) bytes).  Workspace beyond that, counted
 * from the next 256-byte boundary, is split-K space for the two linears:
 * with max(q6_linear_tc_workspace_bytes(M, H, D),
 * q6_linear_tc_workspace_bytes(M, D, H)) bytes there, a linear whose tiles
 * alone would leave SMs idle (a few hundred tokens) splits K.
 * Replaces `fused_q6_mlp` (shardedit_mlx/q6_metal_mlp.py:207-215) and the
 * QwenFeedForward `img_ff(x)` call it stands in for (dense_img_ff_window.py:62-67).
 */
Q6_API int q6_mlp_bf16(const uint16_t* x, const uint32_t* w1, const uint16_t* scales1,
                const uint16_t* qbiases1, const uint16_t* bias1, const uint32_t* w2,
                const uint16_t* scales2, const uint16_t* qbiases2, const uint16_t* bias2,
                const uint16_t* residual, const uint16_t* gate, uint16_t* y, int64_t M, int64_t D,
                int64_t H, int group_size, void* workspace, size_t workspace_bytes,
                q6_stream_t stream);

Q6_API size_t q6_mlp_workspace_bytes(int64_t M, int64_t H);

/*
 * q6_mlp_bf16 for callers that cannot allocate device memory: the same fused
 * MLP, but the bf16 hidden activations live in a library-owned static device
 * array of 32 MiB per GPU (held by every GPU that loads the library until the
 * process exits) instead of a caller workspace.  Fits M * H * 2 <= 32 MiB
 * (1365 tokens at H = 12288); larger problems return Q6_ERR_WORKSPACE.
 * The call allocates nothing.  Its first call on a device looks the array's
 * address up once (make that first call before any stream capture).  All
 * calls share the array: calls whose GPU work overlaps race and give wrong
 * results, so order them on one stream.
 * No counterpart in the reference: it exists for plugin hosts, FFI bindings
 * and serving loops that receive only input/output pointers and must not call
 * cudaMalloc.
 */
Q6_API int q6_mlp_bf16_noalloc(const uint16_t* x, const uint32_t* w1, const uint16_t* scales1,
                               const uint16_t* qbiases1, const uint16_t* bias1, const uint32_t* w2,
                               const uint16_t* scales2, const uint16_t* qbiases2, const uint16_t* bias2,
                               const uint16_t* residual, const uint16_t* gate, uint16_t* y, int64_t M,
                               int64_t D, int64_t H, int group_size, q6_stream_t stream);

/*
 * MMDiT block steps around the q6 linears (the block's adaLN modulation and
 * attention pre-processing, benchmarks/profile_qwen_block.py:172-217).
 *
 * q6_layernorm_modulate_bf16: y[m, :] = LayerNorm(x[m, :]) * (1 + scale) + shift,
 *   LayerNorm without affine parameters (mean and variance over D, eps),
 *   computed in fp32 and rounded to bf16 once; shift / scale bf16 [D] (one
 *   sample's modulation vectors).  Replaces `_modulate(img_norm1(x), mod1)`.
 *   D in {256, 512, 768, 1024, 1536, 2048, 3072, 4096}, 16-byte aligned pointers.
 * q6_qk_rmsnorm_rope_bf16: in place on M rows of `heads` heads of head_dim
 *   (128) values, row stride `row_stride` elements: per head
 *   x <- rope(x * rsqrt(mean(x^2) + eps) * weight), weight bf16 [128]; the
 *   rotation turns interleaved pairs (x[2i], x[2i+1]) by the angle whose
 *   cosine / sine are cos[m, i] / sin[m, i] (fp32 [M, 64]).  Replaces
 *   norm_q / norm_k followed by `_apply_rope_qwen`.
 */
Q6_API int q6_layernorm_modulate_bf16(const uint16_t* x, const uint16_t* shift, const uint16_t* scale, uint16_t* y,
                                      int64_t M, int64_t D, float eps, q6_stream_t stream);

/*
 * The residual add and adaLN modulate of a block over rows of a joint,
 * batched sequence (several samples, each [text; image] rows):
 *   h[m, :] = x[m, :] + add[m, :]        (bf16 rounding once; h = x when add is null)
 *   y[m, :] = LayerNorm(h[m, :]) * (1 + scale[v]) + shift[v]
 * where local row m is global row g = row0 + m of sequences of seq_len rows,
 * the first text_len of each from the text stream:
 *   v = (g / seq_len) * 2 + ((g % seq_len) >= text_len ? 1 : 0),
 * i.e. shift / scale hold [samples][text, image] vectors of D values, vector
 * v starting vec_stride elements after vector v - 1 (vec_stride 0 means D;
 * else a multiple of 8 and >= D, so the vectors can be one chunk of each
 * [samples][text, image][6][D] modulation output in place).  h_out (nullable)
 * receives h.  With seq_len = text_len = 0 every row takes vector 0 (the
 * plain q6_layernorm_modulate_bf16).  Replaces `x + gate * attn_out` /
 * `x + gate * ff` followed by `_modulate(norm2(x), mod2)` and the next block's
 * `_modulate(norm1(x), mod1)` (benchmarks/profile_qwen_block.py:253-263) when
 * the gated term arrives from a reduce-scatter of tensor-parallel partials.
 * D and alignment as q6_layernorm_modulate_bf16.
 */
Q6_API int q6_add_layernorm_modulate_bf16(const uint16_t* x, const uint16_t* add, uint16_t* h_out,
                                          const uint16_t* shift, const uint16_t* scale, int64_t vec_stride,
                                          uint16_t* y, int64_t M, int64_t D, int64_t row0, int64_t seq_len,
                                          int64_t text_len, float eps, q6_stream_t stream);
Q6_API int q6_qk_rmsnorm_rope_bf16(uint16_t* qk, int64_t row_stride, int64_t M, int heads, int head_dim,
                                   const uint16_t* weight, const float* cos, const float* sin, float eps,
                                   q6_stream_t stream);

/*
 * q6_qk_rmsnorm_rope_bf16 over rows of a joint, batched sequence: local row m
 * is global row g = row0 + m of sequences of seq_len rows whose first
 * text_len rows are text.  The row takes angle-table row g % seq_len
 * (cos / sin fp32 [seq_len, 64], text rows first) and the RMSNorm weight
 * weight_text for text rows (norm_added_q / norm_added_k) or weight_image
 * for image rows (norm_q / norm_k), so one launch covers the q (or k)
 * columns of every stream and sample.  seq_len = 0: one sequence of M rows,
 * weight_image throughout.  Replaces the four norm + `_apply_rope_qwen`
 * calls of the block (benchmarks/profile_qwen_block.py:203-217).
 */
Q6_API int q6_qk_rmsnorm_rope_joint_bf16(uint16_t* qk, int64_t row_stride, int64_t M, int heads, int head_dim,
                                         const uint16_t* weight_text, const uint16_t* weight_image, const float* cos,
                                         const float* sin, int64_t row0, int64_t seq_len, int64_t text_len, float eps,
                                         q6_stream_t stream);

/*
 * Sequence-parallel step of the tensor-parallel block over peer memory (one
 * rank per GPU, `world` <= 8 ranks; pointer tables are HOST arrays of `world`
 * device pointers, this rank's own at index `rank`, each addressable from this
 * GPU: CUDA peer mappings of buffers every rank allocated alike).  This rank
 * owns joint rows [rank R, (rank + 1) R) of [world R, D].  The kernel forms
 *   h = x_local + sum_r partials[r][own rows]   (rank order, fp32, one bf16 rounding;
 *                                                h = x_local without partials)
 * writes h to h_out (nullable), and writes
 *   y = LayerNorm(h) * (1 + scale[v]) + shift[v]   (v and vec_stride as q6_add_layernorm_modulate_bf16)
 * into the own-row block of every gathered[r] (gathered null: only h, which
 * then needs partials and h_out; shift / scale may be null).  It is the reduce-scatter of
 * the row-parallel GEMM's partial sums, the residual add, the adaLN modulate
 * and the all-gather the next column-parallel GEMM needs, in one kernel
 * (benchmarks/profile_qwen_block.py:253-263 with the block split over
 * GPUs).  Order it between q6_sp_barrier calls: the partials of every rank
 * complete before it runs, and its stores reach every rank before anyone
 * reads them.  D in {256, 512, 1024, 3072}.
 */
Q6_API int q6_sp_add_layernorm_gather_bf16(const uint16_t* x_local, const uint16_t* const* partials,
                                           uint16_t* h_out, const uint16_t* shift, const uint16_t* scale,
                                           int64_t vec_stride, uint16_t* const* gathered, int world, int rank,
                                           int64_t R, int64_t D, int64_t seq_len, int64_t text_len, float eps,
                                           q6_stream_t stream);

/*
 * Barrier of `world` ranks for the kernels above: one thread per peer
 * publishes this rank's new epoch (system-scope release, after everything
 * this GPU did before on the stream) into slot `rank` of that peer's signal
 * array and waits until the peer's epoch is in slot `peer` of this rank's.
 * signals: host array of `world` device pointers to uint32[world] (zeroed
 * once, like `epoch`, before the first barrier); epoch: this rank's device
 * counter, advanced by the barrier itself, so graph replays see new epochs.
 * A wait longer than timeout_ns (1 us .. 60 s) records
 * Q6_SITE_PEER_BARRIER in the device error word and gives up.
 */
Q6_API int q6_sp_barrier(uint32_t* const* signals, uint32_t* epoch, int world, int rank, int64_t timeout_ns,
                         q6_stream_t stream);

/* Device error word (0 = none, else a q6_error_site code).  Reading it
   synchronises the current device. */
Q6_API int q6_get_device_error(int* code);
Q6_API int q6_clear_device_error(void);

/*
 * Self-test of the failure path every pipeline wait in this library takes:
 * one CTA initialises an mbarrier that nothing ever arrives at and waits on
 * it through the same bounded wait the GEMM's barriers use, with a limit of
 * limit_ns (1 us .. 1 s).  When the limit passes the wait records
 * Q6_SITE_SELFTEST in the device error word and the kernel returns; no copy
 * is in flight.  The call returns Q6_OK once launched; the result is read
 * with q6_get_device_error.  No counterpart in the reference (it has no
 * device-side hang detection).
 */
Q6_API int q6_selftest_bounded_wait(int64_t limit_ns, q6_stream_t stream);

/* Path the last q6_linear_bf16 / q6_mlp_bf16 call on this host thread launched. */
Q6_API int q6_last_path(void);

/* Token tile (MMA N) the tensor path would use for an M x N problem. */
Q6_API int q6_tensor_token_tile(int64_t M, int64_t N);

/* Plan the few-row path (Q6_PATH_SKINNY) would launch for an M x N x K problem at
   this group size on the current device: *tpw 16-row weight tiles per warp (row
   blocks of 32 * tpw rows), *split CTAs per thread-block cluster sharing K, and
   *clusters clusters.  Q6_ERR_UNSUPPORTED when the shape is outside the path. */
Q6_API int q6_skinny_plan(int64_t M, int64_t N, int64_t K, int group_size, int* tpw, int* split,
                          int* clusters);

/* How many tensor-path launches in this process asked for CTA pairs (two-CTA
   clusters sharing one cta_group::2 MMA), were refused by the device before
   anything ran, and ran one CTA per tile instead. */
Q6_API int64_t q6_pair_fallback_count(void);

Q6_API const char* q6_status_string(int status);
Q6_API int q6_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* Q6_B200_H */
