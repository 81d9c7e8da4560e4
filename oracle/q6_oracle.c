/*
 * CPU oracle for the q6 affine linear / image feed-forward path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker: tests/, the smoke()
 * entry and bench.py's cpu_baseline leg may load it; the product library
 * never links it and never falls back to it.
 *
 * It restates, in plain C, the arithmetic of the reference's q6 path:
 *   - 6-bit codes as a continuous little-endian bit stream over uint32 words
 *     (shardedit_mlx/q6_metal_mlp.py:28-40, `extract_q6`);
 *   - affine dequantisation w = scale * q + bias, fp32
 *     (shardedit_mlx/q6_metal_mlp.py:42-54, `dequant_q6`);
 *   - the one-output-per-thread linear with fp32 accumulation in k order,
 *     optional output bias and GELU-tanh epilogue
 *     (shardedit_mlx/q6_metal_mlp.py:58-83, SOURCE_QMM_T; GELU at :21-26);
 *   - the bf16 pre-dequantised variant used by `dequantize_linear` /
 *     `dense_mlp` (shardedit_mlx/q6_metal_mlp.py:143-154, 218-232), where
 *     the dequantised weight is rounded to bf16 once: bf16_rn(fp32(s)*q + fp32(b)).
 *
 * Parity of this restatement is pinned against the reference's own kernel
 * source compiled for the CPU (oracle/build_ref.py -> oracle/_ref/) through
 * the golden vectors in tests/golden/.
 *
 * Build with -ffp-contract=off so that a*b+c is never fused: the reference
 * kernel performs the multiply and the add as separate fp32 operations.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define Q6_GELU_K 0.7978845608028654f /* sqrt(2/pi) */
#define Q6_GELU_C 0.044715f

float q6o_bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, sizeof f);
    return f;
}

/* Round-to-nearest-even fp32 -> bf16 (NaN stays NaN, made quiet). */
uint16_t q6o_f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, sizeof u);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x0040u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

/* Code `index` of one packed row: bits [6*index, 6*index+6) of the row's
 * little-endian word stream (q6_metal_mlp.py:29-40). */
uint32_t q6o_extract(const uint32_t *row, uint32_t index) {
    uint32_t bit = index * 6u;
    uint32_t word = bit >> 5;
    uint32_t shift = bit & 31u;
    uint32_t v = row[word] >> shift;
    if (shift > 26u) v |= row[word + 1] << (32u - shift);
    return v & 63u;
}

/* Inverse of q6o_extract: codes uint8 [rows, k] (values < 64) -> packed
 * uint32 [rows, k*6/32].  k must be a multiple of 16. */
void q6o_pack(const uint8_t *codes, int64_t rows, int64_t k, uint32_t *packed) {
    int64_t words = k * 6 / 32;
    memset(packed, 0, (size_t)(rows * words) * sizeof(uint32_t));
    for (int64_t r = 0; r < rows; ++r) {
        uint32_t *dst = packed + r * words;
        const uint8_t *src = codes + r * k;
        for (int64_t i = 0; i < k; ++i) {
            uint32_t v = (uint32_t)(src[i] & 63u);
            uint64_t bit = (uint64_t)i * 6u;
            uint32_t w = (uint32_t)(bit >> 5), s = (uint32_t)(bit & 31u);
            dst[w] |= v << s;
            if (s > 26u) dst[w + 1] |= v >> (32u - s);
        }
    }
}

void q6o_unpack(const uint32_t *packed, int64_t rows, int64_t k, uint8_t *codes) {
    int64_t words = k * 6 / 32;
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t i = 0; i < k; ++i)
            codes[r * k + i] = (uint8_t)q6o_extract(packed + r * words, (uint32_t)i);
}

static inline float dequant_one(const uint32_t *row, const float *srow, const float *brow,
                                int64_t i, int64_t gs) {
    float q = (float)q6o_extract(row, (uint32_t)i);
    float s = srow[i / gs];
    float b = brow[i / gs];
    float p = s * q; /* exact: 8-bit significand times a 6-bit integer */
    return p + b;
}

/* Dense fp32 weights [n, k] from packed codes and fp32 scales/biases [n, k/gs]. */
void q6o_dequant_f32(const uint32_t *packed, const float *scales, const float *biases,
                     int64_t n, int64_t k, int64_t gs, float *out) {
    int64_t words = k * 6 / 32, groups = k / gs;
    for (int64_t r = 0; r < n; ++r)
        for (int64_t i = 0; i < k; ++i)
            out[r * k + i] = dequant_one(packed + r * words, scales + r * groups,
                                         biases + r * groups, i, gs);
}

/* Dense bf16 weights: bf16_rn(fp32(scale) * q + fp32(bias)), the definition the
 * GPU dequantiser must match bit for bit. */
void q6o_dequant_bf16(const uint32_t *packed, const uint16_t *scales, const uint16_t *biases,
                      int64_t n, int64_t k, int64_t gs, uint16_t *out) {
    int64_t words = k * 6 / 32, groups = k / gs;
    for (int64_t r = 0; r < n; ++r) {
        const uint32_t *row = packed + r * words;
        for (int64_t i = 0; i < k; ++i) {
            float s = q6o_bf16_to_f32(scales[r * groups + i / gs]);
            float b = q6o_bf16_to_f32(biases[r * groups + i / gs]);
            float p = s * (float)q6o_extract(row, (uint32_t)i);
            out[r * k + i] = q6o_f32_to_bf16(p + b);
        }
    }
}

float q6o_gelu(float x) {
    float x3 = x * x * x;
    return 0.5f * x * (1.0f + tanhf(Q6_GELU_K * (x + Q6_GELU_C * x3)));
}

/*
 * y[m, n] = act(sum_k x[m, k] * w[n, k] + bias[n]), fp32, k ascending.
 * x is fp32 [m, k] (bf16 activations are widened by the caller); weights are
 * dequantised on the fly like SOURCE_QMM_T (q6_metal_mlp.py:58-83).
 * round_w_bf16 != 0 rounds every dequantised weight to bf16 first, which is
 * the pre-dequantised dense path (dequantize_linear + matmul).
 * scales/biases are fp32 [n, k/gs]; bias may be NULL.
 */
void q6o_qmm_t(const float *x, const uint32_t *packed, const float *scales,
               const float *biases, const float *bias, int apply_gelu, int round_w_bf16,
               int64_t m, int64_t n, int64_t k, int64_t gs, float *y) {
    int64_t words = k * 6 / 32, groups = k / gs;
    for (int64_t mi = 0; mi < m; ++mi) {
        const float *xr = x + mi * k;
        for (int64_t ni = 0; ni < n; ++ni) {
            const uint32_t *row = packed + ni * words;
            const float *srow = scales + ni * groups, *brow = biases + ni * groups;
            float acc = 0.0f;
            for (int64_t i = 0; i < k; ++i) {
                float w = dequant_one(row, srow, brow, i, gs);
                if (round_w_bf16) w = q6o_bf16_to_f32(q6o_f32_to_bf16(w));
                float prod = xr[i] * w;
                acc = acc + prod;
            }
            if (bias) acc = acc + bias[ni];
            if (apply_gelu) acc = q6o_gelu(acc);
            y[mi * n + ni] = acc;
        }
    }
}

/* Elementwise GELU-tanh over an fp32 buffer (mlx nn.gelu_approx formula). */
void q6o_gelu_inplace(float *v, int64_t count) {
    for (int64_t i = 0; i < count; ++i) v[i] = q6o_gelu(v[i]);
}

/* Round an fp32 buffer to bf16 bit patterns. */
void q6o_round_bf16(const float *v, int64_t count, uint16_t *out) {
    for (int64_t i = 0; i < count; ++i) out[i] = q6o_f32_to_bf16(v[i]);
}

void q6o_widen_bf16(const uint16_t *v, int64_t count, float *out) {
    for (int64_t i = 0; i < count; ++i) out[i] = q6o_bf16_to_f32(v[i]);
}
