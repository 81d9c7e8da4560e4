// Exact register-level unpacking of MLX affine 6-bit codes.
//
// Layout (shardedit_mlx/q6_metal_mlp.py:28-40): code j of a row occupies bits
// [6j, 6j+6) of the row's little-endian uint32 stream, so every 16 codes fill
// exactly three words w0, w1, w2 and codes 5 and 10 straddle a word boundary.
//
// Conversion: a code sitting at bit position P of a word is turned into an
// fp32 value by splicing the masked word into the mantissa of 2^(23-P), which
// gives exactly 2^(23-P) + q; subtracting 2^(23-P) again is exact.  One LOP3
// per code plus one add per code and one packed FMA per code pair, then
//   w = fma(q, scale, bias)            (fp32, rounded once; scale*q is exact)
// and, for the tensor-core operand, bf16_rn(w) two at a time.  This is the
// same value as the reference's `scale * float(code) + qbias`
// (q6_metal_mlp.py:42-54) followed by round-to-nearest-even to bf16.
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

namespace q6 {

template <int P>
__device__ __forceinline__ float code_spliced(uint32_t v) {
    static_assert(P >= 0 && P <= 17, "code must sit in the low 23 mantissa bits");
    constexpr uint32_t kMask = 0x3Fu << P;
    constexpr uint32_t kExp = (127u + 23u - P) << 23;
    return __uint_as_float((v & kMask) | kExp);
}

template <int P>
__device__ __forceinline__ constexpr float code_offset() {
    return static_cast<float>(1u << (23 - P));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}

// Dequantise one code pair given as spliced values with their offsets.  The
// exact subtraction is two scalar adds: their constants are immediates, where
// a packed add would need the constant pair in a register pair.
template <int PA, int PB>
__device__ __forceinline__ float2 pair_f32(float a_spliced, float b_spliced, float2 s2, float2 b2) {
    const float2 q = make_float2(__fadd_rn(a_spliced, -code_offset<PA>()),  // exact integer codes
                                 __fadd_rn(b_spliced, -code_offset<PB>()));
    return __ffma2_rn(q, s2, b2);  // s*q + b, one rounding
}

// Sixteen codes (three packed words) -> sixteen fp32 weights.
__device__ __forceinline__ void dequant16_f32(uint32_t w0, uint32_t w1, uint32_t w2, float s, float b,
                                              float (&out)[16]) {
    const uint32_t t0 = w0 >> 12, t1 = w1 >> 12, t2 = w2 >> 12;
    const uint32_t f5 = __funnelshift_r(w0, w1, 30);
    const uint32_t f10 = __funnelshift_r(w1, w2, 28);
    const float2 s2 = make_float2(s, s), b2 = make_float2(b, b);
    float2 r;
    r = pair_f32<0, 6>(code_spliced<0>(w0), code_spliced<6>(w0), s2, b2);
    out[0] = r.x; out[1] = r.y;
    r = pair_f32<12, 6>(code_spliced<12>(w0), code_spliced<6>(t0), s2, b2);
    out[2] = r.x; out[3] = r.y;
    r = pair_f32<12, 0>(code_spliced<12>(t0), code_spliced<0>(f5), s2, b2);
    out[4] = r.x; out[5] = r.y;
    r = pair_f32<4, 10>(code_spliced<4>(w1), code_spliced<10>(w1), s2, b2);
    out[6] = r.x; out[7] = r.y;
    r = pair_f32<16, 10>(code_spliced<16>(w1), code_spliced<10>(t1), s2, b2);
    out[8] = r.x; out[9] = r.y;
    r = pair_f32<0, 2>(code_spliced<0>(f10), code_spliced<2>(w2), s2, b2);
    out[10] = r.x; out[11] = r.y;
    r = pair_f32<8, 14>(code_spliced<8>(w2), code_spliced<14>(w2), s2, b2);
    out[12] = r.x; out[13] = r.y;
    r = pair_f32<8, 14>(code_spliced<8>(t2), code_spliced<14>(t2), s2, b2);
    out[14] = r.x; out[15] = r.y;
}

// Sixteen codes -> their exact integer values as fp32 (q[i] = code i), no
// scale or bias: for dot products that apply the group's affine map once per
// group instead of once per weight.
__device__ __forceinline__ void codes16_f32(uint32_t w0, uint32_t w1, uint32_t w2, float (&q)[16]) {
    const uint32_t t0 = w0 >> 12, t1 = w1 >> 12, t2 = w2 >> 12;
    const uint32_t f5 = __funnelshift_r(w0, w1, 30);
    const uint32_t f10 = __funnelshift_r(w1, w2, 28);
#define Q6_PAIR(i, PA, VA, PB, VB)                                                                       \
    {                                                                                                    \
        q[2 * (i)] = __fadd_rn(code_spliced<PA>(VA), -code_offset<PA>());                                \
        q[2 * (i) + 1] = __fadd_rn(code_spliced<PB>(VB), -code_offset<PB>());                            \
    }
    Q6_PAIR(0, 0, w0, 6, w0);
    Q6_PAIR(1, 12, w0, 6, t0);
    Q6_PAIR(2, 12, t0, 0, f5);
    Q6_PAIR(3, 4, w1, 10, w1);
    Q6_PAIR(4, 16, w1, 10, t1);
    Q6_PAIR(5, 0, f10, 2, w2);
    Q6_PAIR(6, 8, w2, 14, w2);
    Q6_PAIR(7, 8, t2, 14, t2);
#undef Q6_PAIR
}

// ------------------------------------------------------------------------
// Three-position splice.  Shifting the three words first puts every code of a
// 16-code block at bit 0, 6 or 12 of some word, so a splice needs one of only
// three exponent words.  Passed in as runtime values (kernel arguments, which
// the compiler cannot fold into the instruction), each splice is a single
// logic instruction with the mask as its immediate, where two constants force
// two.  SpliceExp3 holds the exponent words of 2^23, 2^17 and 2^11 (codes at
// bits 0, 6, 12), and of 2^12 and 2^6 (codes at bits 11 and 17, the folded
// dequant below).
struct SpliceExp3 {
    uint32_t e0, e6, e12;
    uint32_t e11, e17;
};

inline SpliceExp3 splice_exp3_host() {
    return SpliceExp3{150u << 23, 144u << 23, 138u << 23, 139u << 23, 133u << 23};
}

template <int P>
__device__ __forceinline__ float code_at(uint32_t v, uint32_t e) {
    return __fadd_rn(__uint_as_float((v & (0x3Fu << P)) | e), -code_offset<P>());
}

// Sixteen codes (three packed words) -> their exact integer values as fp32.
__device__ __forceinline__ void codes16_f32_e3(uint32_t w0, uint32_t w1, uint32_t w2, SpliceExp3 x,
                                               float (&q)[16]) {
    const uint32_t a1 = w0 >> 18;                      // codes 3, 4 at 0, 6
    const uint32_t f5 = __funnelshift_r(w0, w1, 30);   // code 5 at 0
    const uint32_t b0 = w1 >> 4;                       // codes 6, 7, 8 at 0, 6, 12
    const uint32_t b1 = w1 >> 22;                      // code 9 at 0
    const uint32_t f10 = __funnelshift_r(w1, w2, 28);  // code 10 at 0
    const uint32_t c0 = w2 >> 2;                       // codes 11, 12, 13 at 0, 6, 12
    const uint32_t c1 = w2 >> 20;                      // codes 14, 15 at 0, 6
    q[0] = code_at<0>(w0, x.e0);
    q[1] = code_at<6>(w0, x.e6);
    q[2] = code_at<12>(w0, x.e12);
    q[3] = code_at<0>(a1, x.e0);
    q[4] = code_at<6>(a1, x.e6);
    q[5] = code_at<0>(f5, x.e0);
    q[6] = code_at<0>(b0, x.e0);
    q[7] = code_at<6>(b0, x.e6);
    q[8] = code_at<12>(b0, x.e12);
    q[9] = code_at<0>(b1, x.e0);
    q[10] = code_at<0>(f10, x.e0);
    q[11] = code_at<0>(c0, x.e0);
    q[12] = code_at<6>(c0, x.e6);
    q[13] = code_at<12>(c0, x.e12);
    q[14] = code_at<0>(c1, x.e0);
    q[15] = code_at<6>(c1, x.e6);
}

// Sixteen codes -> eight bf16x2 words (low half = even code), three-position
// splice: the same values as dequant16_bf16x2.
__device__ __forceinline__ void dequant16_bf16x2_e3(uint32_t w0, uint32_t w1, uint32_t w2, float s, float b,
                                                    SpliceExp3 x, uint32_t* out) {
    float q[16];
    codes16_f32_e3(w0, w1, w2, x, q);
    const float2 s2 = make_float2(s, s), b2 = make_float2(b, b);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float2 r = __ffma2_rn(make_float2(q[2 * i], q[2 * i + 1]), s2, b2);  // s*q + b, one rounding
        out[i] = pack_bf16x2(r.x, r.y);
    }
}

// Sixteen codes -> eight bf16x2 words (low half = even code).
__device__ __forceinline__ void dequant16_bf16x2(uint32_t w0, uint32_t w1, uint32_t w2, float s, float b,
                                                 uint32_t* out) {
    const uint32_t t0 = w0 >> 12, t1 = w1 >> 12, t2 = w2 >> 12;
    const uint32_t f5 = __funnelshift_r(w0, w1, 30);
    const uint32_t f10 = __funnelshift_r(w1, w2, 28);
    const float2 s2 = make_float2(s, s), b2 = make_float2(b, b);
    float2 r;
    r = pair_f32<0, 6>(code_spliced<0>(w0), code_spliced<6>(w0), s2, b2);
    out[0] = pack_bf16x2(r.x, r.y);
    r = pair_f32<12, 6>(code_spliced<12>(w0), code_spliced<6>(t0), s2, b2);
    out[1] = pack_bf16x2(r.x, r.y);
    r = pair_f32<12, 0>(code_spliced<12>(t0), code_spliced<0>(f5), s2, b2);
    out[2] = pack_bf16x2(r.x, r.y);
    r = pair_f32<4, 10>(code_spliced<4>(w1), code_spliced<10>(w1), s2, b2);
    out[3] = pack_bf16x2(r.x, r.y);
    r = pair_f32<16, 10>(code_spliced<16>(w1), code_spliced<10>(t1), s2, b2);
    out[4] = pack_bf16x2(r.x, r.y);
    r = pair_f32<0, 2>(code_spliced<0>(f10), code_spliced<2>(w2), s2, b2);
    out[5] = pack_bf16x2(r.x, r.y);
    r = pair_f32<8, 14>(code_spliced<8>(w2), code_spliced<14>(w2), s2, b2);
    out[6] = pack_bf16x2(r.x, r.y);
    r = pair_f32<8, 14>(code_spliced<8>(t2), code_spliced<14>(t2), s2, b2);
    out[7] = pack_bf16x2(r.x, r.y);
}

// ------------------------------------------------------------------------
// Folded-offset dequant.  A code spliced at bit 11 under exponent 2^12 reads
// 4096 + q, at bit 17 under 2^6 it reads 64 + q (exact).  Folding the offset
// into the bias, w = fma(s, 4096 + q, b - 4096 s) (resp. 64), drops the
// subtract of the exact path: one FFMA2 per code pair.  The result equals
// bf16_rn(s q + b) exactly whenever b - 4096 s and b - 64 s are exact in fp32
// (the FMA then rounds the same real number once), which holds unless |b| is
// below about s / 32 without being zero.  FoldedBias carries the two folded
// biases and whether both are exact; an inexact group must take the exact
// path (dequant16_bf16x2_e3).
struct FoldedBias {
    float2 b;  // (b - 4096 s, b - 64 s): the even code of a pair sits at bit 11, the odd at 17
    bool exact;
};

__device__ __forceinline__ FoldedBias fold_bias(float s, float b) {
    FoldedBias f;
    f.b.x = fmaf(-4096.0f, s, b);
    f.b.y = fmaf(-64.0f, s, b);
    // Adding the offset back recovers b exactly iff the fold rounded nothing:
    // a rounding error is a multiple of b's bf16 unit, far above half its fp32 ulp.
    f.exact = fmaf(4096.0f, s, f.b.x) == b && fmaf(64.0f, s, f.b.y) == b;
    return f;
}

// Eight shifts of a 16-code block (three packed words) that place code pair
// (2i, 2i+1) at bits 11 and 17 of v[i].
__device__ __forceinline__ void pair_words16(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t (&v)[8]) {
    v[0] = w0 << 11;
    v[1] = w0 >> 1;
    v[2] = __funnelshift_r(w0, w1, 13);
    v[3] = w1 << 7;
    v[4] = w1 >> 5;
    v[5] = __funnelshift_r(w1, w2, 17);
    v[6] = w2 << 3;
    v[7] = w2 >> 9;
}

// The pair of v as fp32 (4096 + even code, 64 + odd code): one splice each.
__device__ __forceinline__ float2 pair_at11_17(uint32_t v, SpliceExp3 x) {
    return make_float2(__uint_as_float((v & (0x3Fu << 11)) | x.e11), __uint_as_float((v & (0x3Fu << 17)) | x.e17));
}

// Sixteen codes -> eight bf16x2 words (low half = even code): per pair one
// shift, two splices, one FFMA2 and one pack.
__device__ __forceinline__ void dequant16_bf16x2_fold(uint32_t w0, uint32_t w1, uint32_t w2, float s, float2 fb,
                                                      SpliceExp3 x, uint32_t* out) {
    uint32_t v[8];
    pair_words16(w0, w1, w2, v);
    const float2 s2 = make_float2(s, s);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float2 r = __ffma2_rn(pair_at11_17(v[i], x), s2, fb);
        out[i] = pack_bf16x2(r.x, r.y);
    }
}

}  // namespace q6
