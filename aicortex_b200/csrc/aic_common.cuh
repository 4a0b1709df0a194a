// Device-side primitives of the packed int4 format used on the whole
// inference path, plus launch/error plumbing shared by the kernels.
//
// Format ("F", AICortex kernels.h:56-85): a group is 32 signed 4-bit codes in
// four little-endian u32 words (code i sits in word i>>3 at bits 4*(i&7)) and
// one int8 exponent s. The value of code q is q * max(2^s / 7, 2^-13).
// Activations are NHWC: position p, group g -> words [p*C/8 + 4g .. +3] and
// exponent [p*C/32 + g].
//
// The quantisation rules (absmax -> stored exponent rn(log2 absmax) clamped to
// +-120, codes rn(v * 7 / absmax) clamped to [-8, 7], absmax < 2^-13 treated
// as 1) are the reference's; they are restated here because parity with packed
// weights and activations produced by the reference must be bit-exact.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_fp16.h>

namespace aic {

constexpr float kEps = 1.0f / 8192.0f;   // kernels.h: epsilon (base_constants.h:33)
constexpr float kQMax = 7.0f;            // quant_int4_max
constexpr float kScaleMin = -120.0f;     // quant_scale_min
constexpr float kScaleMax = 120.0f;      // quant_scale_max
constexpr int kNormChunk = 256;          // RMSNorm chunk of the quantized convs and out-proj

// Sign-extended code e (0..7) of a packed word.
__device__ __forceinline__ int code_of(uint32_t w, int e)
{
    int r;
    asm("bfe.s32 %0, %1, %2, 4;" : "=r"(r) : "r"(w), "r"(e << 2));
    return r;
}

// Stored exponent of a group whose (clamped) absmax is `scale`.
__device__ __forceinline__ int8_t exponent_of(float scale)
{
    return static_cast<int8_t>(__float2int_rn(fmaxf(kScaleMin, fminf(kScaleMax, __log2f(scale)))));
}

// Dequantisation factor max(2^s/7, 2^-13).
__device__ __forceinline__ float unit_of(int8_t s)
{
    return fmaxf(exp2f(static_cast<float>(s)) * (1.0f / kQMax), kEps);
}

// Code of value v given inv = 7 / absmax, round to nearest even.
__device__ __forceinline__ uint32_t code_rn(float v, float inv)
{
    return static_cast<uint32_t>(max(-8, min(7, __float2int_rn(v * inv)))) & 0xFu;
}

// Exact sum over 8 code pairs of qa*qb. Each nibble is moved to the top of
// its byte (16*q as a signed byte) so one dp4a covers four pairs; the two
// partial dot products carry a factor 256 that is shifted out exactly.
__device__ __forceinline__ int dot8(uint32_t a, uint32_t b)
{
    const int hi = __dp4a(static_cast<int>(a & 0xF0F0F0F0u), static_cast<int>(b & 0xF0F0F0F0u), 0);
    const int lo = __dp4a(static_cast<int>((a << 4) & 0xF0F0F0F0u), static_cast<int>((b << 4) & 0xF0F0F0F0u), hi);
    return lo >> 8;
}

// Code e (0..7) of a packed word as a float, without a conversion
// instruction: (n ^ 8) placed in the mantissa of 2^23 gives 2^23 + q + 8.
__device__ __forceinline__ float code_f(uint32_t w, int e)
{
    return __uint_as_float(((w >> (e << 2)) & 0xFu) ^ 0x4B000008u) - 8388616.0f;
}

// Reciprocal of d >= 2^-13 rounded to nearest, results below 2^-126 flushed
// to zero (the rcp.rn.ftz semantics of __frcp_rn under fast math): one
// Newton-Raphson step from the hardware approximation, with the residual
// 1 - d*y formed exactly by an FMA (Markstein's correction). Infinity is
// clamped to the largest float first, whose reciprocal flushes to zero.
// aic_selftest_rcp compares it with __frcp_rn over every significand of
// thirteen binades from 2^-13 to 2^126 and at the clamp: no input differs.
// Its callers are the sigmoid (d = 1 + e >= 1) and the quantisers (d = the
// group's absmax clamped to >= 2^-13).
__device__ __forceinline__ float rcp_rn_pos(float d)
{
    d = fminf(d, 3.40282347e38f);
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(d));
    const float r = fmaf(-d, y, 1.0f);
    return fmaf(r, y, y);
}

// sigmoid(x) = __frcp_rn(1 + __expf(-x)) and silu(x) = x * sigmoid(x), as the
// reference defines them (kernels.h:86-87); 1 + e >= 1, so rcp_rn_pos gives
// the same bits as __frcp_rn.
__device__ __forceinline__ float sigmoid_f(float x) { return rcp_rn_pos(1.0f + __expf(-x)); }
__device__ __forceinline__ float silu_f(float x) { return x * sigmoid_f(x); }

// ---- packed fp32 pairs (the sm_100 two-lane FFMA/FADD/FMUL) -----------------
// Each component of a pair operation is rounded exactly as the scalar
// __fmaf_rn / __fadd_rn / __fmul_rn, so two independent per-channel chains
// run as one instruction stream and keep the scalar bits. One rule: a pair
// multiply must never feed a pair add. The CUDA 12.9 assembler fuses that
// pattern into one FFMA2 (one rounding instead of two) even when both are
// written in PTX with an explicit .rn, which a tie in a requant exposes; the
// scalar __fmul_rn / __fadd_rn are never fused. So a product that is then
// added goes through the scalar intrinsics, and pairs are used for fma chains,
// multiplies of sums and adds of fma results only.
__device__ __forceinline__ float2 dup2(float a) { return make_float2(a, a); }

__device__ __forceinline__ float2 add2(float2 a, float2 b)
{
    float2 d;
    asm("{\n\t.reg .b64 pa, pb, pd;\n\t"
        "mov.b64 pa, {%2, %3};\n\tmov.b64 pb, {%4, %5};\n\t"
        "add.rn.ftz.f32x2 pd, pa, pb;\n\t"
        "mov.b64 {%0, %1}, pd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}

__device__ __forceinline__ float2 mul2(float2 a, float2 b)
{
    float2 d;
    asm("{\n\t.reg .b64 pa, pb, pd;\n\t"
        "mov.b64 pa, {%2, %3};\n\tmov.b64 pb, {%4, %5};\n\t"
        "mul.rn.ftz.f32x2 pd, pa, pb;\n\t"
        "mov.b64 {%0, %1}, pd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}

// fmaf of both components (one rounding each).
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }

// silu_f of both components (the same operations, the arithmetic paired).
__device__ __forceinline__ float2 silu2(float2 x)
{
    const float2 d = add2(dup2(1.0f), make_float2(__expf(-x.x), __expf(-x.y)));
    const float2 dc = make_float2(fminf(d.x, 3.40282347e38f), fminf(d.y, 3.40282347e38f));
    float2 y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y.x) : "f"(dc.x));
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y.y) : "f"(dc.y));
    const float2 r = fma2(make_float2(-dc.x, -dc.y), y, dup2(1.0f));
    return mul2(x, fma2(r, y, y));
}

// ---- group requantisation ------------------------------------------------------
// The reference (kernels.h:68-70) takes absmax with fmaxf (a NaN is skipped),
// scale = absmax < 2^-13 ? 1 : absmax, inv = 7 * __frcp_rn(scale), and codes
// max(-8, min(7, __float2int_rn(v * inv))), where the conversion gives 0 for a
// NaN and saturates infinities. For a group without NaN or infinity,
// |v * inv| <= 7 (1 + 3 * 2^-24) < 7.5, so the clamp never acts and the code is
// rn(v * inv) itself: adding 1.5 * 2^23 rounds it to an integer and leaves the
// bits 0x4B400000 + q, which pack8_magic turns into nibbles without masking.
// A group holding a NaN or an infinity (max.NaN makes its absmax NaN or inf)
// takes the reference's own sequence instead.

// Running absmax with NaN propagation: max.NaN(acc, |v|).
__device__ __forceinline__ float amax_nan(float acc, float v)
{
    float r;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(acc), "f"(fabsf(v)));
    return r;
}
__device__ __forceinline__ float max_nan(float a, float b)
{
    float r;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}
// max.NaN over |v_i| of N values as a pairwise tree (depth log2 N instead of
// N): max.NaN is exact, commutative and associative (NaN if any operand is
// NaN, else the largest magnitude), so the order does not change the result.
template <int N>
__device__ __forceinline__ float amax_tree(const float (&v)[N])
{
    static_assert(N >= 2 && (N & (N - 1)) == 0, "power of two");
    float m[N / 2];
#pragma unroll
    for (int i = 0; i < N / 2; ++i) m[i] = max_nan(fabsf(v[i]), fabsf(v[i + N / 2]));
#pragma unroll
    for (int o = N / 4; o > 0; o >>= 1)
#pragma unroll
        for (int i = 0; i < o; ++i) m[i] = max_nan(m[i], m[i + o]);
    return m[0];
}
__device__ __forceinline__ float amax_tree2(const float2 (&v)[16])
{
    float m[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) m[i] = max_nan(fabsf(v[i].x), fabsf(v[i].y));
#pragma unroll
    for (int o = 8; o > 0; o >>= 1)
#pragma unroll
        for (int i = 0; i < o; ++i) m[i] = max_nan(m[i], m[i + o]);
    return m[0];
}
// false for a NaN or an infinity
__device__ __forceinline__ bool is_finite_amax(float a) { return a <= 3.40282347e38f; }

// Bits of rn(y) + 1.5 * 2^23, i.e. 0x4B400000 + rn(y) for |y| < 2^22.
__device__ __forceinline__ uint32_t magic_bits(float y) { return __float_as_uint(__fadd_rn(y, 12582912.0f)); }

// Word of 8 codes from z_i = 0x4B400000 + q_i (q_i in [-8, 7], code i at bits
// 4i): sum (z_i - 0x4B3FFFF8) 16^i = sum (q_i + 8) 16^i has no carries, and
// q_i + 8 is the two's-complement nibble of q_i with its top bit flipped.
__device__ __forceinline__ uint32_t pack8_magic(const uint32_t (&z)[8])
{
    uint32_t h = z[7];
#pragma unroll
    for (int i = 6; i >= 0; --i) h = (h << 4) + z[i];
    return (h - 0x4B3FFFF8u * 0x11111111u) ^ 0x88888888u;
}

// fmaxf-reduction start that reproduces a butterfly over the values'
// magnitudes, v = fmaxf(v, shfl_xor(v, o)) from |v| on every lane (the conv
// and depthwise epilogues, kernels.h:271, 861): a NaN drops out of fmaxf, so
// the result is NaN only when every value is NaN.
__device__ __forceinline__ float butterfly_start() { return __int_as_float(0x7FFFFFFF); }

// The packed group a quantiser returns: 4 code words and the exponent.
struct QuantGroup {
    uint4 words;
    int exp;
};

// The reference's epilogue sequence for 32 values held by one thread. Not
// inlined (it is the rare path) and returning by value, so that only its
// caller's copy of the values, made on that path, lives in local memory.
static __device__ __noinline__ QuantGroup quantize_group_ref(const float* v)
{
    float amax = butterfly_start();
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
    const float scale = amax < kEps ? 1.0f : amax;
    const float inv = kQMax * rcp_rn_pos(scale);
    uint32_t w[4] = {0u, 0u, 0u, 0u};
    for (int i = 0; i < 32; ++i) w[i >> 3] |= code_rn(v[i], inv) << ((i & 7) << 2);
    return QuantGroup{make_uint4(w[0], w[1], w[2], w[3]), exponent_of(scale)};
}

// Quantise 32 values held by one thread into 4 words + exponent.
__device__ __forceinline__ void quantize_group(const float (&v)[32], uint4* words, int8_t* exp_out)
{
    const float amax = amax_tree(v);
    if (!is_finite_amax(amax)) {
        float f[32];  // a copy, so that only the rare path takes an array's address
#pragma unroll
        for (int i = 0; i < 32; ++i) f[i] = v[i];
        const QuantGroup r = quantize_group_ref(f);
        *words = r.words;
        *exp_out = static_cast<int8_t>(r.exp);
        return;
    }
    const float scale = amax < kEps ? 1.0f : amax;
    const float inv = kQMax * rcp_rn_pos(scale);
    uint32_t w[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        uint32_t z[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) z[i] = magic_bits(__fmul_rn(v[8 * q + i], inv));
        w[q] = pack8_magic(z);
    }
    *words = make_uint4(w[0], w[1], w[2], w[3]);
    *exp_out = exponent_of(scale);
}

// quantize_group over 32 values held as 16 pairs (value 2i + j in v[i].j).
__device__ __forceinline__ void quantize_group2(const float2 (&v)[16], uint4* words, int8_t* exp_out)
{
    const float amax = amax_tree2(v);
    if (!is_finite_amax(amax)) {
        float f[32];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            f[2 * i] = v[i].x;
            f[2 * i + 1] = v[i].y;
        }
        const QuantGroup r = quantize_group_ref(f);
        *words = r.words;
        *exp_out = static_cast<int8_t>(r.exp);
        return;
    }
    const float scale = amax < kEps ? 1.0f : amax;
    const float inv = kQMax * rcp_rn_pos(scale);
    uint32_t w[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        uint32_t z[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {  // scalar: the product must be rounded before the add
            z[2 * i] = magic_bits(__fmul_rn(v[4 * q + i].x, inv));
            z[2 * i + 1] = magic_bits(__fmul_rn(v[4 * q + i].y, inv));
        }
        w[q] = pack8_magic(z);
    }
    *words = make_uint4(w[0], w[1], w[2], w[3]);
    *exp_out = exponent_of(scale);
}

// Quantise 32 values held as 8 per lane across 4 consecutive lanes (lane & 3
// selects the word). Returns this lane's packed word; *exp_out gets the
// exponent on every lane. Every lane of the warp must call it (the NaN test
// is a warp vote, so the slow path's shuffles run on the whole warp).
__device__ __forceinline__ uint32_t quantize_word_x4(const float (&v)[8], int8_t* exp_out)
{
    float amax = amax_tree(v);
    amax = max_nan(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 1));
    amax = max_nan(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 2));
    uint32_t w = 0;
    if (__any_sync(0xFFFFFFFFu, !is_finite_amax(amax))) {
        float a = butterfly_start();
#pragma unroll
        for (int i = 0; i < 8; ++i) a = fmaxf(a, fabsf(v[i]));
        a = fmaxf(a, __shfl_xor_sync(0xFFFFFFFFu, a, 1));
        a = fmaxf(a, __shfl_xor_sync(0xFFFFFFFFu, a, 2));
        const float scale = a < kEps ? 1.0f : a;
        const float inv = kQMax * rcp_rn_pos(scale);
#pragma unroll
        for (int i = 0; i < 8; ++i) w |= code_rn(v[i], inv) << (i << 2);
        *exp_out = exponent_of(scale);
        return w;
    }
    const float scale = amax < kEps ? 1.0f : amax;
    const float inv = kQMax * rcp_rn_pos(scale);
    uint32_t z[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) z[i] = magic_bits(__fmul_rn(v[i], inv));
    *exp_out = exponent_of(scale);
    return pack8_magic(z);
}

}  // namespace aic
