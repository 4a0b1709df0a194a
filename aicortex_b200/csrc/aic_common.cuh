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

// The same code as code_rn for finite v without a float->int conversion: the
// clamped value plus 1.5 * 2^23 is rounded to nearest even by the add, and the
// low four mantissa bits are then the two's-complement code.
// (rn(clamp(x)) == clamp(rn(x)) because rounding is monotonic.)
__device__ __forceinline__ uint32_t code_rn_fast(float v, float inv)
{
    const float y = fminf(fmaxf(v * inv, -8.0f), 7.0f);
    return __float_as_uint(y + 12582912.0f) & 0xFu;
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

// Reciprocal of d >= 1 rounded to nearest, results below 2^-126 flushed to
// zero (the rcp.rn.ftz semantics of __frcp_rn under fast math): one
// Newton-Raphson step from the hardware approximation, with the residual
// 1 - d*y formed exactly by an FMA (Markstein's correction). Infinity is
// clamped to the largest float first, whose reciprocal flushes to zero.
// aic_selftest_rcp compares it with __frcp_rn over every significand of ten
// binades from 1 to 2^126 and at the clamp: no input differs.
__device__ __forceinline__ float rcp_rn_ge1(float d)
{
    d = fminf(d, 3.40282347e38f);
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(d));
    const float r = fmaf(-d, y, 1.0f);
    return fmaf(r, y, y);
}

// sigmoid(x) = __frcp_rn(1 + __expf(-x)) and silu(x) = x * sigmoid(x), as the
// reference defines them (kernels.h:86-87); 1 + e >= 1, so rcp_rn_ge1 gives
// the same bits as __frcp_rn.
__device__ __forceinline__ float sigmoid_f(float x) { return rcp_rn_ge1(1.0f + __expf(-x)); }
__device__ __forceinline__ float silu_f(float x) { return x * sigmoid_f(x); }

// ---- packed fp32 pairs (the sm_100 two-lane FFMA/FADD/FMUL) -----------------
// Each component of __ffma2_rn / __fadd2_rn / __fmul2_rn is rounded exactly as
// the scalar __fmaf_rn / __fadd_rn / __fmul_rn, so two independent
// per-channel chains run as one instruction stream and keep the scalar bits.
__device__ __forceinline__ float2 dup2(float a) { return make_float2(a, a); }

// silu_f of both components (the same operations, the arithmetic paired).
__device__ __forceinline__ float2 silu2(float2 x)
{
    const float2 d = __fadd2_rn(dup2(1.0f), make_float2(__expf(-x.x), __expf(-x.y)));
    const float2 dc = make_float2(fminf(d.x, 3.40282347e38f), fminf(d.y, 3.40282347e38f));
    float2 y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y.x) : "f"(dc.x));
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y.y) : "f"(dc.y));
    const float2 r = __ffma2_rn(make_float2(-dc.x, -dc.y), y, dup2(1.0f));
    return __fmul2_rn(x, __ffma2_rn(r, y, y));
}


// Quantise 32 values held as 8 per lane across 4 consecutive lanes (lane & 3
// selects the word). Returns this lane's packed word; *exp_out gets the
// exponent on every lane.
__device__ __forceinline__ uint32_t quantize_word_x4(const float (&v)[8], int8_t* exp_out)
{
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
    amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 2));
    const float scale = amax < kEps ? 1.0f : amax;
    const float inv = kQMax * __frcp_rn(scale);
    uint32_t w = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) w |= code_rn_fast(v[i], inv) << (i << 2);
    *exp_out = exponent_of(scale);
    return w;
}

// Quantise 32 values held by one thread into 4 words + exponent.
__device__ __forceinline__ void quantize_group(const float (&v)[32], uint4* words, int8_t* exp_out)
{
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
    const float scale = amax < kEps ? 1.0f : amax;
    const float inv = kQMax * __frcp_rn(scale);
    uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
    for (int i = 0; i < 32; ++i) w[i >> 3] |= code_rn_fast(v[i], inv) << ((i & 7) << 2);
    *words = make_uint4(w[0], w[1], w[2], w[3]);
    *exp_out = exponent_of(scale);
}

// quantize_group over 32 values held as 16 pairs (value 2i + j in v[i].j).
__device__ __forceinline__ void quantize_group2(const float2 (&v)[16], uint4* words, int8_t* exp_out)
{
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fmaxf(fabsf(v[i].x), fabsf(v[i].y)));
    const float scale = amax < kEps ? 1.0f : amax;
    const float2 inv = dup2(kQMax * __frcp_rn(scale));
    uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        float2 y = __fmul2_rn(v[i], inv);
        y = make_float2(fminf(fmaxf(y.x, -8.0f), 7.0f), fminf(fmaxf(y.y, -8.0f), 7.0f));
        y = __fadd2_rn(y, dup2(12582912.0f));  // code_rn_fast of both
        const uint32_t two = (__float_as_uint(y.x) & 0xFu) | ((__float_as_uint(y.y) & 0xFu) << 4);
        w[i >> 2] |= two << ((i & 3) << 3);
    }
    *words = make_uint4(w[0], w[1], w[2], w[3]);
    *exp_out = exponent_of(scale);
}

}  // namespace aic
