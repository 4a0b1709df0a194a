// Format kernels of the inference path: weight/activation packing (A1), the
// fp16 stem packer (A2), the per-position residual add (A6), global average
// pooling (A8) and Bernoulli action sampling (A12). All are HBM-bound integer
// and byte work, written as coalesced SIMT kernels.
#include "aic_common.cuh"
#include "aic_kernels.h"

namespace aic {
namespace {

constexpr int kThreads = 256;

// Position hash of the reference packer (kernels.h:21-37, device branch): the
// base is the global thread index, which for the packer is the group index.
__device__ __forceinline__ uint32_t position_seed(uint32_t tid, int32_t sample)
{
    uint32_t s = tid + static_cast<uint32_t>(sample) * 2654435761u;
    s = (s ^ 61u) ^ (s >> 16);
    s *= 9u;
    s ^= s >> 4;
    s *= 668265261u;
    s ^= s >> 15;
    return s == 0u ? 123456789u : s;
}

// xorshift32 mapped to a float with the reference's factor. The reference
// writes `(1.0f / 0xFFFFFFFFf)`, where 0xFFFFFFFFf is the integer 2^36-1, so
// the factor is exactly 2^-36 and the result lies in [0, n/16).
__device__ __forceinline__ float hashed_uniform(uint32_t seed, float n)
{
    seed ^= seed << 13;
    seed ^= seed >> 17;
    seed ^= seed << 5;
    return __uint2float_rn(seed) * (1.0f / 68719476736.0f) * n;
}

template <bool kStochastic>
__global__ void __launch_bounds__(kThreads) pack_f32_kernel(const float* __restrict__ in, uint32_t* __restrict__ out,
                                                          int8_t* __restrict__ out_s, int64_t groups, int32_t add_idx,
                                                          int64_t row_groups)
{
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
    if (idx >= groups) return;
    float v[32];
    const float4* src = reinterpret_cast<const float4*>(in + (idx << 5));
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float4 f = src[i];
        v[4 * i] = f.x; v[4 * i + 1] = f.y; v[4 * i + 2] = f.z; v[4 * i + 3] = f.w;
    }
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
    const float scale = amax < kEps ? 1.0f : amax;
    out_s[idx] = exponent_of(scale);
    const float inv = kQMax * rcp_rn_pos(scale);
    uint32_t w[4] = {0u, 0u, 0u, 0u};
    if (kStochastic) {
        const int64_t rel = row_groups > 0 ? idx % row_groups : idx;
        const uint32_t tid = static_cast<uint32_t>(rel);
        const uint32_t group_seed = position_seed(tid, static_cast<int32_t>(rel + add_idx));
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            const float scaled = fmaxf(-8.0f, fminf(kQMax, v[i] * inv));
            const int lo = __float2int_rd(scaled);
            const float u = hashed_uniform(position_seed(tid, static_cast<int32_t>(group_seed ^ static_cast<uint32_t>(i))), 1.0f);
            const int q = lo + (u < scaled - __int2float_rd(lo));
            w[i >> 3] |= (static_cast<uint32_t>(q) & 0xFu) << ((i & 7) << 2);
        }
    } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) w[i >> 3] |= code_rn(v[i], inv) << ((i & 7) << 2);
    }
    reinterpret_cast<uint4*>(out)[idx] = make_uint4(w[0], w[1], w[2], w[3]);
}

// One thread per pixel: reads the present fp16 planes (coalesced along the
// row), zero-fills the rest of the 32-channel group(s), quantises, writes one
// 16-byte group per 32 channels.
__global__ void __launch_bounds__(kThreads) stem_pack_kernel(const __half* __restrict__ planes, int64_t pixels, int hw,
                                                           int planes_present, int channels, uint32_t* __restrict__ out,
                                                           int8_t* __restrict__ out_s)
{
    const int64_t pix = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
    if (pix >= pixels) return;
    const int64_t frame = pix / hw;
    const int64_t sp = pix - frame * hw;
    const int groups = channels >> 5;
    const __half* src = planes + frame * planes_present * hw + sp;
    for (int g = 0; g < groups; ++g) {
        // channels >= planes_present are zero: code 0, and they do not move the absmax
        const int present = min(32, max(0, planes_present - (g << 5)));
        // the reference's butterfly over 32 lanes, padding lanes holding 0
        float amax = present < 32 ? 0.0f : butterfly_start();
        for (int l = 0; l < present; ++l) amax = fmaxf(amax, fabsf(__half2float(src[static_cast<int64_t>((g << 5) + l) * hw])));
        const float scale = amax < kEps ? 1.0f : amax;
        const float inv = kQMax * rcp_rn_pos(scale);
        uint32_t w[4] = {0u, 0u, 0u, 0u};
        for (int l = 0; l < present; ++l)
            w[l >> 3] |= code_rn(__half2float(src[static_cast<int64_t>((g << 5) + l) * hw]), inv) << ((l & 7) << 2);
        reinterpret_cast<uint4*>(out)[pix * groups + g] = make_uint4(w[0], w[1], w[2], w[3]);
        out_s[pix * groups + g] = exponent_of(scale);
    }
}

// The same with four consecutive pixels of a frame per thread (hw % 4 == 0):
// one 8-byte load per present plane, the pixels' groups stored back to back,
// and their exponents as one packed store when a pixel has a single group.
__global__ void __launch_bounds__(kThreads) stem_pack4_kernel(const __half* __restrict__ planes, int64_t quads, int hw,
                                                            int planes_present, int channels, uint32_t* __restrict__ out,
                                                            int8_t* __restrict__ out_s)
{
    const int64_t qd = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
    if (qd >= quads) return;
    const int64_t pix = qd * 4;
    const int64_t frame = pix / hw;
    const int64_t sp = pix - frame * hw;
    const int groups = channels >> 5;
    const __half* src = planes + frame * planes_present * hw + sp;
    uint4* ov = reinterpret_cast<uint4*>(out) + pix * groups;
    uint32_t packed_s = 0;
    for (int g = 0; g < groups; ++g) {
        const int present = min(32, max(0, planes_present - (g << 5)));
        const float a0 = present < 32 ? 0.0f : butterfly_start();  // as stem_pack_kernel
        float amax[4] = {a0, a0, a0, a0};
        for (int l = 0; l < present; ++l) {
            const uint2 v = __ldg(reinterpret_cast<const uint2*>(src + static_cast<int64_t>((g << 5) + l) * hw));
            const __half2 h01 = *reinterpret_cast<const __half2*>(&v.x), h23 = *reinterpret_cast<const __half2*>(&v.y);
            amax[0] = fmaxf(amax[0], fabsf(__low2float(h01)));
            amax[1] = fmaxf(amax[1], fabsf(__high2float(h01)));
            amax[2] = fmaxf(amax[2], fabsf(__low2float(h23)));
            amax[3] = fmaxf(amax[3], fabsf(__high2float(h23)));
        }
        float inv[4];
        int8_t ex[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float scale = amax[k] < kEps ? 1.0f : amax[k];
            inv[k] = kQMax * rcp_rn_pos(scale);
            ex[k] = exponent_of(scale);
        }
        uint32_t w[4][4] = {};
        for (int l = 0; l < present; ++l) {
            const uint2 v = __ldg(reinterpret_cast<const uint2*>(src + static_cast<int64_t>((g << 5) + l) * hw));
            const __half2 h01 = *reinterpret_cast<const __half2*>(&v.x), h23 = *reinterpret_cast<const __half2*>(&v.y);
            const float x[4] = {__low2float(h01), __high2float(h01), __low2float(h23), __high2float(h23)};
#pragma unroll
            for (int k = 0; k < 4; ++k) w[k][l >> 3] |= code_rn(x[k], inv[k]) << ((l & 7) << 2);
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) ov[k * groups + g] = make_uint4(w[k][0], w[k][1], w[k][2], w[k][3]);
        if (groups == 1) {
            packed_s = static_cast<uint32_t>(static_cast<uint8_t>(ex[0])) | (static_cast<uint32_t>(static_cast<uint8_t>(ex[1])) << 8) |
                       (static_cast<uint32_t>(static_cast<uint8_t>(ex[2])) << 16) |
                       (static_cast<uint32_t>(static_cast<uint8_t>(ex[3])) << 24);
        } else {
#pragma unroll
            for (int k = 0; k < 4; ++k) out_s[(pix + k) * groups + g] = ex[k];
        }
    }
    if (groups == 1) *reinterpret_cast<uint32_t*>(out_s + pix) = packed_s;
}

// stem_pack4_kernel for one 32-channel group and NP <= 8 present planes known
// at compile time: each plane's four pixels are loaded once, before any
// arithmetic, and kept in registers for both the absmax and the codes.
template <int NP>
__global__ void __launch_bounds__(kThreads) stem_pack4_np_kernel(const __half* __restrict__ planes, int64_t quads, int hw,
                                                               int lg_hw, uint32_t* __restrict__ out, int8_t* __restrict__ out_s)
{
    const int64_t qd = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
    if (qd >= quads) return;
    const int64_t pix = qd * 4;
    // frame of the pixel: a shift when the frame size is a power of two (lg_hw >= 0)
    const int64_t frame = lg_hw >= 0 ? pix >> lg_hw : pix / hw;
    const int64_t sp = pix - frame * hw;
    const __half* src = planes + frame * NP * hw + sp;
    float x[NP][4];
#pragma unroll
    for (int c = 0; c < NP; ++c) {
        const uint2 v = __ldg(reinterpret_cast<const uint2*>(src + static_cast<int64_t>(c) * hw));
        const __half2 h01 = *reinterpret_cast<const __half2*>(&v.x), h23 = *reinterpret_cast<const __half2*>(&v.y);
        x[c][0] = __low2float(h01);
        x[c][1] = __high2float(h01);
        x[c][2] = __low2float(h23);
        x[c][3] = __high2float(h23);
    }
    uint4* ov = reinterpret_cast<uint4*>(out) + pix;
    uint32_t packed_s = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        float amax = 0.0f;  // fewer than 32 planes: the padding channels are zeros (as stem_pack_kernel)
#pragma unroll
        for (int c = 0; c < NP; ++c) amax = fmaxf(amax, fabsf(x[c][k]));
        const float scale = amax < kEps ? 1.0f : amax;
        const float inv = kQMax * rcp_rn_pos(scale);
        uint32_t w = 0;
#pragma unroll
        for (int c = 0; c < NP; ++c) w |= code_rn(x[c][k], inv) << (4 * c);
        ov[k] = make_uint4(w, 0u, 0u, 0u);
        packed_s |= static_cast<uint32_t>(static_cast<uint8_t>(exponent_of(scale))) << (8 * k);
    }
    *reinterpret_cast<uint32_t*>(out_s + pix) = packed_s;
}

// Residual add when a position has exactly S = C/32 groups (S a power of two):
// lane gl of a segment of S lanes owns group gl of two positions 32/S apart,
// and all four of its loads are issued before any arithmetic (twice the bytes
// in flight of one position per lane). Per element, as residualAddFwdKernel
// (kernels.h:1020-1026): r = fmaf(q_m, unit(s_m) * mult, q_r * unit(s_r)), two
// channels per packed instruction (the products feed an fma's addend, which is
// never fused). One exponent per position: the absmax (from 0, kernels.h:1008)
// over its S groups, reduced across the segment's lanes; requant as
// quantize_group (the reference's sequence for a group holding a NaN or inf).
template <int S>
__global__ void __launch_bounds__(kThreads) residual_pos2_kernel(const uint32_t* __restrict__ main_in, const int8_t* __restrict__ main_s,
                                                               const uint32_t* __restrict__ res, const int8_t* __restrict__ res_s,
                                                               uint32_t* __restrict__ out, int8_t* __restrict__ out_s,
                                                               int64_t positions, float main_mult, bool skipped)
{
    constexpr int kPos = 32 / S;  // positions per warp row
    const int lane = threadIdx.x & 31;
    const int64_t warp = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) >> 5;
    const int gl = lane % S;
    const int64_t p0 = warp * 2 * kPos + lane / S;
    uint4 a[2], b[2];
    int8_t sa[2], sb[2];
    bool live[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const int64_t pos = p0 + k * kPos;
        live[k] = pos < positions;
        const int64_t gi = (live[k] ? pos : 0) * S + gl;
        a[k] = skipped ? make_uint4(0u, 0u, 0u, 0u) : __ldg(reinterpret_cast<const uint4*>(main_in) + gi);
        b[k] = __ldg(reinterpret_cast<const uint4*>(res) + gi);
        sa[k] = skipped ? static_cast<int8_t>(0) : __ldg(main_s + gi);
        sb[k] = __ldg(res_s + gi);
    }
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const float2 s_res = dup2(unit_of(sb[k]));
        const float2 s_in = dup2(skipped ? 0.0f : unit_of(sa[k]) * main_mult);
        const uint32_t aw[4] = {a[k].x, a[k].y, a[k].z, a[k].w}, bw[4] = {b[k].x, b[k].y, b[k].z, b[k].w};
        float2 r[16];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            // byte j of lo / hi: code 2j / 2j + 1 of the word as n ^ 8, placed in
            // the mantissa of 2^23 (0x4B0000bb = 2^23 + q + 8)
            const uint32_t alo = (aw[q] & 0x0F0F0F0Fu) ^ 0x08080808u, ahi = ((aw[q] >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u;
            const uint32_t blo = (bw[q] & 0x0F0F0F0Fu) ^ 0x08080808u, bhi = ((bw[q] >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float2 qa = add2(make_float2(__uint_as_float(__byte_perm(alo, 0x4B000000u, 0x7440u | j)),
                                                   __uint_as_float(__byte_perm(ahi, 0x4B000000u, 0x7440u | j))),
                                       dup2(-8388616.0f));
                const float2 qb = add2(make_float2(__uint_as_float(__byte_perm(blo, 0x4B000000u, 0x7440u | j)),
                                                   __uint_as_float(__byte_perm(bhi, 0x4B000000u, 0x7440u | j))),
                                       dup2(-8388616.0f));
                r[4 * q + j] = fma2(qa, s_in, mul2(qb, s_res));
            }
        }
        // absmax that keeps a NaN (equal to the reference's when finite), as a tree
        float amaxn = amax_tree2(r);
#pragma unroll
        for (int o = S >> 1; o > 0; o >>= 1) amaxn = max_nan(amaxn, __shfl_xor_sync(0xFFFFFFFFu, amaxn, o));
        // the reference's absmax (fmaxf from 0, a NaN skipped) differs only where
        // a NaN or an infinity is present: recomputed then, warp-wide
        float amax = amaxn;
        if (__any_sync(0xFFFFFFFFu, !is_finite_amax(amaxn))) {
            amax = 0.0f;
#pragma unroll
            for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fmaxf(fabsf(r[i].x), fabsf(r[i].y)));
#pragma unroll
            for (int o = S >> 1; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
        }
        if (!live[k]) continue;
        const float scale = amax < kEps ? 1.0f : amax;
        const float inv = kQMax * rcp_rn_pos(scale);
        uint32_t w[4];
        if (is_finite_amax(amaxn)) {  // rn without the clamp (aic_common.cuh)
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                uint32_t z[8];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    z[2 * i] = magic_bits(__fmul_rn(r[4 * q + i].x, inv));
                    z[2 * i + 1] = magic_bits(__fmul_rn(r[4 * q + i].y, inv));
                }
                w[q] = pack8_magic(z);
            }
        } else {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                w[q] = 0u;
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    w[q] |= (code_rn(r[4 * q + i].x, inv) << (8 * i)) | (code_rn(r[4 * q + i].y, inv) << (8 * i + 4));
            }
        }
        const int64_t gi = (p0 + k * kPos) * S + gl;
        reinterpret_cast<uint4*>(out)[gi] = make_uint4(w[0], w[1], w[2], w[3]);
        out_s[gi] = exponent_of(scale);
    }
}

// Residual add with one exponent per position. A position is handled by a
// segment of S lanes (S = next power of two >= C/32, at most 32); each lane
// walks groups gl, gl+S, ... The values are recomputed in the second pass
// instead of being kept, which is bit-identical and needs no shared memory.
template <int S>
__global__ void __launch_bounds__(kThreads) residual_kernel(const uint32_t* __restrict__ main_in, const int8_t* __restrict__ main_s,
                                                          const uint32_t* __restrict__ res, const int8_t* __restrict__ res_s,
                                                          uint32_t* __restrict__ out, int8_t* __restrict__ out_s,
                                                          int64_t positions, int C, float main_mult, bool skipped)
{
    const int lane = threadIdx.x & 31;
    const int64_t warp = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) >> 5;
    const int64_t pos = warp * (32 / S) + lane / S;
    const int gl = lane % S;
    const bool live = pos < positions;
    const int G = C >> 5;
    const int64_t pbase = live ? pos : 0;
    const uint4* mv = reinterpret_cast<const uint4*>(main_in) + pbase * G;
    const uint4* rv = reinterpret_cast<const uint4*>(res) + pbase * G;
    if (G == S) {
        // One group per lane: keep the 32 values in registers (single pass).
        float r[32];
        float amax1 = 0.0f, amaxn = 0.0f;  // the reference's absmax, and one that keeps a NaN
        if (live) {
            const float s_res = unit_of(res_s[pbase * G + gl]);
            const float s_in = skipped ? 0.0f : unit_of(main_s[pbase * G + gl]) * main_mult;
            const uint4 a = skipped ? make_uint4(0u, 0u, 0u, 0u) : mv[gl];
            const uint4 b = rv[gl];
            const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                r[i] = fmaf(code_f(aw[i >> 3], i & 7), s_in, code_f(bw[i >> 3], i & 7) * s_res);
                amax1 = fmaxf(amax1, fabsf(r[i]));
                amaxn = amax_nan(amaxn, r[i]);
            }
        }
#pragma unroll
        for (int o = S >> 1; o > 0; o >>= 1) {
            amax1 = fmaxf(amax1, __shfl_xor_sync(0xFFFFFFFFu, amax1, o));
            amaxn = max_nan(amaxn, __shfl_xor_sync(0xFFFFFFFFu, amaxn, o));
        }
        if (!live) return;
        const float scale1 = amax1 < kEps ? 1.0f : amax1;
        const float inv1 = kQMax * rcp_rn_pos(scale1);
        uint32_t w[4] = {0u, 0u, 0u, 0u};
        if (is_finite_amax(amaxn)) {  // no NaN or infinity in the group: rn without the clamp (aic_common.cuh)
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                uint32_t z[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) z[i] = magic_bits(__fmul_rn(r[8 * q + i], inv1));
                w[q] = pack8_magic(z);
            }
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) w[i >> 3] |= code_rn(r[i], inv1) << ((i & 7) << 2);
        }
        reinterpret_cast<uint4*>(out)[pos * G + gl] = make_uint4(w[0], w[1], w[2], w[3]);
        out_s[pos * G + gl] = exponent_of(scale1);
        return;
    }
    float amax = 0.0f;
    for (int g = gl; live && g < G; g += S) {
        const float s_res = unit_of(res_s[pbase * G + g]);
        const float s_in = skipped ? 0.0f : unit_of(main_s[pbase * G + g]) * main_mult;
        const uint4 a = skipped ? make_uint4(0u, 0u, 0u, 0u) : mv[g];
        const uint4 b = rv[g];
        const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const float r = fmaf(static_cast<float>(code_of(aw[i], e)), s_in, static_cast<float>(code_of(bw[i], e)) * s_res);
                amax = fmaxf(amax, fabsf(r));
            }
    }
#pragma unroll
    for (int o = S >> 1; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
    if (!live) return;
    const float scale = amax < kEps ? 1.0f : amax;
    const float inv = kQMax * rcp_rn_pos(scale);
    const int8_t e_out = exponent_of(scale);
    uint4* ov = reinterpret_cast<uint4*>(out) + pos * G;
    for (int g = gl; g < G; g += S) {
        const float s_res = unit_of(res_s[pos * G + g]);
        const float s_in = skipped ? 0.0f : unit_of(main_s[pos * G + g]) * main_mult;
        const uint4 a = skipped ? make_uint4(0u, 0u, 0u, 0u) : mv[g];
        const uint4 b = rv[g];
        const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, bw[4] = {b.x, b.y, b.z, b.w};
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            w[i] = 0u;
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const float r = fmaf(static_cast<float>(code_of(aw[i], e)), s_in, static_cast<float>(code_of(bw[i], e)) * s_res);
                w[i] |= code_rn(r, inv) << (e << 2);
            }
        }
        ov[g] = make_uint4(w[0], w[1], w[2], w[3]);
        out_s[pos * G + g] = e_out;
    }
}

// Global average pool: one warp per (frame, 32-channel group), lane = channel.
// Partial sums over blocks of 16 pixels (the reference's per-CTA chunk) are
// combined in block order, which makes the result deterministic.
template <bool kHalf>
__global__ void __launch_bounds__(kThreads) gap_kernel(const uint32_t* __restrict__ in, const int8_t* __restrict__ in_s,
                                                     int64_t frames, int HW, int C, float* __restrict__ out_f32,
                                                     __half* __restrict__ out_f16, uint32_t* __restrict__ out_q,
                                                     int8_t* __restrict__ out_qs)
{
    const int lane = threadIdx.x & 31;
    const int64_t warp = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) >> 5;
    const int G = C >> 5;
    if (warp >= frames * G) return;
    const int64_t frame = warp / G;
    const int g = static_cast<int>(warp - frame * G);
    const int c = (g << 5) + lane;
    const float inv = __frcp_rn(static_cast<float>(HW));
    float acc = 0.0f;
    __half acc_h = __float2half_rn(0.0f);
    for (int start = 0; start < HW; start += 16) {
        const int end = min(start + 16, HW);
        float part = 0.0f;
        for (int i = start; i < end; ++i) {
            const int64_t sp = frame * HW + i;
            const uint32_t w = in[sp * (C >> 3) + (c >> 3)];
            part = fmaf(static_cast<float>(code_of(w, c & 7)), unit_of(in_s[sp * G + g]), part);
        }
        // __fmul_rn keeps the scaled partial separately rounded (as it is when
        // the reference hands it to atomicAdd) instead of letting the
        // compiler fuse it into the running sum.
        if (kHalf) acc_h = __hadd(acc_h, __float2half_rn(__fmul_rn(part, inv)));
        else acc = __fadd_rn(acc, __fmul_rn(part, inv));
    }
    const int64_t oi = frame * C + c;
    if (kHalf) {
        out_f16[oi] = acc_h;
        return;
    }
    if (out_f32) out_f32[oi] = acc;
    if (out_q) {
        float amax = fabsf(acc);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
        const float scale = amax < kEps ? 1.0f : amax;
        uint32_t q = code_rn(acc, kQMax * rcp_rn_pos(scale)) << ((lane & 7) << 2);
#pragma unroll
        for (int o = 4; o > 0; o >>= 1) q |= __shfl_down_sync(0xFFFFFFFFu, q, o);
        if ((lane & 7) == 0) out_q[frame * (C >> 3) + (g << 2) + (lane >> 3)] = q;
        if (lane == 0) out_qs[frame * G + g] = exponent_of(scale);
    }
}

// Action bits: thread per (row, 64-bit word), bit j set when the position hash
// of (int(p * 65504) ^ j) maps below p.
__global__ void __launch_bounds__(kThreads) set_actions_kernel(const float* __restrict__ probs, int64_t rows, int A,
                                                             unsigned long long* __restrict__ actions)
{
    const int words = (A + 63) >> 6;
    const int64_t t = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
    if (t >= rows * words) return;
    const int64_t row = t / words;
    const int wi = static_cast<int>(t - row * words);
    unsigned long long bits = 0ull;
    for (int j = wi << 6; j < min(A, (wi + 1) << 6); ++j) {
        const float p = probs[row * A + j];
        const int32_t sample = static_cast<int32_t>(p * 65504.0f) ^ j;
        if (hashed_uniform(position_seed(static_cast<uint32_t>(j), sample), 1.0f) < p) bits |= 1ull << (j & 63);
    }
    actions[t] = bits;
}

inline unsigned grid_for(int64_t threads) { return static_cast<unsigned>((threads + kThreads - 1) / kThreads); }

}  // namespace

cudaError_t launch_pack_f32(const float* in, int64_t n, uint32_t* out, int8_t* out_s, bool stochastic, int32_t add_idx,
                            int64_t row_groups, cudaStream_t stream)
{
    const int64_t groups = n >> 5;
    if (groups == 0) return cudaSuccess;
    if (stochastic) pack_f32_kernel<true><<<grid_for(groups), kThreads, 0, stream>>>(in, out, out_s, groups, add_idx, row_groups);
    else pack_f32_kernel<false><<<grid_for(groups), kThreads, 0, stream>>>(in, out, out_s, groups, add_idx, row_groups);
    return cudaGetLastError();
}

cudaError_t launch_stem_pack(const __half* planes, int64_t frames, int planes_present, int channels, int dim,
                             uint32_t* out, int8_t* out_s, cudaStream_t stream)
{
    const int64_t pixels = frames * dim * dim;
    if (pixels == 0) return cudaSuccess;
    const int hw = dim * dim;
    if (hw % 4 == 0 && reinterpret_cast<uintptr_t>(planes) % 8 == 0 && reinterpret_cast<uintptr_t>(out_s) % 4 == 0 &&
        channels == 32 && planes_present >= 1 && planes_present <= 8) {
        const int64_t quads = pixels / 4;
        const unsigned grid = grid_for(quads);
        const int lg_hw = (hw & (hw - 1)) == 0 ? 31 - __builtin_clz(static_cast<unsigned>(hw)) : -1;
#define AIC_STEM_NP(NP) stem_pack4_np_kernel<NP><<<grid, kThreads, 0, stream>>>(planes, quads, hw, lg_hw, out, out_s)
        switch (planes_present) {
            case 1: AIC_STEM_NP(1); break;
            case 2: AIC_STEM_NP(2); break;
            case 3: AIC_STEM_NP(3); break;
            case 4: AIC_STEM_NP(4); break;
            case 5: AIC_STEM_NP(5); break;
            case 6: AIC_STEM_NP(6); break;
            case 7: AIC_STEM_NP(7); break;
            default: AIC_STEM_NP(8); break;
        }
#undef AIC_STEM_NP
        return cudaGetLastError();
    }
    if (hw % 4 == 0 && reinterpret_cast<uintptr_t>(planes) % 8 == 0 && reinterpret_cast<uintptr_t>(out_s) % 4 == 0) {
        const int64_t quads = pixels / 4;
        stem_pack4_kernel<<<grid_for(quads), kThreads, 0, stream>>>(planes, quads, hw, planes_present, channels, out, out_s);
    } else {
        stem_pack_kernel<<<grid_for(pixels), kThreads, 0, stream>>>(planes, pixels, hw, planes_present, channels, out, out_s);
    }
    return cudaGetLastError();
}

cudaError_t launch_residual(const uint32_t* main_in, const int8_t* main_s, const uint32_t* res, const int8_t* res_s,
                            uint32_t* out, int8_t* out_s, int64_t positions, int C, float main_mult, bool skipped,
                            cudaStream_t stream)
{
    if (positions == 0) return cudaSuccess;
    const int G = C >> 5;
    int S = 1;
    while (S < G && S < 32) S <<= 1;
    if (S == G) {  // one group per lane, two positions per lane
        const int64_t warps2 = (positions + 2 * (32 / S) - 1) / (2 * (32 / S));
        const unsigned grid2 = grid_for(warps2 * 32);
#define AIC_RES2(SS) residual_pos2_kernel<SS><<<grid2, kThreads, 0, stream>>>(main_in, main_s, res, res_s, out, out_s, positions, main_mult, skipped)
        switch (S) {
            case 1: AIC_RES2(1); break;
            case 2: AIC_RES2(2); break;
            case 4: AIC_RES2(4); break;
            case 8: AIC_RES2(8); break;
            case 16: AIC_RES2(16); break;
            default: AIC_RES2(32); break;
        }
#undef AIC_RES2
        return cudaGetLastError();
    }
    const int64_t warps = (positions + (32 / S) - 1) / (32 / S);
    const unsigned grid = grid_for(warps * 32);
#define AIC_RES(SS) residual_kernel<SS><<<grid, kThreads, 0, stream>>>(main_in, main_s, res, res_s, out, out_s, positions, C, main_mult, skipped)
    switch (S) {
        case 1: AIC_RES(1); break;
        case 2: AIC_RES(2); break;
        case 4: AIC_RES(4); break;
        case 8: AIC_RES(8); break;
        case 16: AIC_RES(16); break;
        default: AIC_RES(32); break;
    }
#undef AIC_RES
    return cudaGetLastError();
}

cudaError_t launch_gap(const uint32_t* in, const int8_t* in_s, int64_t frames, int HW, int C, float* out_f32,
                       uint32_t* out_q, int8_t* out_qs, cudaStream_t stream)
{
    const int64_t warps = frames * (C >> 5);
    if (warps == 0) return cudaSuccess;
    gap_kernel<false><<<grid_for(warps * 32), kThreads, 0, stream>>>(in, in_s, frames, HW, C, out_f32, nullptr, out_q, out_qs);
    return cudaGetLastError();
}

cudaError_t launch_gap_f16(const uint32_t* in, const int8_t* in_s, int64_t frames, int HW, int C, __half* out,
                           cudaStream_t stream)
{
    const int64_t warps = frames * (C >> 5);
    if (warps == 0) return cudaSuccess;
    gap_kernel<true><<<grid_for(warps * 32), kThreads, 0, stream>>>(in, in_s, frames, HW, C, nullptr, out, nullptr, nullptr);
    return cudaGetLastError();
}

cudaError_t launch_set_actions(const float* probs, int64_t rows, int A, unsigned long long* actions, cudaStream_t stream)
{
    const int64_t n = rows * ((A + 63) >> 6);
    if (n == 0) return cudaSuccess;
    set_actions_kernel<<<grid_for(n), kThreads, 0, stream>>>(probs, rows, A, actions);
    return cudaGetLastError();
}

namespace {
// d = (1 + i / 2^23) * 2^e for every i < 2^23 and the exponents below: counts
// the d where rcp_rn_pos and __frcp_rn differ in any bit.
__constant__ int kRcpExps[13] = {-13, -7, -1, 0, 1, 2, 22, 23, 24, 64, 100, 125, 126};
__global__ void selftest_rcp_kernel(unsigned long long* mismatches, float* first_bad)
{
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (1u << 23)) return;
    for (int k = 0; k < 13; ++k) {
        const float d = __uint_as_float((static_cast<uint32_t>(127 + kRcpExps[k]) << 23) | i);
        if (__float_as_uint(rcp_rn_pos(d)) != __float_as_uint(__frcp_rn(d))) {
            if (atomicAdd(mismatches, 1ull) == 0ull) *first_bad = d;
        }
    }
    if (i == 0) {  // the clamped top of the range
        const float top[3] = {3.40282347e38f, __uint_as_float(0x7F800000u), 1.7e38f};
        for (int k = 0; k < 3; ++k)
            if (__float_as_uint(rcp_rn_pos(top[k])) != __float_as_uint(__frcp_rn(top[k]))) {
                if (atomicAdd(mismatches, 1ull) == 0ull) *first_bad = top[k];
            }
    }
}
}  // namespace

cudaError_t launch_selftest_rcp(unsigned long long* mismatches, float* first_bad, cudaStream_t stream)
{
    selftest_rcp_kernel<<<(1u << 23) / 256, 256, 0, stream>>>(mismatches, first_bad);
    return cudaGetLastError();
}

}  // namespace aic
