// Convolution kernels on CUDA cores: the depthwise k x k conv (A5) and the
// quantized implicit-GEMM conv (A3 dense k2/k4, A4 pointwise) with its fused
// RMSNorm + bias + SiLU + requant epilogue. Both reproduce the reference's
// per-output accumulation order, so their results are bit-identical to the
// reference kernels (AICortex kernels.h:217-282, 514-585, 831-870).
#include "aic_common.cuh"
#include "aic_kernels.h"

namespace aic {
namespace {

constexpr int kThreads = 256;

// Depthwise conv: one thread per (output pixel, word of 8 channels); the four
// threads of a 32-channel group sit in consecutive lanes and share the absmax
// through two shuffles. Per channel and tap: fma(x, w, acc[tap & 3]) with
// x = code * unit(s_in) and w the weight dequantised once at load time
// (code * unit(s_w), the value the reference recomputes per tap); the four
// partial sums are folded into the bias in order (kernels.h:848-858).
template <int K>
__global__ void __launch_bounds__(kThreads) conv_dw_kernel(const uint32_t* __restrict__ in, const int8_t* __restrict__ in_s,
                                                         const float* __restrict__ wf, const float* __restrict__ bias,
                                                         uint32_t* __restrict__ out, int8_t* __restrict__ out_s,
                                                         int64_t total_words, int C, int stride, int Din, int Dout)
{
    constexpr int kPad = K >> 1;
    const int64_t t = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
    const bool live = t < total_words;
    const int words = C >> 3, G = C >> 5;
    const int64_t tt = live ? t : 0;
    const int j = static_cast<int>(tt % words);
    const int64_t pix = tt / words;
    const int hw_out = Dout * Dout;
    const int64_t frame = pix / hw_out;
    const int p = static_cast<int>(pix - frame * hw_out);
    const int g = j >> 2;
    const int h0 = (p / Dout) * stride - kPad;
    const int w0 = (p % Dout) * stride - kPad;
    const int64_t frame_base = frame * Din * Din;
    float aa[4][8];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int e = 0; e < 8; ++e) aa[a][e] = 0.0f;
#pragma unroll
    for (int k = 0; k < K * K; ++k) {
        const int hi = h0 + k / K, wi = w0 + k % K;
        const bool valid = hi >= 0 && hi < Din && wi >= 0 && wi < Din;
        const int64_t sp = frame_base + static_cast<int64_t>(valid ? hi : 0) * Din + (valid ? wi : 0);
        const uint32_t xw = valid ? __ldg(in + sp * words + j) : 0u;
        const float xu = unit_of(valid ? __ldg(in_s + sp * G + g) : static_cast<int8_t>(0));
        const float4* wp = reinterpret_cast<const float4*>(wf + static_cast<int64_t>(k) * C + (j << 3));
        const float4 wa = __ldg(wp), wb = __ldg(wp + 1);
        const float wv[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) aa[k & 3][e] = fmaf(code_f(xw, e) * xu, wv[e], aa[k & 3][e]);
    }
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = __ldg(bias + (j << 3) + e) + (aa[0][e] + aa[1][e] + aa[2][e] + aa[3][e]);
    int8_t ex;
    const uint32_t q = quantize_word_x4(v, &ex);
    if (!live) return;
    out[t] = q;
    if ((j & 3) == 0) out_s[pix * G + g] = ex;
}

// Depthwise conv, tiled: a CTA computes a TH x 8 block of output pixels for
// one 32-channel group. The input block it reads (with the halo) is staged once
// in shared memory already dequantised, x = code * unit(s_in) (the value the
// reference forms per tap), with zeros outside the image (the reference's
// invalid taps contribute fma(0, w, acc)). Thread (channel quad cq, pixel pp)
// keeps its 4 channels' k*k weights in registers and runs the reference's
// per-tap chains acc[tap & 3] for pixels pp, pp + 32, ..., then folds them into
// the bias in order and packs the 32-channel group across 8 lanes. Pixel
// quads are stored XOR-swizzled so both the staging stores and the tap loads
// are bank-conflict free.
// CC, DIN: the channel count and input size when known at compile time (0:
// taken from the arguments); the cortex's layers each have their own.
template <int K, int S, int TH, int CC = 0, int DIN = 0>
__global__ void __launch_bounds__(kThreads) conv_dw_tiled_kernel(const uint32_t* __restrict__ in, const int8_t* __restrict__ in_s,
                                                               const float* __restrict__ wf, const float* __restrict__ bias,
                                                               uint32_t* __restrict__ out, int8_t* __restrict__ out_s,
                                                               int C_arg, int Din_arg, int Dout_arg, int tiles_x, int tiles_y,
                                                               int lg_g, int lg_tx, int lg_tpf)
{
    // output block TH rows x 8 columns; input block with its halo
    constexpr int kPad = K >> 1, kHin = (TH - 1) * S + K, kWin = 7 * S + K;
    constexpr int DOUT = DIN ? (DIN + 2 * kPad - K) / S + 1 : 0;
    const int C = CC ? CC : C_arg, Din = DIN ? DIN : Din_arg, Dout = DIN ? DOUT : Dout_arg;
    extern __shared__ float4 xs[];  // [kHin * kWin][8] float4, quad q of pixel i at i * 8 + (q ^ (i & 7))
    const int G = C >> 5;
    // the channel groups of one tile are consecutive blocks, so they run
    // together and share the L2 lines of the tile's pixels (a pixel's groups
    // lie in the same DRAM lines; one group per grid row re-read them per group)
    // block -> (frame, tile row, tile column, group) in 32-bit arithmetic (the
    // launcher keeps the block count below 2^31), by shifts where the counts
    // are powers of two (lg_* >= 0; every layer of the cortex)
    const uint32_t bid = blockIdx.x;
    const int tiles_pf = tiles_x * tiles_y;
    const uint32_t tile = lg_g >= 0 ? bid >> lg_g : bid / static_cast<uint32_t>(G);
    const int g = static_cast<int>(bid - tile * static_cast<uint32_t>(G));
    const uint32_t fr = lg_tpf >= 0 ? tile >> lg_tpf : tile / static_cast<uint32_t>(tiles_pf);
    const int tin = static_cast<int>(tile - fr * static_cast<uint32_t>(tiles_pf));
    const int ty = lg_tx >= 0 ? tin >> lg_tx : tin / tiles_x, tx = tin - ty * tiles_x;
    const int64_t frame = fr;
    const int oy0 = ty * TH, ox0 = tx * 8;
    const int iy0 = oy0 * S - kPad, ix0 = ox0 * S - kPad;
    const int64_t fbase = frame * Din * Din;

    // every load of the thread's input pixels is issued before any is used,
    // so the block waits for one memory round trip instead of one per pixel
    constexpr int kPixIn = kHin * kWin, kPerThread = (kPixIn + kThreads - 1) / kThreads;
    uint4 xw[kPerThread];
    int xe[kPerThread];  // -128 (no exponent is below -120): outside the image
#pragma unroll
    for (int it = 0; it < kPerThread; ++it) {
        const int i = static_cast<int>(threadIdx.x) + it * kThreads;
        const int ry = i / kWin, rx = i - ry * kWin;
        const int iy = iy0 + ry, ix = ix0 + rx;
        xw[it] = make_uint4(0u, 0u, 0u, 0u);
        xe[it] = -128;
        if (i < kPixIn && iy >= 0 && iy < Din && ix >= 0 && ix < Din) {
            const int64_t pix = fbase + static_cast<int64_t>(iy) * Din + ix;
            xw[it] = __ldg(reinterpret_cast<const uint4*>(in) + pix * G + g);
            xe[it] = __ldg(in_s + pix * G + g);
        }
    }
#pragma unroll
    for (int it = 0; it < kPerThread; ++it) {
        const int i = static_cast<int>(threadIdx.x) + it * kThreads;
        if (i >= kPixIn) break;
        float4* dst = xs + i * 8;
        const int sw = i & 7;
        if (xe[it] != -128) {
            const float2 u = dup2(unit_of(static_cast<int8_t>(xe[it])));
            const uint32_t ww[4] = {xw[it].x, xw[it].y, xw[it].z, xw[it].w};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                // byte j of lo / hi: code 2j / 2j + 1 of the word as n ^ 8; each
                // is placed in the mantissa of 2^23 (0x4B0000bb = 2^23 + q + 8)
                const uint32_t lo = (ww[q] & 0x0F0F0F0Fu) ^ 0x08080808u;
                const uint32_t hi = ((ww[q] >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u;
                float2 x[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float2 c = make_float2(__uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7440u | j)),
                                                 __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7440u | j)));
                    x[j] = mul2(add2(c, dup2(-8388616.0f)), u);  // code * unit(s_in)
                }
                dst[(2 * q) ^ sw] = make_float4(x[0].x, x[0].y, x[1].x, x[1].y);
                dst[(2 * q + 1) ^ sw] = make_float4(x[2].x, x[2].y, x[3].x, x[3].y);
            }
        } else {
#pragma unroll
            for (int q = 0; q < 8; ++q) dst[q] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
    }

    const int cq = threadIdx.x & 7, pp = threadIdx.x >> 3;
    const int c0 = (g << 5) + 4 * cq;
    float2 wk[K * K][2];  // channel pairs (4cq, 4cq + 1), (4cq + 2, 4cq + 3)
#pragma unroll
    for (int k = 0; k < K * K; ++k) {
        const float4 w = __ldg(reinterpret_cast<const float4*>(wf + static_cast<int64_t>(k) * C + c0));
        wk[k][0] = make_float2(w.x, w.y);
        wk[k][1] = make_float2(w.z, w.w);
    }
    const float4 bv = __ldg(reinterpret_cast<const float4*>(bias + c0));
    const float2 b01 = make_float2(bv.x, bv.y), b23 = make_float2(bv.z, bv.w);
    // Thread (cq, pp) computes output pixels (oy + 4h, ox), h < TH / 4. Its
    // tap k reads input pixel ip0 + 4 h S kWin + (k / K) kWin + k % K; S kWin
    // is even, so 4 h S kWin is a multiple of 8 and the swizzled quad position
    // of every tap is the same for all h: the offsets are computed once.
    static_assert((S * kWin) % 2 == 0, "the swizzle phase must repeat every 4 output rows");
    const int oy = pp >> 3, ox = pp & 7;
    const int ip0 = oy * S * kWin + ox * S;
    int off[K * K];
#pragma unroll
    for (int k = 0; k < K * K; ++k) {
        const int ip = ip0 + (k / K) * kWin + k % K;
        off[k] = ip * 8 + (cq ^ (ip & 7));
    }
    __syncthreads();

#pragma unroll
    for (int h = 0; h < TH / 4; ++h) {
        const float4* xh = xs + h * 4 * S * kWin * 8;
        float2 a[4][2];
#pragma unroll
        for (int t = 0; t < 4; ++t) a[t][0] = a[t][1] = dup2(0.0f);
#pragma unroll
        for (int k = 0; k < K * K; ++k) {
            const float4 x = xh[off[k]];
            a[k & 3][0] = fma2(make_float2(x.x, x.y), wk[k][0], a[k & 3][0]);
            a[k & 3][1] = fma2(make_float2(x.z, x.w), wk[k][1], a[k & 3][1]);
        }
        const float2 v0 = add2(b01, add2(add2(add2(a[0][0], a[1][0]), a[2][0]), a[3][0]));
        const float2 v1 = add2(b23, add2(add2(add2(a[0][1], a[1][1]), a[2][1]), a[3][1]));
        // 32-channel group = 8 lanes (cq 0..7) of this pixel; requant as
        // quantize_group2 does (a warp whose groups are all finite skips the
        // clamps; any NaN or infinity sends the warp through the reference's
        // sequence)
        float amax = amax_nan(amax_nan(amax_nan(amax_nan(0.0f, v0.x), v0.y), v1.x), v1.y);
        amax = max_nan(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 1));
        amax = max_nan(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 2));
        amax = max_nan(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 4));
        float scale;
        uint32_t h16;
        if (__any_sync(0xFFFFFFFFu, !is_finite_amax(amax))) {
            float a = fmaxf(fmaxf(fmaxf(butterfly_start(), fabsf(v0.x)), fabsf(v0.y)), fmaxf(fabsf(v1.x), fabsf(v1.y)));
            a = fmaxf(a, __shfl_xor_sync(0xFFFFFFFFu, a, 1));
            a = fmaxf(a, __shfl_xor_sync(0xFFFFFFFFu, a, 2));
            a = fmaxf(a, __shfl_xor_sync(0xFFFFFFFFu, a, 4));
            scale = a < kEps ? 1.0f : a;
            const float inv = kQMax * rcp_rn_pos(scale);
            h16 = code_rn(v0.x, inv) | (code_rn(v0.y, inv) << 4) | (code_rn(v1.x, inv) << 8) | (code_rn(v1.y, inv) << 12);
        } else {
            scale = amax < kEps ? 1.0f : amax;
            const float inv = kQMax * rcp_rn_pos(scale);
            // bits 0x4B400000 + q_i -> nibbles, as pack8_magic does for 8 codes
            // (scalar: the product is rounded before the add)
            uint32_t h = magic_bits(__fmul_rn(v1.y, inv));
            h = (h << 4) + magic_bits(__fmul_rn(v1.x, inv));
            h = (h << 4) + magic_bits(__fmul_rn(v0.y, inv));
            h = (h << 4) + magic_bits(__fmul_rn(v0.x, inv));
            h16 = ((h - 0x4B3FFFF8u * 0x1111u) ^ 0x8888u) & 0xFFFFu;
        }
        const uint32_t other = __shfl_xor_sync(0xFFFFFFFFu, h16, 1);
        const int oyy = oy0 + oy + 4 * h, oxx = ox0 + ox;
        if (oyy < Dout && oxx < Dout) {
            const int64_t opix = frame * Dout * Dout + static_cast<int64_t>(oyy) * Dout + oxx;
            if ((cq & 1) == 0) out[opix * (C >> 3) + 4 * g + (cq >> 1)] = h16 | (other << 16);
            if (cq == 0) out_s[opix * G + g] = exponent_of(scale);
        }
    }
}

// Dequantised depthwise weights: wf[i] = code(i) * unit(s[i / 32]), the value
// dequantize_scalar produces for every tap (kernels.h:77, 856-857).
__global__ void dw_weights_kernel(const uint32_t* __restrict__ w, const int8_t* __restrict__ w_s, int64_t n,
                                  float* __restrict__ wf)
{
    const int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
    if (i >= n) return;
    wf[i] = static_cast<float>(code_of(w[i >> 3], static_cast<int>(i & 7))) * unit_of(w_s[i >> 5]);
}

// Implicit-GEMM quantized conv on CUDA cores. A CTA owns TP output pixels and
// one 256-channel chunk (thread = output channel). The TP input rows (all k*k
// taps) are staged in shared memory and read as broadcasts; each thread
// streams its own weight row once per tile. Per (pixel, channel) the
// accumulation is acc[tap & 3] += unit(s_in) * (unit(s_w) * dot) in tap then
// group order, and the epilogue reduces acc^2 with the reference's
// warp-butterfly then cross-warp-butterfly tree.
template <int TP, int KS>
__global__ void __launch_bounds__(kThreads) conv_gemm_simt_kernel(
    const uint32_t* __restrict__ in, const int8_t* __restrict__ in_s, const uint32_t* __restrict__ w,
    const int8_t* __restrict__ w_s, const float* __restrict__ bias, uint32_t* __restrict__ out, int8_t* __restrict__ out_s,
    int64_t total_pix, int InC, int OutC, int stride, int Din, int Dout, bool act)
{
    constexpr int kTaps = KS * KS;
    extern __shared__ uint4 smem_rows[];  // [TP][kTaps][G] groups, then exponents
    __shared__ float part[TP][kThreads / 32];
    __shared__ float total_sq[TP];
    __shared__ unsigned char tap_ok[TP][kTaps];
    const int G = InC >> 5;
    int8_t* smem_exp = reinterpret_cast<int8_t*>(smem_rows + TP * kTaps * G);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int oc = blockIdx.y * kThreads + threadIdx.x;
    const bool active = oc < OutC;
    const int64_t pix0 = static_cast<int64_t>(blockIdx.x) * TP;
    const int pad = KS == stride ? 0 : (KS - 1) >> 1;
    const int hw_out = Dout * Dout;

    // Stage the input rows.
    for (int i = threadIdx.x; i < TP * kTaps * G; i += kThreads) {
        const int pp = i / (kTaps * G);
        const int k = (i / G) % kTaps;
        const int g = i % G;
        const int64_t pix = pix0 + pp;
        bool ok = pix < total_pix;
        int64_t sp = 0;
        if (ok) {
            const int64_t frame = pix / hw_out;
            const int p = static_cast<int>(pix - frame * hw_out);
            const int hi = (p / Dout) * stride - pad + k / KS;
            const int wi = (p % Dout) * stride - pad + k % KS;
            ok = hi >= 0 && hi < Din && wi >= 0 && wi < Din;
            sp = frame * Din * Din + static_cast<int64_t>(hi) * Din + wi;
        }
        smem_rows[i] = ok ? reinterpret_cast<const uint4*>(in)[sp * G + g] : make_uint4(0u, 0u, 0u, 0u);
        smem_exp[i] = ok ? in_s[sp * G + g] : static_cast<int8_t>(0);
        if (g == 0) tap_ok[pp][k] = ok ? 1 : 0;
    }
    __syncthreads();

    float aa[TP][KS == 1 ? 1 : 4];
#pragma unroll
    for (int pp = 0; pp < TP; ++pp)
#pragma unroll
        for (int a = 0; a < (KS == 1 ? 1 : 4); ++a) aa[pp][a] = 0.0f;
    if (active) {
        const uint4* wrow = reinterpret_cast<const uint4*>(w) + static_cast<int64_t>(oc) * kTaps * G;
        const int8_t* wsrow = w_s + static_cast<int64_t>(oc) * kTaps * G;
        for (int k = 0; k < kTaps; ++k) {
            for (int g = 0; g < G; ++g) {
                const uint4 wv = wrow[k * G + g];
                const float wu = unit_of(wsrow[k * G + g]);
#pragma unroll
                for (int pp = 0; pp < TP; ++pp) {
                    if (!tap_ok[pp][k]) continue;
                    const int si = (pp * kTaps + k) * G + g;
                    const uint4 xv = smem_rows[si];
                    const int dot = dot8(xv.x, wv.x) + dot8(xv.y, wv.y) + dot8(xv.z, wv.z) + dot8(xv.w, wv.w);
                    float& acc = aa[pp][KS == 1 ? 0 : (k & 3)];
                    acc = fmaf(unit_of(smem_exp[si]), wu * static_cast<float>(dot), acc);
                }
            }
        }
    }
    float accv[TP];
#pragma unroll
    for (int pp = 0; pp < TP; ++pp) {
        if (KS == 1) accv[pp] = aa[pp][0];
        else accv[pp] = aa[pp][0] + aa[pp][KS == 1 ? 0 : 1] + aa[pp][KS == 1 ? 0 : 2] + aa[pp][KS == 1 ? 0 : 3];
        float sq = active ? accv[pp] * accv[pp] : 0.0f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xFFFFFFFFu, sq, o);
        if (lane == 0) part[pp][warp] = sq;
    }
    __syncthreads();
    for (int pp = warp; pp < TP; pp += kThreads / 32) {
        float s = lane < kThreads / 32 ? part[pp][lane] : 0.0f;
#pragma unroll
        for (int o = (kThreads / 32) >> 1; o > 0; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
        if (lane == 0) total_sq[pp] = s;
    }
    __syncthreads();
    const float inv_div = __frcp_rn(static_cast<float>(min(OutC, kNormChunk)));
    const float b = active ? bias[oc] : 0.0f;
#pragma unroll
    for (int pp = 0; pp < TP; ++pp) {
        const int64_t pix = pix0 + pp;
        float v = fmaf(accv[pp], __frsqrt_rn(fmaf(total_sq[pp], inv_div, kEps)), b);
        if (act) v = silu_f(v);
        float amax = fabsf(v);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
        const float scale = amax < kEps ? 1.0f : amax;
        uint32_t q = code_rn(v, kQMax * __frcp_rn(scale)) << ((lane & 7) << 2);
#pragma unroll
        for (int o = 4; o > 0; o >>= 1) q |= __shfl_down_sync(0xFFFFFFFFu, q, o);
        if (active && pix < total_pix) {
            if ((lane & 7) == 0) out[pix * (OutC >> 3) + (oc >> 3)] = q;
            if (lane == 0) out_s[pix * (OutC >> 5) + (oc >> 5)] = exponent_of(scale);
        }
    }
}

inline unsigned grid_for(int64_t threads) { return static_cast<unsigned>((threads + kThreads - 1) / kThreads); }

template <int TP, int KS>
cudaError_t launch_gemm_tp(const uint32_t* in, const int8_t* in_s, const uint32_t* w, const int8_t* w_s, const float* bias,
                           uint32_t* out, int8_t* out_s, int64_t total_pix, int InC, int OutC, int stride, int Din,
                           int Dout, bool act, cudaStream_t stream)
{
    const int G = InC >> 5;
    const size_t smem = static_cast<size_t>(TP) * KS * KS * G * (sizeof(uint4) + 1);
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(conv_gemm_simt_kernel<TP, KS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem));
        if (e != cudaSuccess) return e;
    }
    dim3 grid(static_cast<unsigned>((total_pix + TP - 1) / TP), static_cast<unsigned>((OutC + kThreads - 1) / kThreads));
    conv_gemm_simt_kernel<TP, KS><<<grid, kThreads, smem, stream>>>(in, in_s, w, w_s, bias, out, out_s, total_pix, InC,
                                                                   OutC, stride, Din, Dout, act);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_dw_weights(const uint32_t* w, const int8_t* w_s, int64_t n, float* wf, cudaStream_t stream)
{
    if (n == 0) return cudaSuccess;
    dw_weights_kernel<<<grid_for(n), kThreads, 0, stream>>>(w, w_s, n, wf);
    return cudaGetLastError();
}

template <int K, int S, int TH = 8, int CC = 0, int DIN = 0>
cudaError_t launch_dw_tiled(const uint32_t* in, const int8_t* in_s, const float* wf, const float* bias, uint32_t* out,
                            int8_t* out_s, int64_t frames, int C, int Din, int Dout, cudaStream_t stream)
{
    constexpr int kHin = (TH - 1) * S + K, kWin = 7 * S + K;
    const size_t smem = static_cast<size_t>(kHin) * kWin * 8 * sizeof(float4);
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(conv_dw_tiled_kernel<K, S, TH, CC, DIN>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
    }
    const int tiles_x = (Dout + 7) / 8, tiles_y = (Dout + TH - 1) / TH;
    const int64_t blocks = frames * tiles_x * tiles_y * (C >> 5);
    if (blocks > 0x7FFFFFFF) return cudaErrorInvalidValue;
    auto lg = [](int v) { return v > 0 && (v & (v - 1)) == 0 ? 31 - __builtin_clz(static_cast<unsigned>(v)) : -1; };
    const dim3 grid(static_cast<unsigned>(blocks), 1u);
    conv_dw_tiled_kernel<K, S, TH, CC, DIN><<<grid, kThreads, smem, stream>>>(in, in_s, wf, bias, out, out_s, C, Din, Dout,
                                                                              tiles_x, tiles_y, lg(C >> 5), lg(tiles_x),
                                                                              lg(tiles_x * tiles_y));
    return cudaGetLastError();
}

cudaError_t launch_conv_dw(const uint32_t* in, const int8_t* in_s, const float* wf, const float* bias, uint32_t* out,
                           int8_t* out_s, int64_t frames, int C, int ksize, int stride, int Din, int Dout,
                           cudaStream_t stream)
{
    if (frames == 0) return cudaSuccess;
    // 3x3 (the stack's kernel) tiled, 16 x 8 output blocks at stride 2 (measured
    // 16 % faster than 8 x 8 on the stack's first block), 8 x 8 when the whole
    // output frame is at most 8 rows (a 16-row block would leave half its
    // threads idle); larger kernels keep k*k weight quads per thread only at
    // very high register counts, so they run direct
    if (ksize == 3 && stride == 1)
        return launch_dw_tiled<3, 1>(in, in_s, wf, bias, out, out_s, frames, C, Din, Dout, stream);
    if (ksize == 3 && stride == 2 && Dout <= 8) {
        if (C == 256 && Din == 16 && Dout == 8)  // the cortex's block 3 (shapes known at compile time)
            return launch_dw_tiled<3, 2, 8, 256, 16>(in, in_s, wf, bias, out, out_s, frames, C, Din, Dout, stream);
        return launch_dw_tiled<3, 2, 8>(in, in_s, wf, bias, out, out_s, frames, C, Din, Dout, stream);
    }
    if (ksize == 3 && stride == 2) {
        // the cortex's blocks 0-2 (shapes known at compile time)
        if (C == 32 && Din == 128 && Dout == 64)
            return launch_dw_tiled<3, 2, 16, 32, 128>(in, in_s, wf, bias, out, out_s, frames, C, Din, Dout, stream);
        if (C == 64 && Din == 64 && Dout == 32)
            return launch_dw_tiled<3, 2, 16, 64, 64>(in, in_s, wf, bias, out, out_s, frames, C, Din, Dout, stream);
        if (C == 128 && Din == 32 && Dout == 16)
            return launch_dw_tiled<3, 2, 16, 128, 32>(in, in_s, wf, bias, out, out_s, frames, C, Din, Dout, stream);
        return launch_dw_tiled<3, 2, 16>(in, in_s, wf, bias, out, out_s, frames, C, Din, Dout, stream);
    }
    return launch_conv_dw_direct(in, in_s, wf, bias, out, out_s, frames, C, ksize, stride, Din, Dout, stream);
}

cudaError_t launch_conv_dw_direct(const uint32_t* in, const int8_t* in_s, const float* wf, const float* bias,
                                  uint32_t* out, int8_t* out_s, int64_t frames, int C, int ksize, int stride, int Din,
                                  int Dout, cudaStream_t stream)
{
    const int64_t total = frames * Dout * Dout * (C >> 3);
    if (total == 0) return cudaSuccess;
    const unsigned grid = grid_for(total);
    switch (ksize) {
        case 3: conv_dw_kernel<3><<<grid, kThreads, 0, stream>>>(in, in_s, wf, bias, out, out_s, total, C, stride, Din, Dout); break;
        case 5: conv_dw_kernel<5><<<grid, kThreads, 0, stream>>>(in, in_s, wf, bias, out, out_s, total, C, stride, Din, Dout); break;
        case 7: conv_dw_kernel<7><<<grid, kThreads, 0, stream>>>(in, in_s, wf, bias, out, out_s, total, C, stride, Din, Dout); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_conv_gemm_simt(const uint32_t* in, const int8_t* in_s, const uint32_t* w, const int8_t* w_s,
                                  const float* bias, uint32_t* out, int8_t* out_s, int64_t frames, int InC, int OutC,
                                  int ksize, int stride, int Din, int Dout, bool act, cudaStream_t stream)
{
    const int64_t total_pix = frames * Dout * Dout;
    if (total_pix == 0) return cudaSuccess;
    switch (ksize) {
        case 1: return launch_gemm_tp<16, 1>(in, in_s, w, w_s, bias, out, out_s, total_pix, InC, OutC, 1, Din, Dout, act, stream);
        case 2: return launch_gemm_tp<8, 2>(in, in_s, w, w_s, bias, out, out_s, total_pix, InC, OutC, stride, Din, Dout, act, stream);
        case 4: return launch_gemm_tp<8, 4>(in, in_s, w, w_s, bias, out, out_s, total_pix, InC, OutC, stride, Din, Dout, act, stream);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace aic
