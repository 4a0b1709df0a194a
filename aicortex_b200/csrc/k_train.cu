// Backward and SGD kernels of the training path (the reference's *Bwd*,
// ApplyTraces and updateParams kernels, kernels.h:196-216, 283-513, 586-830,
// 871-988, 1056-1079, 1260-1419, 1779-1805), on CUDA cores with the
// reference's floating-point order, one layer step (one frame / one env step)
// per call as the reference's layer classes run them.
//
// The reference's gradients are kept as its kernels compute them, including
// three places where they differ from the textbook gradient of its forward:
//  * the RMSNorm is differentiated as a constant scale (dy * inv_rms);
//  * the pointwise weight gradient (kernels.h:359-444) pairs input channel
//    y + 32 by of position p0 + y with output gradient of position p0 + k and
//    takes inv_rms from a 32-channel x 8-position square sum;
//  * Mamba's out-projection recompute reduces its 8-lane partial sums with
//    absolute-lane shuffles (kernels.h:1299), which mix in lanes 1, 2 and 4.
// Where the reference reads memory it did not write (pointwise input gradient
// with fewer than 256 output channels, depthwise weight / bias gradients with
// fewer than 256 channels, positions past the frame), the kernels here skip
// the term or the element instead; every such case is documented at its kernel.
#include <cstdint>

#include "aic_common.cuh"
#include "aic_kernels.h"

namespace aic {
namespace {

constexpr int kT = 256;  // threads per block, gpu_block_threads

// silu_grad / sigmoid_grad (kernels.h:88-97). silu_grad is the product of
// the two factors of silu_parts; the reference's bias-gradient sums add that
// product to their accumulator, which the compiler contracts into one fma.
__device__ __forceinline__ float2 silu_parts(float x, float dy)
{
    const float sig = sigmoid_f(x);
    return make_float2(__fmul_rn(dy, sig), fmaf(x, __fsub_rn(1.0f, sig), 1.0f));
}
__device__ __forceinline__ float silu_grad_f(float x, float dy)
{
    const float2 f = silu_parts(x, dy);
    return __fmul_rn(f.x, f.y);
}
__device__ __forceinline__ float sigmoid_grad_f(float x, float dy)
{
    const float sig = sigmoid_f(x);
    return __fmul_rn(__fmul_rn(dy, sig), __fsub_rn(1.0f, sig));
}

// dequantize_scalar (kernels.h:77): code * unit(s).
__device__ __forceinline__ float deq(const uint32_t* __restrict__ words, const int8_t* __restrict__ exps, int64_t i)
{
    return __fmul_rn(static_cast<float>(code_of(words[i >> 3], static_cast<int>(i & 7))), unit_of(exps[i >> 5]));
}

// Sum of squares over a 256-thread block as the reference forms it: lane
// butterfly (xor 16..1), then warp 0 folds the 8 warp sums (xor 4..1).
// Every thread of the block must call it; returns the total in all threads.
__device__ __forceinline__ float block_sq256(float v, float* smem8)
{
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float s = __fmul_rn(v, v);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xFFFFFFFFu, s, o));
    if (lane == 0) smem8[warp] = s;
    __syncthreads();
    if (warp == 0) {
        float b = lane < 8 ? smem8[lane] : 0.0f;
#pragma unroll
        for (int o = 4; o > 0; o >>= 1) b = __fadd_rn(b, __shfl_xor_sync(0xFFFFFFFFu, b, o));
        if (lane == 0) smem8[8] = b;
    }
    __syncthreads();
    return smem8[8];
}

// ---------------------------------------------------------------- conv

// Forward recompute of one conv layer at every (position, output channel) of
// one frame, in the reference's order (pointwise: one fmaf chain over the
// groups, kernels.h:301-330; dense: one chain per tap & 3, summed, :605-633),
// then the block RMSNorm scale and the activation gradient
//   g = act ? silu_grad(acc * inv + bias, dy) : dy, dyn = g * inv;
// gsa / gst keep silu_grad's two factors (act) or dy and 1 (no act) for the
// bias gradient, facc the raw sum. Grid (positions, ceil(out / 256)), 256 threads.
__global__ void __launch_bounds__(kT) conv_bwd_recompute_kernel(
    const uint32_t* __restrict__ in, const int8_t* __restrict__ in_s, const uint32_t* __restrict__ w,
    const int8_t* __restrict__ w_s, const float* __restrict__ bias, const float* __restrict__ dy, int in_c, int out_c,
    int ks, int stride, int din, int dout, int act, float* __restrict__ gsa, float* __restrict__ gst,
    float* __restrict__ dyn, float* __restrict__ facc)
{
    __shared__ float smem8[9];
    const int p = blockIdx.x;
    const int oc = blockIdx.y * kT + threadIdx.x;
    const bool valid = oc < out_c;
    const int G = in_c >> 5, ksq = ks * ks;
    float acc = 0.0f;
    if (valid) {
        if (ks == 1) {
            const uint4* x = reinterpret_cast<const uint4*>(in) + static_cast<int64_t>(p) * G;
            const uint4* wr = reinterpret_cast<const uint4*>(w) + static_cast<int64_t>(oc) * G;
            for (int g = 0; g < G; ++g) {
                const uint4 a = x[g], b = wr[g];
                const int part = dot8(a.x, b.x) + dot8(a.y, b.y) + dot8(a.z, b.z) + dot8(a.w, b.w);
                acc = fmaf(unit_of(in_s[static_cast<int64_t>(p) * G + g]),
                           __fmul_rn(unit_of(w_s[static_cast<int64_t>(oc) * G + g]), static_cast<float>(part)), acc);
            }
        } else {
            const int pad = ks == stride ? 0 : (ks - 1) >> 1;
            const int hs = p / dout * stride - pad, ws0 = (p % dout) * stride - pad;
            float a4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            for (int k = 0; k < ksq; ++k) {
                const int hi = hs + k / ks, wi = ws0 + k % ks;
                if (hi < 0 || hi >= din || wi < 0 || wi >= din) continue;
                const int64_t pix = static_cast<int64_t>(hi) * din + wi;
                const uint4* x = reinterpret_cast<const uint4*>(in) + pix * G;
                const int64_t wg = (static_cast<int64_t>(oc) * ksq + k) * G;
                const uint4* wr = reinterpret_cast<const uint4*>(w) + wg;
                for (int g = 0; g < G; ++g) {
                    const uint4 a = x[g], b = wr[g];
                    const int part = dot8(a.x, b.x) + dot8(a.y, b.y) + dot8(a.z, b.z) + dot8(a.w, b.w);
                    a4[k & 3] = fmaf(unit_of(in_s[pix * G + g]), __fmul_rn(unit_of(w_s[wg + g]), static_cast<float>(part)),
                                     a4[k & 3]);
                }
            }
            acc = __fadd_rn(__fadd_rn(__fadd_rn(a4[0], a4[1]), a4[2]), a4[3]);
        }
    }
    const float tot = block_sq256(valid ? acc : 0.0f, smem8);
    if (!valid) return;
    const float inv = __frsqrt_rn(fmaf(tot, __frcp_rn(static_cast<float>(min(out_c, kT))), kEps));
    const int64_t o = static_cast<int64_t>(p) * out_c + oc;
    const float d = dy[o];
    const float2 f = act ? silu_parts(fmaf(acc, inv, bias[oc]), d) : make_float2(d, 1.0f);
    gsa[o] = f.x;
    gst[o] = f.y;
    dyn[o] = __fmul_rn(act ? __fmul_rn(f.x, f.y) : d, inv);
    facc[o] = acc;
}

// Bias gradient of the pointwise and dense convs (kernels.h:445-513, 760-830):
// per output channel, the activation gradients summed over positions in order
// (acc += silu_grad(u, dy), contracted: fma(dy * sig, 1 + u (1 - sig), acc)).
__global__ void conv_bwd_bias_kernel(const float* __restrict__ gsa, const float* __restrict__ gst, int positions,
                                     int out_c, int act, float* __restrict__ gb)
{
    const int oc = blockIdx.x * kT + threadIdx.x;
    if (oc >= out_c) return;
    float s = 0.0f;
    for (int p = 0; p < positions; ++p) {
        const int64_t o = static_cast<int64_t>(p) * out_c + oc;
        s = act ? fmaf(gsa[o], gst[o], s) : __fadd_rn(s, gsa[o]);
    }
    gb[oc] = s;
}

// Dense weight gradient (kernels.h:676-759): per (output channel, input
// channel) and tap, sum over output positions of input x dyn, in order.
__global__ void conv_bwd_dense_weight_kernel(const uint32_t* __restrict__ in, const int8_t* __restrict__ in_s,
                                             const float* __restrict__ dyn, int in_c, int out_c, int ks, int stride,
                                             int din, int dout, float* __restrict__ gw)
{
    const int64_t t = static_cast<int64_t>(blockIdx.x) * kT + threadIdx.x;
    if (t >= static_cast<int64_t>(out_c) * in_c) return;
    const int oc = static_cast<int>(t / in_c), ic = static_cast<int>(t % in_c);
    const int ksq = ks * ks, pad = ks == stride ? 0 : (ks - 1) >> 1;
    float s[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) s[k] = 0.0f;
    const int positions = dout * dout;
    for (int p = 0; p < positions; ++p) {
        const int hs = p / dout * stride - pad, ws0 = (p % dout) * stride - pad;
        const float d = dyn[static_cast<int64_t>(p) * out_c + oc];
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            if (k >= ksq) break;
            const int hi = hs + k / ks, wi = ws0 + k % ks;
            if (hi < 0 || hi >= din || wi < 0 || wi >= din) continue;
            s[k] = fmaf(deq(in, in_s, (static_cast<int64_t>(hi) * din + wi) * in_c + ic), d, s[k]);
        }
    }
    for (int k = 0; k < ksq; ++k) gw[(static_cast<int64_t>(oc) * ksq + k) * in_c + ic] = s[k];
}

// The pointwise weight gradient's own RMSNorm scale (kernels.h:415-427): for
// each 32-channel output tile and position p, the square sum of the tile's 32
// pre-norm sums (lane butterfly) is added over the 8 positions of p's
// 8-position group, in order, and dynw = act-gradient x inv of that sum.
// One warp per (position, tile).
__global__ void conv_bwd_pw_dynw_kernel(const float* __restrict__ facc, const float* __restrict__ dy,
                                        const float* __restrict__ bias, int positions, int out_c, int act,
                                        float* __restrict__ dynw)
{
    const int warp = static_cast<int>((static_cast<int64_t>(blockIdx.x) * kT + threadIdx.x) >> 5);
    const int lane = threadIdx.x & 31;
    const int tiles = out_c >> 5;
    if (warp >= (positions >> 3) * tiles) return;
    const int grp = warp / tiles, tile = warp % tiles;  // 8-position group, output tile
    const int oc = tile * 32 + lane;
    float sums[8];
    for (int i = 0; i < 8; ++i) {
        const float a = facc[static_cast<int64_t>(grp * 8 + i) * out_c + oc];
        float s = __fmul_rn(a, a);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xFFFFFFFFu, s, o));
        sums[i] = s;
    }
    float g = 0.0f;
    for (int i = 0; i < 8; ++i) g = __fadd_rn(g, sums[i]);
    const float inv = __frsqrt_rn(fmaf(g, __frcp_rn(static_cast<float>(min(out_c, kT))), kEps));
    const float b = bias[oc];
    for (int i = 0; i < 8; ++i) {
        const int64_t o = static_cast<int64_t>(grp * 8 + i) * out_c + oc;
        const float d = dy[o];
        const float ga = act ? silu_grad_f(fmaf(facc[o], inv, b), d) : d;
        dynw[o] = __fmul_rn(ga, inv);
    }
}

// Pointwise weight gradient (kernels.h:359-444): element (oc, ic) with
// ic = 32 by + y sums, over 32-position chunks p0 and k < 32 in four
// interleaved chains, input channel 32 by + k of position p0 + y times dynw
// of position p0 + k; positions must be a multiple of 32.
__global__ void conv_bwd_pw_weight_kernel(const uint32_t* __restrict__ in, const int8_t* __restrict__ in_s,
                                          const float* __restrict__ dynw, int positions, int in_c, int out_c,
                                          float* __restrict__ gw)
{
    const int64_t t = static_cast<int64_t>(blockIdx.x) * kT + threadIdx.x;
    if (t >= static_cast<int64_t>(out_c) * in_c) return;
    const int oc = static_cast<int>(t / in_c), ic = static_cast<int>(t % in_c);
    const int by = ic >> 5, y = ic & 31;
    float s[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int p0 = 0; p0 < positions; p0 += 32) {
        const int64_t row = static_cast<int64_t>(p0 + y) * in_c + by * 32;
        for (int k = 0; k < 32; k += 4) {
#pragma unroll
            for (int i = 0; i < 4; ++i)
                s[i] = fmaf(deq(in, in_s, row + k + i), dynw[static_cast<int64_t>(p0 + k + i) * out_c + oc], s[i]);
        }
    }
    gw[static_cast<int64_t>(oc) * in_c + ic] = __fadd_rn(__fadd_rn(__fadd_rn(s[0], s[1]), s[2]), s[3]);
}

// Input gradient of the pointwise conv (kernels.h:283-358), one block per
// (position, 256-channel output chunk c), accumulated into grad_in: thread x
// of the chunk's valid threads (x < out - 256 c) covers input channels
// x, x + 256, ..., with sum_i dyn[256 c + i] * master[256 c + i * in + ic]
// (the reference's index). The reference also runs i over the chunk's
// missing channels, whose dyn it never wrote; those terms are skipped here.
__global__ void __launch_bounds__(kT) conv_bwd_pw_input_kernel(const float* __restrict__ dyn,
                                                              const float* __restrict__ master, int in_c, int out_c,
                                                              float* __restrict__ grad_in)
{
    __shared__ float sd[kT];
    const int p = blockIdx.x, base = blockIdx.y * kT;
    const int nvalid = min(kT, out_c - base);
    if (threadIdx.x < nvalid) sd[threadIdx.x] = dyn[static_cast<int64_t>(p) * out_c + base + threadIdx.x];
    __syncthreads();
    if (threadIdx.x >= nvalid) return;
    for (int ic = threadIdx.x; ic < in_c; ic += kT) {
        float acc = 0.0f;
        for (int i = 0; i < nvalid; ++i) acc = fmaf(sd[i], master[base + static_cast<int64_t>(i) * in_c + ic], acc);
        atomicAdd(&grad_in[static_cast<int64_t>(p) * in_c + ic], acc);
    }
}

// Input gradient of the dense conv (kernels.h:586-675): per output position
// and 256-channel output chunk, for each in-bounds tap the chunk's dyn
// against the master weights, added to the tap's input pixel. Input channels
// x (mod 256) with x at or past the chunk's valid threads get nothing, as in
// the reference, whose threads past the output channels have returned.
__global__ void __launch_bounds__(kT) conv_bwd_dense_input_kernel(const float* __restrict__ dyn,
                                                                 const float* __restrict__ master, int in_c, int out_c,
                                                                 int ks, int stride, int din, int dout,
                                                                 float* __restrict__ grad_in)
{
    __shared__ float sd[kT];
    const int p = blockIdx.x, base = blockIdx.y * kT;
    const int nvalid = min(kT, out_c - base);
    if (threadIdx.x < nvalid) sd[threadIdx.x] = dyn[static_cast<int64_t>(p) * out_c + base + threadIdx.x];
    __syncthreads();
    if (threadIdx.x >= nvalid) return;
    const int ksq = ks * ks, pad = ks == stride ? 0 : (ks - 1) >> 1;
    const int hs = p / dout * stride - pad, ws0 = (p % dout) * stride - pad;
    for (int ic = threadIdx.x; ic < in_c; ic += kT) {
        for (int k = 0; k < ksq; ++k) {
            const int hi = hs + k / ks, wi = ws0 + k % ks;
            if (hi < 0 || hi >= din || wi < 0 || wi >= din) continue;
            float acc = 0.0f;
            for (int i = 0; i < nvalid; ++i)
                acc = fmaf(sd[i], master[((static_cast<int64_t>(base) + i) * ksq + k) * in_c + ic], acc);
            atomicAdd(&grad_in[(static_cast<int64_t>(hi) * din + wi) * in_c + ic], acc);
        }
    }
}

// Depthwise input gradient (kernels.h:871-910): one chain over the taps in
// order; written, not added.
__global__ void conv_bwd_dw_input_kernel(const float* __restrict__ go, const float* __restrict__ master, int C, int ks,
                                         int stride, int din, int dout, float* __restrict__ grad_in)
{
    const int64_t t = static_cast<int64_t>(blockIdx.x) * kT + threadIdx.x;
    if (t >= static_cast<int64_t>(din) * din * C) return;
    const int c = static_cast<int>(t % C);
    const int pin = static_cast<int>(t / C);
    const int hi = pin / din, wi = pin % din, pad = ks >> 1;
    float acc = 0.0f;
    for (int k = 0; k < ks * ks; ++k) {
        const int ht = hi - k / ks + pad, wt = wi - k % ks + pad;
        float g = 0.0f;
        if (ht % stride == 0 && wt % stride == 0) {
            const int ho = ht / stride, wo = wt / stride;
            if (ho >= 0 && ho < dout && wo >= 0 && wo < dout) g = go[(static_cast<int64_t>(ho) * dout + wo) * C + c];
        }
        acc = fmaf(g, master[static_cast<int64_t>(k) * C + c], acc);
    }
    grad_in[t] = acc;
}

// Depthwise weight gradient (kernels.h:911-960): per (tap, channel), input x
// output gradient summed over output positions in order. The reference runs
// whole 256-channel blocks and writes past the layer's channels when it has
// fewer than 256; only the layer's channels are computed here.
__global__ void conv_bwd_dw_weight_kernel(const uint32_t* __restrict__ in, const int8_t* __restrict__ in_s,
                                          const float* __restrict__ go, int C, int ks, int stride, int din, int dout,
                                          float* __restrict__ gw)
{
    const int64_t t = static_cast<int64_t>(blockIdx.x) * kT + threadIdx.x;
    const int ksq = ks * ks;
    if (t >= static_cast<int64_t>(ksq) * C) return;
    const int k = static_cast<int>(t / C), c = static_cast<int>(t % C), pad = ks >> 1;
    float acc = 0.0f;
    for (int p = 0; p < dout * dout; ++p) {
        const int hi = p / dout * stride - pad + k / ks, wi = (p % dout) * stride - pad + k % ks;
        const float g = go[static_cast<int64_t>(p) * C + c];
        if (hi >= 0 && hi < din && wi >= 0 && wi < din)
            acc = fmaf(deq(in, in_s, (static_cast<int64_t>(hi) * din + wi) * C + c), g, acc);
    }
    gw[t] = acc;
}

// Depthwise bias gradient (kernels.h:961-988): four chains over positions
// p = 4j + i, summed in order; positions must be a multiple of 4.
__global__ void conv_bwd_dw_bias_kernel(const float* __restrict__ go, int C, int positions, float* __restrict__ gb)
{
    const int c = blockIdx.x * kT + threadIdx.x;
    if (c >= C) return;
    float s[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int p = 0; p < positions; p += 4)
#pragma unroll
        for (int i = 0; i < 4; ++i) s[i] = __fadd_rn(s[i], go[static_cast<int64_t>(p + i) * C + c]);
    gb[c] = __fadd_rn(__fadd_rn(__fadd_rn(s[0], s[1]), s[2]), s[3]);
}

// residualAddBwdKernel (kernels.h:1056-1079): grad_res = grad_next, then
// grad_next *= survival_prob_inv * residual_factor.
__global__ void residual_bwd_kernel(float* __restrict__ gn, float* __restrict__ gr, int64_t n, float combined)
{
    const int64_t i = static_cast<int64_t>(blockIdx.x) * kT + threadIdx.x;
    if (i >= n) return;
    const float v = gn[i];
    gr[i] = v;
    gn[i] = __fmul_rn(v, combined);
}

// ---------------------------------------------------------------- SGD

// Per-block partial square sums of transformReduceKernel (uv.h:9-24): a
// grid-stride sum per thread, lane tree (shfl_down 16..1), warp-0 tree over
// the 8 warp sums (shfl_down 4..1). The reference adds the block results
// with atomics in arrival order; sumsq_final adds them in block order.
__global__ void __launch_bounds__(kT) sumsq_partial_kernel(const float* __restrict__ x, int64_t n,
                                                          float* __restrict__ partial)
{
    __shared__ float sw[8];
    float s = 0.0f;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * kT + threadIdx.x; i < n; i += static_cast<int64_t>(gridDim.x) * kT)
        s = fmaf(x[i], x[i], s);  // sum += x * x, contracted
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_down_sync(0xFFFFFFFFu, s, o));
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) sw[warp] = s;
    __syncthreads();
    if (warp == 0) {
        s = lane < 8 ? sw[lane] : 0.0f;
#pragma unroll
        for (int o = 4; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_down_sync(0xFFFFFFFFu, s, o));
        if (lane == 0) partial[blockIdx.x] = s;
    }
}

// Clip factor of the layer classes' clip_op (conv_layer.h:209-213): norm =
// sqrt(sum + epsilon), 1/norm above 1 (correctly rounded, as the host does).
__global__ void sumsq_final_kernel(const float* __restrict__ partial, int blocks, float* __restrict__ factor)
{
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    float s = 0.0f;  // the reference zeroes its device result, then adds each block's sum
    for (int b = 0; b < blocks; ++b) s = __fadd_rn(s, partial[b]);
    const float norm = __fsqrt_rn(__fadd_rn(s, kEps));
    factor[0] = norm > 1.0f ? __fdiv_rn(1.0f, norm) : 1.0f;
    factor[1] = s;
}

// updateParamsKernel (kernels.h:196-216): data = fma(g, -lr * f, data * (1 - lr
// * penalty)) over the first floor(n / 4) * 4 elements (whole uint4 only, as
// the reference's loop); f is read from the device.
__global__ void sgd_update_kernel(float* __restrict__ data, const float* __restrict__ grad, int64_t n,
                                  const float* __restrict__ factor, float lr, float penalty)
{
    const int64_t i = static_cast<int64_t>(blockIdx.x) * kT + threadIdx.x;
    if (i >= (n >> 2) << 2) return;
    const float c_grad = __fmul_rn(-lr, factor[0]);
    const float c_data = fmaf(-lr, penalty, 1.0f);
    data[i] = fmaf(grad[i], c_grad, __fmul_rn(data[i], c_data));
}

// ---------------------------------------------------------------- Mamba

struct MambaOffsets {
    int64_t c_re, c_im, a_re, a_im, d, w_out;
    __host__ __device__ MambaOffsets(int E, int N)
    {
        c_re = E + 32LL * E;
        c_im = c_re + static_cast<int64_t>(E) * N;
        a_re = c_im + static_cast<int64_t>(E) * N;
        a_im = a_re + static_cast<int64_t>(E) * N;
        d = a_im + static_cast<int64_t>(E) * N;
        w_out = d + E;
    }
};

// y_ssm of channel ch recomputed from the carried state (kernels.h:1277-1288).
// h: [E][P] complex (this sequence), P = N / 32, state c of channel ch is the
// reference's index ch * N + (ch & 31) + 32 c.
__device__ __forceinline__ float y_ssm_of(const uint32_t* __restrict__ in, const int8_t* __restrict__ in_s,
                                          const float2* __restrict__ h, const float* __restrict__ m, const MambaOffsets& o,
                                          int ch, int D, int N)
{
    const int ic = ch & (D - 1);
    float y = __fmul_rn(m[o.d + ch], deq(in, in_s, ic));
    const int P = N >> 5;
    const int64_t base = static_cast<int64_t>(ch) * N + (ch & 31);
    for (int c = 0; c < P; ++c) {
        const float2 hv = h[static_cast<int64_t>(ch) * P + c];
        y = fmaf(hv.x, m[o.c_re + base + 32 * c], y);
        y = fmaf(-hv.y, m[o.c_im + base + 32 * c], y);
    }
    return y;
}

// mambaSSMBwdOutProjKernel (kernels.h:1260-1302): raw[oc] = sum over 256-channel
// chunks (added in chunk order) of the chunk's 8 partial 32-channel sums,
// reduced as the reference does with absolute-lane shuffles: with s_l the
// partial of lane l of the 8-lane group and s_1, s_2, s_4 those of lanes
// 1, 2, 4 of the warp, lane 8 j ends with
//   ((s_8j + s_4) + (s_2 + s_4)) + ((s_1 + s_4) + (s_2 + s_4)).
// One warp per (32-output tile, chunk, warp of the chunk's block), as the
// reference's 256-thread blocks; chunk sums go to partial[chunk][oc].
__global__ void __launch_bounds__(kT) mamba_bwd_outproj_kernel(const uint32_t* __restrict__ in,
                                                              const int8_t* __restrict__ in_s,
                                                              const float2* __restrict__ h,
                                                              const float* __restrict__ m, int D, int N, int out_c,
                                                              float* __restrict__ partial)
{
    __shared__ float sy[8][33];
    const int E = 2 * D;
    const MambaOffsets o(E, N);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int chunk = blockIdx.y;
    const int ch = chunk * kT + warp * 32 + lane;
    sy[warp][lane] = y_ssm_of(in, in_s, h, m, o, ch, D, N);
    __syncthreads();
    const int oc = blockIdx.x * 32 + warp * 4 + (lane >> 3);
    const int v8 = lane & 7;
    const int64_t wb = o.w_out + static_cast<int64_t>(oc) * E + chunk * kT + v8 * 32;
    float s = 0.0f;
#pragma unroll 8
    for (int i = 0; i < 32; ++i) s = fmaf(sy[v8][i], m[wb + i], s);
#pragma unroll
    for (int off = 4; off > 0; off >>= 1) s = __fadd_rn(s, __shfl_sync(0xFFFFFFFFu, s, off));
    if (v8 == 0) partial[static_cast<int64_t>(chunk) * out_c + oc] = s;
}

// mambaSSMBwdNormActKernel (kernels.h:1303-1336) with the out-projection's
// chunk sums added in chunk order first (the reference's zeroed buffer plus
// one atomic add per chunk): raw -> gact (grad_bias) and gnorm = gact * inv.
__global__ void __launch_bounds__(kT) mamba_bwd_normact_kernel(const float* __restrict__ partial, int chunks,
                                                              const float* __restrict__ bias,
                                                              const float* __restrict__ dy, int out_c, int act,
                                                              float* __restrict__ gb, float* __restrict__ gnorm)
{
    __shared__ float smem8[9];
    const int oc = blockIdx.x * kT + threadIdx.x;
    const bool valid = oc < out_c;
    float raw = 0.0f;
    if (valid)
        for (int c = 0; c < chunks; ++c) raw = __fadd_rn(raw, partial[static_cast<int64_t>(c) * out_c + oc]);
    const float tot = block_sq256(valid ? raw : 0.0f, smem8);
    if (!valid) return;
    const float inv = out_c < 2 ? 1.0f : __frsqrt_rn(fmaf(tot, __frcp_rn(static_cast<float>(min(out_c, kT))), kEps));
    const float u = fmaf(raw, inv, bias[oc]);
    const float d = dy[oc];
    const float ga = act == 0 ? d : act == 1 ? silu_grad_f(u, d) : sigmoid_grad_f(u, d);
    gb[oc] = ga;
    gnorm[oc] = __fmul_rn(ga, inv);
}

// mambaSSMApplyTracesKernel (kernels.h:1337-1419): one thread per channel.
// grad_w must be zeroed: the reference adds each of its atomic contributions
// to a zero (one per element), so those are formed as 0 + x here (a -0 reads
// +0); the W_out gradient is a plain store. ta/tb/td: the sequence's traces
// [E][P] complex; gx_ch gets the input-gradient term of every channel.
__global__ void __launch_bounds__(kT) mamba_bwd_traces_kernel(const uint32_t* __restrict__ in,
                                                             const int8_t* __restrict__ in_s,
                                                             const float* __restrict__ gnorm,
                                                             const float2* __restrict__ h,
                                                             const float2* __restrict__ ta_, const float2* __restrict__ tb_,
                                                             const float2* __restrict__ td_, const float* __restrict__ m,
                                                             int D, int N, int out_c, float* __restrict__ gw,
                                                             float* __restrict__ gx_ch)
{
    const int E = 2 * D, P = N >> 5;
    const MambaOffsets o(E, N);
    const int lane = threadIdx.x & 31;
    const int ch = blockIdx.x * kT + threadIdx.x;
    const int block_ch = ch & ~31;
    const int ic = ch & (D - 1);
    const float d_skip = m[o.d + ch], w_delta = m[ch];
    const float x = deq(in, in_s, ic);
    const float y = y_ssm_of(in, in_s, h, m, o, ch, D, N);
    float gy = 0.0f;
    for (int oc = 0; oc < out_c; ++oc) {
        const float g = gnorm[oc];
        const int64_t wi = o.w_out + static_cast<int64_t>(oc) * E + ch;
        gw[wi] = __fmul_rn(g, y);
        gy = fmaf(g, m[wi], gy);
    }
    const int64_t mimo_base = E + static_cast<int64_t>(block_ch >> 5) * 1024;
    const int64_t base = static_cast<int64_t>(ch) * N + lane;
    float g_dt = 0.0f, g_b = 0.0f;
    for (int c = 0; c < P; ++c) {
        const int64_t idx = base + 32 * c, sidx = static_cast<int64_t>(ch) * P + c;
        const float wre = m[o.c_re + idx], wim = m[o.c_im + idx];
        const float2 hv = h[sidx], ta = ta_[sidx], tb = tb_[sidx], td = td_[sidx];
        const float ghr = __fmul_rn(gy, wre), ghi = __fmul_rn(-gy, wim);
        gw[o.c_re + idx] = __fadd_rn(0.0f, __fmul_rn(gy, hv.x));
        gw[o.c_im + idx] = __fadd_rn(0.0f, __fmul_rn(-gy, hv.y));
        gw[o.a_re + idx] = __fadd_rn(0.0f, fmaf(ghr, ta.x, __fmul_rn(ghi, ta.y)));
        gw[o.a_im + idx] = __fadd_rn(0.0f, fmaf(ghi, ta.x, __fmul_rn(-ghr, ta.y)));
        g_b = fmaf(ghr, tb.x, fmaf(ghi, tb.y, g_b));
        g_dt = fmaf(ghr, td.x, fmaf(ghi, td.y, g_dt));
    }
    float gxb[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int k = 0; k < 32; ++k) {
        const int src = (block_ch + k) & (D - 1);
        const float bval = m[mimo_base + lane + 32 * k];
        gw[mimo_base + lane * 32 + k] = __fadd_rn(0.0f, __fmul_rn(g_b, deq(in, in_s, src)));
        gxb[k & 3] = fmaf(__shfl_sync(0xFFFFFFFFu, g_b, k), bval, gxb[k & 3]);
    }
    const float g_xb = __fadd_rn(__fadd_rn(__fadd_rn(gxb[0], gxb[1]), gxb[2]), gxb[3]);
    const float g_pre = __fmul_rn(g_dt, sigmoid_f(__fmul_rn(x, w_delta)));
    gw[ch] = __fadd_rn(0.0f, __fmul_rn(g_pre, x));
    gw[o.d + ch] = __fadd_rn(0.0f, __fmul_rn(gy, x));
    gx_ch[ch] = fmaf(g_pre, w_delta, fmaf(gy, d_skip, g_xb));
}

// The layer's input gradient: the reference zeroes it, then channels ch and
// ch + D add their terms (two additions to a zero commute).
__global__ void mamba_bwd_input_kernel(const float* __restrict__ gx_ch, int D, float* __restrict__ grad_in)
{
    const int ic = blockIdx.x * kT + threadIdx.x;
    if (ic >= D) return;
    grad_in[ic] = __fadd_rn(__fadd_rn(0.0f, gx_ch[ic]), gx_ch[ic + D]);
}

// ---------------------------------------------------------------- critic

// criticApplyTracesKernel + criticOutputGradKernel (kernels.h:1779-1805).
__global__ void critic_bwd_kernel(const float* __restrict__ w2, const float2* __restrict__ tw1,
                                  const float2* __restrict__ tl, const float2* __restrict__ hidden,
                                  const float* __restrict__ pred, float real, int units, int in_c, float* __restrict__ gw1, float* __restrict__ gl,
                                  float* __restrict__ gw2)
{
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * kT + threadIdx.x;
    const float go = __fsub_rn(pred[0], real);
    if (idx < units) {
        const float2 hs = hidden[idx];
        gw2[2 * idx] = __fmul_rn(go, hs.x);
        gw2[2 * idx + 1] = __fmul_rn(go, hs.y);
    }
    if (idx >= static_cast<int64_t>(units) * in_c) return;
    const float2 a = tw1[idx], l = tl[idx];
    const int node = static_cast<int>(idx & (units - 1)) << 1;
    const int lam = static_cast<int>(idx / in_c) << 1;
    gw1[2 * idx] = __fmul_rn(__fmul_rn(go, w2[node]), a.x);
    gw1[2 * idx + 1] = __fmul_rn(__fmul_rn(go, w2[node + 1]), a.y);
    gl[2 * idx] = __fmul_rn(__fmul_rn(go, w2[lam]), l.x);
    gl[2 * idx + 1] = __fmul_rn(__fmul_rn(go, w2[lam + 1]), l.y);
}

unsigned blocks_for(int64_t n) { return static_cast<unsigned>((n + kT - 1) / kT); }

}  // namespace

// ------------------------------------------------------------------ launchers

int sumsq_blocks(int64_t n, int sms)
{
    const int64_t b = (n + kT - 1) / kT, cap = static_cast<int64_t>(sms) * 8;  // uv.h:44-60, 2048 / 256 per SM
    return static_cast<int>(b < 1 ? 1 : b > cap ? cap : b);
}

cudaError_t launch_clip_factor(const float* x, int64_t n, int sms, float* partial, float* factor, cudaStream_t s)
{
    const int blocks = sumsq_blocks(n, sms);
    sumsq_partial_kernel<<<blocks, kT, 0, s>>>(x, n, partial);
    sumsq_final_kernel<<<1, 32, 0, s>>>(partial, blocks, factor);
    return cudaGetLastError();
}

cudaError_t launch_sgd_update(float* data, const float* grad, int64_t n, const float* factor, float lr, float penalty,
                              cudaStream_t s)
{
    if (n >= 4) sgd_update_kernel<<<blocks_for((n >> 2) << 2), kT, 0, s>>>(data, grad, n, factor, lr, penalty);
    return cudaGetLastError();
}

cudaError_t launch_conv_backward_grads(const uint32_t* in, const int8_t* in_s, const uint32_t* w, const int8_t* w_s,
                                       const float* bias, const float* master, const float* dy, int in_c, int out_c,
                                       int ks, int stride, int din, int dout, bool act, float* scratch, float* gw,
                                       float* gb, float* grad_in, cudaStream_t s)
{
    const int positions = dout * dout;
    const bool dw = ks > 1 && (ks & 1);
    if (dw) {
        // the depthwise conv has no norm and no activation: dy is the gradient
        conv_bwd_dw_bias_kernel<<<blocks_for(in_c), kT, 0, s>>>(dy, in_c, positions, gb);
        conv_bwd_dw_weight_kernel<<<blocks_for(static_cast<int64_t>(ks) * ks * in_c), kT, 0, s>>>(
            in, in_s, dy, in_c, ks, stride, din, dout, gw);
        if (grad_in)
            conv_bwd_dw_input_kernel<<<blocks_for(static_cast<int64_t>(din) * din * in_c), kT, 0, s>>>(
                dy, master, in_c, ks, stride, din, dout, grad_in);
        return cudaGetLastError();
    }
    // scratch: 4 planes [positions][out] fp32 (conv_backward_scratch_floats)
    const int64_t plane = static_cast<int64_t>(positions) * out_c;
    float *gsa = scratch, *gst = scratch + plane, *dyn = scratch + 2 * plane, *facc = scratch + 3 * plane;
    dim3 grid(positions, (out_c + kT - 1) / kT);
    conv_bwd_recompute_kernel<<<grid, kT, 0, s>>>(in, in_s, w, w_s, bias, dy, in_c, out_c, ks, stride, din, dout,
                                                  act ? 1 : 0, gsa, gst, dyn, facc);
    conv_bwd_bias_kernel<<<blocks_for(out_c), kT, 0, s>>>(gsa, gst, positions, out_c, act ? 1 : 0, gb);
    if (ks == 1) {
        // dynw reuses gsa's plane: the bias gradient has consumed it
        conv_bwd_pw_dynw_kernel<<<blocks_for(static_cast<int64_t>(positions / 8) * (out_c / 32) * 32), kT, 0, s>>>(
            facc, dy, bias, positions, out_c, act ? 1 : 0, gsa);
        conv_bwd_pw_weight_kernel<<<blocks_for(static_cast<int64_t>(out_c) * in_c), kT, 0, s>>>(
            in, in_s, gsa, positions, in_c, out_c, gw);
        if (grad_in) conv_bwd_pw_input_kernel<<<grid, kT, 0, s>>>(dyn, master, in_c, out_c, grad_in);
    } else {
        conv_bwd_dense_weight_kernel<<<blocks_for(static_cast<int64_t>(out_c) * in_c), kT, 0, s>>>(
            in, in_s, dyn, in_c, out_c, ks, stride, din, dout, gw);
        if (grad_in)
            conv_bwd_dense_input_kernel<<<grid, kT, 0, s>>>(dyn, master, in_c, out_c, ks, stride, din, dout, grad_in);
    }
    return cudaGetLastError();
}

cudaError_t launch_residual_backward(float* grad_next, float* grad_res, int64_t n, float survival_inv,
                                     float residual_factor, cudaStream_t s)
{
    if (n == 0) return cudaSuccess;
    residual_bwd_kernel<<<blocks_for(n), kT, 0, s>>>(grad_next, grad_res, n, survival_inv * residual_factor);  // host IEEE product, as the kernel forms it
    return cudaGetLastError();
}

cudaError_t launch_mamba_backward_grads(const uint32_t* in, const int8_t* in_s, const float2* h, const float2* ta,
                                        const float2* tb, const float2* td, const float* master, const float* bias,
                                        const float* dy, int D, int N, int out_c, int act, float* partial,
                                        float* gnorm, float* gx_ch, float* gw, float* gb, float* grad_in,
                                        cudaStream_t s)
{
    const int E = 2 * D, chunks = E / kT;
    cudaError_t e = cudaMemsetAsync(gw, 0, sizeof(float) * MambaOffsets(E, N).w_out, s);  // every atomic target
    if (e != cudaSuccess) return e;
    mamba_bwd_outproj_kernel<<<dim3(out_c / 32, chunks), kT, 0, s>>>(in, in_s, h, master, D, N, out_c, partial);
    mamba_bwd_normact_kernel<<<blocks_for(out_c), kT, 0, s>>>(partial, chunks, bias, dy, out_c, act, gb, gnorm);
    mamba_bwd_traces_kernel<<<E / kT, kT, 0, s>>>(in, in_s, gnorm, h, ta, tb, td, master, D, N, out_c, gw, gx_ch);
    mamba_bwd_input_kernel<<<blocks_for(D), kT, 0, s>>>(gx_ch, D, grad_in);
    return cudaGetLastError();
}

cudaError_t launch_critic_backward_grads(const float* w2, const float2* tw1, const float2* tl, const float2* hidden,
                                         const float* pred, float real, int units, int in_c, float* gw1, float* gl, float* gw2,
                                         cudaStream_t s)
{
    const int64_t n = static_cast<int64_t>(units) * in_c;
    critic_bwd_kernel<<<blocks_for(n > units ? n : units), kT, 0, s>>>(w2, tw1, tl, hidden, pred, real, units, in_c, gw1,
                                                                       gl, gw2);
    return cudaGetLastError();
}

}  // namespace aic
