// Mamba-layer kernels: the batched, time-looped complex-diagonal SSM scan (A9)
// and the out-projection GEMM with its fused RMSNorm + bias + activation (A10).
//
// Semantics follow AICortex kernels.h:1080-1259: channel ch of d_inner = 2*D
// reads input channel ch & (D-1), uses MIMO row (ch & 31) of block ch >> 5,
// and owns the P = d_state/32 states n = (ch & 31) + 32c of its row. The
// reference advances one step per launch; here a channel's states stay in
// registers (of one thread, or of several lanes when the batch is small) for
// all T steps of a sequence, which is the same recurrence because a layer's
// input at step t does not depend on that layer's own state.
#include <cuda_bf16.h>

#include "aic_common.cuh"
#include "aic_kernels.h"

namespace aic {
namespace {

constexpr int kScanThreads = 64;
constexpr int kThreads = 256;

struct BlobLayout {  // element offsets of the packed weight blob (mamba_layer.h:58)
    int64_t E, N, offB, offCre, offCim, offAre, offAim, offD, offW;
    __host__ __device__ BlobLayout(int D, int d_state)
    {
        E = 2LL * D; N = d_state;
        offB = E; offCre = 33 * E; offCim = offCre + E * N; offAre = offCim + E * N;
        offAim = offAre + E * N; offD = offAim + E * N; offW = offD + E;
    }
};

__device__ __forceinline__ float blob_value(const uint32_t* blob, const int8_t* blob_s, int64_t i)
{
    return static_cast<float>(code_of(blob[i >> 3], static_cast<int>(i & 7))) * unit_of(blob_s[i >> 5]);
}

// Per-channel constants, computed once per weight load instead of per step:
// consts4[ch][c] = {-exp(A_re), A_im, C_re, C_im}; consts2[ch] = {W_delta, D}.
__global__ void __launch_bounds__(kThreads) ssm_prepare_kernel(const uint32_t* __restrict__ blob, const int8_t* __restrict__ blob_s,
                                                             int D, int d_state, float4* __restrict__ consts4,
                                                             float2* __restrict__ consts2)
{
    const BlobLayout L(D, d_state);
    const int P = d_state >> 5;
    const int64_t t = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
    if (t >= L.E * P) return;
    const int ch = static_cast<int>(t / P), c = static_cast<int>(t % P);
    const int64_t off = static_cast<int64_t>(ch) * L.N + (ch & 31) + (c << 5);
    consts4[t] = make_float4(-__expf(blob_value(blob, blob_s, L.offAre + off)), blob_value(blob, blob_s, L.offAim + off),
                             blob_value(blob, blob_s, L.offCre + off), blob_value(blob, blob_s, L.offCim + off));
    if (c == 0) consts2[ch] = make_float2(blob_value(blob, blob_s, ch), blob_value(blob, blob_s, L.offD + ch));
}

// Runs step(t, words, unit) for t = 0..T-1 over one channel's input group
// (words at xv[t * Gx], exponent at xsv[t * Gx]) with the loads of step
// t + PF issued when step t starts: a register ring of PF steps hides the
// global-memory latency behind the serial recurrence.
template <int PF, class Step>
__device__ __forceinline__ void scan_steps(const uint4* __restrict__ xv, const int8_t* __restrict__ xsv, int Gx, int T,
                                           Step& step)
{
    uint4 rw[PF];
    int8_t rs[PF];
#pragma unroll
    for (int j = 0; j < PF; ++j) {
        if (j < T) {
            rw[j] = xv[static_cast<int64_t>(j) * Gx];
            rs[j] = xsv[static_cast<int64_t>(j) * Gx];
        }
    }
    for (int t0 = 0; t0 < T; t0 += PF) {
#pragma unroll
        for (int j = 0; j < PF; ++j) {
            const int t = t0 + j;
            if (t < T) {
                const uint4 xw = rw[j];
                const float xu = unit_of(rs[j]);
                if (t + PF < T) {
                    rw[j] = xv[static_cast<int64_t>(t + PF) * Gx];
                    rs[j] = xsv[static_cast<int64_t>(t + PF) * Gx];
                }
                step(t, xw, xu);
            }
        }
    }
}

// Input steps in flight per thread: threads with few states per step need a
// deeper ring to cover the load latency.
template <int S>
__host__ __device__ constexpr int scan_prefetch() { return S >= 16 ? 2 : (S >= 8 ? 4 : 8); }

// The batched, time-looped scan. Channel ch's P = S * L states are spread over
// L consecutive lanes, S states each (L = 1: one thread per channel; L > 1
// where batch x channels alone cannot fill the GPU). Every lane of a channel
// recomputes the step's channel terms (x, Bx, dt) and advances its S states;
// y = sum_c Re(h_c C_c) is folded in the reference's order c = 0, 1, ... by
// passing the partial sum from lane to lane with shuffles, so every L gives
// the same bits. The reciprocal is rcp_rn_pos, bit-identical to __frcp_rn for
// the operand |1 - dt A / 2|^2 + eps >= eps.
// TRACE: the training-mode forward also advances the eligibility traces
// trace_A, trace_B, trace_Delta (kernels.h:1158-1170), held in registers like
// the state; tr is [3][B][E][P] complex, the layout of h.
// SPLIT: y is written as two bf16 planes [B*T][E], hi = bf16(y) then
// lo = bf16(y - hi), the operands of the tensor-core out-projection;
// otherwise as fp32 [B*T][E].
template <int S, int L, bool TRACE, bool SPLIT>
__global__ void __launch_bounds__(kScanThreads) ssm_scan_kernel(const uint32_t* __restrict__ x, const int8_t* __restrict__ x_s,
                                                              const uint32_t* __restrict__ blob, const int8_t* __restrict__ blob_s,
                                                              const float4* __restrict__ consts4, const float2* __restrict__ consts2,
                                                              int D, float2* __restrict__ h, float2* __restrict__ tr,
                                                              void* __restrict__ y_out, int T)
{
    static_assert(L >= 1 && L <= 32 && (L & (L - 1)) == 0, "lanes per channel");
    constexpr int P = S * L;
    const int E = 2 * D;
    const int gt = blockIdx.x * kScanThreads + threadIdx.x;
    const int ch = gt / L, j = gt & (L - 1);  // channel and this lane's index within it
    const int b = blockIdx.y;
    const int lane = ch & 31, in_ch = ch & (D - 1);
    const int gbase = (threadIdx.x & 31) & ~(L - 1);
    float4 k[S];
#pragma unroll
    for (int i = 0; i < S; ++i) k[i] = consts4[static_cast<int64_t>(ch) * P + j * S + i];
    const float2 wdd = consts2[ch];
    const int64_t brow = E + static_cast<int64_t>(ch >> 5) * 1024 + lane * 32;
    const uint4 bw = reinterpret_cast<const uint4*>(blob)[brow >> 5];
    const float bu = unit_of(blob_s[brow >> 5]);
    float2 st[S];
    float2* hs = h + (static_cast<int64_t>(b) * E + ch) * P + j * S;
#pragma unroll
    for (int i = 0; i < S; ++i) st[i] = hs[i];
    float2 ta[TRACE ? S : 1], tb[TRACE ? S : 1], td[TRACE ? S : 1];
    float2* trs = TRACE ? tr + (static_cast<int64_t>(b) * E + ch) * P + j * S : nullptr;
    const int64_t tr_stride = static_cast<int64_t>(gridDim.y) * E * P;  // one trace of the whole batch
    if (TRACE) {
#pragma unroll
        for (int i = 0; i < S; ++i) {
            ta[i] = trs[i];
            tb[i] = trs[tr_stride + i];
            td[i] = trs[2 * tr_stride + i];
        }
    }
    const int Gx = D >> 5, xg = in_ch >> 5, xword = (in_ch & 31) >> 3, xnib = in_ch & 7;
    const uint4* xv = reinterpret_cast<const uint4*>(x) + static_cast<int64_t>(b) * T * Gx + xg;
    const int8_t* xsv = x_s + static_cast<int64_t>(b) * T * Gx + xg;
    const int64_t yoff = static_cast<int64_t>(b) * T * E + ch;
    float* yv = static_cast<float*>(y_out) + yoff;
    __nv_bfloat16* yh = static_cast<__nv_bfloat16*>(y_out) + yoff;
    const int64_t lo_plane = static_cast<int64_t>(gridDim.y) * T * E;
    auto step = [&](int t, uint4 xw, float xu) {
        const int dot = dot8(xw.x, bw.x) + dot8(xw.y, bw.y) + dot8(xw.z, bw.z) + dot8(xw.w, bw.w);
        const uint32_t xsel = xword == 0 ? xw.x : (xword == 1 ? xw.y : (xword == 2 ? xw.z : xw.w));
        const float x_local = static_cast<float>(code_of(xsel, xnib)) * xu;
        const float bx = static_cast<float>(dot) * (xu * bu);
        const float u = x_local * wdd.x;
        const float dt = u + __logf(1.0f + __expf(-fabsf(u)));
        const float dt_half = dt * 0.5f;
        float ya[S];
#pragma unroll
        for (int i = 0; i < S; ++i) {
            const float are = k[i].x, aim = k[i].y;
            const float dim = -dt_half * aim;
            const float dre = fmaf(-dt_half, are, 1.0f);
            const float inv_s = rcp_rn_pos(fmaf(dre, dre, fmaf(dim, dim, kEps)));
            const float ire = dre * inv_s;
            const float iim = -dim * inv_s;
            const float nre = fmaf(dt_half, are, 1.0f);
            const float abr = fmaf(nre, ire, dim * iim);
            const float abi = fmaf(nre, iim, -dim * ire);
            const float dtbx = dt * bx;
            const float hr = st[i].x, hi = st[i].y;
            st[i] = make_float2(fmaf(abr, hr, fmaf(-abi, hi, dtbx * ire)), fmaf(abr, hi, fmaf(abi, hr, dtbx * iim)));
            if (TRACE) {  // kernels.h:1158-1170, from the state before the step
                const float i2_re = fmaf(ire, ire, -iim * iim);
                const float i2_im = 2.0f * ire * iim;
                const float za_re = fmaf(dt_half, bx, hr);
                const float dt_i2_za_re = dt * fmaf(i2_re, za_re, -i2_im * hi);
                const float dt_i2_za_im = dt * fmaf(i2_re, hi, i2_im * za_re);
                const float zdt_re = fmaf(are, hr, fmaf(-aim, hi, bx));
                const float zdt_im = fmaf(are, hi, aim * hr);
                const float d_dt_re = fmaf(i2_re, zdt_re, -i2_im * zdt_im);
                const float d_dt_im = fmaf(i2_re, zdt_im, i2_im * zdt_re);
                ta[i] = make_float2(fmaf(abr, ta[i].x, fmaf(-abi, ta[i].y, dt_i2_za_re)),
                                    fmaf(abr, ta[i].y, fmaf(abi, ta[i].x, dt_i2_za_im)));
                tb[i] = make_float2(fmaf(abr, tb[i].x, fmaf(-abi, tb[i].y, dt * ire)),
                                    fmaf(abr, tb[i].y, fmaf(abi, tb[i].x, dt * iim)));
                td[i] = make_float2(fmaf(abr, td[i].x, fmaf(-abi, td[i].y, d_dt_re)),
                                    fmaf(abr, td[i].y, fmaf(abi, td[i].x, d_dt_im)));
            }
            ya[i] = fmaf(st[i].x, k[i].z, -st[i].y * k[i].w);
        }
        // y: 0 + ya_0 + ya_1 + ... in state order across the channel's lanes
        float ys = 0.0f;
#pragma unroll
        for (int q = 0; q < L; ++q) {
            if (j == q) {
#pragma unroll
                for (int i = 0; i < S; ++i) ys += ya[i];
            }
            if (L > 1) ys = __shfl_sync(0xFFFFFFFFu, ys, gbase + q);
        }
        if (j == 0) {
            const float yt = fmaf(wdd.y, x_local, ys);
            if (SPLIT) {
                const __nv_bfloat16 hb = __float2bfloat16_rn(yt);
                yh[static_cast<int64_t>(t) * E] = hb;
                yh[lo_plane + static_cast<int64_t>(t) * E] = __float2bfloat16_rn(yt - __bfloat162float(hb));
            } else {
                yv[static_cast<int64_t>(t) * E] = yt;
            }
        }
    };
    scan_steps<scan_prefetch<S>()>(xv, xsv, Gx, T, step);
#pragma unroll
    for (int i = 0; i < S; ++i) hs[i] = st[i];
    if (TRACE) {
#pragma unroll
        for (int i = 0; i < S; ++i) {
            trs[i] = ta[i];
            trs[tr_stride + i] = tb[i];
            trs[2 * tr_stride + i] = td[i];
        }
    }
}

// Out-projection on CUDA cores. A CTA owns R rows and one 256-channel chunk
// (thread = output channel). The y rows are staged 128 channels at a time;
// each weight group is expanded to 32 float codes once and applied to all R
// rows. Per (row, channel) the order is the reference's: four interleaved
// partial sums per 32-group, folded and scaled per group in channel order.
template <int R>
__global__ void __launch_bounds__(kThreads) outproj_kernel(const float* __restrict__ y, const uint32_t* __restrict__ blob,
                                                         const int8_t* __restrict__ blob_s, const float* __restrict__ bias,
                                                         int D, int d_state, int out, int act, int64_t rows,
                                                         float* __restrict__ o)
{
    __shared__ __align__(16) float ys[R][128];
    __shared__ float part[R][kThreads / 32];
    __shared__ float total_sq[R];
    const BlobLayout L(D, d_state);
    const int E = static_cast<int>(L.E);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int oc = blockIdx.y * kThreads + threadIdx.x;
    const bool active = oc < out;
    const int64_t row0 = static_cast<int64_t>(blockIdx.x) * R;
    float acc[R];
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = 0.0f;
    const int64_t wbase = L.offW + static_cast<int64_t>(active ? oc : 0) * E;
    for (int ic0 = 0; ic0 < E; ic0 += 128) {
        __syncthreads();
        for (int i = threadIdx.x; i < R * 32; i += kThreads) {
            const int r = i >> 5, q = i & 31;
            const int64_t row = row0 + r;
            float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (row < rows && ic0 + 4 * q < E) v = reinterpret_cast<const float4*>(y + row * E + ic0)[q];
            reinterpret_cast<float4*>(&ys[r][0])[q] = v;
        }
        __syncthreads();
        if (!active) continue;
#pragma unroll 1
        for (int g = 0; g < 4; ++g) {
            const int ic = ic0 + (g << 5);
            if (ic >= E) break;
            const uint4 wv = reinterpret_cast<const uint4*>(blob)[(wbase + ic) >> 5];
            const float wu = unit_of(blob_s[(wbase + ic) >> 5]);
            const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
            float cf[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) cf[i] = static_cast<float>(code_of(ww[i >> 3], i & 7));
#pragma unroll
            for (int r = 0; r < R; ++r) {
                float gs[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
                for (int i = 0; i < 32; ++i) gs[i & 3] = fmaf(ys[r][(g << 5) + i], cf[i], gs[i & 3]);
                acc[r] = fmaf(gs[0] + gs[1] + gs[2] + gs[3], wu, acc[r]);
            }
        }
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
        float sq = active ? acc[r] * acc[r] : 0.0f;
#pragma unroll
        for (int s = 16; s > 0; s >>= 1) sq += __shfl_xor_sync(0xFFFFFFFFu, sq, s);
        if (lane == 0) part[r][warp] = sq;
    }
    __syncthreads();
    for (int r = warp; r < R; r += kThreads / 32) {
        float s = lane < kThreads / 32 ? part[r][lane] : 0.0f;
#pragma unroll
        for (int q = (kThreads / 32) >> 1; q > 0; q >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, q);
        if (lane == 0) total_sq[r] = s;
    }
    __syncthreads();
    if (!active) return;
    const float inv_div = __frcp_rn(static_cast<float>(min(out, kNormChunk)));
    const float b = bias[oc];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int64_t row = row0 + r;
        if (row >= rows) break;
        const float inv_rms = out < 2 ? 1.0f : __frsqrt_rn(fmaf(total_sq[r], inv_div, kEps));
        float v = fmaf(acc[r], inv_rms, b);
        if (act == 1) v = silu_f(v);
        else if (act == 2) v = sigmoid_f(v);
        o[row * out + oc] = v;
    }
}

// Lanes per channel: the smallest L (a power of two, at most P) that gives the
// scan 16 warps per SM, since each lane's S = P / L states are a serial
// recurrence over T; L = 1 when batch x channels already fills the GPU.
int scan_lanes(int64_t channels, int P)
{
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t want = static_cast<int64_t>(sms) * 512;
    int L = 1;
    while (L < P && channels * L < want) L <<= 1;
    return L;
}

template <int S, int L>
cudaError_t launch_scan_sl(const uint32_t* x, const int8_t* x_s, const uint32_t* blob, const int8_t* blob_s,
                           const float4* c4, const float2* c2, int D, float2* h, float2* traces, void* y, bool split,
                           int B, int T, cudaStream_t stream)
{
    const dim3 grid(static_cast<unsigned>(2LL * D * L / kScanThreads), static_cast<unsigned>(B));
    if (traces)
        ssm_scan_kernel<S, L, true, false><<<grid, kScanThreads, 0, stream>>>(x, x_s, blob, blob_s, c4, c2, D, h, traces, y, T);
    else if (split)
        ssm_scan_kernel<S, L, false, true><<<grid, kScanThreads, 0, stream>>>(x, x_s, blob, blob_s, c4, c2, D, h, nullptr, y, T);
    else
        ssm_scan_kernel<S, L, false, false><<<grid, kScanThreads, 0, stream>>>(x, x_s, blob, blob_s, c4, c2, D, h, nullptr, y, T);
    return cudaGetLastError();
}

// P states per channel over L lanes: S = P / L.
template <int P>
cudaError_t launch_scan_p(int L, const uint32_t* x, const int8_t* x_s, const uint32_t* blob, const int8_t* blob_s,
                          const float4* c4, const float2* c2, int D, float2* h, float2* traces, void* y, bool split, int B,
                          int T, cudaStream_t stream)
{
#define AIC_SCAN_L(LL)                                                                                          \
    if (L == LL) {                                                                                              \
        if constexpr (P % LL == 0)                                                                              \
            return launch_scan_sl<P / LL, LL>(x, x_s, blob, blob_s, c4, c2, D, h, traces, y, split, B, T, stream); \
    }
    AIC_SCAN_L(1)
    AIC_SCAN_L(2)
    AIC_SCAN_L(4)
    AIC_SCAN_L(8)
    AIC_SCAN_L(16)
#undef AIC_SCAN_L
    return cudaErrorInvalidValue;
}

}  // namespace

size_t ssm_consts_floats(int D, int d_state)
{
    const size_t E = 2 * static_cast<size_t>(D), P = static_cast<size_t>(d_state) >> 5;
    return E * P * 4 + E * 2;
}

cudaError_t launch_ssm_prepare(const uint32_t* blob, const int8_t* blob_s, int D, int d_state, float* consts,
                               cudaStream_t stream)
{
    const int64_t E = 2LL * D, P = d_state >> 5;
    float4* c4 = reinterpret_cast<float4*>(consts);
    float2* c2 = reinterpret_cast<float2*>(consts + E * P * 4);
    const unsigned grid = static_cast<unsigned>((E * P + kThreads - 1) / kThreads);
    ssm_prepare_kernel<<<grid, kThreads, 0, stream>>>(blob, blob_s, D, d_state, c4, c2);
    return cudaGetLastError();
}

cudaError_t launch_ssm_scan(const uint32_t* x, const int8_t* x_s, const uint32_t* blob, const int8_t* blob_s,
                            const float* consts, int D, int d_state, float2* h, float2* traces, void* y, bool split,
                            int B, int T, cudaStream_t stream)
{
    if (B == 0 || T == 0) return cudaSuccess;
    const int64_t E = 2LL * D;
    const int P = d_state >> 5;
    const float4* c4 = reinterpret_cast<const float4*>(consts);
    const float2* c2 = reinterpret_cast<const float2*>(consts + E * P * 4);
    const int L = scan_lanes(static_cast<int64_t>(B) * E, P);
    switch (P) {
        case 1: return launch_scan_p<1>(L, x, x_s, blob, blob_s, c4, c2, D, h, traces, y, split, B, T, stream);
        case 2: return launch_scan_p<2>(L, x, x_s, blob, blob_s, c4, c2, D, h, traces, y, split, B, T, stream);
        case 4: return launch_scan_p<4>(L, x, x_s, blob, blob_s, c4, c2, D, h, traces, y, split, B, T, stream);
        case 8: return launch_scan_p<8>(L, x, x_s, blob, blob_s, c4, c2, D, h, traces, y, split, B, T, stream);
        case 16: return launch_scan_p<16>(L, x, x_s, blob, blob_s, c4, c2, D, h, traces, y, split, B, T, stream);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_outproj(const float* y, const uint32_t* blob, const int8_t* blob_s, const float* bias, int D,
                           int d_state, int out, int act, int64_t rows, float* o, cudaStream_t stream)
{
    if (rows == 0) return cudaSuccess;
    constexpr int R = 16;
    dim3 grid(static_cast<unsigned>((rows + R - 1) / R), static_cast<unsigned>((out + kThreads - 1) / kThreads));
    outproj_kernel<R><<<grid, kThreads, 0, stream>>>(y, blob, blob_s, bias, D, d_state, out, act, rows, o);
    return cudaGetLastError();
}

}  // namespace aic
