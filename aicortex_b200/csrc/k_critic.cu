// Critic head (A13): the gated leaky complex recurrent cell and its scalar
// read-out (AICortex kernels.h:1685-1778, critic.h:106-116), batched over
// sequences and looped over time. One warp per (sequence, unit) keeps the
// unit's complex state in registers across all steps and writes it per step;
// a second kernel reduces the per-step states to the score with the
// reference's shuffle-down tree.
#include "aic_common.cuh"
#include "aic_kernels.h"

namespace aic {
namespace {

constexpr int kThreads = 256;

// NI = in/32 inputs per lane whose weights stay in registers across all steps
// (0: any `in`, weights re-read from global memory every step).
// TRACE: the training-mode forward also advances the eligibility traces of w1
// and w_lambda (kernels.h:1731-1751), one set per sequence: tw [B][in][units]
// and tl [B][units][in] complex (the layouts of w1 and wl).
template <int NI, bool TRACE>
__global__ void __launch_bounds__(kThreads) critic_cell_kernel(const __half* __restrict__ x, const float* __restrict__ w1,
                                                             const float* __restrict__ wl, int in, int units,
                                                             float2* __restrict__ h, float2* __restrict__ h_seq,
                                                             float2* __restrict__ tw, float2* __restrict__ tl, int T)
{
    const int lane = threadIdx.x & 31;
    const int j = blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5);
    const int b = blockIdx.y;
    if (j >= units) return;
    float2 w1r[NI > 0 ? NI : 1], wlr[NI > 0 ? NI : 1];
#pragma unroll
    for (int i = 0; i < NI; ++i) {
        const int c = lane + 32 * i;
        w1r[i] = reinterpret_cast<const float2*>(w1)[static_cast<int64_t>(c) * units + j];
        wlr[i] = reinterpret_cast<const float2*>(wl)[static_cast<int64_t>(j) * in + c];
    }
    float2 hv = h[static_cast<int64_t>(b) * units + j];
    for (int t = 0; t < T; ++t) {
        const int64_t row = static_cast<int64_t>(b) * T + t;
        const __half* xr = x + row * in;
        float vr = 0.0f, vi = 0.0f, lr = 0.0f, li = 0.0f;
        if (NI > 0) {
#pragma unroll
            for (int i = 0; i < NI; ++i) {
                const float xf = __half2float(xr[lane + 32 * i]);
                vr = fmaf(xf, w1r[i].x, vr);
                vi = fmaf(xf, w1r[i].y, vi);
                lr = fmaf(xf, wlr[i].x, lr);
                li = fmaf(xf, wlr[i].y, li);
            }
        } else {
            for (int c = lane; c < in; c += 32) {
                const float xf = __half2float(xr[c]);
                const int64_t i1 = (static_cast<int64_t>(c) * units + j) << 1;
                const int64_t il = (static_cast<int64_t>(j) * in + c) << 1;
                vr = fmaf(xf, w1[i1], vr);
                vi = fmaf(xf, w1[i1 + 1], vi);
                lr = fmaf(xf, wl[il], lr);
                li = fmaf(xf, wl[il + 1], li);
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            vr += __shfl_down_sync(0xFFFFFFFFu, vr, o);
            vi += __shfl_down_sync(0xFFFFFFFFu, vi, o);
            lr += __shfl_down_sync(0xFFFFFFFFu, lr, o);
            li += __shfl_down_sync(0xFFFFFFFFu, li, o);
        }
        if (!TRACE) {
            if (lane == 0) {
                const float sr = sigmoid_f(vr), si = sigmoid_f(vi);
                const float lam = sigmoid_f(sqrtf(fmaf(lr, lr, fmaf(li, li, kEps))));
                const float dh = 1.0f - lam;
                const float ar = vr * sr, ai = vi * si;
                hv = make_float2(fmaf(hv.x, lam, dh * ar), fmaf(hv.y, lam, dh * ai));
                h_seq[row * units + j] = hv;
            }
        } else {
            // lane 0's sums and gates to every lane, as the reference broadcasts them
            vr = __shfl_sync(0xFFFFFFFFu, vr, 0);
            vi = __shfl_sync(0xFFFFFFFFu, vi, 0);
            lr = __shfl_sync(0xFFFFFFFFu, lr, 0);
            li = __shfl_sync(0xFFFFFFFFu, li, 0);
            float sr = 0.0f, si = 0.0f, lam = 0.0f, lam_inv = 0.0f;
            if (lane == 0) {
                sr = sigmoid_f(vr);
                si = sigmoid_f(vi);
                const float lam_mod = sqrtf(fmaf(lr, lr, fmaf(li, li, kEps)));
                lam = sigmoid_f(lam_mod);
                lam_inv = __frcp_rn(lam_mod);
            }
            sr = __shfl_sync(0xFFFFFFFFu, sr, 0);
            si = __shfl_sync(0xFFFFFFFFu, si, 0);
            lam = __shfl_sync(0xFFFFFFFFu, lam, 0);
            lam_inv = __shfl_sync(0xFFFFFFFFu, lam_inv, 0);
            const float dh = 1.0f - lam;
            const float2 act = make_float2(vr * sr, vi * si);
            // every lane reads the unit's state, as the reference's lanes do
            const float2 h_old = make_float2(__shfl_sync(0xFFFFFFFFu, hv.x, 0), __shfl_sync(0xFFFFFFFFu, hv.y, 0));
            hv = make_float2(fmaf(h_old.x, lam, dh * act.x), fmaf(h_old.y, lam, dh * act.y));
            if (lane == 0) h_seq[row * units + j] = hv;
            const float g_re = dh * sr * fmaf(vr, 1.0f - sr, 1.0f);
            const float g_im = dh * si * fmaf(vi, 1.0f - si, 1.0f);
            const float dlam = (h_old.x - act.x + h_old.y - act.y) * lam * dh * lam_inv;
            float2* twb = tw + static_cast<int64_t>(b) * in * units;
            float2* tlb = tl + static_cast<int64_t>(b) * units * in;
            for (int c = lane; c < in; c += 32) {
                const float xf = __half2float(xr[c]);
                const int64_t i1 = static_cast<int64_t>(c) * units + j, il = static_cast<int64_t>(j) * in + c;
                float2 a = twb[i1], l = tlb[il];
                a.x = fmaf(a.x, lam, g_re * xf);
                a.y = fmaf(a.y, lam, g_im * xf);
                l.x = fmaf(l.x, lam, dlam * xf * lr);
                l.y = fmaf(l.y, lam, dlam * xf * li);
                twb[i1] = a;
                tlb[il] = l;
            }
        }
    }
    if (lane == 0) h[static_cast<int64_t>(b) * units + j] = hv;
}

// One CTA of `units` threads per (sequence, step).
__global__ void critic_score_kernel(const float2* __restrict__ h_seq, const float* __restrict__ w2, int units,
                                    float* __restrict__ score)
{
    __shared__ float warp_sums[32];
    const int64_t row = blockIdx.x;
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    float s = 0.0f;
    for (int i = threadIdx.x; i < units; i += blockDim.x) {
        const float2 f = h_seq[row * units + i];
        s = fmaf(f.x, w2[i << 1], fmaf(f.y, w2[(i << 1) + 1], s));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_down_sync(0xFFFFFFFFu, s, o);
    if (lane == 0) warp_sums[wid] = s;
    __syncthreads();
    if (wid == 0) {
        float f = lane < nw ? warp_sums[lane] : 0.0f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) f += __shfl_down_sync(0xFFFFFFFFu, f, o);
        if (lane == 0) score[row] = f;
    }
}

}  // namespace

cudaError_t launch_critic(const __half* x, const float* w1, const float* wl, const float* w2, int in, int units,
                          float2* h, float2* h_seq, float2* trace_w1, float2* trace_l, float* score, int B, int T,
                          cudaStream_t stream)
{
    if (B == 0 || T == 0) return cudaSuccess;
    dim3 grid(static_cast<unsigned>((units + kThreads / 32 - 1) / (kThreads / 32)), static_cast<unsigned>(B));
    if (trace_w1 != nullptr) {
        critic_cell_kernel<0, true><<<grid, kThreads, 0, stream>>>(x, w1, wl, in, units, h, h_seq, trace_w1, trace_l, T);
    } else {
#define AIC_CELL(NI) critic_cell_kernel<NI, false><<<grid, kThreads, 0, stream>>>(x, w1, wl, in, units, h, h_seq, nullptr, nullptr, T)
        switch (in) {
            case 32: AIC_CELL(1); break;
            case 64: AIC_CELL(2); break;
            case 128: AIC_CELL(4); break;
            case 256: AIC_CELL(8); break;
            default: AIC_CELL(0); break;
        }
#undef AIC_CELL
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    critic_score_kernel<<<static_cast<unsigned>(static_cast<int64_t>(B) * T), units, 0, stream>>>(h_seq, w2, units, score);
    return cudaGetLastError();
}

}  // namespace aic
