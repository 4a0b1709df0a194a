/*
 * CPU oracle of the training path (the reference's backward and SGD kernels)
 * -- TEST INFRASTRUCTURE ONLY. One layer step per call, as the reference's
 * layer classes run backward: ConvLayer::backward (conv_layer.h:150-219),
 * MambaLayer::backward (mamba_layer.h:146-167), Critic::backward
 * (critic.h:117-131). Each function restates the reference kernels' formulas
 * in their order (kernels.h citations per function), including where they
 * differ from the textbook gradient; libm replaces the fast-math intrinsics.
 * Built with aic_oracle.c (-ffp-contract=off; fmaf() where the reference's
 * code is an fma or a contracted multiply-add).
 */
#include "aic_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#define ORC_EPS (1.0f / 8192.0f)
#define ORC_CPB 256

static inline int nib(uint32_t word, int e)
{
    int v = (int)((word >> (e << 2)) & 0xFu);
    return v >= 8 ? v - 16 : v;
}
static inline int dot8(uint32_t a, uint32_t b)
{
    int s = 0;
    for (int e = 0; e < 8; ++e) s += nib(a, e) * nib(b, e);
    return s;
}
/* dequantize_scalar (kernels.h:77) */
static inline float deq(const uint32_t* w, const int8_t* s, int64_t i)
{
    return (float)nib(w[i >> 3], (int)(i & 7)) * orc_dequantize_scale(s[i >> 5]);
}
static inline float rsqrt_rn(float x) { return (float)(1.0 / sqrt((double)x)); }
static inline float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }
/* silu_grad (kernels.h:88-92) as its two factors dy * sig and 1 + x (1 - sig) */
static inline void silu_parts(float x, float dy, float* a, float* b)
{
    const float sig = sigmoidf_(x);
    *a = dy * sig;
    *b = fmaf(x, 1.0f - sig, 1.0f);
}
/* lane 0's value after `v += __shfl_xor_sync(v, o)` for o = first..1 */
static float xor_sum(const float* vals, int n, int first)
{
    float a[32], b[32];
    for (int l = 0; l < 32; ++l) a[l] = l < n ? vals[l] : 0.0f;
    for (int o = first; o > 0; o >>= 1) {
        for (int l = 0; l < 32; ++l) b[l] = a[l] + a[l ^ o];
        memcpy(a, b, sizeof(a));
    }
    return a[0];
}
/* the 256-thread block's square sum of one position's chunk (kernels.h:330-341) */
static float block_sq(const float* acc, int n)
{
    float warp_part[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int w = 0; w < 8 && 32 * w < n; ++w) {
        float sq[32];
        for (int l = 0; l < 32; ++l) sq[l] = 32 * w + l < n ? acc[32 * w + l] * acc[32 * w + l] : 0.0f;
        warp_part[w] = xor_sum(sq, 32, 16);
    }
    return xor_sum(warp_part, 8, 4);
}

/* updateParamsKernel (kernels.h:196-216) with a given grad_norm_factor: whole
 * uint4 only (the first floor(n / 4) * 4 elements). */
void orc_sgd_update(float* data, const float* grad, int64_t n, float factor, float lr, float penalty)
{
    const float c_grad = -lr * factor;
    const float c_data = fmaf(-lr, penalty, 1.0f);
    const int64_t m = (n >> 2) << 2;
    for (int64_t i = 0; i < m; ++i) data[i] = fmaf(grad[i], c_grad, data[i] * c_data);
}

/* clip_op (conv_layer.h:209-213) of the square sum formed like
 * transformReduceKernel (uv.h:9-24): per-thread sums over a grid of `blocks`
 * 256-thread blocks, lane tree, warp tree, blocks added in order. */
float orc_clip_factor(const float* g, int64_t n, int blocks, float* sum_out)
{
    const int64_t stride = (int64_t)blocks * 256;
    float total = 0.0f;
    for (int b = 0; b < blocks; ++b) {
        float warp_sum[8];
        for (int w = 0; w < 8; ++w) {
            float lane[32];
            for (int l = 0; l < 32; ++l) {
                float s = 0.0f;
                for (int64_t i = (int64_t)b * 256 + w * 32 + l; i < n; i += stride) s = fmaf(g[i], g[i], s);
                lane[l] = s;
            }
            /* shfl_down 16..1: lane 0 */
            for (int o = 16; o > 0; o >>= 1)
                for (int l = 0; l < 32; ++l) lane[l] = l + o < 32 ? lane[l] + lane[l + o] : lane[l] + lane[l];
            warp_sum[w] = lane[0];
        }
        float lane[32];
        for (int l = 0; l < 32; ++l) lane[l] = l < 8 ? warp_sum[l] : 0.0f;
        for (int o = 4; o > 0; o >>= 1)
            for (int l = 0; l < 32; ++l) lane[l] = l + o < 32 ? lane[l] + lane[l + o] : lane[l] + lane[l];
        total = total + lane[0];
    }
    if (sum_out) *sum_out = total;
    const float norm = sqrtf(total + ORC_EPS);
    return norm > 1.0f ? 1.0f / norm : 1.0f;
}

/* ConvLayer::backward's gradient kernels on one frame (conv_layer.h:152-206):
 * gw, gb written; grad_in added to (pointwise, dense) or written (depthwise).
 * in / in_s the layer's forward input, w / w_s the packed weights, master the
 * fp32 masters, dy [Dout^2][OutC]. */
void orc_conv_backward(const uint32_t* in, const int8_t* in_s, const uint32_t* w, const int8_t* w_s,
                       const float* bias, const float* master, const float* dy, int InC, int OutC, int ks,
                       int stride, int Din, int Dout, int act, float* gw, float* gb, float* grad_in)
{
    const int P = Dout * Dout, G = InC >> 5, ksq = ks * ks;
    if (ks > 1 && (ks & 1)) {
        const int pad = ks >> 1;
        /* convDepthwiseBwdGradBiasKernel (kernels.h:961-988): chains p = 4j + i */
        for (int c = 0; c < InC; ++c) {
            float s[4] = {0, 0, 0, 0};
            for (int p = 0; p < P; p += 4)
                for (int i = 0; i < 4; ++i) s[i] = s[i] + dy[(int64_t)(p + i) * InC + c];
            gb[c] = ((s[0] + s[1]) + s[2]) + s[3];
        }
        /* convDepthwiseBwdGradWeightKernel (kernels.h:911-960) */
        for (int k = 0; k < ksq; ++k)
            for (int c = 0; c < InC; ++c) {
                float a = 0.0f;
                for (int p = 0; p < P; ++p) {
                    const int hi = p / Dout * stride - pad + k / ks, wi = (p % Dout) * stride - pad + k % ks;
                    if (hi >= 0 && hi < Din && wi >= 0 && wi < Din)
                        a = fmaf(deq(in, in_s, ((int64_t)hi * Din + wi) * InC + c), dy[(int64_t)p * InC + c], a);
                }
                gw[(int64_t)k * InC + c] = a;
            }
        /* convDepthwiseBwdGradInputKernel (kernels.h:871-910) */
        if (grad_in)
            for (int pin = 0; pin < Din * Din; ++pin)
                for (int c = 0; c < InC; ++c) {
                    const int hi = pin / Din, wi = pin % Din;
                    float a = 0.0f;
                    for (int k = 0; k < ksq; ++k) {
                        const int ht = hi - k / ks + pad, wt = wi - k % ks + pad;
                        float g = 0.0f;
                        if (ht % stride == 0 && wt % stride == 0) {
                            const int ho = ht / stride, wo = wt / stride;
                            if (ho >= 0 && ho < Dout && wo >= 0 && wo < Dout) g = dy[((int64_t)ho * Dout + wo) * InC + c];
                        }
                        a = fmaf(g, master[(int64_t)k * InC + c], a);
                    }
                    grad_in[(int64_t)pin * InC + c] = a;
                }
        return;
    }
    const int pad = ks == stride ? 0 : (ks - 1) >> 1;
    float* facc = (float*)malloc(sizeof(float) * (size_t)P * OutC);
    float* dyn = (float*)malloc(sizeof(float) * (size_t)P * OutC);
    float* ga = (float*)malloc(sizeof(float) * (size_t)P * OutC);
    float* gt = (float*)malloc(sizeof(float) * (size_t)P * OutC);
    const float inv_div = 1.0f / (float)(OutC < ORC_CPB ? OutC : ORC_CPB);
    /* the forward recompute and the activation gradient (kernels.h:301-345, 605-648) */
    for (int p = 0; p < P; ++p) {
        const int hs = p / Dout * stride - pad, ws0 = (p % Dout) * stride - pad;
        for (int oc = 0; oc < OutC; ++oc) {
            float a4[4] = {0, 0, 0, 0}, a = 0.0f;
            for (int k = 0; k < ksq; ++k) {
                const int hi = hs + k / ks, wi = ws0 + k % ks;
                if (ks > 1 && (hi < 0 || hi >= Din || wi < 0 || wi >= Din)) continue;
                const int64_t pix = ks == 1 ? p : (int64_t)hi * Din + wi;
                for (int g = 0; g < G; ++g) {
                    const int64_t wg = ((int64_t)oc * ksq + k) * G + g;
                    int part = 0;
                    for (int i = 0; i < 4; ++i) part += dot8(in[(pix * G + g) * 4 + i], w[wg * 4 + i]);
                    const float t = orc_dequantize_scale(w_s[wg]) * (float)part;
                    if (ks == 1) a = fmaf(orc_dequantize_scale(in_s[pix * G + g]), t, a);
                    else a4[k & 3] = fmaf(orc_dequantize_scale(in_s[pix * G + g]), t, a4[k & 3]);
                }
            }
            facc[(int64_t)p * OutC + oc] = ks == 1 ? a : ((a4[0] + a4[1]) + a4[2]) + a4[3];
        }
        for (int c0 = 0; c0 < OutC; c0 += ORC_CPB) {
            const int n = OutC - c0 < ORC_CPB ? OutC - c0 : ORC_CPB;
            const float inv = rsqrt_rn(fmaf(block_sq(facc + (int64_t)p * OutC + c0, n), inv_div, ORC_EPS));
            for (int oc = c0; oc < c0 + n; ++oc) {
                const int64_t o = (int64_t)p * OutC + oc;
                float fa = dy[o], fb = 1.0f;
                if (act) silu_parts(fmaf(facc[o], inv, bias[oc]), dy[o], &fa, &fb);
                ga[o] = fa;
                gt[o] = fb;
                dyn[o] = (act ? fa * fb : dy[o]) * inv;
            }
        }
    }
    /* bias gradient (kernels.h:445-513, 760-830): acc += silu_grad (contracted) or dy */
    for (int oc = 0; oc < OutC; ++oc) {
        float s = 0.0f;
        for (int p = 0; p < P; ++p) {
            const int64_t o = (int64_t)p * OutC + oc;
            s = act ? fmaf(ga[o], gt[o], s) : s + ga[o];
        }
        gb[oc] = s;
    }
    if (ks == 1) {
        /* convPointwiseBwdGradWeightKernel (kernels.h:359-444): its own inv_rms from
         * the 32-channel tile x 8-position square sums, then the (p0 + y, k)
         * pairing of input channel 32 by + k with the output gradient of p0 + k */
        float* dynw = (float*)malloc(sizeof(float) * (size_t)P * OutC);
        for (int grp = 0; grp < P / 8; ++grp)
            for (int t = 0; t < OutC / 32; ++t) {
                float sums[8];
                for (int i = 0; i < 8; ++i) {
                    float sq[32];
                    for (int l = 0; l < 32; ++l) {
                        const float a = facc[(int64_t)(grp * 8 + i) * OutC + t * 32 + l];
                        sq[l] = a * a;
                    }
                    sums[i] = xor_sum(sq, 32, 16);
                }
                float gs = 0.0f;
                for (int i = 0; i < 8; ++i) gs = gs + sums[i];
                const float inv = rsqrt_rn(fmaf(gs, inv_div, ORC_EPS));
                for (int i = 0; i < 8; ++i)
                    for (int l = 0; l < 32; ++l) {
                        const int64_t o = (int64_t)(grp * 8 + i) * OutC + t * 32 + l;
                        float fa = dy[o], fb = 1.0f;
                        if (act) silu_parts(fmaf(facc[o], inv, bias[t * 32 + l]), dy[o], &fa, &fb);
                        dynw[o] = (act ? fa * fb : dy[o]) * inv;
                    }
            }
        for (int oc = 0; oc < OutC; ++oc)
            for (int ic = 0; ic < InC; ++ic) {
                const int by = ic >> 5, y = ic & 31;
                float s[4] = {0, 0, 0, 0};
                for (int p0 = 0; p0 < P; p0 += 32)
                    for (int k = 0; k < 32; k += 4)
                        for (int i = 0; i < 4; ++i)
                            s[i] = fmaf(deq(in, in_s, (int64_t)(p0 + y) * InC + by * 32 + k + i),
                                        dynw[(int64_t)(p0 + k + i) * OutC + oc], s[i]);
                gw[(int64_t)oc * InC + ic] = ((s[0] + s[1]) + s[2]) + s[3];
            }
        free(dynw);
        /* convPointwiseBwdGradInputKernel (kernels.h:283-358): chunk c's term
         * reads master[256 c + i * InC + ic]; chunks added in order */
        if (grad_in)
            for (int p = 0; p < P; ++p)
                for (int c0 = 0; c0 < OutC; c0 += ORC_CPB) {
                    const int n = OutC - c0 < ORC_CPB ? OutC - c0 : ORC_CPB;
                    for (int ic = 0; ic < InC; ++ic) {
                        if ((ic & (ORC_CPB - 1)) >= n) continue;
                        float a = 0.0f;
                        for (int i = 0; i < n; ++i)
                            a = fmaf(dyn[(int64_t)p * OutC + c0 + i], master[c0 + (int64_t)i * InC + ic], a);
                        grad_in[(int64_t)p * InC + ic] += a;
                    }
                }
    } else {
        /* convDenseBwdGradWeightKernel (kernels.h:676-759) */
        for (int oc = 0; oc < OutC; ++oc)
            for (int ic = 0; ic < InC; ++ic) {
                float s[16];
                for (int k = 0; k < 16; ++k) s[k] = 0.0f;
                for (int p = 0; p < P; ++p) {
                    const int hs = p / Dout * stride - pad, ws0 = (p % Dout) * stride - pad;
                    for (int k = 0; k < ksq; ++k) {
                        const int hi = hs + k / ks, wi = ws0 + k % ks;
                        if (hi < 0 || hi >= Din || wi < 0 || wi >= Din) continue;
                        s[k] = fmaf(deq(in, in_s, ((int64_t)hi * Din + wi) * InC + ic), dyn[(int64_t)p * OutC + oc], s[k]);
                    }
                }
                for (int k = 0; k < ksq; ++k) gw[((int64_t)oc * ksq + k) * InC + ic] = s[k];
            }
        /* convDenseBwdGradInputKernel (kernels.h:586-675) */
        if (grad_in)
            for (int p = 0; p < P; ++p) {
                const int hs = p / Dout * stride - pad, ws0 = (p % Dout) * stride - pad;
                for (int c0 = 0; c0 < OutC; c0 += ORC_CPB) {
                    const int n = OutC - c0 < ORC_CPB ? OutC - c0 : ORC_CPB;
                    for (int ic = 0; ic < InC; ++ic) {
                        if ((ic & (ORC_CPB - 1)) >= n) continue;
                        for (int k = 0; k < ksq; ++k) {
                            const int hi = hs + k / ks, wi = ws0 + k % ks;
                            if (hi < 0 || hi >= Din || wi < 0 || wi >= Din) continue;
                            float a = 0.0f;
                            for (int i = 0; i < n; ++i)
                                a = fmaf(dyn[(int64_t)p * OutC + c0 + i], master[(((int64_t)c0 + i) * ksq + k) * InC + ic], a);
                            grad_in[((int64_t)hi * Din + wi) * InC + ic] += a;
                        }
                    }
                }
            }
    }
    free(facc);
    free(dyn);
    free(ga);
    free(gt);
}

/* MambaLayer::backward's gradient kernels (mamba_layer.h:146-157) for one
 * sequence after a step: h and the traces ta / tb / td compact [E][N/32]
 * complex (state c of channel ch = the reference's index ch*N + (ch & 31) +
 * 32c), m the fp32 blob, dy [OutC]. gw (blob size) is zeroed here; every
 * element the reference adds atomically to a zero is formed as 0 + x. */
void orc_mamba_backward(const uint32_t* in, const int8_t* in_s, const float* h, const float* ta, const float* tb,
                        const float* td, const float* m, const float* bias, const float* dy, int D, int N, int OutC,
                        int act, float* gw, float* gb, float* grad_in)
{
    const int E = 2 * D, P = N >> 5, chunks = E / ORC_CPB;
    const int64_t c_re = 33LL * E, c_im = c_re + (int64_t)E * N, a_re = c_im + (int64_t)E * N,
                  a_im = a_re + (int64_t)E * N, o_d = a_im + (int64_t)E * N, w_out = o_d + E;
    memset(gw, 0, sizeof(float) * (size_t)(w_out + (int64_t)OutC * E));
    float* y = (float*)malloc(sizeof(float) * E);
    float* xv = (float*)malloc(sizeof(float) * D);
    for (int i = 0; i < D; ++i) xv[i] = deq(in, in_s, i);
    /* y_ssm recomputed from the state (kernels.h:1277-1288) */
    for (int ch = 0; ch < E; ++ch) {
        float v = m[o_d + ch] * xv[ch & (D - 1)];
        const int64_t base = (int64_t)ch * N + (ch & 31);
        for (int c = 0; c < P; ++c) {
            const float* hv = h + 2 * ((int64_t)ch * P + c);
            v = fmaf(hv[0], m[c_re + base + 32 * c], v);
            v = fmaf(-hv[1], m[c_im + base + 32 * c], v);
        }
        y[ch] = v;
    }
    /* mambaSSMBwdOutProjKernel (kernels.h:1260-1302): per (32-output tile,
     * chunk, warp) 8-lane partial sums, folded with absolute-lane shuffles */
    float* raw = (float*)calloc((size_t)OutC, sizeof(float));
    for (int ck = 0; ck < chunks; ++ck)
        for (int bx = 0; bx < OutC / 32; ++bx)
            for (int wp = 0; wp < 8; ++wp) {
                float v[32], nv[32];
                for (int l = 0; l < 32; ++l) {
                    const int oc = bx * 32 + wp * 4 + (l >> 3), v8 = l & 7;
                    const int64_t wb = w_out + (int64_t)oc * E + ck * ORC_CPB + v8 * 32;
                    float s = 0.0f;
                    for (int i = 0; i < 32; ++i) s = fmaf(y[ck * ORC_CPB + v8 * 32 + i], m[wb + i], s);
                    v[l] = s;
                }
                for (int off = 4; off > 0; off >>= 1) {
                    for (int l = 0; l < 32; ++l) nv[l] = v[l] + v[off];
                    memcpy(v, nv, sizeof(v));
                }
                for (int j = 0; j < 4; ++j) raw[bx * 32 + wp * 4 + j] = raw[bx * 32 + wp * 4 + j] + v[8 * j];
            }
    /* mambaSSMBwdNormActKernel (kernels.h:1303-1336) */
    float* gn = (float*)malloc(sizeof(float) * OutC);
    const float inv_div = 1.0f / (float)(OutC < ORC_CPB ? OutC : ORC_CPB);
    for (int c0 = 0; c0 < OutC; c0 += ORC_CPB) {
        const int n = OutC - c0 < ORC_CPB ? OutC - c0 : ORC_CPB;
        const float inv = OutC < 2 ? 1.0f : rsqrt_rn(fmaf(block_sq(raw + c0, n), inv_div, ORC_EPS));
        for (int oc = c0; oc < c0 + n; ++oc) {
            const float u = fmaf(raw[oc], inv, bias[oc]), d = dy[oc];
            float g = d;
            if (act != 0) {
                const float sig = sigmoidf_(u);
                g = act == 1 ? (d * sig) * fmaf(u, 1.0f - sig, 1.0f) : (d * sig) * (1.0f - sig);
            }
            gb[oc] = g;
            gn[oc] = g * inv;
        }
    }
    /* mambaSSMApplyTracesKernel (kernels.h:1337-1419) */
    float* gyv = (float*)malloc(sizeof(float) * E);
    float* gbv = (float*)malloc(sizeof(float) * E);
    float* gdv = (float*)malloc(sizeof(float) * E);
    for (int ch = 0; ch < E; ++ch) {
        float gy = 0.0f;
        for (int oc = 0; oc < OutC; ++oc) {
            const int64_t wi = w_out + (int64_t)oc * E + ch;
            gw[wi] = gn[oc] * y[ch];
            gy = fmaf(gn[oc], m[wi], gy);
        }
        float g_dt = 0.0f, g_b = 0.0f;
        const int64_t base = (int64_t)ch * N + (ch & 31);
        for (int c = 0; c < P; ++c) {
            const int64_t idx = base + 32 * c, s2 = 2 * ((int64_t)ch * P + c);
            const float wre = m[c_re + idx], wim = m[c_im + idx];
            const float ghr = gy * wre, ghi = -gy * wim;
            gw[c_re + idx] = 0.0f + gy * h[s2];
            gw[c_im + idx] = 0.0f + -gy * h[s2 + 1];
            gw[a_re + idx] = 0.0f + fmaf(ghr, ta[s2], ghi * ta[s2 + 1]);
            gw[a_im + idx] = 0.0f + fmaf(ghi, ta[s2], -ghr * ta[s2 + 1]);
            g_b = fmaf(ghr, tb[s2], fmaf(ghi, tb[s2 + 1], g_b));
            g_dt = fmaf(ghr, td[s2], fmaf(ghi, td[s2 + 1], g_dt));
        }
        gyv[ch] = gy;
        gbv[ch] = g_b;
        gdv[ch] = g_dt;
    }
    float* gx = (float*)malloc(sizeof(float) * E);
    for (int ch = 0; ch < E; ++ch) {
        const int lane = ch & 31, bc = ch & ~31;
        const int64_t mimo = E + (int64_t)(bc >> 5) * 1024;
        float gxb[4] = {0, 0, 0, 0};
        for (int k = 0; k < 32; ++k) {
            gw[mimo + lane * 32 + k] = 0.0f + gbv[ch] * xv[(bc + k) & (D - 1)];
            gxb[k & 3] = fmaf(gbv[bc + k], m[mimo + lane + 32 * k], gxb[k & 3]);
        }
        const float x = xv[ch & (D - 1)], wd = m[ch];
        const float g_pre = gdv[ch] * sigmoidf_(x * wd);
        gw[ch] = 0.0f + g_pre * x;
        gw[o_d + ch] = 0.0f + gyv[ch] * x;
        gx[ch] = fmaf(g_pre, wd, fmaf(gyv[ch], m[o_d + ch], ((gxb[0] + gxb[1]) + gxb[2]) + gxb[3]));
    }
    for (int ic = 0; ic < D; ++ic) grad_in[ic] = (0.0f + gx[ic]) + gx[ic + D];
    free(y); free(xv); free(raw); free(gn); free(gyv); free(gbv); free(gdv); free(gx);
}

/* criticApplyTracesKernel + criticOutputGradKernel (kernels.h:1779-1805):
 * trace_w1 [in][units], trace_l [units][in], hidden [units], all complex. */
void orc_critic_backward(const float* w2, const float* tw1, const float* tl, const float* hidden, float pred,
                         float real, int units, int in, float* gw1, float* gl, float* gw2)
{
    const float go = pred - real;
    for (int64_t idx = 0; idx < (int64_t)units * in; ++idx) {
        const int node = (int)(idx % units) * 2, lam = (int)(idx / in) * 2;
        gw1[2 * idx] = (go * w2[node]) * tw1[2 * idx];
        gw1[2 * idx + 1] = (go * w2[node + 1]) * tw1[2 * idx + 1];
        gl[2 * idx] = (go * w2[lam]) * tl[2 * idx];
        gl[2 * idx + 1] = (go * w2[lam + 1]) * tl[2 * idx + 1];
    }
    for (int u = 0; u < units; ++u) {
        gw2[2 * u] = go * hidden[2 * u];
        gw2[2 * u + 1] = go * hidden[2 * u + 1];
    }
}
