/*
 * CPU oracle for the AICortex inference hot path -- TEST INFRASTRUCTURE ONLY.
 * See aic_oracle.h. Reference citations are to AICortex's kernels.h and the
 * layer headers (conv_layer.h, conv_block.h, mamba_layer.h, mamba_block.h,
 * critic.h).
 *
 * Build: gcc -O3 -fopenmp -ffp-contract=off -shared -fPIC (oracle/Makefile).
 * -ffp-contract=off keeps every multiply and add separately rounded unless the
 * code calls fmaf() explicitly, which is how the reference kernels are written.
 */
#include "aic_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* kernels.h / base_constants.h constants */
#define ORC_EPS (1.0f / 8192.0f)   /* epsilon, base_constants.h:33 */
#define ORC_QMAX 7.0f              /* quant_int4_max */
#define ORC_SMIN (-120.0f)         /* quant_scale_min */
#define ORC_SMAX 120.0f            /* quant_scale_max */
#define ORC_FMAXIMUM 65504.0f      /* fmaximum */
#define ORC_CPB 256                /* channels_per_block == gpu_block_threads */

/* kernels.h:41: `getFastRandomModifier(seed) * (1.0f / 0xFFFFFFFFf) * n`.
 * `0xFFFFFFFFf` is the hexadecimal INTEGER literal 0xFFFFFFFFF (the trailing f
 * is a hex digit), i.e. 2^36-1, which converts to the float 2^36. The factor
 * is therefore exactly 2^-36 and the "uniform" lies in [0, n/16). */
static const float ORC_U32_TO_UNIFORM = 1.0f / 68719476736.0f;

int orc_num_threads(void)
{
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* kernels.h:21-37, device branch: the base is the global thread index. */
uint32_t orc_unique_seed(uint32_t global_tid, int32_t sample_index)
{
    uint32_t s = global_tid;
    s += (uint32_t)sample_index * 2654435761U;
    s = (s ^ 61u) ^ (s >> 16);
    s *= 9u;
    s ^= s >> 4;
    s *= 668265261u;
    s ^= s >> 15;
    return s == 0 ? 123456789u : s;
}

/* kernels.h:38-44 */
static inline uint32_t orc_xorshift(uint32_t seed)
{
    seed ^= seed << 13;
    seed ^= seed >> 17;
    seed ^= seed << 5;
    return seed;
}

float orc_uniform(uint32_t seed, float n)
{
    float u = (float)orc_xorshift(seed);
    u = u * ORC_U32_TO_UNIFORM;
    return u * n;
}

/* kernels.h:68: rn(clamp(log2(scale), +-120)) */
int8_t orc_quantize_scale(float scale)
{
    float l = log2f(scale);
    l = fmaxf(ORC_SMIN, fminf(ORC_SMAX, l));
    return (int8_t)(int)rintf(l);
}

/* kernels.h:69: max(2^s / 7, 2^-13) */
float orc_dequantize_scale(int8_t s)
{
    float v = ldexpf(1.0f, s) * (1.0f / ORC_QMAX);
    return fmaxf(v, ORC_EPS);
}

static inline int orc_nib(uint32_t word, int e) /* bfe.s32 sign extend, kernels.h:56-72 */
{
    int v = (int)((word >> (4 * e)) & 0xFu);
    return v >= 8 ? v - 16 : v;
}

static inline float orc_rcp(float x) { return 1.0f / x; }              /* __frcp_rn */
static inline float orc_rsqrt(float x) { return (float)(1.0 / sqrt((double)x)); } /* __frsqrt_rn */
static inline float orc_sigmoid(float x) { return orc_rcp(1.0f + expf(-x)); }     /* kernels.h:86 */
static inline float orc_silu(float x) { return x * orc_sigmoid(x); }              /* kernels.h:87 */

/* kernels.h:70: clamp(__float2int_rn(v * inv), -8, 7) & 0xF. The GPU
   conversion (cvt.rni.s32.f32) gives 0 for a NaN and saturates infinities;
   clamping before the conversion gives the same code (rounding is monotonic)
   and keeps the C conversion defined. */
static inline uint32_t orc_q_rn(float v, float inv)
{
    const float p = v * inv;
    if (p != p) return 0u;
    const int q = (int)rintf(fmaxf(-8.0f, fminf(7.0f, p)));
    return (uint32_t)q & 0xFu;
}

/* kernels.h:71-76, element_idx hashed from the calling thread's global id */
static inline uint32_t orc_q_stochastic(float v, float inv, uint32_t tid, int32_t element_idx)
{
    float scaled = fmaxf(-8.0f, fminf(ORC_QMAX, v * inv));
    int fl = (int)floorf(scaled);
    float u = orc_uniform(orc_unique_seed(tid, element_idx), 1.0f);
    int up = u < (scaled - (float)fl);
    return (uint32_t)(fl + up) & 0xFu;
}

/* kernels.h:85: exact integer dot of 8 nibble pairs */
static inline int orc_dot8(uint32_t a, uint32_t b)
{
    int s = 0;
    for (int e = 0; e < 8; ++e) s += orc_nib(a, e) * orc_nib(b, e);
    return s;
}

/* lane 0's value after `v += __shfl_xor_sync(v, o)` for o = first..1 */
static float orc_xor_reduce_sum(const float* vals, int first_offset)
{
    float a[32], b[32];
    memcpy(a, vals, sizeof(a));
    for (int o = first_offset; o > 0; o >>= 1) {
        for (int l = 0; l < 32; ++l) b[l] = a[l] + a[l ^ o];
        memcpy(a, b, sizeof(a));
    }
    return a[0];
}

/* lane 0's value after `v += __shfl_down_sync(v, o)` for o = 16..1 */
static float orc_down_reduce_sum(const float* vals)
{
    float a[32], b[32];
    memcpy(a, vals, sizeof(a));
    for (int o = 16; o > 0; o >>= 1) {
        for (int l = 0; l < 32; ++l) b[l] = l + o < 32 ? a[l] + a[l + o] : a[l] + a[l];
        memcpy(a, b, sizeof(a));
    }
    return a[0];
}

float orc_half_to_float(uint16_t h)
{
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    int exp = (h >> 10) & 0x1F;
    uint32_t man = h & 0x3FFu;
    float f;
    if (exp == 0) {
        f = ldexpf((float)man, -24);
        if (sign) f = -f;
        return f;
    }
    if (exp == 31) {
        uint32_t bits = sign | 0x7F800000u | (man << 13);
        memcpy(&f, &bits, 4);
        return f;
    }
    uint32_t bits = sign | ((uint32_t)(exp - 15 + 127) << 23) | (man << 13);
    memcpy(&f, &bits, 4);
    return f;
}

/* IEEE binary32 -> binary16, round to nearest even */
uint16_t orc_float_to_half(float f)
{
    uint32_t x;
    memcpy(&x, &f, 4);
    uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0u));
    if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u); /* rounds to inf */
    if (ax < 0x38800000u) { /* subnormal half (or zero) */
        float a;
        memcpy(&a, &ax, 4);
        float q = rintf(a * 16777216.0f); /* units of 2^-24, ties to even */
        return (uint16_t)(sign | (uint16_t)q);
    }
    uint32_t e = (ax >> 23) - 127 + 15;
    uint32_t man = ax & 0x7FFFFFu;
    uint32_t h = (e << 10) | (man >> 13);
    uint32_t rem = man & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1;
    return (uint16_t)(sign | h);
}

/* ------------------------------------------------------------------ A1 */
void orc_pack_f32(const float* in, int64_t n, uint32_t* out, int8_t* scales,
                  int stochastic, int32_t add_idx)
{
    const int64_t groups = n >> 5;
#pragma omp parallel for schedule(static)
    for (int64_t idx = 0; idx < groups; ++idx) {
        const float* v = in + (idx << 5);
        float amax = 0.0f;
        for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
        const float scale = amax < ORC_EPS ? 1.0f : amax;
        scales[idx] = orc_quantize_scale(scale);
        const float inv = ORC_QMAX * orc_rcp(scale);
        uint32_t w[4] = {0, 0, 0, 0};
        if (stochastic) {
            const uint32_t tid = (uint32_t)idx;
            const uint32_t tseed = orc_unique_seed(tid, (int32_t)(idx + add_idx));
            for (int i = 0; i < 32; ++i)
                w[i >> 3] |= orc_q_stochastic(v[i], inv, tid, (int32_t)(tseed ^ (uint32_t)i)) << ((i & 7) << 2);
        } else {
            for (int i = 0; i < 32; ++i) w[i >> 3] |= orc_q_rn(v[i], inv) << ((i & 7) << 2);
        }
        memcpy(out + (idx << 2), w, 16);
    }
}

/* ------------------------------------------------------------------ A2 */
void orc_stem_pack(const uint16_t* planes, int64_t frames, int planes_present,
                   int channels, int dim, uint32_t* out, int8_t* out_s)
{
    const int64_t hw = (int64_t)dim * dim;
    const int groups = channels >> 5;
#pragma omp parallel for schedule(static)
    for (int64_t fp = 0; fp < frames * hw; ++fp) {
        const int64_t f = fp / hw, sp = fp % hw;
        for (int g = 0; g < groups; ++g) {
            float v[32];
            float amax = NAN; /* the reference reduces |v| by a lane butterfly: NaN only if every value is */
            for (int l = 0; l < 32; ++l) {
                const int c = (g << 5) + l;
                v[l] = c < planes_present ? orc_half_to_float(planes[(f * planes_present + c) * hw + sp]) : 0.0f;
                amax = fmaxf(amax, fabsf(v[l]));
            }
            const float scale = amax < ORC_EPS ? 1.0f : amax;
            const float inv = ORC_QMAX * orc_rcp(scale);
            uint32_t w[4] = {0, 0, 0, 0};
            for (int l = 0; l < 32; ++l) w[l >> 3] |= orc_q_rn(v[l], inv) << ((l & 7) << 2);
            memcpy(out + fp * (channels >> 3) + g * 4, w, 16);
            out_s[fp * groups + g] = orc_quantize_scale(scale);
        }
    }
}

/* Shared epilogue of the quantized convs (kernels.h:255-281, 565-584):
 * RMSNorm over each 256-channel CTA chunk (divisor min(OutC,256)), bias,
 * optional SiLU, then int4 requant per 32 channels. acc: [OutC]. */
static void orc_conv_epilogue(const float* acc, const float* bias, int OutC, int act,
                              uint32_t* out_words, int8_t* out_s)
{
    const float inv_div = orc_rcp((float)(OutC < ORC_CPB ? OutC : ORC_CPB));
    for (int c0 = 0; c0 < OutC; c0 += ORC_CPB) {
        float warp_part[32];
        for (int w = 0; w < 32; ++w) warp_part[w] = 0.0f;
        for (int w = 0; w < ORC_CPB / 32; ++w) {
            const int base = c0 + w * 32;
            if (base >= OutC) break;
            float sq[32];
            for (int l = 0; l < 32; ++l) sq[l] = acc[base + l] * acc[base + l];
            warp_part[w] = orc_xor_reduce_sum(sq, 16);
        }
        const float block_sq = orc_xor_reduce_sum(warp_part, (ORC_CPB / 32) >> 1);
        const float inv_rms = orc_rsqrt(fmaf(block_sq, inv_div, ORC_EPS));
        for (int base = c0; base < c0 + ORC_CPB && base < OutC; base += 32) {
            float v[32];
            float amax = NAN; /* the reference reduces |v| by a lane butterfly: NaN only if every value is */
            for (int l = 0; l < 32; ++l) {
                float a = fmaf(acc[base + l], inv_rms, bias[base + l]);
                if (act) a = orc_silu(a);
                v[l] = a;
                amax = fmaxf(amax, fabsf(a));
            }
            const float scale = amax < ORC_EPS ? 1.0f : amax;
            const float inv = ORC_QMAX * orc_rcp(scale);
            uint32_t w[4] = {0, 0, 0, 0};
            for (int l = 0; l < 32; ++l) w[l >> 3] |= orc_q_rn(v[l], inv) << ((l & 7) << 2);
            memcpy(out_words + (base >> 3), w, 16);
            out_s[base >> 5] = orc_quantize_scale(scale);
        }
    }
}

/* ------------------------------------------------------------------ A4 */
void orc_conv_pw(const uint32_t* in, const int8_t* in_s, const uint32_t* w,
                 const int8_t* w_s, const float* bias, uint32_t* out,
                 int8_t* out_s, int64_t positions, int InC, int OutC, int act)
{
    const int G = InC >> 5;
#pragma omp parallel
    {
        float* acc = (float*)malloc(sizeof(float) * OutC);
#pragma omp for schedule(static)
        for (int64_t p = 0; p < positions; ++p) {
            const uint32_t* xi = in + p * (InC >> 3);
            const int8_t* xs = in_s + p * G;
            for (int oc = 0; oc < OutC; ++oc) {
                const uint32_t* wr = w + (int64_t)oc * (InC >> 3);
                const int8_t* wsr = w_s + (int64_t)oc * G;
                float a = 0.0f;
                for (int g = 0; g < G; ++g) {
                    int ps = 0;
                    for (int i = 0; i < 4; ++i) ps += orc_dot8(xi[g * 4 + i], wr[g * 4 + i]);
                    a = fmaf(orc_dequantize_scale(xs[g]), orc_dequantize_scale(wsr[g]) * (float)ps, a);
                }
                acc[oc] = a;
            }
            orc_conv_epilogue(acc, bias, OutC, act, out + p * (OutC >> 3), out_s + p * (OutC >> 5));
        }
        free(acc);
    }
}

/* ------------------------------------------------------------------ A3 */
void orc_conv_dense(const uint32_t* in, const int8_t* in_s, const uint32_t* w,
                    const int8_t* w_s, const float* bias, uint32_t* out,
                    int8_t* out_s, int64_t frames, int InC, int OutC, int ksize,
                    int stride, int Din, int Dout, int act)
{
    const int G = InC >> 5, ksq = ksize * ksize;
    const int pad = ksize == stride ? 0 : (ksize - 1) >> 1;
    const int64_t hw_in = (int64_t)Din * Din, hw_out = (int64_t)Dout * Dout;
#pragma omp parallel
    {
        float* acc = (float*)malloc(sizeof(float) * OutC);
#pragma omp for schedule(static)
        for (int64_t fp = 0; fp < frames * hw_out; ++fp) {
            const int64_t f = fp / hw_out;
            const int p = (int)(fp % hw_out);
            const int h0 = p / Dout * stride - pad;
            const int w0 = (p & (Dout - 1)) * stride - pad;
            for (int oc = 0; oc < OutC; ++oc) {
                float aa[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                const int64_t oc_groups = (int64_t)oc * ksq * G;
                for (int k = 0; k < ksq; ++k) {
                    const int hi = h0 + k / ksize, wi = w0 + k % ksize;
                    if (hi < 0 || hi >= Din || wi < 0 || wi >= Din) continue;
                    const int64_t sp = f * hw_in + (int64_t)hi * Din + wi;
                    const uint32_t* xi = in + sp * (InC >> 3);
                    const int8_t* xs = in_s + sp * G;
                    for (int g = 0; g < G; ++g) {
                        const int64_t wg = oc_groups + (int64_t)k * G + g;
                        int ps = 0;
                        for (int i = 0; i < 4; ++i) ps += orc_dot8(xi[g * 4 + i], w[wg * 4 + i]);
                        aa[k & 3] = fmaf(orc_dequantize_scale(xs[g]), orc_dequantize_scale(w_s[wg]) * (float)ps, aa[k & 3]);
                    }
                }
                acc[oc] = aa[0] + aa[1] + aa[2] + aa[3];
            }
            orc_conv_epilogue(acc, bias, OutC, act, out + fp * (OutC >> 3), out_s + fp * (OutC >> 5));
        }
        free(acc);
    }
}

/* ------------------------------------------------------------------ A5 */
void orc_conv_dw(const uint32_t* in, const int8_t* in_s, const uint32_t* w,
                 const int8_t* w_s, const float* bias, uint32_t* out,
                 int8_t* out_s, int64_t frames, int C, int ksize, int stride,
                 int Din, int Dout)
{
    const int G = C >> 5, ksq = ksize * ksize, pad = ksize >> 1;
    const int64_t hw_in = (int64_t)Din * Din, hw_out = (int64_t)Dout * Dout;
#pragma omp parallel for schedule(static)
    for (int64_t fp = 0; fp < frames * hw_out; ++fp) {
        const int64_t f = fp / hw_out;
        const int p = (int)(fp % hw_out);
        const int h0 = p / Dout * stride - pad;
        const int w0 = (p & (Dout - 1)) * stride - pad;
        for (int g = 0; g < G; ++g) {
            float v[32];
            float amax = NAN; /* the reference reduces |v| by a lane butterfly: NaN only if every value is */
            for (int l = 0; l < 32; ++l) {
                const int c = (g << 5) + l;
                float a = bias[c];
                float aa[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                for (int k = 0; k < ksq; ++k) {
                    const int hi = h0 + k / ksize, wi = w0 + k % ksize;
                    const int valid = hi >= 0 && hi < Din && wi >= 0 && wi < Din;
                    float xv = 0.0f;
                    if (valid) {
                        const int64_t sp = f * hw_in + (int64_t)hi * Din + wi;
                        xv = (float)orc_nib(in[sp * (C >> 3) + (c >> 3)], c & 7) * orc_dequantize_scale(in_s[sp * G + g]);
                    } else {
                        xv = 0.0f * orc_dequantize_scale(0);
                    }
                    const int64_t wi_abs = (int64_t)k * C + c;
                    const float wv = (float)orc_nib(w[wi_abs >> 3], (int)(wi_abs & 7)) * orc_dequantize_scale(w_s[wi_abs >> 5]);
                    aa[k & 3] = fmaf(xv, wv, aa[k & 3]);
                }
                a += aa[0] + aa[1] + aa[2] + aa[3];
                v[l] = a;
                amax = fmaxf(amax, fabsf(a));
            }
            const float scale = amax < ORC_EPS ? 1.0f : amax;
            const float inv = ORC_QMAX * orc_rcp(scale);
            uint32_t wd[4] = {0, 0, 0, 0};
            for (int l = 0; l < 32; ++l) wd[l >> 3] |= orc_q_rn(v[l], inv) << ((l & 7) << 2);
            memcpy(out + fp * (C >> 3) + g * 4, wd, 16);
            out_s[fp * G + g] = orc_quantize_scale(scale);
        }
    }
}

/* ------------------------------------------------------------------ A6 */
void orc_residual(const uint32_t* main_in, const int8_t* main_s,
                  const uint32_t* res, const int8_t* res_s, uint32_t* out,
                  int8_t* out_s, int64_t positions, int C, float main_mult,
                  int skipped)
{
    const int G = C >> 5;
#pragma omp parallel
    {
        float* r = (float*)malloc(sizeof(float) * C);
#pragma omp for schedule(static)
        for (int64_t p = 0; p < positions; ++p) {
            float amax = 0.0f;
            for (int g = 0; g < G; ++g) {
                const float s_res = orc_dequantize_scale(res_s[p * G + g]);
                const float s_in = skipped ? 0.0f : orc_dequantize_scale(main_s[p * G + g]) * main_mult;
                for (int l = 0; l < 32; ++l) {
                    const int c = (g << 5) + l;
                    const int64_t wi = p * (C >> 3) + (c >> 3);
                    const float qi = skipped ? 0.0f : (float)orc_nib(main_in[wi], c & 7);
                    const float qr = (float)orc_nib(res[wi], c & 7);
                    const float v = fmaf(qi, s_in, qr * s_res);
                    r[c] = v;
                    amax = fmaxf(amax, fabsf(v));
                }
            }
            const float scale = amax < ORC_EPS ? 1.0f : amax;
            const float inv = ORC_QMAX * orc_rcp(scale);
            const int8_t sq = orc_quantize_scale(scale);
            for (int g = 0; g < G; ++g) {
                uint32_t wd[4] = {0, 0, 0, 0};
                for (int l = 0; l < 32; ++l) wd[l >> 3] |= orc_q_rn(r[(g << 5) + l], inv) << ((l & 7) << 2);
                memcpy(out + p * (C >> 3) + g * 4, wd, 16);
                out_s[p * G + g] = sq;
            }
        }
        free(r);
    }
}

/* ------------------------------------------------------------------ A8 */
static void orc_gap_partials(const uint32_t* in, const int8_t* in_s, int64_t f,
                             int HW, int C, int c, float* blocks_out, int* nblocks)
{
    const int G = C >> 5, g = c >> 5;
    int nb = 0;
    for (int start = 0; start < HW; start += 16) {
        const int end = start + 16 < HW ? start + 16 : HW;
        float s = 0.0f;
        for (int i = start; i < end; ++i) {
            const int64_t sp = f * HW + i;
            s = fmaf((float)orc_nib(in[sp * (C >> 3) + (c >> 3)], c & 7), orc_dequantize_scale(in_s[sp * G + g]), s);
        }
        blocks_out[nb++] = s;
    }
    *nblocks = nb;
}

void orc_gap_f32(const uint32_t* in, const int8_t* in_s, int64_t frames,
                 int HW, int C, float* out)
{
    const float inv = orc_rcp((float)HW);
#pragma omp parallel
    {
        float* blocks = (float*)malloc(sizeof(float) * ((HW + 15) / 16));
#pragma omp for schedule(static)
        for (int64_t fc = 0; fc < frames * C; ++fc) {
            const int64_t f = fc / C;
            const int c = (int)(fc % C);
            int nb = 0;
            orc_gap_partials(in, in_s, f, HW, C, c, blocks, &nb);
            float acc = 0.0f;
            for (int b = 0; b < nb; ++b) acc = acc + blocks[b] * inv;
            out[fc] = acc;
        }
        free(blocks);
    }
}

void orc_gap_f16(const uint32_t* in, const int8_t* in_s, int64_t frames,
                 int HW, int C, uint16_t* out)
{
    const float inv = orc_rcp((float)HW);
#pragma omp parallel
    {
        float* blocks = (float*)malloc(sizeof(float) * ((HW + 15) / 16));
#pragma omp for schedule(static)
        for (int64_t fc = 0; fc < frames * C; ++fc) {
            const int64_t f = fc / C;
            const int c = (int)(fc % C);
            int nb = 0;
            orc_gap_partials(in, in_s, f, HW, C, c, blocks, &nb);
            uint16_t acc = 0; /* fp16 atomicAdd on a zero pool, block order */
            for (int b = 0; b < nb; ++b) {
                const uint16_t add = orc_float_to_half(blocks[b] * inv);
                acc = orc_float_to_half(orc_half_to_float(acc) + orc_half_to_float(add));
            }
            out[fc] = acc;
        }
        free(blocks);
    }
}

/* ------------------------------------------------------------------ A9 */
int64_t orc_mamba_blob_elems(int D, int d_state, int out)
{
    const int64_t E = 2LL * D;
    return E * (2 + 32 + 4LL * d_state + out); /* mamba_layer.h:58 */
}

static inline float orc_blob_dq(const uint32_t* blob, const int8_t* blob_s, int64_t idx)
{
    return (float)orc_nib(blob[idx >> 3], (int)(idx & 7)) * orc_dequantize_scale(blob_s[idx >> 5]);
}

void orc_ssm_scan(const uint32_t* x, const int8_t* x_s, const uint32_t* blob,
                  const int8_t* blob_s, int D, int d_state, int out, float* h,
                  float* y, int B, int T)
{
    orc_ssm_scan_traced(x, x_s, blob, blob_s, D, d_state, out, h, NULL, y, B, T);
}

void orc_ssm_scan_traced(const uint32_t* x, const int8_t* x_s, const uint32_t* blob,
                         const int8_t* blob_s, int D, int d_state, int out, float* h,
                         float* tr, float* y, int B, int T)
{
    (void)out;
    const int E = 2 * D, N = d_state, P = d_state >> 5;
    const int64_t offB = E, offCre = 33LL * E, offCim = offCre + (int64_t)E * N;
    const int64_t offAre = offCim + (int64_t)E * N, offAim = offAre + (int64_t)E * N;
    const int64_t offD = offAim + (int64_t)E * N;
    const int Gx = D >> 5;
#pragma omp parallel
    {
        float* are = (float*)malloc(sizeof(float) * P);
        float* aim = (float*)malloc(sizeof(float) * P);
        float* cre = (float*)malloc(sizeof(float) * P);
        float* cim = (float*)malloc(sizeof(float) * P);
        float* yacc = (float*)malloc(sizeof(float) * P);
#pragma omp for schedule(static)
        for (int64_t bc = 0; bc < (int64_t)B * E; ++bc) {
            const int b = (int)(bc / E), ch = (int)(bc % E);
            const int lane = ch & 31, in_ch = ch & (D - 1);
            for (int c = 0; c < P; ++c) { /* kernels.h:1108-1120 */
                const int64_t w_off = (int64_t)ch * N + lane + (c << 5);
                are[c] = -expf(orc_blob_dq(blob, blob_s, offAre + w_off));
                aim[c] = orc_blob_dq(blob, blob_s, offAim + w_off);
                cre[c] = orc_blob_dq(blob, blob_s, offCre + w_off);
                cim[c] = orc_blob_dq(blob, blob_s, offCim + w_off);
            }
            const int64_t brow = offB + (int64_t)(ch >> 5) * 1024 + lane * 32; /* kernels.h:1122-1125 */
            const int8_t b_scale = blob_s[brow >> 5];
            const uint32_t* bw = blob + (brow >> 3);
            const float wd = orc_blob_dq(blob, blob_s, ch);
            const float dq = orc_blob_dq(blob, blob_s, offD + ch);
            float* hs = h + ((int64_t)b * E + ch) * P * 2;
            /* trace_A, trace_B, trace_Delta: [3][B][E][P] complex, the layout of h */
            float* ta = tr ? tr + ((int64_t)b * E + ch) * P * 2 : NULL;
            float* tb = tr ? ta + (int64_t)B * E * P * 2 : NULL;
            float* td = tr ? tb + (int64_t)B * E * P * 2 : NULL;
            for (int t = 0; t < T; ++t) {
                const int64_t row = (int64_t)b * T + t;
                const uint32_t* xw = x + row * (D >> 3) + (in_ch >> 5) * 4;
                const int8_t xs = x_s[row * Gx + (in_ch >> 5)];
                int dot = 0;
                for (int i = 0; i < 4; ++i) dot += orc_dot8(xw[i], bw[i]);
                const float x_local = (float)orc_nib(xw[(in_ch & 31) >> 3], in_ch & 7) * orc_dequantize_scale(xs);
                const float bx = (float)dot * (orc_dequantize_scale(xs) * orc_dequantize_scale(b_scale));
                const float u = x_local * wd;
                const float dt = u + logf(1.0f + expf(-fabsf(u))); /* kernels.h:1139 */
                const float dt_half = dt * 0.5f;
                for (int c = 0; c < P; ++c) { /* kernels.h:1146-1173 (the traces when tr is given) */
                    const float dim = -dt_half * aim[c];
                    const float dre = fmaf(-dt_half, are[c], 1.0f);
                    const float inv_s = orc_rcp(fmaf(dre, dre, fmaf(dim, dim, ORC_EPS)));
                    const float ire = dre * inv_s;
                    const float iim = -dim * inv_s;
                    const float nre = fmaf(dt_half, are[c], 1.0f);
                    const float abr = fmaf(nre, ire, dim * iim);
                    const float abi = fmaf(nre, iim, -dim * ire);
                    const float dtbx = dt * bx;
                    const float hr = hs[2 * c], hi = hs[2 * c + 1];
                    const float nhr = fmaf(abr, hr, fmaf(-abi, hi, dtbx * ire));
                    const float nhi = fmaf(abr, hi, fmaf(abi, hr, dtbx * iim));
                    hs[2 * c] = nhr;
                    hs[2 * c + 1] = nhi;
                    if (tr) { /* kernels.h:1158-1170, from the state before the step */
                        const float i2_re = fmaf(ire, ire, -iim * iim);
                        const float i2_im = 2.0f * ire * iim;
                        const float za_re = fmaf(dt_half, bx, hr);
                        const float dt_i2_za_re = dt * fmaf(i2_re, za_re, -i2_im * hi);
                        const float dt_i2_za_im = dt * fmaf(i2_re, hi, i2_im * za_re);
                        const float zdt_re = fmaf(are[c], hr, fmaf(-aim[c], hi, bx));
                        const float zdt_im = fmaf(are[c], hi, aim[c] * hr);
                        const float d_dt_re = fmaf(i2_re, zdt_re, -i2_im * zdt_im);
                        const float d_dt_im = fmaf(i2_re, zdt_im, i2_im * zdt_re);
                        float* t3[3] = {ta + 2 * c, tb + 2 * c, td + 2 * c};
                        const float ur[3] = {dt_i2_za_re, dt * ire, d_dt_re};
                        const float ui[3] = {dt_i2_za_im, dt * iim, d_dt_im};
                        for (int k = 0; k < 3; ++k) {
                            const float r = t3[k][0], i = t3[k][1];
                            t3[k][0] = fmaf(abr, r, fmaf(-abi, i, ur[k]));
                            t3[k][1] = fmaf(abr, i, fmaf(abi, r, ui[k]));
                        }
                    }
                    yacc[c] = fmaf(nhr, cre[c], -nhi * cim[c]);
                }
                float ys = 0.0f;
                for (int c = 0; c < P; ++c) ys += yacc[c];
                y[row * E + ch] = fmaf(dq, x_local, ys);
            }
        }
        free(are); free(aim); free(cre); free(cim); free(yacc);
    }
}

/* ------------------------------------------------------------------ A10 */
void orc_outproj(const float* y, const uint32_t* blob, const int8_t* blob_s,
                 const float* bias, int D, int d_state, int out, int act,
                 int64_t rows, float* o)
{
    const int E = 2 * D;
    const int64_t offW = 34LL * E + 4LL * E * d_state;
    const float inv_div = orc_rcp((float)(out < ORC_CPB ? out : ORC_CPB));
#pragma omp parallel
    {
        float* acc = (float*)malloc(sizeof(float) * out);
#pragma omp for schedule(static)
        for (int64_t r = 0; r < rows; ++r) {
            const float* yr = y + r * E;
            for (int oc = 0; oc < out; ++oc) {
                float a = 0.0f;
                for (int ic = 0; ic < E; ic += 32) {
                    const int64_t woff = offW + (int64_t)oc * E + ic;
                    const uint32_t* ww = blob + (woff >> 3);
                    float gs[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                    for (int w = 0; w < 4; ++w)
                        for (int i = 0; i < 8; ++i)
                            gs[i & 3] = fmaf(yr[ic + 8 * w + i], (float)orc_nib(ww[w], i), gs[i & 3]);
                    a = fmaf(gs[0] + gs[1] + gs[2] + gs[3], orc_dequantize_scale(blob_s[woff >> 5]), a);
                }
                acc[oc] = a;
            }
            for (int c0 = 0; c0 < out; c0 += ORC_CPB) {
                float inv_rms = 1.0f;
                if (out >= 2) {
                    float warp_part[32];
                    for (int w = 0; w < 32; ++w) warp_part[w] = 0.0f;
                    for (int w = 0; w < ORC_CPB / 32; ++w) {
                        const int base = c0 + w * 32;
                        if (base >= out) break;
                        float sq[32];
                        for (int l = 0; l < 32; ++l) sq[l] = base + l < out ? acc[base + l] * acc[base + l] : 0.0f;
                        warp_part[w] = orc_xor_reduce_sum(sq, 16);
                    }
                    const float block_sq = orc_xor_reduce_sum(warp_part, (ORC_CPB / 32) >> 1);
                    inv_rms = orc_rsqrt(fmaf(block_sq, inv_div, ORC_EPS));
                }
                for (int oc = c0; oc < c0 + ORC_CPB && oc < out; ++oc) {
                    const float v = fmaf(acc[oc], inv_rms, bias[oc]);
                    o[r * out + oc] = act == 0 ? v : (act == 1 ? orc_silu(v) : orc_sigmoid(v));
                }
            }
        }
        free(acc);
    }
}

/* ------------------------------------------------------------------ A13 */
void orc_critic(const uint16_t* x, const float* w1, const float* wl,
                const float* w2, int in, int units, float* h, float* score,
                int B, int T)
{
    orc_critic_traced(x, w1, wl, w2, in, units, h, NULL, NULL, score, B, T);
}

void orc_critic_traced(const uint16_t* x, const float* w1, const float* wl,
                       const float* w2, int in, int units, float* h, float* trace_w1,
                       float* trace_l, float* score, int B, int T)
{
#pragma omp parallel
    {
        float* xf = (float*)malloc(sizeof(float) * in);
#pragma omp for schedule(static)
        for (int b = 0; b < B; ++b) {
            float* hb = h + (int64_t)b * units * 2;
            for (int t = 0; t < T; ++t) {
                const int64_t row = (int64_t)b * T + t;
                for (int c = 0; c < in; ++c) xf[c] = orc_half_to_float(x[row * in + c]);
                for (int j = 0; j < units; ++j) { /* kernels.h:1685-1732 */
                    float vr[32], vi[32], lr[32], li[32];
                    for (int l = 0; l < 32; ++l) {
                        float ar = 0.0f, ai = 0.0f, br = 0.0f, bi = 0.0f;
                        for (int c = l; c < in; c += 32) {
                            const int64_t i1 = ((int64_t)c * units + j) << 1;
                            const int64_t il = ((int64_t)j * in + c) << 1;
                            ar = fmaf(xf[c], w1[i1], ar);
                            ai = fmaf(xf[c], w1[i1 + 1], ai);
                            br = fmaf(xf[c], wl[il], br);
                            bi = fmaf(xf[c], wl[il + 1], bi);
                        }
                        vr[l] = ar; vi[l] = ai; lr[l] = br; li[l] = bi;
                    }
                    const float accr = orc_down_reduce_sum(vr), acci = orc_down_reduce_sum(vi);
                    const float lamr = orc_down_reduce_sum(lr), lami = orc_down_reduce_sum(li);
                    const float sr = orc_sigmoid(accr), si = orc_sigmoid(acci);
                    const float lam_mod = sqrtf(fmaf(lamr, lamr, fmaf(lami, lami, ORC_EPS)));
                    const float lam = orc_sigmoid(lam_mod);
                    const float dh = 1.0f - lam;
                    const float actr = accr * sr, acti = acci * si;
                    const float hr = hb[2 * j], hi = hb[2 * j + 1];
                    hb[2 * j] = fmaf(hr, lam, dh * actr);
                    hb[2 * j + 1] = fmaf(hi, lam, dh * acti);
                    if (trace_w1) { /* kernels.h:1731-1751: eligibility traces of w1 and w_lambda */
                        float* tw = trace_w1 + (int64_t)b * in * units * 2;
                        float* tl = trace_l + (int64_t)b * in * units * 2;
                        const float inv = orc_rcp(lam_mod);
                        const float gr = dh * sr * fmaf(accr, 1.0f - sr, 1.0f);
                        const float gi = dh * si * fmaf(acci, 1.0f - si, 1.0f);
                        const float dlam = (hr - actr + hi - acti) * lam * dh * inv;
                        for (int c = 0; c < in; ++c) {
                            const int64_t i1 = ((int64_t)c * units + j) << 1;
                            const int64_t il = ((int64_t)j * in + c) << 1;
                            tw[i1] = fmaf(tw[i1], lam, gr * xf[c]);
                            tw[i1 + 1] = fmaf(tw[i1 + 1], lam, gi * xf[c]);
                            tl[il] = fmaf(tl[il], lam, dlam * xf[c] * lamr);
                            tl[il + 1] = fmaf(tl[il + 1], lam, dlam * xf[c] * lami);
                        }
                    }
                }
                /* criticFwd2Kernel (kernels.h:1754-1778), blockDim == units */
                float warp_sums[32];
                for (int w = 0; w < 32; ++w) warp_sums[w] = 0.0f;
                const int nw = units >> 5;
                for (int w = 0; w < nw; ++w) {
                    float ls[32];
                    for (int l = 0; l < 32; ++l) {
                        const int i = w * 32 + l;
                        ls[l] = fmaf(hb[2 * i], w2[2 * i], fmaf(hb[2 * i + 1], w2[2 * i + 1], 0.0f));
                    }
                    warp_sums[w] = orc_down_reduce_sum(ls);
                }
                score[row] = orc_down_reduce_sum(warp_sums);
            }
        }
        free(xf);
    }
}

/* ------------------------------------------------------------------ A12 */
void orc_set_actions(const float* probs, int64_t rows, int A, uint64_t* actions)
{
    const int words = (A + 63) >> 6;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        uint64_t* ar = actions + r * words;
        for (int w = 0; w < words; ++w) ar[w] = 0;
        for (int idx = 0; idx < A; ++idx) {
            const float v = probs[r * A + idx];
            const int32_t seed_in = ((int32_t)(v * ORC_FMAXIMUM)) ^ idx;
            const int set = orc_uniform(orc_unique_seed((uint32_t)idx, seed_in), 1.0f) < v;
            if (set) ar[idx >> 6] |= 1ULL << (idx & 63);
        }
    }
}

/* ------------------------------------------------------------------ A14 */
/* Audio front-end (ca.cu:4-20, 76-117; kernels.h:1420-1459, 1566-1652) in
 * emulated fp16: every fp16 operation is computed in float (exact for the
 * product of two halves) and rounded to half, as the GPU does per op. */
static inline uint16_t orc_hmul(uint16_t a, uint16_t b) { return orc_float_to_half(orc_half_to_float(a) * orc_half_to_float(b)); }
static inline uint16_t orc_hadd(uint16_t a, uint16_t b) { return orc_float_to_half(orc_half_to_float(a) + orc_half_to_float(b)); }
static inline uint16_t orc_hsub(uint16_t a, uint16_t b) { return orc_float_to_half(orc_half_to_float(a) - orc_half_to_float(b)); }

void orc_audio_pcm_to_half(const int16_t* pcm, int n, uint16_t* out)
{
    const uint16_t inv = orc_float_to_half(1.0f / 32768.0f);
    for (int i = 0; i < n; ++i) out[i] = orc_hmul(orc_float_to_half((float)pcm[i]), inv);
}

void orc_resize_half(const uint16_t* src, uint16_t* dst, int src_h, int src_w, int dst_dim, int channels)
{
    const float scale = (float)src_w / (float)dst_dim;
    for (int c = 0; c < channels; ++c) {
        const uint16_t* s = src + (int64_t)c * src_w * src_h;
        for (int y = 0; y < dst_dim; ++y) {
            const float ys = fmaf((float)y + 0.5f, scale, -0.5f);
            const float fy = floorf(ys);
            const int y1 = fy > 0.0f ? (int)fy : 0;
            const float wy = ys - fy;
            const int r1 = y1 * src_w, r2 = (y1 + 1 < src_h - 1 ? y1 + 1 : src_h - 1) * src_w;
            for (int x = 0; x < dst_dim; ++x) {
                const float xs = fmaf((float)x + 0.5f, scale, -0.5f);
                const float fx = floorf(xs);
                const float wx = xs - fx;
                const int x1 = fx > 0.0f ? (int)fx : 0;
                const int x2 = x1 + 1 < src_w - 1 ? x1 + 1 : src_w - 1;
                const float v11 = orc_half_to_float(s[r1 + x1]);
                const float v21 = orc_half_to_float(s[r2 + x1]);
                const float top = fmaf(wx, orc_half_to_float(s[r1 + x2]) - v11, v11);
                const float res = fmaf(wy, fmaf(wx, orc_half_to_float(s[r2 + x2]) - v21, v21) - top, top);
                dst[(int64_t)c * dst_dim * dst_dim + (int64_t)y * dst_dim + x] = orc_float_to_half(res);
            }
        }
    }
}

/* radix-2 DIT on n complex halves (re, im interleaved), input in natural order */
static void orc_fft_half(uint16_t* z, int n)
{
    int log2n = 0;
    while ((1 << log2n) < n) ++log2n;
    uint16_t* t = (uint16_t*)malloc(sizeof(uint16_t) * 2 * n);
    for (int i = 0; i < n; ++i) {
        int r = 0;
        for (int b = 0; b < log2n; ++b) r |= ((i >> b) & 1) << (log2n - 1 - b);
        t[2 * r] = z[2 * i];
        t[2 * r + 1] = z[2 * i + 1];
    }
    for (int s = 1; s <= log2n; ++s) {
        const int m = 1 << s, half_m = m >> 1;
        for (int b = 0; b < n / 2; ++b) {
            const int local = b % half_m;
            const int u = b / half_m * m + local, v = u + half_m;
            const float arg = (-6.2831853f * (float)local) / (float)m;
            const uint16_t wr = orc_float_to_half(cosf(arg)), wi = orc_float_to_half(sinf(arg));
            /* complex_mul_half2 (kernels.h:98-102) */
            const uint16_t ar = t[2 * v], ai = t[2 * v + 1];
            const uint16_t tr = orc_hsub(orc_hmul(ar, wr), orc_hmul(ai, wi));
            const uint16_t ti = orc_hadd(orc_hmul(ai, wr), orc_hmul(ar, wi));
            const uint16_t ur = t[2 * u], ui = t[2 * u + 1];
            t[2 * u] = orc_hadd(ur, tr);
            t[2 * u + 1] = orc_hadd(ui, ti);
            t[2 * v] = orc_hsub(ur, tr);
            t[2 * v + 1] = orc_hsub(ui, ti);
        }
    }
    memcpy(z, t, sizeof(uint16_t) * 2 * n);
    free(t);
}

/* fftRowKernel: row r = complex pairs of in[2nr .. 2nr + 2n) (in holds 2 n^2 halves) */
void orc_fft_rows(const uint16_t* in, int n, uint16_t* out)
{
#pragma omp parallel for schedule(static)
    for (int r = 0; r < n; ++r) {
        memcpy(out + (int64_t)r * 2 * n, in + (int64_t)r * 2 * n, sizeof(uint16_t) * 2 * n);
        orc_fft_half(out + (int64_t)r * 2 * n, n);
    }
}

/* fftColumnKernel, out of place: planes [2][n][n] = |X| / n^2, atan2(im, re) */
void orc_fft_cols(const uint16_t* in, int n, uint16_t* planes)
{
    const float norm = 1.0f / ((float)n * (float)n);
#pragma omp parallel
    {
        uint16_t* col = (uint16_t*)malloc(sizeof(uint16_t) * 2 * n);
#pragma omp for schedule(static)
        for (int x = 0; x < n; ++x) {
            for (int r = 0; r < n; ++r) {
                col[2 * r] = in[((int64_t)r * n + x) * 2];
                col[2 * r + 1] = in[((int64_t)r * n + x) * 2 + 1];
            }
            orc_fft_half(col, n);
            for (int r = 0; r < n; ++r) {
                const float re = orc_half_to_float(col[2 * r]), im = orc_half_to_float(col[2 * r + 1]);
                planes[(int64_t)r * n + x] = orc_float_to_half(sqrtf(fmaf(re, re, im * im)) * norm);
                planes[(int64_t)n * n + (int64_t)r * n + x] = orc_float_to_half(atan2f(im, re));
            }
        }
        free(col);
    }
}

/* ------------------------------------------------------------------ F2 */
/* Screen front-end (cs.cu:5-45): kernels.h:38-45 bounded xorshift hash. */
static uint32_t orc_bounded_hash(uint32_t seed, uint32_t n)
{
    seed ^= seed << 13;
    seed ^= seed >> 17;
    seed ^= seed << 5;
    return (uint32_t)(((uint64_t)seed * n) >> 32);
}

/* A double rounded to the nearest binary16 (ties to even), as fp16 bits. */
static uint16_t orc_double_to_half(double r)
{
    if (r == 0.0) return signbit(r) ? 0x8000u : 0u;
    int e;
    frexp(fabs(r), &e);                       /* |r| in [2^(e-1), 2^e) */
    int ulp_exp = (e - 1) - 10;               /* 11 significant bits */
    if (ulp_exp < -24) ulp_exp = -24;          /* subnormal spacing */
    const double n = nearbyint(ldexp(r, -ulp_exp));
    return orc_float_to_half((float)ldexp(n, ulp_exp));  /* exact in float and half */
}

/* __hfma: a*b + c with one rounding; exact in double for the operands here
 * (the products and sums of halves span well under 53 bits). */
static uint16_t orc_hfma(uint16_t a, uint16_t b, uint16_t c)
{
    return orc_double_to_half((double)orc_half_to_float(a) * (double)orc_half_to_float(b) + (double)orc_half_to_float(c));
}

/* bgra [pixels] (4 bytes each) -> planes [4][pixels] as fp16 bits
 * (ProcessBgraToRgbOP cs.cu:12-31, AugmentBrightnessContrastOP cs.cu:40-44). */
void orc_screen_frontend(const uint8_t* bgra, int pixels, int train, uint32_t frame_seed, float brightness,
                         float contrast, uint16_t* planes)
{
    const uint16_t h_half = orc_float_to_half(0.5f), one = orc_float_to_half(1.0f);
    const uint16_t c = orc_float_to_half(contrast);
    const uint16_t offset = orc_float_to_half(0.5f + orc_half_to_float(orc_float_to_half(brightness)));
    for (int idx = 0; idx < pixels; ++idx) {
        uint8_t px[4] = {bgra[4 * idx], bgra[4 * idx + 1], bgra[4 * idx + 2], bgra[4 * idx + 3]};
        if (train) {
            const uint32_t r = orc_bounded_hash(frame_seed ^ (uint32_t)idx, 10000u);
            if (r < 50u) px[0] = px[1] = px[2] = 0;
            else if (r < 100u) px[0] = px[1] = px[2] = 255;
        }
        for (int ch = 0; ch < 4; ++ch) {
            uint16_t v = orc_float_to_half((float)px[ch] * (1.0f / 255.0f));
            if (train) {
                const uint16_t d = orc_float_to_half(orc_half_to_float(v) - orc_half_to_float(h_half));
                v = orc_hfma(d, c, offset);
                if (orc_half_to_float(v) > 1.0f) v = one;  /* __hmin2(., 1) */
                if (!(orc_half_to_float(v) > 0.0f)) v = 0; /* __hmax2(., +0) */
            }
            planes[(int64_t)ch * pixels + idx] = v;
        }
    }
}
