/*
 * CPU oracle for the AICortex inference hot path -- TEST INFRASTRUCTURE ONLY.
 *
 * This is a plain-C restatement of the reference's forward kernels
 * (AICortex kernels.h and the layer/block composition headers), used as the
 * checker for the CUDA product and as the timed CPU baseline. It is never
 * linked into the product library. Only tests/, __graft_entry__.smoke() and
 * bench.py (its cpu_baseline leg and its `--impl reference` arm) load it.
 *
 * Each function cites the reference file:line it follows. Arithmetic is
 * carried out in float with explicit fmaf() in the reference's order; the
 * only deliberate differences from the GPU reference are the fast-math
 * intrinsics (__expf, __logf, __log2f, sqrt.approx), which are replaced by
 * libm and agree to ~1e-7 relative.
 *
 * Packed int4 activation/weight format ("F"): 32 signed nibbles per group
 * stored as 4 little-endian u32 words (element i in word i>>3, bits 4*(i&7)),
 * one int8 log2 exponent per group; dequantised value q * max(2^s/7, 2^-13)
 * (kernels.h:56-85).
 */
#ifndef AIC_ORACLE_H
#define AIC_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* --- format primitives (kernels.h:21-85) --- */
uint32_t orc_unique_seed(uint32_t global_tid, int32_t sample_index);
float orc_uniform(uint32_t seed, float n);
int8_t orc_quantize_scale(float scale);
float orc_dequantize_scale(int8_t s);
float orc_half_to_float(uint16_t h);
uint16_t orc_float_to_half(float f);

/* A1: quantizeKernel (kernels.h:116-145). n must be a multiple of 32.
 * stochastic != 0 reproduces the weight packer with the reference launch
 * geometry (global thread id == group index). */
void orc_pack_f32(const float* in, int64_t n, uint32_t* out, int8_t* scales,
                  int stochastic, int32_t add_idx);

/* A2: quantizeNCHWtoNHWCKernel<half, true> (kernels.h:146-195) over a batch of
 * frames. planes: [frames][planes_present][dim][dim] fp16 bits; channels
 * planes_present..channels-1 are zero. Output NHWC F [frames*dim*dim][channels]. */
void orc_stem_pack(const uint16_t* planes, int64_t frames, int planes_present,
                   int channels, int dim, uint32_t* out, int8_t* out_s);

/* A4: convPointwiseFwdKernel (kernels.h:217-282). act: 1 = SiLU, 0 = none. */
void orc_conv_pw(const uint32_t* in, const int8_t* in_s, const uint32_t* w,
                 const int8_t* w_s, const float* bias, uint32_t* out,
                 int8_t* out_s, int64_t positions, int InC, int OutC, int act);

/* A3: convDenseFwdKernel (kernels.h:514-585); weights [OutC][k*k][InC]. */
void orc_conv_dense(const uint32_t* in, const int8_t* in_s, const uint32_t* w,
                    const int8_t* w_s, const float* bias, uint32_t* out,
                    int8_t* out_s, int64_t frames, int InC, int OutC, int ksize,
                    int stride, int Din, int Dout, int act);

/* A5: convDepthwiseFwdKernel (kernels.h:831-870); weights [k*k][C]. */
void orc_conv_dw(const uint32_t* in, const int8_t* in_s, const uint32_t* w,
                 const int8_t* w_s, const float* bias, uint32_t* out,
                 int8_t* out_s, int64_t frames, int C, int ksize, int stride,
                 int Din, int Dout);

/* A6: residualAddFwdKernel (kernels.h:989-1055), one scale per position. */
void orc_residual(const uint32_t* main_in, const int8_t* main_s,
                  const uint32_t* res, const int8_t* res_s, uint32_t* out,
                  int8_t* out_s, int64_t positions, int C, float main_mult,
                  int skipped);

/* A8: gapKernel<float> (kernels.h:1653-1684): out [frames][C] fp32, 16-position
 * partial sums added in block order. */
void orc_gap_f32(const uint32_t* in, const int8_t* in_s, int64_t frames,
                 int HW, int C, float* out);
/* gapKernel<__half> on an all-zero pool (critic.h:108-111): out fp16 bits. */
void orc_gap_f16(const uint32_t* in, const int8_t* in_s, int64_t frames,
                 int HW, int C, uint16_t* out);

/* Mamba blob helpers (mamba_layer.h:58, kernels.h:1084-1089, 1192). */
int64_t orc_mamba_blob_elems(int D, int d_state, int out);

/* A9: mambaSSMFwdStateKernel (kernels.h:1080-1187) run for T steps over B
 * independent sequences. x: F [B*T][D] (row = b*T + t); h: compact state
 * [B][E][d_state/32] complex (float pairs), updated in place; y: [B*T][E]. */
void orc_ssm_scan(const uint32_t* x, const int8_t* x_s, const uint32_t* blob,
                  const int8_t* blob_s, int D, int d_state, int out, float* h,
                  float* y, int B, int T);
/* The same with the training-mode eligibility traces (kernels.h:1158-1170):
 * tr = trace_A | trace_B | trace_Delta, each [B][E][d_state/32] complex like h,
 * updated in place (tr may be NULL). */
void orc_ssm_scan_traced(const uint32_t* x, const int8_t* x_s, const uint32_t* blob,
                         const int8_t* blob_s, int D, int d_state, int out, float* h,
                         float* tr, float* y, int B, int T);

/* A10: mambaSSMFwdOutProjKernel<act> (kernels.h:1188-1259) over rows. */
void orc_outproj(const float* y, const uint32_t* blob, const int8_t* blob_s,
                 const float* bias, int D, int d_state, int out, int act,
                 int64_t rows, float* o);

/* A13: criticFwd1Kernel + criticFwd2Kernel (kernels.h:1685-1778) for T steps
 * over B sequences. x: fp16 [B*T][in]; w1 [in][units][2]; wl [units][in][2];
 * w2 [units][2]; h: [B][units][2] in/out; score: [B*T]. */
void orc_critic(const uint16_t* x, const float* w1, const float* wl,
                const float* w2, int in, int units, float* h, float* score,
                int B, int T);
/* The same with the traces (kernels.h:1731-1751): trace_w1 [B][in][units][2]
 * (the layout of w1) and trace_l [B][units][in][2] (the layout of wl), updated
 * in place (both NULL for none). */
void orc_critic_traced(const uint16_t* x, const float* w1, const float* wl,
                       const float* w2, int in, int units, float* h, float* trace_w1,
                       float* trace_l, float* score, int B, int T);

/* A12: setActionsKernel (kernels.h:1473-1485) per row of A probabilities.
 * actions: [rows][(A+63)/64] words, cleared first. */
void orc_set_actions(const float* probs, int64_t rows, int A,
                     uint64_t* actions);

/* A14: audio front-end (ca.cu:4-20, 76-117; kernels.h:1420-1459, 1566-1652),
 * fp16 values as IEEE half bits. */
void orc_audio_pcm_to_half(const int16_t* pcm, int n, uint16_t* out);
void orc_resize_half(const uint16_t* src, uint16_t* dst, int src_h, int src_w, int dst_dim, int channels);
/* in: 2 n^2 halves (row r pairs elements 2nr + 2k, +1); out: n x n complex (re, im) */
void orc_fft_rows(const uint16_t* in, int n, uint16_t* out);
/* in: n x n complex; planes: [2][n][n] = |X|/n^2, atan2(im, re) */
void orc_fft_cols(const uint16_t* in, int n, uint16_t* planes);

/* F2: screen front-end (cs.cu:5-45): bgra [pixels][4] -> fp16 bits [4][pixels]. */
void orc_screen_frontend(const uint8_t* bgra, int pixels, int train, uint32_t frame_seed, float brightness,
                         float contrast, uint16_t* planes);

int orc_num_threads(void);

/* ---- training path (aic_oracle_train.c) ---- */
void orc_sgd_update(float* data, const float* grad, int64_t n, float factor, float lr, float penalty);
float orc_clip_factor(const float* g, int64_t n, int blocks, float* sum_out);
void orc_conv_backward(const uint32_t* in, const int8_t* in_s, const uint32_t* w, const int8_t* w_s,
                       const float* bias, const float* master, const float* dy, int InC, int OutC, int ks,
                       int stride, int Din, int Dout, int act, float* gw, float* gb, float* grad_in);
void orc_mamba_backward(const uint32_t* in, const int8_t* in_s, const float* h, const float* ta, const float* tb,
                        const float* td, const float* m, const float* bias, const float* dy, int D, int N, int OutC,
                        int act, float* gw, float* gb, float* grad_in);
void orc_critic_backward(const float* w2, const float* tw1, const float* tl, const float* hidden, float pred,
                         float real, int units, int in, float* gw1, float* gl, float* gw2);

#ifdef __cplusplus
}
#endif
#endif
