// Host-side launchers for the CUDA kernels of the inference path. Every
// launcher is asynchronous on `stream`, validates nothing beyond what it needs
// to size its grid (the C-ABI layer validates arguments) and returns the
// launch status.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_fp16.h>

namespace aic {

// A1: fp32 [n] -> packed int4 groups (n % 32 == 0). stochastic != 0 selects
// the weight packer (position hash seeded with add_idx). The hash uses the
// group index modulo row_groups (0 = no wrap) as the reference's thread index,
// so a batch of rows packs each row as one reference call would.
cudaError_t launch_pack_f32(const float* in, int64_t n, uint32_t* out, int8_t* out_s, bool stochastic,
                            int32_t add_idx, int64_t row_groups, cudaStream_t stream);

// A2: fp16 planes [frames][planes][dim][dim] (channels >= planes are zero)
// -> NHWC packed int4 [frames*dim*dim][channels].
cudaError_t launch_stem_pack(const __half* planes, int64_t frames, int planes_present, int channels, int dim,
                             uint32_t* out, int8_t* out_s, cudaStream_t stream);

// A5: depthwise k x k conv (k in {3,5,7}), stride 1/2, pad k/2, + bias, requant.
// wf: weights dequantised by launch_dw_weights ([k*k][C] fp32).
cudaError_t launch_dw_weights(const uint32_t* w, const int8_t* w_s, int64_t n, float* wf, cudaStream_t stream);
cudaError_t launch_conv_dw(const uint32_t* in, const int8_t* in_s, const float* wf, const float* bias, uint32_t* out,
                           int8_t* out_s, int64_t frames, int C, int ksize, int stride, int Din, int Dout,
                           cudaStream_t stream);
// The same conv with one thread per (output pixel, 8 channels) and no tiling
// (strides other than 1 and 2; the reference-structure cross-check).
cudaError_t launch_conv_dw_direct(const uint32_t* in, const int8_t* in_s, const float* wf, const float* bias,
                                  uint32_t* out, int8_t* out_s, int64_t frames, int C, int ksize, int stride, int Din,
                                  int Dout, cudaStream_t stream);

// A3/A4 on CUDA cores: quantized conv (pointwise when ksize == 1) with the fused
// RMSNorm(256-chunk) + bias (+SiLU) + requant epilogue; reproduces the
// reference accumulation order exactly.
cudaError_t launch_conv_gemm_simt(const uint32_t* in, const int8_t* in_s, const uint32_t* w, const int8_t* w_s,
                                  const float* bias, uint32_t* out, int8_t* out_s, int64_t frames, int InC,
                                  int OutC, int ksize, int stride, int Din, int Dout, bool act, cudaStream_t stream);

// A3/A4 on the tensor cores (tcgen05, TMEM accumulator) with the same fused
// epilogue. Weights come as swizzled bf16 images built by launch_build_wimg.
size_t conv_tc_wimg_bytes(int in_c, int out_c, int ksize);
cudaError_t launch_build_wimg(const uint32_t* w, const int8_t* w_s, int in_c, int out_c, int ksize, uint8_t* img,
                              cudaStream_t stream);
cudaError_t launch_conv_gemm_tc(const uint32_t* in, const int8_t* in_s, const uint8_t* wimg, const float* bias,
                                uint32_t* out, int8_t* out_s, int64_t frames, int in_c, int out_c, int ksize, int din,
                                int dout, bool act, int* err, cudaStream_t stream);

// A3/A4 on the tensor cores in the reference's accumulation order (exact
// integer dots from the MMA, the fp32 fmaf chain over groups on CUDA cores):
// bit-identical to the reference. ksize 1 or 2 (conv_tc_ord_supported).
bool conv_tc_ord_supported(int ksize);
size_t conv_tc_ord_wimg_bytes(int in_c, int out_c, int ksize);
cudaError_t launch_build_wimg_ord(const uint32_t* w, const int8_t* w_s, int in_c, int out_c, int ksize, uint8_t* img,
                                  cudaStream_t stream);
cudaError_t launch_conv_gemm_tc_ord(const uint32_t* in, const int8_t* in_s, const uint8_t* wimg, const float* bias,
                                    uint32_t* out, int8_t* out_s, int64_t frames, int in_c, int out_c, int ksize,
                                    int din, int dout, bool act, int* err, cudaStream_t stream);

// Compares rcp_rn_pos with __frcp_rn over every significand of several
// binades; *mismatches (zeroed by the caller) counts differing results.
cudaError_t launch_selftest_rcp(unsigned long long* mismatches, float* first_bad, cudaStream_t stream);

// Device-side error word written by kernels whose bounded waits time out.
int* device_error_word();
// One CTA waits on an mbarrier nothing arrives on: the bounded wait records
// `code` in the device error word and *returned becomes 1 (2 if it completed).
cudaError_t launch_selftest_wait(int code, int* returned, cudaStream_t stream);

// A6: out = requant(q_main * s_main * main_mult + q_res * s_res), one exponent per position.
cudaError_t launch_residual(const uint32_t* main_in, const int8_t* main_s, const uint32_t* res, const int8_t* res_s,
                            uint32_t* out, int8_t* out_s, int64_t positions, int C, float main_mult, bool skipped,
                            cudaStream_t stream);

// A8: global average pool of [frames][HW][C] -> fp32 [frames][C] (optional)
// and round-to-nearest packed int4 [frames][C] (optional).
cudaError_t launch_gap(const uint32_t* in, const int8_t* in_s, int64_t frames, int HW, int C, float* out_f32,
                       uint32_t* out_q, int8_t* out_qs, cudaStream_t stream);
// gapKernel<__half> semantics: fp16 [frames][C].
cudaError_t launch_gap_f16(const uint32_t* in, const int8_t* in_s, int64_t frames, int HW, int C, __half* out,
                           cudaStream_t stream);

// A9: batched, time-looped SSM scan. x: F [B*T][D] (row b*T+t); consts: per
// channel prepared constants; h: [B][E][P] float2 in/out; y: [B*T][E].
cudaError_t launch_ssm_prepare(const uint32_t* blob, const int8_t* blob_s, int D, int d_state, float* consts,
                               cudaStream_t stream);
size_t ssm_consts_floats(int D, int d_state);
// traces: nullptr, or trace_A | trace_B | trace_Delta [3][B][E][d_state/32]
// complex, advanced with the state (training-mode forward, kernels.h:1158-1170).
// split: y as two bf16 planes hi | lo [B*T][E] (the tensor-core out-projection's
// operands) instead of fp32 [B*T][E]; both take B*T*E*4 bytes.
cudaError_t launch_ssm_scan(const uint32_t* x, const int8_t* x_s, const uint32_t* blob, const int8_t* blob_s,
                            const float* consts, int D, int d_state, float2* h, float2* traces, void* y, bool split,
                            int B, int T, cudaStream_t stream);

// A10: out-projection GEMM y[rows][E] x W_out -> RMSNorm(256-chunk) + bias + act -> fp32 [rows][out].
cudaError_t launch_outproj(const float* y, const uint32_t* blob, const int8_t* blob_s, const float* bias, int D,
                           int d_state, int out, int act, int64_t rows, float* o, cudaStream_t stream);

// A10 on the tensor cores (k_outproj_tc.cu): the weight image holds W_out as
// bf16 q * F(s) [out][E] (exact), y comes as the scan's split bf16 planes; two
// MMAs per K step, fp32 accumulation, the same fused epilogue. Supported for
// E % 64 == 0 and out a multiple of 32 that is <= 256 or a multiple of 256.
bool outproj_tc_supported(int E, int out_c);
size_t outproj_tc_wimg_bytes(int E, int out_c);
cudaError_t launch_build_outproj_wimg(const uint32_t* blob, const int8_t* blob_s, int64_t off_w, int E, int out_c,
                                      void* img, cudaStream_t stream);
cudaError_t launch_outproj_tc(const void* y_planes, const void* wimg, const float* bias, int E, int out_c, int act,
                              int64_t rows, float* out, int* err, cudaStream_t stream);

// A13: critic recurrence over T for B sequences; x fp16 [B*T][in]. trace_w1
// [B][in][units] and trace_l [B][units][in] complex: nullptr, or the
// training-mode eligibility traces, advanced in place (kernels.h:1731-1751).
cudaError_t launch_critic(const __half* x, const float* w1, const float* wl, const float* w2, int in, int units,
                          float2* h, float2* h_seq, float2* trace_w1, float2* trace_l, float* score, int B, int T,
                          cudaStream_t stream);

// A14: audio front-end (ca.cu): 2048 int16 PCM samples -> two fp16 planes
// (|X|/N^2, phase of the 1024x1024 fp16 FFT) resized to dim x dim, written to
// channels first_channel and first_channel+1 of an fp16 [C][dim][dim] frame.
size_t audio_workspace_bytes();
cudaError_t launch_audio_frontend(const short* pcm, __half* frame, int dim, int first_channel, void* workspace,
                                  cudaStream_t stream);

// F2: screen front-end (cs.cu): BGRA8 [dim*dim] -> fp16 planes B, G, R, A at
// channels first_channel.. of an fp16 [C][dim][dim] frame; train adds the
// reference's pixel dropout and brightness/contrast augmentation. dim even.
cudaError_t launch_screen_frontend(const uint8_t* bgra, __half* frame, int dim, int first_channel, bool train,
                                   uint32_t frame_seed, float brightness, float contrast, cudaStream_t stream);

// A12: Bernoulli action bits, [rows][A] probabilities -> [rows][(A+63)/64] words.
cudaError_t launch_set_actions(const float* probs, int64_t rows, int A, unsigned long long* actions,
                               cudaStream_t stream);

// F4: training path (k_train.cu), one layer step per call as the reference's
// layer classes run it. Clip factor of a gradient (conv_layer.h:207-213):
// factor[0] = 1/norm above 1, factor[1] = the square sum; partial holds
// sumsq_blocks(n, sms) floats.
int sumsq_blocks(int64_t n, int sms);
cudaError_t launch_clip_factor(const float* x, int64_t n, int sms, float* partial, float* factor, cudaStream_t s);
// updateParamsKernel (kernels.h:196-216) with the factor read from the device.
cudaError_t launch_sgd_update(float* data, const float* grad, int64_t n, const float* factor, float lr, float penalty,
                              cudaStream_t s);
// Gradients of one conv layer on one frame (ConvLayer::backward,
// conv_layer.h:150-206): grad_out [dout^2][out] fp32, input the layer's packed
// forward input; gw / gb written, grad_in [din^2][in] added to (pointwise,
// dense) or written (depthwise), or skipped when null. scratch: 4 *
// dout^2 * out floats (unused by the depthwise conv).
cudaError_t launch_conv_backward_grads(const uint32_t* in, const int8_t* in_s, const uint32_t* w, const int8_t* w_s,
                                       const float* bias, const float* master, const float* dy, int in_c, int out_c,
                                       int ks, int stride, int din, int dout, bool act, float* scratch, float* gw,
                                       float* gb, float* grad_in, cudaStream_t s);
// residualAddBwdKernel (kernels.h:1056-1079) over n floats.
cudaError_t launch_residual_backward(float* grad_next, float* grad_res, int64_t n, float survival_inv,
                                     float residual_factor, cudaStream_t s);
// Gradients of one Mamba layer step (MambaLayer::backward, mamba_layer.h:146-
// 167) of one sequence: h and the traces [E][P] complex after the step;
// master the fp32 blob; gw zeroed here and written, gb written, grad_in [D]
// written. partial: (2D / 256) * out floats, gnorm: out, gx_ch: 2D.
cudaError_t launch_mamba_backward_grads(const uint32_t* in, const int8_t* in_s, const float2* h, const float2* ta,
                                        const float2* tb, const float2* td, const float* master, const float* bias,
                                        const float* dy, int D, int N, int out_c, int act, float* partial,
                                        float* gnorm, float* gx_ch, float* gw, float* gb, float* grad_in,
                                        cudaStream_t s);
// Critic gradients (Critic::backward, critic.h:117-124): gw1 / gl [in][units]
// / [units][in] complex, gw2 [units] complex; units a power of two; pred
// points at the step's score on the device.
cudaError_t launch_critic_backward_grads(const float* w2, const float2* tw1, const float2* tl, const float2* hidden,
                                         const float* pred, float real, int units, int in_c, float* gw1, float* gl, float* gw2,
                                         cudaStream_t s);

}  // namespace aic
