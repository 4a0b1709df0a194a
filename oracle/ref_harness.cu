// Reference-kernel harness -- TEST INFRASTRUCTURE ONLY.
//
// Compiled by oracle/build_ref.sh against the reference's own kernels.h (and
// the uv.h / device_constants.h / base_constants.h it pulls in), with the
// reference build flags (-O3 --use_fast_math --extended-lambda), into
// oracle/_ref/libaicref_D<d_model>_N<d_state>.so. Each entry point launches
// one reference kernel with exactly the launch geometry the reference layer
// classes use (file:line cited per function) on raw device pointers, so the
// golden-vector generator (tests/golden/make_golden.py) can drive the
// reference kernels one at a time. Nothing in the product links this.
//
// The Mamba kernels read d_model / d_inner / d_state from compile-time
// constants (kernels.h:1080-1089), which is why one library is built per
// (d_model, d_state) pair.
#include "kernels.h"
#include "ca.cu"      // AudioProcessorOP (ca.cu:4-20)
#include "cs_ops.h"   // ProcessBgraToRgbOP, AugmentBrightnessContrastOP (cs.cu:5-45), cut by build_ref.sh

#define AICREF_API extern "C" __attribute__((visibility("default")))

static int aicref_status() { return (int)cudaGetLastError(); }

AICREF_API int aicref_d_model() { return final_channels; }
AICREF_API int aicref_d_state() { return mamba_d_state; }

// conv_layer.h:98 / mamba_layer.h:137 (weights, stochastic, add_idx = n) and
// mamba_block.h:64,70 (activations, round-to-nearest, add_idx = 0).
AICREF_API int aicref_quantize_f32(const float* in, uint32_t* out, int8_t* scales, int n, int stochastic, int add_idx)
{
    const int groups = n >> 5;
    const int grid = (groups + gpu_block_threads - 1) / gpu_block_threads;
    if (stochastic) quantizeKernel<float, false><<<grid, gpu_block_threads>>>(in, out, scales, n, add_idx);
    else quantizeKernel<float, true><<<grid, gpu_block_threads>>>(in, out, scales, n, add_idx);
    return aicref_status();
}

// cortex.h:294-295: one fp16 NCHW frame [channels][dim][dim] -> NHWC int4.
AICREF_API int aicref_stem(const __half* in, uint32_t* out, int8_t* out_s, int dim, int channels)
{
    dim3 grid((dim + 31) >> 5, dim, channels >> 5);
    quantizeNCHWtoNHWCKernel<__half><<<grid, gpu_block_threads>>>(in, out, out_s, dim, channels, 0);
    return aicref_status();
}

// conv_layer.h:145-147 (one frame of `positions` pixels).
AICREF_API int aicref_conv_pw(const uint32_t* in, const int8_t* in_s, const uint32_t* w, const int8_t* w_s, const float* bias,
                              uint32_t* out, int8_t* out_s, int positions, int InC, int OutC, int act)
{
    dim3 grid(positions, (OutC + gpu_block_threads - 1) / gpu_block_threads);
    if (act) convPointwiseFwdKernel<false><<<grid, gpu_block_threads>>>(in, w, in_s, w_s, bias, out, out_s, InC, OutC);
    else convPointwiseFwdKernel<true><<<grid, gpu_block_threads>>>(in, w, in_s, w_s, bias, out, out_s, InC, OutC);
    return aicref_status();
}

// conv_layer.h:118-142 (one frame).
AICREF_API int aicref_conv_dense(const uint32_t* in, const int8_t* in_s, const uint32_t* w, const int8_t* w_s, const float* bias,
                                 uint32_t* out, int8_t* out_s, int InC, int OutC, int ksize, int stride, int Din, int Dout, int act)
{
    dim3 grid(Dout * Dout, (OutC + gpu_block_threads - 1) / gpu_block_threads);
#define AICREF_DENSE(NOACT, K) convDenseFwdKernel<NOACT, K><<<grid, gpu_block_threads>>>(in, w, in_s, w_s, bias, out, out_s, InC, OutC, Din, Dout, stride)
    if (ksize == 2) { if (act) AICREF_DENSE(false, 2); else AICREF_DENSE(true, 2); }
    else if (ksize == 4) { if (act) AICREF_DENSE(false, 4); else AICREF_DENSE(true, 4); }
    else return -1;
#undef AICREF_DENSE
    return aicref_status();
}

// conv_layer.h:104-116 (one frame).
AICREF_API int aicref_conv_dw(const uint32_t* in, const int8_t* in_s, const uint32_t* w, const int8_t* w_s, const float* bias,
                              uint32_t* out, int8_t* out_s, int C, int ksize, int stride, int Din, int Dout)
{
    dim3 grid(Dout * Dout, (C + gpu_block_threads - 1) / gpu_block_threads);
#define AICREF_DW(K) convDepthwiseFwdKernel<K><<<grid, gpu_block_threads>>>(in, w, in_s, w_s, bias, out, out_s, C, Din, Dout, stride)
    if (ksize == 3) AICREF_DW(3);
    else if (ksize == 5) AICREF_DW(5);
    else if (ksize == 7) AICREF_DW(7);
    else return -1;
#undef AICREF_DW
    return aicref_status();
}

// conv_block.h:80-81 (dim x dim positions) and mamba_block.h:65 (dim = 1).
AICREF_API int aicref_residual(const uint32_t* main_in, const int8_t* main_s, const uint32_t* res, const int8_t* res_s,
                               uint32_t* out, int8_t* out_s, int C, int dim, float survival_prob_inv, int skipped, float residual_factor)
{
    dim3 grid(dim, dim);
    residualAddFwdKernel<><<<grid, gpu_block_threads, C * sizeof(float)>>>(main_in, main_s, res, res_s, out, out_s, C, dim,
                                                                         survival_prob_inv, skipped != 0, residual_factor);
    return aicref_status();
}

// critic.h:108-111; the caller zeroes `pooled` (critic.h:108).
AICREF_API int aicref_gap_f32(const uint32_t* in, const int8_t* in_s, float* pooled, int spatial, int C)
{
    dim3 grid(((C >> 5) + gpu_block_threads - 1) / gpu_block_threads, (spatial + 15) >> 4);
    gapKernel<float><<<grid, gpu_block_threads>>>(in, in_s, pooled, spatial, C);
    return aicref_status();
}
AICREF_API int aicref_gap_f16(const uint32_t* in, const int8_t* in_s, __half* pooled, int spatial, int C)
{
    dim3 grid(((C >> 5) + gpu_block_threads - 1) / gpu_block_threads, (spatial + 15) >> 4);
    gapKernel<__half><<<grid, gpu_block_threads>>>(in, in_s, pooled, spatial, C);
    return aicref_status();
}

// mamba_layer.h:141 -- one time step of one sequence. h/trace buffers are
// [d_inner][d_state] complex; y is [d_inner].
AICREF_API int aicref_ssm_step(const uint32_t* in, const int8_t* in_s, const uint32_t* w, const int8_t* w_s, float2* h,
                               float2* tr_a, float2* tr_b, float2* tr_d, float* y)
{
    mambaSSMFwdStateKernel<><<<mamba_d_inner / gpu_block_threads, gpu_block_threads>>>(in, in_s, w, w_s, h, tr_a, tr_b, tr_d, y);
    return aicref_status();
}

// mamba_layer.h:142-145.
AICREF_API int aicref_outproj(const float* y, const uint32_t* w, const int8_t* w_s, const float* bias, float* out, int OutC, int act)
{
    const int grid = (OutC + gpu_block_threads - 1) / gpu_block_threads;
    if (act == 0) mambaSSMFwdOutProjKernel<0><<<grid, gpu_block_threads>>>(y, w, w_s, bias, out, OutC);
    else if (act == 1) mambaSSMFwdOutProjKernel<1><<<grid, gpu_block_threads>>>(y, w, w_s, bias, out, OutC);
    else mambaSSMFwdOutProjKernel<2><<<grid, gpu_block_threads>>>(y, w, w_s, bias, out, OutC);
    return aicref_status();
}

// critic.h:112-114 -- one time step; units complex units, `in` fp16 inputs.
AICREF_API int aicref_critic(const __half* pooled, const float* w1, const float* wl, const float* w2, float* h,
                             float* trace_w1, float* trace_l, float* score, int units, int in)
{
    criticFwd1Kernel<__half><<<((units << 5) + gpu_block_threads - 1) / gpu_block_threads, gpu_block_threads>>>(
        pooled, w1, wl, h, trace_w1, trace_l, units, in);
    criticFwd2Kernel<><<<1, units>>>(h, w2, score, units);
    return aicref_status();
}

// cortex.h:371-372 -- `actions` must be zeroed by the caller.
AICREF_API int aicref_set_actions(const float* probs, unsigned long long* actions, int count)
{
    setActionsKernel<float><<<(count + gpu_block_threads - 1) / gpu_block_threads, gpu_block_threads>>>(
        probs, reinterpret_cast<action_type*>(actions), count);
    return aicref_status();
}

// ca.cu:106: 2048 int16 samples -> fp16 through AudioProcessorOP.
AICREF_API int aicref_audio_convert(const short* pcm, __half* out)
{
    AudioProcessorOP op{out, pcm};
    forEachNUniversalVectorKernel<<<1, gpu_block_threads>>>(op, 2048 >> 3);
    return aicref_status();
}

// ca.cu:107,112 launch geometry: 16x16 blocks, two outputs per thread.
AICREF_API int aicref_resize(const __half* src, __half* dst, int src_h, int src_w, int dst_dim, int channels)
{
    dim3 block(16, 16);
    dim3 grid(dst_dim / (block.x << 1), dst_dim / block.y, channels);
    resizeKernel<__half><<<grid, block>>>(src, dst, src_h, src_w, dst_dim, channels);
    return aicref_status();
}

// ca.cu:108-109 with an input of 2 x 1024 x 1024 halves (rows 512.. read the upper half).
AICREF_API int aicref_fft_rows(const __half* in, __half2* out)
{
    fftRowKernel<1024><<<1024, gpu_block_threads>>>(in, out);
    return aicref_status();
}

// ca.cu:110, out of place: out holds 2 x 1024 x 1024 halves (|X|/N^2, phase).
AICREF_API int aicref_fft_cols(const __half2* in, __half* out)
{
    fftColumnKernel<1024><<<1024, gpu_block_threads>>>(in, out);
    return aicref_status();
}

template <typename Op>
__global__ void aicref_elementwise(Op op, int n)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) op(i);
}

// cs.cu:116: BGRA8 [pixels] -> fp16 planes [4][pixels] (train: pixel dropout seeded by frame_seed).
AICREF_API int aicref_screen(const uchar4* bgra, __half* out, int pixels, unsigned frame_seed, int train)
{
    ProcessBgraToRgbOP op{bgra, out, pixels, frame_seed, train != 0};
    aicref_elementwise<<<(pixels + 255) / 256, 256>>>(op, pixels);
    return aicref_status();
}

// cs.cu:117-122: the augmentation over `pairs` half2 of the planes.
AICREF_API int aicref_augment(__half2* v, int pairs, float brightness, float contrast)
{
    AugmentBrightnessContrastOP op{v, __float2half2_rn(brightness), __float2half2_rn(contrast)};
    aicref_elementwise<<<(pairs + 255) / 256, 256>>>(op, pairs);
    return aicref_status();
}

// ---- training path (F4)

// updateParamsKernel, launched as conv_layer.h:214-216.
AICREF_API int aicref_update_params(float* data, const float* grad, int n, float grad_norm_factor, float lr, float penalty)
{
    updateParamsKernel<><<<(n + gpu_block_threads - 1) / gpu_block_threads, gpu_block_threads>>>(data, grad, n, grad_norm_factor,
                                                                                                 lr, penalty);
    return aicref_status();
}

// universal_vector::transform_reduce(SquareOp) (uv.h:230-248) over a device
// array: the same kernel and grid, result copied to *out.
AICREF_API int aicref_sum_sq(const float* x, int n, float* out)
{
    static float* d_res = nullptr;
    if (!d_res && cudaMalloc(&d_res, sizeof(float)) != cudaSuccess) return -1;
    int dev = 0, sms = 0, tpm = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&tpm, cudaDevAttrMaxThreadsPerMultiProcessor, dev);
    size_t per_sm = tpm / gpu_block_threads;
    if (per_sm < 1) per_sm = 1;
    const size_t opt = sms * per_sm, need = (static_cast<size_t>(n) + gpu_block_threads - 1) / gpu_block_threads;
    const size_t blocks = std::max<size_t>(1, std::min(opt, need));
    cudaMemset(d_res, 0, sizeof(float));
    transformReduceKernel<float, float, SquareOp<float>><<<blocks, gpu_block_threads>>>(x, d_res, SquareOp<float>{}, n);
    if (cudaMemcpy(out, d_res, sizeof(float), cudaMemcpyDeviceToHost) != cudaSuccess) return -2;
    return aicref_status();
}

// The gradient kernels of ConvLayer::backward (conv_layer.h:152-206), same
// launch geometry; grad_in is accumulated into (dense / pointwise) or written
// (depthwise) as the reference does.
AICREF_API int aicref_conv_bwd(const uint32_t* in, const int8_t* in_s, const uint32_t* w, const int8_t* w_s, const float* bias,
                               const float* master, const float* grad_out, float* grad_in, float* gw, float* gb, int InC,
                               int OutC, int ks, int stride, int Din, int Dout, int act)
{
    const int T = gpu_block_threads;
    if (ks > 1 && (ks & 1)) {
        dim3 grid_b((InC + T - 1) / T), grid_w(grid_b.x), grid_i(Din * Din, grid_b.x);
        convDepthwiseBwdGradBiasKernel<><<<grid_b, T>>>(grad_out, gb, InC, Dout * Dout);
#define AICREF_DWB(K) convDepthwiseBwdGradWeightKernel<K><<<grid_w, T>>>(in, in_s, grad_out, gw, InC, Din, Dout, stride); \
                      convDepthwiseBwdGradInputKernel<K><<<grid_i, T>>>(grad_out, master, grad_in, InC, Din, Dout, stride)
        if (ks == 3) { AICREF_DWB(3); } else if (ks == 5) { AICREF_DWB(5); } else if (ks == 7) { AICREF_DWB(7); } else return -1;
#undef AICREF_DWB
    } else if ((ks & 1) == 0) {
        dim3 grid_b((OutC + T - 1) / T), grid_w((OutC + T - 1) / T, InC), grid_i(Dout * Dout, (OutC + T - 1) / T);
#define AICREF_DB(NOACT, K) \
    convDenseBwdGradBiasKernel<NOACT, K><<<grid_b, T>>>(in, in_s, w, w_s, bias, grad_out, gb, InC, OutC, Din, Dout, stride); \
    convDenseBwdGradWeightKernel<NOACT, K><<<grid_w, T>>>(in, in_s, w, w_s, bias, grad_out, gw, InC, OutC, Din, Dout, stride); \
    convDenseBwdGradInputKernel<NOACT, K><<<grid_i, T>>>(in, in_s, w, w_s, bias, grad_out, master, grad_in, InC, OutC, Din, Dout, stride)
        if (ks == 2) { if (act) { AICREF_DB(false, 2); } else { AICREF_DB(true, 2); } }
        else if (ks == 4) { if (act) { AICREF_DB(false, 4); } else { AICREF_DB(true, 4); } }
        else return -1;
#undef AICREF_DB
    } else {
        dim3 grid_b((OutC + T - 1) / T);
        dim3 block_w(dim_block_pw_bwd_gw_size, dim_block_pw_bwd_gw_size);
        dim3 grid_w(OutC / dim_block_pw_bwd_gw_size, InC / dim_block_pw_bwd_gw_size);
        dim3 grid_in(Dout * Dout, grid_b.x);
        const int nhw = Dout * Dout;
        if (act) {
            convPointwiseBwdGradBiasKernel<false><<<grid_b, T>>>(in, in_s, w, w_s, bias, grad_out, gb, InC, OutC, nhw);
            convPointwiseBwdGradWeightKernel<false><<<grid_w, block_w>>>(in, in_s, w, w_s, bias, grad_out, gw, InC, OutC, nhw);
            convPointwiseBwdGradInputKernel<false><<<grid_in, T>>>(in, in_s, w, w_s, bias, grad_out, master, grad_in, InC, OutC);
        } else {
            convPointwiseBwdGradBiasKernel<true><<<grid_b, T>>>(in, in_s, w, w_s, bias, grad_out, gb, InC, OutC, nhw);
            convPointwiseBwdGradWeightKernel<true><<<grid_w, block_w>>>(in, in_s, w, w_s, bias, grad_out, gw, InC, OutC, nhw);
            convPointwiseBwdGradInputKernel<true><<<grid_in, T>>>(in, in_s, w, w_s, bias, grad_out, master, grad_in, InC, OutC);
        }
    }
    return aicref_status();
}

// conv_block.h:89 residualAddBwdKernel over dim x dim positions.
AICREF_API int aicref_residual_bwd(float* grad_next, float* grad_res, int C, int dim, float survival_prob_inv, float residual_factor)
{
    residualAddBwdKernel<><<<dim3(dim, dim), gpu_block_threads>>>(grad_next, grad_res, C, dim, survival_prob_inv, residual_factor);
    return aicref_status();
}

// The gradient kernels of MambaLayer::backward (mamba_layer.h:148-157); the
// caller zeroes raw_out, gw, gb and grad_in first (:148-151).
AICREF_API int aicref_mamba_bwd(const uint32_t* in, const int8_t* in_s, const float2* h, const float2* ta, const float2* tb,
                                const float2* td, const float* master, const float* bias, const float* grad_out, float* raw_out,
                                float* gw, float* gb, float* grad_in, int OutC, int act)
{
    dim3 proj_grid(OutC >> 5, mamba_d_inner / gpu_block_threads, 1);
    mambaSSMBwdOutProjKernel<><<<proj_grid, gpu_block_threads>>>(in, in_s, h, master, raw_out, OutC);
    const int act_grid = (OutC + gpu_block_threads - 1) / gpu_block_threads;
    if (act == 0) mambaSSMBwdNormActKernel<0><<<act_grid, gpu_block_threads>>>(raw_out, bias, grad_out, gb, OutC);
    else if (act == 1) mambaSSMBwdNormActKernel<1><<<act_grid, gpu_block_threads>>>(raw_out, bias, grad_out, gb, OutC);
    else mambaSSMBwdNormActKernel<2><<<act_grid, gpu_block_threads>>>(raw_out, bias, grad_out, gb, OutC);
    mambaSSMApplyTracesKernel<><<<mamba_d_inner / gpu_block_threads, gpu_block_threads>>>(in, in_s, raw_out, h, ta, tb, td, master,
                                                                                         gw, grad_in, OutC);
    return aicref_status();
}

// The gradient kernels of Critic::backward (critic.h:120-121); w1 / wl are
// [in][units] / [units][in] complex, `out_channels` 2 * units.
AICREF_API int aicref_critic_bwd(const float* w2, const float* trace_w1, const float* trace_l, const float* hidden, float* gw1,
                                 float* gl, float* gw2, float pred, float real, int units, int in)
{
    const int real_size = 2 * units * in;
    criticApplyTracesKernel<><<<((real_size >> 1) + gpu_block_threads - 1) / gpu_block_threads, gpu_block_threads>>>(
        w2, trace_w1, trace_l, gw1, gl, pred, real, units, in);
    criticOutputGradKernel<><<<(units + gpu_block_threads - 1) / gpu_block_threads, gpu_block_threads>>>(hidden, gw2, pred, real,
                                                                                                         units);
    return aicref_status();
}

AICREF_API int aicref_sync() { return (int)cudaDeviceSynchronize(); }
