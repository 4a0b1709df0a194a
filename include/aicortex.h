/*
 * aicortex.h -- C ABI of the B200 (sm_100a) implementation of the AICortex
 * inference hot path: quantized conv/residual feature stack -> recurrent
 * complex-diagonal SSM ("Mamba") layers -> actor and critic heads.
 *
 * The ABI mirrors the reference's layer classes and their two-phase
 * construction (a constructor that reports byte counts, then initData()
 * binding views into caller-owned arenas, then forward()), plus the
 * reference's extern "C" opaque-state idiom (create / init / run / free in
 * ca.cu:68-136 and cs.cu:75-136). Every reference forward() gains a batch
 * dimension (independent environments) and a sequence dimension (successive
 * calls of the reference, state carried between them); batch = seq = 1 is
 * exactly one reference call.
 *
 * Rules:
 *  - Functions never throw; they return an aic_status and leave a message for
 *    aic_last_error() (thread-local).
 *  - Tensor arguments are plain device pointers (device memory, or mapped
 *    pinned host memory where noted), borrowed for the duration of the call.
 *    Streams are cudaStream_t passed as void* (NULL = legacy default stream).
 *  - Handles allocate no device memory: the caller queries the bytes needed,
 *    allocates them and binds them (parameters once, recurrent state per batch
 *    size, workspace per call). Every bound pointer must be 256-byte aligned.
 *  - All launches are asynchronous on the given stream; nothing synchronises
 *    except the functions whose name ends in _sync.
 *  - One handle is used by one host thread / stream at a time.
 *
 * Packed int4 format ("F", reference kernels.h:56-85): a group is 32 signed
 * 4-bit codes in four little-endian u32 words (code i in word i>>3, bits
 * 4*(i&7)) and one int8 exponent s; the value of code q is
 * q * max(2^s/7, 2^-13). Activations are NHWC: pixel p, group g -> words
 * [p*C/8 + 4g .. 4g+3], exponent [p*C/32 + g]. Frames are stacked along the
 * pixel axis; a sequence tensor's row for (env b, step t) is b*seq + t.
 */
#ifndef AICORTEX_H
#define AICORTEX_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define AIC_API __attribute__((visibility("default")))
#else
#define AIC_API
#endif

typedef int aic_status;
#define AIC_OK 0
#define AIC_ERR_INVALID 1     /* bad argument, shape or alignment */
#define AIC_ERR_UNSUPPORTED 2 /* configuration the reference does not support either */
#define AIC_ERR_CUDA 3        /* CUDA launch/runtime error */
#define AIC_ERR_STATE 4       /* handle not bound / state not bound */
#define AIC_ERR_IO 5          /* checkpoint file missing, short or unreadable */

AIC_API const char* aic_last_error(void);
AIC_API int aic_abi_version(void);
/* Synchronises the current device and reads (and clears) the device error
 * word that kernels set when a bounded wait on the tensor-core pipeline times
 * out (the kernel then abandons its tile and returns). *code = 0: no error. */
AIC_API aic_status aic_device_error_sync(int* code);

/* ------------------------------------------------------------------------
 * Stateless format kernels
 * ---------------------------------------------------------------------- */

/* quantizeKernel<float, !stochastic> (reference kernels.h:116-145), as used by
 * ConvLayer/MambaLayer weight packing (conv_layer.h:98, mamba_layer.h:137:
 * stochastic, add_idx = n) and by MambaBlock's activation requant
 * (mamba_block.h:64,70: round-to-nearest, add_idx ignored). n % 32 == 0. */
AIC_API aic_status aic_pack_f32(const float* in, int64_t n, uint32_t* out, int8_t* out_s, int stochastic,
                                int32_t add_idx, void* stream);

/* quantizeNCHWtoNHWCKernel<half> (kernels.h:146-195, cortex.h:294-295) over a
 * batch: fp16 planes [frames][planes_present][dim][dim]; channels
 * planes_present..channels-1 are zero (the reference zero-fills its capture
 * buffer, cortex.h:291). Output F [frames*dim*dim][channels]. */
AIC_API aic_status aic_stem_pack(const uint16_t* planes, int64_t frames, int planes_present, int channels, int dim,
                                 uint32_t* out, int8_t* out_s, void* stream);

/* residualAddFwdKernel (kernels.h:989-1055, conv_block.h:80-81,
 * mamba_block.h:65): out = requant(main * main_mult + res) with one exponent
 * per position; main is ignored when skipped != 0. */
AIC_API aic_status aic_residual_add(const uint32_t* main_in, const int8_t* main_s, const uint32_t* res,
                                    const int8_t* res_s, uint32_t* out, int8_t* out_s, int64_t positions, int channels,
                                    float main_mult, int skipped, void* stream);

/* gapKernel<float> (kernels.h:1653-1684): mean over hw pixels of each frame ->
 * fp32 [frames][C] (out_f32 may be NULL) and/or its round-to-nearest F
 * requant [frames][C] (out_q/out_qs may be NULL). */
AIC_API aic_status aic_gap(const uint32_t* in, const int8_t* in_s, int64_t frames, int hw, int channels, float* out_f32,
                           uint32_t* out_q, int8_t* out_qs, void* stream);
/* gapKernel<__half> on a zeroed pool (critic.h:108-111): fp16 bits [frames][C]. */
AIC_API aic_status aic_gap_f16(const uint32_t* in, const int8_t* in_s, int64_t frames, int hw, int channels,
                               uint16_t* out, void* stream);

/* Audio front-end of the reference's capture path (ca.cu:76-117): 2048 int16
 * PCM samples (1024 interleaved stereo frames, device memory) -> fp16 ->
 * bilinear resize to 1024 x 1024 -> 2-D radix-2 fp16 FFT -> |X|/1024^2 and
 * atan2 planes -> bilinear resize to dim x dim, written to channels
 * first_channel and first_channel + 1 of an fp16 frame [C][dim][dim] (the
 * reference uses channels 4 and 5 of its 32-channel stem input, ca.cu:118-125).
 * The reference's row FFT reads past its input for rows 512..1023 and its
 * column FFT overwrites its own input; here those reads see zeros and the
 * column results go to a separate buffer. workspace: aic_audio_workspace_bytes. */
AIC_API aic_status aic_audio_workspace_bytes(size_t* bytes);

/* Numerics self-test of the library's reciprocal (the sigmoid's 1/(1+e)):
 * counts, into the device word *mismatches (zeroed by the caller), the inputs
 * d >= 1 over every significand of ten binades where it differs from the IEEE
 * round-to-nearest reciprocal __frcp_rn; *first_bad (device) gets one such d. */
AIC_API aic_status aic_selftest_rcp(uint64_t* mismatches, float* first_bad, void* stream);
/* The failure path of the kernels' bounded waits, without a GPU fault: one CTA
 * waits on an mbarrier that nothing arrives on; after the wait's limit (about
 * 1 s) it records `code` in the device error word (read and cleared by
 * aic_device_error_sync) and writes 1 to *returned (device int; 2 would mean
 * the wait completed). The context stays usable. */
AIC_API aic_status aic_selftest_wait_timeout(int code, int* returned, void* stream);
AIC_API aic_status aic_audio_frontend(const int16_t* pcm, uint16_t* frame, int dim, int first_channel,
                                      void* workspace, void* stream);

/* Screen front-end (cs.cu:5-45, run_cuda_processing_visual cs.cu:104-123
 * without the D3D11 texture copy): bgra = dim*dim BGRA8 pixels (device), written
 * as fp16 planes byte/255 in byte order B, G, R, A to channels first_channel ..
 * first_channel + 3 of the fp16 frame [C][dim][dim]. train != 0 applies the
 * reference's training-mode pixel dropout, hashed from frame_seed (the
 * reference draws it with generateUniqueSeed), and the brightness/contrast
 * augmentation with the given values (the reference draws them uniformly from
 * +-0.15 and 1 +- 0.2), all in fp16 arithmetic. dim must be even. */
AIC_API aic_status aic_screen_frontend(const uint8_t* bgra, uint16_t* frame, int dim, int first_channel, int train,
                                       uint32_t frame_seed, float brightness, float contrast, void* stream);

/* setActionsKernel (kernels.h:1473-1485, cortex.h:371-372): per row of
 * `count` probabilities, Bernoulli bits into [rows][(count+63)/64] words. */
AIC_API aic_status aic_set_actions(const float* probs, int64_t rows, int count, uint64_t* actions, void* stream);

/* ------------------------------------------------------------------------
 * ConvLayer (conv_layer.h): depthwise (odd k>1), dense (k = 2, 4; stride = k)
 * or pointwise (k = 1) quantized conv with fused RMSNorm(256-channel chunks)
 * + bias (+SiLU) + int4 requant.
 * ---------------------------------------------------------------------- */
typedef struct aic_conv_layer_t* aic_conv_layer;
typedef struct {
    int in_channels, out_channels, kernel_size, stride, dim_in, dim_out;
    int disable_activation; /* reference ctor argument is_activation_disabled */
} aic_conv_layer_desc;

/* ConvLayer ctor (conv_layer.h:45-63). */
AIC_API aic_status aic_conv_layer_create(const aic_conv_layer_desc* desc, aic_conv_layer* out);
/* Byte count the ctor adds to total_mem_main_device (conv_layer.h:59), plus
 * this implementation's tensor-core copy of the weights. */
AIC_API aic_status aic_conv_layer_sizes(aic_conv_layer l, int64_t* weight_elems, int64_t* bias_elems,
                                        size_t* param_bytes);
/* initData arena carve (conv_layer.h:64-77). */
AIC_API aic_status aic_conv_layer_bind(aic_conv_layer l, void* dev_params);
AIC_API aic_status aic_conv_layer_param_ptrs(aic_conv_layer l, uint32_t** weights, int8_t** weight_scales,
                                             float** bias);
/* loadFromFile's device half (conv_layer.h:31-44): fp32 master weights
 * ([out][k*k][in], or [k*k][C] for depthwise) and bias, device-accessible;
 * packs with the reference's stochastic packer, bit-exact. */
AIC_API aic_status aic_conv_layer_load_weights(aic_conv_layer l, const float* master, const float* bias,
                                               void* stream);
/* ConvLayer::loadFromFile (conv_layer.h:31-44): raw little-endian fp32
 * master weights then fp32 bias. Host-side file read + pack. */
AIC_API aic_status aic_conv_layer_load_file_sync(aic_conv_layer l, const char* path, void* stream);
/* ConvLayer::forward (conv_layer.h:102-149) over `frames` frames, in the
 * layer's conv mode (aic_conv_layer_set_mode; default AIC_CONV_ORDERED). */
AIC_API aic_status aic_conv_layer_forward(aic_conv_layer l, const uint32_t* in, const int8_t* in_s, uint32_t* out,
                                          int8_t* out_s, int64_t frames, void* stream);
/* The same conv on CUDA cores with the reference kernels' structure
 * (convPointwiseFwdKernel / convDenseFwdKernel / convDepthwiseFwdKernel),
 * whatever the layer's mode: bit-identical to the reference. */
AIC_API aic_status aic_conv_layer_forward_exact(aic_conv_layer l, const uint32_t* in, const int8_t* in_s,
                                                uint32_t* out, int8_t* out_s, int64_t frames, void* stream);
/* Arithmetic of the pointwise and dense convs (depthwise convs always run on
 * CUDA cores in the reference order):
 *   AIC_CONV_ORDERED (default) tensor cores compute the exact integer group
 *       dots; the fp32 accumulation over groups follows the reference order,
 *       so outputs are bit-identical to the reference (the 4x4 dense conv
 *       runs as AIC_CONV_SIMT);
 *   AIC_CONV_FAST  NOT a parity mode: tensor cores accumulate all of K in
 *       fp32 in MMA order. A layer matches the reference up to that summation
 *       order (a requant code flips where a value sits on a rounding boundary,
 *       about 1e-4 of the codes), but the flips propagate through the stack:
 *       end to end the features drift (mean error ~0.1 of their scale), so
 *       only use it where the reference's bits do not matter;
 *   AIC_CONV_SIMT  CUDA cores, reference order (bit-identical). */
#define AIC_CONV_ORDERED 0
#define AIC_CONV_FAST 1
#define AIC_CONV_SIMT 2
AIC_API aic_status aic_conv_layer_set_mode(aic_conv_layer l, int mode);
AIC_API aic_status aic_conv_layer_destroy(aic_conv_layer l);

/* ------------------------------------------------------------------------
 * ConvBlock (conv_block.h): dw k x k -> pw1 (SiLU) -> pw2, shortcut (1x1 or
 * 2x2/s2), residual add scaled by residual_factor.
 * ---------------------------------------------------------------------- */
typedef struct aic_conv_block_t* aic_conv_block;
typedef struct {
    int in_channels, mid_channels, out_channels, stride, dim_in, dim_out, dw_kernel;
    float survival_probability, residual_factor;
} aic_conv_block_desc;

AIC_API aic_status aic_conv_block_create(const aic_conv_block_desc* desc, aic_conv_block* out);
/* sub-layer i: 0 depthwise, 1 conv_layer1, 2 conv_layer2, 3 residual_layer (conv_block.h:18-21). */
AIC_API aic_status aic_conv_block_layer(aic_conv_block b, int i, aic_conv_layer* out);
AIC_API aic_status aic_conv_block_param_bytes(aic_conv_block b, size_t* bytes);
AIC_API aic_status aic_conv_block_bind(aic_conv_block b, void* dev_params);
/* Ping-pong buffers a/b (conv_block.h:63-66) for `frames` frames. */
AIC_API aic_status aic_conv_block_workspace_bytes(aic_conv_block b, int64_t frames, size_t* bytes);
/* ConvBlock::loadFromFile (conv_block.h:23-29): <dir>/{depthwise_layer,conv_layer1,conv_layer2,residual_layer}.bin */
AIC_API aic_status aic_conv_block_load_dir_sync(aic_conv_block b, const char* dir, void* stream);
/* ConvBlock::forward (conv_block.h:74-82). train_mode/is_survived select the
 * stochastic-depth scaling of the main branch exactly as the reference. */
AIC_API aic_status aic_conv_block_forward(aic_conv_block b, const uint32_t* in, const int8_t* in_s, uint32_t* out,
                                          int8_t* out_s, int64_t frames, int train_mode, int is_survived,
                                          void* workspace, void* stream);
AIC_API aic_status aic_conv_block_destroy(aic_conv_block b);

/* ------------------------------------------------------------------------
 * MambaLayer (mamba_layer.h): recurrent complex-diagonal SSM step + out-proj
 * + RMSNorm(256-chunks) + bias + activation (0 id, 1 SiLU, 2 sigmoid).
 * d_model must be a power of two >= 32 (the reference indexes ch & (D-1));
 * d_state a multiple of 32; channel ch owns the d_state/32 states
 * (ch & 31) + 32c of its row, as the reference kernel does.
 * ---------------------------------------------------------------------- */
typedef struct aic_mamba_layer_t* aic_mamba_layer;
typedef struct {
    int d_model, d_state, out_channels, activation;
} aic_mamba_layer_desc;

AIC_API aic_status aic_mamba_layer_create(const aic_mamba_layer_desc* desc, aic_mamba_layer* out);
/* weight_elems = 2*d_model*(34 + 4*d_state + out) (mamba_layer.h:58). */
AIC_API aic_status aic_mamba_layer_sizes(aic_mamba_layer l, int64_t* weight_elems, int64_t* bias_elems,
                                         size_t* param_bytes);
AIC_API aic_status aic_mamba_layer_bind(aic_mamba_layer l, void* dev_params);
AIC_API aic_status aic_mamba_layer_param_ptrs(aic_mamba_layer l, uint32_t** weights, int8_t** weight_scales,
                                              float** bias);
/* fp32 master blob [W_delta | B_mimo | C_re | C_im | A_re | A_im | D | W_out]
 * (kernels.h:1084-1089) + bias; packs bit-exactly (mamba_layer.h:137). */
AIC_API aic_status aic_mamba_layer_load_weights(aic_mamba_layer l, const float* master, const float* bias,
                                                void* stream);
AIC_API aic_status aic_mamba_layer_load_file_sync(aic_mamba_layer l, const char* path, void* stream);
/* Recurrent state h: [batch][2*d_model][d_state/32] complex fp32 (the active
 * entries of the reference's h_states, mamba_layer.h:90-92). */
AIC_API aic_status aic_mamba_layer_state_bytes(aic_mamba_layer l, int batch, size_t* bytes);
AIC_API aic_status aic_mamba_layer_bind_state(aic_mamba_layer l, void* dev_state, int batch);
/* Training-mode forward (replaces mambaSSMFwdStateKernel's trace arguments,
 * kernels.h:1080, 1158-1170): with traces bound, every forward also advances
 * trace_A, trace_B and trace_Delta, stored back to back, each in the layout of
 * the state ([batch][2*d_model][d_state/32] complex fp32; 3x state_bytes).
 * Bind after aic_mamba_layer_bind_state with the same batch (binding a state
 * unbinds them); NULL unbinds (the inference forward, which skips them). */
AIC_API aic_status aic_mamba_layer_trace_bytes(aic_mamba_layer l, int batch, size_t* bytes);
AIC_API aic_status aic_mamba_layer_bind_traces(aic_mamba_layer l, void* dev_traces, int batch);
/* MambaLayer::reset (mamba_layer.h:171-177): zeroes the state and, if bound,
 * the traces. */
AIC_API aic_status aic_mamba_layer_reset_state(aic_mamba_layer l, void* stream);
/* y_ssm [rows][2*d_model] fp32 (mamba_layer.h:93-95). */
AIC_API aic_status aic_mamba_layer_workspace_bytes(aic_mamba_layer l, int64_t rows, size_t* bytes);
/* MambaLayer::forward (mamba_layer.h:139-146) for `seq` successive steps of
 * `batch` sequences: in F [batch*seq][d_model], out fp32 [batch*seq][out]. */
AIC_API aic_status aic_mamba_layer_forward(aic_mamba_layer l, const uint32_t* in, const int8_t* in_s, float* out,
                                           int batch, int seq, void* workspace, void* stream);
/* aic_mamba_layer_forward without a workspace: no counterpart in the
 * reference. For callers that cannot allocate device memory themselves, for
 * example a real-time control loop that must not call cudaMalloc (it can
 * synchronise the whole device and stall the frame) or a plugin whose host
 * application owns all device memory through its own allocator. The layer's
 * y_ssm scratch is a 4 MiB array compiled into the library, one per device,
 * held from load until process exit; batch * seq * 2 * d_model must not
 * exceed 1,048,576 floats (AIC_ERR_INVALID otherwise). The first call on a
 * device looks up that array's device address (cudaGetSymbolAddress); make
 * that first call before capturing a stream. The address is then kept per
 * device ordinal until the process exits, which assumes that the device's
 * primary context is not reset (cudaDeviceReset) while the library is
 * loaded. All calls share the one array:
 * calls that can overlap on the GPU (different streams, no ordering) race.
 * The scratch is fully overwritten before it is read, so nothing needs
 * clearing between calls. Parameters and state are bound as usual; the
 * caller passes inputs and outputs. */
AIC_API aic_status aic_mamba_layer_forward_noalloc(aic_mamba_layer l, const uint32_t* in, const int8_t* in_s,
                                                   float* out, int batch, int seq, void* stream);
/* The out-projection alone (mambaSSMFwdOutProjKernel, kernels.h:1188-1259):
 * y_ssm fp32 [rows][2*d_model] -> out fp32 [rows][out], on CUDA cores in the
 * reference's accumulation order (bit-identical to the reference kernel). */
AIC_API aic_status aic_mamba_layer_outproj(aic_mamba_layer l, const float* y, float* out, int64_t rows, void* stream);
/* Out-projection arithmetic of a Mamba layer:
 *   AIC_MAMBA_TENSOR (default) tcgen05 GEMM: W_out held exactly as bf16
 *       q * F(s) (the 1/7 of the int4 unit is applied in the epilogue), y as
 *       two bf16 planes hi + lo (16 significant bits), fp32 accumulation;
 *       within about 1e-5 of the output scale of the reference's fp32 chain
 *       (stated tolerance 1e-3). Out channels: a multiple of 32 that is at most
 *       256 or a multiple of 256 (others run as AIC_MAMBA_EXACT).
 *   AIC_MAMBA_EXACT  CUDA cores in the reference's accumulation order:
 *       bit-identical to mambaSSMFwdOutProjKernel.
 * The SSM scan is the reference's arithmetic in both modes. */
#define AIC_MAMBA_TENSOR 0
#define AIC_MAMBA_EXACT 1
AIC_API aic_status aic_mamba_layer_set_mode(aic_mamba_layer l, int mode);
/* The SSM scan alone (mambaSSMFwdStateKernel, kernels.h:1080-1187, over `seq`
 * steps of `batch` sequences; advances the bound state): y 256-byte aligned,
 * batch*seq*2*d_model*4 bytes, written as fp32 [rows][2*d_model] when
 * y_split == 0, else as the bf16 planes hi [rows][2*d_model] then lo. */
AIC_API aic_status aic_mamba_layer_scan(aic_mamba_layer l, const uint32_t* in, const int8_t* in_s, void* y, int batch,
                                        int seq, int y_split, void* stream);
/* The tensor-core out-projection alone over split-bf16 y planes (as
 * aic_mamba_layer_scan writes them with y_split != 0); AIC_ERR_UNSUPPORTED
 * for out channels without a tensor-core tiling. */
AIC_API aic_status aic_mamba_layer_outproj_split(aic_mamba_layer l, const void* y_planes, float* out, int64_t rows,
                                                 void* stream);
AIC_API aic_status aic_mamba_layer_destroy(aic_mamba_layer l);

/* ------------------------------------------------------------------------
 * MambaBlock (mamba_block.h): strategist (SiLU) -> requant -> residual with
 * the block input -> tactic (SiLU) -> requant -> executor (activation).
 * ---------------------------------------------------------------------- */
typedef struct aic_mamba_block_t* aic_mamba_block;
typedef struct {
    int d_model, d_state, out_channels, activation;
    float survival_probability, residual_factor;
} aic_mamba_block_desc;

AIC_API aic_status aic_mamba_block_create(const aic_mamba_block_desc* desc, aic_mamba_block* out);
/* layer i: 0 strategist, 1 tactic, 2 executor (mamba_block.h:18-20). */
AIC_API aic_status aic_mamba_block_layer(aic_mamba_block b, int i, aic_mamba_layer* out);
AIC_API aic_status aic_mamba_block_param_bytes(aic_mamba_block b, size_t* bytes);
AIC_API aic_status aic_mamba_block_bind(aic_mamba_block b, void* dev_params);
AIC_API aic_status aic_mamba_block_state_bytes(aic_mamba_block b, int batch, size_t* bytes);
AIC_API aic_status aic_mamba_block_bind_state(aic_mamba_block b, void* dev_state, int batch);
/* The three layers' traces (aic_mamba_layer_bind_traces), carved in layer order. */
AIC_API aic_status aic_mamba_block_trace_bytes(aic_mamba_block b, int batch, size_t* bytes);
AIC_API aic_status aic_mamba_block_bind_traces(aic_mamba_block b, void* dev_traces, int batch);
AIC_API aic_status aic_mamba_block_reset_state(aic_mamba_block b, void* stream);
AIC_API aic_status aic_mamba_block_workspace_bytes(aic_mamba_block b, int64_t rows, size_t* bytes);
/* MambaBlock::loadFromFile (mamba_block.h:23-27): <dir>/mamba_{strategist,tactic,executor}.bin */
AIC_API aic_status aic_mamba_block_load_dir_sync(aic_mamba_block b, const char* dir, void* stream);
/* MambaBlock::forward (mamba_block.h:58-72): in F [batch*seq][d_model] ->
 * out fp32 [batch*seq][out]. on_training selects the stochastic requant with
 * add_seed, as in the reference. */
AIC_API aic_status aic_mamba_block_forward(aic_mamba_block b, const uint32_t* in, const int8_t* in_s, float* out,
                                           int batch, int seq, int on_training, int add_seed, int is_survived,
                                           void* workspace, void* stream);
/* AIC_MAMBA_* of the block's three layers. */
AIC_API aic_status aic_mamba_block_set_mode(aic_mamba_block b, int mode);
AIC_API aic_status aic_mamba_block_destroy(aic_mamba_block b);

/* ------------------------------------------------------------------------
 * Critic (critic.h): global average pool of an F frame (fp16) -> gated leaky
 * complex recurrent cell (`units` complex units, fp32 weights) -> scalar.
 * ---------------------------------------------------------------------- */
typedef struct aic_critic_t* aic_critic;
typedef struct {
    int in_channels, units, dim_in; /* reference ctor: out_channels = 2*units */
} aic_critic_desc;

AIC_API aic_status aic_critic_create(const aic_critic_desc* desc, aic_critic* out);
AIC_API aic_status aic_critic_param_bytes(aic_critic c, size_t* bytes);
AIC_API aic_status aic_critic_bind(aic_critic c, void* dev_params);
/* W1 [in][units][2], W2 [units][2], Wlambda [units][in][2], fp32 (critic.h:36-38). */
AIC_API aic_status aic_critic_load_weights(aic_critic c, const float* w1, const float* w2, const float* wl,
                                           void* stream);
AIC_API aic_status aic_critic_load_file_sync(aic_critic c, const char* path, void* stream);
AIC_API aic_status aic_critic_state_bytes(aic_critic c, int batch, size_t* bytes);
AIC_API aic_status aic_critic_bind_state(aic_critic c, void* dev_state, int batch);
/* Training-mode forward (criticFwd1Kernel's trace arguments, kernels.h:1685,
 * 1731-1751): with traces bound, every step also advances trace_w1
 * [batch][in][units] then trace_lambda [batch][units][in] complex fp32 (the
 * layouts of W1 and Wlambda, one set per sequence). Bind after
 * aic_critic_bind_state with the same batch; NULL unbinds. Reset zeroes them. */
AIC_API aic_status aic_critic_trace_bytes(aic_critic c, int batch, size_t* bytes);
AIC_API aic_status aic_critic_bind_traces(aic_critic c, void* dev_traces, int batch);
AIC_API aic_status aic_critic_reset_state(aic_critic c, void* stream);
AIC_API aic_status aic_critic_workspace_bytes(aic_critic c, int64_t rows, size_t* bytes);
/* Critic::forward (critic.h:106-116) for `seq` steps of `batch` sequences:
 * in F [batch*seq][dim_in*dim_in][in], score fp32 [batch*seq]. */
AIC_API aic_status aic_critic_forward(aic_critic c, const uint32_t* in, const int8_t* in_s, float* score, int batch,
                                      int seq, void* workspace, void* stream);
/* criticFwd1Kernel + criticFwd2Kernel on already pooled fp16 features
 * [batch*seq][in] (critic.h:112-114 after the pooling step). */
AIC_API aic_status aic_critic_forward_pooled(aic_critic c, const uint16_t* pooled, float* score, int batch, int seq,
                                             void* workspace, void* stream);
AIC_API aic_status aic_critic_destroy(aic_critic c);

/* ------------------------------------------------------------------------
 * Cortex forward (cortex.h:281-303 composition): stem pack -> conv blocks ->
 * global average pool -> requant -> Mamba units (layer + requant + residual)
 * -> actor layer, and the critic on the trunk output.
 * ---------------------------------------------------------------------- */
typedef struct aic_cortex_t* aic_cortex;
#define AIC_MAX_BLOCKS 16
typedef struct {
    int planes, stem_channels, dim;          /* input fp16 planes, stem channels, input H = W */
    int n_blocks;
    aic_conv_block_desc blocks[AIC_MAX_BLOCKS];
    int d_model, d_state, n_units;           /* Mamba trunk: n_units x (layer D->D SiLU + requant + residual) */
    float unit_residual_factor;
    int actor_out, actor_activation;         /* actor MambaLayer D -> actor_out */
    int critic_units;                        /* 0 = no critic */
    int chunk_frames;                        /* frames per conv-stack pass (0 = 2048) */
} aic_cortex_desc;

AIC_API aic_status aic_cortex_create(const aic_cortex_desc* desc, aic_cortex* out);
AIC_API aic_status aic_cortex_block(aic_cortex c, int i, aic_conv_block* out);
AIC_API aic_status aic_cortex_unit(aic_cortex c, int i, aic_mamba_layer* out);
AIC_API aic_status aic_cortex_actor(aic_cortex c, aic_mamba_layer* out);
AIC_API aic_status aic_cortex_critic(aic_cortex c, aic_critic* out);
AIC_API aic_status aic_cortex_param_bytes(aic_cortex c, size_t* bytes);
AIC_API aic_status aic_cortex_bind(aic_cortex c, void* dev_params);
AIC_API aic_status aic_cortex_state_bytes(aic_cortex c, int batch, size_t* bytes);
AIC_API aic_status aic_cortex_bind_state(aic_cortex c, void* dev_state, int batch);
AIC_API aic_status aic_cortex_reset_state(aic_cortex c, void* stream);
AIC_API aic_status aic_cortex_workspace_bytes(aic_cortex c, int batch, int seq, size_t* bytes);
/* planes fp16 [batch*seq][planes][dim][dim]; actor fp32 [batch*seq][actor_out];
 * critic fp32 [batch*seq] (may be NULL); features (optional) F [batch*seq][d_model]. */
AIC_API aic_status aic_cortex_forward(aic_cortex c, const uint16_t* planes, int batch, int seq, float* actor,
                                      float* critic, uint32_t* features, int8_t* features_s, void* workspace,
                                      void* stream);
/* Host-buffer variant for callers holding the frames in pinned host memory:
 * planes_host [batch*seq][planes][dim][dim] fp16 is copied chunk by chunk on
 * an internal copy stream, overlapped with the conv stack of the previous
 * chunk; actor_host / critic_host (pinned, critic may be NULL) receive the
 * outputs. Needs aic_cortex_host_workspace_bytes of workspace. Returns once
 * the work is queued; synchronise `stream` before reading the outputs. */
AIC_API aic_status aic_cortex_host_workspace_bytes(aic_cortex c, int batch, int seq, size_t* bytes);
AIC_API aic_status aic_cortex_forward_host(aic_cortex c, const uint16_t* planes_host, int batch, int seq,
                                           float* actor_host, float* critic_host, void* workspace, void* stream);
/* Conv mode (AIC_CONV_*) of every conv layer of the cortex. */
AIC_API aic_status aic_cortex_set_conv_mode(aic_cortex c, int mode);
/* AIC_MAMBA_* of every Mamba layer of the cortex (units and actor). */
AIC_API aic_status aic_cortex_set_mamba_mode(aic_cortex c, int mode);
/* exact != 0: AIC_CONV_SIMT and AIC_MAMBA_EXACT (every kernel in the
 * reference's arithmetic order); 0: AIC_CONV_ORDERED and AIC_MAMBA_TENSOR
 * (the defaults). */
AIC_API aic_status aic_cortex_set_exact(aic_cortex c, int exact);
/* Number of kernel launches the last forward issued. */
AIC_API aic_status aic_cortex_last_launches(aic_cortex c, int64_t* launches);
/* Per-launch-site CUDA-event timing (tracing). When enabled, every kernel
 * launch of a forward is bracketed by events on its stream; collecting waits
 * for them. Sites are named like "b0.pw1" (block 0, first pointwise conv),
 * "u2.scan", "actor.outproj". flops/bytes are the algorithmic work and the
 * minimum HBM traffic of ONE launch of the site. */
AIC_API aic_status aic_cortex_profile_enable(aic_cortex c, int enable);
AIC_API aic_status aic_cortex_profile_count(aic_cortex c, int* sites);
AIC_API aic_status aic_cortex_profile_get(aic_cortex c, int site, char name[32], double* total_ms, int64_t* launches,
                                          double* flops_per_launch, double* bytes_per_launch);
AIC_API aic_status aic_cortex_profile_reset(aic_cortex c);
AIC_API aic_status aic_cortex_destroy(aic_cortex c);

/* ---------------------------------------------------------------- training
 * The reference's online training step, one layer at a time, as its layer
 * classes' backward() run it: gradients of one frame (conv) or one env step
 * (Mamba, critic), clip_op + updateParamsKernel on every parameter tensor
 * (norm = sqrt(sum g^2 + epsilon), factor 1/norm above 1; data = g * (-lr *
 * factor) + data * (1 - lr * penalty), biases with penalty 0), then the
 * weights re-quantised from their fp32 masters (quantizeKernel, stochastic,
 * add_idx = n). Replaces ConvLayer::backward (conv_layer.h:150-219),
 * MambaLayer::backward (mamba_layer.h:146-167), Critic::backward
 * (critic.h:117-131), residualAddBwdKernel (kernels.h:1056-1079) and
 * updateParamsKernel (kernels.h:196-216). The gradients are the reference
 * kernels' own formulas (kernels.h:283-988, 1260-1419, 1779-1805), including
 * where they differ from the textbook gradient; the header of k_train.cu
 * lists those and the inputs on which the reference reads unwritten memory. */

/* Square-sum clip factor of a gradient: factor[0] = 1/norm above 1 else 1,
 * factor[1] = sum g^2 (device floats). `partial` holds
 * aic_grad_clip_partials(n) floats. The reference adds its block sums with
 * atomics in arrival order; these are added in block order. */
AIC_API aic_status aic_grad_clip_partials(int64_t n, int64_t* floats);
AIC_API aic_status aic_grad_clip_factor(const float* grad, int64_t n, float* partial, float* factor, void* stream);
/* updateParamsKernel with grad_norm_factor read from factor[0] (device). Like
 * the reference, updates the first floor(n / 4) * 4 elements. */
AIC_API aic_status aic_sgd_update(float* data, const float* grad, int64_t n, const float* factor, float lr,
                                  float penalty, void* stream);
/* grad_res = grad_next; grad_next *= survival_prob_inv * residual_factor. */
AIC_API aic_status aic_residual_backward(float* grad_next, float* grad_res, int64_t n, float survival_prob_inv,
                                         float residual_factor, void* stream);

/* Training state of a conv layer: bytes of the 256-byte-aligned device buffer,
 * and binding it with the fp32 master weights (weight layout of
 * aic_conv_layer_load, device or host memory), from which the packed weights
 * are re-derived. */
AIC_API aic_status aic_conv_layer_train_bytes(aic_conv_layer l, size_t* bytes);
AIC_API aic_status aic_conv_layer_train_bind(aic_conv_layer l, void* buffer, const float* master, float learning_rate,
                                             float penalty, void* stream);
/* One frame: grad_out fp32 [dim_out^2][out]; in / in_s the layer's forward
 * input (F); grad_in fp32 [dim_in^2][in] is added to (pointwise and dense
 * convs, the reference's atomic adds) or written (depthwise), or NULL.
 * Pointwise convs need dim_out^2 % 32 == 0, depthwise dim_out^2 % 4 == 0. */
AIC_API aic_status aic_conv_layer_backward(aic_conv_layer l, const float* grad_out, const uint32_t* in,
                                           const int8_t* in_s, float* grad_in, void* stream);
/* Device pointers into the training state (any may be NULL): masters,
 * gradients of the last backward, and the fp32 biases. */
AIC_API aic_status aic_conv_layer_train_views(aic_conv_layer l, float** master, float** grad_w, float** grad_b,
                                              float** bias);

/* Training state of a Mamba layer (master = the fp32 blob of
 * aic_mamba_layer_load); d_model a multiple of 128. */
AIC_API aic_status aic_mamba_layer_train_bytes(aic_mamba_layer l, size_t* bytes);
AIC_API aic_status aic_mamba_layer_train_bind(aic_mamba_layer l, void* buffer, const float* master,
                                              float learning_rate, float penalty, void* stream);
/* The step just run: state bound for batch 1 with traces bound; in / in_s the
 * step's input; grad_out fp32 [out]; grad_in fp32 [d_model] written. */
AIC_API aic_status aic_mamba_layer_backward(aic_mamba_layer l, const float* grad_out, const uint32_t* in,
                                            const int8_t* in_s, float* grad_in, void* stream);
AIC_API aic_status aic_mamba_layer_train_views(aic_mamba_layer l, float** master, float** grad_w, float** grad_b,
                                               float** bias);

/* Training state of the critic (its weights are fp32 and updated in place);
 * units a power of two. */
AIC_API aic_status aic_critic_train_bytes(aic_critic c, size_t* bytes);
AIC_API aic_status aic_critic_train_bind(aic_critic c, void* buffer, float learning_rate, float penalty);
/* The step just run (batch 1, traces bound): pred_score the score it wrote
 * (device pointer), real_score the target. */
AIC_API aic_status aic_critic_backward(aic_critic c, const float* pred_score, float real_score, void* stream);
AIC_API aic_status aic_critic_train_views(aic_critic c, float** grad_w1, float** grad_w2, float** grad_lambda);

#ifdef __cplusplus
}
#endif
#endif /* AICORTEX_H */
