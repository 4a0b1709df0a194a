/*
 * aicortex_layers.hpp -- the reference's layer classes for the inference
 * path, with their constructor / initData / forward / reset / loadFromFile
 * signatures unchanged, implemented over the C ABI of aicortex.h.
 *
 * A maintainer replaces the reference headers conv_layer.h, conv_block.h,
 * mamba_layer.h, mamba_block.h and critic.h with this one header (for the
 * inference path) and links libaicortex_b200.so; Cortex and the rest of the
 * reference keep their code. Signatures follow conv_layer.h:45-47,64,102,
 * conv_block.h:30-33,57,74, mamba_layer.h:54-56,73,139,171, mamba_block.h:28-30,
 * 43,58,105 and critic.h:58,70,106,134.
 *
 * Memory follows the reference's two-phase scheme: each constructor adds the
 * bytes it needs to the caller's counters (here the C ABI's parameter,
 * state and workspace sizes, each rounded up to 256 bytes plus 256 bytes of
 * alignment slack, since the reference carves its arenas at 16-byte
 * granularity); initData carves views from the caller's arenas by advancing
 * the same cursors. Host master weights are carved from the host arena as the
 * reference does (it must be pinned host memory, as the reference allocates
 * it, because the packer reads it from the GPU). Nothing here allocates device
 * memory. The d_model and d_state of the Mamba layers are the reference's
 * compile-time final_channels and mamba_d_state (base_constants.h); define
 * AIC_LAYERS_D_MODEL / AIC_LAYERS_D_STATE to give them without that header.
 *
 * Training: ConvLayer, MambaLayer and Critic keep the reference's backward()
 * (conv_layer.h:150, mamba_layer.h:146, critic.h:117) over the C ABI's layer
 * backward. Their training state (fp32 master copy on the device, gradients,
 * scratch) is counted into the main device arena by every constructor, since
 * only initData learns whether the layer trains, and is bound when
 * is_in_inference is false (the critic always trains, as in the reference).
 * After each backward the updated masters are copied back into the host
 * arena, where the reference's update kernel writes them.
 *
 * Differences from the reference classes: errors (status codes of the C ABI)
 * are thrown as std::runtime_error with aic_last_error()'s message, as the
 * reference's checkCudaError does; the block-level backward (ConvBlock,
 * MambaBlock) and saveToFile are not provided; a short checkpoint file is an
 * error (the reference reads it silently); weights drawn when no checkpoint
 * is loaded come from a seeded std::mt19937 (the reference's generator
 * hashes thread indices and is not reproducible).
 */
#ifndef AICORTEX_LAYERS_HPP
#define AICORTEX_LAYERS_HPP

#include <cuda_runtime.h>

#include <cmath>
#include <cstddef>
#include <cstdint>
#include <filesystem>
#include <fstream>
#include <memory>
#include <random>
#include <stdexcept>
#include <string>
#include <vector>

#include "aicortex.h"

#ifndef AIC_LAYERS_D_MODEL
#define AIC_LAYERS_D_MODEL final_channels
#endif
#ifndef AIC_LAYERS_D_STATE
#define AIC_LAYERS_D_STATE mamba_d_state
#endif

namespace aic_dropin {

inline void check(aic_status st)
{
    if (st != AIC_OK) throw std::runtime_error(std::string("[aicortex_b200] ") + aic_last_error());
}
inline void check_cuda(cudaError_t e)
{
    if (e != cudaSuccess) throw std::runtime_error(std::string("[aicortex_b200] ") + cudaGetErrorString(e));
}
inline size_t align16(size_t n) { return (n + 15) & ~size_t(15); }
// bytes a 256-byte aligned view of n bytes takes from a 16-byte aligned cursor
inline size_t carve_bytes(size_t n) { return ((n + 255) & ~size_t(255)) + 256; }
inline uint8_t* carve(uint8_t*& cur, size_t n)
{
    const uintptr_t p = (reinterpret_cast<uintptr_t>(cur) + 255) & ~uintptr_t(255);
    cur += carve_bytes(n);
    return reinterpret_cast<uint8_t*>(p);
}
inline uint8_t* carve_host(uint8_t*& cur, size_t n)
{
    uint8_t* p = cur;
    cur += align16(n);
    return p;
}
// fp32 values of a reference checkpoint file: the counts in order
inline void read_floats(const std::string& path, std::vector<float*> dst, std::vector<size_t> counts)
{
    std::ifstream f(path, std::ios::binary);
    if (!f.is_open()) throw std::runtime_error("[SYSTEM ERROR] Failed to open file for reading: " + path);
    for (size_t i = 0; i < dst.size(); ++i) {
        f.read(reinterpret_cast<char*>(dst[i]), static_cast<std::streamsize>(counts[i] * sizeof(float)));
        if (static_cast<size_t>(f.gcount()) != counts[i] * sizeof(float))
            throw std::runtime_error("[SYSTEM ERROR] Short checkpoint file: " + path);
    }
}
inline void fill_normal(float* p, size_t n, float stddev, uint32_t seed)
{
    std::mt19937 gen(seed);
    std::normal_distribution<float> d(0.0f, stddev);
    for (size_t i = 0; i < n; ++i) p[i] = d(gen);
}

// A view of device output with the data()/size() of the reference's universal_vector.
template <class T>
struct DeviceSpan {
    T* ptr = nullptr;
    size_t count = 0;
    T* data() const { return ptr; }
    size_t size() const { return count; }
};

// ---------------------------------------------------------------- ConvLayer
class ConvLayer {
    aic_conv_layer h_ = nullptr;
    cudaStream_t stream_forward, stream_backward;
    int in_channels, out_channels, kernel_size;
    bool is_dw, disable_activation;
    int64_t weight_elems = 0;
    size_t param_bytes = 0, train_bytes = 0;
    float learning_rate, f_penalty;
    float* master_weights = nullptr;  // host arena view
    float* master_dev = nullptr;      // the training state's device copy
    bool training = false;
    std::vector<float> bias_host;

public:
    ConvLayer(int inChannels, int outChannels, int kernelSize, int str_ide, int in_dimension, int out_dimension,
              cudaStream_t stream_fwd, int* total_size_grad_weights, int* total_size_grad_biases, cudaStream_t stream_bwd,
              float learningRate, float penalty, size_t* total_mem_main_device, size_t* total_mem_main_host,
              size_t* total_learnable_data, size_t* total_learnable_data_count, bool is_activation_disabled = false)
        : stream_forward(stream_fwd), stream_backward(stream_bwd), in_channels(inChannels), out_channels(outChannels),
          kernel_size(kernelSize), is_dw(kernelSize > 1 && (kernelSize & 1) == 1),
          disable_activation(is_activation_disabled), learning_rate(learningRate), f_penalty(penalty)
    {
        const aic_conv_layer_desc d{inChannels, outChannels, kernelSize, str_ide, in_dimension, out_dimension,
                                    is_activation_disabled ? 1 : 0};
        check(aic_conv_layer_create(&d, &h_));
        int64_t be = 0;
        check(aic_conv_layer_sizes(h_, &weight_elems, &be, &param_bytes));
        check(aic_conv_layer_train_bytes(h_, &train_bytes));
        if (*total_size_grad_weights < weight_elems) *total_size_grad_weights = static_cast<int>(weight_elems);
        if (*total_size_grad_biases < out_channels) *total_size_grad_biases = out_channels;
        *total_mem_main_device += carve_bytes(param_bytes) + carve_bytes(train_bytes);
        *total_mem_main_host += align16(static_cast<size_t>(weight_elems) * sizeof(float));
        if (total_learnable_data) *total_learnable_data += static_cast<size_t>(weight_elems) + out_channels;
        if (total_learnable_data_count) *total_learnable_data_count += 2;
    }
    ConvLayer(const ConvLayer&) = delete;
    ConvLayer& operator=(const ConvLayer&) = delete;
    ~ConvLayer()
    {
        if (h_) aic_conv_layer_destroy(h_);
    }
    aic_conv_layer handle() const { return h_; }

    void initData(bool isLoaded, std::string dir_path, uint8_t*& current_dev_main_ptr, uint8_t*& current_host_main_ptr,
                  uint8_t*&, uint8_t*&, bool is_in_inference, float*** meta_adapted_data, size_t** meta_adapted_offsets,
                  int, int)
    {
        check(aic_conv_layer_bind(h_, carve(current_dev_main_ptr, param_bytes)));
        void* train_buf = carve(current_dev_main_ptr, train_bytes);
        init_weights(isLoaded, dir_path, current_host_main_ptr);
        if (is_in_inference) return;
        // conv_layer.h:82-92: the training state, and the parameter list of the meta-learner
        check(aic_conv_layer_train_bind(h_, train_buf, master_weights, learning_rate, f_penalty, stream_backward));
        check_cuda(cudaStreamSynchronize(stream_backward));
        float* bias_dev = nullptr;
        check(aic_conv_layer_train_views(h_, &master_dev, nullptr, nullptr, &bias_dev));
        training = true;
        if (meta_adapted_data && *meta_adapted_data) {
            *(*meta_adapted_data)++ = master_weights;
            *(*meta_adapted_data)++ = bias_dev;
        }
        if (meta_adapted_offsets && *meta_adapted_offsets) {
            *(*meta_adapted_offsets)++ = static_cast<size_t>(weight_elems);
            *(*meta_adapted_offsets)++ = static_cast<size_t>(out_channels);
        }
    }
    // conv_layer.h:150-219: one frame; grad_input is added to (pointwise and
    // dense convs) or written (depthwise), as the reference's kernels do
    void backward(const float* grad_output, const uint32_t* input, const int8_t* input_scales, float* grad_input)
    {
        if (!training) throw std::runtime_error("[aicortex_b200] ConvLayer::backward needs initData in training mode");
        check(aic_conv_layer_backward(h_, grad_output, input, input_scales, grad_input, stream_backward));
        check_cuda(cudaMemcpyAsync(master_weights, master_dev, static_cast<size_t>(weight_elems) * sizeof(float),
                                   cudaMemcpyDeviceToHost, stream_backward));
    }

private:
    void init_weights(bool isLoaded, const std::string& dir_path, uint8_t*& current_host_main_ptr)
    {
        master_weights = reinterpret_cast<float*>(
            carve_host(current_host_main_ptr, static_cast<size_t>(weight_elems) * sizeof(float)));
        bias_host.assign(out_channels, 0.0f);
        if (isLoaded) {
            loadFromFile(dir_path);
        } else {  // conv_layer.h:90-95: N(0, sqrt(1/k^2)) depthwise, N(0, sqrt(2/fan)) otherwise; zero bias
            const float sd = is_dw ? std::sqrt(1.0f / (kernel_size * kernel_size))
                                   : std::sqrt(2.0f / (in_channels + (disable_activation ? out_channels : 0)));
            fill_normal(master_weights, static_cast<size_t>(weight_elems), sd, static_cast<uint32_t>(weight_elems));
            check(aic_conv_layer_load_weights(h_, master_weights, bias_host.data(), stream_forward));
            check_cuda(cudaStreamSynchronize(stream_forward));
        }
    }

public:
    // conv_layer.h:31-44: fp32 master weights then fp32 bias; packed bit-exactly
    void loadFromFile(std::string pathFile)
    {
        read_floats(pathFile, {master_weights, bias_host.data()},
                    {static_cast<size_t>(weight_elems), static_cast<size_t>(out_channels)});
        check(aic_conv_layer_load_weights(h_, master_weights, bias_host.data(), stream_forward));
        check_cuda(cudaStreamSynchronize(stream_forward));
    }
    void forward(const uint32_t* input, const int8_t* input_scales, uint32_t* output, int8_t* output_scales)
    {
        check(aic_conv_layer_forward(h_, input, input_scales, output, output_scales, 1, stream_forward));
    }
};

// ---------------------------------------------------------------- ConvBlock
class ConvBlock {
    aic_conv_block h_ = nullptr;
    cudaStream_t stream_forward;
    int *pipo_db, *pipo_db_num_groups;
    int dims[4][2];  // (in, out) channels of the four sub-layers
    size_t param_bytes = 0, ws_bytes = 0;
    int64_t weight_elems[4] = {0, 0, 0, 0};
    float* master_weights[4] = {nullptr, nullptr, nullptr, nullptr};
    std::vector<float> bias_host[4];
    void* workspace = nullptr;
    static constexpr const char* kFiles[4] = {"depthwise_layer.bin", "conv_layer1.bin", "conv_layer2.bin",
                                              "residual_layer.bin"};

public:
    ConvBlock(int in_channels, int mid_channels, int out_channels, int stride, int in_dimension, int out_dimension,
              cudaStream_t stream_fwd, int* total_size_grad_weights, int* total_size_grad_biases, int* db_pipo,
              int* db_pipo_num_groups, int kernel_size_dw, float survival_probability, float res_factor, cudaStream_t,
              float, float, size_t* total_mem_main_device, size_t* total_mem_main_host, size_t* total_learnable_data,
              size_t* total_learnable_data_count)
        : stream_forward(stream_fwd), pipo_db(db_pipo), pipo_db_num_groups(db_pipo_num_groups),
          dims{{in_channels, in_channels}, {in_channels, mid_channels}, {mid_channels, out_channels},
               {in_channels, out_channels}}
    {
        const aic_conv_block_desc d{in_channels,   mid_channels,   out_channels,         stride,    in_dimension,
                                    out_dimension, kernel_size_dw, survival_probability, res_factor};
        check(aic_conv_block_create(&d, &h_));
        check(aic_conv_block_param_bytes(h_, &param_bytes));
        check(aic_conv_block_workspace_bytes(h_, 1, &ws_bytes));
        *total_mem_main_device += carve_bytes(param_bytes);
        for (int i = 0; i < 4; ++i) {
            aic_conv_layer l;
            int64_t be = 0;
            check(aic_conv_block_layer(h_, i, &l));
            check(aic_conv_layer_sizes(l, &weight_elems[i], &be, nullptr));
            if (*total_size_grad_weights < weight_elems[i]) *total_size_grad_weights = static_cast<int>(weight_elems[i]);
            if (*total_size_grad_biases < dims[i][1]) *total_size_grad_biases = dims[i][1];
            *total_mem_main_host += align16(static_cast<size_t>(weight_elems[i]) * sizeof(float));
            if (total_learnable_data) *total_learnable_data += static_cast<size_t>(weight_elems[i]) + dims[i][1];
            if (total_learnable_data_count) *total_learnable_data_count += 2;
        }
        // conv_block.h:44-47: the ping-pong buffers; buffer a holds this
        // implementation's per-frame workspace (groups of 16 bytes)
        const int local_pipo_db = mid_channels * out_dimension * out_dimension;
        const int ws_groups = static_cast<int>((carve_bytes(ws_bytes) + 15) / 16);
        if (*pipo_db < local_pipo_db) *pipo_db = local_pipo_db;
        if (*pipo_db_num_groups < ws_groups) *pipo_db_num_groups = ws_groups;
        if (*pipo_db_num_groups < (local_pipo_db >> 5)) *pipo_db_num_groups = local_pipo_db >> 5;
    }
    ConvBlock(const ConvBlock&) = delete;
    ConvBlock& operator=(const ConvBlock&) = delete;
    ~ConvBlock()
    {
        if (h_) aic_conv_block_destroy(h_);
    }
    aic_conv_block handle() const { return h_; }

    void initData(bool isLoaded, std::string dir_path, uint8_t*& current_dev_main_ptr, uint8_t*& current_host_main_ptr,
                  uint8_t*&, uint8_t*&, bool, float**&, size_t*&, uint8_t*&, uint8_t*&, uint8_t*&,
                  uint8_t*& dev_main_ptr_buffer_a, uint8_t*&, uint8_t*&, uint8_t*&, int, int)
    {
        check(aic_conv_block_bind(h_, carve(current_dev_main_ptr, param_bytes)));
        uint8_t* a = dev_main_ptr_buffer_a;
        workspace = carve(a, ws_bytes);
        for (int i = 0; i < 4; ++i) {
            master_weights[i] = reinterpret_cast<float*>(
                carve_host(current_host_main_ptr, static_cast<size_t>(weight_elems[i]) * sizeof(float)));
            bias_host[i].assign(dims[i][1], 0.0f);
        }
        if (isLoaded) {
            loadFromFile(dir_path);
            return;
        }
        for (int i = 0; i < 4; ++i) {
            aic_conv_layer l;
            check(aic_conv_block_layer(h_, i, &l));
            const bool dw = i == 0, noact = i != 1;
            const float sd = dw ? std::sqrt(1.0f / static_cast<float>(weight_elems[0] / dims[0][0]))
                                : std::sqrt(2.0f / (dims[i][0] + (noact ? dims[i][1] : 0)));
            fill_normal(master_weights[i], static_cast<size_t>(weight_elems[i]), sd, static_cast<uint32_t>(i + 1));
            check(aic_conv_layer_load_weights(l, master_weights[i], bias_host[i].data(), stream_forward));
        }
        check_cuda(cudaStreamSynchronize(stream_forward));
    }
    // conv_block.h:23-29
    void loadFromFile(std::string pathFile)
    {
        for (int i = 0; i < 4; ++i) {
            aic_conv_layer l;
            check(aic_conv_block_layer(h_, i, &l));
            read_floats((std::filesystem::path(pathFile) / kFiles[i]).string(), {master_weights[i], bias_host[i].data()},
                        {static_cast<size_t>(weight_elems[i]), static_cast<size_t>(dims[i][1])});
            check(aic_conv_layer_load_weights(l, master_weights[i], bias_host[i].data(), stream_forward));
        }
        check_cuda(cudaStreamSynchronize(stream_forward));
    }
    void forward(const uint32_t* input, const int8_t* input_scales, uint32_t* output, int8_t* output_scales,
                 bool train_mode = true, bool is_survived = true)
    {
        check(aic_conv_block_forward(h_, input, input_scales, output, output_scales, 1, train_mode ? 1 : 0,
                                     is_survived ? 1 : 0, workspace, stream_forward));
    }
};

// ---------------------------------------------------------------- MambaLayer
class MambaLayer {
    aic_mamba_layer h_ = nullptr;
    cudaStream_t stream_forward, stream_backward;
    int out_channels;
    int64_t weight_elems = 0;
    size_t param_bytes = 0, state_bytes = 0, ws_bytes = 0, trace_bytes = 0, train_bytes = 0;
    float learning_rate, f_penalty;
    float* master_weights = nullptr;
    float* master_dev = nullptr;
    bool training = false;
    std::vector<float> bias_host;
    DeviceSpan<float> mamba_output;
    void* workspace = nullptr;

public:
    static constexpr int d_model = AIC_LAYERS_D_MODEL, d_state = AIC_LAYERS_D_STATE;

    MambaLayer(int output_channels, cudaStream_t stream_fwd, int* total_size_grad_weights, int* total_size_grad_biases,
               cudaStream_t stream_bwd, float learningRate, float penalty, size_t* total_mem_device,
               size_t* total_mem_host, size_t* total_learnable_data, size_t* total_learnable_data_count,
               int type_activation)
        : stream_forward(stream_fwd), stream_backward(stream_bwd), out_channels(output_channels),
          learning_rate(learningRate), f_penalty(penalty)
    {
        const aic_mamba_layer_desc d{d_model, d_state, output_channels, type_activation};
        check(aic_mamba_layer_create(&d, &h_));
        // one step of one sequence per call, as the reference runs it: the
        // reference-order out-projection (bit-identical; a one-row GEMM gains
        // nothing from the tensor cores)
        check(aic_mamba_layer_set_mode(h_, AIC_MAMBA_EXACT));
        int64_t be = 0;
        check(aic_mamba_layer_sizes(h_, &weight_elems, &be, &param_bytes));
        check(aic_mamba_layer_state_bytes(h_, 1, &state_bytes));
        check(aic_mamba_layer_workspace_bytes(h_, 1, &ws_bytes));
        check(aic_mamba_layer_trace_bytes(h_, 1, &trace_bytes));
        check(aic_mamba_layer_train_bytes(h_, &train_bytes));
        if (*total_size_grad_weights < weight_elems) *total_size_grad_weights = static_cast<int>(weight_elems);
        if (*total_size_grad_biases < out_channels) *total_size_grad_biases = out_channels;
        // mamba_layer.h:68: output, parameters, state and y_ssm in the main device
        // arena; then the training state
        *total_mem_device += carve_bytes(out_channels * sizeof(float)) + carve_bytes(param_bytes) +
                             carve_bytes(state_bytes) + carve_bytes(ws_bytes) + carve_bytes(train_bytes);
        *total_mem_host += align16(static_cast<size_t>(weight_elems) * sizeof(float));
        if (total_learnable_data) *total_learnable_data += static_cast<size_t>(weight_elems) + out_channels;
        if (total_learnable_data_count) *total_learnable_data_count += 2;
    }
    MambaLayer(const MambaLayer&) = delete;
    MambaLayer& operator=(const MambaLayer&) = delete;
    ~MambaLayer()
    {
        if (h_) aic_mamba_layer_destroy(h_);
    }
    aic_mamba_layer handle() const { return h_; }
    DeviceSpan<float>& get_output() { return mamba_output; }

    // mamba_layer.h:73-118; the training-mode traces (mamba_layer.h:101-105)
    // come from the side arena when is_in_inference is false
    void initData(bool isLoaded, std::string dir_path, uint8_t*& current_dev_main_ptr, uint8_t*& current_host_main_ptr,
                  uint8_t*& current_dev_side_ptr, uint8_t*&, uint8_t*&, bool is_in_inference, float***, size_t**, int,
                  int)
    {
        mamba_output.ptr = reinterpret_cast<float*>(carve(current_dev_main_ptr, out_channels * sizeof(float)));
        mamba_output.count = static_cast<size_t>(out_channels);
        check(aic_mamba_layer_bind(h_, carve(current_dev_main_ptr, param_bytes)));
        check(aic_mamba_layer_bind_state(h_, carve(current_dev_main_ptr, state_bytes), 1));
        workspace = carve(current_dev_main_ptr, ws_bytes);
        void* train_buf = carve(current_dev_main_ptr, train_bytes);
        if (!is_in_inference) check(aic_mamba_layer_bind_traces(h_, carve(current_dev_side_ptr, trace_bytes), 1));
        master_weights = reinterpret_cast<float*>(
            carve_host(current_host_main_ptr, static_cast<size_t>(weight_elems) * sizeof(float)));
        bias_host.assign(out_channels, 0.0f);
        reset(stream_forward);
        init_weights(isLoaded, dir_path);
        if (is_in_inference) return;
        check(aic_mamba_layer_train_bind(h_, train_buf, master_weights, learning_rate, f_penalty, stream_backward));
        check_cuda(cudaStreamSynchronize(stream_backward));
        check(aic_mamba_layer_train_views(h_, &master_dev, nullptr, nullptr, nullptr));
        training = true;
    }
    // mamba_layer.h:146-167: the step just run; grad_input (the reference's
    // universal_vector, or anything with data()) receives d_model floats
    template <class Vec>
    void backward(const float* grad_output, const uint32_t* input, const int8_t* input_scales, Vec& grad_input)
    {
        if (!training) throw std::runtime_error("[aicortex_b200] MambaLayer::backward needs initData in training mode");
        check(aic_mamba_layer_backward(h_, grad_output, input, input_scales, grad_input.data(), stream_backward));
        check_cuda(cudaMemcpyAsync(master_weights, master_dev, static_cast<size_t>(weight_elems) * sizeof(float),
                                   cudaMemcpyDeviceToHost, stream_backward));
    }

private:
    void init_weights(bool isLoaded, const std::string& dir_path)
    {
        if (isLoaded) {
            loadFromFile(dir_path);
            return;
        }
        // mamba_layer.h:120-135: N(0, sqrt(2/d_inner)), MIMO blocks near identity,
        // A_re from -12.1 to -12.5 across a row, A_im = 0.001, zero bias
        const int E = 2 * d_model;
        fill_normal(master_weights, static_cast<size_t>(weight_elems), std::sqrt(2.0f / E), 7u);
        std::mt19937 gen(11u);
        std::uniform_real_distribution<float> u(-std::sqrt(1.0f / 32.0f), std::sqrt(1.0f / 32.0f));
        for (int b = 0; b < E / 32; ++b)
            for (int r = 0; r < 32; ++r)
                for (int c = 0; c < 32; ++c)
                    master_weights[E + b * 1024 + r * 32 + c] = std::fma(u(gen), 0.1f, r == c ? 1.0f : 0.0f);
        const size_t n_st = static_cast<size_t>(E) * d_state, off_are = static_cast<size_t>(E) * 33 + 2 * n_st;
        for (size_t i = 0; i < n_st; ++i) {
            master_weights[off_are + i] =
                -12.1f - 0.4f * static_cast<float>(i & (d_state - 1)) / static_cast<float>(d_state - 1);
            master_weights[off_are + n_st + i] = 0.001f;
        }
        check(aic_mamba_layer_load_weights(h_, master_weights, bias_host.data(), stream_forward));
        check_cuda(cudaStreamSynchronize(stream_forward));
    }

public:
    // mamba_layer.h:40-53
    void loadFromFile(std::string pathFile)
    {
        read_floats(pathFile, {master_weights, bias_host.data()},
                    {static_cast<size_t>(weight_elems), static_cast<size_t>(out_channels)});
        check(aic_mamba_layer_load_weights(h_, master_weights, bias_host.data(), stream_forward));
        check_cuda(cudaStreamSynchronize(stream_forward));
    }
    void forward(const uint32_t* input, const int8_t* input_scales)
    {
        check(aic_mamba_layer_forward(h_, input, input_scales, mamba_output.ptr, 1, 1, workspace, stream_forward));
    }
    void reset(cudaStream_t stream_lnk = 0) { check(aic_mamba_layer_reset_state(h_, stream_lnk)); }
};

// ---------------------------------------------------------------- MambaBlock
class MambaBlock {
    aic_mamba_block h_ = nullptr;
    cudaStream_t stream_forward;
    int output_channels;
    size_t param_bytes = 0, state_bytes = 0, ws_bytes = 0, trace_bytes = 0;
    int64_t weight_elems[3] = {0, 0, 0};
    int outs[3];
    float* master_weights[3] = {nullptr, nullptr, nullptr};
    std::vector<float> bias_host[3];
    DeviceSpan<float> output;
    void* workspace = nullptr;
    static constexpr const char* kFiles[3] = {"mamba_strategist.bin", "mamba_tactic.bin", "mamba_executor.bin"};

public:
    static constexpr int d_model = AIC_LAYERS_D_MODEL, d_state = AIC_LAYERS_D_STATE;

    MambaBlock(int in_channels, int out_channels, cudaStream_t stream_fwd, int* total_size_grad_weights,
               int* total_size_grad_biases, float survival_probability, float res_factor, cudaStream_t, float, float,
               size_t* total_mem_main_device, size_t* total_mem_main_host, size_t* total_learnable_data,
               size_t* total_learnable_data_count, int activation_type = 2)
        : stream_forward(stream_fwd), output_channels(out_channels), outs{in_channels, in_channels, out_channels}
    {
        if (in_channels != d_model) throw std::runtime_error("[aicortex_b200] MambaBlock input channels must equal d_model");
        const aic_mamba_block_desc d{d_model, d_state, out_channels, activation_type, survival_probability, res_factor};
        check(aic_mamba_block_create(&d, &h_));
        check(aic_mamba_block_set_mode(h_, AIC_MAMBA_EXACT));  // as MambaLayer above
        check(aic_mamba_block_param_bytes(h_, &param_bytes));
        check(aic_mamba_block_state_bytes(h_, 1, &state_bytes));
        check(aic_mamba_block_workspace_bytes(h_, 1, &ws_bytes));
        check(aic_mamba_block_trace_bytes(h_, 1, &trace_bytes));
        *total_mem_main_device += carve_bytes(out_channels * sizeof(float)) + carve_bytes(param_bytes) +
                                  carve_bytes(state_bytes) + carve_bytes(ws_bytes);
        for (int i = 0; i < 3; ++i) {
            aic_mamba_layer l;
            int64_t be = 0;
            check(aic_mamba_block_layer(h_, i, &l));
            check(aic_mamba_layer_sizes(l, &weight_elems[i], &be, nullptr));
            if (*total_size_grad_weights < weight_elems[i]) *total_size_grad_weights = static_cast<int>(weight_elems[i]);
            if (*total_size_grad_biases < outs[i]) *total_size_grad_biases = outs[i];
            *total_mem_main_host += align16(static_cast<size_t>(weight_elems[i]) * sizeof(float));
            if (total_learnable_data) *total_learnable_data += static_cast<size_t>(weight_elems[i]) + outs[i];
            if (total_learnable_data_count) *total_learnable_data_count += 2;
        }
    }
    MambaBlock(const MambaBlock&) = delete;
    MambaBlock& operator=(const MambaBlock&) = delete;
    ~MambaBlock()
    {
        if (h_) aic_mamba_block_destroy(h_);
    }
    aic_mamba_block handle() const { return h_; }
    DeviceSpan<float>& get_output() { return output; }

    void initData(bool isLoaded, std::string dir_path, uint8_t*& current_dev_main_ptr, uint8_t*& current_host_main_ptr,
                  uint8_t*& dev_side_ptr, uint8_t*&, uint8_t*&, bool is_in_inference, float**&, size_t*&, uint8_t*&,
                  uint8_t*&, uint8_t*&, uint8_t*&, uint8_t*&, uint8_t*&, int, int, int)
    {
        output.ptr = reinterpret_cast<float*>(carve(current_dev_main_ptr, output_channels * sizeof(float)));
        output.count = static_cast<size_t>(output_channels);
        check(aic_mamba_block_bind(h_, carve(current_dev_main_ptr, param_bytes)));
        check(aic_mamba_block_bind_state(h_, carve(current_dev_main_ptr, state_bytes), 1));
        workspace = carve(current_dev_main_ptr, ws_bytes);
        if (!is_in_inference) check(aic_mamba_block_bind_traces(h_, carve(dev_side_ptr, trace_bytes), 1));
        for (int i = 0; i < 3; ++i) {
            master_weights[i] = reinterpret_cast<float*>(
                carve_host(current_host_main_ptr, static_cast<size_t>(weight_elems[i]) * sizeof(float)));
            bias_host[i].assign(outs[i], 0.0f);
        }
        reset(stream_forward);
        if (isLoaded) loadFromFile(dir_path);
    }
    // mamba_block.h:22-27
    void loadFromFile(std::string pathFile)
    {
        for (int i = 0; i < 3; ++i) {
            aic_mamba_layer l;
            check(aic_mamba_block_layer(h_, i, &l));
            read_floats((std::filesystem::path(pathFile) / kFiles[i]).string(), {master_weights[i], bias_host[i].data()},
                        {static_cast<size_t>(weight_elems[i]), static_cast<size_t>(outs[i])});
            check(aic_mamba_layer_load_weights(l, master_weights[i], bias_host[i].data(), stream_forward));
        }
        check_cuda(cudaStreamSynchronize(stream_forward));
    }
    void forward(const uint32_t* input, const int8_t* input_scales, bool on_training = true, int add_seed = 1234,
                 bool is_survived = true)
    {
        check(aic_mamba_block_forward(h_, input, input_scales, output.ptr, 1, 1, on_training ? 1 : 0, add_seed,
                                      is_survived ? 1 : 0, workspace, stream_forward));
    }
    void reset(cudaStream_t stream_lnk = 0) { check(aic_mamba_block_reset_state(h_, stream_lnk)); }
};

// ---------------------------------------------------------------- Critic
class Critic {
    aic_critic h_ = nullptr;
    cudaStream_t stream_forward, stream_backward;
    int in_channels, units;
    size_t param_bytes = 0, state_bytes = 0, ws_bytes = 0, trace_bytes = 0, train_bytes = 0;
    float learning_rate, f_penalty;
    float* score_dev = nullptr;
    void* workspace = nullptr;
    float score_host = 0.0f;

public:
    Critic(int inChannels, int outChannels, int in_dimension, cudaStream_t stream_fwd, int* total_size_grad_weights,
           int* total_size_grad_biases, cudaStream_t stream_bwd, float learningRate, float penalty,
           size_t* total_mem_main_device)
        : stream_forward(stream_fwd), stream_backward(stream_bwd), in_channels(inChannels), units(outChannels / 2),
          learning_rate(learningRate), f_penalty(penalty)
    {
        const aic_critic_desc d{inChannels, units, in_dimension};
        check(aic_critic_create(&d, &h_));
        check(aic_critic_param_bytes(h_, &param_bytes));
        check(aic_critic_state_bytes(h_, 1, &state_bytes));
        check(aic_critic_workspace_bytes(h_, 1, &ws_bytes));
        check(aic_critic_trace_bytes(h_, 1, &trace_bytes));
        check(aic_critic_train_bytes(h_, &train_bytes));
        if (*total_size_grad_weights < inChannels * outChannels) *total_size_grad_weights = inChannels * outChannels;
        if (*total_size_grad_biases < outChannels) *total_size_grad_biases = outChannels;
        // critic.h:68: parameters, traces and gradients in the main device arena (the
        // reference's critic always keeps its traces and trains)
        *total_mem_main_device += carve_bytes(param_bytes) + carve_bytes(state_bytes) + carve_bytes(ws_bytes) +
                                  carve_bytes(sizeof(float)) + carve_bytes(trace_bytes) + carve_bytes(train_bytes);
    }
    Critic(const Critic&) = delete;
    Critic& operator=(const Critic&) = delete;
    ~Critic()
    {
        if (h_) aic_critic_destroy(h_);
    }
    aic_critic handle() const { return h_; }
    // critic.h:22: the score of the last forward (on the host once forward returns)
    float get_score_output() const { return score_host; }

    void initData(bool isLoaded, std::string dir_path, uint8_t*& current_dev_main_ptr, uint8_t*&, uint8_t*&, int, int)
    {
        check(aic_critic_bind(h_, carve(current_dev_main_ptr, param_bytes)));
        check(aic_critic_bind_state(h_, carve(current_dev_main_ptr, state_bytes), 1));
        workspace = carve(current_dev_main_ptr, ws_bytes);
        score_dev = reinterpret_cast<float*>(carve(current_dev_main_ptr, sizeof(float)));
        check(aic_critic_bind_traces(h_, carve(current_dev_main_ptr, trace_bytes), 1));
        if (units & (units - 1))  // the reference's backward indexes units with a mask (kernels.h:1786)
            current_dev_main_ptr += carve_bytes(train_bytes);
        else
            check(aic_critic_train_bind(h_, carve(current_dev_main_ptr, train_bytes), learning_rate, f_penalty));
        reset(stream_forward);
        if (isLoaded) {
            loadFromFile(dir_path);
            return;
        }
        // critic.h:99-103: W1 ~ N(0, sqrt(2/in)), W2 ~ N(0, sqrt(1/out)); Wlambda small
        const size_t n1 = static_cast<size_t>(in_channels) * units * 2;
        std::vector<float> w1(n1), w2(static_cast<size_t>(units) * 2), wl(n1);
        fill_normal(w1.data(), n1, std::sqrt(2.0f / in_channels), 3u);
        fill_normal(w2.data(), w2.size(), std::sqrt(1.0f / (2 * units)), 5u);
        fill_normal(wl.data(), n1, 0.01f, 9u);
        check(aic_critic_load_weights(h_, w1.data(), w2.data(), wl.data(), stream_forward));
        check_cuda(cudaStreamSynchronize(stream_forward));
    }
    void loadFromFile(std::string pathFile) { check(aic_critic_load_file_sync(h_, pathFile.c_str(), stream_forward)); }
    // critic.h:106-116, including its stream synchronisation
    void forward(const uint32_t* input, const int8_t* input_scales)
    {
        check(aic_critic_forward(h_, input, input_scales, score_dev, 1, 1, workspace, stream_forward));
        check_cuda(cudaMemcpyAsync(&score_host, score_dev, sizeof(float), cudaMemcpyDeviceToHost, stream_forward));
        check_cuda(cudaStreamSynchronize(stream_forward));
    }
    void reset(cudaStream_t stream_lnk = 0) { check(aic_critic_reset_state(h_, stream_lnk)); }
    // critic.h:117-131: against the last forward's score
    void backward(float real_score) { check(aic_critic_backward(h_, score_dev, real_score, stream_backward)); }
};

}  // namespace aic_dropin

#ifndef AIC_LAYERS_NO_GLOBAL_NAMES
using aic_dropin::ConvBlock;
using aic_dropin::ConvLayer;
using aic_dropin::Critic;
using aic_dropin::MambaBlock;
using aic_dropin::MambaLayer;
#endif

#endif  // AICORTEX_LAYERS_HPP
