// C++ layer classes of the inference path and the extern "C" boundary
// declared in include/aicortex.h.
//
// The classes keep the reference's ownership model: a layer owns no memory,
// reports the bytes it needs, and is bound to caller-owned device memory
// (ConvLayer ctor/initData, conv_layer.h:45-101; MambaLayer,
// mamba_layer.h:54-138; Critic, critic.h:58-105). forward() gains batch and
// sequence extents; the kernels it launches are in k_*.cu.
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <exception>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "aic_common.cuh"
#include "aic_kernels.h"
#include "aicortex.h"

namespace aic {
namespace {

thread_local std::string g_last_error;

struct Failure {
    aic_status code;
    std::string msg;
};

[[noreturn]] void fail(aic_status code, const std::string& msg) { throw Failure{code, msg}; }
void require(bool ok, const std::string& msg)
{
    if (!ok) fail(AIC_ERR_INVALID, msg);
}
void cuda_ok(cudaError_t e, const char* what)
{
    if (e != cudaSuccess) fail(AIC_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}
bool aligned256(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 255u) == 0; }
bool is_pow2(int v) { return v > 0 && (v & (v - 1)) == 0; }

template <class F>
aic_status guarded(F&& f)
{
    try {
        f();
        return AIC_OK;
    } catch (const Failure& e) {
        g_last_error = e.msg;
        return e.code;
    } catch (const std::exception& e) {
        g_last_error = e.what();
        return AIC_ERR_INVALID;
    } catch (...) {
        g_last_error = "unknown error";
        return AIC_ERR_INVALID;
    }
}

// Sequential 256-byte aligned carve of a caller arena. With base == nullptr it
// only counts, so sizing and binding share one code path.
struct Carver {
    char* base;
    size_t off = 0;
    explicit Carver(void* b) : base(static_cast<char*>(b)) {}
    template <class T>
    T* take(size_t count)
    {
        off = (off + 255) & ~static_cast<size_t>(255);
        T* p = base ? reinterpret_cast<T*>(base + off) : nullptr;
        off += count * sizeof(T);
        return p;
    }
    size_t bytes() const { return (off + 255) & ~static_cast<size_t>(255); }
};

cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

int device_sms()
{
    int dev = 0, sms = 0;
    cuda_ok(cudaGetDevice(&dev), "device");
    cuda_ok(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "SM count");
    return sms;
}

// Training state of a layer (the reference's master weights, gradients and
// SGD hyper-parameters, conv_layer.h / mamba_layer.h / critic.h), in one
// caller-provided device buffer. The fp32 master copies of the packed
// weights live here; fp32 parameters (biases, the critic) are updated in place.
struct TrainState {
    float* master = nullptr;          // fp32 masters of the packed weights (null when all weights are fp32)
    float* gw = nullptr;              // weight gradients
    float* gb = nullptr;              // bias / second-tensor gradients
    float* gx = nullptr;              // third gradient tensor (critic lambda)
    float* scratch = nullptr;         // kernel scratch
    float* partial = nullptr;         // clip-factor block sums
    float* factor = nullptr;          // [3][2] clip factors and square sums
    float lr = 0.0f, penalty = 0.0f;  // learning_rate, f_penalty
    int sms = 0;
    bool bound = false;
    static size_t bytes(int64_t master_n, int64_t gw_n, int64_t gb_n, int64_t gx_n, int64_t scratch_n, int sms)
    {
        Carver c(nullptr);
        TrainState t;
        t.carve(c, master_n, gw_n, gb_n, gx_n, scratch_n, sms);
        return c.bytes();
    }
    void carve(Carver& c, int64_t master_n, int64_t gw_n, int64_t gb_n, int64_t gx_n, int64_t scratch_n, int n_sms)
    {
        const int64_t biggest = std::max(std::max(gw_n, gb_n), gx_n);
        master = master_n ? c.take<float>(master_n) : nullptr;
        gw = c.take<float>(gw_n);
        gb = c.take<float>(gb_n);
        gx = gx_n ? c.take<float>(gx_n) : nullptr;
        scratch = scratch_n ? c.take<float>(scratch_n) : nullptr;
        partial = c.take<float>(sumsq_blocks(biggest, n_sms));
        factor = c.take<float>(6);
        sms = n_sms;
    }
    // clip_op + updateParamsKernel (conv_layer.h:207-216) of one tensor
    void step(float* data, const float* grad, int64_t n, int slot, float pen, cudaStream_t s)
    {
        cuda_ok(launch_clip_factor(grad, n, sms, partial, factor + 2 * slot, s), "clip factor");
        cuda_ok(launch_sgd_update(data, grad, n, factor + 2 * slot, lr, pen, s), "sgd update");
    }
};

// Host staging of fp32 checkpoint data in mapped pinned memory, which the
// packer reads directly, as the reference keeps its master weights
// (uv.h:122, conv_layer.h:80-82). The file is read and checked before any
// CUDA call, so a missing or short file fails without touching the device.
struct MappedHost {
    float* host = nullptr;
    float* dev = nullptr;
    explicit MappedHost(const std::vector<float>& src)
    {
        cuda_ok(cudaHostAlloc(reinterpret_cast<void**>(&host), src.size() * sizeof(float), cudaHostAllocMapped),
                "cudaHostAlloc");
        cuda_ok(cudaHostGetDevicePointer(reinterpret_cast<void**>(&dev), host, 0), "cudaHostGetDevicePointer");
        std::memcpy(host, src.data(), src.size() * sizeof(float));
    }
    ~MappedHost()
    {
        if (host) cudaFreeHost(host);
    }
    MappedHost(const MappedHost&) = delete;
    MappedHost& operator=(const MappedHost&) = delete;
};

// Reads sum(counts) little-endian floats; a missing or short file is an error
// (the reference reads short files silently, conv_layer.h:37-38).
std::vector<float> read_floats(const char* path, const std::vector<size_t>& counts)
{
    require(path != nullptr, "null path");
    size_t total = 0;
    for (size_t c : counts) total += c;
    std::vector<float> out(total);
    FILE* f = std::fopen(path, "rb");
    if (!f) fail(AIC_ERR_IO, std::string("cannot open ") + path);
    const size_t got = std::fread(out.data(), sizeof(float), total, f);
    std::fclose(f);
    if (got != total) fail(AIC_ERR_IO, std::string("short read in ") + path);
    return out;
}

// Per-launch-site CUDA-event timing. Each traced launch is bracketed by two
// events on its own stream; collect() waits for them and accumulates the
// elapsed time, the launch count and the algorithmic work of the site.
struct Profiler {
    struct Site {
        std::string name;
        double ms = 0.0, flops = 0.0, bytes = 0.0;
        int64_t launches = 0;
        std::vector<std::pair<cudaEvent_t, cudaEvent_t>> pending;
    };
    bool enabled = false;
    std::vector<Site> sites;
    std::vector<cudaEvent_t> pool;

    ~Profiler()
    {
        for (auto& s : sites)
            for (auto& p : s.pending) pool.push_back(p.first), pool.push_back(p.second);
        for (cudaEvent_t e : pool) cudaEventDestroy(e);
    }
    cudaEvent_t event()
    {
        if (!pool.empty()) {
            cudaEvent_t e = pool.back();
            pool.pop_back();
            return e;
        }
        cudaEvent_t e;
        cuda_ok(cudaEventCreate(&e), "cudaEventCreate");
        return e;
    }
    Site& site(const std::string& name)
    {
        for (auto& s : sites)
            if (s.name == name) return s;
        sites.push_back(Site{});
        sites.back().name = name;
        return sites.back();
    }
    // Accumulates and recycles the oldest `count` pending event pairs of a site
    // (waiting for them if the device has not reached them yet).
    void settle(Site& s, size_t count)
    {
        count = std::min(count, s.pending.size());
        for (size_t i = 0; i < count; ++i) {
            auto& p = s.pending[i];
            cuda_ok(cudaEventSynchronize(p.second), "profile sync");
            float ms = 0.0f;
            cuda_ok(cudaEventElapsedTime(&ms, p.first, p.second), "profile elapsed");
            s.ms += ms;
            pool.push_back(p.first);
            pool.push_back(p.second);
        }
        s.pending.erase(s.pending.begin(), s.pending.begin() + static_cast<std::ptrdiff_t>(count));
    }
    void collect()
    {
        for (auto& s : sites) settle(s, s.pending.size());
    }
    void reset()
    {
        collect();
        sites.clear();
    }
};

// Launches through `launch` (returning cudaError_t), traced under `name` when
// a profiler is attached and enabled.
template <class F>
void traced(Profiler* p, const std::string& name, cudaStream_t s, double flops, double bytes, const char* what, F&& launch)
{
    if (!p || !p->enabled) {
        cuda_ok(launch(), what);
        return;
    }
    Profiler::Site& site = p->site(name);
    cudaEvent_t a = p->event(), b = p->event();
    cuda_ok(cudaEventRecord(a, s), "profile record");
    cuda_ok(launch(), what);
    cuda_ok(cudaEventRecord(b, s), "profile record");
    site.pending.emplace_back(a, b);
    // bounded event count on long runs: once a site holds kMaxPending pairs,
    // the older half is settled (the host is then still half that many
    // launches of the site ahead of the device)
    constexpr size_t kMaxPending = 256;
    if (site.pending.size() >= kMaxPending) p->settle(site, kMaxPending / 2);
    site.launches += 1;
    site.flops += flops;
    site.bytes += bytes;
}

// Bytes of `elems` values in the packed int4 format (codes + exponents).
inline double f_bytes(double elems) { return elems * (0.5 + 1.0 / 32.0); }

std::string join(const char* dir, const char* name)
{
    require(dir != nullptr, "null directory");
    std::string d(dir);
    if (!d.empty() && d.back() != '/') d.push_back('/');
    return d + name;
}

// ---------------------------------------------------------------- ConvLayer
struct ConvLayer {
    aic_conv_layer_desc d;
    bool is_dw;
    int64_t weight_elems, groups;
    uint32_t* w = nullptr;
    int8_t* ws = nullptr;
    float* bias = nullptr;
    bool bound = false;
    Profiler* prof = nullptr;
    std::string tag = "conv";

    explicit ConvLayer(const aic_conv_layer_desc& desc) : d(desc)
    {
        require(d.in_channels > 0 && d.out_channels > 0 && d.in_channels % 32 == 0 && d.out_channels % 32 == 0,
                "conv channels must be positive multiples of 32");
        require(d.kernel_size >= 1 && d.stride >= 1 && d.dim_in >= 1 && d.dim_out >= 1, "bad conv geometry");
        is_dw = d.kernel_size > 1 && (d.kernel_size & 1) == 1;  // conv_layer.h:49
        if (is_dw) {
            if (d.kernel_size != 3 && d.kernel_size != 5 && d.kernel_size != 7)
                fail(AIC_ERR_UNSUPPORTED, "depthwise kernel size must be 3, 5 or 7");
            require(d.in_channels == d.out_channels, "depthwise conv needs in == out channels");
            require(is_pow2(d.dim_out), "depthwise output dimension must be a power of two");
            require(d.dim_out == (d.dim_in - 1) / d.stride + 1, "depthwise output dimension mismatch");
        } else if (d.kernel_size == 1) {
            require(d.stride == 1 && d.dim_in == d.dim_out, "pointwise conv keeps the dimension");
        } else {
            if (d.kernel_size != 2 && d.kernel_size != 4) fail(AIC_ERR_UNSUPPORTED, "dense kernel size must be 2 or 4");
            require(d.stride == d.kernel_size, "dense conv is supported with stride == kernel size");
            require(is_pow2(d.dim_out) && d.dim_in == d.dim_out * d.stride, "dense conv dimension mismatch");
        }
        weight_elems = static_cast<int64_t>(d.in_channels) * d.kernel_size * d.kernel_size * (is_dw ? 1 : d.out_channels);
        groups = weight_elems >> 5;
    }
    uint8_t* wimg = nullptr;      // tensor-core weight images, AIC_CONV_FAST (dense/pointwise only)
    uint8_t* wimg_ord = nullptr;  // tensor-core images, AIC_CONV_ORDERED (k = 1, 2)
    float* wf = nullptr;          // dequantised weights (depthwise only)
    int mode = AIC_CONV_ORDERED;
    TrainState train;

    int64_t train_scratch() const { return is_dw ? 0 : 4LL * d.dim_out * d.dim_out * d.out_channels; }
    size_t train_bytes() const
    {
        return TrainState::bytes(weight_elems, weight_elems, d.out_channels, 0, train_scratch(), device_sms());
    }
    // Binds the training state and takes `m` (weight_elems fp32, device or
    // host) as the master weights; the packed weights are re-derived from it.
    void train_bind(void* buf, const float* m, float lr, float penalty, cudaStream_t s)
    {
        check_bound();
        require(buf && aligned256(buf) && m, "training buffer must be 256-byte aligned; master weights required");
        Carver c(buf);
        train.carve(c, weight_elems, weight_elems, d.out_channels, 0, train_scratch(), device_sms());
        train.lr = lr;
        train.penalty = penalty;
        cuda_ok(cudaMemcpyAsync(train.master, m, sizeof(float) * weight_elems, cudaMemcpyDefault, s), "copy master");
        repack(s);
        train.bound = true;
    }
    // quantizeKernel of the masters (conv_layer.h:98, 218) and the images
    void repack(cudaStream_t s)
    {
        cuda_ok(launch_pack_f32(train.master, weight_elems, w, ws, true, static_cast<int32_t>(weight_elems), 0, s),
                "pack weights");
        prepare(s);
    }
    // ConvLayer::backward (conv_layer.h:150-219) on one frame: gradients,
    // clipped SGD on the masters and biases, re-quantised weights. grad_in:
    // added to (pointwise, dense; the reference's atomics) or written
    // (depthwise), or null.
    void backward(const float* dy, const uint32_t* in, const int8_t* in_s, float* grad_in, cudaStream_t s)
    {
        check_bound();
        if (!train.bound) fail(AIC_ERR_STATE, "conv layer training state not bound");
        require(dy && in && in_s, "null tensor");
        const int positions = d.dim_out * d.dim_out;
        if (d.kernel_size == 1 && positions % 32 != 0)
            fail(AIC_ERR_UNSUPPORTED, "pointwise backward needs a multiple of 32 positions (kernels.h:375-379)");
        if (is_dw && positions % 4 != 0) fail(AIC_ERR_UNSUPPORTED, "depthwise backward needs a multiple of 4 positions");
        cuda_ok(launch_conv_backward_grads(in, in_s, w, ws, bias, train.master, dy, d.in_channels, d.out_channels,
                                           d.kernel_size, d.stride, d.dim_in, d.dim_out, !is_dw && !d.disable_activation,
                                           train.scratch, train.gw, train.gb, grad_in, s),
                "conv backward");
        train.step(train.master, train.gw, weight_elems, 0, train.penalty, s);
        train.step(bias, train.gb, d.out_channels, 1, 0.0f, s);
        repack(s);
    }

    size_t carve(void* base)
    {
        Carver c(base);
        w = c.take<uint32_t>(groups * 4);
        ws = c.take<int8_t>(groups);
        bias = c.take<float>(d.out_channels);
        wimg = is_dw ? nullptr : c.take<uint8_t>(conv_tc_wimg_bytes(d.in_channels, d.out_channels, d.kernel_size));
        wimg_ord = is_dw || !conv_tc_ord_supported(d.kernel_size)
                       ? nullptr
                       : c.take<uint8_t>(conv_tc_ord_wimg_bytes(d.in_channels, d.out_channels, d.kernel_size));
        wf = is_dw ? c.take<float>(weight_elems) : nullptr;
        return c.bytes();
    }
    void check_bound() const
    {
        if (!bound) fail(AIC_ERR_STATE, "conv layer parameters not bound");
    }
    // After the packed weights change: derive the tensor-core images.
    void prepare(cudaStream_t s)
    {
        if (is_dw)
            cuda_ok(launch_dw_weights(w, ws, weight_elems, wf, s), "depthwise weights");
        else
            cuda_ok(launch_build_wimg(w, ws, d.in_channels, d.out_channels, d.kernel_size, wimg, s), "weight images");
        if (wimg_ord)
            cuda_ok(launch_build_wimg_ord(w, ws, d.in_channels, d.out_channels, d.kernel_size, wimg_ord, s),
                    "weight images");
    }
    void load(const float* master, const float* b, cudaStream_t s)
    {
        check_bound();
        require(master != nullptr && b != nullptr, "null weights");
        cuda_ok(launch_pack_f32(master, weight_elems, w, ws, true, static_cast<int32_t>(weight_elems), 0, s), "pack weights");
        cuda_ok(cudaMemcpyAsync(bias, b, sizeof(float) * d.out_channels, cudaMemcpyDefault, s), "copy bias");
        prepare(s);
    }
    // Reference accumulation order on CUDA cores (bit-exact with the reference kernels).
    void forward_exact(const uint32_t* in, const int8_t* in_s, uint32_t* out, int8_t* out_s, int64_t frames,
                       cudaStream_t s)
    {
        check_bound();
        if (frames == 0) return;
        require(in && in_s && out && out_s, "null tensor");
        if (is_dw)
            cuda_ok(launch_conv_dw_direct(in, in_s, wf, bias, out, out_s, frames, d.in_channels, d.kernel_size, d.stride,
                                   d.dim_in, d.dim_out, s),
                    "conv_dw");
        else
            cuda_ok(launch_conv_gemm_simt(in, in_s, w, ws, bias, out, out_s, frames, d.in_channels, d.out_channels,
                                          d.kernel_size, d.stride, d.dim_in, d.dim_out, !d.disable_activation, s),
                    "conv_gemm_simt");
    }
    void load_file(const char* path, cudaStream_t s)
    {
        check_bound();
        MappedHost h(read_floats(path, {static_cast<size_t>(weight_elems), static_cast<size_t>(d.out_channels)}));
        load(h.dev, h.dev + weight_elems, s);
        cuda_ok(cudaStreamSynchronize(s), "load sync");
    }
    int64_t forward(const uint32_t* in, const int8_t* in_s, uint32_t* out, int8_t* out_s, int64_t frames, cudaStream_t s)
    {
        check_bound();
        if (frames == 0) return 0;
        require(in && in_s && out && out_s, "null tensor");
        const double pix_in = static_cast<double>(frames) * d.dim_in * d.dim_in;
        const double pix_out = static_cast<double>(frames) * d.dim_out * d.dim_out;
        const double ksq = static_cast<double>(d.kernel_size) * d.kernel_size;
        const double bytes = f_bytes(pix_in * d.in_channels) + f_bytes(pix_out * d.out_channels) +
                             f_bytes(static_cast<double>(weight_elems)) + 4.0 * d.out_channels;
        if (is_dw)
            traced(prof, tag, s, 2.0 * ksq * d.in_channels * pix_out, bytes, "conv_dw", [&] {
                return launch_conv_dw(in, in_s, wf, bias, out, out_s, frames, d.in_channels, d.kernel_size, d.stride,
                                      d.dim_in, d.dim_out, s);
            });
        else if (mode == AIC_CONV_FAST)
            traced(prof, tag, s, 2.0 * pix_out * d.out_channels * ksq * d.in_channels, bytes, "conv_gemm", [&] {
                return launch_conv_gemm_tc(in, in_s, wimg, bias, out, out_s, frames, d.in_channels, d.out_channels,
                                           d.kernel_size, d.dim_in, d.dim_out, !d.disable_activation,
                                           device_error_word(), s);
            });
        else if (mode == AIC_CONV_ORDERED && wimg_ord)
            traced(prof, tag, s, 2.0 * pix_out * d.out_channels * ksq * d.in_channels, bytes, "conv_gemm_ord", [&] {
                return launch_conv_gemm_tc_ord(in, in_s, wimg_ord, bias, out, out_s, frames, d.in_channels,
                                               d.out_channels, d.kernel_size, d.dim_in, d.dim_out,
                                               !d.disable_activation, device_error_word(), s);
            });
        else  // AIC_CONV_SIMT, and the 4x4 dense conv in AIC_CONV_ORDERED
            traced(prof, tag, s, 2.0 * pix_out * d.out_channels * ksq * d.in_channels, bytes, "conv_gemm_simt", [&] {
                return launch_conv_gemm_simt(in, in_s, w, ws, bias, out, out_s, frames, d.in_channels, d.out_channels,
                                             d.kernel_size, d.stride, d.dim_in, d.dim_out, !d.disable_activation, s);
            });
        return 1;
    }
};

// ---------------------------------------------------------------- ConvBlock
struct ConvBlock {
    aic_conv_block_desc d;
    std::unique_ptr<ConvLayer> layers[4];
    int final_stride;
    Profiler* prof = nullptr;
    std::string tag = "block";

    void attach(Profiler* p, const std::string& t)
    {
        prof = p;
        tag = t;
        static const char* names[4] = {".dw", ".pw1", ".pw2", ".sc"};
        for (int i = 0; i < 4; ++i) {
            layers[i]->prof = p;
            layers[i]->tag = t + names[i];
        }
    }

    explicit ConvBlock(const aic_conv_block_desc& desc) : d(desc)
    {
        require(d.survival_probability > 0.0f, "survival probability must be positive");
        final_stride = d.dim_in == d.dim_out ? 1 : d.stride;  // conv_block.h:47
        // conv_block.h:52-55
        layers[0].reset(new ConvLayer({d.in_channels, d.in_channels, d.dw_kernel, final_stride, d.dim_in, d.dim_out, 1}));
        layers[1].reset(new ConvLayer({d.in_channels, d.mid_channels, 1, 1, d.dim_out, d.dim_out, 0}));
        layers[2].reset(new ConvLayer({d.mid_channels, d.out_channels, 1, 1, d.dim_out, d.dim_out, 1}));
        layers[3].reset(new ConvLayer({d.in_channels, d.out_channels, final_stride, final_stride, d.dim_in, d.dim_out, 1}));
    }
    size_t carve(void* base)
    {
        Carver c(base);
        for (auto& l : layers) {
            char* p = c.take<char>(l->carve(nullptr));
            l->carve(p);
            if (base) l->bound = true;
        }
        return c.bytes();
    }
    int64_t buffer_words(int64_t frames) const
    {
        const int cmax = std::max(d.in_channels, std::max(d.mid_channels, d.out_channels));
        return frames * d.dim_out * d.dim_out * (cmax >> 3);
    }
    size_t workspace(int64_t frames, void* base, uint32_t** a, int8_t** as, uint32_t** b, int8_t** bs) const
    {
        Carver c(base);
        const int64_t words = buffer_words(frames);
        uint32_t* pa = c.take<uint32_t>(words);
        int8_t* pas = c.take<int8_t>(words / 4);
        uint32_t* pb = c.take<uint32_t>(words);
        int8_t* pbs = c.take<int8_t>(words / 4);
        if (a) { *a = pa; *as = pas; *b = pb; *bs = pbs; }
        return c.bytes();
    }
    int64_t forward(const uint32_t* in, const int8_t* in_s, uint32_t* out, int8_t* out_s, int64_t frames, bool train,
                    bool survived, void* ws, cudaStream_t s)
    {
        if (frames == 0) return 0;
        require(ws != nullptr && aligned256(ws), "block workspace must be 256-byte aligned");
        uint32_t *a, *b;
        int8_t *as, *bs;
        workspace(frames, ws, &a, &as, &b, &bs);
        int64_t n = 0;
        n += layers[0]->forward(in, in_s, a, as, frames, s);
        n += layers[1]->forward(a, as, b, bs, frames, s);
        n += layers[2]->forward(b, bs, a, as, frames, s);
        n += layers[3]->forward(in, in_s, b, bs, frames, s);
        const float surv_inv = 1.0f / d.survival_probability;
        const float main_mult = d.residual_factor * (train && survived ? surv_inv : 1.0f);
        const int64_t pos = frames * d.dim_out * d.dim_out;
        traced(prof, tag + ".res", s, 3.0 * pos * d.out_channels, 3.0 * f_bytes(static_cast<double>(pos) * d.out_channels),
               "residual", [&] {
                   return launch_residual(a, as, b, bs, out, out_s, pos, d.out_channels, main_mult, train && !survived, s);
               });
        return n + 1;
    }
};

// ---------------------------------------------------------------- MambaLayer
struct MambaLayer {
    aic_mamba_layer_desc d;
    int E, P;
    int64_t weight_elems, groups;
    uint32_t* w = nullptr;
    int8_t* ws = nullptr;
    float* bias = nullptr;
    float* consts = nullptr;
    void* wimg = nullptr;      // W_out as exact bf16 q * F(s) [out][E] for the tensor-core out-projection
    float2* h = nullptr;
    float2* traces = nullptr;  // trace_A | trace_B | trace_Delta [3][batch][E][P]; null: inference forward
    int batch_bound = -1;
    int mode = AIC_MAMBA_TENSOR;
    bool bound = false;
    TrainState train;
    Profiler* prof = nullptr;
    std::string tag = "mamba";

    explicit MambaLayer(const aic_mamba_layer_desc& desc) : d(desc)
    {
        require(is_pow2(d.d_model) && d.d_model >= 32, "d_model must be a power of two >= 32");
        if (d.d_state < 32 || d.d_state % 32 != 0)
            fail(AIC_ERR_UNSUPPORTED, "d_state must be a positive multiple of 32 (reference kernels.h:1089)");
        if (d.d_state / 32 > 16) fail(AIC_ERR_UNSUPPORTED, "at most 16 states per channel (d_state <= 512)");
        require(!((d.d_state / 32) & (d.d_state / 32 - 1)), "d_state/32 must be a power of two");
        require(d.out_channels >= 1 && d.out_channels % 32 == 0, "out channels must be a multiple of 32");
        require(d.activation >= 0 && d.activation <= 2, "activation must be 0, 1 or 2");
        E = 2 * d.d_model;
        P = d.d_state / 32;
        weight_elems = static_cast<int64_t>(E) * (2 + 32 + 4LL * d.d_state + d.out_channels);  // mamba_layer.h:58
        groups = weight_elems >> 5;
    }
    size_t carve(void* base)
    {
        Carver c(base);
        w = c.take<uint32_t>(groups * 4);
        ws = c.take<int8_t>(groups);
        bias = c.take<float>(d.out_channels);
        consts = c.take<float>(ssm_consts_floats(d.d_model, d.d_state));
        wimg = tc_ok() ? c.take<char>(outproj_tc_wimg_bytes(E, d.out_channels)) : nullptr;
        return c.bytes();
    }
    bool tc_ok() const { return outproj_tc_supported(E, d.out_channels); }
    // the out-projection runs on the tensor cores (split-bf16 operands) unless
    // the reference-order CUDA-core kernel is selected or the shape has no
    // tensor-core tiling
    bool use_tc() const { return mode == AIC_MAMBA_TENSOR && tc_ok(); }
    int64_t off_w() const { return static_cast<int64_t>(E) * (34 + 4LL * d.d_state); }
    size_t state_bytes(int batch) const { return static_cast<size_t>(batch) * E * P * sizeof(float2); }
    void check_bound() const
    {
        if (!bound) fail(AIC_ERR_STATE, "mamba layer parameters not bound");
    }
    void load(const float* master, const float* b, cudaStream_t s)
    {
        check_bound();
        require(master != nullptr && b != nullptr, "null weights");
        cuda_ok(launch_pack_f32(master, weight_elems, w, ws, true, static_cast<int32_t>(weight_elems), 0, s), "pack blob");
        cuda_ok(cudaMemcpyAsync(bias, b, sizeof(float) * d.out_channels, cudaMemcpyDefault, s), "copy bias");
        cuda_ok(launch_ssm_prepare(w, ws, d.d_model, d.d_state, consts, s), "ssm prepare");
        if (wimg) cuda_ok(launch_build_outproj_wimg(w, ws, off_w(), E, d.out_channels, wimg, s), "out-proj image");
    }
    void load_file(const char* path, cudaStream_t s)
    {
        check_bound();
        MappedHost m(read_floats(path, {static_cast<size_t>(weight_elems), static_cast<size_t>(d.out_channels)}));
        load(m.dev, m.dev + weight_elems, s);
        cuda_ok(cudaStreamSynchronize(s), "load sync");
    }
    // training scratch: out-projection chunk sums, normalised gradient, per-channel input terms
    int64_t train_scratch() const { return static_cast<int64_t>(E / 256) * d.out_channels + d.out_channels + E; }
    size_t train_bytes() const
    {
        return TrainState::bytes(weight_elems, weight_elems, d.out_channels, 0, train_scratch(), device_sms());
    }
    void train_bind(void* buf, const float* m, float lr, float penalty, cudaStream_t s)
    {
        check_bound();
        require(buf && aligned256(buf) && m, "training buffer must be 256-byte aligned; master weights required");
        require(E % 256 == 0, "the backward kernels run 256-channel blocks: d_model must be a multiple of 128");
        Carver c(buf);
        train.carve(c, weight_elems, weight_elems, d.out_channels, 0, train_scratch(), device_sms());
        train.lr = lr;
        train.penalty = penalty;
        cuda_ok(cudaMemcpyAsync(train.master, m, sizeof(float) * weight_elems, cudaMemcpyDefault, s), "copy master");
        repack(s);
        train.bound = true;
    }
    void repack(cudaStream_t s)
    {
        cuda_ok(launch_pack_f32(train.master, weight_elems, w, ws, true, static_cast<int32_t>(weight_elems), 0, s),
                "pack blob");
        cuda_ok(launch_ssm_prepare(w, ws, d.d_model, d.d_state, consts, s), "ssm prepare");
        if (wimg) cuda_ok(launch_build_outproj_wimg(w, ws, off_w(), E, d.out_channels, wimg, s), "out-proj image");
    }
    // MambaLayer::backward (mamba_layer.h:146-167) of the step just run: the
    // state and traces of sequence 0 after it, the step's packed input;
    // grad_in [d_model] written.
    void backward(const float* dy, const uint32_t* in, const int8_t* in_s, float* grad_in, cudaStream_t s)
    {
        check_bound();
        if (!train.bound) fail(AIC_ERR_STATE, "mamba layer training state not bound");
        if (batch_bound != 1 || !traces) fail(AIC_ERR_STATE, "backward needs the state bound for batch 1 and traces bound");
        require(dy && in && in_s && grad_in, "null tensor");
        const int64_t plane = static_cast<int64_t>(E) * P;
        float* partial = train.scratch;
        float* gnorm = partial + static_cast<int64_t>(E / 256) * d.out_channels;
        float* gx_ch = gnorm + d.out_channels;
        cuda_ok(launch_mamba_backward_grads(in, in_s, h, traces, traces + plane, traces + 2 * plane, train.master, bias, dy,
                                            d.d_model, d.d_state, d.out_channels, d.activation, partial, gnorm, gx_ch,
                                            train.gw, train.gb, grad_in, s),
                "mamba backward");
        train.step(train.master, train.gw, weight_elems, 0, train.penalty, s);
        train.step(bias, train.gb, d.out_channels, 1, 0.0f, s);
        repack(s);
    }
    void reset(cudaStream_t s)
    {
        if (batch_bound < 0) fail(AIC_ERR_STATE, "mamba state not bound");
        cuda_ok(cudaMemsetAsync(h, 0, state_bytes(batch_bound), s), "reset state");
        // mamba_layer.h:171-177 zeroes the traces with the state
        if (traces) cuda_ok(cudaMemsetAsync(traces, 0, 3 * state_bytes(batch_bound), s), "reset traces");
    }
    size_t workspace_bytes(int64_t rows) const { return ((static_cast<size_t>(rows) * E * sizeof(float)) + 255) & ~size_t(255); }
    int64_t forward(const uint32_t* in, const int8_t* in_s, float* out, int batch, int seq, void* wsp, cudaStream_t s)
    {
        check_bound();
        if (batch_bound < 0) fail(AIC_ERR_STATE, "mamba state not bound");
        require(batch == batch_bound, "batch differs from the bound state's batch");
        require(seq >= 0, "negative sequence length");
        if (seq == 0 || batch == 0) return 0;
        require(in && in_s && out && wsp && aligned256(wsp), "null or misaligned tensor");
        const bool tc = use_tc();
        scan(in, in_s, wsp, tc, batch, seq, s);
        const int64_t rows = static_cast<int64_t>(batch) * seq;
        if (tc)
            outproj_split(wsp, out, rows, s);
        else
            traced(prof, tag + ".outproj", s, 2.0 * rows * E * d.out_channels,
                   4.0 * rows * E + f_bytes(static_cast<double>(E) * d.out_channels) + 4.0 * rows * d.out_channels,
                   "outproj", [&] {
                       return launch_outproj(static_cast<const float*>(wsp), w, ws, bias, d.d_model, d.d_state,
                                             d.out_channels, d.activation, rows, out, s);
                   });
        return 2;
    }
    // The SSM scan alone: y as fp32 [rows][E], or (split) as the bf16 planes hi | lo.
    void scan(const uint32_t* in, const int8_t* in_s, void* y, bool split, int batch, int seq, cudaStream_t s)
    {
        const double rows = static_cast<double>(batch) * seq;
        // per (row, channel): 31 flops per state plus ~15 (kernels.h:1126-1176)
        traced(prof, tag + ".scan", s, rows * E * (31.0 * P + 15.0),
               f_bytes(rows * d.d_model) + 4.0 * rows * E + 2.0 * batch * E * P * 8.0 + E * P * 16.0, "ssm scan",
               [&] {
                   return launch_ssm_scan(in, in_s, w, ws, consts, d.d_model, d.d_state, h, traces, y, split, batch, seq,
                                          s);
               });
    }
    // The tensor-core out-projection of split-bf16 y planes.
    void outproj_split(const void* y_planes, float* out, int64_t rows, cudaStream_t s)
    {
        // algorithmic work 2 * rows * E * out (the tensor pipe runs it twice: hi and lo)
        traced(prof, tag + ".outproj", s, 2.0 * rows * E * d.out_channels,
               4.0 * rows * E + 2.0 * E * d.out_channels + 4.0 * rows * d.out_channels, "tensor-core outproj", [&] {
                   return launch_outproj_tc(y_planes, wimg, bias, E, d.out_channels, d.activation, rows, out,
                                            device_error_word(), s);
               });
    }
};

// ---------------------------------------------------------------- MambaBlock
struct MambaBlock {
    aic_mamba_block_desc d;
    std::unique_ptr<MambaLayer> layers[3];

    explicit MambaBlock(const aic_mamba_block_desc& desc) : d(desc)
    {
        require(d.survival_probability > 0.0f, "survival probability must be positive");
        // mamba_block.h:39-41
        layers[0].reset(new MambaLayer({d.d_model, d.d_state, d.d_model, 1}));
        layers[1].reset(new MambaLayer({d.d_model, d.d_state, d.d_model, 1}));
        layers[2].reset(new MambaLayer({d.d_model, d.d_state, d.out_channels, d.activation}));
    }
    size_t carve(void* base)
    {
        Carver c(base);
        for (auto& l : layers) {
            char* p = c.take<char>(l->carve(nullptr));
            l->carve(p);
            if (base) l->bound = true;
        }
        return c.bytes();
    }
    size_t state_bytes(int batch) const
    {
        Carver c(nullptr);
        for (auto& l : layers) c.take<char>(l->state_bytes(batch));
        return c.bytes();
    }
    void bind_state(void* base, int batch)
    {
        Carver c(base);
        for (auto& l : layers) {
            l->h = reinterpret_cast<float2*>(c.take<char>(l->state_bytes(batch)));
            l->batch_bound = batch;
            l->traces = nullptr;  // bound again after the state
        }
    }
    size_t trace_bytes(int batch) const
    {
        Carver c(nullptr);
        for (auto& l : layers) c.take<char>(3 * l->state_bytes(batch));
        return c.bytes();
    }
    void bind_traces(void* base, int batch)
    {
        Carver c(base);
        for (auto& l : layers) {
            require(batch == l->batch_bound, "traces must be bound for the bound state's batch");
            l->traces = base ? reinterpret_cast<float2*>(c.take<char>(3 * l->state_bytes(batch))) : nullptr;
        }
    }
    size_t workspace(int64_t rows, void* base, float** y, float** o, uint32_t** a, int8_t** as, uint32_t** b,
                     int8_t** bs) const
    {
        Carver c(base);
        size_t ybytes = 0;
        for (auto& l : layers) ybytes = std::max(ybytes, l->workspace_bytes(rows));
        float* py = reinterpret_cast<float*>(c.take<char>(ybytes));
        float* po = c.take<float>(static_cast<size_t>(rows) * d.d_model);
        uint32_t* pa = c.take<uint32_t>(static_cast<size_t>(rows) * d.d_model / 8);
        int8_t* pas = c.take<int8_t>(static_cast<size_t>(rows) * d.d_model / 32);
        uint32_t* pb = c.take<uint32_t>(static_cast<size_t>(rows) * d.d_model / 8);
        int8_t* pbs = c.take<int8_t>(static_cast<size_t>(rows) * d.d_model / 32);
        if (y) { *y = py; *o = po; *a = pa; *as = pas; *b = pb; *bs = pbs; }
        return c.bytes();
    }
    int64_t forward(const uint32_t* in, const int8_t* in_s, float* out, int batch, int seq, bool on_training,
                    int add_seed, bool survived, void* wsp, cudaStream_t s)
    {
        if (batch == 0 || seq == 0) return 0;
        require(wsp != nullptr && aligned256(wsp), "block workspace must be 256-byte aligned");
        const int64_t rows = static_cast<int64_t>(batch) * seq;
        float *y, *o;
        uint32_t *a, *b;
        int8_t *as, *bs;
        workspace(rows, wsp, &y, &o, &a, &as, &b, &bs);
        const int64_t n_el = rows * d.d_model, row_groups = d.d_model / 32;
        int64_t n = 0;
        // mamba_block.h:60-65
        n += layers[0]->forward(in, in_s, o, batch, seq, y, s);
        cuda_ok(launch_pack_f32(o, n_el, a, as, on_training, add_seed, row_groups, s), "requant");
        const float surv_inv = 1.0f / d.survival_probability;
        const float main_mult = d.residual_factor * (on_training && survived ? surv_inv : 1.0f);
        cuda_ok(launch_residual(a, as, in, in_s, b, bs, rows, d.d_model, main_mult, on_training && !survived, s), "residual");
        // mamba_block.h:66-71
        n += layers[1]->forward(b, bs, o, batch, seq, y, s);
        cuda_ok(launch_pack_f32(o, n_el, a, as, on_training, add_seed, row_groups, s), "requant");
        n += layers[2]->forward(a, as, out, batch, seq, y, s);
        return n + 3;
    }
};

// ---------------------------------------------------------------- Critic
struct Critic {
    aic_critic_desc d;
    float *w1 = nullptr, *w2 = nullptr, *wl = nullptr;
    float2* h = nullptr;
    float2* traces = nullptr;  // trace_w1 [batch][in][units] | trace_lambda [batch][units][in]; null: inference
    int batch_bound = -1;
    bool bound = false;
    Profiler* prof = nullptr;
    std::string tag = "critic";

    explicit Critic(const aic_critic_desc& desc) : d(desc)
    {
        require(d.in_channels > 0 && d.in_channels % 32 == 0, "critic input channels must be a multiple of 32");
        require(d.units >= 32 && d.units % 32 == 0 && d.units <= 1024, "critic units must be a multiple of 32 in [32, 1024]");
        require(d.dim_in >= 1, "bad critic input dimension");
    }
    int64_t w1_elems() const { return 2LL * d.in_channels * d.units; }
    TrainState train;
    size_t train_bytes() const { return TrainState::bytes(0, w1_elems(), 2 * d.units, w1_elems(), 0, device_sms()); }
    void train_bind(void* buf, float lr, float penalty)
    {
        check_bound();
        require(buf && aligned256(buf), "training buffer must be 256-byte aligned");
        if (d.units & (d.units - 1)) fail(AIC_ERR_UNSUPPORTED, "critic backward needs a power-of-two unit count (kernels.h:1786)");
        Carver c(buf);
        train.carve(c, 0, w1_elems(), 2 * d.units, w1_elems(), 0, device_sms());
        train.lr = lr;
        train.penalty = penalty;
        train.bound = true;
    }
    // Critic::backward (critic.h:117-131) of the step just run (batch 1): the
    // score it produced (device pointer) against real_score.
    void backward(const float* pred, float real, cudaStream_t s)
    {
        check_bound();
        if (!train.bound) fail(AIC_ERR_STATE, "critic training state not bound");
        if (batch_bound != 1 || !traces) fail(AIC_ERR_STATE, "backward needs the state bound for batch 1 and traces bound");
        require(pred != nullptr, "null score");
        cuda_ok(launch_critic_backward_grads(w2, traces, trace_l(), h, pred, real, d.units, d.in_channels, train.gw,
                                             train.gx, train.gb, s),
                "critic backward");
        train.step(w1, train.gw, w1_elems(), 0, train.penalty, s);
        train.step(w2, train.gb, 2 * d.units, 1, train.penalty, s);
        train.step(wl, train.gx, w1_elems(), 2, train.penalty, s);
    }
    size_t carve(void* base)
    {
        Carver c(base);
        w1 = c.take<float>(w1_elems());
        w2 = c.take<float>(2 * d.units);
        wl = c.take<float>(w1_elems());
        return c.bytes();
    }
    void check_bound() const
    {
        if (!bound) fail(AIC_ERR_STATE, "critic parameters not bound");
    }
    void load(const float* a, const float* b, const float* l, cudaStream_t s)
    {
        check_bound();
        require(a && b && l, "null weights");
        cuda_ok(cudaMemcpyAsync(w1, a, sizeof(float) * w1_elems(), cudaMemcpyDefault, s), "copy w1");
        cuda_ok(cudaMemcpyAsync(w2, b, sizeof(float) * 2 * d.units, cudaMemcpyDefault, s), "copy w2");
        cuda_ok(cudaMemcpyAsync(wl, l, sizeof(float) * w1_elems(), cudaMemcpyDefault, s), "copy wl");
    }
    void load_file(const char* path, cudaStream_t s)
    {
        check_bound();
        const size_t n1 = static_cast<size_t>(w1_elems()), n2 = 2 * static_cast<size_t>(d.units);
        MappedHost m(read_floats(path, {n1, n2, n1}));  // critic.h:36-38: W1, W2, Wlambda
        load(m.dev, m.dev + n1, m.dev + n1 + n2, s);
        cuda_ok(cudaStreamSynchronize(s), "load sync");
    }
    size_t state_bytes(int batch) const { return static_cast<size_t>(batch) * d.units * sizeof(float2); }
    size_t trace_bytes(int batch) const { return 2 * static_cast<size_t>(batch) * d.in_channels * d.units * sizeof(float2); }
    float2* trace_l() const { return traces ? traces + static_cast<int64_t>(batch_bound) * d.in_channels * d.units : nullptr; }
    void reset(cudaStream_t s)
    {
        if (batch_bound < 0) fail(AIC_ERR_STATE, "critic state not bound");
        cuda_ok(cudaMemsetAsync(h, 0, state_bytes(batch_bound), s), "reset critic");
        // critic.h:133-139 zeroes the traces with the state
        if (traces) cuda_ok(cudaMemsetAsync(traces, 0, trace_bytes(batch_bound), s), "reset critic traces");
    }
    size_t workspace(int64_t rows, void* base, __half** pooled, float2** hseq) const
    {
        Carver c(base);
        __half* p = c.take<__half>(static_cast<size_t>(rows) * d.in_channels);
        float2* q = c.take<float2>(static_cast<size_t>(rows) * d.units);
        if (pooled) { *pooled = p; *hseq = q; }
        return c.bytes();
    }
    int64_t forward(const uint32_t* in, const int8_t* in_s, float* score, int batch, int seq, void* wsp, cudaStream_t s)
    {
        check_bound();
        if (batch_bound < 0) fail(AIC_ERR_STATE, "critic state not bound");
        require(batch == batch_bound, "batch differs from the bound state's batch");
        if (batch == 0 || seq == 0) return 0;
        require(in && in_s && score && wsp && aligned256(wsp), "null or misaligned tensor");
        const int64_t rows = static_cast<int64_t>(batch) * seq;
        __half* pooled;
        float2* hseq;
        workspace(rows, wsp, &pooled, &hseq);
        const double hw = static_cast<double>(d.dim_in) * d.dim_in;
        traced(prof, tag + ".gap", s, rows * hw * d.in_channels, f_bytes(rows * hw * d.in_channels) + 2.0 * rows * d.in_channels,
               "critic gap", [&] { return launch_gap_f16(in, in_s, rows, d.dim_in * d.dim_in, d.in_channels, pooled, s); });
        traced(prof, tag + ".cell", s, 8.0 * rows * d.units * d.in_channels,
               2.0 * rows * d.in_channels + 16.0 * d.units * d.in_channels + 16.0 * rows * d.units + 4.0 * rows, "critic",
               [&] {
                   return launch_critic(pooled, w1, wl, w2, d.in_channels, d.units, h, hseq, traces, trace_l(), score, batch,
                                        seq, s);
               });
        return 3;
    }
    void forward_pooled(const __half* pooled, float* score, int batch, int seq, void* wsp, cudaStream_t s)
    {
        check_bound();
        if (batch_bound < 0) fail(AIC_ERR_STATE, "critic state not bound");
        require(batch == batch_bound, "batch differs from the bound state's batch");
        if (batch == 0 || seq == 0) return;
        require(pooled && score && wsp && aligned256(wsp), "null or misaligned tensor");
        __half* unused;
        float2* hseq;
        workspace(static_cast<int64_t>(batch) * seq, wsp, &unused, &hseq);
        cuda_ok(launch_critic(pooled, w1, wl, w2, d.in_channels, d.units, h, hseq, traces, trace_l(), score, batch, seq, s),
                "critic");
    }
};

// ---------------------------------------------------------------- Cortex
struct Cortex {
    aic_cortex_desc d;
    std::vector<std::unique_ptr<ConvBlock>> blocks;
    std::vector<std::unique_ptr<MambaLayer>> units;
    std::unique_ptr<MambaLayer> actor;
    std::unique_ptr<Critic> critic;
    int chunk;
    int64_t last_launches = 0;

    explicit Cortex(const aic_cortex_desc& desc) : d(desc)
    {
        require(d.n_blocks >= 1 && d.n_blocks <= AIC_MAX_BLOCKS, "n_blocks out of range");
        require(d.planes >= 1 && d.planes <= d.stem_channels && d.stem_channels % 32 == 0, "bad stem planes/channels");
        require(d.dim >= 1, "bad input dimension");
        int c = d.stem_channels, dim = d.dim;
        for (int i = 0; i < d.n_blocks; ++i) {
            const auto& b = d.blocks[i];
            require(b.in_channels == c && b.dim_in == dim, "block " + std::to_string(i) + " does not chain");
            blocks.emplace_back(new ConvBlock(b));
            c = b.out_channels;
            dim = b.dim_out;
        }
        require(c == d.d_model, "last block's channels must equal d_model");
        for (int i = 0; i < d.n_units; ++i) units.emplace_back(new MambaLayer({d.d_model, d.d_state, d.d_model, 1}));
        actor.reset(new MambaLayer({d.d_model, d.d_state, d.actor_out, d.actor_activation}));
        if (d.critic_units > 0) critic.reset(new Critic({d.d_model, d.critic_units, 1}));
        chunk = d.chunk_frames > 0 ? d.chunk_frames : 2048;
        attach_profiler();
    }
    int final_dim() const { return d.blocks[d.n_blocks - 1].dim_out; }
    size_t carve(void* base)
    {
        Carver c(base);
        auto put = [&](auto& obj) {
            char* p = c.take<char>(obj->carve(nullptr));
            obj->carve(p);
        };
        for (auto& b : blocks) put(b);
        for (auto& u : units) put(u);
        put(actor);
        if (critic) put(critic);
        if (base) {
            for (auto& b : blocks)
                for (auto& l : b->layers) l->bound = true;
            for (auto& u : units) u->bound = true;
            actor->bound = true;
            if (critic) critic->bound = true;
        }
        return c.bytes();
    }
    size_t state(int batch, void* base)
    {
        Carver c(base);
        auto take = [&](float2*& h, int& bound, size_t bytes) {
            float2* p = reinterpret_cast<float2*>(c.take<char>(bytes));
            if (base) {
                h = p;
                bound = batch;
            }
        };
        for (auto& u : units) take(u->h, u->batch_bound, u->state_bytes(batch));
        take(actor->h, actor->batch_bound, actor->state_bytes(batch));
        if (critic) take(critic->h, critic->batch_bound, critic->state_bytes(batch));
        return c.bytes();
    }
    struct Work {
        uint32_t *stem, *x, *y, *feat, *ua, *ub, *uc;
        int8_t *stem_s, *x_s, *y_s, *feat_s, *ua_s, *ub_s, *uc_s;
        void *block_ws, *layer_ws, *critic_ws;
        float* o;
    };
    size_t workspace(int batch, int seq, void* base, Work* w) const
    {
        const int64_t rows = static_cast<int64_t>(batch) * seq;
        const int64_t ch = std::min<int64_t>(rows, chunk);
        Carver c(base);
        Work t{};
        t.stem = c.take<uint32_t>(ch * d.dim * d.dim * d.stem_channels / 8);
        t.stem_s = c.take<int8_t>(ch * d.dim * d.dim * d.stem_channels / 32);
        int64_t act_words = 0, block_ws = 0;
        for (auto& b : blocks) {
            act_words = std::max<int64_t>(act_words, ch * b->d.dim_out * b->d.dim_out * b->d.out_channels / 8);
            block_ws = std::max<int64_t>(block_ws, b->workspace(ch, nullptr, nullptr, nullptr, nullptr, nullptr));
        }
        t.x = c.take<uint32_t>(act_words);
        t.x_s = c.take<int8_t>(act_words / 4);
        t.y = c.take<uint32_t>(act_words);
        t.y_s = c.take<int8_t>(act_words / 4);
        t.block_ws = c.take<char>(block_ws);
        const int64_t fw = rows * d.d_model / 8;
        t.feat = c.take<uint32_t>(fw);
        t.feat_s = c.take<int8_t>(fw / 4);
        t.ua = c.take<uint32_t>(fw);
        t.ua_s = c.take<int8_t>(fw / 4);
        t.ub = c.take<uint32_t>(fw);
        t.ub_s = c.take<int8_t>(fw / 4);
        t.uc = c.take<uint32_t>(fw);
        t.uc_s = c.take<int8_t>(fw / 4);
        t.o = c.take<float>(rows * d.d_model);
        size_t lw = actor->workspace_bytes(rows);
        for (auto& u : units) lw = std::max(lw, u->workspace_bytes(rows));
        t.layer_ws = c.take<char>(lw);
        t.critic_ws = critic ? c.take<char>(critic->workspace(rows, nullptr, nullptr, nullptr)) : nullptr;
        if (w) *w = t;
        return c.bytes();
    }
    int64_t plane_elems() const { return static_cast<int64_t>(d.planes) * d.dim * d.dim; }

    // Host-mode extras after the device workspace: two staging buffers for the
    // input planes of one chunk each, and device copies of the outputs.
    size_t host_workspace(int batch, int seq, void* base, Work* w, __half** stage, float** actor_dev,
                          float** critic_dev) const
    {
        const int64_t rows = static_cast<int64_t>(batch) * seq;
        const int64_t ch = std::min<int64_t>(rows, chunk);
        Carver c(base);
        void* dev = c.take<char>(workspace(batch, seq, nullptr, nullptr));
        __half* s0 = c.take<__half>(ch * plane_elems());
        __half* s1 = c.take<__half>(ch * plane_elems());
        float* a = c.take<float>(rows * d.actor_out);
        float* k = c.take<float>(rows);
        if (base) {
            workspace(batch, seq, dev, w);
            stage[0] = s0;
            stage[1] = s1;
            *actor_dev = a;
            *critic_dev = k;
        }
        return c.bytes();
    }

    cudaStream_t copy_stream = nullptr;
    cudaEvent_t ev_ready[2] = {nullptr, nullptr}, ev_free[2] = {nullptr, nullptr};
    Profiler prof;

    ~Cortex()
    {
        for (int i = 0; i < 2; ++i) {
            if (ev_ready[i]) cudaEventDestroy(ev_ready[i]);
            if (ev_free[i]) cudaEventDestroy(ev_free[i]);
        }
        if (copy_stream) cudaStreamDestroy(copy_stream);
    }
    void attach_profiler()
    {
        for (size_t i = 0; i < blocks.size(); ++i) blocks[i]->attach(&prof, "b" + std::to_string(i));
        for (size_t i = 0; i < units.size(); ++i) {
            units[i]->prof = &prof;
            units[i]->tag = "u" + std::to_string(i);
        }
        actor->prof = &prof;
        actor->tag = "actor";
        if (critic) critic->prof = &prof;
    }

    // Shared body of the device- and host-buffer forwards. With `host_planes`
    // set, chunk i is copied into stage[i & 1] on copy_stream while chunk i-1
    // runs; the stem kernel of chunk i waits for that copy, and the copy of
    // chunk i+2 waits for that stem kernel.
    void run(const __half* dev_planes, const __half* host_planes, __half* const* stage, int batch, int seq,
             float* actor_out, float* critic_out, uint32_t* features, int8_t* features_s, const Work& w, cudaStream_t s)
    {
        const int64_t rows = static_cast<int64_t>(batch) * seq;
        uint32_t* feat = features ? features : w.feat;
        int8_t* feat_s = features ? features_s : w.feat_s;
        require(feat_s != nullptr, "features exponents missing");
        const int64_t pe = plane_elems();
        if (host_planes) {
            if (!copy_stream) cuda_ok(cudaStreamCreateWithFlags(&copy_stream, cudaStreamNonBlocking), "copy stream");
            for (int i = 0; i < 2; ++i) {
                if (!ev_ready[i]) cuda_ok(cudaEventCreateWithFlags(&ev_ready[i], cudaEventDisableTiming), "event");
                if (!ev_free[i]) cuda_ok(cudaEventCreateWithFlags(&ev_free[i], cudaEventDisableTiming), "event");
            }
            // the staging buffers are free once everything queued before this call has run
            for (int i = 0; i < 2; ++i) cuda_ok(cudaEventRecord(ev_free[i], s), "event record");
        }
        int64_t n = 0;
        int64_t ci = 0;
        for (int64_t f0 = 0; f0 < rows; f0 += chunk, ++ci) {
            const int64_t fc = std::min<int64_t>(chunk, rows - f0);
            const __half* src = dev_planes ? dev_planes + f0 * pe : nullptr;
            if (host_planes) {
                const int b = static_cast<int>(ci & 1);
                cuda_ok(cudaStreamWaitEvent(copy_stream, ev_free[b], 0), "wait free");
                cuda_ok(cudaMemcpyAsync(stage[b], host_planes + f0 * pe, sizeof(__half) * fc * pe, cudaMemcpyHostToDevice,
                                        copy_stream),
                        "planes H2D");
                cuda_ok(cudaEventRecord(ev_ready[b], copy_stream), "event record");
                cuda_ok(cudaStreamWaitEvent(s, ev_ready[b], 0), "wait ready");
                src = stage[b];
            }
            const double pix = static_cast<double>(fc) * d.dim * d.dim;
            traced(&prof, "stem", s, pix * d.stem_channels, pix * d.planes * 2.0 + f_bytes(pix * d.stem_channels), "stem",
                   [&] { return launch_stem_pack(src, fc, d.planes, d.stem_channels, d.dim, w.stem, w.stem_s, s); });
            if (host_planes) cuda_ok(cudaEventRecord(ev_free[ci & 1], s), "event record");
            ++n;
            const uint32_t* cur = w.stem;
            const int8_t* cur_s = w.stem_s;
            for (size_t i = 0; i < blocks.size(); ++i) {
                uint32_t* dst = (i & 1) ? w.y : w.x;
                int8_t* dst_s = (i & 1) ? w.y_s : w.x_s;
                n += blocks[i]->forward(cur, cur_s, dst, dst_s, fc, false, true, w.block_ws, s);
                cur = dst;
                cur_s = dst_s;
            }
            const int fd = final_dim();
            const double gp = static_cast<double>(fc) * fd * fd * d.d_model;
            traced(&prof, "gap", s, gp, f_bytes(gp) + f_bytes(static_cast<double>(fc) * d.d_model), "gap", [&] {
                return launch_gap(cur, cur_s, fc, fd * fd, d.d_model, nullptr, feat + f0 * d.d_model / 8,
                                  feat_s + f0 * d.d_model / 32, s);
            });
            ++n;
        }
        // Mamba trunk: units of layer -> requant -> residual with the unit input.
        const uint32_t* cur = feat;
        const int8_t* cur_s = feat_s;
        uint32_t* bufs[2] = {w.ub, w.uc};
        int8_t* bufs_s[2] = {w.ub_s, w.uc_s};
        const double el = static_cast<double>(rows) * d.d_model;
        for (size_t i = 0; i < units.size(); ++i) {
            const std::string tag = "u" + std::to_string(i);
            n += units[i]->forward(cur, cur_s, w.o, batch, seq, w.layer_ws, s);
            traced(&prof, tag + ".requant", s, 3.0 * el, 4.0 * el + f_bytes(el), "unit requant",
                   [&] { return launch_pack_f32(w.o, rows * d.d_model, w.ua, w.ua_s, false, 0, 0, s); });
            uint32_t* nxt = bufs[i & 1];
            int8_t* nxt_s = bufs_s[i & 1];
            traced(&prof, tag + ".res", s, 3.0 * el, 3.0 * f_bytes(el), "unit residual", [&] {
                return launch_residual(w.ua, w.ua_s, cur, cur_s, nxt, nxt_s, rows, d.d_model, d.unit_residual_factor,
                                       false, s);
            });
            n += 2;
            cur = nxt;
            cur_s = nxt_s;
        }
        n += actor->forward(cur, cur_s, actor_out, batch, seq, w.layer_ws, s);
        if (critic && critic_out) n += critic->forward(cur, cur_s, critic_out, batch, seq, w.critic_ws, s);
        last_launches = n;
    }

    void forward(const uint16_t* planes, int batch, int seq, float* actor_out, float* critic_out, uint32_t* features,
                 int8_t* features_s, void* wsp, cudaStream_t s)
    {
        last_launches = 0;
        if (batch == 0 || seq == 0) return;
        require(planes && actor_out && wsp && aligned256(wsp), "null or misaligned tensor");
        Work w;
        workspace(batch, seq, wsp, &w);
        run(reinterpret_cast<const __half*>(planes), nullptr, nullptr, batch, seq, actor_out, critic_out, features,
            features_s, w, s);
    }

    void forward_host(const uint16_t* planes_host, int batch, int seq, float* actor_host, float* critic_host, void* wsp,
                      cudaStream_t s)
    {
        last_launches = 0;
        if (batch == 0 || seq == 0) return;
        require(planes_host && actor_host && wsp && aligned256(wsp), "null or misaligned buffer");
        Work w;
        __half* stage[2];
        float *actor_dev, *critic_dev;
        host_workspace(batch, seq, wsp, &w, stage, &actor_dev, &critic_dev);
        const bool want_critic = critic && critic_host;
        run(nullptr, reinterpret_cast<const __half*>(planes_host), stage, batch, seq, actor_dev,
            want_critic ? critic_dev : nullptr, nullptr, nullptr, w, s);
        const int64_t rows = static_cast<int64_t>(batch) * seq;
        cuda_ok(cudaMemcpyAsync(actor_host, actor_dev, sizeof(float) * rows * d.actor_out, cudaMemcpyDeviceToHost, s),
                "actor D2H");
        if (want_critic)
            cuda_ok(cudaMemcpyAsync(critic_host, critic_dev, sizeof(float) * rows, cudaMemcpyDeviceToHost, s), "critic D2H");
    }
};

template <class T>
T* handle(void* p, const char* what)
{
    if (!p) fail(AIC_ERR_INVALID, std::string("null ") + what + " handle");
    return static_cast<T*>(p);
}

// ---- fixed scratch for aic_mamba_layer_forward_noalloc ------------------
// Scratch for callers that cannot allocate device memory themselves: the
// Mamba layer's per-row SSM output y_ssm lives in this array instead of a
// caller-provided workspace. One instance per device, resident from the time
// the library is loaded on that device until the process exits.
constexpr size_t kNoAllocScratchFloats = size_t(1) << 20;  // 4 MiB: rows * 2 * d_model <= 1,048,576
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];

constexpr int kMaxDevices = 64;
float* g_noalloc_addr[kMaxDevices] = {};
std::mutex g_noalloc_mu;

// Device address of g_noalloc_scratch on the current device. In host code the
// symbol is only a host-side stand-in, so the address is looked up once per
// device (with that device current) and cached.
float* noalloc_scratch()
{
    int dev = 0;
    cuda_ok(cudaGetDevice(&dev), "cudaGetDevice");
    require(dev >= 0 && dev < kMaxDevices, "device ordinal out of range");
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_addr[dev]) {
        void* p = nullptr;
        cuda_ok(cudaGetSymbolAddress(&p, g_noalloc_scratch), "cudaGetSymbolAddress(g_noalloc_scratch)");
        g_noalloc_addr[dev] = static_cast<float*>(p);
    }
    return g_noalloc_addr[dev];
}

}  // namespace
}  // namespace aic

using namespace aic;

extern "C" {

AIC_API const char* aic_last_error(void) { return g_last_error.c_str(); }
AIC_API int aic_abi_version(void) { return 1; }

AIC_API aic_status aic_device_error_sync(int* code)
{
    return guarded([&] {
        require(code != nullptr, "null output");
        cuda_ok(cudaDeviceSynchronize(), "device synchronize");
        int* word = device_error_word();
        if (!word) fail(AIC_ERR_CUDA, "device error word unavailable");
        int v = 0;
        cuda_ok(cudaMemcpy(&v, word, sizeof(int), cudaMemcpyDeviceToHost), "read error word");
        const int zero = 0;
        cuda_ok(cudaMemcpy(word, &zero, sizeof(int), cudaMemcpyHostToDevice), "clear error word");
        *code = v;
    });
}

AIC_API aic_status aic_pack_f32(const float* in, int64_t n, uint32_t* out, int8_t* out_s, int stochastic,
                                int32_t add_idx, void* stream)
{
    return guarded([&] {
        require(n >= 0 && n % 32 == 0, "n must be a non-negative multiple of 32");
        require(n == 0 || (in && out && out_s), "null tensor");
        cuda_ok(launch_pack_f32(in, n, out, out_s, stochastic != 0, add_idx, 0, as_stream(stream)), "pack");
    });
}

AIC_API aic_status aic_stem_pack(const uint16_t* planes, int64_t frames, int planes_present, int channels, int dim,
                                 uint32_t* out, int8_t* out_s, void* stream)
{
    return guarded([&] {
        require(frames >= 0 && dim >= 1 && channels > 0 && channels % 32 == 0, "bad stem geometry");
        require(planes_present >= 0 && planes_present <= channels, "planes_present out of range");
        require(frames == 0 || (planes && out && out_s), "null tensor");
        cuda_ok(launch_stem_pack(reinterpret_cast<const __half*>(planes), frames, planes_present, channels, dim, out, out_s,
                                 as_stream(stream)),
                "stem");
    });
}

AIC_API aic_status aic_residual_add(const uint32_t* main_in, const int8_t* main_s, const uint32_t* res,
                                    const int8_t* res_s, uint32_t* out, int8_t* out_s, int64_t positions, int channels,
                                    float main_mult, int skipped, void* stream)
{
    return guarded([&] {
        require(positions >= 0 && channels > 0 && channels % 32 == 0, "bad residual geometry");
        require(positions == 0 || (res && res_s && out && out_s && (skipped || (main_in && main_s))), "null tensor");
        cuda_ok(launch_residual(main_in, main_s, res, res_s, out, out_s, positions, channels, main_mult, skipped != 0,
                                as_stream(stream)),
                "residual");
    });
}

AIC_API aic_status aic_gap(const uint32_t* in, const int8_t* in_s, int64_t frames, int hw, int channels, float* out_f32,
                           uint32_t* out_q, int8_t* out_qs, void* stream)
{
    return guarded([&] {
        require(frames >= 0 && hw >= 1 && channels > 0 && channels % 32 == 0, "bad gap geometry");
        require(frames == 0 || (in && in_s), "null tensor");
        require((out_q == nullptr) == (out_qs == nullptr), "out_q and out_qs go together");
        cuda_ok(launch_gap(in, in_s, frames, hw, channels, out_f32, out_q, out_qs, as_stream(stream)), "gap");
    });
}

AIC_API aic_status aic_gap_f16(const uint32_t* in, const int8_t* in_s, int64_t frames, int hw, int channels,
                               uint16_t* out, void* stream)
{
    return guarded([&] {
        require(frames >= 0 && hw >= 1 && channels > 0 && channels % 32 == 0, "bad gap geometry");
        require(frames == 0 || (in && in_s && out), "null tensor");
        cuda_ok(launch_gap_f16(in, in_s, frames, hw, channels, reinterpret_cast<__half*>(out), as_stream(stream)), "gap");
    });
}

AIC_API aic_status aic_selftest_wait_timeout(int code, int* returned, void* stream)
{
    return guarded([&] {
        require(returned != nullptr && code != 0, "bad self-test arguments");
        cuda_ok(launch_selftest_wait(code, returned, as_stream(stream)), "wait self-test");
    });
}
AIC_API aic_status aic_selftest_rcp(uint64_t* mismatches, float* first_bad, void* stream)
{
    return guarded([&] {
        require(mismatches && first_bad, "null buffer");
        cuda_ok(launch_selftest_rcp(reinterpret_cast<unsigned long long*>(mismatches), first_bad, as_stream(stream)),
                "rcp self-test");
    });
}

AIC_API aic_status aic_audio_workspace_bytes(size_t* bytes)
{
    return guarded([&] {
        require(bytes != nullptr, "null output");
        *bytes = audio_workspace_bytes();
    });
}

AIC_API aic_status aic_audio_frontend(const int16_t* pcm, uint16_t* frame, int dim, int first_channel, void* workspace,
                                      void* stream)
{
    return guarded([&] {
        require(pcm && frame && workspace && aligned256(workspace), "null or misaligned buffer");
        require(dim >= 2 && dim <= 1024 && dim % 2 == 0, "dim must be even and at most 1024");
        require(first_channel >= 0, "bad channel");
        cuda_ok(launch_audio_frontend(reinterpret_cast<const short*>(pcm), reinterpret_cast<__half*>(frame), dim,
                                      first_channel, workspace, as_stream(stream)),
                "audio front-end");
    });
}

AIC_API aic_status aic_screen_frontend(const uint8_t* bgra, uint16_t* frame, int dim, int first_channel, int train,
                                      uint32_t frame_seed, float brightness, float contrast, void* stream)
{
    return guarded([&] {
        require(bgra && frame, "null buffer");
        require(dim >= 2 && dim % 2 == 0, "dim must be even");
        require(first_channel >= 0, "bad channel");
        cuda_ok(launch_screen_frontend(bgra, reinterpret_cast<__half*>(frame), dim, first_channel, train != 0, frame_seed,
                                       brightness, contrast, as_stream(stream)),
                "screen front-end");
    });
}

AIC_API aic_status aic_set_actions(const float* probs, int64_t rows, int count, uint64_t* actions, void* stream)
{
    return guarded([&] {
        require(rows >= 0 && count >= 0, "bad action geometry");
        require(rows == 0 || count == 0 || (probs && actions), "null tensor");
        cuda_ok(launch_set_actions(probs, rows, count, reinterpret_cast<unsigned long long*>(actions), as_stream(stream)),
                "actions");
    });
}

// ---- ConvLayer
AIC_API aic_status aic_conv_layer_create(const aic_conv_layer_desc* desc, aic_conv_layer* out)
{
    return guarded([&] {
        require(desc && out, "null argument");
        *out = reinterpret_cast<aic_conv_layer>(new ConvLayer(*desc));
    });
}
AIC_API aic_status aic_conv_layer_sizes(aic_conv_layer l, int64_t* weight_elems, int64_t* bias_elems, size_t* param_bytes)
{
    return guarded([&] {
        auto* c = handle<ConvLayer>(l, "conv layer");
        if (weight_elems) *weight_elems = c->weight_elems;
        if (bias_elems) *bias_elems = c->d.out_channels;
        if (param_bytes) {
            ConvLayer tmp(*c);
            *param_bytes = tmp.carve(nullptr);
        }
    });
}
AIC_API aic_status aic_conv_layer_bind(aic_conv_layer l, void* dev_params)
{
    return guarded([&] {
        auto* c = handle<ConvLayer>(l, "conv layer");
        require(dev_params && aligned256(dev_params), "parameters must be 256-byte aligned");
        c->carve(dev_params);
        c->bound = true;
    });
}
AIC_API aic_status aic_conv_layer_param_ptrs(aic_conv_layer l, uint32_t** weights, int8_t** weight_scales, float** bias)
{
    return guarded([&] {
        auto* c = handle<ConvLayer>(l, "conv layer");
        c->check_bound();
        if (weights) *weights = c->w;
        if (weight_scales) *weight_scales = c->ws;
        if (bias) *bias = c->bias;
    });
}
AIC_API aic_status aic_conv_layer_load_weights(aic_conv_layer l, const float* master, const float* bias, void* stream)
{
    return guarded([&] { handle<ConvLayer>(l, "conv layer")->load(master, bias, as_stream(stream)); });
}
AIC_API aic_status aic_conv_layer_load_file_sync(aic_conv_layer l, const char* path, void* stream)
{
    return guarded([&] { handle<ConvLayer>(l, "conv layer")->load_file(path, as_stream(stream)); });
}
AIC_API aic_status aic_conv_layer_forward(aic_conv_layer l, const uint32_t* in, const int8_t* in_s, uint32_t* out,
                                          int8_t* out_s, int64_t frames, void* stream)
{
    return guarded([&] {
        require(frames >= 0, "negative frame count");
        handle<ConvLayer>(l, "conv layer")->forward(in, in_s, out, out_s, frames, as_stream(stream));
    });
}
AIC_API aic_status aic_conv_layer_forward_exact(aic_conv_layer l, const uint32_t* in, const int8_t* in_s,
                                                uint32_t* out, int8_t* out_s, int64_t frames, void* stream)
{
    return guarded([&] {
        require(frames >= 0, "negative frame count");
        handle<ConvLayer>(l, "conv layer")->forward_exact(in, in_s, out, out_s, frames, as_stream(stream));
    });
}
AIC_API aic_status aic_conv_layer_set_mode(aic_conv_layer l, int mode)
{
    return guarded([&] {
        require(mode == AIC_CONV_ORDERED || mode == AIC_CONV_FAST || mode == AIC_CONV_SIMT, "unknown conv mode");
        handle<ConvLayer>(l, "conv layer")->mode = mode;
    });
}
AIC_API aic_status aic_conv_layer_destroy(aic_conv_layer l)
{
    return guarded([&] { delete reinterpret_cast<ConvLayer*>(l); });
}

// ---- ConvBlock
AIC_API aic_status aic_conv_block_create(const aic_conv_block_desc* desc, aic_conv_block* out)
{
    return guarded([&] {
        require(desc && out, "null argument");
        *out = reinterpret_cast<aic_conv_block>(new ConvBlock(*desc));
    });
}
AIC_API aic_status aic_conv_block_layer(aic_conv_block b, int i, aic_conv_layer* out)
{
    return guarded([&] {
        auto* c = handle<ConvBlock>(b, "conv block");
        require(i >= 0 && i < 4 && out, "layer index out of range");
        *out = reinterpret_cast<aic_conv_layer>(c->layers[i].get());
    });
}
AIC_API aic_status aic_conv_block_param_bytes(aic_conv_block b, size_t* bytes)
{
    return guarded([&] {
        auto* c = handle<ConvBlock>(b, "conv block");
        require(bytes != nullptr, "null output");
        *bytes = c->carve(nullptr);
    });
}
AIC_API aic_status aic_conv_block_bind(aic_conv_block b, void* dev_params)
{
    return guarded([&] {
        auto* c = handle<ConvBlock>(b, "conv block");
        require(dev_params && aligned256(dev_params), "parameters must be 256-byte aligned");
        c->carve(dev_params);
    });
}
AIC_API aic_status aic_conv_block_workspace_bytes(aic_conv_block b, int64_t frames, size_t* bytes)
{
    return guarded([&] {
        auto* c = handle<ConvBlock>(b, "conv block");
        require(bytes && frames >= 0, "bad argument");
        *bytes = c->workspace(frames, nullptr, nullptr, nullptr, nullptr, nullptr);
    });
}
AIC_API aic_status aic_conv_block_load_dir_sync(aic_conv_block b, const char* dir, void* stream)
{
    return guarded([&] {
        auto* c = handle<ConvBlock>(b, "conv block");
        static const char* names[4] = {"depthwise_layer.bin", "conv_layer1.bin", "conv_layer2.bin", "residual_layer.bin"};
        for (int i = 0; i < 4; ++i) c->layers[i]->load_file(join(dir, names[i]).c_str(), as_stream(stream));
    });
}
AIC_API aic_status aic_conv_block_forward(aic_conv_block b, const uint32_t* in, const int8_t* in_s, uint32_t* out,
                                          int8_t* out_s, int64_t frames, int train_mode, int is_survived, void* workspace,
                                          void* stream)
{
    return guarded([&] {
        require(frames >= 0, "negative frame count");
        handle<ConvBlock>(b, "conv block")
            ->forward(in, in_s, out, out_s, frames, train_mode != 0, is_survived != 0, workspace, as_stream(stream));
    });
}
AIC_API aic_status aic_conv_block_destroy(aic_conv_block b)
{
    return guarded([&] { delete reinterpret_cast<ConvBlock*>(b); });
}

// ---- MambaLayer
AIC_API aic_status aic_mamba_layer_create(const aic_mamba_layer_desc* desc, aic_mamba_layer* out)
{
    return guarded([&] {
        require(desc && out, "null argument");
        *out = reinterpret_cast<aic_mamba_layer>(new MambaLayer(*desc));
    });
}
AIC_API aic_status aic_mamba_layer_sizes(aic_mamba_layer l, int64_t* weight_elems, int64_t* bias_elems, size_t* param_bytes)
{
    return guarded([&] {
        auto* m = handle<MambaLayer>(l, "mamba layer");
        if (weight_elems) *weight_elems = m->weight_elems;
        if (bias_elems) *bias_elems = m->d.out_channels;
        if (param_bytes) {
            MambaLayer tmp(*m);
            *param_bytes = tmp.carve(nullptr);
        }
    });
}
AIC_API aic_status aic_mamba_layer_bind(aic_mamba_layer l, void* dev_params)
{
    return guarded([&] {
        auto* m = handle<MambaLayer>(l, "mamba layer");
        require(dev_params && aligned256(dev_params), "parameters must be 256-byte aligned");
        m->carve(dev_params);
        m->bound = true;
    });
}
AIC_API aic_status aic_mamba_layer_param_ptrs(aic_mamba_layer l, uint32_t** weights, int8_t** weight_scales, float** bias)
{
    return guarded([&] {
        auto* m = handle<MambaLayer>(l, "mamba layer");
        m->check_bound();
        if (weights) *weights = m->w;
        if (weight_scales) *weight_scales = m->ws;
        if (bias) *bias = m->bias;
    });
}
AIC_API aic_status aic_mamba_layer_load_weights(aic_mamba_layer l, const float* master, const float* bias, void* stream)
{
    return guarded([&] { handle<MambaLayer>(l, "mamba layer")->load(master, bias, as_stream(stream)); });
}
AIC_API aic_status aic_mamba_layer_load_file_sync(aic_mamba_layer l, const char* path, void* stream)
{
    return guarded([&] { handle<MambaLayer>(l, "mamba layer")->load_file(path, as_stream(stream)); });
}
AIC_API aic_status aic_mamba_layer_state_bytes(aic_mamba_layer l, int batch, size_t* bytes)
{
    return guarded([&] {
        auto* m = handle<MambaLayer>(l, "mamba layer");
        require(bytes && batch >= 0, "bad argument");
        *bytes = m->state_bytes(batch);
    });
}
AIC_API aic_status aic_mamba_layer_bind_state(aic_mamba_layer l, void* dev_state, int batch)
{
    return guarded([&] {
        auto* m = handle<MambaLayer>(l, "mamba layer");
        require(batch >= 0 && (batch == 0 || (dev_state && aligned256(dev_state))), "state must be 256-byte aligned");
        m->h = static_cast<float2*>(dev_state);
        m->batch_bound = batch;
        m->traces = nullptr;  // bound again after the state
    });
}
AIC_API aic_status aic_mamba_layer_trace_bytes(aic_mamba_layer l, int batch, size_t* bytes)
{
    return guarded([&] {
        auto* m = handle<MambaLayer>(l, "mamba layer");
        require(bytes && batch >= 0, "bad argument");
        *bytes = 3 * m->state_bytes(batch);
    });
}
AIC_API aic_status aic_mamba_layer_bind_traces(aic_mamba_layer l, void* dev_traces, int batch)
{
    return guarded([&] {
        auto* m = handle<MambaLayer>(l, "mamba layer");
        require(batch == m->batch_bound, "traces must be bound for the bound state's batch");
        require(!dev_traces || aligned256(dev_traces), "traces must be 256-byte aligned");
        m->traces = static_cast<float2*>(dev_traces);
    });
}
AIC_API aic_status aic_mamba_layer_reset_state(aic_mamba_layer l, void* stream)
{
    return guarded([&] { handle<MambaLayer>(l, "mamba layer")->reset(as_stream(stream)); });
}
AIC_API aic_status aic_mamba_layer_workspace_bytes(aic_mamba_layer l, int64_t rows, size_t* bytes)
{
    return guarded([&] {
        auto* m = handle<MambaLayer>(l, "mamba layer");
        require(bytes && rows >= 0, "bad argument");
        *bytes = m->workspace_bytes(rows);
    });
}
AIC_API aic_status aic_mamba_layer_forward(aic_mamba_layer l, const uint32_t* in, const int8_t* in_s, float* out,
                                           int batch, int seq, void* workspace, void* stream)
{
    return guarded([&] {
        handle<MambaLayer>(l, "mamba layer")->forward(in, in_s, out, batch, seq, workspace, as_stream(stream));
    });
}
AIC_API aic_status aic_mamba_layer_outproj(aic_mamba_layer l, const float* y, float* out, int64_t rows, void* stream)
{
    return guarded([&] {
        auto* m = handle<MambaLayer>(l, "mamba layer");
        m->check_bound();
        require(rows >= 0 && (rows == 0 || (y && out)), "bad out-projection arguments");
        cuda_ok(launch_outproj(y, m->w, m->ws, m->bias, m->d.d_model, m->d.d_state, m->d.out_channels, m->d.activation,
                               rows, out, as_stream(stream)),
                "outproj");
    });
}
AIC_API aic_status aic_mamba_layer_set_mode(aic_mamba_layer l, int mode)
{
    return guarded([&] {
        require(mode == AIC_MAMBA_TENSOR || mode == AIC_MAMBA_EXACT, "unknown mamba mode");
        handle<MambaLayer>(l, "mamba layer")->mode = mode;
    });
}
AIC_API aic_status aic_mamba_layer_scan(aic_mamba_layer l, const uint32_t* in, const int8_t* in_s, void* y, int batch,
                                        int seq, int y_split, void* stream)
{
    return guarded([&] {
        auto* m = handle<MambaLayer>(l, "mamba layer");
        m->check_bound();
        if (m->batch_bound < 0) fail(AIC_ERR_STATE, "mamba state not bound");
        require(batch == m->batch_bound, "batch differs from the bound state's batch");
        require(seq >= 0, "negative sequence length");
        if (batch == 0 || seq == 0) return;
        require(in && in_s && y && aligned256(y), "null or misaligned tensor");
        m->scan(in, in_s, y, y_split != 0, batch, seq, as_stream(stream));
    });
}
AIC_API aic_status aic_mamba_layer_outproj_split(aic_mamba_layer l, const void* y_planes, float* out, int64_t rows,
                                                 void* stream)
{
    return guarded([&] {
        auto* m = handle<MambaLayer>(l, "mamba layer");
        m->check_bound();
        if (!m->tc_ok())
            fail(AIC_ERR_UNSUPPORTED, "out channels have no tensor-core tiling (multiple of 32, <= 256 or a multiple of 256)");
        require(rows >= 0 && (rows == 0 || (y_planes && out)), "bad out-projection arguments");
        require(rows == 0 || aligned256(y_planes), "y planes must be 256-byte aligned");
        m->outproj_split(y_planes, out, rows, as_stream(stream));
    });
}
AIC_API aic_status aic_mamba_layer_forward_noalloc(aic_mamba_layer l, const uint32_t* in, const int8_t* in_s,
                                                   float* out, int batch, int seq, void* stream)
{
    return guarded([&] {
        auto* m = handle<MambaLayer>(l, "mamba layer");
        require(batch >= 0 && seq >= 0, "bad extents");
        const size_t need = static_cast<size_t>(batch) * seq * m->E;
        if (need > kNoAllocScratchFloats)
            fail(AIC_ERR_INVALID, "aic_mamba_layer_forward_noalloc: batch * seq * 2 * d_model = " + std::to_string(need) +
                                      " floats exceeds the fixed scratch of " + std::to_string(kNoAllocScratchFloats) +
                                      " floats (4 MiB); use aic_mamba_layer_forward with a workspace");
        // empty extents still go through forward()'s checks of the bound
        // parameters, state and batch, so both entry points agree on them
        m->forward(in, in_s, out, batch, seq, need ? noalloc_scratch() : nullptr, as_stream(stream));
    });
}
AIC_API aic_status aic_mamba_layer_destroy(aic_mamba_layer l)
{
    return guarded([&] { delete reinterpret_cast<MambaLayer*>(l); });
}

// ---- MambaBlock
AIC_API aic_status aic_mamba_block_create(const aic_mamba_block_desc* desc, aic_mamba_block* out)
{
    return guarded([&] {
        require(desc && out, "null argument");
        *out = reinterpret_cast<aic_mamba_block>(new MambaBlock(*desc));
    });
}
AIC_API aic_status aic_mamba_block_layer(aic_mamba_block b, int i, aic_mamba_layer* out)
{
    return guarded([&] {
        auto* m = handle<MambaBlock>(b, "mamba block");
        require(i >= 0 && i < 3 && out, "layer index out of range");
        *out = reinterpret_cast<aic_mamba_layer>(m->layers[i].get());
    });
}
AIC_API aic_status aic_mamba_block_param_bytes(aic_mamba_block b, size_t* bytes)
{
    return guarded([&] {
        auto* m = handle<MambaBlock>(b, "mamba block");
        require(bytes != nullptr, "null output");
        *bytes = m->carve(nullptr);
    });
}
AIC_API aic_status aic_mamba_block_bind(aic_mamba_block b, void* dev_params)
{
    return guarded([&] {
        auto* m = handle<MambaBlock>(b, "mamba block");
        require(dev_params && aligned256(dev_params), "parameters must be 256-byte aligned");
        m->carve(dev_params);
    });
}
AIC_API aic_status aic_mamba_block_state_bytes(aic_mamba_block b, int batch, size_t* bytes)
{
    return guarded([&] {
        auto* m = handle<MambaBlock>(b, "mamba block");
        require(bytes && batch >= 0, "bad argument");
        *bytes = m->state_bytes(batch);
    });
}
AIC_API aic_status aic_mamba_block_bind_state(aic_mamba_block b, void* dev_state, int batch)
{
    return guarded([&] {
        auto* m = handle<MambaBlock>(b, "mamba block");
        require(batch >= 0 && (batch == 0 || (dev_state && aligned256(dev_state))), "state must be 256-byte aligned");
        m->bind_state(dev_state, batch);
    });
}
AIC_API aic_status aic_mamba_block_trace_bytes(aic_mamba_block b, int batch, size_t* bytes)
{
    return guarded([&] {
        auto* m = handle<MambaBlock>(b, "mamba block");
        require(bytes && batch >= 0, "bad argument");
        *bytes = m->trace_bytes(batch);
    });
}
AIC_API aic_status aic_mamba_block_bind_traces(aic_mamba_block b, void* dev_traces, int batch)
{
    return guarded([&] {
        auto* m = handle<MambaBlock>(b, "mamba block");
        require(!dev_traces || aligned256(dev_traces), "traces must be 256-byte aligned");
        m->bind_traces(dev_traces, batch);
    });
}
AIC_API aic_status aic_mamba_block_reset_state(aic_mamba_block b, void* stream)
{
    return guarded([&] {
        auto* m = handle<MambaBlock>(b, "mamba block");
        for (auto& l : m->layers) l->reset(as_stream(stream));
    });
}
AIC_API aic_status aic_mamba_block_workspace_bytes(aic_mamba_block b, int64_t rows, size_t* bytes)
{
    return guarded([&] {
        auto* m = handle<MambaBlock>(b, "mamba block");
        require(bytes && rows >= 0, "bad argument");
        *bytes = m->workspace(rows, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr);
    });
}
AIC_API aic_status aic_mamba_block_load_dir_sync(aic_mamba_block b, const char* dir, void* stream)
{
    return guarded([&] {
        auto* m = handle<MambaBlock>(b, "mamba block");
        static const char* names[3] = {"mamba_strategist.bin", "mamba_tactic.bin", "mamba_executor.bin"};
        for (int i = 0; i < 3; ++i) m->layers[i]->load_file(join(dir, names[i]).c_str(), as_stream(stream));
    });
}
AIC_API aic_status aic_mamba_block_forward(aic_mamba_block b, const uint32_t* in, const int8_t* in_s, float* out,
                                           int batch, int seq, int on_training, int add_seed, int is_survived,
                                           void* workspace, void* stream)
{
    return guarded([&] {
        handle<MambaBlock>(b, "mamba block")
            ->forward(in, in_s, out, batch, seq, on_training != 0, add_seed, is_survived != 0, workspace, as_stream(stream));
    });
}
AIC_API aic_status aic_mamba_block_set_mode(aic_mamba_block b, int mode)
{
    return guarded([&] {
        require(mode == AIC_MAMBA_TENSOR || mode == AIC_MAMBA_EXACT, "unknown mamba mode");
        for (auto& l : handle<MambaBlock>(b, "mamba block")->layers) l->mode = mode;
    });
}
AIC_API aic_status aic_mamba_block_destroy(aic_mamba_block b)
{
    return guarded([&] { delete reinterpret_cast<MambaBlock*>(b); });
}

// ---- Critic
AIC_API aic_status aic_critic_create(const aic_critic_desc* desc, aic_critic* out)
{
    return guarded([&] {
        require(desc && out, "null argument");
        *out = reinterpret_cast<aic_critic>(new Critic(*desc));
    });
}
AIC_API aic_status aic_critic_param_bytes(aic_critic c, size_t* bytes)
{
    return guarded([&] {
        auto* k = handle<Critic>(c, "critic");
        require(bytes != nullptr, "null output");
        Critic tmp(*k);
        *bytes = tmp.carve(nullptr);
    });
}
AIC_API aic_status aic_critic_bind(aic_critic c, void* dev_params)
{
    return guarded([&] {
        auto* k = handle<Critic>(c, "critic");
        require(dev_params && aligned256(dev_params), "parameters must be 256-byte aligned");
        k->carve(dev_params);
        k->bound = true;
    });
}
AIC_API aic_status aic_critic_load_weights(aic_critic c, const float* w1, const float* w2, const float* wl, void* stream)
{
    return guarded([&] { handle<Critic>(c, "critic")->load(w1, w2, wl, as_stream(stream)); });
}
AIC_API aic_status aic_critic_load_file_sync(aic_critic c, const char* path, void* stream)
{
    return guarded([&] { handle<Critic>(c, "critic")->load_file(path, as_stream(stream)); });
}
AIC_API aic_status aic_critic_state_bytes(aic_critic c, int batch, size_t* bytes)
{
    return guarded([&] {
        auto* k = handle<Critic>(c, "critic");
        require(bytes && batch >= 0, "bad argument");
        *bytes = k->state_bytes(batch);
    });
}
AIC_API aic_status aic_critic_bind_state(aic_critic c, void* dev_state, int batch)
{
    return guarded([&] {
        auto* k = handle<Critic>(c, "critic");
        require(batch >= 0 && (batch == 0 || (dev_state && aligned256(dev_state))), "state must be 256-byte aligned");
        k->h = static_cast<float2*>(dev_state);
        k->batch_bound = batch;
        k->traces = nullptr;  // bound again after the state
    });
}
AIC_API aic_status aic_critic_trace_bytes(aic_critic c, int batch, size_t* bytes)
{
    return guarded([&] {
        auto* k = handle<Critic>(c, "critic");
        require(bytes && batch >= 0, "bad argument");
        *bytes = k->trace_bytes(batch);
    });
}
AIC_API aic_status aic_critic_bind_traces(aic_critic c, void* dev_traces, int batch)
{
    return guarded([&] {
        auto* k = handle<Critic>(c, "critic");
        require(batch == k->batch_bound, "traces must be bound for the bound state's batch");
        require(!dev_traces || aligned256(dev_traces), "traces must be 256-byte aligned");
        k->traces = static_cast<float2*>(dev_traces);
    });
}
AIC_API aic_status aic_critic_reset_state(aic_critic c, void* stream)
{
    return guarded([&] { handle<Critic>(c, "critic")->reset(as_stream(stream)); });
}
AIC_API aic_status aic_critic_workspace_bytes(aic_critic c, int64_t rows, size_t* bytes)
{
    return guarded([&] {
        auto* k = handle<Critic>(c, "critic");
        require(bytes && rows >= 0, "bad argument");
        *bytes = k->workspace(rows, nullptr, nullptr, nullptr);
    });
}
AIC_API aic_status aic_critic_forward(aic_critic c, const uint32_t* in, const int8_t* in_s, float* score, int batch,
                                      int seq, void* workspace, void* stream)
{
    return guarded([&] { handle<Critic>(c, "critic")->forward(in, in_s, score, batch, seq, workspace, as_stream(stream)); });
}
AIC_API aic_status aic_critic_forward_pooled(aic_critic c, const uint16_t* pooled, float* score, int batch, int seq,
                                             void* workspace, void* stream)
{
    return guarded([&] {
        auto* k = handle<Critic>(c, "critic");
        k->forward_pooled(reinterpret_cast<const __half*>(pooled), score, batch, seq, workspace, as_stream(stream));
    });
}
AIC_API aic_status aic_critic_destroy(aic_critic c)
{
    return guarded([&] { delete reinterpret_cast<Critic*>(c); });
}

// ---- Cortex
AIC_API aic_status aic_cortex_create(const aic_cortex_desc* desc, aic_cortex* out)
{
    return guarded([&] {
        require(desc && out, "null argument");
        *out = reinterpret_cast<aic_cortex>(new Cortex(*desc));
    });
}
AIC_API aic_status aic_cortex_block(aic_cortex c, int i, aic_conv_block* out)
{
    return guarded([&] {
        auto* x = handle<Cortex>(c, "cortex");
        require(out && i >= 0 && i < static_cast<int>(x->blocks.size()), "block index out of range");
        *out = reinterpret_cast<aic_conv_block>(x->blocks[i].get());
    });
}
AIC_API aic_status aic_cortex_unit(aic_cortex c, int i, aic_mamba_layer* out)
{
    return guarded([&] {
        auto* x = handle<Cortex>(c, "cortex");
        require(out && i >= 0 && i < static_cast<int>(x->units.size()), "unit index out of range");
        *out = reinterpret_cast<aic_mamba_layer>(x->units[i].get());
    });
}
AIC_API aic_status aic_cortex_actor(aic_cortex c, aic_mamba_layer* out)
{
    return guarded([&] {
        auto* x = handle<Cortex>(c, "cortex");
        require(out != nullptr, "null output");
        *out = reinterpret_cast<aic_mamba_layer>(x->actor.get());
    });
}
AIC_API aic_status aic_cortex_critic(aic_cortex c, aic_critic* out)
{
    return guarded([&] {
        auto* x = handle<Cortex>(c, "cortex");
        require(out != nullptr, "null output");
        *out = reinterpret_cast<aic_critic>(x->critic.get());
    });
}
AIC_API aic_status aic_cortex_param_bytes(aic_cortex c, size_t* bytes)
{
    return guarded([&] {
        auto* x = handle<Cortex>(c, "cortex");
        require(bytes != nullptr, "null output");
        *bytes = x->carve(nullptr);
    });
}
AIC_API aic_status aic_cortex_bind(aic_cortex c, void* dev_params)
{
    return guarded([&] {
        auto* x = handle<Cortex>(c, "cortex");
        require(dev_params && aligned256(dev_params), "parameters must be 256-byte aligned");
        x->carve(dev_params);
    });
}
AIC_API aic_status aic_cortex_state_bytes(aic_cortex c, int batch, size_t* bytes)
{
    return guarded([&] {
        auto* x = handle<Cortex>(c, "cortex");
        require(bytes && batch >= 0, "bad argument");
        *bytes = x->state(batch, nullptr);
    });
}
AIC_API aic_status aic_cortex_bind_state(aic_cortex c, void* dev_state, int batch)
{
    return guarded([&] {
        auto* x = handle<Cortex>(c, "cortex");
        require(batch >= 0 && dev_state && aligned256(dev_state), "state must be 256-byte aligned");
        x->state(batch, dev_state);
    });
}
AIC_API aic_status aic_cortex_reset_state(aic_cortex c, void* stream)
{
    return guarded([&] {
        auto* x = handle<Cortex>(c, "cortex");
        for (auto& u : x->units) u->reset(as_stream(stream));
        x->actor->reset(as_stream(stream));
        if (x->critic) x->critic->reset(as_stream(stream));
    });
}
AIC_API aic_status aic_cortex_workspace_bytes(aic_cortex c, int batch, int seq, size_t* bytes)
{
    return guarded([&] {
        auto* x = handle<Cortex>(c, "cortex");
        require(bytes && batch >= 0 && seq >= 0, "bad argument");
        *bytes = x->workspace(batch, seq, nullptr, nullptr);
    });
}
AIC_API aic_status aic_cortex_forward(aic_cortex c, const uint16_t* planes, int batch, int seq, float* actor,
                                      float* critic, uint32_t* features, int8_t* features_s, void* workspace,
                                      void* stream)
{
    return guarded([&] {
        require(batch >= 0 && seq >= 0, "bad extents");
        handle<Cortex>(c, "cortex")
            ->forward(planes, batch, seq, actor, critic, features, features_s, workspace, as_stream(stream));
    });
}
AIC_API aic_status aic_cortex_host_workspace_bytes(aic_cortex c, int batch, int seq, size_t* bytes)
{
    return guarded([&] {
        auto* x = handle<Cortex>(c, "cortex");
        require(bytes && batch >= 0 && seq >= 0, "bad argument");
        *bytes = x->host_workspace(batch, seq, nullptr, nullptr, nullptr, nullptr, nullptr);
    });
}
AIC_API aic_status aic_cortex_forward_host(aic_cortex c, const uint16_t* planes_host, int batch, int seq,
                                           float* actor_host, float* critic_host, void* workspace, void* stream)
{
    return guarded([&] {
        require(batch >= 0 && seq >= 0, "bad extents");
        handle<Cortex>(c, "cortex")->forward_host(planes_host, batch, seq, actor_host, critic_host, workspace,
                                                  as_stream(stream));
    });
}
AIC_API aic_status aic_cortex_set_conv_mode(aic_cortex c, int mode)
{
    return guarded([&] {
        require(mode == AIC_CONV_ORDERED || mode == AIC_CONV_FAST || mode == AIC_CONV_SIMT, "unknown conv mode");
        auto* x = handle<Cortex>(c, "cortex");
        for (auto& b : x->blocks)
            for (auto& l : b->layers) l->mode = mode;
    });
}
AIC_API aic_status aic_cortex_set_mamba_mode(aic_cortex c, int mode)
{
    return guarded([&] {
        require(mode == AIC_MAMBA_TENSOR || mode == AIC_MAMBA_EXACT, "unknown mamba mode");
        auto* x = handle<Cortex>(c, "cortex");
        for (auto& u : x->units) u->mode = mode;
        x->actor->mode = mode;
    });
}
AIC_API aic_status aic_cortex_set_exact(aic_cortex c, int exact)
{
    const aic_status st = aic_cortex_set_conv_mode(c, exact ? AIC_CONV_SIMT : AIC_CONV_ORDERED);
    return st != AIC_OK ? st : aic_cortex_set_mamba_mode(c, exact ? AIC_MAMBA_EXACT : AIC_MAMBA_TENSOR);
}
AIC_API aic_status aic_cortex_profile_enable(aic_cortex c, int enable)
{
    return guarded([&] { handle<Cortex>(c, "cortex")->prof.enabled = enable != 0; });
}
AIC_API aic_status aic_cortex_profile_count(aic_cortex c, int* sites)
{
    return guarded([&] {
        auto* x = handle<Cortex>(c, "cortex");
        require(sites != nullptr, "null output");
        x->prof.collect();
        *sites = static_cast<int>(x->prof.sites.size());
    });
}
AIC_API aic_status aic_cortex_profile_get(aic_cortex c, int site, char name[32], double* total_ms, int64_t* launches,
                                          double* flops_per_launch, double* bytes_per_launch)
{
    return guarded([&] {
        auto* x = handle<Cortex>(c, "cortex");
        x->prof.collect();
        require(site >= 0 && site < static_cast<int>(x->prof.sites.size()), "site index out of range");
        const auto& s = x->prof.sites[site];
        if (name) {
            std::strncpy(name, s.name.c_str(), 31);
            name[31] = '\0';
        }
        if (total_ms) *total_ms = s.ms;
        if (launches) *launches = s.launches;
        const double n = s.launches > 0 ? static_cast<double>(s.launches) : 1.0;
        if (flops_per_launch) *flops_per_launch = s.flops / n;
        if (bytes_per_launch) *bytes_per_launch = s.bytes / n;
    });
}
AIC_API aic_status aic_cortex_profile_reset(aic_cortex c)
{
    return guarded([&] { handle<Cortex>(c, "cortex")->prof.reset(); });
}
AIC_API aic_status aic_cortex_last_launches(aic_cortex c, int64_t* launches)
{
    return guarded([&] {
        auto* x = handle<Cortex>(c, "cortex");
        require(launches != nullptr, "null output");
        *launches = x->last_launches;
    });
}
AIC_API aic_status aic_cortex_destroy(aic_cortex c)
{
    return guarded([&] { delete reinterpret_cast<Cortex*>(c); });
}

// ---------------------------------------------------------------- training (F4)
AIC_API aic_status aic_grad_clip_factor(const float* grad, int64_t n, float* partial, float* factor, void* stream)
{
    return guarded([&] {
        require(grad && partial && factor && n > 0, "bad clip arguments");
        cuda_ok(launch_clip_factor(grad, n, device_sms(), partial, factor, as_stream(stream)), "clip factor");
    });
}
AIC_API aic_status aic_grad_clip_partials(int64_t n, int64_t* floats)
{
    return guarded([&] {
        require(floats && n > 0, "bad arguments");
        *floats = sumsq_blocks(n, device_sms());
    });
}
AIC_API aic_status aic_sgd_update(float* data, const float* grad, int64_t n, const float* factor, float lr,
                                  float penalty, void* stream)
{
    return guarded([&] {
        require(data && grad && factor && n >= 0, "bad update arguments");
        cuda_ok(launch_sgd_update(data, grad, n, factor, lr, penalty, as_stream(stream)), "sgd update");
    });
}
AIC_API aic_status aic_residual_backward(float* grad_next, float* grad_res, int64_t n, float survival_prob_inv,
                                         float residual_factor, void* stream)
{
    return guarded([&] {
        require(n >= 0 && (n == 0 || (grad_next && grad_res)), "bad residual arguments");
        cuda_ok(launch_residual_backward(grad_next, grad_res, n, survival_prob_inv, residual_factor, as_stream(stream)),
                "residual backward");
    });
}
AIC_API aic_status aic_conv_layer_train_bytes(aic_conv_layer l, size_t* bytes)
{
    return guarded([&] {
        require(bytes != nullptr, "null output");
        *bytes = handle<ConvLayer>(l, "conv layer")->train_bytes();
    });
}
AIC_API aic_status aic_conv_layer_train_bind(aic_conv_layer l, void* buffer, const float* master, float learning_rate,
                                             float penalty, void* stream)
{
    return guarded([&] { handle<ConvLayer>(l, "conv layer")->train_bind(buffer, master, learning_rate, penalty, as_stream(stream)); });
}
AIC_API aic_status aic_conv_layer_backward(aic_conv_layer l, const float* grad_out, const uint32_t* in,
                                           const int8_t* in_s, float* grad_in, void* stream)
{
    return guarded([&] { handle<ConvLayer>(l, "conv layer")->backward(grad_out, in, in_s, grad_in, as_stream(stream)); });
}
AIC_API aic_status aic_conv_layer_train_views(aic_conv_layer l, float** master, float** grad_w, float** grad_b,
                                              float** bias)
{
    return guarded([&] {
        auto* c = handle<ConvLayer>(l, "conv layer");
        if (!c->train.bound) fail(AIC_ERR_STATE, "conv layer training state not bound");
        if (master) *master = c->train.master;
        if (grad_w) *grad_w = c->train.gw;
        if (grad_b) *grad_b = c->train.gb;
        if (bias) *bias = c->bias;
    });
}
AIC_API aic_status aic_mamba_layer_train_bytes(aic_mamba_layer l, size_t* bytes)
{
    return guarded([&] {
        require(bytes != nullptr, "null output");
        *bytes = handle<MambaLayer>(l, "mamba layer")->train_bytes();
    });
}
AIC_API aic_status aic_mamba_layer_train_bind(aic_mamba_layer l, void* buffer, const float* master,
                                              float learning_rate, float penalty, void* stream)
{
    return guarded([&] { handle<MambaLayer>(l, "mamba layer")->train_bind(buffer, master, learning_rate, penalty, as_stream(stream)); });
}
AIC_API aic_status aic_mamba_layer_backward(aic_mamba_layer l, const float* grad_out, const uint32_t* in,
                                            const int8_t* in_s, float* grad_in, void* stream)
{
    return guarded([&] { handle<MambaLayer>(l, "mamba layer")->backward(grad_out, in, in_s, grad_in, as_stream(stream)); });
}
AIC_API aic_status aic_mamba_layer_train_views(aic_mamba_layer l, float** master, float** grad_w, float** grad_b,
                                               float** bias)
{
    return guarded([&] {
        auto* m = handle<MambaLayer>(l, "mamba layer");
        if (!m->train.bound) fail(AIC_ERR_STATE, "mamba layer training state not bound");
        if (master) *master = m->train.master;
        if (grad_w) *grad_w = m->train.gw;
        if (grad_b) *grad_b = m->train.gb;
        if (bias) *bias = m->bias;
    });
}
AIC_API aic_status aic_critic_train_bytes(aic_critic c, size_t* bytes)
{
    return guarded([&] {
        require(bytes != nullptr, "null output");
        *bytes = handle<Critic>(c, "critic")->train_bytes();
    });
}
AIC_API aic_status aic_critic_train_bind(aic_critic c, void* buffer, float learning_rate, float penalty)
{
    return guarded([&] { handle<Critic>(c, "critic")->train_bind(buffer, learning_rate, penalty); });
}
AIC_API aic_status aic_critic_backward(aic_critic c, const float* pred_score, float real_score, void* stream)
{
    return guarded([&] { handle<Critic>(c, "critic")->backward(pred_score, real_score, as_stream(stream)); });
}
AIC_API aic_status aic_critic_train_views(aic_critic c, float** grad_w1, float** grad_w2, float** grad_lambda)
{
    return guarded([&] {
        auto* k = handle<Critic>(c, "critic");
        if (!k->train.bound) fail(AIC_ERR_STATE, "critic training state not bound");
        if (grad_w1) *grad_w1 = k->train.gw;
        if (grad_w2) *grad_w2 = k->train.gb;
        if (grad_lambda) *grad_lambda = k->train.gx;
    });
}

}  // extern "C"
