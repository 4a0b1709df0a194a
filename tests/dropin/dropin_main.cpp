// Test driver of the drop-in layer classes (include/aicortex_layers.hpp): it
// uses them the way the reference's Cortex does (cortex.h:600-720, 281-303):
// the constructors add up arena bytes, the arenas are allocated once (device,
// pinned host, ping-pong buffers), initData carves them and loads the
// reference-format checkpoint trees, and forward runs one environment step per
// call with the state carried between calls.
//
//   dropin_main <dir>
//
// <dir>/spec.txt (written by tests/test_dropin_gpu.py):
//   conv in mid out stride din dout k residual_factor
//   mamba steps out activation
//   critic in units dim steps
// Inputs <dir>/{conv,mamba,critic}_in_{w,s}.bin, checkpoints <dir>/conv_block/,
// <dir>/mamba_block/, <dir>/critic.bin; outputs <dir>/*_out*.bin.
//
// With <dir>/train_spec.txt it also trains one ConvLayer frame and one
// MambaLayer step through the classes' backward (conv_layer.h:150,
// mamba_layer.h:146) in training mode (is_in_inference = false):
//   convtrain in out k stride din dout act lr penalty
//   mambatrain steps out activation lr penalty
// Inputs train_conv.bin / train_mamba.bin (checkpoints), train_conv_in_{w,s},
// train_conv_gout, train_mamba_in_{w,s}, train_mamba_gout; outputs
// train_{conv,mamba}_gin.bin and the host masters train_{conv,mamba}_master.bin.
#include <cstdio>
#include <fstream>
#include <iostream>
#include <iterator>
#include <string>
#include <vector>

#include "aicortex_layers.hpp"

namespace {

std::vector<char> read_file(const std::string& path)
{
    std::ifstream f(path, std::ios::binary);
    if (!f) throw std::runtime_error("cannot read " + path);
    return std::vector<char>((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
}

void write_file(const std::string& path, const void* p, size_t n)
{
    std::ofstream f(path, std::ios::binary);
    f.write(static_cast<const char*>(p), static_cast<std::streamsize>(n));
}

template <class T>
T* to_device(const std::vector<char>& v)
{
    void* p = nullptr;
    aic_dropin::check_cuda(cudaMalloc(&p, v.size()));
    aic_dropin::check_cuda(cudaMemcpy(p, v.data(), v.size(), cudaMemcpyHostToDevice));
    return static_cast<T*>(p);
}

struct Arenas {
    uint8_t *dev = nullptr, *host = nullptr, *buf_a = nullptr, *buf_a_s = nullptr, *buf_b = nullptr, *buf_b_s = nullptr;
    uint8_t *side = nullptr, *side_w = nullptr, *side_b = nullptr, *grad_a = nullptr, *grad_b = nullptr, *grad_r = nullptr;
    void alloc(size_t dev_bytes, size_t host_bytes, int pipo_groups)
    {
        aic_dropin::check_cuda(cudaMalloc(&dev, dev_bytes));
        aic_dropin::check_cuda(cudaMallocHost(&host, host_bytes + 16));
        aic_dropin::check_cuda(cudaMalloc(&buf_a, static_cast<size_t>(pipo_groups) * 16));
        aic_dropin::check_cuda(cudaMalloc(&buf_a_s, static_cast<size_t>(pipo_groups)));
        aic_dropin::check_cuda(cudaMalloc(&buf_b, static_cast<size_t>(pipo_groups) * 16));
        aic_dropin::check_cuda(cudaMalloc(&buf_b_s, static_cast<size_t>(pipo_groups)));
    }
};

}  // namespace

int main(int argc, char** argv)
{
    if (argc != 2) {
        std::cerr << "usage: dropin_main <dir>\n";
        return 2;
    }
    const std::string dir = argv[1];
    try {
        std::ifstream spec(dir + "/spec.txt");
        std::string tag;
        int cin, mid, cout_, stride, din, dout, kdw, steps, mout, mact, c_in, c_units, c_dim, c_steps;
        float rf;
        spec >> tag >> cin >> mid >> cout_ >> stride >> din >> dout >> kdw >> rf;
        spec >> tag >> steps >> mout >> mact;
        spec >> tag >> c_in >> c_units >> c_dim >> c_steps;
        if (!spec) throw std::runtime_error("bad spec.txt");
        cudaStream_t stream = nullptr;
        aic_dropin::check_cuda(cudaStreamCreate(&stream));

        // two-phase construction: the constructors count, then one allocation per arena
        int grad_w = 0, grad_b = 0, pipo_db = 0, pipo_groups = 0;
        size_t dev_bytes = 0, host_bytes = 0, learn = 0, learn_cnt = 0, critic_bytes = 0;
        ConvBlock conv(cin, mid, cout_, stride, din, dout, stream, &grad_w, &grad_b, &pipo_db, &pipo_groups, kdw, 1.0f, rf,
                       stream, 0.0f, 0.0f, &dev_bytes, &host_bytes, &learn, &learn_cnt);
        MambaBlock mamba(MambaBlock::d_model, mout, stream, &grad_w, &grad_b, 1.0f, 1.0f, stream, 0.0f, 0.0f, &dev_bytes,
                         &host_bytes, &learn, &learn_cnt, mact);
        Critic critic(c_in, 2 * c_units, c_dim, stream, &grad_w, &grad_b, stream, 0.0f, 0.0f, &critic_bytes);
        Arenas ar;
        ar.alloc(dev_bytes + critic_bytes + 16, host_bytes, pipo_groups);
        uint8_t* dev = ar.dev;
        uint8_t* host = ar.host;
        float** meta_data = nullptr;
        size_t* meta_offsets = nullptr;
        conv.initData(true, dir + "/conv_block", dev, host, ar.side_w, ar.side_b, true, meta_data, meta_offsets,
                      ar.grad_a, ar.grad_b, ar.grad_r, ar.buf_a, ar.buf_a_s, ar.buf_b, ar.buf_b_s, grad_w, grad_b);
        mamba.initData(true, dir + "/mamba_block", dev, host, ar.side, ar.side_w, ar.side_b, true, meta_data,
                       meta_offsets, ar.grad_a, ar.grad_r, ar.buf_a, ar.buf_a_s, ar.buf_b, ar.buf_b_s, pipo_groups, grad_w,
                       grad_b);
        critic.initData(true, dir + "/critic.bin", dev, ar.side_w, ar.side_b, grad_w, grad_b);
        if (dev > ar.dev + dev_bytes + critic_bytes + 16 || host > ar.host + host_bytes + 16)
            throw std::runtime_error("initData carved past the counted arena");

        // ConvBlock: one frame
        {
            auto* in_w = to_device<uint32_t>(read_file(dir + "/conv_in_w.bin"));
            auto* in_s = to_device<int8_t>(read_file(dir + "/conv_in_s.bin"));
            const size_t pos = static_cast<size_t>(dout) * dout, groups = pos * cout_ / 32;
            uint32_t* out_w;
            int8_t* out_s;
            aic_dropin::check_cuda(cudaMalloc(&out_w, groups * 16));
            aic_dropin::check_cuda(cudaMalloc(&out_s, groups));
            conv.forward(in_w, in_s, out_w, out_s, false, true);
            std::vector<uint32_t> hw(groups * 4);
            std::vector<int8_t> hs(groups);
            aic_dropin::check_cuda(cudaMemcpy(hw.data(), out_w, groups * 16, cudaMemcpyDeviceToHost));
            aic_dropin::check_cuda(cudaMemcpy(hs.data(), out_s, groups, cudaMemcpyDeviceToHost));
            write_file(dir + "/conv_out_w.bin", hw.data(), hw.size() * 4);
            write_file(dir + "/conv_out_s.bin", hs.data(), hs.size());
        }
        // MambaBlock: `steps` successive calls, one row each, state carried
        {
            auto* in_w = to_device<uint32_t>(read_file(dir + "/mamba_in_w.bin"));
            auto* in_s = to_device<int8_t>(read_file(dir + "/mamba_in_s.bin"));
            const int D = MambaBlock::d_model;
            std::vector<float> out(static_cast<size_t>(steps) * mout);
            for (int t = 0; t < steps; ++t) {
                mamba.forward(in_w + static_cast<size_t>(t) * D / 8, in_s + static_cast<size_t>(t) * D / 32, false, 0,
                              true);
                if (mamba.get_output().size() != static_cast<size_t>(mout)) throw std::runtime_error("output size");
                aic_dropin::check_cuda(cudaMemcpyAsync(out.data() + static_cast<size_t>(t) * mout,
                                                       mamba.get_output().data(), mout * sizeof(float),
                                                       cudaMemcpyDeviceToHost, stream));
            }
            aic_dropin::check_cuda(cudaStreamSynchronize(stream));
            write_file(dir + "/mamba_out.bin", out.data(), out.size() * 4);
        }
        // Critic: `c_steps` successive calls on F input frames of c_dim x c_dim pixels
        {
            auto* in_w = to_device<uint32_t>(read_file(dir + "/critic_in_w.bin"));
            auto* in_s = to_device<int8_t>(read_file(dir + "/critic_in_s.bin"));
            const size_t frame = static_cast<size_t>(c_dim) * c_dim * c_in;
            std::vector<float> scores(c_steps);
            for (int t = 0; t < c_steps; ++t) {
                critic.forward(in_w + t * frame / 8, in_s + t * frame / 32);
                scores[t] = critic.get_score_output();
            }
            write_file(dir + "/critic_out.bin", scores.data(), scores.size() * 4);
        }
        std::ifstream tspec(dir + "/train_spec.txt");
        if (tspec) {
            int tci, tco, tk, tst, tdi, tdo, tact, msteps, mo, ma;
            float clr, cpen, mlr, mpen;
            tspec >> tag >> tci >> tco >> tk >> tst >> tdi >> tdo >> tact >> clr >> cpen;
            tspec >> tag >> msteps >> mo >> ma >> mlr >> mpen;
            if (!tspec) throw std::runtime_error("bad train_spec.txt");
            int gw = 0, gb = 0;
            size_t tdev = 0, thost = 0;
            ConvLayer layer(tci, tco, tk, tst, tdi, tdo, stream, &gw, &gb, stream, clr, cpen, &tdev, &thost, nullptr,
                            nullptr, tact == 0);
            MambaLayer ml(mo, stream, &gw, &gb, stream, mlr, mpen, &tdev, &thost, nullptr, nullptr, ma);
            uint8_t *tdev_base = nullptr, *thost_base = nullptr, *side = nullptr;
            aic_dropin::check_cuda(cudaMalloc(&tdev_base, tdev + 16));
            aic_dropin::check_cuda(cudaMallocHost(&thost_base, thost + 16));
            aic_dropin::check_cuda(cudaMalloc(&side, 64u << 20));  // traces (side arena)
            uint8_t *d = tdev_base, *h = thost_base, *sd = side, *unused = nullptr;
            float** no_data = nullptr;
            size_t* no_offsets = nullptr;
            layer.initData(true, dir + "/train_conv.bin", d, h, unused, unused, false, &no_data, &no_offsets, gw, gb);
            ml.initData(true, dir + "/train_mamba.bin", d, h, sd, unused, unused, false, &no_data, &no_offsets, gw, gb);
            if (d > tdev_base + tdev + 16 || h > thost_base + thost + 16)
                throw std::runtime_error("initData carved past the counted training arena");
            // the conv layer: one frame, grad_in accumulated into zeros
            auto* cin_w = to_device<uint32_t>(read_file(dir + "/train_conv_in_w.bin"));
            auto* cin_s = to_device<int8_t>(read_file(dir + "/train_conv_in_s.bin"));
            auto* cgout = to_device<float>(read_file(dir + "/train_conv_gout.bin"));
            const size_t n_in = static_cast<size_t>(tdi) * tdi * tci;
            float* cgin = nullptr;
            aic_dropin::check_cuda(cudaMalloc(&cgin, n_in * sizeof(float)));
            aic_dropin::check_cuda(cudaMemset(cgin, 0, n_in * sizeof(float)));
            layer.backward(cgout, cin_w, cin_s, cgin);
            aic_dropin::check_cuda(cudaStreamSynchronize(stream));
            std::vector<float> hg(n_in);
            aic_dropin::check_cuda(cudaMemcpy(hg.data(), cgin, n_in * sizeof(float), cudaMemcpyDeviceToHost));
            write_file(dir + "/train_conv_gin.bin", hg.data(), hg.size() * 4);
            const size_t n_cw = static_cast<size_t>(tco) * tk * tk * tci;
            write_file(dir + "/train_conv_master.bin", thost_base, n_cw * sizeof(float));
            // the Mamba layer: `msteps` training-mode steps, then the last step's backward
            auto* min_w = to_device<uint32_t>(read_file(dir + "/train_mamba_in_w.bin"));
            auto* min_s = to_device<int8_t>(read_file(dir + "/train_mamba_in_s.bin"));
            auto* mgout = to_device<float>(read_file(dir + "/train_mamba_gout.bin"));
            const int D = MambaLayer::d_model;
            for (int t = 0; t < msteps; ++t)
                ml.forward(min_w + static_cast<size_t>(t) * D / 8, min_s + static_cast<size_t>(t) * D / 32);
            aic_dropin::DeviceSpan<float> mgin;
            aic_dropin::check_cuda(cudaMalloc(&mgin.ptr, D * sizeof(float)));
            mgin.count = D;
            ml.backward(mgout, min_w + static_cast<size_t>(msteps - 1) * D / 8,
                        min_s + static_cast<size_t>(msteps - 1) * D / 32, mgin);
            aic_dropin::check_cuda(cudaStreamSynchronize(stream));
            std::vector<float> hm(D);
            aic_dropin::check_cuda(cudaMemcpy(hm.data(), mgin.ptr, D * sizeof(float), cudaMemcpyDeviceToHost));
            write_file(dir + "/train_mamba_gin.bin", hm.data(), hm.size() * 4);
            const size_t n_mw = static_cast<size_t>(2 * D) * (34 + 4 * MambaLayer::d_state + mo);
            write_file(dir + "/train_mamba_master.bin", thost_base + ((n_cw * sizeof(float) + 15) & ~size_t(15)),
                       n_mw * sizeof(float));
        }
        int code = -1;
        aic_dropin::check(aic_device_error_sync(&code));
        if (code != 0) throw std::runtime_error("device error word " + std::to_string(code));
        std::printf("dropin ok: device arena %zu bytes, host arena %zu bytes, ping-pong groups %d\n",
                    dev_bytes + critic_bytes, host_bytes, pipo_groups);
    } catch (const std::exception& e) {
        std::cerr << "dropin failed: " << e.what() << "\n";
        return 1;
    }
    return 0;
}
