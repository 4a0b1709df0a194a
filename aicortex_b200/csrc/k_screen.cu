// Screen front-end (AICortex cs.cu:5-45, ProcessBgraToRgbOP and
// AugmentBrightnessContrastOP): a BGRA8 frame -> four fp16 planes
// (byte / 255 in the byte order B, G, R, A), and in training mode the
// reference's per-pixel dropout (with probability 50/10000 the three colour
// bytes become 0, with the next 50/10000 they become 255, chosen by the
// xorshift hash of frame_seed ^ pixel) followed by the brightness/contrast
// augmentation clamp(fma(v - 1/2, contrast, 1/2 + brightness), 0, 1) in fp16
// arithmetic on all four planes. Both steps run in one pass: a thread owns two
// horizontally adjacent pixels, reads 8 bytes and writes one half2 per plane,
// which is exactly the half2 lane pair the reference's augmentation reads.
#include <cuda_fp16.h>

#include "aic_common.cuh"
#include "aic_kernels.h"

namespace aic {
namespace {

// kernels.h:38-45: xorshift32, then the top 32 bits of x * n
__device__ __forceinline__ uint32_t bounded_hash(uint32_t seed, uint32_t n)
{
    seed ^= seed << 13;
    seed ^= seed >> 17;
    seed ^= seed << 5;
    return static_cast<uint32_t>((static_cast<uint64_t>(seed) * n) >> 32);
}

template <bool TRAIN>
__global__ void screen_kernel(const uchar4* __restrict__ bgra, __half* __restrict__ planes, int pairs, int plane_size,
                              uint32_t frame_seed, __half2 brightness, __half2 contrast)
{
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= pairs) return;
    const int idx = 2 * t;
    uchar4 px[2] = {__ldg(bgra + idx), __ldg(bgra + idx + 1)};
    if (TRAIN) {
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const uint32_t r = bounded_hash(frame_seed ^ static_cast<uint32_t>(idx + k), 10000u);
            if (r < 50u) px[k] = make_uchar4(0, 0, 0, px[k].w);
            else if (r < 100u) px[k] = make_uchar4(255, 255, 255, px[k].w);
        }
    }
    const unsigned char b[2][4] = {{px[0].x, px[0].y, px[0].z, px[0].w}, {px[1].x, px[1].y, px[1].z, px[1].w}};
    const __half2 h_half = __float2half2_rn(0.5f);
    const __half2 offset = __hadd2(h_half, brightness);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        __half2 v = __halves2half2(__float2half(b[0][c] * (1.0f / 255.0f)), __float2half(b[1][c] * (1.0f / 255.0f)));
        if (TRAIN) v = __hmax2(__hmin2(__hfma2(__hsub2(v, h_half), contrast, offset), __float2half2_rn(1.0f)),
                               __float2half2_rn(0.0f));
        *reinterpret_cast<__half2*>(planes + static_cast<int64_t>(c) * plane_size + idx) = v;
    }
}

}  // namespace

cudaError_t launch_screen_frontend(const uint8_t* bgra, __half* frame, int dim, int first_channel, bool train,
                                   uint32_t frame_seed, float brightness, float contrast, cudaStream_t stream)
{
    const int plane = dim * dim;
    const int pairs = plane / 2;
    if (pairs == 0) return cudaSuccess;
    const __half2 b = __float2half2_rn(brightness), c = __float2half2_rn(contrast);
    __half* out = frame + static_cast<int64_t>(first_channel) * plane;
    const unsigned grid = static_cast<unsigned>((pairs + 255) / 256);
    const uchar4* px = reinterpret_cast<const uchar4*>(bgra);
    if (train) screen_kernel<true><<<grid, 256, 0, stream>>>(px, out, pairs, plane, frame_seed, b, c);
    else screen_kernel<false><<<grid, 256, 0, stream>>>(px, out, pairs, plane, frame_seed, b, c);
    return cudaGetLastError();
}

}  // namespace aic
