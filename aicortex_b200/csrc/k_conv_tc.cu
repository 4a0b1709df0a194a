// Quantized conv (pointwise k=1, dense k=2/4 with stride k) as an implicit
// GEMM on the 5th-generation tensor cores (tcgen05.mma, accumulator in TMEM),
// with the RMSNorm(256-chunk) + bias (+SiLU) + int4 requant epilogue fused.
//
// Numerics. A packed int4 code q with exponent s stands for q * max(2^s/7,
// 2^-13) (AICortex kernels.h:69). Both operands are staged in shared memory as
// bf16 values q * F(s), F(s) = 2^s for s >= -10 and 7 * 2^-13 below (where the
// reference's dequantisation clamps), which bf16 represents exactly (|q*7| <
// 2^6). Every product is therefore exact, the tensor core accumulates in fp32,
// and the epilogue multiplies by fl(1/7)^2. The result equals the reference's
// sum over groups of unit(s_in) * unit(s_w) * dot up to fp32 summation order.
//
// Structure of one CTA (256 threads, one 128-pixel x up-to-256-channel tile):
//   - for each 64-wide K stage, thread t converts group (t >> 7) of pixel row
//     (t & 127) of the A tile from the packed activations (im2col on the fly
//     for the dense convs) into a 128B-swizzled K-major bf16 tile;
//   - the B tile (weights) is a pre-swizzled bf16 image built at weight-load
//     time, fetched per stage with one cp.async.bulk into the same layout;
//   - thread 0 issues four tcgen05.mma (M128 x N x K16) per stage and commits
//     to the stage's mbarrier; stages are double-buffered;
//   - after the last stage warp w reads TMEM lanes 32*(w&3).. (its 32 pixel
//     rows) with tcgen05.ld; the two warpgroups take alternate 32-channel
//     groups, exchange the rows' sums of squares once through shared memory,
//     and each thread normalises, activates and packs whole 32-channel groups
//     of its own row, so the requant needs no cross-thread reduction.
// Shared memory is sized per launch (1-2 stages, B tile of the layer's width)
// so 2-4 CTAs share an SM, never more than its 512 TMEM columns can hold.
// All mbarrier waits are bounded; on timeout the kernel records an error code
// in *err, skips the remaining work, waits (bounded) for its own outstanding
// operations and releases its TMEM before returning.
#include <cuda_bf16.h>

#include "aic_common.cuh"
#include "aic_kernels.h"
#include "tc_ptx.cuh"

namespace aic {
namespace {

using namespace tc;

constexpr int kBK = 64;           // K elements per stage (128 bytes of bf16)
constexpr int kStages = 2;        // smem pipeline depth
constexpr int kThreads = 256;
constexpr int kTileA = kBM * kBK * 2;          // 16 KB
constexpr int kMaxN = 256;
constexpr int kTileBMax = kMaxN * kBK * 2;     // 32 KB

struct TcParams {
    const uint32_t* in;
    const int8_t* in_s;
    const uint8_t* wimg;
    const float* bias;
    uint32_t* out;
    int8_t* out_s;
    int64_t rows;
    int in_c, out_c, ksize, din, dout, stages, act;
    int smem_stages, n_max;
    int* err;
};

__global__ void __launch_bounds__(kThreads, 4) conv_gemm_tc_kernel(TcParams p)
{
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte aligned tiles (swizzle atoms), then bias, row partial sums, barriers.
    uint8_t* base = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);  // stays a shared-space pointer
    const int nst = p.smem_stages;
    const int n0 = blockIdx.y * kMaxN;
    const int n_cta = min(kMaxN, p.out_c - n0);
    const int tile_b = n_cta * kBK * 2;
    const int tile_b_max = p.n_max * kBK * 2;
    uint8_t* a_tiles = base;
    uint8_t* b_tiles = base + nst * kTileA;
    float* bias_s = reinterpret_cast<float*>(b_tiles + nst * tile_b_max);
    float* part = bias_s + kMaxN;  // [2][kBM] partial sums of squares
    uint64_t* bars = reinterpret_cast<uint64_t*>(part + 2 * kBM);
    // bars[0..nst): B full, bars[nst..2nst): stage free, bars[2nst]: accumulator ready
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * nst + 1);
    int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t tmem_cols = n_cta <= 32 ? 32u : n_cta <= 64 ? 64u : n_cta <= 128 ? 128u : 256u;
    if (tid < n_cta) bias_s[tid] = p.bias[n0 + tid];
    if (tid == 0) {
        for (int i = 0; i < 2 * nst + 1; ++i) mbar_init(smem_addr(&bars[i]), 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) tmem_alloc(smem_addr(tmem_slot), tmem_cols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    const int64_t m0 = static_cast<int64_t>(blockIdx.x) * kBM;
    // producer role: one (row, group-of-stage) per thread
    const int prow = tid & (kBM - 1), pg = tid >> 7;
    const int64_t prow_g = m0 + prow;
    const bool prow_ok = prow_g < p.rows;
    const int G = p.in_c >> 5;
    const int GK = G * p.ksize * p.ksize;
    const uint8_t* wimg = p.wimg + (static_cast<int64_t>(n0) * p.stages * kBK * 2);
    const uint32_t idesc = instr_desc(n_cta);

    for (int s = 0; s < p.stages; ++s) {
        const int buf = s % nst;
        const uint32_t use = static_cast<uint32_t>(s / nst);
        uint8_t* a_tile = a_tiles + buf * kTileA;
        uint8_t* b_tile = b_tiles + buf * tile_b_max;
        if (use > 0 && !*abort_flag) {
            if (!mbar_wait(smem_addr(&bars[nst + buf]), (use - 1) & 1u, p.err, 1)) *abort_flag = 1;
        }
        __syncthreads();
        if (*abort_flag) break;
        if (tid == 0) {
            mbar_expect_tx(smem_addr(&bars[buf]), static_cast<uint32_t>(tile_b));
            bulk_g2s(smem_addr(b_tile), wimg + static_cast<int64_t>(s) * tile_b, static_cast<uint32_t>(tile_b),
                     smem_addr(&bars[buf]));
        }
        const int gk = 2 * s + pg;
        if (prow_ok && gk < GK) {
            const int tap = gk / G, g = gk - tap * G;
            const int64_t pix = tap_pixel(prow_g, tap, p.ksize, p.din, p.dout);
            const uint4 words = __ldg(reinterpret_cast<const uint4*>(p.in) + pix * G + g);
            stage_group(a_tile, prow, pg, words, __ldg(p.in_s + pix * G + g));
        } else {
            stage_zero(a_tile, prow, pg);
        }
        fence_async_smem();
        __syncthreads();
        if (tid == 0) {
            if (mbar_wait(smem_addr(&bars[buf]), use & 1u, p.err, 2)) {
                tc_fence_after();
                const uint32_t a_addr = smem_addr(a_tile), b_addr = smem_addr(b_tile);
#pragma unroll
                for (int j = 0; j < kBK / 16; ++j)
                    mma_f16(tmem, smem_desc(a_addr + 32 * j), smem_desc(b_addr + 32 * j), idesc,
                             (s > 0 || j > 0) ? 1u : 0u);
                mma_commit(smem_addr(&bars[nst + buf]));
            } else {
                *abort_flag = 1;
            }
        }
    }
    if (tid == 0) mma_commit(smem_addr(&bars[2 * nst]));
    const bool acc_ok = mbar_wait(smem_addr(&bars[2 * nst]), 0u, p.err, 3);
    tc_fence_after();

    // Epilogue: warp w reads TMEM lanes 32*(w&3).. (its pixel rows); the two
    // warpgroups take alternate 32-channel groups and share the row's sum of
    // squares through shared memory.
    const int q = warp & 3, half = warp >> 2;
    const int erow = q * 32 + lane;
    const int64_t row = m0 + erow;
    const bool ok = acc_ok && !*abort_flag;
    const uint32_t taddr = tmem + (static_cast<uint32_t>(q * 32) << 16);
    const int ngroups = n_cta >> 5;
    float ss = 0.0f;
    if (ok) {
        for (int g = half; g < ngroups; g += 2) {
            float v[32];
            tmem_ld32(taddr + 32 * g, v);
#pragma unroll
            for (int i = 0; i < 32; ++i) ss = fmaf(v[i], v[i], ss);
        }
    }
    part[half * kBM + erow] = ss;
    asm volatile("bar.sync 1, %0;" ::"n"(kThreads) : "memory");
    if (ok) {
        const float inv49 = (1.0f / kQMax) * (1.0f / kQMax);
        const float inv_div = __frcp_rn(static_cast<float>(min(p.out_c, kNormChunk)));
        const float total = (part[erow] + part[kBM + erow]) * (inv49 * inv49);
        const float sc = inv49 * __frsqrt_rn(fmaf(total, inv_div, kEps));
        const int groups_out = p.out_c >> 5;
        for (int g = half; g < ngroups; g += 2) {
            float v[32];
            tmem_ld32(taddr + 32 * g, v);
            const float4* b4 = reinterpret_cast<const float4*>(bias_s + 32 * g);
#pragma unroll
            for (int i4 = 0; i4 < 8; ++i4) {
                const float4 b = b4[i4];
                const float bb[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const float x = fmaf(v[4 * i4 + k], sc, bb[k]);
                    v[4 * i4 + k] = p.act ? __fdividef(x, 1.0f + __expf(-x)) : x;
                }
            }
            uint4 words;
            int8_t e;
            quantize_group(v, &words, &e);
            if (row < p.rows) {
                const int64_t gi = row * groups_out + (n0 >> 5) + g;
                reinterpret_cast<uint4*>(p.out)[gi] = words;
                p.out_s[gi] = e;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, tmem_cols);
}

// Builds the per-(chunk, stage) swizzled bf16 images of the weights from the
// packed int4 rows [out_c][ksize^2 * in_c]. One thread per (out channel,
// 32-element group slot of the padded K).
__global__ void build_wimg_kernel(const uint32_t* __restrict__ w, const int8_t* __restrict__ w_s, int out_c, int gk_total,
                                  int stages, uint8_t* __restrict__ img)
{
    const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int slots = 2 * stages;
    if (t >= static_cast<int64_t>(out_c) * slots) return;
    const int n = static_cast<int>(t / slots);
    const int gk = static_cast<int>(t % slots);
    const int chunk = n / kMaxN, nl = n % kMaxN;
    const int n_chunk = min(kMaxN, out_c - chunk * kMaxN);
    const int s = gk >> 1, gl = gk & 1;
    uint8_t* tile = img + (static_cast<int64_t>(chunk) * kMaxN * stages + static_cast<int64_t>(s) * n_chunk) * kBK * 2;
    if (gk < gk_total) {
        const int64_t gi = static_cast<int64_t>(n) * gk_total + gk;
        stage_group(tile, nl, gl, reinterpret_cast<const uint4*>(w)[gi], w_s[gi]);
    } else {
        stage_zero(tile, nl, gl);
    }
}

__device__ int g_device_error;

}  // namespace

// Address of the device error word of the current device (looked up per
// call: the symbol has one instance per device).
int* device_error_word()
{
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
    return static_cast<int*>(p);
}

size_t conv_tc_wimg_bytes(int in_c, int out_c, int ksize)
{
    const int gk_total = (in_c >> 5) * ksize * ksize;
    const int stages = (gk_total + 1) / 2;
    return static_cast<size_t>(out_c) * stages * kBK * 2;
}

cudaError_t launch_build_wimg(const uint32_t* w, const int8_t* w_s, int in_c, int out_c, int ksize, uint8_t* img,
                              cudaStream_t stream)
{
    const int gk_total = (in_c >> 5) * ksize * ksize;
    const int stages = (gk_total + 1) / 2;
    const int64_t n = static_cast<int64_t>(out_c) * 2 * stages;
    build_wimg_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, stream>>>(w, w_s, out_c, gk_total, stages, img);
    return cudaGetLastError();
}

cudaError_t launch_conv_gemm_tc(const uint32_t* in, const int8_t* in_s, const uint8_t* wimg, const float* bias,
                                uint32_t* out, int8_t* out_s, int64_t frames, int in_c, int out_c, int ksize, int din,
                                int dout, bool act, int* err, cudaStream_t stream)
{
    const int64_t rows = frames * dout * dout;
    if (rows == 0) return cudaSuccess;
    TcParams p;
    p.in = in; p.in_s = in_s; p.wimg = wimg; p.bias = bias; p.out = out; p.out_s = out_s;
    p.rows = rows; p.in_c = in_c; p.out_c = out_c; p.ksize = ksize; p.din = din; p.dout = dout;
    p.stages = ((in_c >> 5) * ksize * ksize + 1) / 2;
    p.act = act ? 1 : 0;
    p.smem_stages = p.stages < kStages ? p.stages : kStages;
    p.n_max = out_c < kMaxN ? out_c : kMaxN;
    p.err = err;
    size_t smem = 1024 + static_cast<size_t>(p.smem_stages) * (kTileA + p.n_max * kBK * 2) + (kMaxN + 2 * kBM) * 4 +
                  (2 * p.smem_stages + 1) * 8 + 16;
    // Never let more CTAs share an SM than its 512 TMEM columns can serve:
    // pad the shared-memory request so the smem limit binds first.
    const int tmem_cols = p.n_max <= 32 ? 32 : p.n_max <= 64 ? 64 : p.n_max <= 128 ? 128 : 256;
    const int max_ctas = 512 / tmem_cols;
    const size_t smem_per_sm = 233472;  // 228 KB
    const size_t floor_smem = smem_per_sm / (max_ctas + 1) + 1;
    if (smem < floor_smem) smem = floor_smem;
    cudaError_t e = cudaFuncSetAttribute(conv_gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    dim3 grid(static_cast<unsigned>((rows + kBM - 1) / kBM), static_cast<unsigned>((out_c + kMaxN - 1) / kMaxN));
    conv_gemm_tc_kernel<<<grid, kThreads, smem, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace aic
