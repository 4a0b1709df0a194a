// Mamba out-projection on the tensor cores (A10: mambaSSMFwdOutProjKernel,
// AICortex kernels.h:1188-1259, batched): out = act(acc * rsqrt(sum_chunk
// acc^2 / min(out, 256) + eps) + bias), acc = sum_ic y[ic] * W_out[oc][ic].
//
// Operands. A weight of the packed int4 format is q * max(2^s / 7, 2^-13)
// (kernels.h:69,77) = (q * F(s)) / 7 with F(s) = 2^s, or 7 * 2^-13 where the
// reference clamps; q * F(s) has at most 6 significant bits, so the weight
// image holds it exactly in bf16 ([out][E], built at load time) and the 1/7
// moves to the epilogue. The fp32 activations y are carried as two bf16
// planes, hi = bf16(y) and lo = bf16(y - hi) (16 significant bits, relative
// error <= 2^-17), written that way by the SSM scan. Two kind::f16 MMAs per
// K16 step (hi x W, lo x W) accumulate in one fp32 TMEM accumulator; every
// product is exact, so the result differs from the reference's fp32 fmaf
// chain only by the accumulation order and the 2^-17 truncation of y (about
// 1e-5 of the output scale; the stated tolerance is 1e-3).
//
// Pipeline (persistent, one CTA of 6 warps per SM, tiles of 128 rows x BN
// output channels, BN = min(out, 256) = one RMSNorm chunk):
//   warp 0      TMA producer: A_hi, A_lo (128 x 64 bf16) and W (BN x 64 bf16)
//               tiles per 64-wide K stage, 128-byte swizzle, onto full[s];
//   warp 1      MMA issue (one thread): 8 MMAs per stage into one of two TMEM
//               accumulators, commit to empty[s] and, per tile, acc_full[b];
//   warps 2..5  epilogue: each thread owns one row (TMEM lane), folds the
//               row's sum of squares over the chunk, then normalises, adds the
//               bias, applies the activation and stores fp32; frees the
//               accumulator on acc_empty[b], so it overlaps the next tile.
// Every mbarrier wait is bounded; on timeout the kernel records an error code
// in the device error word, stops issuing work, drains its MMAs and releases
// TMEM. No cluster multicast.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>

#include <algorithm>
#include <mutex>

#include "aic_common.cuh"
#include "aic_kernels.h"
#include "tc_ptx.cuh"

namespace aic {
namespace {
using namespace tc;

constexpr int kOpBK = 64;                   // K elements per stage: one 128-byte swizzle row of bf16
constexpr int kOpThreads = 192;             // TMA warp, MMA warp, 4 epilogue warps
constexpr uint32_t kOpATile = 128 * 128;    // bytes of a 128 x 64 bf16 A tile
constexpr int kOpSmemBudget = 200 * 1024;   // stage ring budget

struct OpParams {
    const float* bias;
    float* out;
    int64_t rows;
    int64_t n_tiles;
    int E, out_c, bn, act, n_tiles_n, stages;
    int* err;
};

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

__device__ __forceinline__ void tma_prefetch_map(const CUtensorMap* map)
{
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__global__ void __launch_bounds__(kOpThreads, 1)
    outproj_tc_kernel(const __grid_constant__ CUtensorMap ta_hi, const __grid_constant__ CUtensorMap ta_lo,
                      const __grid_constant__ CUtensorMap tb, OpParams p)
{
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    const int S = p.stages, bn = p.bn;
    const uint32_t b_bytes = static_cast<uint32_t>(bn) * 128u;
    const uint32_t stage_bytes = 2 * kOpATile + b_bytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(base + S * stage_bytes);
    uint64_t* full = bars;
    uint64_t* empty = bars + S;
    uint64_t* acc_full = bars + 2 * S;
    uint64_t* acc_empty = acc_full + 2;
    uint64_t* drain = acc_empty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    uint32_t tmem_cols = 32;
    while (tmem_cols < 2u * static_cast<uint32_t>(bn)) tmem_cols <<= 1;
    if (tid == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(smem_addr(&full[i]), 1);
            mbar_init(smem_addr(&empty[i]), 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(smem_addr(&acc_full[i]), 1);
            mbar_init(smem_addr(&acc_empty[i]), 4);
        }
        mbar_init(smem_addr(drain), 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) tmem_alloc(smem_addr(tmem_slot), tmem_cols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int KB = p.E / kOpBK;

    if (warp == 0) {
        if (lane == 0) {
            tma_prefetch_map(&ta_hi);
            tma_prefetch_map(&ta_lo);
            tma_prefetch_map(&tb);
            uint32_t it = 0;
            for (int64_t tile = blockIdx.x; tile < p.n_tiles && !*abort_flag; tile += gridDim.x) {
                const int m_blk = static_cast<int>(tile / p.n_tiles_n), n_blk = static_cast<int>(tile % p.n_tiles_n);
                for (int kb = 0; kb < KB; ++kb, ++it) {
                    const int s = static_cast<int>(it % S);
                    const uint32_t use = it / S;
                    if (use > 0 && !mbar_wait(smem_addr(&empty[s]), (use - 1) & 1u, p.err, 41)) {
                        *abort_flag = 1;
                        break;
                    }
                    uint8_t* st = base + s * stage_bytes;
                    const uint32_t bar = smem_addr(&full[s]);
                    mbar_expect_tx(bar, stage_bytes);
                    tma_load_2d(smem_addr(st), &ta_hi, kb * kOpBK, m_blk * 128, bar);
                    tma_load_2d(smem_addr(st + kOpATile), &ta_lo, kb * kOpBK, m_blk * 128, bar);
                    tma_load_2d(smem_addr(st + 2 * kOpATile), &tb, kb * kOpBK, n_blk * bn, bar);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = instr_desc(bn);
            uint32_t it = 0, local = 0;
            for (int64_t tile = blockIdx.x; tile < p.n_tiles && !*abort_flag; tile += gridDim.x, ++local) {
                const uint32_t ab = local & 1u, au = local >> 1;
                if (au > 0 && !mbar_wait(smem_addr(&acc_empty[ab]), (au - 1) & 1u, p.err, 42)) {
                    *abort_flag = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem + ab * static_cast<uint32_t>(bn);
                bool ok = true;
                for (int kb = 0; kb < KB; ++kb, ++it) {
                    const int s = static_cast<int>(it % S);
                    if (!mbar_wait(smem_addr(&full[s]), (it / S) & 1u, p.err, 43)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_hi = smem_addr(base + s * stage_bytes), a_lo = a_hi + kOpATile,
                                   b = a_hi + 2 * kOpATile;
#pragma unroll
                    for (int j = 0; j < kOpBK / 16; ++j) {
                        mma_f16(d, smem_desc(a_hi + 32 * j), smem_desc(b + 32 * j), idesc, (kb > 0 || j > 0) ? 1u : 0u);
                        mma_f16(d, smem_desc(a_lo + 32 * j), smem_desc(b + 32 * j), idesc, 1u);
                    }
                    mma_commit(smem_addr(&empty[s]));
                }
                if (!ok) {
                    *abort_flag = 1;
                    break;
                }
                mma_commit(smem_addr(&acc_full[ab]));
            }
            // every MMA this CTA issued has completed before TMEM is released (a
            // timeout records 44 and gets one more bounded window)
            mma_commit(smem_addr(drain));
            if (!mbar_wait(smem_addr(drain), 0u, p.err, 44)) mbar_wait(smem_addr(drain), 0u, p.err, 44);
        }
    } else {
        const int q = warp & 3;  // this warp's quarter of the TMEM lanes
        const int erow = q * 32 + lane;
        const float inv7 = 1.0f / kQMax;
        const float inv_div = __frcp_rn(static_cast<float>(min(p.out_c, kNormChunk)));
        uint32_t local = 0;
        for (int64_t tile = blockIdx.x; tile < p.n_tiles; tile += gridDim.x, ++local) {
            const uint32_t ab = local & 1u, au = local >> 1;
            bool ok = !*abort_flag && mbar_wait(smem_addr(&acc_full[ab]), au & 1u, p.err, 45);
            ok = __all_sync(0xFFFFFFFFu, ok);
            if (!ok) {
                *abort_flag = 1;
                break;
            }
            tc_fence_after();
            const int m_blk = static_cast<int>(tile / p.n_tiles_n), n_blk = static_cast<int>(tile % p.n_tiles_n);
            const uint32_t taddr = tmem + (static_cast<uint32_t>(q * 32) << 16) + ab * static_cast<uint32_t>(bn);
            float ss = 0.0f;
            for (int c = 0; c < bn; c += 32) {
                float v[32];
                tmem_ld32(taddr + c, v);
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const float x = v[i] * inv7;
                    ss = fmaf(x, x, ss);
                }
            }
            const float inv_rms = p.out_c < 2 ? 1.0f : __frsqrt_rn(fmaf(ss, inv_div, kEps));
            const int64_t row = static_cast<int64_t>(m_blk) * 128 + erow;
            const int n0 = n_blk * bn;
            float* orow = p.out + row * p.out_c + n0;
            for (int c = 0; c < bn; c += 32) {
                float v[32];
                tmem_ld32(taddr + c, v);
                const float4* b4 = reinterpret_cast<const float4*>(p.bias + n0 + c);
#pragma unroll
                for (int i4 = 0; i4 < 8; ++i4) {
                    const float4 bb = __ldg(b4 + i4);
                    float o[4] = {fmaf(v[4 * i4] * inv7, inv_rms, bb.x), fmaf(v[4 * i4 + 1] * inv7, inv_rms, bb.y),
                                  fmaf(v[4 * i4 + 2] * inv7, inv_rms, bb.z), fmaf(v[4 * i4 + 3] * inv7, inv_rms, bb.w)};
                    if (p.act == 1) {
#pragma unroll
                        for (int k = 0; k < 4; ++k) o[k] = silu_f(o[k]);
                    } else if (p.act == 2) {
#pragma unroll
                        for (int k = 0; k < 4; ++k) o[k] = sigmoid_f(o[k]);
                    }
                    if (row < p.rows) reinterpret_cast<float4*>(orow + c)[i4] = make_float4(o[0], o[1], o[2], o[3]);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_addr(&acc_empty[ab]));
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, tmem_cols);
    }
}

// W_out of the packed blob -> bf16 [out][E] holding q * F(s) (exact).
__global__ void build_outproj_wimg_kernel(const uint32_t* __restrict__ blob, const int8_t* __restrict__ blob_s,
                                          int64_t off_w, int E, int out_c, __nv_bfloat16* __restrict__ img)
{
    const int64_t gi = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;  // group of W_out
    const int64_t groups = static_cast<int64_t>(out_c) * (E >> 5);
    if (gi >= groups) return;
    const int64_t g = (off_w >> 5) + gi;  // off_w is a multiple of 32
    const uint4 w = reinterpret_cast<const uint4*>(blob)[g];
    const float f = stage_factor(blob_s[g]);
    const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
    uint32_t o[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(static_cast<float>(code_of(ww[i >> 2], (2 * i) & 7)) * f,
                                                       static_cast<float>(code_of(ww[i >> 2], (2 * i + 1) & 7)) * f);
        o[i] = *reinterpret_cast<const uint32_t*>(&h);
    }
    uint4* dst = reinterpret_cast<uint4*>(img + gi * 32);
#pragma unroll
    for (int i = 0; i < 4; ++i) dst[i] = make_uint4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder()
{
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// 2-D bf16 tensor map over a row-major [outer][inner] array, box of
// 64 (inner, 128 bytes) x box_outer, 128-byte swizzle; out-of-range rows read 0.
bool bf16_map(CUtensorMap* m, const void* ptr, uint64_t inner, uint64_t outer, uint32_t box_outer)
{
    auto enc = tensor_map_encoder();
    if (!enc) return false;
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {inner * 2};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(kOpBK), box_outer};
    const cuuint32_t estr[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int outproj_bn(int out_c) { return out_c <= kNormChunk ? out_c : kNormChunk; }

}  // namespace

bool outproj_tc_supported(int E, int out_c)
{
    return E >= kOpBK && E % kOpBK == 0 && out_c >= 32 && out_c % 32 == 0 &&
           (out_c <= kNormChunk || out_c % kNormChunk == 0);
}

size_t outproj_tc_wimg_bytes(int E, int out_c) { return static_cast<size_t>(E) * out_c * 2; }

cudaError_t launch_build_outproj_wimg(const uint32_t* blob, const int8_t* blob_s, int64_t off_w, int E, int out_c,
                                      void* img, cudaStream_t stream)
{
    const int64_t groups = static_cast<int64_t>(out_c) * (E >> 5);
    build_outproj_wimg_kernel<<<static_cast<unsigned>((groups + 255) / 256), 256, 0, stream>>>(
        blob, blob_s, off_w, E, out_c, static_cast<__nv_bfloat16*>(img));
    return cudaGetLastError();
}

cudaError_t launch_outproj_tc(const void* y_planes, const void* wimg, const float* bias, int E, int out_c, int act,
                              int64_t rows, float* out, int* err, cudaStream_t stream)
{
    if (rows == 0) return cudaSuccess;
    if (!outproj_tc_supported(E, out_c)) return cudaErrorInvalidValue;
    const int bn = outproj_bn(out_c);
    const __nv_bfloat16* hi = static_cast<const __nv_bfloat16*>(y_planes);
    CUtensorMap ta_hi, ta_lo, tb;
    if (!bf16_map(&ta_hi, hi, E, rows, 128) || !bf16_map(&ta_lo, hi + rows * E, E, rows, 128) ||
        !bf16_map(&tb, wimg, E, out_c, bn))
        return cudaErrorInvalidValue;
    const uint32_t stage_bytes = 2 * kOpATile + static_cast<uint32_t>(bn) * 128u;
    const int stages = std::min(6, kOpSmemBudget / static_cast<int>(stage_bytes));
    const size_t smem = 1024 + stages * stage_bytes + (2 * stages + 5) * 8 + 16;
    const cudaError_t attr_err =
        cudaFuncSetAttribute(outproj_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (attr_err != cudaSuccess) return attr_err;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    OpParams p;
    p.bias = bias;
    p.out = out;
    p.rows = rows;
    p.E = E;
    p.out_c = out_c;
    p.bn = bn;
    p.act = act;
    p.n_tiles_n = out_c / bn;
    p.n_tiles = ((rows + 127) / 128) * p.n_tiles_n;
    p.stages = stages;
    p.err = err;
    const unsigned grid = static_cast<unsigned>(std::min<int64_t>(p.n_tiles, sms));
    outproj_tc_kernel<<<grid, kOpThreads, smem, stream>>>(ta_hi, ta_lo, tb, p);
    return cudaGetLastError();
}

}  // namespace aic
