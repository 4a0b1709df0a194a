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
// Structure: a persistent, warp-specialised kernel, one CTA per SM walking
// tiles of 128 pixel rows x one 256-channel chunk:
//   - producer warps convert, per 64-wide K stage, the A rows from the packed
//     activations (im2col on the fly for the dense convs) into a 128B-swizzled
//     K-major bf16 tile of a multi-stage shared-memory ring; the B stage
//     (weights) is a pre-swizzled bf16 image built at weight-load time and
//     fetched with one cp.async.bulk into the same layout;
//   - one thread issues four tcgen05.mma (M128 x N x K16) per stage into one
//     of two TMEM accumulators and commits stages and tiles to mbarriers;
//   - epilogue warps read a finished accumulator with tcgen05.ld (warp w owns
//     TMEM lanes 32*(w&3)..: its 32 pixel rows; two warpgroups take alternate
//     32-channel groups and exchange the rows' sums of squares once through
//     shared memory); each thread normalises, activates and packs whole
//     32-channel groups of its own row, so the requant needs no cross-thread
//     reduction. The epilogue of one tile overlaps the main loop of the next.
// All mbarrier waits are bounded; on timeout the kernel records an error code
// in *err, every role skips its remaining work, and the TMEM columns are
// released only after the CTA's last tcgen05.commit has completed.
#include <cuda_bf16.h>

#include "aic_common.cuh"
#include "aic_kernels.h"

namespace aic {
namespace {

constexpr int kBM = 128;          // pixel rows per tile (= TMEM lanes)
constexpr int kBK = 64;           // K elements per stage (128 bytes of bf16)
constexpr int kStages = 2;        // smem pipeline depth
constexpr int kProducerWarps = 4;
constexpr int kProducerThreads = kProducerWarps * 32;
constexpr int kMmaWarp = 4;
constexpr int kEpiWarp0 = 5;
constexpr int kEpiWarps = 8;
constexpr int kPThreads = (kEpiWarp0 + kEpiWarps) * 32;  // 416
constexpr int kTileA = kBM * kBK * 2;          // 16 KB
constexpr int kMaxN = 256;
constexpr int kTileBMax = kMaxN * kBK * 2;     // 32 KB
constexpr uint32_t kWaitLimit = 1u << 22;

struct TcParams {
    const uint32_t* in;
    const int8_t* in_s;
    const uint8_t* wimg;
    const float* bias;
    uint32_t* out;
    int8_t* out_s;
    int64_t rows;
    int in_c, out_c, ksize, din, dout, stages, act;
    int smem_stages, n_max, m_tiles, n_chunks;
    int* err;
};

// ---- PTX wrappers ---------------------------------------------------------

__device__ __forceinline__ uint32_t smem_addr(const void* p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait; returns false (and records `code`) when the phase never completes.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int* err, int code)
{
    for (uint32_t i = 0; i < kWaitLimit; ++i) {
        if (mbar_try(bar, parity)) return true;
        if (i > 256) __nanosleep(128);
    }
    atomicCAS(err, 0, code);
    return false;
}

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar)
{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t cols)
{
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(cols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols)
{
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols));
}

// K-major operand, 128-byte swizzle: rows of 128 B, 8-row atoms of 1024 B.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr)
{
    uint64_t d = 0;
    d |= static_cast<uint64_t>((addr >> 4) & 0x3FFFu);        // start address
    d |= static_cast<uint64_t>(1u) << 16;                      // leading byte offset (unused for SW128 K-major)
    d |= static_cast<uint64_t>(1024u >> 4) << 32;              // stride byte offset: next 8-row atom
    d |= static_cast<uint64_t>(1u) << 46;                      // descriptor version (sm_100)
    d |= static_cast<uint64_t>(2u) << 61;                      // layout: SWIZZLE_128B
    return d;
}

// kind::f16 instruction descriptor: bf16 x bf16 -> f32, both K-major, M = 128.
__host__ __device__ constexpr uint32_t instr_desc(int n)
{
    return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(kBM >> 4) << 24);
}

__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint32_t bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32])
{
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// ---- int4 -> bf16 staging ----------------------------------------------------

// bf16 factor F(s): 2^s where the reference's unit is 2^s/7, 7*2^-13 where it
// clamps to 2^-13.
__device__ __forceinline__ float stage_factor(int8_t s) { return s >= -10 ? exp2f(static_cast<float>(s)) : 7.0f * kEps; }

// 8 codes of `word` -> 4 bf16x2 words holding (code j, code j+4) * f. The
// nibble pair (n_j, n_j+4) lands in the two halves as 0x43.. | (n ^ 8), i.e.
// the bf16 value 128 + q + 8; one fma with (f, -136 f) leaves q * f exactly.
// A and B use the same K permutation, so the dot products are unchanged.
__device__ __forceinline__ uint4 unpack_word(uint32_t word, __nv_bfloat162 f, __nv_bfloat162 c)
{
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        uint32_t x = ((word >> (4 * j)) & 0x000F000Fu) ^ 0x43084308u;
        __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162*>(&x);
        v = __hfma2(v, f, c);
        o[j] = *reinterpret_cast<uint32_t*>(&v);
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
}

// Writes one 32-element group (4 chunks of 16 B) of a K-major SW128 row.
__device__ __forceinline__ void stage_group(uint8_t* tile, int row, int group_in_stage, uint4 words, int8_t s)
{
    const float f = stage_factor(s);
    const __nv_bfloat162 fv = __floats2bfloat162_rn(f, f);
    const __nv_bfloat162 cv = __floats2bfloat162_rn(-136.0f * f, -136.0f * f);
    uint8_t* rowp = tile + (row >> 3) * 1024 + (row & 7) * 128;
    const uint32_t w[4] = {words.x, words.y, words.z, words.w};
#pragma unroll
    for (int cl = 0; cl < 4; ++cl) {
        const int chunk = (group_in_stage << 2) + cl;
        *reinterpret_cast<uint4*>(rowp + ((chunk ^ (row & 7)) << 4)) = unpack_word(w[cl], fv, cv);
    }
}

__device__ __forceinline__ void stage_zero(uint8_t* tile, int row, int group_in_stage)
{
    uint8_t* rowp = tile + (row >> 3) * 1024 + (row & 7) * 128;
#pragma unroll
    for (int cl = 0; cl < 4; ++cl) {
        const int chunk = (group_in_stage << 2) + cl;
        *reinterpret_cast<uint4*>(rowp + ((chunk ^ (row & 7)) << 4)) = make_uint4(0u, 0u, 0u, 0u);
    }
}

// Input pixel of output row r for tap `tap` (stride == ksize, no padding).
__device__ __forceinline__ int64_t tap_pixel(int64_t r, int tap, int ksize, int din, int dout)
{
    if (ksize == 1) return r;
    const int64_t hw = static_cast<int64_t>(dout) * dout;
    const int64_t frame = r / hw;
    const int p = static_cast<int>(r - frame * hw);
    const int hi = (p / dout) * ksize + tap / ksize;
    const int wi = (p % dout) * ksize + tap % ksize;
    return frame * din * din + static_cast<int64_t>(hi) * din + wi;
}

__device__ __forceinline__ void mbar_expect_tx_noarrive(uint32_t bar, uint32_t bytes)
{
    asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar)
{
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Bounded wait that also gives up at once when another role has aborted.
__device__ __forceinline__ bool role_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* err, int code)
{
    if (*abort_flag) return false;
    for (uint32_t i = 0; i < kWaitLimit; ++i) {
        if (mbar_try(bar, parity)) return true;
        if (i > 256) {
            if (*abort_flag) return false;
            __nanosleep(128);
        }
    }
    atomicCAS(err, 0, code);
    *abort_flag = 1;
    return false;
}

// Persistent, warp-specialised kernel. One CTA per SM walks tiles
// t = blockIdx.x, blockIdx.x + gridDim.x, ... (tile = 128 pixel rows x one
// 256-channel chunk). Roles:
//   warps 0-3   producers: fill the A ring (one pixel row per thread, both
//               groups of each 64-wide K stage); thread 0 also fetches the B
//               stage with cp.async.bulk; all 128 arrive on full[slot];
//   warp  4     allocates TMEM (two accumulators) and, on lane 0, issues the
//               tcgen05.mma of every stage, committing each stage to
//               empty[slot] and each finished tile to acc_full[buf];
//   warps 5-12  epilogue: wait acc_full[buf], read the accumulator, normalise,
//               activate, requant and store; release acc_empty[buf].
// The epilogue of tile i overlaps the main loop of tile i+1.
__global__ void __launch_bounds__(kPThreads, 1) conv_gemm_tc_kernel(TcParams p)
{
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int nst = p.smem_stages;
    const int tile_b_max = p.n_max * kBK * 2;
    uint8_t* a_tiles = base;
    uint8_t* b_tiles = base + nst * kTileA;
    float* part = reinterpret_cast<float*>(b_tiles + nst * tile_b_max);  // [2 bufs][2 halves][kBM]
    uint64_t* bars = reinterpret_cast<uint64_t*>(part + 4 * kBM);
    uint64_t* full = bars;
    uint64_t* empty = bars + nst;
    uint64_t* acc_full = bars + 2 * nst;
    uint64_t* acc_empty = acc_full + 2;
    uint64_t* final_bar = acc_empty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(final_bar + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t acc_cols = p.n_max <= 32 ? 32u : p.n_max <= 64 ? 64u : p.n_max <= 128 ? 128u : 256u;
    if (tid == 0) {
        for (int i = 0; i < nst; ++i) {
            mbar_init(smem_addr(&full[i]), kProducerThreads);
            mbar_init(smem_addr(&empty[i]), 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(smem_addr(&acc_full[i]), 1);
            mbar_init(smem_addr(&acc_empty[i]), kEpiWarps);
        }
        mbar_init(smem_addr(final_bar), 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kMmaWarp) tmem_alloc(smem_addr(tmem_slot), 2 * acc_cols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int num_tiles = p.m_tiles * p.n_chunks;
    const int G = p.in_c >> 5;
    const int GK = G * p.ksize * p.ksize;

    if (warp < kProducerWarps) {
        uint32_t gs = 0;
        for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x) {
            const int m_tile = tile / p.n_chunks, chunk = tile - m_tile * p.n_chunks;
            const int n0 = chunk * kMaxN;
            const int tile_b = min(kMaxN, p.out_c - n0) * kBK * 2;
            const uint8_t* wimg = p.wimg + static_cast<int64_t>(n0) * p.stages * kBK * 2;
            const int64_t row = static_cast<int64_t>(m_tile) * kBM + tid;
            const bool row_ok = row < p.rows;
            for (int s = 0; s < p.stages; ++s, ++gs) {
                const int slot = static_cast<int>(gs % nst);
                const uint32_t r = gs / nst;
                if (!role_wait(smem_addr(&empty[slot]), (r & 1u) ^ 1u, abort_flag, p.err, 1)) break;
                uint8_t* a_tile = a_tiles + slot * kTileA;
                if (tid == 0) {
                    mbar_expect_tx_noarrive(smem_addr(&full[slot]), static_cast<uint32_t>(tile_b));
                    bulk_g2s(smem_addr(b_tiles + slot * tile_b_max), wimg + static_cast<int64_t>(s) * tile_b,
                             static_cast<uint32_t>(tile_b), smem_addr(&full[slot]));
                }
#pragma unroll
                for (int gl = 0; gl < 2; ++gl) {
                    const int gk = 2 * s + gl;
                    if (row_ok && gk < GK) {
                        const int tap = gk / G, g = gk - tap * G;
                        const int64_t pix = tap_pixel(row, tap, p.ksize, p.din, p.dout);
                        const uint4 words = __ldg(reinterpret_cast<const uint4*>(p.in) + pix * G + g);
                        stage_group(a_tile, tid, gl, words, __ldg(p.in_s + pix * G + g));
                    } else {
                        stage_zero(a_tile, tid, gl);
                    }
                }
                fence_async_smem();
                mbar_arrive(smem_addr(&full[slot]));
            }
        }
    } else if (warp == kMmaWarp) {
        if (lane == 0) {
            uint32_t gs = 0, i = 0;
            for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x, ++i) {
                const int chunk = tile % p.n_chunks;
                const int n_cta = min(kMaxN, p.out_c - chunk * kMaxN);
                const uint32_t idesc = instr_desc(n_cta);
                const uint32_t b = i & 1u;
                if (!role_wait(smem_addr(&acc_empty[b]), ((i >> 1) & 1u) ^ 1u, abort_flag, p.err, 4)) break;
                tc_fence_after();
                const uint32_t tacc = tmem + b * acc_cols;
                for (int s = 0; s < p.stages; ++s, ++gs) {
                    const int slot = static_cast<int>(gs % nst);
                    if (!role_wait(smem_addr(&full[slot]), (gs / nst) & 1u, abort_flag, p.err, 2)) break;
                    tc_fence_after();
                    const uint32_t a_addr = smem_addr(a_tiles + slot * kTileA);
                    const uint32_t b_addr = smem_addr(b_tiles + slot * tile_b_max);
#pragma unroll
                    for (int j = 0; j < kBK / 16; ++j)
                        mma_bf16(tacc, smem_desc(a_addr + 32 * j), smem_desc(b_addr + 32 * j), idesc,
                                 (s > 0 || j > 0) ? 1u : 0u);
                    mma_commit(smem_addr(&empty[slot]));
                }
                mma_commit(smem_addr(&acc_full[b]));
            }
            mma_commit(smem_addr(final_bar));
        }
        __syncwarp();
    } else {
        const int q = warp & 3, half = (warp - kEpiWarp0) >> 2;
        const int erow = q * 32 + lane;
        const float inv49 = (1.0f / kQMax) * (1.0f / kQMax);
        const float inv_div = __frcp_rn(static_cast<float>(min(p.out_c, kNormChunk)));
        const int groups_out = p.out_c >> 5;
        uint32_t i = 0;
        // Every epilogue warp runs the same number of iterations and always
        // reaches the named barrier, even after an abort (it then skips work).
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++i) {
            const int m_tile = tile / p.n_chunks, chunk = tile - m_tile * p.n_chunks;
            const int n0 = chunk * kMaxN;
            const int ngroups = min(kMaxN, p.out_c - n0) >> 5;
            const uint32_t b = i & 1u;
            const bool ok = role_wait(smem_addr(&acc_full[b]), (i >> 1) & 1u, abort_flag, p.err, 3);
            tc_fence_after();
            const uint32_t taddr = tmem + b * acc_cols + (static_cast<uint32_t>(q * 32) << 16);
            float ss = 0.0f;
            if (ok) {
                for (int g = half; g < ngroups; g += 2) {
                    float v[32];
                    tmem_ld32(taddr + 32 * g, v);
#pragma unroll
                    for (int k = 0; k < 32; ++k) ss = fmaf(v[k], v[k], ss);
                }
            }
            float* pb = part + b * 2 * kBM;
            pb[half * kBM + erow] = ss;
            asm volatile("bar.sync 1, %0;" ::"n"(kEpiWarps * 32) : "memory");
            if (ok) {
                const float total = (pb[erow] + pb[kBM + erow]) * (inv49 * inv49);
                const float sc = inv49 * __frsqrt_rn(fmaf(total, inv_div, kEps));
                const int64_t row = static_cast<int64_t>(m_tile) * kBM + erow;
                for (int g = half; g < ngroups; g += 2) {
                    float v[32];
                    tmem_ld32(taddr + 32 * g, v);
                    const float4* b4 = reinterpret_cast<const float4*>(p.bias + n0 + 32 * g);
#pragma unroll
                    for (int i4 = 0; i4 < 8; ++i4) {
                        const float4 bb = __ldg(b4 + i4);
                        const float bv[4] = {bb.x, bb.y, bb.z, bb.w};
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            const float x = fmaf(v[4 * i4 + k], sc, bv[k]);
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
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_addr(&acc_empty[b]));
            }
        }
    }
    __syncthreads();
    if (warp == kMmaWarp) {
        // every MMA this CTA issued has completed before the columns are freed
        role_wait(smem_addr(final_bar), 0u, abort_flag, p.err, 5);
        tc_fence_after();
        tmem_dealloc(tmem, 2 * acc_cols);
    }
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
    int dev = 0, sms = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    TcParams p;
    p.in = in; p.in_s = in_s; p.wimg = wimg; p.bias = bias; p.out = out; p.out_s = out_s;
    p.rows = rows; p.in_c = in_c; p.out_c = out_c; p.ksize = ksize; p.din = din; p.dout = dout;
    p.stages = ((in_c >> 5) * ksize * ksize + 1) / 2;
    p.act = act ? 1 : 0;
    p.n_max = out_c < kMaxN ? out_c : kMaxN;
    p.m_tiles = static_cast<int>((rows + kBM - 1) / kBM);
    p.n_chunks = (out_c + kMaxN - 1) / kMaxN;
    p.err = err;
    const int stage_bytes = kTileA + p.n_max * kBK * 2;
    int nst = (200 * 1024) / stage_bytes;
    nst = nst < 2 ? 2 : (nst > 8 ? 8 : nst);
    p.smem_stages = nst;
    const size_t smem = 1024 + static_cast<size_t>(nst) * stage_bytes + 4 * kBM * 4 + (2 * nst + 5) * 8 + 16;
    e = cudaFuncSetAttribute(conv_gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    const int64_t tiles = static_cast<int64_t>(p.m_tiles) * p.n_chunks;
    const unsigned grid = static_cast<unsigned>(tiles < sms ? tiles : sms);
    conv_gemm_tc_kernel<<<grid, kPThreads, smem, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace aic
