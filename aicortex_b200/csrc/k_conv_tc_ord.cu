// Quantized conv (pointwise k=1, dense k=2 with stride 2) on the 5th-generation
// tensor cores with the reference's floating-point accumulation order, so the
// packed outputs are bit-identical to the reference kernels
// (AICortex kernels.h:217-282 convPointwiseFwdKernel, 514-585
// convDenseFwdKernel).
//
// The reference accumulates, per output (pixel, channel), over taps k and
// 32-element groups g in order:
//     acc[k & 3] = fmaf(unit(s_in[k][g]), unit(s_w[k][g]) * dot[k][g], acc[k & 3])
// where dot is the exact integer dot product of the two groups' codes, and
// folds the partial sums as ((acc0 + acc1) + acc2) + acc3. The integer dots
// are what a tensor core computes exactly: with the codes themselves as fp16
// operands (q and 16 q against w and w / 16, see unpack_word_h), a K=32
// kind::f16 MMA sums 32 integer products of magnitude <= 64 in fp32, which is
// exact. So each stage of two groups issues
// two MMAs per group into a group-private TMEM accumulator, and the CUDA cores
// run the reference's fmaf chain over the groups, in group order, from those
// exact dots. Only the chain runs in fp32, exactly as the reference does.
//
// Tile: 128 pixel rows x 64 output channels, so a thread's chain state is
// 32 accumulators (plus 32 for the finished taps of a 2x2 conv) and two CTAs
// (128 registers per thread) fit on an SM. The RMSNorm spans up to 256 channels, so the CTAs covering
// one norm chunk form a cluster (2 for 128 channels, 4 for 256) and exchange
// their rows' per-32-channel sums of squares through distributed shared
// memory; the sums are then folded with the reference's butterfly tree (32
// lanes, then 8 warps). Layers with <= 64 output channels use no cluster.
//
// Pipeline (256 threads, a run of consecutive row tiles per CTA): the CTA
// walks one sequence of stages across its tiles. For stage s every thread stages one
// (row, group) of the A tile (interleaved K-major layout) from the packed
// activations (im2col on the fly for k=2) and records unit(s_in); thread 0
// fetches the stage's B image (fp16 codes in the SW128 layout, followed by
// unit(s_w) of both groups)
// with one cp.async.bulk and issues the MMAs for stage s; meanwhile all
// threads run the chain for stage s-1 from TMEM (tcgen05.ld), and after a
// tile's last stage its epilogue, which so overlaps the next tile's first
// MMAs. A, B and the per-group accumulators are double buffered. Thread
// (row r, half h) owns the chain of row r over the tile's 32-channel group h.
//
// All mbarrier waits are bounded; on timeout the kernel records an error code
// in *err, skips the remaining work, still takes part in every CTA and
// cluster barrier, waits (bounded) for its MMAs and releases its TMEM.
#include <cuda_bf16.h>

#include "aic_common.cuh"
#include "aic_kernels.h"
#include "tc_ptx.cuh"

namespace aic {
namespace {

using namespace tc;

constexpr int kThreads = 256;
constexpr int kBK = 64;                   // two 32-element groups per stage
constexpr int kTileA = kBM * kBK * 2;     // 16 KB of fp16
constexpr int kNCta = 64;                 // output channels per CTA
constexpr int kImgRow = kBK * 2 + 2 * 4;  // image bytes per channel per stage: 128 B codes + 2 units
constexpr int kResidentStages = 8;        // up to this many stages per tile stay resident in shared memory

struct OrdParams {
    const uint32_t* in;
    const int8_t* in_s;
    const uint8_t* wimg;
    const float* bias;
    uint32_t* out;
    int8_t* out_s;
    int64_t rows;
    int in_c, out_c, din, dout, stages, gk_total, act;
    int n_max;          // largest channel count of any CTA of the launch
    int tiles_per_cta;  // consecutive 128-row tiles each CTA column processes
    int* err;
};

// Barrier over every thread of the cluster with release/acquire ordering of
// shared memory (local and distributed).
__device__ __forceinline__ void cluster_sync_all()
{
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Store to the same shared-memory offset in the cluster CTA of rank `peer`.
__device__ __forceinline__ void st_peer_f32(uint32_t local_addr, uint32_t peer, float v)
{
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_addr), "r"(peer));
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(remote), "f"(v) : "memory");
}

// Lane 0's value of the reference's `v += __shfl_xor_sync(v, o)` for
// o = 16..1 over the 32 lanes' squares acc[i]^2 (kernels.h:266-267): a
// pairwise tree with stride halving. The products and sums are separately
// rounded (no contraction into fma).
__device__ __forceinline__ float tree_sq32(const float (&a)[32])
{
    float t[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) t[i] = __fadd_rn(__fmul_rn(a[i], a[i]), __fmul_rn(a[i + 16], a[i + 16]));
#pragma unroll
    for (int o = 8; o > 0; o >>= 1)
#pragma unroll
        for (int i = 0; i < o; ++i) t[i] = __fadd_rn(t[i], t[i + o]);
    return t[0];
}

// tree_sq32 over 32 values held as 16 pairs (value 2i + j in a[i].j), in
// scalar arithmetic (a square feeding a sum must not be fused).
__device__ __forceinline__ float tree_sq32x2(const float2 (&a)[16])
{
    float f[32];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        f[2 * i] = a[i].x;
        f[2 * i + 1] = a[i].y;
    }
    return tree_sq32(f);
}

// TMEM columns: per-group accumulators of n channels, double buffered over
// stages (a single stage needs one buffer, a single group one slot).
__host__ __device__ inline uint32_t ord_tmem_cols(int n, int stages, int gk_total)
{
    const int need = (stages > 1 ? 4 : gk_total > 1 ? 2 : 1) * n;
    return need <= 32 ? 32u : need <= 64 ? 64u : need <= 128 ? 128u : need <= 256 ? 256u : 512u;
}

// G1: a 2x2 conv with one group per tap. Each tap's chain is then a single
// term fmaf(unit(s_in), unit(s_w) * dot, 0), so ((a0 + a1) + a2) + a3 is
// accumulated directly into one register set (the products differ from the
// fmaf form only in the sign of a zero, which the sum and the requant erase).
template <int KS, int CS, bool ACT, bool G1 = false>
__global__ void __launch_bounds__(kThreads, 2) conv_gemm_tc_ord_kernel(OrdParams p)
{
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);  // stays a shared-space pointer
    // CTA y covers channels [n0, n0 + n_cta) of norm chunk y / CS
    const int n0 = static_cast<int>(blockIdx.y / CS) * kNormChunk + static_cast<int>(blockIdx.y % CS) * kNCta;
    const int n_cta = min(kNCta, p.out_c - n0);  // <= 0: a CTA past the end of a narrow chunk
    const bool live = n_cta > 0;
    // Weights: with at most kResidentStages stages per tile every stage's image
    // stays in shared memory (fetched once per CTA); otherwise two slots rotate
    // and each stage is fetched in turn. Codes and units sit in separate arrays
    // so that every code slot stays 1024-byte aligned for the SW128 layout.
    const int S = p.stages;
    const bool resident = S <= kResidentStages;
    const int nb = resident ? S : 2;
    uint8_t* a_tiles = base;                                   // [2][kTileA]
    uint8_t* b_codes = base + 2 * kTileA;                      // [nb][n_max][128 B]
    float* b_units = reinterpret_cast<float*>(b_codes + nb * p.n_max * 128);  // [nb][2][n_max]
    float* din_s = b_units + nb * 2 * p.n_max;                 // [2 buffers][2 groups][kBM] unit(s_in)
    float* bias_s = din_s + 4 * kBM;               // [kNCta]
    float* part = bias_s + kNCta;                  // [2 tiles][8][kBM] group sums of squares of the norm chunk
    uint64_t* bars = reinterpret_cast<uint64_t*>(part + 16 * kBM);  // 0,1: B full; 2,3: MMAs done; 4: drain
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 5);
    int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t ncols = live ? ord_tmem_cols(n_cta, p.stages, p.gk_total) : 0u;
    for (int i = tid; i < 16 * kBM; i += kThreads) part[i] = 0.0f;
    if (live && tid < n_cta) bias_s[tid] = p.bias[n0 + tid];
    if (tid == 0) {
        for (int i = 0; i < 5; ++i) mbar_init(smem_addr(&bars[i]), 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (live && warp == 0) tmem_alloc(smem_addr(tmem_slot), ncols);
    tc_fence_before();
    __syncthreads();
    if (CS > 1) cluster_sync_all();  // every peer's `part` is initialised before any remote store
    tc_fence_after();
    const uint32_t tmem = live ? *tmem_slot : 0u;

    // Row tiles of this CTA: tiles_per_cta consecutive tiles from tile0 (the
    // same tiles for every CTA of a cluster, which therefore run in lockstep).
    const int64_t n_tiles = (p.rows + kBM - 1) / kBM;
    const int64_t tile0 = static_cast<int64_t>(blockIdx.x) * p.tiles_per_cta;
    const int my_tiles = tile0 < n_tiles ? static_cast<int>(min(static_cast<int64_t>(p.tiles_per_cta), n_tiles - tile0)) : 0;
    const int total = my_tiles * S;

    const int prow = tid & (kBM - 1), pg = tid >> 7;  // producer: (row, group of the stage)
    const int G = p.in_c >> 5;
    const int GK = p.gk_total;
    const int stage_bytes = n_cta * kImgRow;
    const uint8_t* wimg = p.wimg + static_cast<int64_t>(n0) * S * kImgRow;
    const uint32_t idesc = instr_desc_h(n_cta);
    const float inv_div = __frcp_rn(static_cast<float>(min(p.out_c, kNormChunk)));

    // chain role: row erow (== prow), 32-channel group hw of the tile
    const int q = warp & 3, hw = warp >> 2;
    const int erow = q * 32 + lane;
    const bool has_cols = hw < (n_cta >> 5);
    const uint32_t tl = tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(32 * hw);
    constexpr bool kFold = KS == 2 && !G1;  // finished taps kept apart from the running chain
    float2 acc[16], sacc[kFold ? 16 : 1];  // channel pairs
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i] = dup2(0.0f);
#pragma unroll
    for (int i = 0; i < (kFold ? 16 : 1); ++i) sacc[i] = dup2(0.0f);

    // fmaf chain over the groups of global stage gc (stage sc of its tile);
    // next_fold: the group index at which the current tap's chain ends (the
    // stages of a tile arrive in order, so no division per group)
    int next_fold = G;
    auto chain = [&](int gc, int sc) -> bool {
        if (sc == 0) next_fold = G;
        const int buf = gc & 1;
        if (!mbar_wait(smem_addr(&bars[2 + buf]), static_cast<uint32_t>(gc >> 1) & 1u, p.err, 12)) return false;
        tc_fence_after();
        const float* units = b_units + (resident ? sc : buf) * 2 * p.n_max + 32 * hw;
        const float* dins = din_s + buf * 2 * kBM + erow;
        const uint32_t tb = tl + static_cast<uint32_t>(buf * 2 * n_cta);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int gk = 2 * sc + j;
            if (gk >= GK) break;
            if (kFold && gk == next_fold) {  // a tap's chain ends: fold it, start the next from 0
                next_fold += G;
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    sacc[kFold ? i : 0] = add2(sacc[kFold ? i : 0], acc[i]);
                    acc[i] = dup2(0.0f);
                }
            }
            if (has_cols) {
                const float2 du = dup2(dins[j * kBM]);
                const float4* u4 = reinterpret_cast<const float4*>(units + j * n_cta);
#pragma unroll
                for (int h16 = 0; h16 < 2; ++h16) {
                    float pv[16];
                    tmem_ld16(tb + static_cast<uint32_t>(j * n_cta + 16 * h16), pv);
#pragma unroll
                    for (int i4 = 0; i4 < 4; ++i4) {
                        const float4 u = u4[4 * h16 + i4];
                        const int b = 8 * h16 + 2 * i4;
                        const float2 p0 = mul2(make_float2(u.x, u.y), make_float2(pv[4 * i4], pv[4 * i4 + 1]));
                        const float2 p1 = mul2(make_float2(u.z, u.w), make_float2(pv[4 * i4 + 2], pv[4 * i4 + 3]));
                        if (G1) {  // scalar: the product is rounded before the add
                            acc[b].x = __fadd_rn(acc[b].x, __fmul_rn(du.x, p0.x));
                            acc[b].y = __fadd_rn(acc[b].y, __fmul_rn(du.y, p0.y));
                            acc[b + 1].x = __fadd_rn(acc[b + 1].x, __fmul_rn(du.x, p1.x));
                            acc[b + 1].y = __fadd_rn(acc[b + 1].y, __fmul_rn(du.y, p1.y));
                        } else {
                            acc[b] = fma2(du, p0, acc[b]);
                            acc[b + 1] = fma2(du, p1, acc[b + 1]);
                        }
                    }
                }
            }
        }
        tc_fence_before();
        return true;
    };

    // One loop over this CTA's global stages; iteration gs stages and issues
    // stage gs, then runs the chain of stage gs - 1 and, after a tile's last
    // stage, its epilogue. Every CTA runs every iteration and every barrier
    // (work is skipped, not the barriers, after an abort or in an empty CTA).
    bool ok = true;  // this thread's chain of the current tile completed
    // producer position (stage sp of local tile tp) and consumer position
    // (stage sc of local tile tc) advance by one stage per iteration
    int sp = 0, sc = 0, tp = 0, tc = 0;
    const int lg_dout = 31 - __clz(p.dout), lg_din = 31 - __clz(p.din);
    // This thread's A group of the next stage to produce (group gk = 2 * s + pg
    // of its row's im2col), loaded one stage ahead so the global-memory latency
    // overlaps the chain and epilogue.
    uint4 pf_words = make_uint4(0u, 0u, 0u, 0u);
    int8_t pf_s = 0;
    bool pf_ok = false;
    // Per producer tile: the group base of the row's input pixel (pointwise) or
    // of the top-left pixel of its 2x2 window; within the tile the im2col
    // position (tap, group g) of group gk = 2 s + pg advances by two groups per
    // stage, so a stage costs one small offset and no division.
    const uint4* pf_base = reinterpret_cast<const uint4*>(p.in);
    const int8_t* pf_sbase = p.in_s;
    bool pf_row_ok = false;
    int pf_tap = 0, pf_g = 0;
    auto start_tile = [&](int t_local) {
        const int64_t row = (tile0 + t_local) * kBM + prow;
        pf_row_ok = live && row < p.rows;
        const int64_t pix0 = KS == 2 ? (pf_row_ok ? tap_pixel_pow2(row, 0, KS, lg_din, lg_dout) : 0) : row;
        pf_base = reinterpret_cast<const uint4*>(p.in) + pix0 * G;
        pf_sbase = p.in_s + pix0 * G;
        pf_tap = 0;
        pf_g = pg;
        while (pf_g >= G) {  // G == 1: group 1 is tap 1
            pf_g -= G;
            ++pf_tap;
        }
    };
    auto prefetch = [&](int s_local) {  // stage s_local of the current producer tile
        pf_ok = pf_row_ok && 2 * s_local + pg < GK;
        if (pf_ok) {
            const int off = (KS == 2 ? (((pf_tap >> 1) << lg_din) + (pf_tap & 1)) * G : 0) + pf_g;
            pf_words = __ldg(pf_base + off);
            pf_s = __ldg(pf_sbase + off);
        }
        pf_g += 2;
        while (pf_g >= G) {
            pf_g -= G;
            ++pf_tap;
        }
    };
    // stage k of the tile's weight image (codes, then the units of its two
    // groups) into slot j, completing on barrier bar (thread 0 only)
    auto fetch_stage = [&](int k, int j, int bar) {
        const uint8_t* img = wimg + static_cast<int64_t>(k) * stage_bytes;
        if (bar >= 0) mbar_expect_tx(smem_addr(&bars[bar]), static_cast<uint32_t>(stage_bytes));
        bulk_g2s(smem_addr(b_codes + j * p.n_max * 128), img, static_cast<uint32_t>(n_cta * 128),
                 smem_addr(&bars[bar < 0 ? 0 : bar]));
        bulk_g2s(smem_addr(b_units + j * 2 * p.n_max), img + n_cta * 128, static_cast<uint32_t>(n_cta * 8),
                 smem_addr(&bars[bar < 0 ? 0 : bar]));
    };
    if (resident && live && tid == 0 && total > 0) {  // every stage once, on barrier 0
        mbar_expect_tx(smem_addr(&bars[0]), static_cast<uint32_t>(S * stage_bytes));
        for (int k = 0; k < S; ++k) fetch_stage(k, k, -1);
    }
    if (total > 0) {
        start_tile(0);
        prefetch(0);
    }
    for (int gs = 0; gs <= total; ++gs) {
        const int buf = gs & 1;
        __syncthreads();  // stage gs-2's chain is done with this buffer's units and accumulators
        const bool run = live && !*abort_flag;
        const bool produce = run && gs < total;
        uint8_t* a_tile = a_tiles + buf * kTileA;
        const uint32_t a_row = smem_addr(a_tile) + static_cast<uint32_t>((prow >> 3) * 1024 + (prow & 7) * 16);
        const int bslot = resident ? sp : buf;
        if (produce) {
            if (tid == 0 && !resident) fetch_stage(sp, buf, buf);
            // interleaved A layout (smem_desc_il); a padding (row, group) is
            // staged from zero words (zero codes) with unit 0
            const float du = pf_ok ? unit_of(pf_s) : 0.0f;
            stage_group_h_il(a_row, pg, pf_ok ? pf_words : make_uint4(0u, 0u, 0u, 0u));
            din_s[(buf * 2 + pg) * kBM + prow] = du;
            fence_async_smem();
            // the stage after this one
            if (gs + 1 < total) {
                if (sp + 1 == S) {
                    start_tile(tp + 1);
                    prefetch(0);
                } else {
                    prefetch(sp + 1);
                }
            }
        }
        tc_fence_before();
        __syncthreads();
        if (produce && tid == 0) {
            const bool ready = resident ? (gs > 0 || mbar_wait(smem_addr(&bars[0]), 0u, p.err, 11))
                                        : mbar_wait(smem_addr(&bars[buf]), static_cast<uint32_t>(gs >> 1) & 1u, p.err, 11);
            if (ready) {
                tc_fence_after();
                // K16 steps advance A (interleaved) by 256 bytes and B (SW128) by
                // 32 bytes: 16 and 2 in the address field
                const uint64_t da = smem_desc_il(smem_addr(a_tile)),
                               db = smem_desc(smem_addr(b_codes + bslot * p.n_max * 128));
                // two K16 MMAs per group; a padding group (odd group count) has no
                // accumulator slot and is skipped
                const int n_mma = 2 * sp + 1 < GK ? kBK / 16 : kBK / 32;
#pragma unroll
                for (int j = 0; j < kBK / 16; ++j)
                    if (j < n_mma)
                        mma_f16(tmem + static_cast<uint32_t>((buf * 2 + (j >> 1)) * n_cta), da + 16 * j, db + 2 * j, idesc,
                                 static_cast<uint32_t>(j & 1));
                mma_commit(smem_addr(&bars[2 + buf]));
            } else {
                *abort_flag = 1;
            }
        }
        if (gs < total && ++sp == S) {
            sp = 0;
            ++tp;
        }
        if (gs == 0) continue;
        const int gc = gs - 1;
        const int sc_now = sc;
        if (++sc == S) sc = 0;
        if (run && ok) {
            if (!chain(gc, sc_now)) {
                ok = false;
                *abort_flag = 1;
            }
        }
        if (sc_now != S - 1) continue;

        // Epilogue of local tile tc: fold the taps, square-sum the 32-channel
        // group, share the sums across the norm chunk, normalise, activate, pack.
        const int64_t tile = tile0 + tc;
        float* part_t = part + (tc & 1) * 8 * kBM;
        ++tc;
        const bool emit = run && ok && has_cols;
        if (kFold) {
#pragma unroll
            for (int i = 0; i < 16; ++i) acc[i] = add2(sacc[kFold ? i : 0], acc[i]);
        }
        if (emit) {
            const float gs2 = tree_sq32x2(acc);
            float* dst = &part_t[(((n0 & (kNormChunk - 1)) >> 5) + hw) * kBM + erow];
            if (CS > 1) {
#pragma unroll
                for (int r = 0; r < CS; ++r) st_peer_f32(smem_addr(dst), static_cast<uint32_t>(r), gs2);
            } else {
                *dst = gs2;
            }
        }
        __syncthreads();
        if (CS > 1) cluster_sync_all();
        if (emit) {
            // the reference's cross-warp butterfly over the chunk's 8 group sums (kernels.h:271-276)
            float w8[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) w8[i] = part_t[i * kBM + erow];
#pragma unroll
            for (int o = 4; o > 0; o >>= 1)
#pragma unroll
                for (int i = 0; i < o; ++i) w8[i] = __fadd_rn(w8[i], w8[i + o]);
            const float sc_norm = __frsqrt_rn(fmaf(w8[0], inv_div, kEps));
            const int64_t row = tile * kBM + erow;
            const float2 sc2 = dup2(sc_norm);
            const float4* b4 = reinterpret_cast<const float4*>(bias_s + 32 * hw);
#pragma unroll
            for (int i4 = 0; i4 < 8; ++i4) {
                const float4 b = b4[i4];
                acc[2 * i4] = fma2(acc[2 * i4], sc2, make_float2(b.x, b.y));
                acc[2 * i4 + 1] = fma2(acc[2 * i4 + 1], sc2, make_float2(b.z, b.w));
                if (ACT) {
                    acc[2 * i4] = silu2(acc[2 * i4]);
                    acc[2 * i4 + 1] = silu2(acc[2 * i4 + 1]);
                }
            }
            uint4 words;
            int8_t e;
            quantize_group2(acc, &words, &e);
            if (row < p.rows) {
                const int64_t gi = row * (p.out_c >> 5) + (n0 >> 5) + hw;
                reinterpret_cast<uint4*>(p.out)[gi] = words;
                p.out_s[gi] = e;
            }
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) acc[i] = dup2(0.0f);
#pragma unroll
        for (int i = 0; i < (kFold ? 16 : 1); ++i) sacc[i] = dup2(0.0f);
    }
    if (live) {
        // every MMA this CTA issued has completed before TMEM is released
        // A timeout here (error 13 recorded) means an MMA has not completed within
        // the wait's limit; one more bounded wait gives it a second window before
        // TMEM is released. The outputs of such a launch are undefined and the host
        // learns of it through the error word.
        if (tid == 0) mma_commit(smem_addr(&bars[4]));
        if (warp == 0 && !mbar_wait(smem_addr(&bars[4]), 0u, p.err, 13)) mbar_wait(smem_addr(&bars[4]), 0u, p.err, 13);
        tc_fence_before();
        __syncthreads();
        if (warp == 0) {
            tc_fence_after();
            tmem_dealloc(tmem, ncols);
        }
    }
}

// ---- chain at the end: pointwise convs with one or two groups -------------
//
// With in_c <= 64 the whole K of a tile is one stage of at most two 32-element
// groups, and every group's dot products stay resident in TMEM (group g in
// slice g). Per row tile the CTA stages A once and issues the MMAs, and the
// epilogue then runs the reference's fmaf chain over the groups one 32-channel
// group of columns at a time, so a thread's chain state is transient: pass 1
// folds the chain, square-sums the group and parks the pre-norm sums back in
// TMEM slice 0; pass 2 normalises, activates and packs. Tiles are 128 rows x
// 128 channels; the two CTAs of a 256-channel RMSNorm chunk form a cluster as
// in the streaming kernel. The weights of the CTA's channels are fetched once
// for its run of up to 8 row tiles. Shared memory holds one A tile and one
// stage of weights (about 45 KB), so with a single group (128 TMEM columns,
// 64 registers per thread) four CTAs share an SM.
constexpr int kCaeW = 128;

template <int CS, bool ACT, bool ONE>
__global__ void __launch_bounds__(kThreads, ONE ? 4 : 2) conv_gemm_tc_cae_kernel(OrdParams p)
{
    constexpr int W = kCaeW, kChunks = W / kNCta;  // 64-channel image chunks per CTA
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);  // stays a shared-space pointer
    const int n0 = static_cast<int>(blockIdx.y / CS) * kNormChunk + static_cast<int>(blockIdx.y % CS) * W;
    const int n_cta = min(W, p.out_c - n0);  // <= 0: a CTA past the end of a narrow chunk
    const bool live = n_cta > 0;
    const int GK = ONE ? 1 : p.gk_total;  // 1 or 2 (a compile-time 1 with one group: 7 % faster; a compile-time 2 measured 3 % slower)
    uint8_t* a_tile = base;                                         // [kTileA]
    uint8_t* b_codes = base + kTileA;                               // [W][128 B]
    float* b_units = reinterpret_cast<float*>(b_codes + W * 128);  // [2][W]
    float* din_s = b_units + 2 * W;                                 // [2][kBM] unit(s_in)
    float* bias_s = din_s + 2 * kBM;                                // [W]
    float* part = bias_s + W;                                       // [2 tiles][8][kBM]
    uint64_t* bars = reinterpret_cast<uint64_t*>(part + 16 * kBM);  // 0: B; 1: accumulators ready
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2);
    int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int need = GK * (n_cta > 0 ? n_cta : 0);
    const uint32_t ncols = need <= 32 ? 32u : need <= 64 ? 64u : need <= 128 ? 128u : 256u;
    for (int i = tid; i < 16 * kBM; i += kThreads) part[i] = 0.0f;
    if (live && tid < n_cta) bias_s[tid] = p.bias[n0 + tid];
    if (tid == 0) {
        for (int i = 0; i < 2; ++i) mbar_init(smem_addr(&bars[i]), 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (live && warp == 0) tmem_alloc(smem_addr(tmem_slot), ncols);
    tc_fence_before();
    __syncthreads();
    if (CS > 1) cluster_sync_all();  // every peer's `part` is initialised before any remote store
    tc_fence_after();
    const uint32_t tmem = live ? *tmem_slot : 0u;

    // The weights, once: per 64-channel chunk the codes, then the units of
    // group 0 and group 1 (image layout of build_wimg_ord_kernel, one stage).
    if (live && tid == 0) {
        mbar_expect_tx(smem_addr(&bars[0]), static_cast<uint32_t>(n_cta * kImgRow));
        for (int c = 0; c < kChunks; ++c) {
            const int cn0 = n0 + c * kNCta;
            const int n_c = min(kNCta, p.out_c - cn0);
            if (n_c <= 0) break;
            const uint8_t* img = p.wimg + static_cast<int64_t>(cn0) * kImgRow;
            bulk_g2s(smem_addr(b_codes + c * kNCta * 128), img, static_cast<uint32_t>(n_c * 128), smem_addr(&bars[0]));
            for (int j = 0; j < 2; ++j)
                bulk_g2s(smem_addr(b_units + j * W + c * kNCta), img + n_c * 128 + j * n_c * 4,
                         static_cast<uint32_t>(n_c * 4), smem_addr(&bars[0]));
        }
    }

    const int prow = tid & (kBM - 1), pg = tid >> 7;
    const uint32_t idesc = instr_desc_h(n_cta > 0 ? n_cta : 32);
    const int q = warp & 3, hw = warp >> 2;
    const int erow = q * 32 + lane;
    const int ngroups = n_cta >> 5;
    const uint32_t tl = tmem + (static_cast<uint32_t>(q * 32) << 16);
    const int gbase = (n0 & (kNormChunk - 1)) >> 5;
    const float inv_div = __frcp_rn(static_cast<float>(min(p.out_c, kNormChunk)));

    // A run of consecutive row tiles per CTA (the same for every CTA of a
    // cluster); each tile's MMAs have completed (the accumulator barrier)
    // before the next tile restages A and reuses TMEM.
    const int64_t n_tiles = (p.rows + kBM - 1) / kBM;
    const int64_t tile0 = static_cast<int64_t>(blockIdx.x) * p.tiles_per_cta;
    const int my_tiles = tile0 < n_tiles ? static_cast<int>(min(static_cast<int64_t>(p.tiles_per_cta), n_tiles - tile0)) : 0;
    // this thread's (row, group) of a tile; with two groups it is loaded one
    // tile ahead so the loads overlap the current tile's MMAs and epilogue
    // (measured: 6 % faster with two groups, 2 % slower with one, where four
    // CTAs per SM already overlap each other's loads)
    uint4 nw = make_uint4(0u, 0u, 0u, 0u);
    int8_t ns = 0;
    auto load_row = [&](int t_local) {
        const int64_t row = (tile0 + t_local) * kBM + prow;
        if (live && pg < GK && t_local < my_tiles && row < p.rows) {
            const int64_t gi = row * GK + pg;  // pointwise: the row's own pixel, group pg
            nw = __ldg(reinterpret_cast<const uint4*>(p.in) + gi);
            ns = __ldg(p.in_s + gi);
        }
    };
    if (!ONE) load_row(0);
    for (int t = 0; t < my_tiles; ++t) {
        const int64_t m0 = (tile0 + t) * kBM;
        const int64_t prow_g = m0 + prow;
        __syncthreads();  // the previous tile's chain has read din_s
        if (ONE) load_row(t);
        if (live && pg < GK && !*abort_flag) {
            // interleaved A layout (smem_desc_il); rows past the end staged as zero codes
            const bool in_rows = prow_g < p.rows;
            const float du = in_rows ? unit_of(ns) : 0.0f;
            stage_group_h_il(smem_addr(a_tile) + static_cast<uint32_t>((prow >> 3) * 1024 + (prow & 7) * 16), pg,
                             in_rows ? nw : make_uint4(0u, 0u, 0u, 0u));
            din_s[pg * kBM + prow] = du;
        }
        if (!ONE) load_row(t + 1);
        fence_async_smem();
        __syncthreads();
        if (live && tid == 0) {
            if (!*abort_flag && (t > 0 || mbar_wait(smem_addr(&bars[0]), 0u, p.err, 22))) {
                tc_fence_after();
                const uint32_t a_addr = smem_addr(a_tile), b_addr = smem_addr(b_codes);
                // two K16 MMAs per group; group 1's half of A is not read with one group
                const int n_mma = GK == 2 ? kBK / 16 : kBK / 32;
#pragma unroll
                for (int j = 0; j < kBK / 16; ++j)
                    if (j < n_mma)
                        mma_f16(tmem + static_cast<uint32_t>((j >> 1) * n_cta), smem_desc_il(a_addr + 256 * j),
                                 smem_desc(b_addr + 32 * j), idesc, static_cast<uint32_t>(j & 1));
            } else {
                *abort_flag = 1;
            }
            mma_commit(smem_addr(&bars[1]));  // arrives once the MMAs (if any) complete
        }
        __syncthreads();
        bool ok = live && !*abort_flag;
        if (live) {
            if (!mbar_wait(smem_addr(&bars[1]), static_cast<uint32_t>(t & 1), p.err, 23)) ok = false;
            tc_fence_after();
        }

        // Pass 1: chain and square-sum per 32-channel group; the pre-norm
        // sums go back to TMEM slice 0.
        float* part_t = part + (t & 1) * 8 * kBM;
        if (ok) {
            for (int cg = hw; cg < ngroups; cg += 2) {
                float2 acc[16];  // channel pairs
#pragma unroll
                for (int i = 0; i < 16; ++i) acc[i] = dup2(0.0f);
                for (int g = 0; g < GK; ++g) {
                    const float2 du = dup2(din_s[g * kBM + erow]);
                    const float4* u4 = reinterpret_cast<const float4*>(b_units + g * W + 32 * cg);
#pragma unroll
                    for (int h16 = 0; h16 < 2; ++h16) {
                        float pv[16];
                        tmem_ld16(tl + static_cast<uint32_t>(g * n_cta + 32 * cg + 16 * h16), pv);
#pragma unroll
                        for (int i4 = 0; i4 < 4; ++i4) {
                            const float4 u = u4[4 * h16 + i4];
                            const int b = 8 * h16 + 2 * i4;
                            acc[b] = fma2(du, mul2(make_float2(u.x, u.y), make_float2(pv[4 * i4], pv[4 * i4 + 1])),
                                                acc[b]);
                            acc[b + 1] = fma2(
                                du, mul2(make_float2(u.z, u.w), make_float2(pv[4 * i4 + 2], pv[4 * i4 + 3])), acc[b + 1]);
                        }
                    }
                }
                const float gs2 = tree_sq32x2(acc);
                float* dst = &part_t[(gbase + cg) * kBM + erow];
                if (CS > 1) {
#pragma unroll
                    for (int r = 0; r < CS; ++r) st_peer_f32(smem_addr(dst), static_cast<uint32_t>(r), gs2);
                } else {
                    *dst = gs2;
                }
                tmem_st32(tl + static_cast<uint32_t>(32 * cg), acc);
            }
        }
        __syncthreads();
        if (CS > 1) cluster_sync_all();
        // Pass 2: the reference's cross-warp butterfly over the chunk's 8 group
        // sums (kernels.h:271-276), then bias, activation and requant.
        if (ok) {
            float w8[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) w8[i] = part_t[i * kBM + erow];
#pragma unroll
            for (int o = 4; o > 0; o >>= 1)
#pragma unroll
                for (int i = 0; i < o; ++i) w8[i] = __fadd_rn(w8[i], w8[i + o]);
            const float sc_norm = __frsqrt_rn(fmaf(w8[0], inv_div, kEps));
            const int64_t row = m0 + erow;
            const float2 sc2 = dup2(sc_norm);
            for (int cg = hw; cg < ngroups; cg += 2) {
                float v[32];
                tmem_ld32(tl + static_cast<uint32_t>(32 * cg), v);
                const float4* b4 = reinterpret_cast<const float4*>(bias_s + 32 * cg);
                float2 x[16];
#pragma unroll
                for (int i4 = 0; i4 < 8; ++i4) {
                    const float4 b = b4[i4];
                    x[2 * i4] = fma2(make_float2(v[4 * i4], v[4 * i4 + 1]), sc2, make_float2(b.x, b.y));
                    x[2 * i4 + 1] = fma2(make_float2(v[4 * i4 + 2], v[4 * i4 + 3]), sc2, make_float2(b.z, b.w));
                    if (ACT) {
                        x[2 * i4] = silu2(x[2 * i4]);
                        x[2 * i4 + 1] = silu2(x[2 * i4 + 1]);
                    }
                }
                uint4 words;
                int8_t e;
                quantize_group2(x, &words, &e);
                if (row < p.rows) {
                    const int64_t gi = row * (p.out_c >> 5) + (n0 >> 5) + cg;
                    reinterpret_cast<uint4*>(p.out)[gi] = words;
                    p.out_s[gi] = e;
                }
            }
        }
        tc_fence_before();  // this tile's TMEM reads precede the next tile's MMAs
    }
    if (live) {
        tc_fence_before();
        __syncthreads();
        if (warp == 0) {
            tc_fence_after();
            tmem_dealloc(tmem, ncols);
        }
    }
}

// ---- warp-specialised streaming kernel ----------------------------------------
//
// The streaming kernel's pipeline with its roles on separate warps and its
// hand-offs on mbarriers instead of CTA-wide barriers. Tiles of ROWS = 128 or
// 256 rows x NC = 64 channels, or 128 rows x NC = 128 channels (WsCfg), with
// C = ROWS * NC / 1024 consumer warps:
// * warps C..C+2 (after setmaxnreg, kStageRegs registers): staging. Thread pt
//   stages rows pt, pt + 96 (and pt + 192) < ROWS of the tile (both groups of
//   a stage, loaded one stage ahead into registers) and records unit(s_in);
//   each warp then arrives on staged[slot].
// * warp C+3 (the same warpgroup): one thread fetches the weight images and
//   issues each staged stage's MMAs (ROWS / 128 M = 128 halves x two groups x
//   two K16 steps, N = NC) into one of two TMEM buffers, committed to
//   full_acc[buf].
//   On its own warp the MMA issue, which waits for the tensor pipe, overlaps
//   the staging of the next stage.
// * warps 0..C-1 (kConsumerRegs registers): consumers. Warp w owns the rows of
//   TMEM lane quarter w & 3 in row half w / (NC / 8) and the 32-channel group
//   (w >> 2) % (NC / 32) of the CTA's channels; it runs the reference's fmaf
//   chain stage by stage from TMEM and, after a tile's last stage, the
//   epilogue. Every consumer thread so owns one row x 32 channels, whatever
//   the shape.
// The weight images of all stages (at most kResidentStages) stay in shared
// memory, fetched once per CTA. Stage slots (A tile halves, unit(s_in)) rotate
// over ws_slots(); a slot is free again once all consumer warps have run the
// chain of the stage it held (empty[slot]), and a TMEM buffer once the chain of
// the stage two before has run (the same barrier). The RMSNorm's per-32-channel sums go
// to the cluster peers through distributed shared memory, after which each
// consumer warp arrives on every peer's part_full[tile & 1] (release/acquire
// at cluster scope): no cluster-wide barrier per tile, so the producers run on.
// TMEM: column (half h, buffer b, group j, channel c) = 4 NC h + 2 NC b + NC j + c.
// With NC = 128 the A tile that the staging warps fill per stage serves twice
// the output channels, and a 256-channel norm chunk needs a cluster of two
// CTAs instead of four; the weights of both 64-channel image chunks are
// fetched side by side, so one N = 128 MMA covers them (the SW128 atoms of
// the second chunk continue those of the first).
constexpr int kWsStageWarps = 3;
constexpr int kWsStageRows = kWsStageWarps * 32;  // 96 staging threads
// Tile shapes: 128 rows x 64 channels (8 consumer warps, 384 threads, two
// CTAs per SM, each with 256 TMEM columns); 256 rows x 64 channels or 128 rows
// x 128 channels (16 consumer warps, 640 threads, one CTA per SM with all 512
// columns). The block launches with kLaunchRegs x kThreads
// registers, exactly the consumers' kConsumerRegs plus the staging/MMA
// warpgroup's kStageRegs (a setmaxnreg.inc that cannot be granted never returns).
template <int ROWS, int NC = kNCta>
struct WsCfg {
    static_assert((ROWS == kBM || ROWS == 2 * kBM) && (NC == kNCta || NC == 2 * kNCta) && ROWS * NC <= 2 * kBM * kNCta,
                  "tile shape");
    static constexpr bool kSmall = ROWS == kBM && NC == kNCta;
    static constexpr int kHalves = ROWS / kBM;
    static constexpr int kGroups = NC / 32;  // 32-channel groups per CTA
    static constexpr int kConsumerWarps = 4 * kGroups * kHalves;
    static constexpr int kThreads = (kConsumerWarps + kWsStageWarps + 1) * 32;
    static constexpr int kTmemCols = 4 * NC * kHalves;
    static constexpr int kRowsPerThread = (ROWS + kWsStageRows - 1) / kWsStageRows;
    static constexpr int kLaunchRegs = kSmall ? 80 : 96;
    static constexpr int kConsumerRegs = kSmall ? 96 : 104;
    static constexpr int kStageRegs = kSmall ? 48 : 64;
    static_assert(kConsumerWarps * 32 * kConsumerRegs + 128 * kStageRegs == kThreads * kLaunchRegs, "register split");
    // the register file admits at most this many CTAs per SM; their TMEM
    // allocations must fit the SM's 512 columns, or an alloc would wait for a
    // CTA that may itself wait on a cluster peer
    static constexpr int kMaxCtasPerSm = 65536 / (kThreads * kLaunchRegs);
    static_assert(kMaxCtasPerSm * kTmemCols <= 512, "TMEM columns per SM");
};
// A-tile slots: 3, or 4 for pointwise convs on 128-channel CTAs (measured 7 %
// faster on the 512 -> 256 layer with 8 stages per tile; equal or slower on
// the 2x2 convs, whose shared memory the fold's shapes need elsewhere)
__host__ __device__ constexpr int ws_slots(int ks, int nc) { return ks == 1 && nc == 128 ? 4 : 3; }
constexpr int kWsMaxStages = 4;  // stages per tile up to which the 64-channel warp-specialised kernel is used
constexpr int kWsCodeSlots = 4;  // ring of weight-code stages when a tile's stages do not all stay resident

// GV: the input's 32-channel groups per tap when known at compile time (0:
// from the arguments); it fixes the stage count and the tap boundaries, so the
// consumers' stage loop unrolls with its folds resolved.
template <int KS, int CS, bool ACT, bool G1, int ROWS, int NC, int GV = 0>
__global__ void __maxnreg__((WsCfg<ROWS, NC>::kLaunchRegs)) conv_gemm_tc_ws_kernel(OrdParams p)
{
    using Cfg = WsCfg<ROWS, NC>;
    constexpr int kWsSlots = ws_slots(KS, NC);
    constexpr int kWsConsumerWarps = Cfg::kConsumerWarps, kWsThreads = Cfg::kThreads, kWsRows = ROWS,
                  kWsRowsPerThread = Cfg::kRowsPerThread, kWsHalves = Cfg::kHalves;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);  // stays a shared-space pointer
    const int n0 = static_cast<int>(blockIdx.y / CS) * kNormChunk + static_cast<int>(blockIdx.y % CS) * NC;
    const int n_cta = min(NC, p.out_c - n0);  // <= 0: a CTA past the end of a narrow chunk (NC = 64 only)
    const bool live = n_cta > 0;
    constexpr int kGkFixed = GV * KS * KS, kStagesFixed = (kGkFixed + 1) / 2;
    const int S = GV ? kStagesFixed : p.stages, GK = GV ? kGkFixed : p.gk_total, G = GV ? GV : p.in_c >> 5;
    // More stages than stay resident (128-channel CTAs only): the weight codes
    // stream through a ring of kWsCodeSlots stages; the units stay resident.
    const bool stream_w = S > kResidentStages;
    const int code_stages = stream_w ? kWsCodeSlots : S;
    uint8_t* a_slots = base;                                                   // [slot][half][kTileA]
    uint8_t* b_codes = a_slots + kWsSlots * kWsHalves * kTileA;                        // [stage or ring slot][n_max][128 B]
    float* b_units = reinterpret_cast<float*>(b_codes + code_stages * p.n_max * 128);  // [stage][2][n_max]
    float* din_s = b_units + S * 2 * p.n_max;                                 // [slot][2 groups][kWsRows]
    float* bias_s = din_s + kWsSlots * 2 * kWsRows;                           // [NC]
    float* part = bias_s + NC;                                                // [2 tiles][8][kWsRows]
    uint64_t* bars = reinterpret_cast<uint64_t*>(part + 2 * 8 * kWsRows);
    uint64_t* full_b = bars;                       // every stage's weights landed
    uint64_t* staged = bars + 1;                   // [slot] the staging warps filled the slot
    uint64_t* empty = staged + kWsSlots;           // [slot] every consumer warp ran the stage's chain
    uint64_t* full_acc = empty + kWsSlots;         // [buf] the stage's MMAs completed
    uint64_t* part_full = full_acc + 2;        // [tile & 1] the chunk's sums of squares arrived
    uint64_t* drain = part_full + 2;
    uint64_t* code_full = drain + 1;               // [ring slot] a stage's codes landed (streamed weights)
    uint64_t* code_free = code_full + kWsCodeSlots;  // [ring slot] the MMAs reading the slot completed
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(code_free + kWsCodeSlots);
    int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    for (int i = tid; i < 2 * 8 * kWsRows; i += kWsThreads) part[i] = 0.0f;
    if (live && tid < n_cta) bias_s[tid] = p.bias[n0 + tid];
    if (tid == 0) {
        mbar_init(smem_addr(&full_b[0]), 1);
        for (int i = 0; i < kWsSlots; ++i) {
            mbar_init(smem_addr(&staged[i]), kWsStageWarps);
            mbar_init(smem_addr(&empty[i]), kWsConsumerWarps);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(smem_addr(&full_acc[i]), 1);
            mbar_init(smem_addr(&part_full[i]), CS * kWsConsumerWarps);
        }
        mbar_init(smem_addr(drain), 1);
        for (int i = 0; i < kWsCodeSlots; ++i) {
            mbar_init(smem_addr(&code_full[i]), 1);
            mbar_init(smem_addr(&code_free[i]), 1);
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (live && warp == 0) tmem_alloc(smem_addr(tmem_slot), Cfg::kTmemCols);
    tc_fence_before();
    __syncthreads();
    if (CS > 1) cluster_sync_all();  // every peer's barriers and `part` are initialised before any remote access
    tc_fence_after();
    const uint32_t tmem = live ? *tmem_slot : 0u;

    const int64_t n_tiles = (p.rows + kWsRows - 1) / kWsRows;
    const int64_t tile0 = static_cast<int64_t>(blockIdx.x) * p.tiles_per_cta;
    const int my_tiles = tile0 < n_tiles ? static_cast<int>(min(static_cast<int64_t>(p.tiles_per_cta), n_tiles - tile0)) : 0;
    const int total = my_tiles * S;
    const int lg_dout = 31 - __clz(p.dout), lg_din = 31 - __clz(p.din);

    if (warp == kWsConsumerWarps + kWsStageWarps) {
        // ------------------------------------------------------------ MMA issuer
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(Cfg::kStageRegs));  // with the staging warps: one warpgroup
        // One thread fetches every
        // stage's weights once, then issues each staged stage's MMAs into the
        // TMEM buffer the consumers freed.
        if (live && lane == 0 && total > 0) {
            const int stage_bytes = n_cta * kImgRow;
            const uint8_t* wimg = p.wimg + static_cast<int64_t>(n0) * S * kImgRow;
            const uint32_t idesc = instr_desc_h(n_cta);
            // streamed codes: stage k's codes of both 64-channel image chunks into
            // ring slot ws, completing on code_full[ws]
            auto fetch_codes = [&](int k, int ws) {
                mbar_expect_tx(smem_addr(&code_full[ws]), static_cast<uint32_t>(n_cta * 128));
                for (int hn = 0; hn < NC / kNCta; ++hn) {
                    const uint8_t* img = p.wimg + static_cast<int64_t>(n0 + hn * kNCta) * S * kImgRow +
                                         static_cast<int64_t>(k) * kNCta * kImgRow;
                    bulk_g2s(smem_addr(b_codes + (ws * p.n_max + hn * kNCta) * 128), img, kNCta * 128u,
                             smem_addr(&code_full[ws]));
                }
            };
            int fills = 0;  // code stages fetched into the ring (streamed weights)
            if (stream_w) {
                // units of every stage once; the first kWsCodeSlots stages' codes
                mbar_expect_tx(smem_addr(&full_b[0]), static_cast<uint32_t>(S * n_cta * 8));
                for (int hn = 0; hn < NC / kNCta; ++hn) {
                    const uint8_t* wimg_h = p.wimg + static_cast<int64_t>(n0 + hn * kNCta) * S * kImgRow;
                    for (int k = 0; k < S; ++k)
#pragma unroll
                        for (int j = 0; j < 2; ++j)
                            bulk_g2s(smem_addr(b_units + (k * 2 + j) * p.n_max + hn * kNCta),
                                     wimg_h + static_cast<int64_t>(k) * kNCta * kImgRow + kNCta * 128 + j * kNCta * 4,
                                     kNCta * 4u, smem_addr(&full_b[0]));
                }
                for (; fills < kWsCodeSlots && fills < total; ++fills) fetch_codes(fills % S, fills);
            } else {  // every stage's codes and units, once
                mbar_expect_tx(smem_addr(&full_b[0]), static_cast<uint32_t>(S * stage_bytes));
                if constexpr (NC == kNCta) {
                    for (int k = 0; k < S; ++k) {
                        const uint8_t* img = wimg + static_cast<int64_t>(k) * stage_bytes;
                        bulk_g2s(smem_addr(b_codes + k * p.n_max * 128), img, static_cast<uint32_t>(n_cta * 128),
                                 smem_addr(&full_b[0]));
                        bulk_g2s(smem_addr(b_units + k * 2 * p.n_max), img + n_cta * 128, static_cast<uint32_t>(n_cta * 8),
                                 smem_addr(&full_b[0]));
                    }
                } else {
                    // the 64-channel image chunks side by side (every chunk of a layer
                    // on this shape is full): codes [stage][NC][128 B], units
                    // [stage][group][NC]
                    for (int hn = 0; hn < NC / kNCta; ++hn) {
                        const uint8_t* wimg_h = p.wimg + static_cast<int64_t>(n0 + hn * kNCta) * S * kImgRow;
                        for (int k = 0; k < S; ++k) {
                            const uint8_t* img = wimg_h + static_cast<int64_t>(k) * kNCta * kImgRow;
                            bulk_g2s(smem_addr(b_codes + (k * p.n_max + hn * kNCta) * 128), img, kNCta * 128u,
                                     smem_addr(&full_b[0]));
#pragma unroll
                            for (int j = 0; j < 2; ++j)
                                bulk_g2s(smem_addr(b_units + (k * 2 + j) * p.n_max + hn * kNCta), img + kNCta * 128 + j * kNCta * 4,
                                         kNCta * 4u, smem_addr(&full_b[0]));
                        }
                    }
                }
            }
            int sp = 0, landed = 0;  // landed: ring fills whose codes were awaited
            for (int gs = 0; gs < total; ++gs) {
                const int slot = gs % kWsSlots, buf = gs & 1, ws = gs % kWsCodeSlots;
                // staged; weights landed; TMEM buffer free once the consumers ran the chain of gs - 2
                bool ok = !*abort_flag &&
                          mbar_wait(smem_addr(&staged[slot]), static_cast<uint32_t>(gs / kWsSlots) & 1u, p.err, 39) &&
                          (gs > 0 || mbar_wait(smem_addr(&full_b[0]), 0u, p.err, 32)) &&
                          (gs < 2 || mbar_wait(smem_addr(&empty[(gs - 2) % kWsSlots]),
                                               static_cast<uint32_t>((gs - 2) / kWsSlots) & 1u, p.err, 33)) &&
                          (!stream_w ||
                           mbar_wait(smem_addr(&code_full[ws]), static_cast<uint32_t>(gs / kWsCodeSlots) & 1u, p.err, 46));
                if (ok && stream_w) landed = gs + 1;
                if (ok) {
                    tc_fence_after();
                    const uint64_t db = smem_desc(smem_addr(b_codes + (stream_w ? ws : sp) * p.n_max * 128));
                    const int n_mma = 2 * sp + 1 < GK ? kBK / 16 : kBK / 32;
#pragma unroll
                    for (int hh = 0; hh < kWsHalves; ++hh) {
                        const uint64_t da = smem_desc_il(smem_addr(a_slots + (slot * kWsHalves + hh) * kTileA));
#pragma unroll
                        for (int j = 0; j < kBK / 16; ++j)
                            if (j < n_mma)
                                mma_f16(tmem + static_cast<uint32_t>(4 * NC * hh + 2 * NC * buf + NC * (j >> 1)),
                                        da + 16 * j, db + 2 * j, idesc, static_cast<uint32_t>(j & 1));
                    }
                    mma_commit(smem_addr(&full_acc[buf]));
                    if (stream_w) mma_commit(smem_addr(&code_free[ws]));  // the slot's MMAs completed
                } else {
                    *abort_flag = 1;
                }
                // streamed codes: once the MMAs of stage gs - 1 completed, its ring slot
                // takes the stage kWsCodeSlots further on
                if (stream_w && ok && gs >= 1 && fills < total) {
                    const int wf = (gs - 1) % kWsCodeSlots;
                    if (mbar_wait(smem_addr(&code_free[wf]), static_cast<uint32_t>((gs - 1) / kWsCodeSlots) & 1u, p.err, 47)) {
                        fetch_codes(fills % S, wf);
                        ++fills;
                    } else {
                        *abort_flag = 1;
                    }
                }
                if (++sp == S) sp = 0;
            }
            // every MMA issued has completed (and the weight copies landed) before TMEM is released
            // (a timeout records 37 / 48 / 34; the drain gets a second bounded window, as above)
            mbar_wait(smem_addr(&full_b[0]), 0u, p.err, 37);
            for (int f = landed; f < fills; ++f)  // ring fills not awaited after an abort
                mbar_wait(smem_addr(&code_full[f % kWsCodeSlots]), static_cast<uint32_t>(f / kWsCodeSlots) & 1u, p.err, 48);
            mma_commit(smem_addr(drain));
            if (!mbar_wait(smem_addr(drain), 0u, p.err, 34)) mbar_wait(smem_addr(drain), 0u, p.err, 34);
        }
    } else if (warp >= kWsConsumerWarps) {
        // ------------------------------------------------------------ staging
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(Cfg::kStageRegs));
        const int pt = tid - kWsConsumerWarps * 32;  // rows pt + kWsStageRows * i of each tile
        const uint32_t a_base = smem_addr(a_slots);
        // this thread's rows: pixel of the row (pointwise) or of the top-left
        // pixel of its 2x2 window, per tile (-1: past the end)
        int pix[kWsRowsPerThread];
        auto start_tile = [&](int t_local) {
#pragma unroll
            for (int i = 0; i < kWsRowsPerThread; ++i) {
                const int rl = pt + kWsStageRows * i;
                const int64_t row = (tile0 + t_local) * kWsRows + rl;
                pix[i] = rl < kWsRows && row < p.rows
                             ? static_cast<int>(KS == 2 ? tap_pixel_pow2(row, 0, KS, lg_din, lg_dout) : row)
                             : -1;
            }
        };
        // im2col position of group gk = 2 sp (j = 0) of the stage being loaded
        int tap0 = 0, g0 = 0;
        uint4 pw[kWsRowsPerThread][2];
        int8_t ps[kWsRowsPerThread][2];
        auto load_stage = [&](int sp) {  // into pw/ps, then advance (tap0, g0) by two groups
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                int tap = tap0, g = g0 + j;
                if (g >= G) {
                    g -= G;
                    ++tap;
                }
                const bool gok = 2 * sp + j < GK;
                const int off = (KS == 2 ? (((tap >> 1) << lg_din) + (tap & 1)) * G : 0) + g;
#pragma unroll
                for (int i = 0; i < kWsRowsPerThread; ++i) {
                    if (gok && pix[i] >= 0) {
                        const int64_t gi = static_cast<int64_t>(pix[i]) * G + off;
                        pw[i][j] = __ldg(reinterpret_cast<const uint4*>(p.in) + gi);
                        ps[i][j] = __ldg(p.in_s + gi);
                    } else {
                        pw[i][j] = make_uint4(0u, 0u, 0u, 0u);
                        ps[i][j] = -128;  // marks a padding (row, group): staged as zeros
                    }
                }
            }
            g0 += 2;
            while (g0 >= G) {
                g0 -= G;
                ++tap0;
            }
        };
        if (live && total > 0) {
            start_tile(0);
            load_stage(0);
        }
        int sp = 0, tp = 0;
        for (int gs = 0; live && gs < total; ++gs) {
            const int slot = gs % kWsSlots;
            bool run = !*abort_flag;
            // the slot is free once the consumers ran the chain of stage gs - kWsSlots
            if (run && gs >= kWsSlots &&
                !mbar_wait(smem_addr(&empty[slot]), static_cast<uint32_t>(gs / kWsSlots - 1) & 1u, p.err, 31)) {
                *abort_flag = 1;
                run = false;
            }
            if (run) {
                const uint32_t slot_base = a_base + static_cast<uint32_t>(slot * kWsHalves * kTileA);
#pragma unroll
                for (int i = 0; i < kWsRowsPerThread; ++i) {
                    const int rl = pt + kWsStageRows * i;
                    if (rl >= kWsRows) break;
                    // the row's place in the interleaved layout of its 128-row half
                    const uint32_t row_base = slot_base + static_cast<uint32_t>((rl >> 7) * kTileA + ((rl & (kBM - 1)) >> 3) * 1024 +
                                                                             (rl & 7) * 16);
#pragma unroll
                    for (int j = 0; j < 2; ++j) {
                        // a padding (row, group) was loaded as zero words: zero codes, unit 0
                        const float du = ps[i][j] != -128 ? unit_of(ps[i][j]) : 0.0f;
                        stage_group_h_il(row_base, j, pw[i][j]);
                        din_s[(slot * 2 + j) * kWsRows + rl] = du;
                    }
                }
                fence_async_smem();  // the tile is read by the MMAs (async proxy)
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_addr(&staged[slot]));  // also after an abort: the MMA thread never waits in vain
            // the next stage's activations, one stage ahead
            if (gs + 1 < total) {
                if (sp + 1 == S) {
                    start_tile(tp + 1);
                    tap0 = 0;
                    g0 = 0;
                    load_stage(0);
                } else {
                    load_stage(sp + 1);
                }
            }
            if (++sp == S) {
                sp = 0;
                ++tp;
            }
        }
    } else {
        // ------------------------------------------------------------ consumers
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(Cfg::kConsumerRegs));
        const int h = warp / (4 * Cfg::kGroups), q = warp & 3, hw = (warp >> 2) % Cfg::kGroups;
        const int erow = q * 32 + lane;    // TMEM lane = row within the half
        const int trow = h * kBM + erow;   // row within the 256-row tile
        // 128-channel CTAs are always full; known at compile time for the tap-fold
        // convs (7-12 % faster), left to the runtime test otherwise (measured 1-2 %
        // faster that way on the pointwise ones)
        const bool has_cols = (NC == 2 * kNCta && KS == 2 && !G1) || hw < (n_cta >> 5);
        const uint32_t tl = tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(4 * NC * h + 32 * hw);
        const float inv_div = __frcp_rn(static_cast<float>(min(p.out_c, kNormChunk)));
        const int gidx = ((n0 & (kNormChunk - 1)) >> 5) + hw;  // this warp's group within the norm chunk
        constexpr bool kFold = KS == 2 && !G1;
        float2 acc[16], sacc[kFold ? 16 : 1];
#pragma unroll
        for (int i = 0; i < 16; ++i) acc[i] = dup2(0.0f);
#pragma unroll
        for (int i = 0; i < (kFold ? 16 : 1); ++i) sacc[i] = dup2(0.0f);
        for (int t = 0; t < my_tiles; ++t) {
            bool ok = !*abort_flag;
            int next_fold = G;  // the group index at which the current tap's chain ends
#pragma unroll(GV ? kStagesFixed : 1)
            for (int sc = 0; sc < S; ++sc) {
                const int gs = t * S + sc, slot = gs % kWsSlots, buf = gs & 1;
                if (live && ok) {
                    if (!mbar_wait(smem_addr(&full_acc[buf]), static_cast<uint32_t>(gs >> 1) & 1u, p.err, 35)) {
                        ok = false;
                        *abort_flag = 1;
                    }
                }
                if (live && ok) {
                    tc_fence_after();
                    const float* units = b_units + sc * 2 * p.n_max + 32 * hw;
                    const float* dins = din_s + slot * 2 * kWsRows + trow;
                    const uint32_t tb = tl + static_cast<uint32_t>(2 * NC * buf);
#pragma unroll
                    for (int j = 0; j < 2; ++j) {
                        const int gk = 2 * sc + j;
                        if (gk >= GK) break;
                        if (kFold && gk == next_fold) {  // a tap's chain ends: fold it, start the next from 0
                            next_fold += G;
#pragma unroll
                            for (int i = 0; i < 16; ++i) {
                                sacc[kFold ? i : 0] = add2(sacc[kFold ? i : 0], acc[i]);
                                acc[i] = dup2(0.0f);
                            }
                        }
                        if (has_cols) {
                            const float2 du = dup2(dins[j * kWsRows]);
                            const float4* u4 = reinterpret_cast<const float4*>(units + j * n_cta);
#pragma unroll
                            for (int h16 = 0; h16 < 2; ++h16) {
                                float pv[16];
                                tmem_ld16(tb + static_cast<uint32_t>(NC * j + 16 * h16), pv);
#pragma unroll
                                for (int i4 = 0; i4 < 4; ++i4) {
                                    const float4 u = u4[4 * h16 + i4];
                                    const int b = 8 * h16 + 2 * i4;
                                    const float2 p0 = mul2(make_float2(u.x, u.y), make_float2(pv[4 * i4], pv[4 * i4 + 1]));
                                    const float2 p1 = mul2(make_float2(u.z, u.w), make_float2(pv[4 * i4 + 2], pv[4 * i4 + 3]));
                                    if (G1) {  // scalar: the product is rounded before the add
                                        acc[b].x = __fadd_rn(acc[b].x, __fmul_rn(du.x, p0.x));
                                        acc[b].y = __fadd_rn(acc[b].y, __fmul_rn(du.y, p0.y));
                                        acc[b + 1].x = __fadd_rn(acc[b + 1].x, __fmul_rn(du.x, p1.x));
                                        acc[b + 1].y = __fadd_rn(acc[b + 1].y, __fmul_rn(du.y, p1.y));
                                    } else {
                                        acc[b] = fma2(du, p0, acc[b]);
                                        acc[b + 1] = fma2(du, p1, acc[b + 1]);
                                    }
                                }
                            }
                        }
                    }
                    tc_fence_before();
                }
                // slot and TMEM buffer may be reused once every consumer warp is here
                __syncwarp();
                if (live && lane == 0) mbar_arrive(smem_addr(&empty[slot]));
            }

            // Epilogue of the tile: fold the taps, square-sum the 32-channel group,
            // share the sums across the norm chunk, normalise, activate, pack.
            float* part_t = part + (t & 1) * 8 * kWsRows;
            const bool emit = live && ok && has_cols;
            if (kFold) {
#pragma unroll
                for (int i = 0; i < 16; ++i) acc[i] = add2(sacc[kFold ? i : 0], acc[i]);
            }
            if (emit) {
                const float gs2 = tree_sq32x2(acc);
                float* dst = &part_t[gidx * kWsRows + trow];
                if (CS > 1) {
#pragma unroll
                    for (int r = 0; r < CS; ++r) st_peer_f32(smem_addr(dst), static_cast<uint32_t>(r), gs2);
                } else {
                    *dst = gs2;
                }
            }
            bool got = true;
            if (CS > 1) {
                asm volatile("fence.acq_rel.cluster;" ::: "memory");
                __syncwarp();
                if (lane == 0) {
#pragma unroll
                    for (int r = 0; r < CS; ++r) mbar_arrive_peer(smem_addr(&part_full[t & 1]), static_cast<uint32_t>(r));
                }
                if (!*abort_flag && !mbar_wait_cluster(smem_addr(&part_full[t & 1]), static_cast<uint32_t>(t >> 1) & 1u, p.err, 36)) {
                    got = false;
                    *abort_flag = 1;
                }
            } else {
                asm volatile("bar.sync 2, %0;" ::"n"(kWsConsumerWarps * 32) : "memory");  // every consumer warp's sums are in `part`
            }
            if (emit && got) {
                // the reference's cross-warp butterfly over the chunk's 8 group sums (kernels.h:271-276)
                float w8[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) w8[i] = part_t[i * kWsRows + trow];
#pragma unroll
                for (int o = 4; o > 0; o >>= 1)
#pragma unroll
                    for (int i = 0; i < o; ++i) w8[i] = __fadd_rn(w8[i], w8[i + o]);
                const float sc_norm = __frsqrt_rn(fmaf(w8[0], inv_div, kEps));
                const int64_t row = (tile0 + t) * kWsRows + trow;
                const float2 sc2 = dup2(sc_norm);
                const float4* b4 = reinterpret_cast<const float4*>(bias_s + 32 * hw);
#pragma unroll
                for (int i4 = 0; i4 < 8; ++i4) {
                    const float4 b = b4[i4];
                    acc[2 * i4] = fma2(acc[2 * i4], sc2, make_float2(b.x, b.y));
                    acc[2 * i4 + 1] = fma2(acc[2 * i4 + 1], sc2, make_float2(b.z, b.w));
                    if (ACT) {
                        acc[2 * i4] = silu2(acc[2 * i4]);
                        acc[2 * i4 + 1] = silu2(acc[2 * i4 + 1]);
                    }
                }
                uint4 words;
                int8_t e;
                quantize_group2(acc, &words, &e);
                if (row < p.rows) {
                    const int64_t gi = row * (p.out_c >> 5) + (n0 >> 5) + hw;
                    reinterpret_cast<uint4*>(p.out)[gi] = words;
                    p.out_s[gi] = e;
                }
            }
#pragma unroll
            for (int i = 0; i < 16; ++i) acc[i] = dup2(0.0f);
#pragma unroll
            for (int i = 0; i < (kFold ? 16 : 1); ++i) sacc[i] = dup2(0.0f);
        }
    }
    // every role is done; no CTA of the cluster leaves while a peer may still
    // write into its shared memory, and TMEM is released after all MMAs completed
    tc_fence_before();
    __syncthreads();
    if (CS > 1) cluster_sync_all();
    if (live && warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, Cfg::kTmemCols);
    }
}

// Per (64-channel chunk, stage) image: the codes of both groups as fp16 in the
// SW128 K-major layout ([n][64] elements, pairs ordered and scaled as
// stage_group_w16 writes them), then unit(s_w) of group 0 and group 1
// ([2][n] fp32). One thread per (output channel, group slot).
__global__ void build_wimg_ord_kernel(const uint32_t* __restrict__ w, const int8_t* __restrict__ w_s, int out_c,
                                      int gk_total, int stages, uint8_t* __restrict__ img)
{
    const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int slots = 2 * stages;
    if (t >= static_cast<int64_t>(out_c) * slots) return;
    const int n = static_cast<int>(t / slots);
    const int gk = static_cast<int>(t % slots);
    const int chunk = n / kNCta, nl = n % kNCta;
    const int n_chunk = min(kNCta, out_c - chunk * kNCta);
    const int s = gk >> 1, gl = gk & 1;
    uint8_t* tile = img + (static_cast<int64_t>(chunk) * kNCta * stages + static_cast<int64_t>(s) * n_chunk) * kImgRow;
    float* units = reinterpret_cast<float*>(tile + n_chunk * 128);
    if (gk < gk_total) {
        const int64_t gi = static_cast<int64_t>(n) * gk_total + gk;
        stage_group_w16(tile, nl, gl, reinterpret_cast<const uint4*>(w)[gi]);
        units[gl * n_chunk + nl] = unit_of(w_s[gi]);
    } else {
        stage_zero(tile, nl, gl);
        units[gl * n_chunk + nl] = 0.0f;
    }
}

// Clusters of CS CTAs along y cover a norm chunk (chunks along y as well);
// along x each CTA column takes tiles_per_cta consecutive row tiles.
template <int KS, int CS>
cudaError_t launch_ord(const OrdParams& p, size_t smem, unsigned chunks, cudaStream_t stream)
{
    auto kern = p.act ? conv_gemm_tc_ord_kernel<KS, CS, true> : conv_gemm_tc_ord_kernel<KS, CS, false>;
    if constexpr (KS == 2) {
        if (p.in_c == 32)  // one group per tap
            kern = p.act ? conv_gemm_tc_ord_kernel<KS, CS, true, true> : conv_gemm_tc_ord_kernel<KS, CS, false, true>;
    }
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = CS;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = CS > 1 ? 1 : 0;
    const int64_t n_tiles = (p.rows + kBM - 1) / kBM;
    cfg.gridDim = dim3(static_cast<unsigned>((n_tiles + p.tiles_per_cta - 1) / p.tiles_per_cta), chunks * CS, 1);
    e = cudaLaunchKernelEx(&cfg, kern, p);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

template <int KS>
cudaError_t launch_ord_cs(const OrdParams& p, size_t smem, cudaStream_t stream)
{
    // CTAs per norm chunk: ceil(min(out_c, 256) / 64) rounded up to 1, 2 or 4
    const int w = p.out_c < kNormChunk ? p.out_c : kNormChunk;
    const int cs = w <= kNCta ? 1 : w <= 2 * kNCta ? 2 : 4;
    const unsigned chunks = static_cast<unsigned>((p.out_c + kNormChunk - 1) / kNormChunk);
    // Tiles per CTA: amortise the per-CTA set-up while keeping >= ~8 CTAs per
    // SM's worth of work in the grid (so the scheduler balances the tail).
    const int64_t n_tiles = (p.rows + kBM - 1) / kBM;
    const int64_t ctas_per_tile_row = static_cast<int64_t>(chunks) * cs;
    int64_t t = n_tiles * ctas_per_tile_row / (148 * 8);
    OrdParams q = p;
    q.tiles_per_cta = static_cast<int>(t < 1 ? 1 : t > 8 ? 8 : t);
    if (cs == 1) return launch_ord<KS, 1>(q, smem, chunks, stream);
    if (cs == 2) return launch_ord<KS, 2>(q, smem, chunks, stream);
    return launch_ord<KS, 4>(q, smem, chunks, stream);
}

template <int KS, int CS, int ROWS, int NC = kNCta, int GV = 0>
cudaError_t launch_ws(const OrdParams& p, unsigned chunks, cudaStream_t stream)
{
    using Cfg = WsCfg<ROWS, NC>;
    if (GV && p.in_c != 32 * GV) return cudaErrorInvalidValue;
    auto kern = p.act ? conv_gemm_tc_ws_kernel<KS, CS, true, false, ROWS, NC, GV>
                      : conv_gemm_tc_ws_kernel<KS, CS, false, false, ROWS, NC, GV>;
    if constexpr (KS == 2 && NC == kNCta) {
        if (p.in_c == 32)  // one group per tap
            kern = p.act ? conv_gemm_tc_ws_kernel<KS, CS, true, true, ROWS, NC, GV>
                         : conv_gemm_tc_ws_kernel<KS, CS, false, true, ROWS, NC, GV>;
    }
    if (NC != kNCta && (p.out_c % NC != 0 || p.n_max != NC || (KS == 2 && p.in_c == 32)))
        return cudaErrorNotSupported;  // 128-channel CTAs: full chunks only, no one-group-per-tap form
    // The role split (setmaxnreg) draws on the block's launch allocation of
    // kLaunchRegs x kThreads; with any other compiled count the increase could
    // never be granted.
    cudaFuncAttributes fa;
    cudaError_t e = cudaFuncGetAttributes(&fa, kern);
    if (e != cudaSuccess) return e;
    if (fa.numRegs != Cfg::kLaunchRegs) return cudaErrorNotSupported;
    // 64-channel CTAs keep every stage's weights resident; 128-channel CTAs
    // stream the codes of longer layers through a ring (the units stay resident)
    const bool stream_w = p.stages > kResidentStages;
    if (stream_w && NC == kNCta) return cudaErrorNotSupported;
    if (p.rows * KS * KS > 0x7FFFFFFFll) return cudaErrorNotSupported;  // input pixel indices are 32-bit
    constexpr int kWsSlots = ws_slots(KS, NC);
    const size_t smem = 1024 + static_cast<size_t>(kWsSlots) * Cfg::kHalves * kTileA +
                        static_cast<size_t>(stream_w ? kWsCodeSlots : p.stages) * p.n_max * 128 +
                        static_cast<size_t>(p.stages) * p.n_max * 8 +
                        (static_cast<size_t>(kWsSlots) * 2 * ROWS + NC + 16 * ROWS) * sizeof(float) +
                        (2 * kWsSlots + 6 + 2 * kWsCodeSlots) * 8 + 16;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return e;
    const int64_t n_tiles = (p.rows + ROWS - 1) / ROWS;
    OrdParams q = p;
    if constexpr (Cfg::kSmall) {
        // Two CTAs per SM (TMEM columns, shared memory); runs of tiles sized
        // for about four CTA runs per SM over the launch.
        const int64_t t = n_tiles * chunks * CS / (148 * 4);
        q.tiles_per_cta = static_cast<int>(t < 1 ? 1 : t > 16 ? 16 : t);
    } else {
        // One CTA per SM: runs of at most 16 tiles, sized so the CTAs fill a
        // whole number of waves over the 148 SMs (a partial last wave of
        // single-CTA SMs idles the rest of the GPU)
        const int64_t per_sm = (n_tiles * chunks * CS + 147) / 148;
        const int64_t waves = (per_sm + 15) / 16;
        const int64_t t = (per_sm + waves - 1) / waves;
        q.tiles_per_cta = static_cast<int>(t < 1 ? 1 : t);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>((n_tiles + q.tiles_per_cta - 1) / q.tiles_per_cta), chunks * CS, 1);
    cfg.blockDim = dim3(Cfg::kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = CS;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = CS > 1 ? 1 : 0;
    e = cudaLaunchKernelEx(&cfg, kern, q);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

template <int KS>
cudaError_t launch_ws_cs(const OrdParams& p, cudaStream_t stream)
{
    const int w = p.out_c < kNormChunk ? p.out_c : kNormChunk;
    const int cs = w <= kNCta ? 1 : w <= 2 * kNCta ? 2 : 4;
    const unsigned chunks = static_cast<unsigned>((p.out_c + kNormChunk - 1) / kNormChunk);
    // 128-row tiles, two CTAs per SM, except where a 2x2 conv folds taps of
    // several groups: the fold's second accumulator set does not fit the
    // 96 consumer registers of that shape (measured 10 % slower), so 256 rows
    if (cs > 2) return cudaErrorNotSupported;  // clusters of 4 take the two-role kernel
    if constexpr (KS == 2) {
        if (p.in_c > 32)
            return cs == 1 ? launch_ws<KS, 1, 2 * kBM>(p, chunks, stream) : launch_ws<KS, 2, 2 * kBM>(p, chunks, stream);
    }
    // the cortex's block-0 layers with their group count fixed at compile time
    if (cs == 1 && p.in_c == (KS == 1 ? 128 : 32)) return launch_ws<KS, 1, kBM, kNCta, KS == 1 ? 4 : 1>(p, chunks, stream);
    return cs == 1 ? launch_ws<KS, 1, kBM>(p, chunks, stream) : launch_ws<KS, 2, kBM>(p, chunks, stream);
}

// 128-row x 128-channel CTAs: one per 128 channels, a cluster of two per
// 256-channel norm chunk.
template <int KS>
cudaError_t launch_ws_wide(const OrdParams& p, cudaStream_t stream)
{
    const unsigned chunks = static_cast<unsigned>((p.out_c + kNormChunk - 1) / kNormChunk);
    constexpr int N = 2 * kNCta;
    const bool pair = p.out_c >= kNormChunk;
    // the cortex's layers with their group count fixed at compile time
    if constexpr (KS == 1) {
        if (p.in_c == 256 && pair) return launch_ws<1, 2, kBM, N, 8>(p, chunks, stream);
        if (p.in_c == 128 && pair) return launch_ws<1, 2, kBM, N, 4>(p, chunks, stream);
        if (p.in_c == 512 && pair) return launch_ws<1, 2, kBM, N, 16>(p, chunks, stream);
    } else {
        if (p.in_c == 64 && !pair) return launch_ws<2, 1, kBM, N, 2>(p, chunks, stream);
        if (p.in_c == 128 && pair) return launch_ws<2, 2, kBM, N, 4>(p, chunks, stream);
    }
    return pair ? launch_ws<KS, 2, kBM, N>(p, chunks, stream) : launch_ws<KS, 1, kBM, N>(p, chunks, stream);
}

}  // namespace

bool conv_tc_ord_supported(int ksize) { return ksize == 1 || ksize == 2; }

size_t conv_tc_ord_wimg_bytes(int in_c, int out_c, int ksize)
{
    const int gk_total = (in_c >> 5) * ksize * ksize;
    const int stages = (gk_total + 1) / 2;
    return static_cast<size_t>(out_c) * stages * kImgRow;
}

cudaError_t launch_build_wimg_ord(const uint32_t* w, const int8_t* w_s, int in_c, int out_c, int ksize, uint8_t* img,
                                  cudaStream_t stream)
{
    const int gk_total = (in_c >> 5) * ksize * ksize;
    const int stages = (gk_total + 1) / 2;
    const int64_t n = static_cast<int64_t>(out_c) * 2 * stages;
    build_wimg_ord_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, stream>>>(w, w_s, out_c, gk_total, stages,
                                                                                     img);
    return cudaGetLastError();
}

template <int CS, bool ONE>
cudaError_t launch_cae(const OrdParams& p, unsigned chunks, cudaStream_t stream)
{
    auto kern = p.act ? conv_gemm_tc_cae_kernel<CS, true, ONE> : conv_gemm_tc_cae_kernel<CS, false, ONE>;
    size_t smem = 1024 + static_cast<size_t>(kTileA) + kCaeW * 128 + 2 * kCaeW * 4 +
                  (2 * kBM + kCaeW + 16 * kBM) * sizeof(float) + 2 * 8 + 8;
    // Never let more CTAs share an SM than its 512 TMEM columns can serve.
    const int need = p.gk_total * (p.out_c < kCaeW ? p.out_c : kCaeW);
    const int tmem_cols = need <= 32 ? 32 : need <= 64 ? 64 : need <= 128 ? 128 : 256;
    const size_t floor_smem = 233472 / (512 / tmem_cols + 1) + 1;
    if (smem < floor_smem) smem = floor_smem;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = CS;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = CS > 1 ? 1 : 0;
    // runs of tiles amortise the weight fetch and set-up (measured on the
    // 32 -> 128 pointwise conv at 2048 x 64 x 64: 1.43 ms with runs of 8,
    // 1.76 ms with one tile per CTA)
    const int64_t n_tiles = (p.rows + kBM - 1) / kBM;
    int64_t t = n_tiles * chunks * CS / (148 * 8);
    OrdParams q = p;
    q.tiles_per_cta = static_cast<int>(t < 1 ? 1 : t > 8 ? 8 : t);
    cfg.gridDim = dim3(static_cast<unsigned>((n_tiles + q.tiles_per_cta - 1) / q.tiles_per_cta), chunks * CS, 1);
    e = cudaLaunchKernelEx(&cfg, kern, q);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

// Chain-at-end dispatch (pointwise, one or two groups): one CTA per 128
// channels, a cluster of two per 256-channel norm chunk.
cudaError_t launch_cae_pw(const OrdParams& p, cudaStream_t stream)
{
    const unsigned chunks = static_cast<unsigned>((p.out_c + kNormChunk - 1) / kNormChunk);
    const bool narrow = p.out_c <= kCaeW;
    if (p.gk_total == 1) return narrow ? launch_cae<1, true>(p, chunks, stream) : launch_cae<2, true>(p, chunks, stream);
    return narrow ? launch_cae<1, false>(p, chunks, stream) : launch_cae<2, false>(p, chunks, stream);
}

cudaError_t launch_conv_gemm_tc_ord(const uint32_t* in, const int8_t* in_s, const uint8_t* wimg, const float* bias,
                                    uint32_t* out, int8_t* out_s, int64_t frames, int in_c, int out_c, int ksize,
                                    int din, int dout, bool act, int* err, cudaStream_t stream)
{
    if (!conv_tc_ord_supported(ksize)) return cudaErrorInvalidValue;
    const int64_t rows = frames * dout * dout;
    if (rows == 0) return cudaSuccess;
    OrdParams p;
    p.in = in; p.in_s = in_s; p.wimg = wimg; p.bias = bias; p.out = out; p.out_s = out_s;
    p.rows = rows; p.in_c = in_c; p.out_c = out_c; p.din = din; p.dout = dout;
    p.gk_total = (in_c >> 5) * ksize * ksize;
    p.stages = (p.gk_total + 1) / 2;
    p.act = act ? 1 : 0;
    p.n_max = out_c < kNCta ? out_c : kNCta;
    p.tiles_per_cta = 1;
    p.err = err;
    const bool one_group_taps = ksize == 2 && in_c == 32;
    // measured: the chain at the end wins with one or two groups per output,
    // the streaming kernel from three on
    if (p.gk_total <= 2)  // only pointwise convs have so few groups (a 2x2 conv has >= 4)
        return launch_cae_pw(p, stream);
    // 128-channel CTAs where the channels come in whole 128-channel CTAs: the
    // staged A tile serves twice the channels, and a 256-channel norm chunk is
    // a cluster of two (weights resident up to kResidentStages stages per tile,
    // the codes of longer layers streamed through a ring)
    if (p.out_c % (2 * kNCta) == 0 && !one_group_taps) {
        OrdParams w = p;
        w.n_max = 2 * kNCta;
        const cudaError_t e = ksize == 1 ? launch_ws_wide<1>(w, stream) : launch_ws_wide<2>(w, stream);
        if (e != cudaErrorNotSupported) return e;
        (void)cudaGetLastError();  // that build is unusable: the kernels below
    }
    // 64-channel CTAs otherwise. Measured: the warp-specialised kernel wins up
    // to four stages per tile and norm clusters of up to two CTAs (two 128-row
    // CTAs per SM: 15-19 % on the block-0 layers of the cortex); on clusters of
    // four it is equal or slower, and longer K needs more resident weights than
    // two CTAs' shared memory holds, so those shapes take the two-role kernel
    const int w_chunk = p.out_c < kNormChunk ? p.out_c : kNormChunk;
    if (p.stages <= kWsMaxStages && w_chunk <= 2 * kNCta) {
        const cudaError_t e = ksize == 1 ? launch_ws_cs<1>(p, stream) : launch_ws_cs<2>(p, stream);
        if (e != cudaErrorNotSupported) return e;
        (void)cudaGetLastError();  // the warp-specialised build is unusable: the two-role kernel below
    }
    const int nb = p.stages <= kResidentStages ? p.stages : 2;  // weight slots (the kernel's `nb`)
    size_t smem = 1024 + 2 * static_cast<size_t>(kTileA) + static_cast<size_t>(nb) * p.n_max * kImgRow +
                  (4 * kBM + kNCta + 16 * kBM) * sizeof(float) + 5 * 8 + 16;
    // Never let more CTAs share an SM than its 512 TMEM columns can serve.
    const int max_ctas = static_cast<int>(512u / ord_tmem_cols(p.n_max, p.stages, p.gk_total));
    const size_t smem_per_sm = 233472;  // 228 KB
    const size_t floor_smem = smem_per_sm / (max_ctas + 1) + 1;
    if (smem < floor_smem) smem = floor_smem;
    return ksize == 1 ? launch_ord_cs<1>(p, smem, stream) : launch_ord_cs<2>(p, smem, stream);
}

}  // namespace aic
