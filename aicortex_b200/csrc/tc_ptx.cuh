// tcgen05 / mbarrier / bulk-copy PTX wrappers and the int4 -> bf16 / fp16
// operand staging shared by the tensor-core conv kernels (k_conv_tc.cu,
// k_conv_tc_ord.cu).
#pragma once
#include <cstdint>
#include <cuda_bf16.h>

#include "aic_common.cuh"

namespace aic {
namespace tc {

constexpr int kBM = 128;                 // pixel rows per tile (= TMEM lanes)
constexpr uint32_t kWaitLimit = 1u << 22;          // mbarrier polls before a wait gives up
constexpr uint64_t kWaitNs = 1000000000ull;         // ... or this many nanoseconds, whichever is first

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

// One poll of the phase with parity `parity`: try_wait may park the thread
// for a system-dependent time until the phase completes (measured 1 % faster
// on the warp-specialised conv than a 20 us suspend hint).
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

__device__ __forceinline__ uint64_t global_ns()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Bounded wait: at most kWaitLimit polls and about kWaitNs nanoseconds;
// returns false (and records `code`) when the phase never completes.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int* err, int code)
{
    if (mbar_try(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (uint32_t i = 0; i < kWaitLimit; ++i) {
        if (mbar_try(bar, parity)) return true;
        if (global_ns() - t0 > kWaitNs) break;
    }
    atomicCAS(err, 0, code);
    return false;
}

// Arrive once on a barrier of this CTA (release at CTA scope).
__device__ __forceinline__ void mbar_arrive(uint32_t bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Arrive once on the barrier at the same offset in cluster CTA `peer`, with
// release at cluster scope (orders this thread's prior distributed-shared
// stores before the peer's acquire).
__device__ __forceinline__ void mbar_arrive_peer(uint32_t local_bar, uint32_t peer)
{
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_bar), "r"(peer));
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(remote) : "memory");
}

// mbar_wait with acquire at cluster scope: after it, stores that cluster peers
// made before their releasing arrive are visible.
__device__ __forceinline__ bool mbar_wait_cluster(uint32_t bar, uint32_t parity, int* err, int code)
{
    const uint64_t t0 = global_ns();
    for (uint32_t i = 0; i < kWaitLimit; ++i) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(bar), "r"(parity)
            : "memory");
        if (ok) return true;
        if (global_ns() - t0 > kWaitNs) break;
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

// K-major operand without swizzle: 8-row x 16-byte core matrices of 128
// contiguous bytes, the next along K at +128 B (leading byte offset), the next
// 8 rows at +1024 B (stride byte offset), so element chunk c (8 fp16) of row r
// sits at (r / 8) * 1024 + c * 128 + (r % 8) * 16 of a 128-row x 64-element
// tile. A K16 step advances the start address by two core matrices (256 B).
__device__ __forceinline__ uint64_t smem_desc_il(uint32_t addr)
{
    uint64_t d = 0;
    d |= static_cast<uint64_t>((addr >> 4) & 0x3FFFu);   // start address
    d |= static_cast<uint64_t>(128u >> 4) << 16;          // leading byte offset: next core matrix along K
    d |= static_cast<uint64_t>(1024u >> 4) << 32;         // stride byte offset: next 8 rows
    d |= static_cast<uint64_t>(1u) << 46;                 // descriptor version (sm_100)
    return d;                                             // layout 0: no swizzle
}

// kind::f16 instruction descriptor: bf16 x bf16 -> f32, both K-major, M = 128.
__host__ __device__ constexpr uint32_t instr_desc(int n)
{
    return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(kBM >> 4) << 24);
}

// The same for fp16 x fp16 -> f32 (the reference-order kernels' operands).
__host__ __device__ constexpr uint32_t instr_desc_h(int n)
{
    return (1u << 4) | (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(kBM >> 4) << 24);
}

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate)
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

// 8 consecutive TMEM columns of this warp's 32 lanes (one row per thread).
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8])
{
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

// 16 consecutive TMEM columns of this warp's 32 lanes (one row per thread).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16])
{
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Stores 32 consecutive TMEM columns of this warp's 32 lanes (one row per thread).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32])
{
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
        "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
        "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
        "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
        "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
        "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
        "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
        "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
        "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
        : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
// tmem_st32 of 32 values held as 16 pairs (value 2i + j in v[i].j)
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float2 (&v)[16])
{
    float f[32];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        f[2 * i] = v[i].x;
        f[2 * i + 1] = v[i].y;
    }
    tmem_st32(taddr, f);
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

// Writes one 32-element group (4 chunks of 16 B) of a K-major SW128 row as the
// bf16 values code * f.
__device__ __forceinline__ void stage_group_f(uint8_t* tile, int row, int group_in_stage, uint4 words, float f)
{
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

// The group scaled by its exponent's factor F(s).
__device__ __forceinline__ void stage_group(uint8_t* tile, int row, int group_in_stage, uint4 words, int8_t s)
{
    stage_group_f(tile, row, group_in_stage, words, stage_factor(s));
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

// ---- int4 -> fp16 staging of the reference-order kernels ------------------------
//
// A word's 8 codes n_0..n_7 become the fp16 pairs (n_0, n_4), (n_1, n_5),
// (n_2, n_6), (n_3, n_7). An even-indexed code is placed at mantissa bit 0 of
// a half with exponent 2^10 (the half 0x6400 | (n ^ 8) is 1032 + q), an
// odd-indexed one at mantissa bit 4 (0x6400 | (n ^ 8) << 4 is 1152 + 16 q): one
// LOP3 per pair and one shift per word; one HADD2 per pair then removes the
// offset exactly, leaving q and 16 q. The weight image holds w at the even
// slots and w / 16 at the odd ones, so every product is q * w exactly, and A
// and B share the K permutation.
__device__ __forceinline__ uint4 unpack_word_h(uint32_t w)
{
    const uint32_t t = w >> 8;
    uint32_t o[4] = {(w & 0x000F000Fu) ^ 0x64086408u, (w & 0x00F000F0u) ^ 0x64806480u, (t & 0x000F000Fu) ^ 0x64086408u,
                     (t & 0x00F000F0u) ^ 0x64806480u};
    const __half2 ce = __halves2half2(__ushort_as_half(0xE408u), __ushort_as_half(0xE408u));  // -1032
    const __half2 co = __halves2half2(__ushort_as_half(0xE480u), __ushort_as_half(0xE480u));  // -1152
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        __half2 v = *reinterpret_cast<__half2*>(&o[j]);
        v = __hadd2(v, (j & 1) ? co : ce);
        o[j] = *reinterpret_cast<uint32_t*>(&v);
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
}

__device__ __forceinline__ uint8_t* sw128_row(uint8_t* tile, int row) { return tile + (row >> 3) * 1024 + (row & 7) * 128; }

// One group into the interleaved (no-swizzle) layout of smem_desc_il: the row's
// chunk c at row_base + c * 128, row_base = (r / 8) * 1024 + (r % 8) * 16.
__device__ __forceinline__ void stage_group_h_il(uint32_t row_base, int group_in_stage, uint4 words)
{
    const uint32_t w[4] = {words.x, words.y, words.z, words.w};
#pragma unroll
    for (int cl = 0; cl < 4; ++cl) {
        const uint4 v = unpack_word_h(w[cl]);
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(row_base + ((group_in_stage * 4 + cl) << 7)),
                     "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                     : "memory");
    }
}

// A weight group for the fp16 operands: w at the even slots, w / 16 at the odd.
__device__ __forceinline__ void stage_group_w16(uint8_t* tile, int row, int group_in_stage, uint4 words)
{
    uint8_t* rowp = sw128_row(tile, row);
    const uint32_t w[4] = {words.x, words.y, words.z, words.w};
#pragma unroll
    for (int cl = 0; cl < 4; ++cl) {
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {  // pair j: codes (j, j + 4), as unpack_word_h orders them
            const float s = (j & 1) ? 0.0625f : 1.0f;
            const __half2 h = __floats2half2_rn(static_cast<float>(code_of(w[cl], j)) * s,
                                                static_cast<float>(code_of(w[cl], j + 4)) * s);
            o[j] = *reinterpret_cast<const uint32_t*>(&h);
        }
        const int chunk = (group_in_stage << 2) + cl;
        *reinterpret_cast<uint4*>(rowp + ((chunk ^ (row & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
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

// tap_pixel for power-of-two dimensions (shifts instead of divisions).
__device__ __forceinline__ int64_t tap_pixel_pow2(int64_t r, int tap, int ksize, int lg_din, int lg_dout)
{
    if (ksize == 1) return r;
    const int64_t frame = r >> (2 * lg_dout);
    const int p = static_cast<int>(r & ((int64_t(1) << (2 * lg_dout)) - 1));
    const int hi = (p >> lg_dout) * ksize + tap / ksize;
    const int wi = (p & ((1 << lg_dout) - 1)) * ksize + tap % ksize;
    return (frame << (2 * lg_din)) + (static_cast<int64_t>(hi) << lg_din) + wi;
}

}  // namespace tc
}  // namespace aic
