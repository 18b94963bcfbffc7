// Blackwell (sm_100a) tensor-core implicit-GEMM convolution.
//
// GEMM view: D[M = batch*Ho*Wo pixels, N = Cout] = A[M, K] * W[N, K]^T with
// K = kh*kw*Cin ordered (tap, channel), cut into 128 x BN output tiles. The kernel
// is persistent (1-4 CTAs per SM as TMEM, registers and shared memory allow; tiles
// taken round-robin) and warp-specialized:
//   * warp 0 / lane 0 issues TMA loads into a ring of `stages` shared-memory slots
//     that runs on across tile boundaries:
//       A: im2col-mode tensor map (3x3 / strided / padded convs: the TMA unit walks
//          128 consecutive output pixels and applies the tap offset, zero-filling
//          padding) or a plain 2-D tiled map (1x1 stride-1 convs, GEMMs);
//       W: 2-D tiled map over the [Cout, K] weight matrix.
//     Each load covers `CH` channels (CH*elem = 32/64/128 bytes, the swizzle width).
//     No load uses cluster multicast.
//   * warp 1 / lane 0 issues tcgen05.mma (kind::f16 for BF16, kind::tf32 for TF32)
//     into one of 1, 2 or 4 TMEM accumulators (128 lanes x BN fp32 columns each),
//     releases ring slots with tcgen05.commit and hands a finished accumulator to the
//     epilogue.
//   * 4 or 8 epilogue warps run the epilogue of tile t while tile t+1 accumulates
//     (with a single accumulator, after it): tcgen05.ld of
//     their 32 TMEM lanes, bias, activation, optional residual add, and a strided
//     store (bf16 or fp32) that can land inside a channel slice of a concat buffer.
// Every mbarrier wait is bounded; on timeout the kernel records an error in the
// device error word, stops issuing work, drains its outstanding copies, frees TMEM
// and exits.
#include <cuda.h>
#include <cstdlib>
#include <cstring>
#include <algorithm>
#include <mutex>

#include "common.h"
#include "device_common.cuh"

namespace pb {

namespace {

constexpr int BM = 128;
constexpr int kMaxBuf = 4;                        // TMEM accumulator buffers at most
constexpr int kMaxHalo = 4;                       // window slots (a_mode 2)
constexpr uint32_t kBarrierBytes = 512;           // mbarriers, TMEM slot, abort flag
// Epilogue warps per CTA: EPI = 4 (one group, one warp per TMEM lane quarter) or 8
// (two groups that split the columns). Threads: producer warp, MMA warp, epilogue.
template <int EPI> constexpr int conv_threads() { return 64 + 32 * EPI; }

// Division by a launch-invariant divisor for n < 2^31: q = (n * m) >> p with
// p = 31 + ceil(log2 d) and m = ceil(2^p / d) (the round-up method of Granlund and
// Montgomery, "Division by invariant integers using multiplication", 1994).
struct FastDiv {
    uint64_t m = 1;
    uint32_t p = 0, d = 1;
};
FastDiv make_fastdiv(uint32_t d) {
    FastDiv f;
    int k = 0;
    while ((1ull << k) < d) ++k;
    f.d = d;
    f.p = 31u + (uint32_t)k;
    f.m = ((1ull << f.p) + d - 1) / d;
    return f;
}
__device__ __forceinline__ uint32_t fdiv(uint32_t n, const FastDiv& f) {
    return (uint32_t)(((uint64_t)n * f.m) >> f.p);
}

// Position in a ring of n slots: slot index and the parity of the pass, advanced
// without division. The pipeline roles are single threads (or one warp) that step
// their rings once per k-block; a 64-bit division by a runtime ring size is a long
// software sequence on the GPU and cost those threads thousands of cycles per tile.
struct RingPos {
    int slot = 0;
    uint32_t phase = 0;     // completed passes & 1
    bool wrapped = false;   // at least one full pass: every slot was used before
    __device__ __forceinline__ void next(int n) {
        if (++slot == n) { slot = 0; phase ^= 1u; wrapped = true; }
    }
};

struct TcParams {
    int64_t M;
    int Ho, Wo;
    int sh, sw, ph, pw, dh, dw, kw;
    int taps, cin_chunks, ch, cin;
    int bn, stages, a_mode, tmem_cols, swb;
    int nbuf;                             // TMEM accumulator buffers (2 or 4), bufcols columns each
    uint32_t bufcols;
    uint32_t idesc;
    uint32_t stage_a_bytes, stage_b_bytes;
    void* out; int out_dt; int64_t out_img, out_sh, out_sw;
    const void* res; int res_dt; int64_t res_img, res_sh, res_sw;
    const float* bias; int act; float slope; int cout;
    int64_t m_tiles; int n_tiles;
    FastDiv div_ntiles, div_hw, div_wo;   // tile -> (m_tile, n_tile), pixel -> (image, row, col)
    // a_mode 2 (halo): stride-1 convs read one zero-padded input window per tile and
    // 64/32/16-channel chunk; tap (r, s) is the window shifted by r*Wp + s rows.
    int Wp, NR, hstages;                  // padded row width, window rows, window slots
    uint32_t Q;                           // output positions per image (Ho * Wp)
    uint32_t halo_bytes, halo_tx;         // window slot stride, bytes one window load brings
    // b_res: the whole weight matrix (every k-block's bn x ch tile, in k-block order)
    // sits in shared memory for the CTA's lifetime, loaded once (n_tiles == 1).
    int b_res;
    uint32_t bres_bytes, btile_bytes;
    FastDiv div_tpi, div_wp;              // tile -> (image, tile in image), position -> (row, col)
    int tma_store;                        // 1: stage output chunks in shared memory, TMA-store them
    uint32_t staging_bytes;               // bn * 128 * out element size (0 without tma_store)
    int* err;
    long long wait_limit;                 // SM cycles a bounded wait on a pipeline barrier may take
    // Narrow tail chunk: Cin = q * ch + tail_ch (tail_ch * elem = 32 bytes) is read as q
    // full chunks and one tail chunk of tail_ch channels with its own 32-byte-swizzle
    // tensor maps (tmA2 / tmB2), instead of a full chunk padded with zeros.
    int tail_ch;
    uint32_t tail_a_bytes, tail_b_bytes;
};

__device__ __forceinline__ uint64_t make_smem_desc(uint32_t addr, int swb) {
    // K-major, swizzled canonical layout: rows of `swb` bytes, 8-row groups `8*swb`
    // bytes apart (SBO), LBO = 16 bytes (unused for swizzled K-major), version 1.
    const uint64_t layout = swb == 128 ? 2ull : (swb == 64 ? 4ull : 6ull);
    uint64_t d = 0;
    d |= (uint64_t)((addr & 0x3FFFF) >> 4);
    d |= (uint64_t)1 << 16;                         // LBO = 16 B
    d |= (uint64_t)((8 * swb) >> 4) << 32;          // SBO
    d |= (uint64_t)1 << 46;                         // descriptor version (sm100)
    d |= layout << 61;
    return d;
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
        : "memory");
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2, int c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], [%2];"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
        : "memory");
}

__device__ __forceinline__ void tma_load_im2col_4d(uint32_t dst, const CUtensorMap* map, uint64_t* bar,
                                                   int c, int w, int h, int n, uint16_t ow, uint16_t oh) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.im2col.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5, %6}], [%2], {%7, %8};"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)),
          "r"(c), "r"(w), "r"(h), "r"(n), "h"(ow), "h"(oh)
        : "memory");
}

// One k-block: ksteps (1, 2 or 4) MMAs over consecutive 32-byte K slices of the A and
// B rows, then a commit of all of them to `bar`, in one branch-free instruction
// sequence (the extra MMAs are predicated off). A branch between a tcgen05.mma and the
// next one costs the issuing thread tens of cycles, so the k-slices are never issued
// from a loop. acc = 0 starts a fresh accumulator with the first slice;
// bar == nullptr issues no commit.
template <int KIND>
__device__ __forceinline__ void umma_kblock(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc,
                                            int ksteps, uint64_t* bar) {
    // a 32-byte step is +2 in the descriptor's 16-byte start-address field
    if (KIND == 0) {
        asm volatile(
            "{\n\t.reg .pred pa, pt, p1, p2, pc;\n\t.reg .b64 a1, b1, a2, b2, a3, b3;\n\t"
            "setp.ne.b32 pa, %4, 0;\n\tsetp.eq.u32 pt, 0, 0;\n\tsetp.ne.b32 pc, %7, 0;\n\t"
            "setp.gt.s32 p1, %5, 1;\n\tsetp.gt.s32 p2, %5, 2;\n\t"
            "add.s64 a1, %1, 2;\n\tadd.s64 b1, %2, 2;\n\tadd.s64 a2, %1, 4;\n\tadd.s64 b2, %2, 4;\n\t"
            "add.s64 a3, %1, 6;\n\tadd.s64 b3, %2, 6;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, pa;\n\t"
            "@p1 tcgen05.mma.cta_group::1.kind::f16 [%0], a1, b1, %3, pt;\n\t"
            "@p2 tcgen05.mma.cta_group::1.kind::f16 [%0], a2, b2, %3, pt;\n\t"
            "@p2 tcgen05.mma.cta_group::1.kind::f16 [%0], a3, b3, %3, pt;\n\t"
            "@pc tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%6];\n\t}"
            ::"r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(acc), "r"(ksteps), "r"(bar ? smem_u32(bar) : 0u),
              "r"(bar ? 1u : 0u)
            : "memory");
    } else {
        asm volatile(
            "{\n\t.reg .pred pa, pt, p1, p2, pc;\n\t.reg .b64 a1, b1, a2, b2, a3, b3;\n\t"
            "setp.ne.b32 pa, %4, 0;\n\tsetp.eq.u32 pt, 0, 0;\n\tsetp.ne.b32 pc, %7, 0;\n\t"
            "setp.gt.s32 p1, %5, 1;\n\tsetp.gt.s32 p2, %5, 2;\n\t"
            "add.s64 a1, %1, 2;\n\tadd.s64 b1, %2, 2;\n\tadd.s64 a2, %1, 4;\n\tadd.s64 b2, %2, 4;\n\t"
            "add.s64 a3, %1, 6;\n\tadd.s64 b3, %2, 6;\n\t"
            "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, pa;\n\t"
            "@p1 tcgen05.mma.cta_group::1.kind::tf32 [%0], a1, b1, %3, pt;\n\t"
            "@p2 tcgen05.mma.cta_group::1.kind::tf32 [%0], a2, b2, %3, pt;\n\t"
            "@p2 tcgen05.mma.cta_group::1.kind::tf32 [%0], a3, b3, %3, pt;\n\t"
            "@pc tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%6];\n\t}"
            ::"r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(acc), "r"(ksteps), "r"(bar ? smem_u32(bar) : 0u),
              "r"(bar ? 1u : 0u)
            : "memory");
    }
}

// The same with exactly KS MMAs (KS = ksteps, a launch constant). A predicated-off
// tcgen05.mma still costs the issuing thread about as much as an issued one (9
// k-blocks of one 32-byte slice: 1574 cycles with three predicated-off MMAs each,
// 658 without, measured on B200), so narrow chunks (KS 1, 2) issue no padding.
template <int KIND, int KS>
__device__ __forceinline__ void umma_kblock_n(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc,
                                              uint64_t* bar) {
    if (KS == 4) {
        umma_kblock<KIND>(tmem_d, da, db, idesc, acc, 4, bar);
    } else if (KS == 2) {
        if (KIND == 0)
            asm volatile(
                "{\n\t.reg .pred pa, pt, pc;\n\t.reg .b64 a1, b1;\n\t"
                "setp.ne.b32 pa, %4, 0;\n\tsetp.eq.u32 pt, 0, 0;\n\tsetp.ne.b32 pc, %6, 0;\n\t"
                "add.s64 a1, %1, 2;\n\tadd.s64 b1, %2, 2;\n\t"
                "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, pa;\n\t"
                "tcgen05.mma.cta_group::1.kind::f16 [%0], a1, b1, %3, pt;\n\t"
                "@pc tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%5];\n\t}"
                ::"r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(acc), "r"(bar ? smem_u32(bar) : 0u),
                  "r"(bar ? 1u : 0u)
                : "memory");
        else
            asm volatile(
                "{\n\t.reg .pred pa, pt, pc;\n\t.reg .b64 a1, b1;\n\t"
                "setp.ne.b32 pa, %4, 0;\n\tsetp.eq.u32 pt, 0, 0;\n\tsetp.ne.b32 pc, %6, 0;\n\t"
                "add.s64 a1, %1, 2;\n\tadd.s64 b1, %2, 2;\n\t"
                "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, pa;\n\t"
                "tcgen05.mma.cta_group::1.kind::tf32 [%0], a1, b1, %3, pt;\n\t"
                "@pc tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%5];\n\t}"
                ::"r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(acc), "r"(bar ? smem_u32(bar) : 0u),
                  "r"(bar ? 1u : 0u)
                : "memory");
    } else {
        if (KIND == 0)
            asm volatile(
                "{\n\t.reg .pred pa, pc;\n\t"
                "setp.ne.b32 pa, %4, 0;\n\tsetp.ne.b32 pc, %6, 0;\n\t"
                "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, pa;\n\t"
                "@pc tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%5];\n\t}"
                ::"r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(acc), "r"(bar ? smem_u32(bar) : 0u),
                  "r"(bar ? 1u : 0u)
                : "memory");
        else
            asm volatile(
                "{\n\t.reg .pred pa, pc;\n\t"
                "setp.ne.b32 pa, %4, 0;\n\tsetp.ne.b32 pc, %6, 0;\n\t"
                "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, pa;\n\t"
                "@pc tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%5];\n\t}"
                ::"r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(acc), "r"(bar ? smem_u32(bar) : 0u),
                  "r"(bar ? 1u : 0u)
                : "memory");
    }
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 ::"r"(smem_u32(bar)) : "memory");
}

// 16 consecutive fp32 columns of this thread's TMEM lane; no wait (tmem_wait_ld).
__device__ __forceinline__ void tmem_ld16_async(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Activation of the tensor-core epilogue. The operands are BF16/TF32, so SiLU and
// sigmoid use the hardware exponential (__expf, ~2 ulp) and a fast divide; the
// reference's Winograd SiLU flavour and the rarer activations keep their exact form.
__device__ __forceinline__ float tanh_approx(float x) {
    float y;
    asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Activation of the tensor-core epilogue. The operands are BF16/TF32 (results are
// held to 1e-2), so SiLU and sigmoid use the hardware tanh (one MUFU op):
// sigmoid(x) = 0.5 + 0.5 tanh(x/2), SiLU(x) = x/2 + x/2 tanh(x/2). The reference's
// Winograd SiLU flavour keeps its steps with an approximate final divide; the rarer
// activations keep their exact form.
template <int ACT>
__device__ __forceinline__ float tc_act(float x, float slope) {
    if (ACT == ACT_NONE) return x;
    if (ACT == ACT_SILU) { const float h = 0.5f * x; return fmaf(h, tanh_approx(h), h); }
    if (ACT == ACT_SIGMOID) return fmaf(0.5f, tanh_approx(0.5f * x), 0.5f);
    if (ACT == ACT_SILU_WINO) return silu_wino_fast(x);
    return apply_act(x, ACT, slope, 0.0f);
}

__device__ __forceinline__ void prefetch_l2(const void* a) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(a));
}

__device__ __forceinline__ void load_res_chunk(const TcParams& p, int64_t rb, uint4 (&r)[4]) {
    const uint4* src = p.res_dt == BF16
        ? reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(p.res) + rb)
        : reinterpret_cast<const uint4*>(reinterpret_cast<const float*>(p.res) + rb);
    r[0] = __ldg(src);
    r[1] = __ldg(src + 1);
    if (p.res_dt != BF16) { r[2] = __ldg(src + 2); r[3] = __ldg(src + 3); }
}

// Epilogue math for one 16-column chunk of one accumulator row: bias, activation,
// residual add (16 contiguous channels of one pixel).
template <int ACT>
__device__ __forceinline__ void epilogue_math(const TcParams& p, float (&v)[16], const uint4 (&r)[4], int ncol) {
    if (p.bias) {
        const float4* b4 = reinterpret_cast<const float4*>(p.bias + ncol);
#pragma unroll
        for (int q = 0; q < 4; ++q) {      // packed fp32x2 adds: one instruction per pair
            const float4 b = __ldg(b4 + q);
            const float2 lo = __fadd2_rn(make_float2(v[4 * q], v[4 * q + 1]), make_float2(b.x, b.y));
            const float2 hi = __fadd2_rn(make_float2(v[4 * q + 2], v[4 * q + 3]), make_float2(b.z, b.w));
            v[4 * q] = lo.x; v[4 * q + 1] = lo.y; v[4 * q + 2] = hi.x; v[4 * q + 3] = hi.y;
        }
    }
    if (ACT == ACT_SILU) {
        // x/2 + x/2 tanh(x/2) with packed multiplies and fused multiply-adds
#pragma unroll
        for (int i = 0; i < 16; i += 2) {
            const float2 h = __fmul2_rn(make_float2(v[i], v[i + 1]), make_float2(0.5f, 0.5f));
            const float2 y = __ffma2_rn(h, make_float2(tanh_approx(h.x), tanh_approx(h.y)), h);
            v[i] = y.x;
            v[i + 1] = y.y;
        }
    } else if (ACT == ACT_SILU_WINO) {
#pragma unroll
        for (int i = 0; i < 16; i += 2) {
            const float2 y = silu_wino_fast2(make_float2(v[i], v[i + 1]));
            v[i] = y.x;
            v[i + 1] = y.y;
        }
    } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = tc_act<ACT>(v[i], p.slope);
    }
    if (p.res) {
        if (p.res_dt == BF16) {
#pragma unroll
            for (int q = 0; q < 2; ++q) {
                const uint32_t w4[4] = {r[q].x, r[q].y, r[q].z, r[q].w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const __nv_bfloat162 h2 = *reinterpret_cast<const __nv_bfloat162*>(&w4[j]);
                    v[q * 8 + 2 * j] += __low2float(h2);
                    v[q * 8 + 2 * j + 1] += __high2float(h2);
                }
            }
        } else {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                v[4 * q] += __uint_as_float(r[q].x); v[4 * q + 1] += __uint_as_float(r[q].y);
                v[4 * q + 2] += __uint_as_float(r[q].z); v[4 * q + 3] += __uint_as_float(r[q].w);
            }
        }
    }
}

__device__ __forceinline__ uint4 pack_bf16x8(const float* v) {
    uint32_t w4[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        __nv_bfloat162 h2 = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
        w4[j] = *reinterpret_cast<uint32_t*>(&h2);
    }
    return make_uint4(w4[0], w4[1], w4[2], w4[3]);
}

// 16 channels of one pixel straight to global memory (views a TMA store cannot take).
__device__ __forceinline__ void store_chunk_global(const TcParams& p, const float (&v)[16], int64_t ob) {
    if (p.out_dt == BF16) {
        uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.out) + ob);
        dst[0] = pack_bf16x8(v);
        dst[1] = pack_bf16x8(v + 8);
    } else {
        float4* dst = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + ob);
#pragma unroll
        for (int q = 0; q < 4; ++q) dst[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    }
}

// 16 channels of accumulator row `row` into the staging block of its chunk, in the
// swizzled layout of the output tensor map (32-byte rows with SWIZZLE_32B for bf16,
// 64-byte rows with SWIZZLE_64B for fp32): the 16-byte piece j of row r sits at
// piece j ^ ((r >> 2) & 1), resp. j ^ ((r >> 1) & 3), so a quarter-warp's stores
// hit distinct banks.
__device__ __forceinline__ void store_chunk_staging(const TcParams& p, const float (&v)[16], uint8_t* blk, int row) {
    if (p.out_dt == BF16) {
        const int sw = (row >> 2) & 1;
        uint4* r = reinterpret_cast<uint4*>(blk + row * 32);
        r[0 ^ sw] = pack_bf16x8(v);
        r[1 ^ sw] = pack_bf16x8(v + 8);
    } else {
        const int sw = (row >> 1) & 3;
        float4* r = reinterpret_cast<float4*>(blk + row * 64);
#pragma unroll
        for (int q = 0; q < 4; ++q) r[q ^ sw] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    }
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int c0, int c1) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];"
                 ::"l"(reinterpret_cast<uint64_t>(map)), "r"(src), "r"(c0), "r"(c1) : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Named barriers 1 and 2 (one per epilogue group of 128 threads); the ids are
// immediates so the kernel reserves only the barriers it uses.
__device__ __forceinline__ void group_bar(int grp) {
    if (grp == 0) asm volatile("bar.sync 1, 128;" ::: "memory");
    else asm volatile("bar.sync 2, 128;" ::: "memory");
}
// Group barrier that also ORs a predicate over the group (every thread gets the result).
__device__ __forceinline__ bool group_bar_or(int grp, bool pred) {
    uint32_t r;
    if (grp == 0)
        asm volatile("{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbarrier.red.or.pred q, 1, 128, p;\n\t"
                     "selp.u32 %0, 1, 0, q;\n\t}" : "=r"(r) : "r"((uint32_t)pred) : "memory");
    else
        asm volatile("{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbarrier.red.or.pred q, 2, 128, p;\n\t"
                     "selp.u32 %0, 1, 0, q;\n\t}" : "=r"(r) : "r"((uint32_t)pred) : "memory");
    return r != 0;
}

// Epilogue warps 2..EPI+1: drain accumulator tiles in the order the MMA warp filled
// them. Warp w reads TMEM lanes 32*(w%4).. (its row quarter); with EPI = 8 the two
// groups of four warps (2-5, 6-9) split the 16-column chunks (group g takes chunks
// g, g+2, ..).
// Addresses come from launch-invariant fast divisions and are computed before the
// accumulator wait, with the first residual chunk; TMEM is read two chunks per
// wait. With tma_store each group stages its chunks in shared memory and one of its
// threads TMA-stores them (full, coalesced rows; the tensor map clips rows past M).
// Hands the accumulator back to the MMA warp once this warp's TMEM loads have landed.
__device__ __forceinline__ void tmem_release(uint64_t* tempty_buf, int lane) {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncwarp();
    if (lane == 0) mbar_arrive(tempty_buf);
}

template <int ACT, int EPI>
__device__ void epilogue_loop(const TcParams& p, const CUtensorMap* tmOut, uint8_t* staging, uint32_t tmem,
                              uint64_t* tfull, uint64_t* tempty, volatile int* abort_flag,
                              int64_t total) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q = warp & 3;               // TMEM lane quarter this warp may access
    constexpr int G = EPI / 4;            // groups
    const int grp = (warp - 2) >> 2;      // 0: warps 2-5, 1: warps 6-9
    const int row = q * 32 + lane;
    const bool leader = (warp & 3) == 2 && lane == 0;   // warp 2 / warp 6, lane 0
    const int nchunks = p.bn >> 4;
    const uint32_t chunk_bytes = p.out_dt == BF16 ? 128u * 32u : 128u * 64u;
    // this thread's output pixel (image b, row ho, column wo) and column base n0 in tile t
    auto locate = [&](int64_t t, uint32_t& mt, int& n0, uint32_t& b, uint32_t& ho, uint32_t& wo) -> bool {
        mt = fdiv((uint32_t)t, p.div_ntiles);
        n0 = (int)((uint32_t)t - mt * (uint32_t)p.n_tiles) * p.bn;
        if (p.a_mode == 2) {
            // row -> padded position P of image b; columns x >= Wo are padding
            b = fdiv(mt, p.div_tpi);
            const uint32_t P = (mt - b * p.div_tpi.d) * (uint32_t)BM + (uint32_t)row;
            ho = fdiv(P, p.div_wp);
            wo = P - ho * p.div_wp.d;
            return P < p.Q && (int)wo < p.Wo;
        }
        const uint32_t m = mt * (uint32_t)BM + (uint32_t)row;
        b = fdiv(m, p.div_hw);
        const uint32_t r = m - b * p.div_hw.d;
        ho = fdiv(r, p.div_wo);
        wo = r - ho * p.div_wo.d;
        return (int64_t)m < p.M;
    };
    RingPos acc;
    for (int64_t t = blockIdx.x; t < total; t += gridDim.x, acc.next(p.nbuf)) {
        const int buf = acc.slot;
        const uint32_t use = acc.phase;                  // parity of this buffer's fills before
        uint32_t mt, b, ho, wo;
        int n0;
        const bool live = locate(t, mt, n0, b, ho, wo);
        int64_t ob = 0, rb = 0;
        if (live) {
            ob = (int64_t)b * p.out_img + (int64_t)ho * p.out_sh + (int64_t)wo * p.out_sw + n0;
            rb = (int64_t)b * p.res_img + (int64_t)ho * p.res_sh + (int64_t)wo * p.res_sw + n0;
        }
        // The residual loads below run just before the accumulator wait, so a tile whose
        // accumulator is ready waits for them: bring this thread's residual pixel of its
        // next tile into L2 now, a tile ahead.
        if (p.res && t + gridDim.x < total) {
            uint32_t mt2, b2, ho2, wo2;
            int n2;
            if (locate(t + gridDim.x, mt2, n2, b2, ho2, wo2)) {
                const int64_t rb2 = (int64_t)b2 * p.res_img + (int64_t)ho2 * p.res_sh + (int64_t)wo2 * p.res_sw + n2;
                const char* a = static_cast<const char*>(p.res) + rb2 * (p.res_dt == BF16 ? 2 : 4);
                const int bytes = p.bn * (p.res_dt == BF16 ? 2 : 4);
                for (int o = 0; o < bytes; o += 128) prefetch_l2(a + o);
            }
        }
        uint4 rn[4] = {};
        if (p.res && live && grp < nchunks) load_res_chunk(p, rb + 16 * grp, rn);
        bool ok = mbar_wait_bounded(&tfull[buf], use & 1u, p.wait_limit);
        ok = __all_sync(0xffffffffu, ok);
        if (p.tma_store) {
            // One decision for the whole group (its warps meet at named barriers, so
            // none may leave alone); the barrier also gates the staging writes on the
            // previous tile's stores having read it.
            if (leader) bulk_wait_read0();
            if (group_bar_or(grp, !ok || *abort_flag != 0)) {
                if (!ok && lane == 0) { atomicExch(p.err, 3); *abort_flag = 1; }
                break;
            }
        } else if (!ok) {
            if (lane == 0) { atomicExch(p.err, 3); *abort_flag = 1; }
            break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)buf * p.bufcols;
        // EPI = 4 hands the accumulator back to the MMA warp as soon as this warp's last
        // TMEM load has landed, before that chunk's math and stores: the next tile's
        // MMAs then wait for the loads only (3x3 64 -> 80 at 80x80 -9%, 64 -> 64 -4%).
        if (EPI == 8) {
            // two chunks per TMEM wait
            for (int c = grp; c < nchunks; c += 2 * G) {
                const bool two = c + G < nchunks;
                uint32_t r0[16], r1[16];
                tmem_ld16_async(tbase + (uint32_t)(16 * c), r0);
                if (two) tmem_ld16_async(tbase + (uint32_t)(16 * (c + G)), r1);
                tmem_wait_ld();
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    if (h == 1 && !two) break;
                    const int cc = c + G * h;           // chunk index
                    const uint4 rc[4] = {rn[0], rn[1], rn[2], rn[3]};
                    if (p.res && live && cc + G < nchunks) load_res_chunk(p, rb + 16 * (cc + G), rn);
                    float v[16];
#pragma unroll
                    for (int k = 0; k < 16; ++k) v[k] = __uint_as_float(h ? r1[k] : r0[k]);
                    epilogue_math<ACT>(p, v, rc, n0 + 16 * cc);
                    if (p.tma_store) store_chunk_staging(p, v, staging + cc * chunk_bytes, row);
                    else if (live) store_chunk_global(p, v, ob + 16 * cc);
                }
            }
        } else {
            // one chunk per TMEM wait (EPI = 4: fewer registers, so four CTAs fit per SM);
            // the last chunk is peeled so the release sits outside the loop
            auto chunk = [&](int cc, bool last) {
                uint32_t r0[16];
                tmem_ld16_async(tbase + (uint32_t)(16 * cc), r0);
                tmem_wait_ld();
                if (last) tmem_release(tempty + buf, lane);
                float v[16];
#pragma unroll
                for (int k = 0; k < 16; ++k) v[k] = __uint_as_float(r0[k]);
                const uint4 rc[4] = {rn[0], rn[1], rn[2], rn[3]};
                if (p.res && live && cc + G < nchunks) load_res_chunk(p, rb + 16 * (cc + G), rn);
                epilogue_math<ACT>(p, v, rc, n0 + 16 * cc);
                if (p.tma_store) store_chunk_staging(p, v, staging + cc * chunk_bytes, row);
                else if (live) store_chunk_global(p, v, ob + 16 * cc);
            };
            int cc = grp;
            for (; cc + G < nchunks; cc += G) chunk(cc, false);
            if (cc < nchunks) chunk(cc, true);
        }
        // EPI = 8 releases after its loop (an earlier release there cost the 1x1 convs
        // 5-12% in register spills); a group without columns releases here too
        if (EPI == 8 || grp >= nchunks) tmem_release(tempty + buf, lane);
        if (p.tma_store) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            group_bar(grp);
            if (leader) {
                for (int c = grp; c < nchunks; c += G)
                    tma_store_2d(tmOut, smem_u32(staging + c * chunk_bytes), n0 + 16 * c, (int)(mt * BM));
                bulk_commit();
            }
        } else if (__any_sync(0xffffffffu, *abort_flag != 0)) {
            break;
        }
    }
    if (p.tma_store && leader) bulk_wait0();
}

struct MmaSmem {
    uint32_t ring, halo, bres, a_bytes, b_bytes;
    int S, HS;
    uint64_t *full, *empty, *tfull, *tempty, *hfull, *hempty, *bres_full, *mma_done;
    uint32_t tmem;
};

// MMA issuer (one thread). Every branch this thread takes while MMAs are in flight
// costs it tens of cycles, so the operand mode is a template parameter and the tap
// and chunk loops carry no per-k-block mode tests. WIN: a_mode 2 (windows; taps are
// shifted windows); otherwise A comes from the ring (im2col or 2-D tiles). BRES:
// weights resident in shared memory instead of streamed through the ring. KS: MMAs
// per k-block (swb / 32).
template <int KIND, int WIN, bool BRES, int KS>
__device__ __forceinline__ void mma_issuer(const TcParams& p, const MmaSmem& m, volatile int* abort_flag, int64_t total) {
    const int taps = p.taps, chunks = p.cin_chunks, kw = p.kw;
    const uint64_t bdesc0 = make_smem_desc(m.bres, p.swb);
    const uint32_t bstep = (p.btile_bytes >> 4);          // descriptor units per resident k-block
    const int rows = taps / kw;
    RingPos ring, win, acc;                               // operand ring, window slots, accumulators
    if (BRES && blockIdx.x < total && !mbar_wait_bounded(m.bres_full, 0, p.wait_limit)) {
        atomicExch(p.err, 2);
        *abort_flag = 1;
    }
    for (int64_t t = blockIdx.x; t < total && !*abort_flag; t += gridDim.x, acc.next(p.nbuf)) {
        const int buf = acc.slot;
        if (acc.wrapped && !mbar_wait_bounded(&m.tempty[buf], acc.phase ^ 1u, p.wait_limit)) {
            atomicExch(p.err, 5);
            *abort_flag = 1;
            break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t d = m.tmem + (uint32_t)buf * p.bufcols;
        bool ok = true;
        if (WIN == 2) {
            const uint32_t mt = fdiv((uint32_t)t, p.div_ntiles);
            const uint32_t b = fdiv(mt, p.div_tpi);
            const uint32_t P0 = (mt - b * p.div_tpi.d) * (uint32_t)BM;
            const uint32_t off0 = P0 - fdiv(P0, p.div_wp) * p.div_wp.d;
            for (int cc = 0; cc < chunks && ok; ++cc) {
                const int hs = win.slot;
                if (!mbar_wait_bounded(&m.hfull[hs], win.phase, p.wait_limit)) { ok = false; break; }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint64_t adesc0 = make_smem_desc(m.halo + (uint32_t)hs * p.halo_bytes + off0 * (uint32_t)p.swb, p.swb);
                for (int r = 0, tap = 0; r < rows; ++r) {
                    for (int s2 = 0; s2 < kw; ++s2, ++tap) {
                        const uint64_t da = adesc0 + ((uint64_t)((uint32_t)(r * p.Wp + s2) * (uint32_t)p.swb) >> 4);
                        uint64_t db;
                        uint64_t* release = nullptr;
                        if (BRES) {
                            db = bdesc0 + (uint64_t)(cc * taps + tap) * bstep;
                        } else {
                            const int st = ring.slot;
                            if (!mbar_wait_bounded(&m.full[st], ring.phase, p.wait_limit)) { ok = false; break; }
                            ring.next(m.S);
                            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                            db = make_smem_desc(m.ring + (uint32_t)m.S * m.a_bytes + (uint32_t)st * m.b_bytes, p.swb);
                            release = &m.empty[st];
                        }
                        umma_kblock_n<KIND, KS>(d, da, db, p.idesc, (cc | tap) != 0, release);
                    }
                    if (!ok) break;
                }
                if (!ok) break;
                umma_commit(&m.hempty[hs]);
                win.next(m.HS);
            }
        } else {
            for (int tap = 0; tap < taps && ok; ++tap) {
                for (int cc = 0; cc < chunks; ++cc) {
                    const int st = ring.slot;
                    if (!mbar_wait_bounded(&m.full[st], ring.phase, p.wait_limit)) { ok = false; break; }
                    ring.next(m.S);
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    // the tail chunk (if any) has 32-byte rows: its own swizzle, one K slice
                    const bool tail = p.tail_ch && cc == chunks - 1;
                    const int swbk = tail ? 32 : p.swb;
                    const uint64_t da = make_smem_desc(m.ring + (uint32_t)st * m.a_bytes, swbk);
                    const uint64_t db = BRES ? bdesc0 + (uint64_t)(tap * chunks + cc) * bstep
                                             : make_smem_desc(m.ring + (uint32_t)m.S * m.a_bytes + (uint32_t)st * m.b_bytes, swbk);
                    if (KS == 4) umma_kblock<KIND>(d, da, db, p.idesc, (tap | cc) != 0, tail ? 1 : 4, &m.empty[st]);
                    else umma_kblock_n<KIND, KS>(d, da, db, p.idesc, (tap | cc) != 0, &m.empty[st]);
                }
            }
        }
        if (!ok) { atomicExch(p.err, 2); *abort_flag = 1; break; }
        umma_commit(&m.tfull[buf]);
    }
    umma_commit(m.mma_done);
}

template <int KIND, int KS>
__device__ __forceinline__ void mma_issuer_ks(const TcParams& p, const MmaSmem& m, volatile int* abort_flag,
                                              int64_t total) {
    if (p.a_mode == 2) {
        if (p.b_res) mma_issuer<KIND, 2, true, KS>(p, m, abort_flag, total);
        else mma_issuer<KIND, 2, false, KS>(p, m, abort_flag, total);
    } else {
        if (p.b_res) mma_issuer<KIND, 0, true, KS>(p, m, abort_flag, total);
        else mma_issuer<KIND, 0, false, KS>(p, m, abort_flag, total);
    }
}

// Persistent, warp-specialized kernel. 64 + 32*EPI threads:
//   warp 0  (lane 0): TMA producer, streams (tile, k-block) loads through the ring
//                     without stopping at tile boundaries;
//   warp 1  (lane 0): MMA issuer; owns two TMEM accumulators and alternates between
//                     them, so tile t+1 accumulates while tile t is drained;
//   warps 2..EPI+1:   epilogue (see epilogue_loop).
// Tiles are taken round-robin (tile = blockIdx.x + i*gridDim.x), N-tiles innermost
// so CTAs working on the same pixel rows run close together (A re-reads hit L2).
// MINB: resident CTAs per SM the launch plans for (the register budget per thread is
// 64K / (threads * MINB)); a launch with fewer CTAs per SM uses the variant with the
// larger budget, so the epilogue does not spill.
template <int KIND, int EPI, int MINB>
__global__ void __launch_bounds__(conv_threads<EPI>(), MINB)
conv_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               const __grid_constant__ CUtensorMap tmOut, const __grid_constant__ CUtensorMap tmA2,
               const __grid_constant__ CUtensorMap tmB2, const TcParams p) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t* const smem = smem_raw + (base - raw);
    const int S = p.stages;
    const uint32_t a_bytes = p.stage_a_bytes, b_bytes = p.stage_b_bytes;
    // [output staging | window slots | resident weights | A slots | B slots | barriers],
    // 1024-aligned parts
    uint8_t* const staging = smem;
    const int HS = p.hstages;
    const uint32_t halo = base + p.staging_bytes;
    const uint32_t bres = halo + (uint32_t)HS * p.halo_bytes;
    const uint32_t ring = bres + p.bres_bytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + (ring - base) + (size_t)S * (a_bytes + b_bytes));
    uint64_t* empty = full + S;
    uint64_t* tfull = empty + S;          // [kMaxBuf] MMA -> epilogue
    uint64_t* tempty = tfull + kMaxBuf;   // [kMaxBuf] epilogue -> MMA
    uint64_t* mma_done = tempty + kMaxBuf;  // all issued MMAs finished (before TMEM is freed)
    uint64_t* hfull = mma_done + 1;       // [kMaxHalo] window landed
    uint64_t* hempty = hfull + kMaxHalo;  // [kMaxHalo] window consumed
    uint64_t* bres_full = hempty + kMaxHalo;  // resident weights landed
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bres_full + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nk = p.taps * p.cin_chunks;
    const int64_t total = p.m_tiles * (int64_t)p.n_tiles;

    // A CTA that starts after another one recorded a timeout does no work at all.
    if (threadIdx.x == 0) *abort_flag = *reinterpret_cast<volatile int*>(p.err) != 0;
    __syncthreads();
    if (*abort_flag) return;
    __syncthreads();

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) { mbar_init(&full[i], 1); mbar_init(&empty[i], 1); }
        for (int i = 0; i < p.nbuf; ++i) { mbar_init(&tfull[i], 1); mbar_init(&tempty[i], EPI); }
        mbar_init(mma_done, 1);
        mbar_init(bres_full, 1);
        for (int i = 0; i < HS; ++i) { mbar_init(&hfull[i], 1); mbar_init(&hempty[i], 1); }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32(tmem_slot)), "r"(p.tmem_cols) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            int64_t it = 0;   // global ring counter across tiles
            int64_t hit = 0;  // global window counter (a_mode 2)
            RingPos rp, wp;   // the same as ring / window slot positions
            const bool ring_used = S > 0;     // no ring: windows + resident weights only
            if (p.b_res && blockIdx.x < total) {
                mbar_expect_tx(bres_full, p.bres_bytes);
                for (int kb = 0; kb < nk; ++kb) {
                    int tap, cc;
                    if (p.a_mode == 2) { cc = kb / p.taps; tap = kb - cc * p.taps; }
                    else { tap = kb / p.cin_chunks; cc = kb - tap * p.cin_chunks; }
                    tma_load_3d(bres + (uint32_t)kb * p.btile_bytes, &tmB, bres_full, cc * p.ch, tap, 0);
                }
            }
            for (int64_t t = blockIdx.x; t < total && !*abort_flag; t += gridDim.x) {
                const uint32_t mt = fdiv((uint32_t)t, p.div_ntiles);
                const int n0 = (int)((uint32_t)t - mt * (uint32_t)p.n_tiles) * p.bn;
                const uint32_t m0 = mt * (uint32_t)BM;
                uint32_t b = 0; int ho = 0, wo = 0;
                if (p.a_mode == 0) {
                    b = fdiv(m0, p.div_hw);
                    const uint32_t r = m0 - b * p.div_hw.d;
                    ho = (int)fdiv(r, p.div_wo);
                    wo = (int)(r - (uint32_t)ho * p.div_wo.d);
                } else if (p.a_mode == 2) {
                    b = fdiv(mt, p.div_tpi);
                    const uint32_t P0 = (mt - b * p.div_tpi.d) * (uint32_t)BM;
                    ho = (int)fdiv(P0, p.div_wp);     // first window row (output row of P0)
                }
                bool stop = false;
                // k-block coordinates, stepped in k order: windows run through the taps
                // of one channel chunk, the ring through the chunks of one tap (r, s)
                int tap = 0, cc = 0, r = 0, s = 0;
                for (int kb = 0; kb < nk && !stop; ++kb) {
                    if (p.a_mode == 2 && tap == 0) {
                        const int hs = wp.slot;
                        if (wp.wrapped && !mbar_wait_bounded(&hempty[hs], wp.phase ^ 1u, p.wait_limit)) {
                            atomicExch(p.err, 7);
                            *abort_flag = 1;
                            stop = true;
                            break;
                        }
                        mbar_expect_tx(&hfull[hs], p.halo_tx);
                        tma_load_4d(halo + (uint32_t)hs * p.halo_bytes, &tmA, &hfull[hs], cc * p.ch, -p.pw,
                                    ho - p.ph, (int)b);
                        wp.next(HS);
                        ++hit;
                    }
                    if (ring_used) {
                        const int st = rp.slot;
                        if (rp.wrapped && !mbar_wait_bounded(&empty[st], rp.phase ^ 1u, p.wait_limit)) {
                            atomicExch(p.err, 1);
                            *abort_flag = 1;
                            break;
                        }
                        const uint32_t sa = ring + (uint32_t)st * a_bytes;
                        const uint32_t sb = ring + (uint32_t)S * a_bytes + (uint32_t)st * b_bytes;
                        rp.next(S);
                        ++it;
                        const bool tail = p.tail_ch && cc == p.cin_chunks - 1;
                        mbar_expect_tx(&full[st], tail ? p.tail_a_bytes + (p.b_res ? 0u : p.tail_b_bytes) : a_bytes + b_bytes);
                        const CUtensorMap* mA = tail ? &tmA2 : &tmA;
                        if (p.a_mode == 0) {
                            tma_load_im2col_4d(sa, mA, &full[st], cc * p.ch, wo * p.sw - p.pw, ho * p.sh - p.ph,
                                               (int)b, (uint16_t)(s * p.dw), (uint16_t)(r * p.dh));
                        } else if (p.a_mode == 1) {
                            tma_load_2d(sa, mA, &full[st], cc * p.ch, (int)m0);
                        }
                        if (!p.b_res) tma_load_3d(sb, tail ? &tmB2 : &tmB, &full[st], cc * p.ch, tap, n0);
                    }
                    if (p.a_mode == 2) {
                        if (++tap == p.taps) { tap = 0; ++cc; }
                    } else if (++cc == p.cin_chunks) {
                        cc = 0;
                        ++tap;
                        if (++s == p.kw) { s = 0; ++r; }
                    }
                }
            }
            // Drain: the last use of every slot must have landed before the CTA exits.
            for (int64_t k = it > S ? it - S : 0; k < it; ++k)
                if (!mbar_wait_bounded(&full[k % S], (uint32_t)((k / S) & 1))) atomicExch(p.err, 4);
            if (p.b_res && blockIdx.x < total && !mbar_wait_bounded(bres_full, 0)) atomicExch(p.err, 4);
            for (int64_t k = hit > HS ? hit - HS : 0; k < hit; ++k)
                if (!mbar_wait_bounded(&hfull[k % HS], (uint32_t)((k / HS) & 1))) atomicExch(p.err, 4);
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            MmaSmem m{ring, halo, bres, a_bytes, b_bytes, S, HS, full, empty, tfull, tempty, hfull, hempty, bres_full,
                      mma_done, tmem};
            if (p.swb == 32) mma_issuer_ks<KIND, 1>(p, m, abort_flag, total);
            else if (p.swb == 64) mma_issuer_ks<KIND, 2>(p, m, abort_flag, total);
            else mma_issuer_ks<KIND, 4>(p, m, abort_flag, total);
        }
        __syncwarp();
    } else {
        // ---------------- epilogue (warps 2..EPI+1) ----------------
        switch (p.act) {
            case ACT_NONE: epilogue_loop<ACT_NONE, EPI>(p, &tmOut, staging, tmem, tfull, tempty, abort_flag, total); break;
            case ACT_SILU: epilogue_loop<ACT_SILU, EPI>(p, &tmOut, staging, tmem, tfull, tempty, abort_flag, total); break;
            case ACT_SILU_WINO: epilogue_loop<ACT_SILU_WINO, EPI>(p, &tmOut, staging, tmem, tfull, tempty, abort_flag, total); break;
            case ACT_RELU: epilogue_loop<ACT_RELU, EPI>(p, &tmOut, staging, tmem, tfull, tempty, abort_flag, total); break;
            case ACT_LEAKY: epilogue_loop<ACT_LEAKY, EPI>(p, &tmOut, staging, tmem, tfull, tempty, abort_flag, total); break;
            case ACT_SIGMOID: epilogue_loop<ACT_SIGMOID, EPI>(p, &tmOut, staging, tmem, tfull, tempty, abort_flag, total); break;
            default: epilogue_loop<ACT_GELU_TANH, EPI>(p, &tmOut, staging, tmem, tfull, tempty, abort_flag, total); break;  // host-checked
        }
    }

    // Free TMEM only after every issued MMA has completed.
    __syncthreads();
    if (warp == 1) {
        if (!mbar_wait_bounded(mma_done, 0) && lane == 0) atomicExch(p.err, 6);
        __syncwarp();
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(p.tmem_cols) : "memory");
    }
}

// ---------------------------------------------------------------------------
// Host side: tensor-map encoding through the driver entry points.
// ---------------------------------------------------------------------------
typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
typedef CUresult (*PFN_encodeIm2col)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                     const cuuint64_t*, const int*, const int*, cuuint32_t, cuuint32_t,
                                     const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                     CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

PFN_encodeTiled g_tiled = nullptr;
PFN_encodeIm2col g_im2col = nullptr;
std::once_flag g_once;

void load_driver_fns() {
    std::call_once(g_once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_tiled = reinterpret_cast<PFN_encodeTiled>(f);
        f = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeIm2col", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_im2col = reinterpret_cast<PFN_encodeIm2col>(f);
    });
    if (!g_tiled || !g_im2col) fail(ENGINE_ERR_RUNTIME, "CUDA driver lacks tensor-map encoding entry points");
}

CUtensorMapSwizzle swizzle_of(int swb) {
    return swb == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : (swb == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B);
}

// Channels per k-block (one swizzled smem row of 128, 64 or 32 bytes). The largest
// row that divides Cin, except that Cin with only 32-byte rows and more than 64
// bytes per pixel (Cin = 48, 80, 112 ... in bf16) takes 128-byte rows with a zero
// padded last chunk: on B200 a k-block costs about the same whatever its row width,
// so 80 -> 80 3x3 at 80x80 runs 1.85x faster in two 64-channel chunks (of which 48
// channels read as zeros) than in five 16-channel ones (swept per layer).
int pick_chunk(int cin, int esz) {
    const int c128 = 128 / esz, c64 = 64 / esz, c32 = 32 / esz;
    if (cin % c128 == 0) return c128;
    if (cin % c64 == 0) return c64;
    if (cin % c32 == 0) return cin * esz > 64 ? c128 : c32;
    return 0;
}

int pick_bn(int cout) {
    if (cout % 16) return 0;
    if (cout <= 256) return cout;
    for (int bn = 256; bn >= 16; bn -= 16)
        if (cout % bn == 0) return bn;
    return 0;
}

bool pixel_dense(const TView& v) {
    // rows of the view are equally spaced over (b, h, w): stride[2] = pixel step,
    // stride[1] = W * pixel step and img_stride = H * W * pixel step.
    return v.stride[1] == v.shape[2] * v.stride[2] && v.img_stride == v.shape[1] * v.stride[1];
}

}  // namespace

bool encode_box_map(void* map, int elem_bytes, int rank, const void* ptr, const uint64_t* dims,
                    const uint64_t* strides_bytes, const uint32_t* box) {
    if (rank < 1 || rank > 5 || (elem_bytes != 1 && elem_bytes != 4)) return false;
    load_driver_fns();
    cuuint64_t d[5], st[4];
    cuuint32_t bx[5], es[5];
    for (int i = 0; i < rank; ++i) { d[i] = dims[i]; bx[i] = box[i]; es[i] = 1; }
    for (int i = 0; i + 1 < rank; ++i) st[i] = strides_bytes[i];
    return g_tiled(static_cast<CUtensorMap*>(map),
                   elem_bytes == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, (cuuint32_t)rank,
                   const_cast<void*>(ptr), d, st, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool conv_tc_supported(const ConvArgs& a, int op_dt, const char** why) {
    const int esz = op_dt == BF16 ? 2 : 4;
    auto no = [&](const char* m) { if (why) *why = m; return false; };
    if (a.in.dt != op_dt) return no("input dtype differs from operand dtype");
    if (a.in.stride[3] != 1 || a.out.stride[3] != 1) return no("channel stride must be 1");
    if (!pick_chunk(a.cin, esz)) return no("Cin not a multiple of the minimal chunk");
    if (!pick_bn(a.cout)) return no("Cout not a multiple of 16");
    if (a.act < ACT_NONE || a.act > ACT_SILU_WINO) return no("activation not fusable");
    {
        // tile and pixel indices use 32-bit fast division (n < 2^31)
        // (padded positions when a_mode 2 applies: Ho * (W + 2*pad_w) per image)
        const int64_t M = a.batch * a.out.shape[1] * std::max<int64_t>(a.out.shape[2], a.in.shape[2] + 2 * a.pw) + BM;
        const int bn = pick_bn(a.cout);
        if (M + BM >= (int64_t(1) << 31) || ((M + BM - 1) / BM) * (a.cout / bn) >= (int64_t(1) << 31))
            return no("more than 2^31 output pixels");
    }
    if (a.bias && ((uintptr_t)a.bias) % 16) return no("bias not 16-byte aligned");
    if (((uintptr_t)a.in.ptr) % 16 || ((a.in.stride[2] * esz) % 16) || ((a.in.img_stride * esz) % 16) ||
        ((a.in.stride[1] * esz) % 16))
        return no("input view not 16-byte aligned");
    const int oes = a.out.dt == BF16 ? 2 : 4;
    if (((uintptr_t)a.out.ptr) % 16 || (a.out.stride[2] * oes) % 16 || (a.out.stride[1] * oes) % 16 ||
        (a.out.img_stride * oes) % 16)
        return no("output view not 16-byte aligned");
    if (a.res.ptr) {
        const int res = a.res.dt == BF16 ? 2 : 4;
        if (((uintptr_t)a.res.ptr) % 16 || (a.res.stride[2] * res) % 16 || (a.res.stride[1] * res) % 16 ||
            (a.res.img_stride * res) % 16 || a.res.stride[3] != 1)
            return no("residual view not 16-byte aligned");
    }
    const bool one = a.kh == 1 && a.kw == 1 && a.sh == 1 && a.sw == 1 && a.ph == 0 && a.pw == 0;
    if (!one) {
        if (a.ph > 127 || a.pw > 127 || a.kh > 16 || a.kw > 16) return no("im2col corner out of range");
        if (a.in.shape[1] > 65535 || a.in.shape[2] > 65535) return no("spatial extent too large");
    }
    return true;
}

void launch_conv_tc(const ConvArgs& a, int op_dt, int* err, cudaStream_t s) {
    const char* why = nullptr;
    if (!conv_tc_supported(a, op_dt, &why)) fail(ENGINE_ERR_INVALID_ARG, std::string("conv_tc: ") + why);
    load_driver_fns();
    const int esz = op_dt == BF16 ? 2 : 4;
    const int bn = pick_bn(a.cout);
    const int Ho = (int)a.out.shape[1], Wo = (int)a.out.shape[2];
    const int64_t M = a.batch * Ho * Wo;
    if (M == 0) return;
    const CUtensorMapDataType tdt = op_dt == BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;

    TcParams p{};
    p.M = M; p.Ho = Ho; p.Wo = Wo;
    p.sh = a.sh; p.sw = a.sw; p.ph = a.ph; p.pw = a.pw; p.dh = a.dh; p.dw = a.dw; p.kw = a.kw;
    p.taps = a.kh * a.kw; p.cin = a.cin;
    p.bn = bn;
    p.bufcols = 32;
    while (p.bufcols < (uint32_t)bn) p.bufcols <<= 1;
    p.nbuf = 2;
    p.tmem_cols = 2 * (int)p.bufcols;                   // two accumulators (four when TMEM allows, below)
    int dev = 0;
    PB_CUDA(cudaGetDevice(&dev));
    static int sm_count[64] = {};
    int sms = 148;
    if (dev < 64) {
        if (!sm_count[dev]) PB_CUDA(cudaDeviceGetAttribute(&sm_count[dev], cudaDevAttrMultiProcessorCount, dev));
        sms = sm_count[dev];
    }
    {
        // Multi-tap convs with 64 < Cout < 128 (80 for the YOLO class branches) round
        // an accumulator up to 128 columns, so two of them cap TMEM at two CTAs per
        // SM. One accumulator per CTA allows four CTAs but makes every tile's MMAs wait
        // for the previous tile's whole epilogue. Measured on B200 (batch 256): the one
        // layer with at least 8 tiles per CTA slot at four CTAs per SM, 80 -> 80 3x3 at
        // 80x80, runs 0.480 ms with one accumulator against 0.521 with two; the smaller
        // ones are faster with two (128 -> 80 at 40x40 0.117 -> 0.108 ms, 256 -> 80 at
        // 20x20 0.064 -> 0.059, 80 -> 80 at 20x20 0.044 -> 0.040).
        const bool one_ = a.kh == 1 && a.kw == 1 && a.sh == 1 && a.sw == 1 && a.ph == 0 && a.pw == 0;
        if (!one_ && bn > 64 && bn < 128 && (M + BM - 1) / BM >= (int64_t)8 * 4 * sms) {
            p.nbuf = 1;
            p.tmem_cols = (int)p.bufcols;
        }
    }
    // ---- operand plan --------------------------------------------------------
    // Operand modes:
    //   a_mode 1: 1x1 stride-1 conv on a pixel-dense input, plain 2-D tiles of A;
    //   a_mode 0: TMA im2col, one 128-pixel load per tap and channel chunk;
    //   a_mode 2: stride-1, dilation-1 convs whose padded rows fit one TMA box: one
    //             zero-padded window of NR padded rows per tile and channel chunk, each
    //             tap read as the window shifted by r*Wp + s rows;
    // weights streamed per k-block through the ring, or (b_res, one N tile) resident
    // in shared memory, loaded once per CTA. The choices follow per-layer sweeps of
    // every combination on B200 (YOLOv8 layer shapes):
    //   * CTAs per SM matter most: as many as TMEM allows (two accumulators of
    //     bufcols columns each, or one for multi-tap convs with 64 < Cout < 128),
    //     four at most with 4 epilogue warps, two with 8, even when that leaves a
    //     ring of two slots;
    //   * windows win where im2col moves narrow rows (channel chunks under 128
    //     bytes: Cin = 16, 32, 80, ...), im2col elsewhere;
    //   * resident weights whenever they fit without costing a CTA, and always for
    //     windows (streamed weights would dominate the window's rows).
    const bool one = a.kh == 1 && a.kw == 1 && a.sh == 1 && a.sw == 1 && a.ph == 0 && a.pw == 0;
    const int Wp = (int)a.in.shape[2] + 2 * a.pw;
    const int NR = (a.kh * Wp + a.kw + BM - 2 + Wp - 1) / Wp;   // window rows covering row offsets + 128
    const int ch = pick_chunk(a.cin, esz);
    const int swb = ch * esz;
    // Cin = q full 128-byte chunks + one 32-byte chunk (Cin = 80, 144, ... in bf16): a
    // multi-tap conv reads the last chunk as a narrow tail (own tensor maps, 32-byte
    // swizzle, one K slice) rather than as a full chunk of which three quarters are
    // zeros: 80 -> 80 3x3 at 80x80 0.74 -> 0.51 ms (batch 256). 1x1 convs keep the
    // padded chunk: their extra tail k-block cost more than the zeros (0.13 -> 0.17 ms).
    const int tail_ch = (swb == 128 && p.taps > 1 && a.cin > ch && a.cin % ch == 32 / esz) ? 32 / esz : 0;
    const int chunks = tail_ch ? a.cin / ch + 1 : (a.cin + ch - 1) / ch;   // a partial chunk reads zeros past Cin
    const int nk = p.taps * chunks;
    const int tmem_ctas = 512 / p.tmem_cols;                     // p.nbuf accumulators per CTA
    // 8 epilogue warps for 1x1 convs from 128 output channels up and for multi-tap
    // convs whose accumulators leave TMEM room for two CTAs at most (Cout >= 128 with
    // two accumulators); the single-accumulator convs (64 < Cout < 128) fit four CTAs
    // and take 4 epilogue warps. 1x1 convs stage their output for TMA stores.
    const int epi = (one ? bn >= 128 : tmem_ctas <= 2) ? 8 : 4;
    const int max_ctas = std::min(epi == 8 ? 2 : 4, tmem_ctas);  // register file, TMEM
    const int oes = a.out.dt == BF16 ? 2 : 4;
    const uint32_t staging = (uint32_t)bn * BM * oes;
    const bool tma_store = p.taps == 1 && pixel_dense(a.out) && staging <= 64u * 1024u;
    const uint32_t fixed = 1024 + kBarrierBytes + 1024 + (tma_store ? staging : 0u);   // alignment, barriers, reserve
    const uint32_t btile = (uint32_t)bn * swb;
    const uint32_t bres_all = (uint32_t)nk * btile;
    const uint32_t win_tx = (uint32_t)NR * (uint32_t)Wp * (uint32_t)swb;
    const uint32_t win_slot = (win_tx + 1023u) & ~1023u;
    const bool window_ok = !one && a.sh == 1 && a.sw == 1 && a.dh == 1 && a.dw == 1 && Wp <= 256 && NR <= 256 &&
                           Wo == Wp - a.kw + 1;
    struct Cand { int mode, bres, ctas, stages; };
    // most CTAs (<= max_ctas) a configuration fits, with its ring depth; ctas 0 = none
    auto fit = [&](int mode, int bres) {
        Cand c{mode, bres, 0, 0};
        if (bres && (bn != a.cout || bres_all > 200u * 1024u || tail_ch)) return c;
        const uint32_t a_st = mode == 2 ? 0u : (uint32_t)BM * swb;
        const uint32_t b_st = bres ? 0u : btile;
        const uint32_t st = a_st + b_st;
        const uint32_t fixed_c = fixed + (bres ? bres_all : 0u) + (mode == 2 ? 2u * win_slot : 0u);
        // two ring slots suffice: more CTAs beat a deeper ring (swept on B200), except
        // for tail chunks (below)
        // with a tail chunk (two k-blocks per tap, one of them small) a third slot
        // pays: 80 -> 80 3x3 at 80x80 0.534 -> 0.483 ms; other convs lost with it
        // (64 -> 80 0.275 -> 0.341, the stride-2 convs 25-35%)
        const int min_st = st == 0 ? 0 : (tail_ch ? 3 : 2);
        auto room = [&](int n) { return (int64_t)(228u * 1024u) / n - (int64_t)fixed_c; };
        for (int n = max_ctas; n >= 1; --n) {
            if (room(n) >= 0 && room(n) >= (int64_t)min_st * st) {
                c.ctas = n;
                c.stages = st == 0 ? 0 : (int)std::min<int64_t>(12, room(n) / st);
                return c;
            }
        }
        return c;
    };
    Cand best{-1, 0, 0, 0};
    if (one && pixel_dense(a.in)) {
        const Cand s0 = fit(1, 0), s1 = fit(1, 1);
        best = s1.ctas > 0 && s1.ctas >= s0.ctas ? s1 : s0;
    } else {
        if (window_ok && swb < 128 && !tail_ch) {
            const Cand w1 = fit(2, 1), w0 = fit(2, 0);
            if (w1.ctas > 0) best = w1;
            else if (w0.ctas > 0) best = w0;
        }
        if (best.ctas == 0 || best.mode < 0) {
            const Cand s0 = fit(0, 0), s1 = fit(0, 1);
            best = s1.ctas > 0 && s1.ctas >= s0.ctas ? s1 : s0;
        }
    }
    if (best.mode < 0 || best.ctas == 0) fail(ENGINE_ERR_INVALID_ARG, "conv_tc: tile does not fit in shared memory");
    p.a_mode = best.mode;
    p.b_res = best.bres;
    int ctas = best.ctas;
    const int stages = best.stages;
    p.tma_store = tma_store;
    p.staging_bytes = tma_store ? staging : 0u;
    p.ch = ch; p.swb = swb; p.cin_chunks = chunks;
    p.tail_ch = tail_ch;
    p.tail_a_bytes = tail_ch ? (uint32_t)BM * 32u : 0u;
    p.tail_b_bytes = tail_ch ? (uint32_t)bn * 32u : 0u;
    p.stage_a_bytes = p.a_mode == 2 ? 0u : (uint32_t)BM * swb;
    p.stage_b_bytes = p.b_res ? 0u : btile;
    const uint32_t stage2 = p.stage_a_bytes + p.stage_b_bytes;
    p.btile_bytes = btile;
    p.bres_bytes = p.b_res ? bres_all : 0u;
    p.hstages = p.a_mode == 2 ? 2 : 0;
    const uint32_t halo_tx = p.a_mode == 2 ? win_tx : 0u;
    const uint32_t halo_slot = p.a_mode == 2 ? win_slot : 0u;
    p.Wp = Wp; p.NR = NR;
    p.halo_tx = halo_tx;
    p.halo_bytes = halo_slot;
    p.stages = stages;
    // With spare TMEM the MMA warp may run up to four tiles ahead of the epilogue
    // (MMA completion latency is hidden behind more than one epilogue).
    if (ctas * 4 * (int)p.bufcols <= 512) { p.nbuf = 4; p.tmem_cols = 4 * (int)p.bufcols; }
    const uint32_t fmt = op_dt == BF16 ? 1u : 2u;
    p.idesc = (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)(bn >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
    p.out = const_cast<void*>(a.out.ptr); p.out_dt = a.out.dt;
    p.out_img = a.out.img_stride; p.out_sh = a.out.stride[1]; p.out_sw = a.out.stride[2];
    p.res = a.res.ptr; p.res_dt = a.res.dt;
    p.res_img = a.res.img_stride; p.res_sh = a.res.stride[1]; p.res_sw = a.res.stride[2];
    p.bias = a.bias; p.act = a.act; p.slope = a.slope; p.cout = a.cout;
    p.err = err;
    // Pipeline waits give up after wait_limit cycles (~0.5 s by default); the drains
    // before exit always use the default, so no copy or MMA is left in flight.
    p.wait_limit = a.wait_limit > 0 ? a.wait_limit : 1000000000LL;

    CUtensorMap tmA, tmB, tmOut, tmA2, tmB2;
    std::memset(&tmOut, 0, sizeof(tmOut));
    if (p.tma_store) {
        // [pixels, Cout] view of the output, 16-channel boxes of 128 rows, swizzled
        // like the staging blocks (32-byte rows for bf16, 64-byte rows for fp32)
        cuuint64_t dims[2] = {(cuuint64_t)a.cout, (cuuint64_t)M};
        cuuint64_t strides[1] = {(cuuint64_t)(a.out.stride[2] * oes)};
        cuuint32_t box[2] = {16, (cuuint32_t)BM};
        cuuint32_t es[2] = {1, 1};
        CUresult r = g_tiled(&tmOut, a.out.dt == BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                             2, p.out, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                             a.out.dt == BF16 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_64B,
                             CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) fail(ENGINE_ERR_RUNTIME, "cuTensorMapEncodeTiled(out) failed: " + std::to_string((int)r));
    }
    if (p.a_mode == 1) {
        cuuint64_t dims[2] = {(cuuint64_t)a.cin, (cuuint64_t)(a.batch * a.in.shape[1] * a.in.shape[2])};
        cuuint64_t strides[1] = {(cuuint64_t)(a.in.stride[2] * esz)};
        cuuint32_t es[2] = {1, 1};
        for (int part = 0; part < (tail_ch ? 2 : 1); ++part) {
            cuuint32_t box[2] = {(cuuint32_t)(part ? tail_ch : ch), (cuuint32_t)BM};
            CUresult r = g_tiled(part ? &tmA2 : &tmA, tdt, 2, const_cast<void*>(a.in.ptr), dims, strides, box, es,
                                 CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle_of(part ? 32 : swb),
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
            if (r != CUDA_SUCCESS) fail(ENGINE_ERR_RUNTIME, "cuTensorMapEncodeTiled(A) failed: " + std::to_string((int)r));
        }
    } else if (p.a_mode == 2) {
        // [N, H, W, C] input; box = one channel chunk of NR padded rows of Wp pixels,
        // out-of-image pixels read as zeros (the padding)
        cuuint64_t dims[4] = {(cuuint64_t)a.cin, (cuuint64_t)a.in.shape[2], (cuuint64_t)a.in.shape[1], (cuuint64_t)a.batch};
        cuuint64_t strides[3] = {(cuuint64_t)(a.in.stride[2] * esz), (cuuint64_t)(a.in.stride[1] * esz),
                                 (cuuint64_t)(a.in.img_stride * esz)};
        cuuint32_t box[4] = {(cuuint32_t)ch, (cuuint32_t)Wp, (cuuint32_t)NR, 1};
        cuuint32_t es[4] = {1, 1, 1, 1};
        CUresult r = g_tiled(&tmA, tdt, 4, const_cast<void*>(a.in.ptr), dims, strides, box, es,
                             CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle_of(swb), CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) fail(ENGINE_ERR_RUNTIME, "cuTensorMapEncodeTiled(window) failed: " + std::to_string((int)r));
    } else {
        cuuint64_t dims[4] = {(cuuint64_t)a.cin, (cuuint64_t)a.in.shape[2], (cuuint64_t)a.in.shape[1], (cuuint64_t)a.batch};
        cuuint64_t strides[3] = {(cuuint64_t)(a.in.stride[2] * esz), (cuuint64_t)(a.in.stride[1] * esz),
                                 (cuuint64_t)(a.in.img_stride * esz)};
        int lower[2] = {-a.pw, -a.ph};
        int upper[2] = {a.pw - (a.kw - 1) * a.dw, a.ph - (a.kh - 1) * a.dh};
        cuuint32_t es[4] = {1, (cuuint32_t)a.sw, (cuuint32_t)a.sh, 1};
        for (int part = 0; part < (tail_ch ? 2 : 1); ++part) {
            CUresult r = g_im2col(part ? &tmA2 : &tmA, tdt, 4, const_cast<void*>(a.in.ptr), dims, strides, lower, upper,
                                  (cuuint32_t)(part ? tail_ch : ch), (cuuint32_t)BM, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                  swizzle_of(part ? 32 : swb), CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
            if (r != CUDA_SUCCESS) fail(ENGINE_ERR_RUNTIME, "cuTensorMapEncodeIm2col(A) failed: " + std::to_string((int)r));
        }
    }
    {
        // [Cout, taps, Cin] weights: one box = one channel chunk of one tap for bn
        // output channels; channels past Cin (a partial last chunk) read as zeros
        cuuint64_t dims[3] = {(cuuint64_t)a.cin, (cuuint64_t)p.taps, (cuuint64_t)a.cout};
        cuuint64_t strides[2] = {(cuuint64_t)a.cin * esz, (cuuint64_t)p.taps * a.cin * esz};
        cuuint32_t es[3] = {1, 1, 1};
        for (int part = 0; part < (tail_ch ? 2 : 1); ++part) {
            cuuint32_t box[3] = {(cuuint32_t)(part ? tail_ch : ch), 1, (cuuint32_t)bn};
            CUresult r = g_tiled(part ? &tmB2 : &tmB, tdt, 3, const_cast<void*>(a.weight), dims, strides, box, es,
                                 CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle_of(part ? 32 : swb),
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
            if (r != CUDA_SUCCESS) fail(ENGINE_ERR_RUNTIME, "cuTensorMapEncodeTiled(W) failed: " + std::to_string((int)r));
        }
        if (!tail_ch) { tmA2 = tmA; tmB2 = tmB; }   // unused
    }
    p.n_tiles = a.cout / bn;
    if (p.a_mode == 2) {
        // tiles never straddle images: positions P = y*Wp + x of one image, Ho*Wp of them
        p.Q = (uint32_t)Ho * (uint32_t)Wp;
        const uint32_t tpi = (p.Q + BM - 1) / BM;
        p.div_tpi = make_fastdiv(tpi);
        p.div_wp = make_fastdiv((uint32_t)Wp);
        p.m_tiles = (int64_t)tpi * a.batch;
    } else {
        p.m_tiles = (M + BM - 1) / BM;
    }
    p.div_ntiles = make_fastdiv((uint32_t)p.n_tiles);
    p.div_hw = make_fastdiv((uint32_t)((int64_t)Ho * Wo));
    p.div_wo = make_fastdiv((uint32_t)Wo);
    const size_t smem = (size_t)stages * stage2 + p.staging_bytes + (size_t)p.hstages * p.halo_bytes + p.bres_bytes +
                        1024 + kBarrierBytes;
    const int64_t tiles = p.m_tiles * p.n_tiles;
    dim3 grid((unsigned)std::min<int64_t>(tiles, (int64_t)sms * ctas));
    static bool attr[10][64] = {};
    const int kind = op_dt == BF16 ? 0 : 1;
    // register-budget variant: EPI 4 at 4, 3 or <= 2 CTAs per SM; EPI 8 at 2 or 1
    const int vsub = epi == 8 ? (ctas >= 2 ? 3 : 4) : (ctas >= 4 ? 0 : (ctas == 3 ? 1 : 2));
    const int variant = kind * 5 + vsub;
    void (*const fns[10])(CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap, TcParams) = {
        conv_tc_kernel<0, 4, 4>, conv_tc_kernel<0, 4, 3>, conv_tc_kernel<0, 4, 2>, conv_tc_kernel<0, 8, 2>,
        conv_tc_kernel<0, 8, 1>, conv_tc_kernel<1, 4, 4>, conv_tc_kernel<1, 4, 3>, conv_tc_kernel<1, 4, 2>,
        conv_tc_kernel<1, 8, 2>, conv_tc_kernel<1, 8, 1>};
    if (dev < 64 && !attr[variant][dev]) {
        PB_CUDA(cudaFuncSetAttribute(fns[variant], cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
        attr[variant][dev] = true;
    }
    const int threads = epi == 8 ? conv_threads<8>() : conv_threads<4>();
    fns[variant]<<<grid, threads, smem, s>>>(tmA, tmB, tmOut, tmA2, tmB2, p);
    PB_CUDA(cudaGetLastError());
}

void launch_gemm_tc(const float* A, const float* B, float* C, int64_t M, int64_t N, int64_t K, int op_dt,
                    void* scratch, int* err, cudaStream_t s) {
    // GEMM as a 1x1 convolution over M "pixels": operands staged in the operand type,
    // B transposed to the K-major [N, K] layout the weight tensor map expects.
    const int esz = op_dt == BF16 ? 2 : 4;
    char* sc = static_cast<char*>(scratch);
    const size_t a_bytes = (((size_t)M * K * esz) + 255) & ~size_t(255);
    void* a_op = sc;
    void* bt = sc + a_bytes;
    const void* a_ptr = A;
    if (op_dt == BF16) {
        TView src, dst;
        src.ptr = A; src.dt = F32; src.rank = 2; src.shape[0] = M; src.shape[1] = K;
        src.stride[0] = K; src.stride[1] = 1; src.img_stride = M * K;
        dst = src; dst.ptr = a_op; dst.dt = BF16;
        launch_strided_copy(src, dst, 1, s);
        a_ptr = a_op;
    }
    {
        TView src, dst;
        src.ptr = B; src.dt = F32; src.rank = 2; src.shape[0] = N; src.shape[1] = K;
        src.stride[0] = 1; src.stride[1] = N; src.img_stride = N * K;
        dst.ptr = bt; dst.dt = op_dt; dst.rank = 2; dst.shape[0] = N; dst.shape[1] = K;
        dst.stride[0] = K; dst.stride[1] = 1; dst.img_stride = N * K;
        launch_strided_copy(src, dst, 1, s);
    }
    ConvArgs a;
    a.in.ptr = a_ptr; a.in.dt = op_dt; a.in.rank = 4;
    a.in.shape[0] = 1; a.in.shape[1] = 1; a.in.shape[2] = M; a.in.shape[3] = K;
    a.in.stride[0] = M * K; a.in.stride[1] = M * K; a.in.stride[2] = K; a.in.stride[3] = 1;
    a.in.img_stride = M * K;
    a.out.ptr = C; a.out.dt = F32; a.out.rank = 4;
    a.out.shape[0] = 1; a.out.shape[1] = 1; a.out.shape[2] = M; a.out.shape[3] = N;
    a.out.stride[0] = M * N; a.out.stride[1] = M * N; a.out.stride[2] = N; a.out.stride[3] = 1;
    a.out.img_stride = M * N;
    a.weight = bt;
    a.cin = (int)K; a.cout = (int)N;
    a.batch = 1;
    launch_conv_tc(a, op_dt, err, s);
}

}  // namespace pb
