// Blackwell (sm_100a) tensor-core implicit-GEMM convolution.
//
// GEMM view: D[M = batch*Ho*Wo pixels, N = Cout] = A[M, K] * W[N, K]^T with
// K = kh*kw*Cin ordered (tap, channel), cut into 128 x BN output tiles. The kernel
// is persistent (one CTA per SM, tiles taken round-robin) and warp-specialized:
//   * warp 0 / lane 0 issues TMA loads into a ring of `stages` shared-memory slots
//     that runs on across tile boundaries:
//       A: im2col-mode tensor map (3x3 / strided / padded convs: the TMA unit walks
//          128 consecutive output pixels and applies the tap offset, zero-filling
//          padding) or a plain 2-D tiled map (1x1 stride-1 convs, GEMMs);
//       W: 2-D tiled map over the [Cout, K] weight matrix.
//     Each load covers `CH` channels (CH*elem = 32/64/128 bytes, the swizzle width).
//     No load uses cluster multicast.
//   * warp 1 / lane 0 issues tcgen05.mma (kind::f16 for BF16, kind::tf32 for TF32)
//     into one of two TMEM accumulators (128 lanes x BN fp32 columns each), releases
//     ring slots with tcgen05.commit and hands a finished accumulator to the epilogue.
//   * warps 2-5 run the epilogue of tile t while tile t+1 accumulates: tcgen05.ld of
//     their 32 TMEM lanes, bias, activation, optional residual add, and a strided
//     store (bf16 or fp32) that can land inside a channel slice of a concat buffer.
// Every mbarrier wait is bounded; on timeout the kernel records an error in the
// device error word, stops issuing work, drains its outstanding copies, frees TMEM
// and exits.
#include <cuda.h>
#include <algorithm>
#include <mutex>

#include "common.h"
#include "device_common.cuh"

namespace pb {

namespace {

constexpr int BM = 128;

struct TcParams {
    int64_t M;
    int Ho, Wo;
    int sh, sw, ph, pw, dh, dw, kw;
    int taps, cin_chunks, ch, cin;
    int bn, stages, a_mode, tmem_cols, swb;
    uint32_t idesc;
    uint32_t stage_a_bytes, stage_b_bytes;
    void* out; int out_dt; int64_t out_img, out_sh, out_sw;
    const void* res; int res_dt; int64_t res_img, res_sh, res_sw;
    const float* bias; int act; float slope; int cout;
    int64_t m_tiles; int n_tiles;
    int* err;
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

__device__ __forceinline__ void tma_load_im2col_4d(uint32_t dst, const CUtensorMap* map, uint64_t* bar,
                                                   int c, int w, int h, int n, uint16_t ow, uint16_t oh) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.im2col.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5, %6}], [%2], {%7, %8};"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)),
          "r"(c), "r"(w), "r"(h), "r"(n), "h"(ow), "h"(oh)
        : "memory");
}

template <int KIND>  // 0: kind::f16 (bf16 operands), 1: kind::tf32
__device__ __forceinline__ void umma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
    if (KIND == 0) {
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
            ::"r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(acc));
    } else {
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}"
            ::"r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(acc));
    }
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Activation of the tensor-core epilogue. The operands are BF16/TF32, so SiLU and
// sigmoid use the hardware exponential (__expf, ~2 ulp) and a fast divide; the
// reference's Winograd SiLU flavour and the rarer activations keep their exact form.
template <int ACT>
__device__ __forceinline__ float tc_act(float x, float slope) {
    if (ACT == ACT_NONE) return x;
    if (ACT == ACT_SILU) return __fdividef(x, 1.0f + __expf(-x));
    if (ACT == ACT_SILU_WINO) return silu_wino_f(x);
    return apply_act(x, ACT, slope, 0.0f);
}

__device__ __forceinline__ void load_res_chunk(const TcParams& p, int64_t rb, uint4 (&r)[4]) {
    const uint4* src = p.res_dt == BF16
        ? reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(p.res) + rb)
        : reinterpret_cast<const uint4*>(reinterpret_cast<const float*>(p.res) + rb);
    r[0] = __ldg(src);
    r[1] = __ldg(src + 1);
    if (p.res_dt != BF16) { r[2] = __ldg(src + 2); r[3] = __ldg(src + 3); }
}

// Epilogue for one 16-column chunk of one accumulator row: bias, activation,
// residual, bf16/fp32 store (16 contiguous channels of one pixel).
template <int ACT>
__device__ __forceinline__ void epilogue_chunk(const TcParams& p, float (&v)[16], const uint4 (&r)[4],
                                               int64_t ob, int ncol) {
    if (p.bias) {
        const float4* b4 = reinterpret_cast<const float4*>(p.bias + ncol);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float4 b = __ldg(b4 + q);
            v[4 * q] += b.x; v[4 * q + 1] += b.y; v[4 * q + 2] += b.z; v[4 * q + 3] += b.w;
        }
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = tc_act<ACT>(v[i], p.slope);
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
    if (p.out_dt == BF16) {
        uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.out) + ob);
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            uint32_t w4[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                __nv_bfloat162 h2 = __floats2bfloat162_rn(v[q * 8 + 2 * j], v[q * 8 + 2 * j + 1]);
                w4[j] = *reinterpret_cast<uint32_t*>(&h2);
            }
            dst[q] = make_uint4(w4[0], w4[1], w4[2], w4[3]);
        }
    } else {
        float4* dst = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + ob);
#pragma unroll
        for (int q = 0; q < 4; ++q) dst[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    }
}

// Epilogue warps 2..5: drain accumulator tiles in the order the MMA warp filled them.
// The residual of the next 16 columns is loaded before the current chunk is
// processed (the first chunk's before the accumulator wait), hiding its latency.
template <int ACT>
__device__ void epilogue_loop(const TcParams& p, uint32_t tmem, uint32_t half, uint64_t* tfull, uint64_t* tempty,
                              volatile int* abort_flag, int64_t total) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q = warp & 3;               // TMEM lane quarter this warp may access
    const int row = q * 32 + lane;
    const int64_t hw = (int64_t)p.Ho * p.Wo;
    int64_t i = 0;
    for (int64_t t = blockIdx.x; t < total; t += gridDim.x, ++i) {
        const int buf = (int)(i & 1);
        const int64_t mt = t / p.n_tiles;
        const int n0 = (int)(t - mt * p.n_tiles) * p.bn;
        const int64_t m = mt * BM + row;
        const bool live = m < p.M;
        int64_t ob = 0, rb = 0;
        if (live) {
            const int64_t b = m / hw, r = m - b * hw;
            const int64_t ho = r / p.Wo, wo = r - ho * p.Wo;
            ob = b * p.out_img + ho * p.out_sh + wo * p.out_sw + n0;
            rb = b * p.res_img + ho * p.res_sh + wo * p.res_sw + n0;
        }
        uint4 rn[4] = {};
        if (p.res && live) load_res_chunk(p, rb, rn);
        bool ok = mbar_wait_bounded(&tfull[buf], (uint32_t)((i >> 1) & 1));
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) { if (lane == 0) { atomicExch(p.err, 3); *abort_flag = 1; } break; }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)buf * half;
        for (int c0 = 0; c0 < p.bn; c0 += 16) {
            const uint4 rc[4] = {rn[0], rn[1], rn[2], rn[3]};
            if (p.res && live && c0 + 16 < p.bn) load_res_chunk(p, rb + c0 + 16, rn);
            float v[16];
            tmem_ld16(tbase + (uint32_t)c0, v);
            if (live) epilogue_chunk<ACT>(p, v, rc, ob + c0, n0 + c0);
        }
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[buf]);
        if (__any_sync(0xffffffffu, *abort_flag != 0)) break;
    }
}

// Persistent, warp-specialized kernel. 192 threads:
//   warp 0  (lane 0): TMA producer, streams (tile, k-block) loads through the ring
//                     without stopping at tile boundaries;
//   warp 1  (lane 0): MMA issuer; owns two TMEM accumulators and alternates between
//                     them, so tile t+1 accumulates while tile t is drained;
//   warps 2-5:        epilogue; warp w reads TMEM lanes 32*(w%4).. (its row quarter).
// Tiles are taken round-robin (tile = blockIdx.x + i*gridDim.x), N-tiles innermost
// so CTAs working on the same pixel rows run close together (A re-reads hit L2).
template <int KIND>
__global__ void __launch_bounds__(192, 4)
conv_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const TcParams p) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t* const smem = smem_raw + (base - raw);
    const int S = p.stages;
    const uint32_t a_bytes = p.stage_a_bytes, b_bytes = p.stage_b_bytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)S * (a_bytes + b_bytes));
    uint64_t* empty = full + S;
    uint64_t* tfull = empty + S;          // [2] MMA -> epilogue
    uint64_t* tempty = tfull + 2;         // [2] epilogue -> MMA
    uint64_t* mma_done = tempty + 2;      // all issued MMAs finished (before TMEM is freed)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
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
        for (int i = 0; i < 2; ++i) { mbar_init(&tfull[i], 1); mbar_init(&tempty[i], 4); }
        mbar_init(mma_done, 1);
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
    const uint32_t half = (uint32_t)(p.tmem_cols >> 1);

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            int64_t it = 0;   // global k-block counter across tiles
            for (int64_t t = blockIdx.x; t < total && !*abort_flag; t += gridDim.x) {
                const int64_t mt = t / p.n_tiles;
                const int n0 = (int)(t - mt * p.n_tiles) * p.bn;
                const int64_t m0 = mt * BM;
                int64_t b = 0; int ho = 0, wo = 0;
                if (p.a_mode == 0) {
                    const int64_t hw = (int64_t)p.Ho * p.Wo;
                    b = m0 / hw;
                    const int64_t r = m0 - b * hw;
                    ho = (int)(r / p.Wo);
                    wo = (int)(r - (int64_t)ho * p.Wo);
                }
                for (int kb = 0; kb < nk; ++kb, ++it) {
                    const int st = (int)(it % S);
                    if (it >= S && !mbar_wait_bounded(&empty[st], (uint32_t)(((it / S) & 1) ^ 1))) {
                        atomicExch(p.err, 1);
                        *abort_flag = 1;
                        break;
                    }
                    const int tap = kb / p.cin_chunks, cc = kb - tap * p.cin_chunks;
                    const uint32_t sa = base + (uint32_t)st * a_bytes;
                    const uint32_t sb = base + (uint32_t)S * a_bytes + (uint32_t)st * b_bytes;
                    mbar_expect_tx(&full[st], a_bytes + b_bytes);
                    if (p.a_mode == 0) {
                        const int r = tap / p.kw, s = tap - r * p.kw;
                        tma_load_im2col_4d(sa, &tmA, &full[st], cc * p.ch, wo * p.sw - p.pw, ho * p.sh - p.ph,
                                           (int)b, (uint16_t)(s * p.dw), (uint16_t)(r * p.dh));
                    } else {
                        tma_load_2d(sa, &tmA, &full[st], cc * p.ch, (int)m0);
                    }
                    tma_load_2d(sb, &tmB, &full[st], tap * p.cin + cc * p.ch, n0);
                }
            }
            // Drain: the last use of every slot must have landed before the CTA exits.
            for (int64_t k = it > S ? it - S : 0; k < it; ++k)
                if (!mbar_wait_bounded(&full[k % S], (uint32_t)((k / S) & 1))) atomicExch(p.err, 4);
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            const int ksteps = p.swb / 32;
            int64_t it = 0;
            int64_t i = 0;    // local tile counter
            for (int64_t t = blockIdx.x; t < total && !*abort_flag; t += gridDim.x, ++i) {
                const int buf = (int)(i & 1);
                if (i >= 2 && !mbar_wait_bounded(&tempty[buf], (uint32_t)(((i >> 1) & 1) ^ 1))) {
                    atomicExch(p.err, 5);
                    *abort_flag = 1;
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t d = tmem + (uint32_t)buf * half;
                bool ok = true;
                for (int kb = 0; kb < nk; ++kb, ++it) {
                    const int st = (int)(it % S);
                    if (!mbar_wait_bounded(&full[st], (uint32_t)((it / S) & 1))) { ok = false; break; }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const uint32_t sa = base + (uint32_t)st * a_bytes;
                    const uint32_t sb = base + (uint32_t)S * a_bytes + (uint32_t)st * b_bytes;
                    for (int k = 0; k < ksteps; ++k)
                        umma<KIND>(d, make_smem_desc(sa + 32u * k, p.swb), make_smem_desc(sb + 32u * k, p.swb),
                                   p.idesc, (kb | k) != 0);
                    umma_commit(&empty[st]);
                }
                if (!ok) { atomicExch(p.err, 2); *abort_flag = 1; break; }
                umma_commit(&tfull[buf]);
            }
            umma_commit(mma_done);
        }
        __syncwarp();
    } else {
        // ---------------- epilogue (warps 2..5) ----------------
        switch (p.act) {
            case ACT_NONE: epilogue_loop<ACT_NONE>(p, tmem, half, tfull, tempty, abort_flag, total); break;
            case ACT_SILU: epilogue_loop<ACT_SILU>(p, tmem, half, tfull, tempty, abort_flag, total); break;
            case ACT_SILU_WINO: epilogue_loop<ACT_SILU_WINO>(p, tmem, half, tfull, tempty, abort_flag, total); break;
            case ACT_RELU: epilogue_loop<ACT_RELU>(p, tmem, half, tfull, tempty, abort_flag, total); break;
            case ACT_LEAKY: epilogue_loop<ACT_LEAKY>(p, tmem, half, tfull, tempty, abort_flag, total); break;
            case ACT_SIGMOID: epilogue_loop<ACT_SIGMOID>(p, tmem, half, tfull, tempty, abort_flag, total); break;
            default: epilogue_loop<ACT_GELU_TANH>(p, tmem, half, tfull, tempty, abort_flag, total); break;  // host-checked
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

int pick_chunk(int cin, int esz) {
    const int c128 = 128 / esz, c64 = 64 / esz, c32 = 32 / esz;
    if (cin % c128 == 0) return c128;
    if (cin % c64 == 0) return c64;
    if (cin % c32 == 0) return c32;
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

bool conv_tc_supported(const ConvArgs& a, int op_dt, const char** why) {
    const int esz = op_dt == BF16 ? 2 : 4;
    auto no = [&](const char* m) { if (why) *why = m; return false; };
    if (a.in.dt != op_dt) return no("input dtype differs from operand dtype");
    if (a.in.stride[3] != 1 || a.out.stride[3] != 1) return no("channel stride must be 1");
    if (!pick_chunk(a.cin, esz)) return no("Cin not a multiple of the minimal chunk");
    if (!pick_bn(a.cout)) return no("Cout not a multiple of 16");
    if (a.act < ACT_NONE || a.act > ACT_SILU_WINO) return no("activation not fusable");
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
    const int ch = pick_chunk(a.cin, esz);
    const int swb = ch * esz;
    const int bn = pick_bn(a.cout);
    const int Ho = (int)a.out.shape[1], Wo = (int)a.out.shape[2];
    const int64_t M = a.batch * Ho * Wo;
    if (M == 0) return;
    const CUtensorMapDataType tdt = op_dt == BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;

    TcParams p{};
    p.M = M; p.Ho = Ho; p.Wo = Wo;
    p.sh = a.sh; p.sw = a.sw; p.ph = a.ph; p.pw = a.pw; p.dh = a.dh; p.dw = a.dw; p.kw = a.kw;
    p.taps = a.kh * a.kw; p.ch = ch; p.cin = a.cin; p.cin_chunks = a.cin / ch;
    p.bn = bn; p.swb = swb;
    p.tmem_cols = 32;
    while (p.tmem_cols < 2 * bn) p.tmem_cols <<= 1;    // two accumulators
    p.stage_a_bytes = BM * swb;
    p.stage_b_bytes = bn * swb;
    const uint32_t stage = p.stage_a_bytes + p.stage_b_bytes;
    // Persistent CTAs, several per SM when TMEM and shared memory allow: each CTA
    // is one producer/MMA/epilogue pipeline, and small-K layers are limited by how
    // fast epilogues drain, so more pipelines per SM beat a deeper ring. Each CTA
    // keeps at least 4 ring slots (the ring runs on across tiles).
    const uint32_t fixed = 1024 + 256 + 1024;     // alignment slack, barriers, per-CTA reserve
    auto stages_for = [&](int c) { return (int)(((228u * 1024u) / (uint32_t)c - fixed) / stage); };
    int ctas = std::min(4, 512 / p.tmem_cols);
    while (ctas > 1 && stages_for(ctas) < 4) --ctas;
    int stages = std::min(12, stages_for(ctas));
    if (stages < 2) fail(ENGINE_ERR_INVALID_ARG, "conv_tc: tile does not fit in shared memory");
    p.stages = stages;
    const uint32_t fmt = op_dt == BF16 ? 1u : 2u;
    p.idesc = (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)(bn >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
    p.out = const_cast<void*>(a.out.ptr); p.out_dt = a.out.dt;
    p.out_img = a.out.img_stride; p.out_sh = a.out.stride[1]; p.out_sw = a.out.stride[2];
    p.res = a.res.ptr; p.res_dt = a.res.dt;
    p.res_img = a.res.img_stride; p.res_sh = a.res.stride[1]; p.res_sw = a.res.stride[2];
    p.bias = a.bias; p.act = a.act; p.slope = a.slope; p.cout = a.cout;
    p.err = err;

    CUtensorMap tmA, tmB;
    const bool one = a.kh == 1 && a.kw == 1 && a.sh == 1 && a.sw == 1 && a.ph == 0 && a.pw == 0;
    if (one && pixel_dense(a.in)) {
        p.a_mode = 1;
        cuuint64_t dims[2] = {(cuuint64_t)a.cin, (cuuint64_t)(a.batch * a.in.shape[1] * a.in.shape[2])};
        cuuint64_t strides[1] = {(cuuint64_t)(a.in.stride[2] * esz)};
        cuuint32_t box[2] = {(cuuint32_t)ch, (cuuint32_t)BM};
        cuuint32_t es[2] = {1, 1};
        CUresult r = g_tiled(&tmA, tdt, 2, const_cast<void*>(a.in.ptr), dims, strides, box, es,
                             CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle_of(swb), CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) fail(ENGINE_ERR_RUNTIME, "cuTensorMapEncodeTiled(A) failed: " + std::to_string((int)r));
    } else {
        p.a_mode = 0;
        cuuint64_t dims[4] = {(cuuint64_t)a.cin, (cuuint64_t)a.in.shape[2], (cuuint64_t)a.in.shape[1], (cuuint64_t)a.batch};
        cuuint64_t strides[3] = {(cuuint64_t)(a.in.stride[2] * esz), (cuuint64_t)(a.in.stride[1] * esz),
                                 (cuuint64_t)(a.in.img_stride * esz)};
        int lower[2] = {-a.pw, -a.ph};
        int upper[2] = {a.pw - (a.kw - 1) * a.dw, a.ph - (a.kh - 1) * a.dh};
        cuuint32_t es[4] = {1, (cuuint32_t)a.sw, (cuuint32_t)a.sh, 1};
        CUresult r = g_im2col(&tmA, tdt, 4, const_cast<void*>(a.in.ptr), dims, strides, lower, upper,
                              (cuuint32_t)ch, (cuuint32_t)BM, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle_of(swb),
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) fail(ENGINE_ERR_RUNTIME, "cuTensorMapEncodeIm2col(A) failed: " + std::to_string((int)r));
    }
    {
        const int64_t K = (int64_t)a.kh * a.kw * a.cin;
        cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)a.cout};
        cuuint64_t strides[1] = {(cuuint64_t)(K * esz)};
        cuuint32_t box[2] = {(cuuint32_t)ch, (cuuint32_t)bn};
        cuuint32_t es[2] = {1, 1};
        CUresult r = g_tiled(&tmB, tdt, 2, const_cast<void*>(a.weight), dims, strides, box, es,
                             CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle_of(swb), CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) fail(ENGINE_ERR_RUNTIME, "cuTensorMapEncodeTiled(W) failed: " + std::to_string((int)r));
    }
    p.m_tiles = (M + BM - 1) / BM;
    p.n_tiles = a.cout / bn;
    const size_t smem = (size_t)stages * stage + 1024 + 256;
    int dev = 0;
    PB_CUDA(cudaGetDevice(&dev));
    static int sm_count[64] = {};
    int sms = 148;
    if (dev < 64) {
        if (!sm_count[dev]) PB_CUDA(cudaDeviceGetAttribute(&sm_count[dev], cudaDevAttrMultiProcessorCount, dev));
        sms = sm_count[dev];
    }
    const int64_t tiles = p.m_tiles * p.n_tiles;
    dim3 grid((unsigned)std::min<int64_t>(tiles, (int64_t)sms * ctas));
    static bool attr[2][64] = {};
    const int kind = op_dt == BF16 ? 0 : 1;
    if (dev < 64 && !attr[kind][dev]) {
        PB_CUDA(cudaFuncSetAttribute(kind == 0 ? conv_tc_kernel<0> : conv_tc_kernel<1>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
        attr[kind][dev] = true;
    }
    if (kind == 0) conv_tc_kernel<0><<<grid, 192, smem, s>>>(tmA, tmB, p);
    else conv_tc_kernel<1><<<grid, 192, smem, s>>>(tmA, tmB, p);
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
