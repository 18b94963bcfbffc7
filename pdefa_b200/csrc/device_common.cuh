// Device-side helpers shared by the kernels: element load/store for fp32/bf16,
// strided-view indexing, activations and bounded mbarrier waits.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "kernels.h"

namespace pb {

__device__ __forceinline__ float ld_elem(const void* p, int dt, int64_t i) {
    return dt == BF16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i])
                      : reinterpret_cast<const float*>(p)[i];
}
__device__ __forceinline__ void st_elem(void* p, int dt, int64_t i, float v) {
    if (dt == BF16) reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
    else reinterpret_cast<float*>(p)[i] = v;
}

// Offset of linear element `i` (row-major over v.shape) inside one image of view v.
__device__ __forceinline__ int64_t view_offset(const TView& v, int64_t i) {
    int64_t off = 0;
    for (int d = v.rank - 1; d >= 0; --d) {
        const int64_t n = v.shape[d];
        const int64_t q = i / n;
        off += (i - q * n) * v.stride[d];
        i = q;
    }
    return off;
}

// SiLU with an accurate exponential (the reference's direct and GEMM conv paths
// use a Cephes-style expf accurate to ~1 ulp: conv2d_avx2.cpp:48-88, 01_math.inc:9-56).
__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }

// SiLU exactly as the reference's Winograd epilogue evaluates it
// (PDEFA1.0/src/kernels/simd/avx2/conv2d_winograd.cpp:81-101): with
// t = -x*log2(e), n = round(t), f = t - n, it forms q(f) = 1 + f/2 + f^2/6 + ...
// (degree-6 Horner with the listed coefficients) and returns x / (1 + q(f)*2^n),
// where 2^n is built from the exponent bits of (n + 127). Outside |x| <= 88.37626
// it returns x (large x) or 0 (very negative x). Horner steps are fused
// multiply-adds, as the reference is compiled with -ffp-contract=fast.
__device__ __forceinline__ float silu_wino_f(float x) {
    const float nx = -x;
    if (nx < -88.37626f) return x;
    if (nx > 88.37626f) return 0.0f;
    const float fx = nx * 1.44269504088896341f;
    const float n = roundf(fx);
    const float f = fx - n;
    float p = 1.9875691500e-4f;
    p = fmaf(p, f, 1.3981999507e-3f);
    p = fmaf(p, f, 8.3334519073e-3f);
    p = fmaf(p, f, 4.1665795894e-2f);
    p = fmaf(p, f, 1.6666665459e-1f);
    p = fmaf(p, f, 5.0000001201e-1f);
    p = fmaf(p, f, 1.0f);
    const uint32_t bits = (uint32_t)((int32_t)n + 127) << 23;
    const float scale = __uint_as_float(bits);
    return x / fmaf(p, scale, 1.0f);
}

// The same flavour for the BF16/TF32 epilogues (results held to 1e-2): branch-free,
// round-to-nearest-even for n (differs from round-half-away only at exact ties, where
// both neighbours are valid results of the flavour's jump), n clamped so 2^n stays a
// normal float, and an approximate divide (~2 ulp).
__device__ __forceinline__ float silu_wino_fast(float x) {
    const float fx = -x * 1.44269504088896341f;
    const float n = fminf(fmaxf(rintf(fx), -126.0f), 127.0f);
    const float f = fx - n;
    float p = 1.9875691500e-4f;
    p = fmaf(p, f, 1.3981999507e-3f);
    p = fmaf(p, f, 8.3334519073e-3f);
    p = fmaf(p, f, 4.1665795894e-2f);
    p = fmaf(p, f, 1.6666665459e-1f);
    p = fmaf(p, f, 5.0000001201e-1f);
    p = fmaf(p, f, 1.0f);
    const float scale = __int_as_float(((int)n + 127) << 23);
    float y = __fdividef(x, fmaf(p, scale, 1.0f));
    y = x > 88.37626f ? x : y;
    y = x < -88.37626f ? 0.0f : y;
    return y;
}

// The same flavour on two values with the packed fp32x2 pipe of sm_100, in about 20
// instructions per pair (the epilogue of the 3x3 convs spends most of its issue slots
// here):
//   * t = -x*log2(e) is clamped to [-127, 127] first, so no range selects are needed:
//     t = -127 gives n = -127, whose exponent field (n + 127) << 23 is 0, so 2^n reads
//     as 0 and y = x (the flavour returns x above 88.37626); t = 127 gives
//     den = 1 + 2^127 and y = x * rcp(den), which the flush-to-zero reciprocal makes
//     0 (the flavour returns 0 below -88.37626);
//   * n = rint(t) by the 1.5 * 2^23 magic-number addition (round to nearest even,
//     exact for |t| < 2^22); the sum's bit pattern is 0x4B400000 + n, and
//     (0x4B400000 << 23) vanishes mod 2^32, so the exponent field of 2^n is
//     (bits + 127) << 23 with no float-to-int conversion;
//   * the divide is an approximate reciprocal (rcp.approx.ftz) and a packed multiply.
// Inside |x| <= 88 the steps match silu_wino_fast (same polynomial, same fused
// multiply-adds, ~2 ulp divide).
__device__ __forceinline__ float rcp_approx_ftz(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float2 silu_wino_fast2(float2 x) {
    const float kMagic = 12582912.0f;   // 1.5 * 2^23
    float2 t = __fmul2_rn(x, make_float2(-1.44269504088896341f, -1.44269504088896341f));
    t.x = fminf(fmaxf(t.x, -127.0f), 127.0f);
    t.y = fminf(fmaxf(t.y, -127.0f), 127.0f);
    const float2 tm = __fadd2_rn(t, make_float2(kMagic, kMagic));
    // -n = M - tm (exact: both are within 2^7 of M), then f = t - n
    const float2 neg_n = __ffma2_rn(tm, make_float2(-1.0f, -1.0f), make_float2(kMagic, kMagic));
    const float2 f = __fadd2_rn(t, neg_n);
    float2 p = make_float2(1.9875691500e-4f, 1.9875691500e-4f);
    p = __ffma2_rn(p, f, make_float2(1.3981999507e-3f, 1.3981999507e-3f));
    p = __ffma2_rn(p, f, make_float2(8.3334519073e-3f, 8.3334519073e-3f));
    p = __ffma2_rn(p, f, make_float2(4.1665795894e-2f, 4.1665795894e-2f));
    p = __ffma2_rn(p, f, make_float2(1.6666665459e-1f, 1.6666665459e-1f));
    p = __ffma2_rn(p, f, make_float2(5.0000001201e-1f, 5.0000001201e-1f));
    p = __ffma2_rn(p, f, make_float2(1.0f, 1.0f));
    const float2 scale = make_float2(__uint_as_float((__float_as_uint(tm.x) + 127u) << 23),
                                     __uint_as_float((__float_as_uint(tm.y) + 127u) << 23));
    const float2 den = __ffma2_rn(p, scale, make_float2(1.0f, 1.0f));
    return __fmul2_rn(x, make_float2(rcp_approx_ftz(den.x), rcp_approx_ftz(den.y)));
}

__device__ __forceinline__ float apply_act(float v, int act, float p0, float p1) {
    switch (act) {
        case ACT_RELU: return v > 0.0f ? v : 0.0f;
        case ACT_LEAKY: return v > 0.0f ? v : p0 * v;
        case ACT_SIGMOID: return 1.0f / (1.0f + expf(-v));
        case ACT_GELU_TANH: {
            const float inner = 0.7978845608f * (v + 0.044715f * v * v * v);
            return 0.5f * v * (1.0f + tanhf(inner));
        }
        case ACT_SILU: return silu_f(v);
        case ACT_SILU_WINO: return silu_wino_f(v);
        case UN_TANH: return tanhf(v);
        case UN_GELU: return 0.5f * v * (1.0f + erff(v * 0.70710678118654752f));
        case UN_HARDSWISH: {
            float t = v * (1.0f / 6.0f) + 0.5f;
            t = t < 0.0f ? 0.0f : (t > 1.0f ? 1.0f : t);
            return v * t;
        }
        case UN_HARDSIGMOID: {
            float t = v * (1.0f / 6.0f) + 0.5f;
            return t < 0.0f ? 0.0f : (t > 1.0f ? 1.0f : t);
        }
        case UN_CLIP: return v < p0 ? p0 : (v > p1 ? p1 : v);
        default: return v;
    }
}

// ---------------------------------------------------------------------------
// mbarrier helpers (shared::cta addresses) with bounded waits.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
    return ok != 0;
}
// Waits for the phase with the given parity to complete; gives up after roughly
// `limit_cycles` SM clocks and returns false (the caller records the error).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  long long limit_cycles = 1000000000LL) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > limit_cycles) return false;
    }
    return true;
}

}  // namespace pb
