// Tensor-core stem convolution for BF16 precision: convs whose whole reduction
// (kh*kw*Cin, e.g. 27 for the 3x3 RGB stem) fits one 32-wide K slab.
//
// K is too small for a TMA operand stream, so the CTA's threads build the A tile
// themselves: thread m gathers the kh*kw*Cin input values of output pixel m (any
// input view; the fp32 NCHW graph input is read in place), converts them to bf16
// and writes one 64-byte K-major row (zero-padded to K = 32) into shared memory in
// the SWIZZLE_64B layout. One thread issues two tcgen05.mma (M = 128, K = 16 each)
// into a TMEM accumulator of Cout columns. The tile loop is double-buffered: while
// the tensor core works on tile t, the threads drain tile t-1 (tcgen05.ld, bias,
// activation, bf16 NHWC store). The weights sit in shared memory for the whole
// persistent CTA. Every mbarrier wait is bounded (error word + early exit).
#include <cuda.h>
#include <cstdlib>
#include <cstring>
#include <algorithm>

#include "common.h"
#include "device_common.cuh"

namespace pb {

namespace {

constexpr int kRows = 128;     // output pixels per tile (MMA M)
constexpr int kRowBytes = 64;  // 32 bf16 K values

__device__ __forceinline__ uint64_t sw64_desc(uint32_t addr) {
    // K-major, SWIZZLE_64B: 64-byte rows, 8-row groups 512 bytes apart (SBO).
    uint64_t d = 0;
    d |= (uint64_t)((addr & 0x3FFFF) >> 4);
    d |= (uint64_t)1 << 16;
    d |= (uint64_t)(512 >> 4) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)4 << 61;
    return d;
}

// Byte offset of 16-byte piece j of row r in a SWIZZLE_64B tile (512-byte aligned).
__device__ __forceinline__ uint32_t sw64_off(int r, int j) { return (uint32_t)(r * kRowBytes + ((j ^ ((r >> 1) & 3)) << 4)); }

__device__ __forceinline__ float stem_act(float x, int act, float slope) {
    if (act == ACT_SILU) {
        const float h = 0.5f * x;
        float t;
        asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(h));
        return fmaf(h, t, h);
    }
    return apply_act(x, act, slope, 0.0f);
}

struct StemParams {
    ConvArgs a;
    int Ho, Wo, K;
    int64_t M, tiles;
    int ncols;            // TMEM columns per accumulator (power of two >= cout)
    int* err;
};

// The K = kh*kw*Cin input values of output pixel m in (tap, channel) order, zero
// beyond K and outside the image. KH/KW/CIN > 0 fix the shape at compile time (the
// 3x3 RGB stem) so the values stay in registers.
template <int KH, int KW, int CIN>
__device__ __forceinline__ void gather_row(const ConvArgs& a, const StemParams& P, int64_t m, int H, int W,
                                           int64_t hw, float (&v)[32]) {
#pragma unroll
    for (int k = 0; k < 32; ++k) v[k] = 0.0f;
    if (m >= P.M) return;
    const int64_t b = m / hw, r = m - b * hw;
    const int ho = (int)(r / P.Wo), wo = (int)(r - (int64_t)ho * P.Wo);
    const int64_t ib = b * a.in.img_stride;
    if (KH > 0) {
#pragma unroll
        for (int kr = 0; kr < KH; ++kr) {
            const int hi = ho * a.sh - a.ph + kr * a.dh;
#pragma unroll
            for (int ks = 0; ks < KW; ++ks) {
                const int wi = wo * a.sw - a.pw + ks * a.dw;
                const bool in = hi >= 0 && hi < H && wi >= 0 && wi < W;
                const int64_t off = ib + (int64_t)hi * a.in.stride[1] + (int64_t)wi * a.in.stride[2];
#pragma unroll
                for (int c = 0; c < CIN; ++c)
                    v[(kr * KW + ks) * CIN + c] = in ? ld_elem(a.in.ptr, a.in.dt, off + (int64_t)c * a.in.stride[3]) : 0.0f;
            }
        }
    } else {
        float tmp[32];
        int k = 0;
        for (int kr = 0; kr < a.kh; ++kr) {
            const int hi = ho * a.sh - a.ph + kr * a.dh;
            for (int ks = 0; ks < a.kw; ++ks) {
                const int wi = wo * a.sw - a.pw + ks * a.dw;
                const bool in = hi >= 0 && hi < H && wi >= 0 && wi < W;
                const int64_t off = ib + (int64_t)hi * a.in.stride[1] + (int64_t)wi * a.in.stride[2];
                for (int c = 0; c < a.cin; ++c, ++k)
                    tmp[k] = in ? ld_elem(a.in.ptr, a.in.dt, off + (int64_t)c * a.in.stride[3]) : 0.0f;
            }
        }
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = j < k ? tmp[j] : 0.0f;
    }
}

template <int KH, int KW, int CIN>
__global__ void __launch_bounds__(128, 8) conv_stem_tc_kernel(const StemParams P) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t* const smem = smem_raw + (base - raw);
    const ConvArgs& a = P.a;
    const int cout = a.cout;
    uint8_t* const sA = smem;                               // 2 x 128 rows x 64 B
    uint8_t* const sB = smem + 2 * kRows * kRowBytes;       // cout rows x 64 B
    uint64_t* const mbar = reinterpret_cast<uint64_t*>(sB + ((cout * kRowBytes + 1023) & ~1023));   // [2]
    uint32_t* const tmem_slot = reinterpret_cast<uint32_t*>(mbar + 2);
    volatile int* const abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5;
    if (tid == 0) *abort_flag = *reinterpret_cast<volatile int*>(P.err) != 0;
    __syncthreads();
    if (*abort_flag) return;

    // weights: [kh][kw][cin][cout] fp32 -> B row n = output channel, K-major bf16
    const float* w = reinterpret_cast<const float*>(a.weight);
    for (int i = tid; i < cout * 32; i += blockDim.x) {
        const int n = i >> 5, k = i & 31;
        const float v = k < P.K ? w[(int64_t)k * cout + n] : 0.0f;
        __nv_bfloat16* row = reinterpret_cast<__nv_bfloat16*>(sB + sw64_off(n, k >> 3));
        row[k & 7] = __float2bfloat16_rn(v);
    }
    if (tid == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&mbar[0])) : "memory");
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&mbar[1])) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32(tmem_slot)), "r"(2 * P.ncols) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;
    // BF16 A/B, F32 accumulate, K-major both, N = cout, M = 128
    const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(cout >> 3) << 17) | ((uint32_t)(kRows >> 4) << 24);

    const int H = (int)a.in.shape[1], W = (int)a.in.shape[2];
    const int64_t hw = (int64_t)P.Ho * P.Wo;
    const bool vec_out = a.out.stride[3] == 1 && ((uintptr_t)a.out.ptr % 16) == 0 && (a.out.stride[2] % 8) == 0 &&
                         (a.out.stride[1] % 8) == 0 && (a.out.img_stride % 8) == 0;
    int64_t prev_tile = -1;
    int it = 0;
    bool failed = false;
    for (int64_t t = blockIdx.x;; t += gridDim.x, ++it) {
        const bool have = t < P.tiles;
        const int buf = it & 1;
        if (have) {
            // ---- gather: this thread's output pixel -> one A row (bf16, K padded to 32)
            const int64_t m = t * kRows + tid;
            float v[32];
            gather_row<KH, KW, CIN>(a, P, m, H, W, hw, v);
            uint8_t* const rowA = sA + buf * kRows * kRowBytes;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                uint32_t wd[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    __nv_bfloat162 h2 = __floats2bfloat162_rn(v[8 * j + 2 * q], v[8 * j + 2 * q + 1]);
                    wd[q] = *reinterpret_cast<uint32_t*>(&h2);
                }
                *reinterpret_cast<uint4*>(rowA + sw64_off(tid, j)) = make_uint4(wd[0], wd[1], wd[2], wd[3]);
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        }
        __syncthreads();
        if (have && tid == 0) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t a0 = smem_u32(sA + buf * kRows * kRowBytes), b0 = smem_u32(sB);
            const uint32_t d = tmem + (uint32_t)(buf * P.ncols);
            for (int k = 0; k < 2; ++k) {
                const uint64_t da = sw64_desc(a0 + 32u * k), db = sw64_desc(b0 + 32u * k);
                asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                             "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
                             ::"r"(d), "l"(da), "l"(db), "r"(idesc), "r"(k));
            }
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                         ::"r"(smem_u32(&mbar[buf])) : "memory");
        }
        // ---- drain the previous tile while this one is on the tensor core
        if (prev_tile >= 0) {
            const int pb = buf ^ 1;
            const uint32_t parity = (uint32_t)(((it - 1) >> 1) & 1);
            bool ok = mbar_wait_bounded(&mbar[pb], parity, 200000000LL);
            ok = __syncthreads_and(ok);
            if (!ok) {
                if (tid == 0) atomicExch(P.err, 8);
                failed = true;
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const int64_t m = prev_tile * kRows + tid;
            const bool live = m < P.M;
            int64_t ob = 0;
            if (live) {
                const int64_t b = m / hw, r = m - b * hw;
                const int64_t ho = r / P.Wo, wo = r - ho * P.Wo;
                ob = b * a.out.img_stride + ho * a.out.stride[1] + wo * a.out.stride[2];
            }
            const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(pb * P.ncols);
            for (int c0 = 0; c0 < cout; c0 += 16) {
                uint32_t r[16];
                asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                    : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                      "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
                    : "r"(taddr + (uint32_t)c0));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                if (!live) continue;
                float o[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    float x = __uint_as_float(r[i]) + (a.bias ? __ldg(a.bias + c0 + i) : 0.0f);
                    o[i] = stem_act(x, a.act, a.slope);
                }
                if (vec_out && a.out.dt == BF16) {
                    uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(const_cast<void*>(a.out.ptr)) + ob + c0);
#pragma unroll
                    for (int q = 0; q < 2; ++q) {
                        uint32_t wd[4];
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            __nv_bfloat162 h2 = __floats2bfloat162_rn(o[8 * q + 2 * j], o[8 * q + 2 * j + 1]);
                            wd[j] = *reinterpret_cast<uint32_t*>(&h2);
                        }
                        dst[q] = make_uint4(wd[0], wd[1], wd[2], wd[3]);
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < 16; ++i)
                        st_elem(const_cast<void*>(a.out.ptr), a.out.dt, ob + (int64_t)(c0 + i) * a.out.stride[3], o[i]);
                }
            }
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        }
        if (!have) break;
        prev_tile = t;
    }
    // Every issued MMA has completed once its tile was drained. On the error path the
    // MMAs of this iteration and the previous one may still run: wait (bounded) for
    // both before freeing TMEM.
    if (failed && tid == 0) {
        mbar_wait_bounded(&mbar[(it - 1) & 1], (uint32_t)(((it - 1) >> 1) & 1), 200000000LL);
        if ((int64_t)blockIdx.x + (int64_t)it * gridDim.x < P.tiles)
            mbar_wait_bounded(&mbar[it & 1], (uint32_t)((it >> 1) & 1), 200000000LL);
    }
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * P.ncols) : "memory");
    }
}

// The YOLO stem (3x3, stride 2, pad 1, Cin = 3, fp32 NCHW input with rows of a
// multiple of 4 floats) on 2-D tiles of 8 x 16 output pixels. The tile's input
// region, 17 rows of 33 columns per channel, is copied into shared memory as 9
// aligned 16-byte pieces per row (columns 32*tw - 4 ... 32*tw + 31; zero fill outside
// the image) with cp.async, one tile ahead, so the copy of tile t+1 overlaps the work
// on tile t. Thread m reads its 27 taps from shared memory at offsets fixed at compile
// time. The A rows, MMAs and epilogue are those of conv_stem_tc_kernel, so the
// outputs are identical; only the gather changes.
constexpr int kTileH = 8, kTileW = 16;
constexpr int kRegH = (kTileH - 1) * 2 + 3;     // 17 input rows
constexpr int kRegP = 9;                         // 16-byte pieces per region row (36 floats)
constexpr int kRegW = 4 * kRegP;
constexpr int kRegPlane = kRegH * kRegW;

// q = n / d for n < 2^31 as (n * m) >> p, p = 31 + ceil(log2 d), m = ceil(2^p / d)
// (Granlund and Montgomery, "Division by invariant integers using multiplication", 1994).
struct StemDiv {
    uint64_t m;
    uint32_t p, d;
};

StemDiv make_stem_div(uint32_t d) {
    uint32_t l = 0;
    while ((1ull << l) < d) ++l;
    StemDiv f;
    f.p = 31 + l;
    f.m = ((1ull << f.p) + d - 1) / d;      // p <= 62: no overflow
    f.d = d;
    return f;
}

__device__ __forceinline__ uint32_t stem_div(uint32_t n, const StemDiv& f) {
    return (uint32_t)(((uint64_t)n * f.m) >> f.p);   // n < 2^31, m <= 2^32 + 1: fits 64 bits
}

struct StemTileParams {
    ConvArgs a;
    const uint8_t* u8;    // 8-bit RGB frames instead of the fp32 input (U8 variant)
    float u8_scale;
    int Ho, Wo, K;
    int tiles_h, tiles_w;
    StemDiv div_img, div_tw;   // tile -> (image, tile row, tile column)
    int64_t tiles;
    int RH, RW;           // input region of one tile (rows, columns)
    int ncols;
    int* err;
    // fp32 input whose regions one thread loads as one TMA box (tensor map passed
    // beside the parameters) instead of 459 cp.async pieces from all threads
    int tma_region;
};

__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src, bool in) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(in ? 4 : 0) : "memory");
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool in) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(in ? 16 : 0) : "memory");
}

// Queue the input region of tile t into region buffer dst: 3 planes x 17 rows x 9
// pieces of 16 bytes, piece j of a row holding input columns 32*tw - 4 + 4j ... + 3.
__device__ __forceinline__ void stem_region_load(const StemTileParams& P, int64_t t, float* dst, int H, int W) {
    const ConvArgs& a = P.a;
    // tile counts stay below 2^31 (host-checked): 32-bit multiply-shift divisions
    const uint32_t b = stem_div((uint32_t)t, P.div_img);
    const int r = (int)((uint32_t)t - b * P.div_img.d);
    const int th = (int)stem_div((uint32_t)r, P.div_tw), tw = r - th * P.tiles_w;
    const int h0 = th * (2 * kTileH) - 1, c0 = tw * (2 * kTileW) - 4;
    const float* const in = static_cast<const float*>(a.in.ptr) + b * a.in.img_stride;
    for (int i = threadIdx.x; i < 3 * kRegH * kRegP; i += blockDim.x) {
        const int row = i / kRegP, j = i - row * kRegP;
        const int c = row / kRegH, y = row - c * kRegH;
        const int hi = h0 + y, wi = c0 + 4 * j;
        const bool ok = hi >= 0 && hi < H && wi >= 0 && wi < W;     // W % 4 == 0: pieces are all in or all out
        const float* src = ok ? in + (int64_t)hi * a.in.stride[1] + (int64_t)c * a.in.stride[3] + wi : in;
        cp_async16(smem_u32(dst + row * kRegW + 4 * j), src, ok);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
}

// The same region from 8-bit RGB frames [N, H, W, 3] (U8 variant): 17 rows of 36 pixels
// = 108 bytes, as 27 pieces of 4 bytes; W % 4 == 0 and the region starts at a multiple
// of 4 pixels, so each group of three pieces (four pixels) is all in or all out.
constexpr int kRegU8Row = kRegW * 3;                       // 108 bytes
// In shared memory a region row sits at pitch 112 and byte offset 4: the layout of a
// TMA box that starts 4 bytes earlier, at a 16-byte boundary (see stem_region_tma_u8)
constexpr int kRegU8Pitch = 112;
constexpr int kRegU8Off = 4;
constexpr int kRegU8Bytes = (kRegH * kRegU8Pitch + 127) & ~127;

__device__ __forceinline__ void cp_async4_u8(uint32_t dst, const void* src, bool in) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(in ? 4 : 0) : "memory");
}

__device__ __forceinline__ void stem_region_load_u8(const StemTileParams& P, int64_t t, uint8_t* dst, int H, int W) {
    const uint32_t b = stem_div((uint32_t)t, P.div_img);
    const int r = (int)((uint32_t)t - b * P.div_img.d);
    const int th = (int)stem_div((uint32_t)r, P.div_tw), tw = r - th * P.tiles_w;
    const int h0 = th * (2 * kTileH) - 1, c0 = tw * (2 * kTileW) - 4;
    const uint8_t* const img = P.u8 + (int64_t)b * H * W * 3;
    for (int i = threadIdx.x; i < kRegH * (kRegU8Row / 4); i += blockDim.x) {
        const int row = i / (kRegU8Row / 4), j = i - row * (kRegU8Row / 4);
        const int hi = h0 + row, px = c0 + 4 * (j / 3);
        const bool ok = hi >= 0 && hi < H && px >= 0 && px < W;
        const uint8_t* src = ok ? img + ((int64_t)hi * W + c0) * 3 + 4 * j : P.u8;
        cp_async4_u8(smem_u32(dst + row * kRegU8Pitch + kRegU8Off + 4 * j), src, ok);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
}

// Tile t's input region as one 4-D TMA box [36 columns, 17 rows, 3 planes, 1 image]
// of the NCHW fp32 input (the same layout stem_region_load produces; out-of-image
// elements read as zeros). The column origin 32*tw - 4 is a multiple of 4 floats, as
// TMA requires of the innermost coordinate. Issued by one thread.
__device__ __forceinline__ void stem_region_tma(const StemTileParams& P, const CUtensorMap* map, uint64_t* bar,
                                                float* dst, int64_t t) {
    const uint32_t b = stem_div((uint32_t)t, P.div_img);
    const int r = (int)((uint32_t)t - b * P.div_img.d);
    const int th = (int)stem_div((uint32_t)r, P.div_tw), tw = r - th * P.tiles_w;
    const int h0 = th * (2 * kTileH) - 1, c0 = tw * (2 * kTileW) - 4;
    mbar_expect_tx(bar, 3 * kRegPlane * 4);
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], [%2];"
        ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(h0), "r"(0),
          "r"((int)b)
        : "memory");
}

// The 8-bit frames' region as one 3-D TMA box [112 bytes, 17 rows, 1 image] of the
// [N, H, W*3] byte view: the region's 108 bytes start at byte 96*tw - 12, so the box
// starts 4 bytes earlier, at 96*tw - 16 (a 16-byte boundary, as TMA requires of the
// innermost coordinate; negative at the left edge, where it reads zeros).
__device__ __forceinline__ void stem_region_tma_u8(const StemTileParams& P, const CUtensorMap* map, uint64_t* bar,
                                                   uint8_t* dst, int64_t t) {
    const uint32_t b = stem_div((uint32_t)t, P.div_img);
    const int r = (int)((uint32_t)t - b * P.div_img.d);
    const int th = (int)stem_div((uint32_t)r, P.div_tw), tw = r - th * P.tiles_w;
    const int h0 = th * (2 * kTileH) - 1, x0 = (tw * (2 * kTileW) - 4) * 3 - kRegU8Off;
    mbar_expect_tx(bar, kRegH * kRegU8Pitch);
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];"
        ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x0), "r"(h0), "r"((int)b)
        : "memory");
}

template <bool U8>
__global__ void __launch_bounds__(128, 8) conv_stem_tile_kernel(const StemTileParams P,
                                                                 const __grid_constant__ CUtensorMap tmR) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 511u) & ~511u;
    uint8_t* const smem = smem_raw + (base - raw);
    const ConvArgs& a = P.a;
    const int cout = a.cout;
    // [A: 128 rows x 64 B | B: cout rows x 64 B | region x 2 | barrier, TMEM slot, flag]
    uint8_t* const sA = smem;
    uint8_t* const sB = smem + kRows * kRowBytes;
    // region slots 128-byte aligned (TMA destinations): 7344 bytes of fp32 region -> 7424
    constexpr int rbytes = U8 ? kRegU8Bytes : ((3 * kRegPlane * 4 + 127) & ~127);
    float* const sR0 = reinterpret_cast<float*>(sB + ((cout * kRowBytes + 511) & ~511));
    float* const sR1 = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(sR0) + rbytes);
    uint64_t* const mbar = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(sR1) + rbytes);
    uint32_t* const tmem_slot = reinterpret_cast<uint32_t*>(mbar + 1);
    volatile int* const abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    float* const sBias = reinterpret_cast<float*>(mbar + 2);     // [cout], 16-byte aligned
    uint64_t* const rbar = reinterpret_cast<uint64_t*>(sBias + ((cout + 3) & ~3));   // [2] region slots (TMA)
    const bool tma = P.tma_region != 0;

    const int tid = threadIdx.x, warp = tid >> 5;
    if (tid == 0) *abort_flag = *reinterpret_cast<volatile int*>(P.err) != 0;
    __syncthreads();
    if (*abort_flag) return;

    const int H = (int)a.in.shape[1], W = (int)a.in.shape[2];
    // TMA region loads: issued / consumed counts (load k uses slot k & 1, phase k >> 1)
    int r_issued = 0, r_done = 0;
    if (tma && tid == 0) {
        mbar_init(&rbar[0], 1);
        mbar_init(&rbar[1], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if ((int64_t)blockIdx.x < P.tiles) {
        if (tma) {
            if (tid == 0) {
                if (U8) stem_region_tma_u8(P, &tmR, &rbar[0], reinterpret_cast<uint8_t*>(sR0), blockIdx.x);
                else stem_region_tma(P, &tmR, &rbar[0], sR0, blockIdx.x);
            }
        } else if (U8) {
            stem_region_load_u8(P, blockIdx.x, reinterpret_cast<uint8_t*>(sR0), H, W);
        } else {
            stem_region_load(P, blockIdx.x, sR0, H, W);
        }
        r_issued = tma ? 1 : 0;
    }

    const float* w = reinterpret_cast<const float*>(a.weight);
    for (int i = tid; i < cout * 32; i += blockDim.x) {
        const int n = i >> 5, k = i & 31;
        const float v = k < P.K ? w[(int64_t)k * cout + n] : 0.0f;
        __nv_bfloat16* row = reinterpret_cast<__nv_bfloat16*>(sB + sw64_off(n, k >> 3));
        row[k & 7] = __float2bfloat16_rn(v);
    }
    for (int i = tid; i < cout; i += blockDim.x) sBias[i] = a.bias ? a.bias[i] : 0.0f;
    if (tid == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(mbar)) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32(tmem_slot)), "r"(P.ncols) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;
    const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(cout >> 3) << 17) | ((uint32_t)(kRows >> 4) << 24);

    const int py = tid / kTileW, px = tid - py * kTileW;
    const bool fast_epi = cout == 16 && a.act == ACT_SILU && a.out.dt == BF16 && a.out.stride[3] == 1 &&
                          ((uintptr_t)a.out.ptr % 16) == 0 && (a.out.stride[2] % 8) == 0 && (a.out.stride[1] % 8) == 0 &&
                          (a.out.img_stride % 8) == 0;
    const int rbase = 2 * py * kRegW + 2 * px + 3;          // this pixel's first tap (column 2*px - 1 -> piece offset 3)
    const bool vec_out = a.out.stride[3] == 1 && ((uintptr_t)a.out.ptr % 16) == 0 && (a.out.stride[2] % 8) == 0 &&
                         (a.out.stride[1] % 8) == 0 && (a.out.img_stride % 8) == 0;
    const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16);
    int it = 0;
    bool failed = false;
    for (int64_t t = blockIdx.x; t < P.tiles; t += gridDim.x, ++it) {
        // queue the next tile's region, then wait for this one's
        const int64_t tn = t + gridDim.x;
        float* const cur = (it & 1) ? sR1 : sR0;
        float* const nxt = (it & 1) ? sR0 : sR1;
        if (tn < P.tiles) {
            if (tma) {
                if (tid == 0) {
                    // the slot's previous region was read (generic proxy) before the
                    // last barrier; order those reads before the async-proxy write
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    if (U8) stem_region_tma_u8(P, &tmR, &rbar[r_issued & 1], reinterpret_cast<uint8_t*>(nxt), tn);
                    else stem_region_tma(P, &tmR, &rbar[r_issued & 1], nxt, tn);
                }
                ++r_issued;
            } else if (U8) {
                stem_region_load_u8(P, tn, reinterpret_cast<uint8_t*>(nxt), H, W);
            } else {
                stem_region_load(P, tn, nxt, H, W);
            }
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        bool rok = true;
        if (tma) {
            rok = mbar_wait_bounded(&rbar[r_done & 1], (uint32_t)((r_done >> 1) & 1), 200000000LL);
            ++r_done;
        }
        rok = __syncthreads_and(rok);     // region visible; previous tile's TMEM reads finished
        if (!rok) {
            if (tid == 0) atomicExch(P.err, 9);
            --r_done;
            break;
        }
        {
            float v[32];
            if (U8) {
                // pixel * scale: the identity letterbox's value, bit for bit
                const uint8_t* cu =
                    reinterpret_cast<const uint8_t*>(cur) + 2 * py * kRegU8Pitch + kRegU8Off + (2 * px + 3) * 3;
#pragma unroll
                for (int kr = 0; kr < 3; ++kr)
#pragma unroll
                    for (int ks = 0; ks < 3; ++ks)
#pragma unroll
                        for (int c = 0; c < 3; ++c)
                            v[(kr * 3 + ks) * 3 + c] = __fmul_rn((float)cu[kr * kRegU8Pitch + ks * 3 + c], P.u8_scale);
            } else {
#pragma unroll
                for (int c = 0; c < 3; ++c)
#pragma unroll
                    for (int kr = 0; kr < 3; ++kr)
#pragma unroll
                        for (int ks = 0; ks < 3; ++ks)
                            v[(kr * 3 + ks) * 3 + c] = cur[rbase + c * kRegPlane + kr * kRegW + ks];
            }
#pragma unroll
            for (int k = 27; k < 32; ++k) v[k] = 0.0f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                uint32_t wd[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    __nv_bfloat162 h2 = __floats2bfloat162_rn(v[8 * j + 2 * q], v[8 * j + 2 * q + 1]);
                    wd[q] = *reinterpret_cast<uint32_t*>(&h2);
                }
                *reinterpret_cast<uint4*>(sA + sw64_off(tid, j)) = make_uint4(wd[0], wd[1], wd[2], wd[3]);
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        }
        __syncthreads();          // A rows complete; region `cur` free for the load after next
        if (tid == 0) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t a0 = smem_u32(sA), b0 = smem_u32(sB);
            for (int k = 0; k < 2; ++k) {
                const uint64_t da = sw64_desc(a0 + 32u * k), db = sw64_desc(b0 + 32u * k);
                asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                             "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
                             ::"r"(tmem), "l"(da), "l"(db), "r"(idesc), "r"(k));
            }
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                         ::"r"(smem_u32(mbar)) : "memory");
        }
        // one warp waits for the MMAs; the others wait at the barrier without issuing
        bool ok = true;
        if (warp == 0) ok = mbar_wait_bounded(mbar, (uint32_t)(it & 1), 200000000LL);
        ok = __syncthreads_and(ok);
        if (!ok) {
            if (tid == 0) atomicExch(P.err, 8);
            failed = true;
            break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t b = stem_div((uint32_t)t, P.div_img);
        const int r = (int)((uint32_t)t - b * P.div_img.d);
        const int th = (int)stem_div((uint32_t)r, P.div_tw), tw = r - th * P.tiles_w;
        const int ho = th * kTileH + py, wo = tw * kTileW + px;
        const bool live = ho < P.Ho && wo < P.Wo;
        const int64_t ob = b * a.out.img_stride + (int64_t)ho * a.out.stride[1] + (int64_t)wo * a.out.stride[2];
        for (int c0 = 0; c0 < cout; c0 += 16) {
            uint32_t rr[16];
            asm volatile(
                "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                : "=r"(rr[0]), "=r"(rr[1]), "=r"(rr[2]), "=r"(rr[3]), "=r"(rr[4]), "=r"(rr[5]), "=r"(rr[6]), "=r"(rr[7]),
                  "=r"(rr[8]), "=r"(rr[9]), "=r"(rr[10]), "=r"(rr[11]), "=r"(rr[12]), "=r"(rr[13]), "=r"(rr[14]), "=r"(rr[15])
                : "r"(taddr + (uint32_t)c0));
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
            if (!live) continue;
            float o[16];
            float bv[16];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float4 b4 = reinterpret_cast<const float4*>(sBias + c0)[q];
                bv[4 * q] = b4.x; bv[4 * q + 1] = b4.y; bv[4 * q + 2] = b4.z; bv[4 * q + 3] = b4.w;
            }
            if (fast_epi) {
                // bias + SiLU (x/2 + x/2 tanh(x/2)) on the packed fp32x2 pipe
#pragma unroll
                for (int i = 0; i < 16; i += 2) {
                    const float2 x = __fadd2_rn(make_float2(__uint_as_float(rr[i]), __uint_as_float(rr[i + 1])),
                                                make_float2(bv[i], bv[i + 1]));
                    const float2 h = __fmul2_rn(x, make_float2(0.5f, 0.5f));
                    float t0, t1;
                    asm("tanh.approx.f32 %0, %1;" : "=f"(t0) : "f"(h.x));
                    asm("tanh.approx.f32 %0, %1;" : "=f"(t1) : "f"(h.y));
                    const float2 y = __ffma2_rn(h, make_float2(t0, t1), h);
                    o[i] = y.x;
                    o[i + 1] = y.y;
                }
            } else {
#pragma unroll
                for (int i = 0; i < 16; ++i) o[i] = stem_act(__uint_as_float(rr[i]) + bv[i], a.act, a.slope);
            }
            if (vec_out && a.out.dt == BF16) {
                uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(const_cast<void*>(a.out.ptr)) + ob + c0);
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    uint32_t wd[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        __nv_bfloat162 h2 = __floats2bfloat162_rn(o[8 * q + 2 * j], o[8 * q + 2 * j + 1]);
                        wd[j] = *reinterpret_cast<uint32_t*>(&h2);
                    }
                    dst[q] = make_uint4(wd[0], wd[1], wd[2], wd[3]);
                }
            } else {
#pragma unroll
                for (int i = 0; i < 16; ++i)
                    st_elem(const_cast<void*>(a.out.ptr), a.out.dt, ob + (int64_t)(c0 + i) * a.out.stride[3], o[i]);
            }
        }
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    if (failed && tid == 0) mbar_wait_bounded(mbar, (uint32_t)(it & 1), 200000000LL);
    // no region copy may still be landing when the CTA exits (after a failed wait)
    if (tid == 0)
        for (int k = r_done; k < r_issued; ++k) mbar_wait_bounded(&rbar[k & 1], (uint32_t)((k >> 1) & 1), 200000000LL);
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(P.ncols) : "memory");
    }
}

}  // namespace

bool conv_stem_tc_supported(const ConvArgs& a) {
    return a.kh * a.kw * a.cin <= 32 && a.cout % 16 == 0 && a.cout >= 16 && a.cout <= 256 && !a.res.ptr &&
           a.out.dt == BF16 && (a.act >= ACT_NONE && a.act <= ACT_SILU);
}

void launch_conv_stem_tc(const ConvArgs& a, int* err, cudaStream_t s) {
    if (!conv_stem_tc_supported(a)) fail(ENGINE_ERR_INVALID_ARG, "conv_stem_tc: layer not supported");
    StemParams P;
    P.a = a;
    P.Ho = (int)a.out.shape[1];
    P.Wo = (int)a.out.shape[2];
    P.K = a.kh * a.kw * a.cin;
    P.M = a.batch * P.Ho * P.Wo;
    if (P.M == 0) return;
    P.ncols = 32;
    while (P.ncols < a.cout) P.ncols <<= 1;
    int dev0 = 0;
    PB_CUDA(cudaGetDevice(&dev0));
    const int esz_in = 4;
    const bool u8 = a.in_u8 != nullptr;
    const bool geom = a.kh == 3 && a.kw == 3 && a.cin == 3 && a.sh == 2 && a.sw == 2 && a.ph == 1 && a.pw == 1 &&
                      a.dh == 1 && a.dw == 1 && a.in.shape[2] % 4 == 0;
    if (u8 && !(geom && ((uintptr_t)a.in_u8 % 4) == 0))
        fail(ENGINE_ERR_NOT_IMPL, "conv_stem_tc: 8-bit input needs a 3x3 stride-2 RGB stem with W % 4 == 0");
    if (geom && (u8 || (a.in.dt == F32 && a.in.stride[2] == 1 && ((uintptr_t)a.in.ptr % 16) == 0 &&
                        (a.in.stride[1] * esz_in) % 16 == 0 && (a.in.stride[3] * esz_in) % 16 == 0 &&
                        (a.in.img_stride * esz_in) % 16 == 0))) {
        StemTileParams T;
        T.a = a;
        T.u8 = a.in_u8;
        T.u8_scale = a.in_u8_scale;
        T.Ho = P.Ho; T.Wo = P.Wo; T.K = P.K;
        T.tiles_h = (P.Ho + kTileH - 1) / kTileH;
        T.tiles_w = (P.Wo + kTileW - 1) / kTileW;
        T.tiles = (int64_t)T.tiles_h * T.tiles_w * a.batch;
        T.div_img = make_stem_div((uint32_t)(T.tiles_h * T.tiles_w));
        T.div_tw = make_stem_div((uint32_t)T.tiles_w);
        T.RH = kRegH;
        T.RW = kRegW;
        T.ncols = P.ncols;
        T.err = err;
        // fp32 input: each tile's region as one TMA box (dims W, H, planes, images); one
        // instruction of one thread instead of 459 cp.async pieces with their index
        // arithmetic on all 128 threads (the kernel was issue bound): 0.608 -> 0.445 ms
        // for 256 images
        alignas(64) CUtensorMap tmR;
        std::memset(&tmR, 0, sizeof(tmR));
        T.tma_region = 0;
        if (!u8) {
            const uint64_t dims[4] = {(uint64_t)a.in.shape[2], (uint64_t)a.in.shape[1], 3, (uint64_t)a.batch};
            const uint64_t st[3] = {(uint64_t)(a.in.stride[1] * esz_in), (uint64_t)(a.in.stride[3] * esz_in),
                                    (uint64_t)(a.in.img_stride * esz_in)};
            const uint32_t box[4] = {(uint32_t)kRegW, (uint32_t)kRegH, 3, 1};
            T.tma_region = encode_box_map(&tmR, 4, 4, a.in.ptr, dims, st, box) ? 1 : 0;
        } else if (((uintptr_t)a.in_u8 % 16) == 0 && (a.in.shape[2] * 3) % 16 == 0) {
            // [N, H, W*3] bytes: rows of W*3 bytes (a multiple of 16), images of H*W*3
            const int64_t Wb = a.in.shape[2] * 3, Hh = a.in.shape[1];
            const uint64_t dims[3] = {(uint64_t)Wb, (uint64_t)Hh, (uint64_t)a.batch};
            const uint64_t st[2] = {(uint64_t)Wb, (uint64_t)(Wb * Hh)};
            const uint32_t box[3] = {(uint32_t)kRegU8Pitch, (uint32_t)kRegH, 1};
            T.tma_region = encode_box_map(&tmR, 1, 3, a.in_u8, dims, st, box) ? 1 : 0;
        }
        const size_t rbytes = u8 ? (size_t)kRegU8Bytes : (size_t)((3 * kRegPlane * 4 + 127) & ~127);
        // tail: barrier, TMEM slot, flag (16 B), the biases (cout floats), the two
        // region barriers (16 B, inside the 48 B of slack)
        const size_t smem = 512 + kRows * kRowBytes + ((a.cout * kRowBytes + 511) & ~511) + 2 * rbytes + 16 +
                            (((size_t)a.cout * 4 + 15) & ~size_t(15)) + 48;
        if (smem <= 48 * 1024 && T.tiles < (int64_t(1) << 31)) {
            static int sms_t[64] = {};
            int sms = 148;
            if (dev0 < 64) {
                if (!sms_t[dev0]) PB_CUDA(cudaDeviceGetAttribute(&sms_t[dev0], cudaDevAttrMultiProcessorCount, dev0));
                sms = sms_t[dev0];
            }
            // resident CTAs per SM: 8 by registers (64 a thread), 228 KB of shared memory
            // (1 KB reserved per CTA), TMEM ncols columns each within 512
            const int by_smem = (int)((228u * 1024u) / (smem + 1024));
            const int per_sm = std::max(1, std::min({8, by_smem, 512 / T.ncols}));
            const int64_t grid = std::min<int64_t>(T.tiles, (int64_t)sms * per_sm);
            if (u8) conv_stem_tile_kernel<true><<<(unsigned)grid, 128, smem, s>>>(T, tmR);
            else conv_stem_tile_kernel<false><<<(unsigned)grid, 128, smem, s>>>(T, tmR);
            PB_CUDA(cudaGetLastError());
            return;
        }
    }
    if (u8) fail(ENGINE_ERR_NOT_IMPL, "conv_stem_tc: 8-bit input needs the tiled stem kernel");
    P.tiles = (P.M + kRows - 1) / kRows;
    P.ncols = 32;
    while (P.ncols < a.cout) P.ncols <<= 1;
    P.err = err;
    const size_t smem = 1024 + 2 * kRows * kRowBytes + ((a.cout * kRowBytes + 1023) & ~1023) + 64;
    int dev = 0;
    PB_CUDA(cudaGetDevice(&dev));
    static int sm_count[64] = {};
    int sms = 148;
    if (dev < 64) {
        if (!sm_count[dev]) PB_CUDA(cudaDeviceGetAttribute(&sm_count[dev], cudaDevAttrMultiProcessorCount, dev));
        sms = sm_count[dev];
    }
    // Each CTA works its tiles one after another (gather, MMA, drain), so throughput
    // comes from CTAs per SM: up to 8 (64 registers a thread), TMEM 2 * ncols columns
    // each within 512.
    const int per_sm = std::max(1, std::min(8, 512 / (2 * P.ncols)));
    const int64_t grid = std::min<int64_t>(P.tiles, (int64_t)sms * per_sm);
    if (a.kh == 3 && a.kw == 3 && a.cin == 3) conv_stem_tc_kernel<3, 3, 3><<<(unsigned)grid, 128, smem, s>>>(P);
    else conv_stem_tc_kernel<0, 0, 0><<<(unsigned)grid, 128, smem, s>>>(P);
    PB_CUDA(cudaGetLastError());
}

}  // namespace pb
