// GPU letterbox preprocess: 8-bit images -> float32 NCHW model input.
//
// Replaces imageloader/src/preprocess.cpp:15-147 (preprocess_letterbox_direct) for
// images already decoded to 8-bit pixels, with the same arithmetic, so the results
// are bit-identical to the reference build:
//   ratio  = min(W / src_w, H / src_h), scaled = clamp(round(src * ratio), 1, target),
//   pad    = (target - scaled) / 2, inv = 1 / ratio                    (host, :27-54)
//   sx = dx * inv, x0 = (int)sx (clamped to src_w - 2), x1 = min(x0 + 1, src_w - 1),
//   fx = sx - x0; the same per row with wy0 = (1 - fy) * scale, wy1 = fy * scale
//   value = fma(fma(p00, w0, p10 * w1), wy0, fma(p01, w0, p11 * w1) * wy1)  (:59-108)
// The nested fma is the value the reference's -ffp-contract=fast build computes for
// (p00*w0 + p10*w1)*wy0 + (p01*w0 + p11*w1)*wy1; every operation below is an explicit
// round-to-nearest intrinsic so that nvcc contracts nothing else.
// Gray images are replicated to the three planes, RGBA drops alpha, pad_value fills
// the border.
//
// One thread writes four consecutive output pixels of one row (three planes); rows
// are grid.y and images grid.z, so the three plane stores of a warp are coalesced
// 512-byte runs. The kernel is bound by the float32 output (12 bytes per pixel).
#include <algorithm>
#include <cmath>
#include <cstdint>

#include "common.h"
#include "kernels.h"

namespace pb {

namespace {

template <int CH>
__device__ __forceinline__ float tap(const uint8_t* __restrict__ row, int x, int c) {
    return (float)__ldg(row + (size_t)x * CH + (CH == 1 ? 0 : c));
}

template <int CH, bool VEC>
__global__ void __launch_bounds__(128) letterbox_kernel(const uint8_t* __restrict__ src, float* __restrict__ out,
                                                        LetterboxGeom g) {
    const int y = blockIdx.y;
    const int64_t b = blockIdx.z;
    const int x0p = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (x0p >= g.W) return;
    const size_t plane = (size_t)g.W * g.H;
    float* const o = out + b * 3 * plane + (size_t)y * g.W;
    const uint8_t* const img = src + (size_t)b * g.src_h * g.src_w * CH;
    float v[3][4];
    const int dy = y - g.py;
    const bool row_in = dy >= 0 && dy < g.sh;
    const uint8_t *r0 = img, *r1 = img;
    float wy0 = 0.f, wy1 = 0.f;
    if (row_in) {
        const float sy = __fmul_rn((float)dy, g.inv);
        int yy0 = __float2int_rz(sy);
        if (yy0 > g.src_h - 2 && g.src_h > 1) yy0 = g.src_h - 2;
        const int yy1 = yy0 + 1 < g.src_h ? yy0 + 1 : yy0;
        const float fy = __fsub_rn(sy, (float)yy0);
        wy0 = __fmul_rn(__fsub_rn(1.0f, fy), g.scale);
        wy1 = __fmul_rn(fy, g.scale);
        r0 = img + (size_t)yy0 * g.src_w * CH;
        r1 = img + (size_t)yy1 * g.src_w * CH;
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int dx = x0p + k - g.px;
        if (row_in && dx >= 0 && dx < g.sw) {
            const float sx = __fmul_rn((float)dx, g.inv);
            int xa = __float2int_rz(sx);
            if (xa > g.src_w - 2 && g.src_w > 1) xa = g.src_w - 2;
            const int xb = xa + 1 < g.src_w ? xa + 1 : xa;
            const float fx = __fsub_rn(sx, (float)xa);
            const float w0 = __fsub_rn(1.0f, fx), w1 = fx;
#pragma unroll
            for (int c = 0; c < 3; ++c) {
                const float top = __fmaf_rn(tap<CH>(r0, xa, c), w0, __fmul_rn(tap<CH>(r0, xb, c), w1));
                const float bot = __fmaf_rn(tap<CH>(r1, xa, c), w0, __fmul_rn(tap<CH>(r1, xb, c), w1));
                v[c][k] = __fmaf_rn(top, wy0, __fmul_rn(bot, wy1));
            }
        } else {
#pragma unroll
            for (int c = 0; c < 3; ++c) v[c][k] = g.pad;
        }
    }
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        float* const dst = o + c * plane + x0p;
        if (VEC) {
            __stcs(reinterpret_cast<float4*>(dst), make_float4(v[c][0], v[c][1], v[c][2], v[c][3]));
        } else {
#pragma unroll
            for (int k = 0; k < 4; ++k)
                if (x0p + k < g.W) dst[k] = v[c][k];
        }
    }
}

// Identity geometry (the image already has the target size: ratio 1, no border). The
// blend above then reduces exactly to one product per sample: inside the image fx = fy
// = 0, so top = fma(p00, 1, p10 * 0) = p00 and value = fma(p00, scale, bot * 0) =
// round(p00 * scale); on the last column (row) the clamped index gives fx (fy) = 1, so
// the weights select p10 (the bottom row) exactly and the same single rounding follows.
// One thread converts four pixels (one 12-byte RGB read) into three float4 stores.
template <int CH>
__global__ void __launch_bounds__(128) letterbox_identity_kernel(const uint8_t* __restrict__ src,
                                                                 float* __restrict__ out, LetterboxGeom g) {
    const int y = blockIdx.y;
    const int64_t b = blockIdx.z;
    const int x0p = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (x0p >= g.W) return;
    const size_t plane = (size_t)g.W * g.H;
    const uint8_t* const row = src + ((size_t)b * g.H + y) * g.W * CH + (size_t)x0p * CH;
    uint8_t px[4 * CH];
    if (CH == 3) {
        const uint32_t* w = reinterpret_cast<const uint32_t*>(row);     // 4-byte aligned: W % 4 == 0
        const uint32_t a = __ldcs(w), bb = __ldcs(w + 1), c = __ldcs(w + 2);
        const uint32_t u[3] = {a, bb, c};
#pragma unroll
        for (int i = 0; i < 12; ++i) px[i] = (uint8_t)(u[i >> 2] >> (8 * (i & 3)));
    } else if (CH == 4) {
        const uint4 q = __ldcs(reinterpret_cast<const uint4*>(row));     // 16-byte aligned: W % 4 == 0
        const uint32_t u[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int i = 0; i < 16; ++i) px[i] = (uint8_t)(u[i >> 2] >> (8 * (i & 3)));
    } else {
        const uint32_t a = __ldcs(reinterpret_cast<const uint32_t*>(row));
#pragma unroll
        for (int i = 0; i < 4; ++i) px[i] = (uint8_t)(a >> (8 * i));
    }
    float* const o = out + b * 3 * plane + (size_t)y * g.W + x0p;
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        const int cc = CH == 1 ? 0 : c;
        __stcs(reinterpret_cast<float4*>(o + c * plane),
               make_float4(__fmul_rn((float)px[0 * CH + cc], g.scale), __fmul_rn((float)px[1 * CH + cc], g.scale),
                           __fmul_rn((float)px[2 * CH + cc], g.scale), __fmul_rn((float)px[3 * CH + cc], g.scale)));
    }
}

}  // namespace

LetterboxGeom letterbox_geometry(int src_w, int src_h, int W, int H, float scale, float pad) {
    LetterboxGeom g{};
    g.W = W; g.H = H; g.src_w = src_w; g.src_h = src_h;
    g.ratio = std::min((float)W / (float)src_w, (float)H / (float)src_h);
    g.sw = std::min(std::max((int)std::round((float)src_w * g.ratio), 1), W);
    g.sh = std::min(std::max((int)std::round((float)src_h * g.ratio), 1), H);
    g.px = (W - g.sw) / 2;
    g.py = (H - g.sh) / 2;
    g.inv = 1.0f / g.ratio;
    g.scale = scale;
    g.pad = pad;
    return g;
}

void launch_letterbox_u8(const uint8_t* d_src, int64_t n, int channels, const LetterboxGeom& g, float* d_out,
                         cudaStream_t s) {
    if (n <= 0) return;
    if (n > 65535 || g.H > 65535) fail(ENGINE_ERR_INVALID_ARG, "letterbox: more than 65535 images or rows per launch");
    const dim3 block(128);
    const dim3 grid((unsigned)((g.W + 4 * 128 - 1) / (4 * 128)), (unsigned)g.H, (unsigned)n);
    const bool vec = g.W % 4 == 0 && ((uintptr_t)d_out % 16) == 0;
    const bool identity = g.ratio == 1.0f && g.inv == 1.0f && g.src_w == g.W && g.src_h == g.H && g.sw == g.W &&
                          g.sh == g.H && g.px == 0 && g.py == 0;
    if (identity && vec && ((uintptr_t)d_src % 16) == 0) {
        switch (channels) {
            case 1: letterbox_identity_kernel<1><<<grid, block, 0, s>>>(d_src, d_out, g); break;
            case 3: letterbox_identity_kernel<3><<<grid, block, 0, s>>>(d_src, d_out, g); break;
            case 4: letterbox_identity_kernel<4><<<grid, block, 0, s>>>(d_src, d_out, g); break;
            default: fail(ENGINE_ERR_INVALID_ARG, "letterbox: channels must be 1, 3 or 4");
        }
        PB_CUDA(cudaGetLastError());
        return;
    }
    switch (channels * 2 + (vec ? 1 : 0)) {
        case 2: letterbox_kernel<1, false><<<grid, block, 0, s>>>(d_src, d_out, g); break;
        case 3: letterbox_kernel<1, true><<<grid, block, 0, s>>>(d_src, d_out, g); break;
        case 6: letterbox_kernel<3, false><<<grid, block, 0, s>>>(d_src, d_out, g); break;
        case 7: letterbox_kernel<3, true><<<grid, block, 0, s>>>(d_src, d_out, g); break;
        case 8: letterbox_kernel<4, false><<<grid, block, 0, s>>>(d_src, d_out, g); break;
        case 9: letterbox_kernel<4, true><<<grid, block, 0, s>>>(d_src, d_out, g); break;
        default: fail(ENGINE_ERR_INVALID_ARG, "letterbox: channels must be 1, 3 or 4");
    }
    PB_CUDA(cudaGetLastError());
}

}  // namespace pb
