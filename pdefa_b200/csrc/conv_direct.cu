// Direct convolution for layers with very few input channels (the YOLO stem:
// Cin = 3). K = kh*kw*Cin is too small for tensor cores to pay and the layer is
// bound by HBM (it reads the fp32 NCHW graph input once and writes its NHWC output
// once), so one thread computes one output pixel for all Cout (<= 64) channels with
// fp32 FMAs in (tap, channel) order. Weights sit in shared memory and are read as
// warp-wide broadcasts; the input is read through a strided view (NCHW in place);
// outputs are stored 16 bytes at a time when the view allows it.
#include "common.h"
#include "device_common.cuh"

namespace pb {

namespace {

template <int COUT>
__global__ void __launch_bounds__(256) conv_direct_kernel(ConvArgs a, int Ho, int Wo, int64_t M) {
    extern __shared__ float ws[];                 // [kh*kw*cin][COUT], zero-padded
    const int K = a.kh * a.kw * a.cin;
    const float* w = reinterpret_cast<const float*>(a.weight);   // [kh][kw][cin][cout]
    for (int i = threadIdx.x; i < K * COUT; i += blockDim.x) {
        const int k = i / COUT, co = i - k * COUT;
        ws[i] = co < a.cout ? w[(int64_t)k * a.cout + co] : 0.0f;
    }
    __syncthreads();
    const int H = (int)a.in.shape[1], W = (int)a.in.shape[2];
    const int64_t sH = a.in.stride[1], sW = a.in.stride[2], sC = a.in.stride[3];
    const int64_t hw = (int64_t)Ho * Wo;
    const bool vec_out = a.out.dt == BF16 && a.out.stride[3] == 1 && (a.cout % 8) == 0 && !a.res.ptr &&
                         ((uintptr_t)a.out.ptr % 16) == 0 && (a.out.stride[2] % 8) == 0 &&
                         (a.out.stride[1] % 8) == 0 && (a.out.img_stride % 8) == 0;
    for (int64_t m = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; m < M; m += (int64_t)gridDim.x * blockDim.x) {
        const int64_t b = m / hw;
        const int64_t r = m - b * hw;
        const int ho = (int)(r / Wo), wo = (int)(r - (int64_t)(r / Wo) * Wo);
        float acc[COUT];
#pragma unroll
        for (int co = 0; co < COUT; ++co) acc[co] = 0.0f;
        const int64_t base = b * a.in.img_stride;
        for (int kr = 0; kr < a.kh; ++kr) {
            const int hi = ho * a.sh - a.ph + kr * a.dh;
            if (hi < 0 || hi >= H) continue;
            for (int ks = 0; ks < a.kw; ++ks) {
                const int wi = wo * a.sw - a.pw + ks * a.dw;
                if (wi < 0 || wi >= W) continue;
                const float* wt = ws + ((kr * a.kw + ks) * a.cin) * COUT;
                const int64_t off = base + hi * sH + wi * sW;
                for (int c = 0; c < a.cin; ++c) {
                    const float x = ld_elem(a.in.ptr, a.in.dt, off + c * sC);
#pragma unroll
                    for (int co = 0; co < COUT; ++co) acc[co] = fmaf(x, wt[c * COUT + co], acc[co]);
                }
            }
        }
        const int64_t ob = b * a.out.img_stride + ho * a.out.stride[1] + wo * a.out.stride[2];
        const int64_t rb = a.res.ptr ? b * a.res.img_stride + ho * a.res.stride[1] + wo * a.res.stride[2] : 0;
#pragma unroll
        for (int co = 0; co < COUT; ++co) {
            if (co < a.cout) {
                float v = acc[co] + (a.bias ? __ldg(a.bias + co) : 0.0f);
                v = apply_act(v, a.act, a.slope, 0.0f);
                if (a.res.ptr) v += ld_elem(a.res.ptr, a.res.dt, rb + co * a.res.stride[3]);
                acc[co] = v;
            }
        }
        if (vec_out) {
            uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(const_cast<void*>(a.out.ptr)) + ob);
#pragma unroll
            for (int q = 0; q < COUT / 8; ++q) {
                if (q * 8 < a.cout) {
                    uint32_t w4[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        __nv_bfloat162 h2 = __floats2bfloat162_rn(acc[q * 8 + 2 * j], acc[q * 8 + 2 * j + 1]);
                        w4[j] = *reinterpret_cast<uint32_t*>(&h2);
                    }
                    dst[q] = make_uint4(w4[0], w4[1], w4[2], w4[3]);
                }
            }
        } else {
#pragma unroll
            for (int co = 0; co < COUT; ++co)
                if (co < a.cout) st_elem(const_cast<void*>(a.out.ptr), a.out.dt, ob + co * a.out.stride[3], acc[co]);
        }
    }
}

}  // namespace

bool conv_direct_supported(const ConvArgs& a) {
    return a.cin <= 8 && a.cout <= 64 && (size_t)a.kh * a.kw * a.cin * 64 * 4 <= 48 * 1024;
}

void launch_conv_direct(const ConvArgs& a, cudaStream_t s) {
    if (!conv_direct_supported(a)) fail(ENGINE_ERR_INVALID_ARG, "conv_direct: layer too large");
    const int Ho = (int)a.out.shape[1], Wo = (int)a.out.shape[2];
    const int64_t M = a.batch * Ho * Wo;
    if (M == 0) return;
    int64_t blocks = (M + 255) / 256;
    if (blocks > 148 * 16) blocks = 148 * 16;
    const int K = a.kh * a.kw * a.cin;
    if (a.cout <= 16)
        conv_direct_kernel<16><<<(unsigned)blocks, 256, K * 16 * 4, s>>>(a, Ho, Wo, M);
    else if (a.cout <= 32)
        conv_direct_kernel<32><<<(unsigned)blocks, 256, K * 32 * 4, s>>>(a, Ho, Wo, M);
    else
        conv_direct_kernel<64><<<(unsigned)blocks, 256, K * 64 * 4, s>>>(a, Ho, Wo, M);
    PB_CUDA(cudaGetLastError());
}

}  // namespace pb
