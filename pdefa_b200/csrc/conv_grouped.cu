// Grouped and depthwise convolution (NHWC), replacing the reference's
// engine_conv2d_depthwise_avx2 and engine_conv2d_grouped_gemm
// (PDEFA1.0/src/ops/conv2d.cpp:164-393).
//
// One thread per output element (pixel, output channel), output channels fastest so a
// warp reads and writes consecutive channels. Group g = co / Cout_g reads input
// channels g*Cin_g ... (g+1)*Cin_g - 1. The sum starts at the bias and adds the taps
// in (kh, kw, ci) order with fp32 fma, skipping taps outside the image: for depthwise
// (Cin_g = 1) exactly the reference kernel's accumulation (conv2d.cpp:236-303: acc =
// bias, fma per in-image tap in kh, kw order); grouped convs run the reference's
// per-group GEMM, whose blocking sums in another order (results within the fp32
// tolerance). Then the fused activation and an optional residual, like the other
// conv epilogues. Any input/output view (fp32 or bf16), fp32 arithmetic in every
// precision; memory bound (a depthwise 3x3 does 9 MACs per output).
#include "common.h"
#include "device_common.cuh"

namespace pb {

namespace {

__global__ void __launch_bounds__(256) conv_grouped_kernel(ConvArgs a, int Ho, int Wo, int cin_g, int cout_g,
                                                           int64_t total) {
    const float* wt = reinterpret_cast<const float*>(a.weight);   // [cout][kh][kw][cin_g]
    const int H = (int)a.in.shape[1], W = (int)a.in.shape[2];
    const int64_t sH = a.in.stride[1], sW = a.in.stride[2], sC = a.in.stride[3];
    const int taps = a.kh * a.kw;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int co = (int)(t % a.cout);
        const int64_t m = t / a.cout;
        const int64_t hw = (int64_t)Ho * Wo;
        const int64_t b = m / hw;
        const int64_t r = m - b * hw;
        const int ho = (int)(r / Wo), wo = (int)(r - (int64_t)(r / Wo) * Wo);
        const int g = co / cout_g;
        const int64_t ib = b * a.in.img_stride + (int64_t)g * cin_g * sC;
        const float* w = wt + (int64_t)co * taps * cin_g;
        float acc = a.bias ? a.bias[co] : 0.0f;
        for (int kr = 0; kr < a.kh; ++kr) {
            const int hi = ho * a.sh - a.ph + kr * a.dh;
            if (hi < 0 || hi >= H) continue;
            for (int ks = 0; ks < a.kw; ++ks) {
                const int wi = wo * a.sw - a.pw + ks * a.dw;
                if (wi < 0 || wi >= W) continue;
                const int64_t off = ib + hi * sH + wi * sW;
                const float* wk = w + (kr * a.kw + ks) * cin_g;
                for (int ci = 0; ci < cin_g; ++ci)
                    acc = fmaf(ld_elem(a.in.ptr, a.in.dt, off + ci * sC), wk[ci], acc);
            }
        }
        float v = apply_act(acc, a.act, a.slope, 0.0f);
        if (a.res.ptr)
            v += ld_elem(a.res.ptr, a.res.dt,
                         b * a.res.img_stride + (int64_t)ho * a.res.stride[1] + (int64_t)wo * a.res.stride[2] +
                             (int64_t)co * a.res.stride[3]);
        st_elem(const_cast<void*>(a.out.ptr), a.out.dt,
                b * a.out.img_stride + (int64_t)ho * a.out.stride[1] + (int64_t)wo * a.out.stride[2] +
                    (int64_t)co * a.out.stride[3],
                v);
    }
}

}  // namespace

void launch_conv_grouped(const ConvArgs& a, int groups, cudaStream_t s) {
    if (groups < 1 || a.cin % groups || a.cout % groups) fail(ENGINE_ERR_INVALID_SHAPE, "grouped conv: channels not divisible by groups");
    const int Ho = (int)a.out.shape[1], Wo = (int)a.out.shape[2];
    const int64_t total = a.batch * Ho * Wo * a.cout;
    if (total == 0) return;
    int64_t blocks = (total + 255) / 256;
    if (blocks > 148 * 32) blocks = 148 * 32;
    conv_grouped_kernel<<<(unsigned)blocks, 256, 0, s>>>(a, Ho, Wo, a.cin / groups, a.cout / groups, total);
    PB_CUDA(cudaGetLastError());
}

}  // namespace pb
