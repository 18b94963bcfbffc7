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
#include <algorithm>
#include <cstdlib>

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

// Depthwise 3x3 (groups = Cin = Cout), stride S, dilation 1, channel stride 1.
// A thread owns two adjacent channels (one 4- or 8-byte load per pixel) and kRows
// output rows of one column: it loads the (kRows-1)*S+3 x 3 input window once and
// reuses it across the rows (18 paired loads for 8 outputs at stride 1, against 72 in
// the generic kernel), with 32-bit index math. Per output the sum is the same as the
// generic kernel's: bias, then fma over the in-image taps in (kh, kw) order.
constexpr int kDwRows = 4;

template <int S, bool BIN, bool BOUT>
__global__ void __launch_bounds__(256) conv_dw3_kernel(ConvArgs a, int H, int W, int Ho, int Wo, int CP, int NS,
                                                        int total) {
    constexpr int NR = (kDwRows - 1) * S + 3;
    const float* wt = reinterpret_cast<const float*>(a.weight);   // [C][3][3]
    const int sH = (int)a.in.stride[1], sW = (int)a.in.stride[2];
    const int oH = (int)a.out.stride[1], oW = (int)a.out.stride[2];
    for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < total; t += gridDim.x * blockDim.x) {
        const int cp = t % CP;
        int rem = t / CP;
        const int wo = rem % Wo;
        rem /= Wo;
        const int strip = rem % NS;
        const int b = rem / NS;
        const int c0 = 2 * cp;
        const int ho0 = strip * kDwRows;
        const int hi0 = ho0 * S - a.ph, wi0 = wo * S - a.pw;
        float w0[9], w1[9];
#pragma unroll
        for (int k = 0; k < 9; ++k) { w0[k] = wt[c0 * 9 + k]; w1[k] = wt[c0 * 9 + 9 + k]; }
        const float b0 = a.bias ? a.bias[c0] : 0.0f, b1 = a.bias ? a.bias[c0 + 1] : 0.0f;
        float2 x[NR][3];
        bool rv[NR], cv[3];
#pragma unroll
        for (int j = 0; j < 3; ++j) cv[j] = (unsigned)(wi0 + j) < (unsigned)W;
        const char* ib = static_cast<const char*>(a.in.ptr) + ((int64_t)b * a.in.img_stride + c0) * (BIN ? 2 : 4);
#pragma unroll
        for (int r = 0; r < NR; ++r) {
            const int hi = hi0 + r;
            rv[r] = (unsigned)hi < (unsigned)H;
#pragma unroll
            for (int j = 0; j < 3; ++j) {
                x[r][j] = make_float2(0.0f, 0.0f);
                if (rv[r] && cv[j]) {
                    const int64_t off = (int64_t)hi * sH + (int64_t)(wi0 + j) * sW;
                    if (BIN) x[r][j] = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(ib + off * 2));
                    else x[r][j] = *reinterpret_cast<const float2*>(ib + off * 4);
                }
            }
        }
#pragma unroll
        for (int i = 0; i < kDwRows; ++i) {
            const int ho = ho0 + i;
            if (ho >= Ho) break;
            float acc0 = b0, acc1 = b1;
#pragma unroll
            for (int kr = 0; kr < 3; ++kr) {
                if (!rv[i * S + kr]) continue;
#pragma unroll
                for (int ks = 0; ks < 3; ++ks) {
                    if (!cv[ks]) continue;
                    acc0 = fmaf(x[i * S + kr][ks].x, w0[kr * 3 + ks], acc0);
                    acc1 = fmaf(x[i * S + kr][ks].y, w1[kr * 3 + ks], acc1);
                }
            }
            float v0 = apply_act(acc0, a.act, a.slope, 0.0f), v1 = apply_act(acc1, a.act, a.slope, 0.0f);
            if (a.res.ptr) {
                const int64_t ro = (int64_t)b * a.res.img_stride + (int64_t)ho * a.res.stride[1] +
                                   (int64_t)wo * a.res.stride[2] + (int64_t)c0 * a.res.stride[3];
                v0 += ld_elem(a.res.ptr, a.res.dt, ro);
                v1 += ld_elem(a.res.ptr, a.res.dt, ro + a.res.stride[3]);
            }
            char* ob = static_cast<char*>(const_cast<void*>(a.out.ptr)) +
                       ((int64_t)b * a.out.img_stride + (int64_t)ho * oH + (int64_t)wo * oW + c0) * (BOUT ? 2 : 4);
            if (BOUT) *reinterpret_cast<__nv_bfloat162*>(ob) = __floats2bfloat162_rn(v0, v1);
            else *reinterpret_cast<float2*>(ob) = make_float2(v0, v1);
        }
    }
}

bool dw3_eligible(const ConvArgs& a, int groups) {
    if (!(groups == a.cin && groups == a.cout && a.cin % 2 == 0 && a.kh == 3 && a.kw == 3 && a.dh == 1 &&
          a.dw == 1 && a.sh == a.sw && (a.sh == 1 || a.sh == 2)))
        return false;
    if (a.in.stride[3] != 1 || a.out.stride[3] != 1) return false;
    const int64_t* st[] = {a.in.stride, a.out.stride};
    for (const int64_t* x : st)
        if ((x[1] | x[2]) & 1) return false;
    if ((a.in.img_stride | a.out.img_stride) & 1) return false;
    const uintptr_t ai = reinterpret_cast<uintptr_t>(a.in.ptr), ao = reinterpret_cast<uintptr_t>(a.out.ptr);
    if (ai % (a.in.dt == BF16 ? 4 : 8) || ao % (a.out.dt == BF16 ? 4 : 8)) return false;
    const int64_t Ho = a.out.shape[1], Wo = a.out.shape[2];
    const int64_t n = a.batch * ((Ho + kDwRows - 1) / kDwRows) * Wo * (a.cout / 2);
    return n < (int64_t)1 << 31 && a.in.shape[1] * a.in.stride[1] < (int64_t)1 << 31;
}

template <int S>
void launch_dw3(const ConvArgs& a, cudaStream_t s) {
    const int H = (int)a.in.shape[1], W = (int)a.in.shape[2];
    const int Ho = (int)a.out.shape[1], Wo = (int)a.out.shape[2];
    const int CP = a.cout / 2, NS = (Ho + kDwRows - 1) / kDwRows;
    const int total = (int)(a.batch * NS * Wo * CP);
    if (total == 0) return;
    const int blocks = (int)std::min<int64_t>((total + 255) / 256, 148 * 16);
    const bool bi = a.in.dt == BF16, bo = a.out.dt == BF16;
    if (bi && bo) conv_dw3_kernel<S, true, true><<<blocks, 256, 0, s>>>(a, H, W, Ho, Wo, CP, NS, total);
    else if (bi) conv_dw3_kernel<S, true, false><<<blocks, 256, 0, s>>>(a, H, W, Ho, Wo, CP, NS, total);
    else if (bo) conv_dw3_kernel<S, false, true><<<blocks, 256, 0, s>>>(a, H, W, Ho, Wo, CP, NS, total);
    else conv_dw3_kernel<S, false, false><<<blocks, 256, 0, s>>>(a, H, W, Ho, Wo, CP, NS, total);
    PB_CUDA(cudaGetLastError());
}

}  // namespace

void launch_conv_grouped(const ConvArgs& a, int groups, cudaStream_t s) {
    if (groups < 1 || a.cin % groups || a.cout % groups) fail(ENGINE_ERR_INVALID_SHAPE, "grouped conv: channels not divisible by groups");
    const char* no_dw3 = std::getenv("PDEFA_NO_DW3");   // 1: the generic kernel for every grouped conv
    if (!(no_dw3 && no_dw3[0] == '1') && dw3_eligible(a, groups)) {
        if (a.sh == 1) launch_dw3<1>(a, s);
        else launch_dw3<2>(a, s);
        return;
    }
    const int Ho = (int)a.out.shape[1], Wo = (int)a.out.shape[2];
    const int64_t total = a.batch * Ho * Wo * a.cout;
    if (total == 0) return;
    int64_t blocks = (total + 255) / 256;
    if (blocks > 148 * 32) blocks = 148 * 32;
    conv_grouped_kernel<<<(unsigned)blocks, 256, 0, s>>>(a, Ho, Wo, a.cin / groups, a.cout / groups, total);
    PB_CUDA(cudaGetLastError());
}

}  // namespace pb
