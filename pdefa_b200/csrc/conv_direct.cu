// Direct convolution for layers with very few input channels (the YOLO stem:
// Cin = 3). K = kh*kw*Cin is too small for tensor cores to pay and the layer is
// bound by HBM (it reads the fp32 NCHW graph input once and writes its NHWC output
// once), so one thread computes one output pixel for all Cout (<= 64) channels with
// fp32 FMAs in (tap, channel) order. Weights sit in shared memory and are read as
// warp-wide broadcasts; the input is read through a strided view (NCHW in place);
// outputs are stored 16 bytes at a time when the view allows it.
#include <algorithm>

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


// Row-tiled variant for inputs whose W axis is contiguous (the fp32 NCHW graph
// input): a CTA stages the input rows its R output rows need (all Cin planes, zero
// padded) in shared memory with cp.async, then each thread computes PX output
// pixels x COUT channels, so every weight read from shared memory (float4, warp
// broadcast) feeds PX pixels. A thread's pixels are tpr apart (tpr = threads per
// output row), so the lanes of a warp read neighbouring input columns (at most
// stride-way bank conflicts) and store neighbouring pixels.
constexpr int kLM = 4;   // left margin of a staged row (>= pad_w, keeps the interior 16-byte aligned)

// KK / CIN > 0 fix the kernel size and input channels at compile time (the 3x3,
// Cin = 3 stem) so the tap loops unroll; 0 reads them from the arguments. FAST
// selects the hardware-exponential SiLU (BF16 outputs).
template <int COUT, int PX, int KK, int CIN, bool FAST>
__global__ void __launch_bounds__(256, KK ? 2 : 3) conv_direct_rows_kernel(ConvArgs a, int Ho, int Wo, int R,
                                                                        int rows_in, int pitch, int tiles_h) {
    extern __shared__ float sm[];
    const int kh = KK ? KK : a.kh, kw = KK ? KK : a.kw, cin = CIN ? CIN : a.cin;
    const int K = kh * kw * cin;
    float* ws = sm;                                     // [K][COUT]
    float* xs = sm + K * COUT;                          // [cin][rows_in][pitch]
    const float* w = reinterpret_cast<const float*>(a.weight);   // [kh][kw][cin][cout]
    for (int i = threadIdx.x; i < K * COUT; i += blockDim.x) {
        const int k = i / COUT, co = i - k * COUT;
        ws[i] = co < a.cout ? w[(int64_t)k * a.cout + co] : 0.0f;
    }
    const int b = blockIdx.x / tiles_h;
    const int yo0 = (blockIdx.x - b * tiles_h) * R;
    const int H = (int)a.in.shape[1], W = (int)a.in.shape[2];
    const int64_t sH = a.in.stride[1], sC = a.in.stride[3];
    const int64_t ibase = (int64_t)b * a.in.img_stride;
    const int yi0 = yo0 * a.sh - a.ph;
    // stage rows: element (c, j, x) -> xs[(c*rows_in + j)*pitch + kLM + x], zeros outside the image
    const int nrow = cin * rows_in;
    const bool vec = a.in.dt == F32 && (W % 4) == 0 && (sH % 4) == 0 && (sC % 4) == 0 &&
                     (a.in.img_stride % 4) == 0 && ((uintptr_t)a.in.ptr % 16) == 0;
    if (vec) {
        // cp.async (global -> shared, 16 bytes, no register round trip): every copy of
        // the tile is in flight at once; rows outside the image are zero-filled by a
        // source size of 0.
        const int w4 = W / 4;
        const float* src0 = reinterpret_cast<const float*>(a.in.ptr) + ibase;
        for (int i = threadIdx.x; i < nrow * w4; i += blockDim.x) {
            const int row = i / w4, x4 = i - row * w4;
            const int c = row / rows_in, j = row - c * rows_in;
            const int yi = yi0 + j;
            const bool in = yi >= 0 && yi < H;
            const float* src = in ? src0 + c * sC + (int64_t)yi * sH + 4 * x4 : src0;
            const uint32_t dst = smem_u32(xs + row * pitch + kLM + 4 * x4);
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(in ? 16 : 0)
                         : "memory");
        }
        asm volatile("cp.async.wait_all;" ::: "memory");
    } else {
        for (int i = threadIdx.x; i < nrow * W; i += blockDim.x) {
            const int row = i / W, x = i - row * W;
            const int c = row / rows_in, j = row - c * rows_in;
            const int yi = yi0 + j;
            xs[row * pitch + kLM + x] = (yi >= 0 && yi < H)
                ? ld_elem(a.in.ptr, a.in.dt, ibase + c * sC + (int64_t)yi * sH + x) : 0.0f;
        }
    }
    // zero margins: [0, kLM) and [kLM + W, pitch)
    const int marg = pitch - W;
    for (int i = threadIdx.x; i < nrow * marg; i += blockDim.x) {
        const int row = i / marg, m = i - row * marg;
        xs[row * pitch + (m < kLM ? m : W + m)] = 0.0f;
    }
    __syncthreads();

    const int tpr = (Wo + PX - 1) / PX;                 // threads per output row
    const int ry = threadIdx.x / tpr, g = threadIdx.x - ry * tpr;
    const int yo = yo0 + ry;
    if (ry >= R || yo >= Ho) return;
    float acc[PX][COUT];
#pragma unroll
    for (int p = 0; p < PX; ++p)
#pragma unroll
        for (int co = 0; co < COUT; ++co) acc[p][co] = 0.0f;
    int xcol[PX];
#pragma unroll
    for (int p = 0; p < PX; ++p) xcol[p] = (g + p * tpr) * a.sw + kLM - a.pw;
#pragma unroll 1
    for (int kr = 0; kr < kh; ++kr) {
        const int j = ry * a.sh + kr * a.dh;
#pragma unroll
        for (int ks = 0; ks < kw; ++ks) {
            const int xoff = ks * a.dw;
#pragma unroll
            for (int c = 0; c < cin; ++c) {
                const float* row = xs + (c * rows_in + j) * pitch + xoff;
                float v[PX];
#pragma unroll
                for (int p = 0; p < PX; ++p) v[p] = row[xcol[p]];
                const float4* wt = reinterpret_cast<const float4*>(ws + ((kr * kw + ks) * cin + c) * COUT);
#pragma unroll
                for (int q = 0; q < COUT / 4; ++q) {
                    const float4 wv = wt[q];
#pragma unroll
                    for (int p = 0; p < PX; ++p) {
                        acc[p][4 * q] = fmaf(v[p], wv.x, acc[p][4 * q]);
                        acc[p][4 * q + 1] = fmaf(v[p], wv.y, acc[p][4 * q + 1]);
                        acc[p][4 * q + 2] = fmaf(v[p], wv.z, acc[p][4 * q + 2]);
                        acc[p][4 * q + 3] = fmaf(v[p], wv.w, acc[p][4 * q + 3]);
                    }
                }
            }
        }
    }
    const bool vec_out = a.out.dt == BF16 && a.out.stride[3] == 1 && (a.cout % 8) == 0 &&
                         ((uintptr_t)a.out.ptr % 16) == 0 && (a.out.stride[2] % 8) == 0 &&
                         (a.out.stride[1] % 8) == 0 && (a.out.img_stride % 8) == 0;
#pragma unroll
    for (int p = 0; p < PX; ++p) {
        const int xo = g + p * tpr;
        if (xo >= Wo) break;
        const int64_t ob = (int64_t)b * a.out.img_stride + (int64_t)yo * a.out.stride[1] + (int64_t)xo * a.out.stride[2];
        const int64_t rb = a.res.ptr ? (int64_t)b * a.res.img_stride + (int64_t)yo * a.res.stride[1] +
                                           (int64_t)xo * a.res.stride[2] : 0;
#pragma unroll
        for (int co = 0; co < COUT; ++co) {
            if (co < a.cout) {
                float v = acc[p][co] + (a.bias ? __ldg(a.bias + co) : 0.0f);
                if (FAST && a.act == ACT_SILU) v = __fdividef(v, 1.0f + __expf(-v));
                else v = apply_act(v, a.act, a.slope, 0.0f);
                if (a.res.ptr) v += ld_elem(a.res.ptr, a.res.dt, rb + co * a.res.stride[3]);
                acc[p][co] = v;
            }
        }
        if (vec_out) {
            uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(const_cast<void*>(a.out.ptr)) + ob);
#pragma unroll
            for (int q = 0; q < COUT / 8; ++q) {
                if (q * 8 < a.cout) {
                    uint32_t w4[4];
#pragma unroll
                    for (int t = 0; t < 4; ++t) {
                        __nv_bfloat162 h2 = __floats2bfloat162_rn(acc[p][q * 8 + 2 * t], acc[p][q * 8 + 2 * t + 1]);
                        w4[t] = *reinterpret_cast<uint32_t*>(&h2);
                    }
                    dst[q] = make_uint4(w4[0], w4[1], w4[2], w4[3]);
                }
            }
        } else {
#pragma unroll
            for (int co = 0; co < COUT; ++co)
                if (co < a.cout) st_elem(const_cast<void*>(a.out.ptr), a.out.dt, ob + co * a.out.stride[3], acc[p][co]);
        }
    }
}

template <int COUT, int PX, int KK, int CIN, bool FAST>
void launch_rows_kernel(const ConvArgs& a, int Ho, int Wo, int R, int rows_in, int pitch, int tiles_h, int threads,
                        size_t smem, int64_t grid, cudaStream_t s) {
    int dev = 0;
    PB_CUDA(cudaGetDevice(&dev));
    static bool attr[64] = {};
    if (dev >= 64 || !attr[dev]) {
        PB_CUDA(cudaFuncSetAttribute(conv_direct_rows_kernel<COUT, PX, KK, CIN, FAST>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024));
        if (dev < 64) attr[dev] = true;
    }
    conv_direct_rows_kernel<COUT, PX, KK, CIN, FAST><<<(unsigned)grid, threads, smem, s>>>(a, Ho, Wo, R, rows_in,
                                                                                         pitch, tiles_h);
}

template <int COUT, int PX>
bool launch_rows(const ConvArgs& a, int Ho, int Wo, cudaStream_t s) {
    const int W = (int)a.in.shape[2];
    if (a.in.stride[2] != 1 || a.pw > kLM || Wo > 256 * PX) return false;
    const int tpr = (Wo + PX - 1) / PX;
    int R = std::max(1, 256 / tpr);
    R = std::min(R, Ho);
    const int K = a.kh * a.kw * a.cin;
    // the last thread's pixels reach tpr*PX - 1 (computed, not stored): stage
    // enough right margin that their reads stay inside the row
    const int right = std::max(0, (tpr * PX - 1) * a.sw - a.pw + (a.kw - 1) * a.dw + 1 - W);
    const int pitch = (kLM + W + right + 3) / 4 * 4;
    auto bytes = [&](int r) {
        const int rin = (r - 1) * a.sh + (a.kh - 1) * a.dh + 1;
        return (size_t)(K * COUT + a.cin * rin * pitch) * 4;
    };
    while (R > 1 && bytes(R) > 96 * 1024) --R;
    if (bytes(R) > 96 * 1024) return false;
    const int rows_in = (R - 1) * a.sh + (a.kh - 1) * a.dh + 1;
    const int tiles_h = (Ho + R - 1) / R;
    const int64_t grid = a.batch * tiles_h;
    if (grid > 0x7fffffff) return false;
    const bool stem = a.kh == 3 && a.kw == 3 && a.cin == 3;
    const bool fast = a.out.dt == BF16;
    const size_t smem = bytes(R);
    const int threads = R * tpr;
    if (stem && fast) launch_rows_kernel<COUT, PX, 3, 3, true>(a, Ho, Wo, R, rows_in, pitch, tiles_h, threads, smem, grid, s);
    else if (stem) launch_rows_kernel<COUT, PX, 3, 3, false>(a, Ho, Wo, R, rows_in, pitch, tiles_h, threads, smem, grid, s);
    else if (fast) launch_rows_kernel<COUT, PX, 0, 0, true>(a, Ho, Wo, R, rows_in, pitch, tiles_h, threads, smem, grid, s);
    else launch_rows_kernel<COUT, PX, 0, 0, false>(a, Ho, Wo, R, rows_in, pitch, tiles_h, threads, smem, grid, s);
    PB_CUDA(cudaGetLastError());
    return true;
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
    if (a.cout <= 16 ? launch_rows<16, 4>(a, Ho, Wo, s)
                     : a.cout <= 32 ? launch_rows<32, 2>(a, Ho, Wo, s) : launch_rows<64, 1>(a, Ho, Wo, s))
        return;
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
