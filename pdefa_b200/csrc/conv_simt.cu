// Strict-fp32 SIMT kernels: implicit-GEMM convolution over strided views and a
// row-major GEMM. These are the <= 1e-5 parity path (fp32 FMA accumulation, no
// tensor cores) and serve layers the tensor-core kernel cannot take.
//
// Convolution as GEMM: M = batch*Ho*Wo output pixels, N = Cout, K = kh*kw*Cin in
// (tap, channel) order. A block computes a BM x BN tile; each of its 256 threads
// owns 4 pixels x 4 output channels. Input taps outside the image read as zero,
// which is the reference's zero padding (conv2d.cpp:401-439 naive form).
#include "common.h"
#include "device_common.cuh"

namespace pb {

namespace {

constexpr int KC = 16;   // K elements staged per step

template <int BN>
__global__ void __launch_bounds__(256) conv_simt_kernel(ConvArgs a, int Ho, int Wo, int64_t M) {
    constexpr int TN = BN / 4;           // threads along N
    constexpr int TM = 256 / TN;         // threads along M
    constexpr int BM = TM * 4;
    constexpr int LA = BM * KC / 256;    // A elements loaded per thread
    __shared__ float As[KC][BM];
    __shared__ float Ws[KC][BN];

    const int tid = threadIdx.x;
    const int64_t m0 = (int64_t)blockIdx.x * BM;
    const int n0 = blockIdx.y * BN;
    const float* wt = reinterpret_cast<const float*>(a.weight);

    // Each thread loads channels (tid % KC) of pixels p = tid / KC + j * (256 / KC).
    const int lk = tid % KC;
    int64_t pbase[LA];
    int hi0[LA], wi0[LA];
    for (int j = 0; j < LA; ++j) {
        const int p = tid / KC + j * (256 / KC);
        const int64_t m = m0 + p;
        if (m < M) {
            const int64_t b = m / ((int64_t)Ho * Wo);
            const int64_t r = m - b * (int64_t)Ho * Wo;
            const int ho = (int)(r / Wo), wo = (int)(r - (int64_t)(r / Wo) * Wo);
            hi0[j] = ho * a.sh - a.ph;
            wi0[j] = wo * a.sw - a.pw;
            pbase[j] = b * a.in.img_stride;
        } else {
            hi0[j] = -1000000;  // forces the bounds check to fail
            wi0[j] = -1000000;
            pbase[j] = 0;
        }
    }
    const int H = (int)a.in.shape[1], W = (int)a.in.shape[2];
    const int64_t sH = a.in.stride[1], sW = a.in.stride[2], sC = a.in.stride[3];

    const int tx = tid % TN, ty = tid / TN;
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;

    for (int r = 0; r < a.kh; ++r) {
        for (int s = 0; s < a.kw; ++s) {
            const int tap = r * a.kw + s;
            for (int c0 = 0; c0 < a.cin; c0 += KC) {
                const int c = c0 + lk;
#pragma unroll
                for (int j = 0; j < LA; ++j) {
                    const int p = tid / KC + j * (256 / KC);
                    const int hi = hi0[j] + r * a.dh, wi = wi0[j] + s * a.dw;
                    float v = 0.0f;
                    if (c < a.cin && hi >= 0 && hi < H && wi >= 0 && wi < W)
                        v = ld_elem(a.in.ptr, a.in.dt, pbase[j] + hi * sH + wi * sW + c * sC);
                    As[lk][p] = v;
                }
#pragma unroll
                for (int j = 0; j < BN * KC / 256; ++j) {
                    const int e = tid + j * 256;
                    const int kk = e / BN, nn = e % BN;
                    const int cc = c0 + kk, co = n0 + nn;
                    Ws[kk][nn] = (cc < a.cin && co < a.cout) ? wt[((int64_t)tap * a.cin + cc) * a.cout + co] : 0.0f;
                }
                __syncthreads();
#pragma unroll
                for (int kk = 0; kk < KC; ++kk) {
                    float av[4], wv[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) av[i] = As[kk][ty + i * TM];
#pragma unroll
                    for (int j = 0; j < 4; ++j) wv[j] = Ws[kk][tx * 4 + j];
#pragma unroll
                    for (int i = 0; i < 4; ++i)
#pragma unroll
                        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], wv[j], acc[i][j]);
                }
                __syncthreads();
            }
        }
    }

    // Epilogue: bias, activation, optional residual, strided store.
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int64_t m = m0 + ty + i * TM;
        if (m >= M) continue;
        const int64_t b = m / ((int64_t)Ho * Wo);
        const int64_t rr = m - b * (int64_t)Ho * Wo;
        const int64_t ho = rr / Wo, wo = rr - ho * Wo;
        const int64_t ob = b * a.out.img_stride + ho * a.out.stride[1] + wo * a.out.stride[2];
        const int64_t rb = a.res.ptr ? b * a.res.img_stride + ho * a.res.stride[1] + wo * a.res.stride[2] : 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int co = n0 + tx * 4 + j;
            if (co >= a.cout) continue;
            float v = acc[i][j];
            if (a.bias) v += a.bias[co];
            v = apply_act(v, a.act, a.slope, 0.0f);
            if (a.res.ptr) v += ld_elem(a.res.ptr, a.res.dt, rb + co * a.res.stride[3]);
            st_elem(const_cast<void*>(a.out.ptr), a.out.dt, ob + co * a.out.stride[3], v);
        }
    }
}

// C[b] = A[b] * B[b] (+ bias); 64x64 tiles, 4x4 per thread, fp32 FMA in k order.
__global__ void __launch_bounds__(256) gemm_f32_kernel(const float* A, const float* B, float* C, const float* bias,
                                                       int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb,
                                                       int64_t ldc, int64_t sA, int64_t sB, int64_t sC) {
    __shared__ float As[KC][64];
    __shared__ float Bs[KC][64];
    const int tid = threadIdx.x;
    const int64_t bz = blockIdx.z;
    A += bz * sA; B += bz * sB; C += bz * sC;
    const int64_t m0 = (int64_t)blockIdx.x * 64, n0 = (int64_t)blockIdx.y * 64;
    const int tx = tid % 16, ty = tid / 16;
    float acc[4][4] = {};
    for (int64_t k0 = 0; k0 < K; k0 += KC) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int e = tid + j * 256;
            // A tile: element (row p, k kk) with kk fastest for coalescing.
            const int kk = e % KC, p = e / KC;
            const int64_t gm = m0 + p, gk = k0 + kk;
            As[kk][p] = (gm < M && gk < K) ? A[gm * lda + gk] : 0.0f;
            const int nn = e % 64, kb = e / 64;
            const int64_t gn = n0 + nn, gk2 = k0 + kb;
            Bs[kb][nn] = (gn < N && gk2 < K) ? B[gk2 * ldb + gn] : 0.0f;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < KC; ++kk) {
            float av[4], bv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) av[i] = As[kk][ty + i * 16];
#pragma unroll
            for (int j = 0; j < 4; ++j) bv[j] = Bs[kk][tx * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int64_t gm = m0 + ty + i * 16;
        if (gm >= M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int64_t gn = n0 + tx * 4 + j;
            if (gn >= N) continue;
            C[gm * ldc + gn] = acc[i][j] + (bias ? bias[gn] : 0.0f);
        }
    }
}

}  // namespace

void launch_conv_simt(const ConvArgs& a, cudaStream_t s) {
    const int Ho = (int)a.out.shape[1], Wo = (int)a.out.shape[2];
    const int64_t M = a.batch * Ho * Wo;
    if (M == 0 || a.cout == 0) return;
    if (a.cout <= 16) {
        dim3 grid((unsigned)((M + 255) / 256), (unsigned)((a.cout + 15) / 16));
        conv_simt_kernel<16><<<grid, 256, 0, s>>>(a, Ho, Wo, M);
    } else if (a.cout <= 32) {
        dim3 grid((unsigned)((M + 127) / 128), (unsigned)((a.cout + 31) / 32));
        conv_simt_kernel<32><<<grid, 256, 0, s>>>(a, Ho, Wo, M);
    } else {
        dim3 grid((unsigned)((M + 63) / 64), (unsigned)((a.cout + 63) / 64));
        conv_simt_kernel<64><<<grid, 256, 0, s>>>(a, Ho, Wo, M);
    }
    PB_CUDA(cudaGetLastError());
}

void launch_gemm_f32(const float* A, const float* B, float* C, const float* bias,
                     int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldc,
                     int64_t batch, int64_t sA, int64_t sB, int64_t sC, cudaStream_t s) {
    if (M == 0 || N == 0 || batch == 0) return;
    dim3 grid((unsigned)((M + 63) / 64), (unsigned)((N + 63) / 64), (unsigned)batch);
    gemm_f32_kernel<<<grid, 256, 0, s>>>(A, B, C, bias, M, N, K, lda, ldb, ldc, sA, sB, sC);
    PB_CUDA(cudaGetLastError());
}

}  // namespace pb
