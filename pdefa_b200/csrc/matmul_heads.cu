// Head-batched matrix product of the attention blocks (YOLOv10 / YOLO11 PSA),
// replacing the reference's 4-D x 4-D MatMul branch
// (PDEFA1.0/src/core/session_parts/session_ops_nn.inc:68-108).
//
// The engine keeps 4-D tensors with the ONNX channel axis last, so an attention
// operand [B, heads, rows, cols] is stored as [B, rows, cols, heads] and the
// product is C[b, i, j, h] = sum_k A[b, i, k, h] * B[b, k, j, h]. Each output is an
// fp32 fma chain over k in ascending order starting from +0, the reference's
// contracted loop, so results are bit-identical to it in every precision.
//
// Operands are strided views (fp32 or bf16; a Transpose feeding the product is read
// through permuted strides instead of being copied), and a scalar Mul after the
// product is applied to each finished sum (the same single rounding as the separate
// Mul). A 256-thread CTA computes a 64 x 64 tile of one (b, h) plane; k advances in
// chunks of 16 staged through shared memory (A as [k][i], B as [k][j]); each
// thread owns a 4 x 4 block of outputs strided by 16 so that a warp reads
// consecutive shared-memory words. The attention products of a 20 x 20 P5 map
// (400 x 400 x 32 and 64 x 400 x 400 per head) are small; this SIMT kernel keeps
// the exact summation order instead of a tensor-core path.
#include <cuda_bf16.h>

#include "common.h"
#include "kernels.h"

namespace pb {

namespace {

constexpr int kTile = 64, kChunk = 16, kThreads = 256;

template <bool BF>
__device__ __forceinline__ float ld_op(const void* p, int64_t i) {
    if (BF) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
    return static_cast<const float*>(p)[i];
}

template <bool ABF, bool BBF>
__global__ void __launch_bounds__(kThreads)
matmul_heads_kernel(HeadOperand A, HeadOperand B, float* __restrict__ C, int M, int K, int N, int H, float scale,
                    int64_t sc) {
    __shared__ float As[kChunk][kTile + 1];
    __shared__ float Bs[kChunk][kTile];
    const int plane = blockIdx.z;              // image * H + h
    const int b = plane / H, h = plane - b * H;
    const int i0 = blockIdx.y * kTile, j0 = blockIdx.x * kTile;
    const int64_t abase = (int64_t)b * A.sb + (int64_t)h * A.s3;
    const int64_t bbase = (int64_t)b * B.sb + (int64_t)h * B.s3;
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    float acc[4][4];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[r][c] = 0.0f;
    for (int k0 = 0; k0 < K; k0 += kChunk) {
#pragma unroll
        for (int q = 0; q < (kTile * kChunk) / kThreads; ++q) {
            const int e = tid + q * kThreads;
            const int kk = e & (kChunk - 1), ii = e >> 4;          // A: k fastest
            const int gi = i0 + ii, gk = k0 + kk;
            As[kk][ii] = (gi < M && gk < K) ? ld_op<ABF>(A.p, abase + gi * A.s1 + gk * A.s2) : 0.0f;
            const int jj = e & (kTile - 1), kb = e >> 6;            // B: j fastest
            const int gj = j0 + jj, gkb = k0 + kb;
            Bs[kb][jj] = (gj < N && gkb < K) ? ld_op<BBF>(B.p, bbase + gkb * B.s1 + gj * B.s2) : 0.0f;
        }
        __syncthreads();
        const int kn = min(kChunk, K - k0);
        for (int kk = 0; kk < kn; ++kk) {
            float av[4], bv[4];
#pragma unroll
            for (int r = 0; r < 4; ++r) av[r] = As[kk][ty + 16 * r];
#pragma unroll
            for (int c = 0; c < 4; ++c) bv[c] = Bs[kk][tx + 16 * c];
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int c = 0; c < 4; ++c) acc[r][c] = fmaf(av[r], bv[c], acc[r][c]);
        }
        __syncthreads();
    }
    float* o = C + (int64_t)b * sc + h;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const int gi = i0 + ty + 16 * r;
        if (gi >= M) continue;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int gj = j0 + tx + 16 * c;
            if (gj < N) o[((int64_t)gi * N + gj) * H] = acc[r][c] * scale;
        }
    }
}

}  // namespace

void launch_matmul_heads(const HeadOperand& A, const HeadOperand& B, float* C, int64_t batch, int64_t M, int64_t K,
                         int64_t N, int64_t H, float scale, int64_t sC, cudaStream_t s) {
    if (batch <= 0 || M <= 0 || N <= 0 || H <= 0) return;
    if (M > INT32_MAX || K > INT32_MAX || N > INT32_MAX || batch * H > 65535 || (M + kTile - 1) / kTile > 65535)
        fail(ENGINE_ERR_INVALID_SHAPE, "matmul_heads: extents out of range");
    const dim3 grid((unsigned)((N + kTile - 1) / kTile), (unsigned)((M + kTile - 1) / kTile), (unsigned)(batch * H));
    const int m = (int)M, k = (int)K, n = (int)N, h = (int)H;
    if (A.bf && B.bf) matmul_heads_kernel<true, true><<<grid, kThreads, 0, s>>>(A, B, C, m, k, n, h, scale, sC);
    else if (A.bf) matmul_heads_kernel<true, false><<<grid, kThreads, 0, s>>>(A, B, C, m, k, n, h, scale, sC);
    else if (B.bf) matmul_heads_kernel<false, true><<<grid, kThreads, 0, s>>>(A, B, C, m, k, n, h, scale, sC);
    else matmul_heads_kernel<false, false><<<grid, kThreads, 0, s>>>(A, B, C, m, k, n, h, scale, sC);
    PB_CUDA(cudaGetLastError());
}

}  // namespace pb
