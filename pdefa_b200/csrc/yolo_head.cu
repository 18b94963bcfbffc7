// Fused YOLOv8 Detect tail. Replaces the exported node chain
//   per-level Concat -> Reshape [1,no,-1] -> Concat(axis 2) -> Split(box, cls)
//   -> DFL (Reshape, Transpose, Softmax over 16 bins, 1x1 conv with arange weights,
//      Reshape) -> Split(lt, rb) -> anchor Sub/Add -> (x1y1+x2y2)/2, x2y2-x1y1
//   -> Concat -> Mul strides ; cls Sigmoid -> Concat -> [1, 4+nc, A]
// with one pass: each thread owns one anchor, reads its 4*reg_max + nc logits from
// the NHWC level tensor, and writes its 4 + nc output rows (coalesced over anchors).
// Arithmetic follows the reference's fp32 op sequence
// (session_ops_math.inc:223-318 softmax, :4-220 elementwise, activation_avx2.cpp:110
// sigmoid): max-shifted exp, sum, multiply by 1/sum, dot with the DFL weights,
// x1 = a - l, x2 = a + r, c = (x1 + x2) / 2, wh = x2 - x1, times the stride.
#include "common.h"
#include "device_common.cuh"

namespace pb {

namespace {

__global__ void yolo_head_kernel(YoloHeadArgs a) {
    const int64_t A = a.A;
    const int64_t total = A * a.batch;
    const int reg = a.reg_max, nc = a.nc;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total;
         t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t b = t / A, i = t - b * A;
        int lvl = 0;
        int64_t li = i;
        while (lvl < a.nlevels - 1 && li >= a.level_anchors[lvl]) { li -= a.level_anchors[lvl]; ++lvl; }
        const TView& v = a.level[lvl];
        const int64_t W = v.shape[2];
        const int64_t h = li / W, w = li - h * W;
        const int64_t base = b * v.img_stride + h * v.stride[1] + w * v.stride[2];
        float dist[4];
        for (int side = 0; side < 4; ++side) {
            float x[32];
            float mx = -1e30f;
            for (int k = 0; k < reg; ++k) {
                x[k] = ld_elem(v.ptr, v.dt, base + (side * reg + k) * v.stride[3]);
                mx = fmaxf(mx, x[k]);
            }
            float sum = 0.0f;
            for (int k = 0; k < reg; ++k) { x[k] = expf(x[k] - mx); sum += x[k]; }
            const float inv = sum > 0.0f ? __frcp_rn(sum) : 0.0f;   // = 1.0f / sum (both correctly rounded)
            float d = 0.0f;
            for (int k = 0; k < reg; ++k) d = fmaf(x[k] * inv, a.dfl_w[k], d);
            dist[side] = d;
        }
        const float ax = a.anchors[i], ay = a.anchors[A + i], st = a.strides[i];
        const float x1 = __fsub_rn(ax, dist[0]), y1 = __fsub_rn(ay, dist[1]);
        const float x2 = __fadd_rn(ax, dist[2]), y2 = __fadd_rn(ay, dist[3]);
        const float cx = __fdiv_rn(__fadd_rn(x1, x2), 2.0f), cy = __fdiv_rn(__fadd_rn(y1, y2), 2.0f);
        const float bw = __fsub_rn(x2, x1), bh = __fsub_rn(y2, y1);
        float* o = a.out + b * (int64_t)(4 + nc) * A + i;
        o[0] = __fmul_rn(cx, st);
        o[A] = __fmul_rn(cy, st);
        o[2 * A] = __fmul_rn(bw, st);
        o[3 * A] = __fmul_rn(bh, st);
        for (int c = 0; c < nc; ++c) {
            const float z = ld_elem(v.ptr, v.dt, base + (4 * reg + c) * v.stride[3]);
            o[(4 + c) * A] = __frcp_rn(1.0f + expf(-z));   // = 1.0f / (1.0f + e), correctly rounded
        }
    }
}

// Tiled variant for the usual layout (channels contiguous, 16-byte aligned pixel
// rows, reg_max 16): a CTA stages the logit rows of 64 consecutive anchors of one
// image in shared memory with coalesced 16-byte loads, then each thread decodes its
// anchor from shared memory with the arithmetic of yolo_head_kernel (same operation
// order, so the outputs are identical) and writes its 4 + nc output rows.
constexpr int kHeadAnchors = 64;

template <bool BF>
__device__ __forceinline__ void unpack8(uint4 q, float* f) {
    if (BF) {
        const uint32_t u[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const __nv_bfloat162 h2 = *reinterpret_cast<const __nv_bfloat162*>(&u[j]);
            f[2 * j] = __low2float(h2);
            f[2 * j + 1] = __high2float(h2);
        }
    } else {
        f[0] = __uint_as_float(q.x); f[1] = __uint_as_float(q.y);
        f[2] = __uint_as_float(q.z); f[3] = __uint_as_float(q.w);
    }
}

// BF16 plans (bf16 logits, results held to 1e-2) evaluate the exponentials with the
// hardware ex2 (__expf, ~2 ulp), the softmax normalisation with an approximate
// reciprocal, and the class sigmoid as 0.5 + 0.5 tanh(z / 2) with the hardware tanh:
// 148 special-function operations per anchor instead of 144 accurate expf and 84
// correctly rounded reciprocals, which made the kernel issue bound. FP32/TF32 plans
// (fp32 logits) keep the accurate sequence above.
__device__ __forceinline__ float head_tanh(float x) {
    float y;
    asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float head_rcp(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

template <bool BF>
__global__ void __launch_bounds__(kHeadAnchors) yolo_head_tile_kernel(YoloHeadArgs a, int tiles, int chunks,
                                                                      int row_chunks) {
    constexpr int kReg = 16;
    constexpr int kPer = BF ? 8 : 4;                   // values per 16-byte chunk
    extern __shared__ uint4 rows[];                    // [kHeadAnchors][row_chunks]
    __shared__ const char* src[kHeadAnchors];
    const int j = threadIdx.x;
    const int64_t b = blockIdx.x / tiles;
    const int64_t i = (int64_t)(blockIdx.x - b * tiles) * kHeadAnchors + j;
    const int64_t A = a.A;
    const int esz = BF ? 2 : 4;
    if (i < A) {
        int lvl = 0;
        int64_t li = i;
        while (lvl < a.nlevels - 1 && li >= a.level_anchors[lvl]) { li -= a.level_anchors[lvl]; ++lvl; }
        const TView& v = a.level[lvl];
        const int W = (int)v.shape[2];
        const int h = (int)(li / W), w = (int)(li - (int64_t)h * W);
        src[j] = static_cast<const char*>(v.ptr) + (b * v.img_stride + h * v.stride[1] + w * v.stride[2]) * esz;
    } else {
        src[j] = nullptr;
    }
    __syncthreads();
    // chunk idx = j + k * kHeadAnchors of the tile is (row r, piece q); (r, q) advance
    // by (kHeadAnchors / chunks, kHeadAnchors % chunks) per step, no division per load
    {
        int r = j / chunks, q = j - r * chunks;
        const int dr = kHeadAnchors / chunks, dq = kHeadAnchors - dr * chunks;
        for (int idx = j; idx < kHeadAnchors * chunks; idx += kHeadAnchors) {
            const char* p = src[r];
            if (p) rows[r * row_chunks + q] = __ldg(reinterpret_cast<const uint4*>(p) + q);
            r += dr;
            q += dq;
            if (q >= chunks) { q -= chunks; ++r; }
        }
    }
    __syncthreads();
    if (i >= A) return;
    const uint4* const row = rows + j * row_chunks;
    float dist[4];
#pragma unroll
    for (int side = 0; side < 4; ++side) {
        float x[kReg];
#pragma unroll
        for (int c = 0; c < kReg / kPer; ++c) unpack8<BF>(row[side * (kReg / kPer) + c], x + c * kPer);
        float mx = -1e30f;
#pragma unroll
        for (int k = 0; k < kReg; ++k) mx = fmaxf(mx, x[k]);
        float sum = 0.0f;
#pragma unroll
        for (int k = 0; k < kReg; ++k) { x[k] = BF ? __expf(x[k] - mx) : expf(x[k] - mx); sum += x[k]; }
        // = 1.0f / sum (correctly rounded on the fp32 path)
        const float inv = sum > 0.0f ? (BF ? head_rcp(sum) : __frcp_rn(sum)) : 0.0f;
        float d = 0.0f;
#pragma unroll
        for (int k = 0; k < kReg; ++k) d = fmaf(x[k] * inv, a.dfl_w[k], d);
        dist[side] = d;
    }
    const float ax = a.anchors[i], ay = a.anchors[A + i], st = a.strides[i];
    const float x1 = __fsub_rn(ax, dist[0]), y1 = __fsub_rn(ay, dist[1]);
    const float x2 = __fadd_rn(ax, dist[2]), y2 = __fadd_rn(ay, dist[3]);
    const float cx = __fdiv_rn(__fadd_rn(x1, x2), 2.0f), cy = __fdiv_rn(__fadd_rn(y1, y2), 2.0f);
    const float bw = __fsub_rn(x2, x1), bh = __fsub_rn(y2, y1);
    float* o = a.out + b * (int64_t)(4 + a.nc) * A + i;
    o[0] = __fmul_rn(cx, st);
    o[A] = __fmul_rn(cy, st);
    o[2 * A] = __fmul_rn(bw, st);
    o[3 * A] = __fmul_rn(bh, st);
    const int cls_chunks = a.nc / kPer;
    for (int c = 0; c < cls_chunks; ++c) {
        float z[kPer];
        unpack8<BF>(row[4 * kReg / kPer + c], z);
#pragma unroll
        for (int e = 0; e < kPer; ++e)
            o[(4 + c * kPer + e) * A] = BF ? fmaf(0.5f, head_tanh(0.5f * z[e]), 0.5f)
                                           : __frcp_rn(1.0f + expf(-z[e]));   // = 1 / (1 + e), correctly rounded
    }
}

// BF16 variant as a persistent kernel: each thread owns one anchor slot of the
// 64-anchor tiles its CTA walks (tile = blockIdx.x + n*gridDim.x) and prefetches its
// own anchor's next row (chunks x 16-byte cp.async; the row is contiguous in NHWC)
// into the other half of a double buffer while it computes the current one. No
// thread reads another's row, so there are no block barriers, and the HBM reads of
// tile n+1 overlap the special-function work of tile n (which the one-tile-per-CTA
// kernel above serialises with its own loads). Same arithmetic as its BF16 path.
__device__ __forceinline__ void head_cp16(uint4* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
                 : "memory");
}

__global__ void __launch_bounds__(kHeadAnchors) yolo_head_stream_kernel(YoloHeadArgs a, int tiles, int chunks,
                                                                        int row_chunks, int total_tiles) {
    constexpr int kReg = 16;
    constexpr int kPer = 8;                            // bf16 values per 16-byte chunk
    extern __shared__ uint4 rows[];                    // [2][kHeadAnchors][row_chunks]
    const int j = threadIdx.x;
    const int64_t A = a.A;
    // this thread's anchor of tile t: image b, index i; false past the last anchor
    auto anchor_of = [&](int t, int64_t& b, int64_t& i) {
        const int bt = t / tiles;
        b = bt;
        i = (int64_t)(t - bt * tiles) * kHeadAnchors + j;
        return i < A;
    };
    auto issue = [&](int t, uint4* dst) {
        int64_t b, i;
        if (!anchor_of(t, b, i)) return;
        int lvl = 0;
        int64_t li = i;
        while (lvl < a.nlevels - 1 && li >= a.level_anchors[lvl]) { li -= a.level_anchors[lvl]; ++lvl; }
        const TView& v = a.level[lvl];
        const int W = (int)v.shape[2];
        const int h = (int)li / W, w = (int)li - h * W;
        const uint4* src = reinterpret_cast<const uint4*>(static_cast<const char*>(v.ptr) +
                                                          (b * v.img_stride + h * v.stride[1] + w * v.stride[2]) * 2);
        for (int q = 0; q < chunks; ++q) head_cp16(dst + q, src + q);
    };
    // this thread's row in buffer k is rows + (k * kHeadAnchors + j) * row_chunks
    int k = 0;
    if ((int)blockIdx.x < total_tiles) issue(blockIdx.x, rows + j * row_chunks);
    asm volatile("cp.async.commit_group;" ::: "memory");
    for (int t = blockIdx.x; t < total_tiles; t += gridDim.x, k ^= 1) {
        const int tn = t + (int)gridDim.x;
        if (tn < total_tiles) issue(tn, rows + ((k ^ 1) * kHeadAnchors + j) * row_chunks);
        // one group per tile (possibly empty), so "all but the newest" is tile t's row
        asm volatile("cp.async.commit_group;" ::: "memory");
        asm volatile("cp.async.wait_group 1;" ::: "memory");
        int64_t b, i;
        if (!anchor_of(t, b, i)) continue;
        const uint4* const row = rows + (k * kHeadAnchors + j) * row_chunks;
        float dist[4];
#pragma unroll
        for (int side = 0; side < 4; ++side) {
            float x[kReg];
#pragma unroll
            for (int c = 0; c < kReg / kPer; ++c) unpack8<true>(row[side * (kReg / kPer) + c], x + c * kPer);
            float mx = -1e30f;
#pragma unroll
            for (int q = 0; q < kReg; ++q) mx = fmaxf(mx, x[q]);
            float sum = 0.0f;
#pragma unroll
            for (int q = 0; q < kReg; ++q) { x[q] = __expf(x[q] - mx); sum += x[q]; }
            const float inv = sum > 0.0f ? head_rcp(sum) : 0.0f;
            float d = 0.0f;
#pragma unroll
            for (int q = 0; q < kReg; ++q) d = fmaf(x[q] * inv, a.dfl_w[q], d);
            dist[side] = d;
        }
        const float ax = a.anchors[i], ay = a.anchors[A + i], st = a.strides[i];
        const float x1 = __fsub_rn(ax, dist[0]), y1 = __fsub_rn(ay, dist[1]);
        const float x2 = __fadd_rn(ax, dist[2]), y2 = __fadd_rn(ay, dist[3]);
        const float cx = __fdiv_rn(__fadd_rn(x1, x2), 2.0f), cy = __fdiv_rn(__fadd_rn(y1, y2), 2.0f);
        const float bw = __fsub_rn(x2, x1), bh = __fsub_rn(y2, y1);
        float* o = a.out + b * (int64_t)(4 + a.nc) * A + i;
        o[0] = __fmul_rn(cx, st);
        o[A] = __fmul_rn(cy, st);
        o[2 * A] = __fmul_rn(bw, st);
        o[3 * A] = __fmul_rn(bh, st);
        const int cls_chunks = a.nc / kPer;
        for (int c = 0; c < cls_chunks; ++c) {
            float z[kPer];
            unpack8<true>(row[4 * kReg / kPer + c], z);
#pragma unroll
            for (int e = 0; e < kPer; ++e) o[(4 + c * kPer + e) * A] = fmaf(0.5f, head_tanh(0.5f * z[e]), 0.5f);
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
}

bool head_tileable(const YoloHeadArgs& a) {
    if (a.reg_max != 16 || a.nlevels < 1 || a.nlevels > 3) return false;
    const int dt = a.level[0].dt;
    const int esz = dt == BF16 ? 2 : 4;
    if (dt != BF16 && dt != F32) return false;
    if ((a.nc * esz) % 16) return false;
    for (int l = 0; l < a.nlevels; ++l) {
        const TView& v = a.level[l];
        if (v.dt != dt || v.rank != 4 || v.stride[3] != 1 || ((uintptr_t)v.ptr) % 16) return false;
        if ((v.stride[2] * esz) % 16 || (v.stride[1] * esz) % 16 || (v.img_stride * esz) % 16) return false;
        if (v.shape[3] < 4 * a.reg_max + a.nc) return false;
    }
    return true;
}

}  // namespace

void launch_yolo_head(const YoloHeadArgs& a, cudaStream_t s) {
    if (a.reg_max > 32) fail(ENGINE_ERR_NOT_IMPL, "yolo head: reg_max > 32");
    const int64_t total = a.A * a.batch;
    if (!total) return;
    if (head_tileable(a)) {
        const bool bf = a.level[0].dt == BF16;
        const int chunks = (4 * a.reg_max + a.nc) * (bf ? 2 : 4) / 16;
        const int row_chunks = chunks | 1;         // odd: conflict-free 16-byte reads of one row per thread
        const int tiles = (int)((a.A + kHeadAnchors - 1) / kHeadAnchors);
        const int64_t blocks = (int64_t)tiles * a.batch;
        const size_t smem = (size_t)kHeadAnchors * row_chunks * 16;
        if (bf && blocks < (int64_t(1) << 31) && 2 * smem <= 48 * 1024) {
            // persistent grid: as many CTAs as fit on the device at once
            int dev = 0;
            PB_CUDA(cudaGetDevice(&dev));
            static int per_sm[64] = {}, sms[64] = {};
            int ps = 4, ns = 148;
            if (dev >= 0 && dev < 64) {
                if (!sms[dev]) {
                    PB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm[dev], yolo_head_stream_kernel,
                                                                          kHeadAnchors, 2 * smem));
                    PB_CUDA(cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev));
                }
                ps = per_sm[dev] > 0 ? per_sm[dev] : 1;
                ns = sms[dev];
            }
            const int64_t grid = std::min<int64_t>(blocks, (int64_t)ps * ns);
            yolo_head_stream_kernel<<<(unsigned)grid, kHeadAnchors, 2 * smem, s>>>(a, tiles, chunks, row_chunks,
                                                                                   (int)blocks);
            PB_CUDA(cudaGetLastError());
            return;
        }
        if (blocks < (int64_t(1) << 31) && smem <= 48 * 1024) {
            if (bf) yolo_head_tile_kernel<true><<<(unsigned)blocks, kHeadAnchors, smem, s>>>(a, tiles, chunks, row_chunks);
            else yolo_head_tile_kernel<false><<<(unsigned)blocks, kHeadAnchors, smem, s>>>(a, tiles, chunks, row_chunks);
            PB_CUDA(cudaGetLastError());
            return;
        }
    }
    int64_t blocks = (total + 127) / 128;
    if (blocks > 148 * 64) blocks = 148 * 64;
    yolo_head_kernel<<<(unsigned)blocks, 128, 0, s>>>(a);
    PB_CUDA(cudaGetLastError());
}

}  // namespace pb
