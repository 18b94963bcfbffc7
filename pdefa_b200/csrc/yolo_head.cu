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
            const float inv = sum > 0.0f ? 1.0f / sum : 0.0f;
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
            o[(4 + c) * A] = 1.0f / (1.0f + expf(-z));
        }
    }
}

}  // namespace

void launch_yolo_head(const YoloHeadArgs& a, cudaStream_t s) {
    if (a.reg_max > 32) fail(ENGINE_ERR_NOT_IMPL, "yolo head: reg_max > 32");
    const int64_t total = a.A * a.batch;
    if (!total) return;
    int64_t blocks = (total + 127) / 128;
    if (blocks > 148 * 64) blocks = 148 * 64;
    yolo_head_kernel<<<(unsigned)blocks, 128, 0, s>>>(a);
    PB_CUDA(cudaGetLastError());
}

}  // namespace pb
