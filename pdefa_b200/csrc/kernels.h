// Host-callable launchers for every device kernel of the engine. All kernels run
// on the caller's stream; none allocates memory.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace pb {

enum DType : int { F32 = 0, BF16 = 1 };

// Activation codes used in conv epilogues and unary kernels. 1-5 follow the
// reference's fused_activation numbering (session_fusion.inc:76-98 and
// Conv2dConfig::FusedActivation); 6 is SiLU evaluated the way the reference's
// Winograd kernel does (conv2d_winograd.cpp:81-101); >= 10 are unary-op kinds.
enum Act : int {
    ACT_NONE = 0, ACT_RELU = 1, ACT_LEAKY = 2, ACT_SIGMOID = 3, ACT_GELU_TANH = 4,
    ACT_SILU = 5, ACT_SILU_WINO = 6,
    UN_TANH = 10, UN_GELU = 11, UN_HARDSWISH = 12, UN_HARDSIGMOID = 13, UN_CLIP = 14,
    UN_COPY = 15,
};

enum BinOp : int { BIN_ADD = 0, BIN_SUB = 1, BIN_MUL = 2, BIN_DIV = 3 };

constexpr int kMaxRank = 8;

// A strided view of one image's worth of a tensor; `img_stride` advances to the
// next image (0 broadcasts one tensor over the batch). Strides are in elements.
struct TView {
    const void* ptr = nullptr;
    int dt = F32;
    int rank = 0;
    int64_t shape[kMaxRank] = {};
    int64_t stride[kMaxRank] = {};
    int64_t img_stride = 0;
};

// out[b, i...] = convert(in[b, i...]); shapes of in and out must match.
void launch_strided_copy(const TView& in, const TView& out, int64_t batch, cudaStream_t s);
// out = a (op) b with broadcasting expressed by zero strides; all views have out's rank.
void launch_binary(int op, const TView& a, const TView& b, const TView& out, int64_t batch, cudaStream_t s);
// out = act(in) for the unary kinds above (p0/p1: leaky slope or clip bounds).
void launch_unary(int kind, const TView& in, const TView& out, int64_t batch, float p0, float p1, cudaStream_t s);
// Softmax over `axis_len` elements spaced `inner` apart; dense fp32 in/out per image.
void launch_softmax(const float* in, float* out, int64_t outer, int64_t axis_len, int64_t inner,
                    int64_t img_elems, int64_t batch, cudaStream_t s);

// Reduction along one axis of a dense fp32 tensor laid out as [outer, axis_len, inner].
// mode: 0 max (init -3.4e38), 1 sum, 2 mean, 3 argmax (int32 out, strict '>' keeps the first).
void launch_reduce(int mode, const float* in, void* out, int64_t outer, int64_t axis_len, int64_t inner,
                   cudaStream_t s);
// out[o, j, i] = data[o, clamp(idx[j]), i] with negative indices wrapped and
// out-of-range ones mapped to 0 (engine_api.cpp gather semantics).
void launch_gather(const float* data, const int64_t* idx, float* out, int64_t outer, int64_t ax_dim,
                   int64_t n_idx, int64_t inner, cudaStream_t s);

struct Pool2dArgs {
    TView in, out;      // rank-4 NHWC views [1,H,W,C]
    int kh, kw, sh, sw, ph, pw;
    int mode;           // 0 max, 1 avg (count excludes padding), 2 global max, 3 global avg
    int64_t batch;
};
void launch_pool2d(const Pool2dArgs& a, cudaStream_t s);
// A chain of n <= 3 identical stride-1 'same' max pools (SPPF: y1 = pool(x), y2 =
// pool(y1), y3 = pool(y2)) in one launch: x is read once, every y_k written to out[k].
// Returns false (nothing launched) when the shapes or layouts do not allow it.
bool launch_maxpool_chain(const Pool2dArgs& a, const TView* out, int n, cudaStream_t s);
bool maxpool_chain_supported(const Pool2dArgs& a, const TView* out, int n);
// Nearest resize: out(h,w) = in(min(floor(h*Hin/H), Hin-1), ...) (session_ops_shape.inc:182-196).
void launch_resize_nearest(const TView& in, const TView& out, int64_t batch, cudaStream_t s);

// ---------------------------------------------------------------------------
// Convolution (NHWC implicit GEMM). Input/output/residual are strided rank-4 views.
// ---------------------------------------------------------------------------
struct ConvArgs {
    TView in;                 // [1,H,W,Cin]
    TView out;                // [1,Ho,Wo,Cout]
    TView res;                // optional residual added after the activation (ptr null = none)
    const void* weight = nullptr;   // packed per kernel family (see conv_*.cu)
    const float* bias = nullptr;
    int cin = 0, cout = 0, kh = 1, kw = 1, sh = 1, sw = 1, ph = 0, pw = 0, dh = 1, dw = 1;
    int act = ACT_NONE;
    float slope = 0.01f;
    int64_t batch = 1;
    long long wait_limit = 0;   // tcgen05 kernels: bounded-wait limit in SM cycles (0: default)
    // stem only: read the input as 8-bit RGB frames [batch, H, W, 3] (pixel * in_u8_scale,
    // the identity letterbox) instead of the fp32 NCHW view `in` (which still gives H, W)
    const uint8_t* in_u8 = nullptr;
    float in_u8_scale = 0.0f;
};
// Strict fp32 SIMT implicit GEMM. weight: fp32 [kh][kw][cin][cout].
void launch_conv_simt(const ConvArgs& a, cudaStream_t s);

// Grouped / depthwise conv: a.cin and a.cout are the full channel counts, each of the
// `groups` groups maps cin/groups input to cout/groups output channels; weight: fp32
// [cout][kh][kw][cin/groups].
void launch_conv_grouped(const ConvArgs& a, int groups, cudaStream_t s);

// Direct conv for tiny Cin (<= 8) and Cout <= 64 (the stem): fp32 FMA, weight
// packing as for launch_conv_simt.
bool conv_direct_supported(const ConvArgs& a);
void launch_conv_direct(const ConvArgs& a, cudaStream_t s);

// tcgen05 stem conv (BF16): kh*kw*Cin <= 32, Cout % 16 == 0 (<= 256), bf16 output, no
// residual; threads gather im2col rows into shared memory. weight: as launch_conv_simt.
// err: device error word for bounded waits.
// TMA tensor map over uint8 (elem_bytes 1) or fp32 (4) data of `rank` dims (innermost
// first; byte strides of dims 1..rank-1), no swizzle, zero fill out of bounds; `map`
// is a 64-byte-aligned CUtensorMap. False when the driver refuses the parameters.
bool encode_box_map(void* map, int elem_bytes, int rank, const void* ptr, const uint64_t* dims,
                    const uint64_t* strides_bytes, const uint32_t* box);
bool conv_stem_tc_supported(const ConvArgs& a);
void launch_conv_stem_tc(const ConvArgs& a, int* err, cudaStream_t s);

// tcgen05 / TMA implicit GEMM. weight: [cout][kh][kw][cin] in the operand type
// (bf16 for BF16, fp32 for TF32). Requires channel stride 1, 16-byte aligned pixel
// strides and channel offsets, cin % chunk == 0 and cout % 16 == 0 (checked by
// conv_tc_supported). err: device error word for bounded waits.
bool conv_tc_supported(const ConvArgs& a, int op_dt, const char** why);
void launch_conv_tc(const ConvArgs& a, int op_dt, int* err, cudaStream_t s);

// Strict fp32 GEMM: C[b] = A[b] (M x K, lda) * B[b] (K x N, ldb) (+ bias[N]); row-major.
void launch_gemm_f32(const float* A, const float* B, float* C, const float* bias,
                     int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldc,
                     int64_t batch, int64_t sA, int64_t sB, int64_t sC, cudaStream_t s);
// Attention MatMul on head-last 4-D tensors: C[b,i,j,h] = scale * sum_k A[b,i,k,h] * B[b,k,j,h]
// (fp32 fma over k in ascending order). Operands are strided views: element (b, r, c, h)
// of an operand is at p[b*sb + r*s1 + c*s2 + h*s3], fp32 or bf16 (bf = 1). C is dense
// [batch][M][N][H] with batch stride sC.
struct HeadOperand {
    const void* p = nullptr;
    int bf = 0;
    int64_t s1 = 0, s2 = 0, s3 = 0, sb = 0;
};
void launch_matmul_heads(const HeadOperand& A, const HeadOperand& B, float* C, int64_t batch, int64_t M, int64_t K,
                         int64_t N, int64_t H, float scale, int64_t sC, cudaStream_t s);
// Tensor-core GEMM for ops_matmul (TF32 or BF16 operands, fp32 accumulate/output).
// scratch must hold M*K + N*K operand-sized elements.
void launch_gemm_tc(const float* A, const float* B, float* C, int64_t M, int64_t N, int64_t K,
                    int op_dt, void* scratch, int* err, cudaStream_t s);

// ---------------------------------------------------------------------------
// YOLO head and decode.
// ---------------------------------------------------------------------------
struct YoloHeadArgs {
    TView level[3];           // rank-4 NHWC [1,H,W,4*reg+nc] views, one per stride level
    int nlevels = 3;
    int64_t level_anchors[3] = {};
    int reg_max = 16, nc = 80;
    const float* anchors = nullptr;    // [2, A] anchor points (x row then y row)
    const float* strides = nullptr;    // [A]
    const float* dfl_w = nullptr;      // [reg_max] DFL conv weights
    float* out = nullptr;              // [batch, 4+nc, A] fp32
    int64_t A = 0;
    int64_t batch = 1;
};
void launch_yolo_head(const YoloHeadArgs& a, cudaStream_t s);

struct DecodeArgs {
    const float* preds;         // [batch, channels, anchors]
    int64_t batch, channels, anchors;
    const int32_t* meta;        // [batch, 9] PdefaPreprocessMeta words or null
    double conf, iou;
    int max_det;
    // device outputs
    int32_t* counts;            // [batch]
    void* dets;                 // [batch, max_det] PdefaDetection records
    void* work;                 // scratch: decode_work_bytes(batch, anchors)
    int* err;
};
size_t decode_work_bytes(int64_t batch, int64_t anchors);
void launch_decode_nms(const DecodeArgs& a, cudaStream_t s);

// Letterbox preprocess geometry (imageloader/src/preprocess.cpp:22-54): target W x H,
// source src_w x src_h, scaled size sw x sh placed at (px, py), inv = 1 / ratio.
struct LetterboxGeom {
    int W, H, src_w, src_h, sw, sh, px, py;
    float ratio, inv, scale, pad;
};
LetterboxGeom letterbox_geometry(int src_w, int src_h, int W, int H, float scale, float pad);
// d_src: [n, src_h, src_w, channels] uint8 (channels 1, 3 or 4) -> d_out [n, 3, H, W] f32.
void launch_letterbox_u8(const uint8_t* d_src, int64_t n, int channels, const LetterboxGeom& g, float* d_out,
                         cudaStream_t s);

// TopK along the middle axis of [outer, L, inner] (dense fp32): the k largest values,
// descending, equal values lowest position first; positions written as exact floats
// (indices may be null). GatherElements: out[o, a, i] = data[o, idx[o, a, i], i]
// for idx [outer, K, inner], data [outer, L, inner] (negative counted from the end,
// out of range -> 0).
void launch_topk(const float* in, float* values, float* indices, int64_t outer, int64_t L, int64_t inner, int64_t k,
                 cudaStream_t s);
void launch_gather_elements(const float* data, const float* idx, float* out, int64_t outer, int64_t K, int64_t L,
                            int64_t inner, cudaStream_t s);

// GEMM on device pointers (engine_gemm_f32_device, engine_ops_matmul): strict FP32
// SIMT, or tcgen05 with operands staged in `scratch` (gemm_device_scratch_bytes).
size_t gemm_device_scratch_bytes(int64_t m, int64_t n, int64_t k, int precision);
void gemm_device(const float* d_a, const float* d_b, float* d_c, int64_t m, int64_t n, int64_t k, int precision,
                 void* scratch, cudaStream_t s);

}  // namespace pb
