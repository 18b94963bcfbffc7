// Layout and memory-bound kernels: strided copy/convert, broadcast binary ops,
// unary activations, softmax, 2-D pooling and nearest resize. All operate on
// strided per-image views (TView) so the planner can express NHWC channel slices,
// NCHW<->NHWC conversions, permutations and broadcasts without extra copies.
#include <cfloat>

#include "common.h"
#include "device_common.cuh"

namespace pb {

namespace {

inline int grid_for(int64_t n, int threads) {
    int64_t b = (n + threads - 1) / threads;
    if (b > 148 * 32) b = 148 * 32;
    return (int)(b < 1 ? 1 : b);
}

int64_t view_numel(const TView& v) {
    int64_t n = 1;
    for (int d = 0; d < v.rank; ++d) n *= v.shape[d];
    return n;
}

__global__ void strided_copy_kernel(TView in, TView out, int64_t per_img, int64_t total) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t b = i / per_img, e = i - b * per_img;
        const float v = ld_elem(in.ptr, in.dt, b * in.img_stride + view_offset(in, e));
        st_elem(const_cast<void*>(out.ptr), out.dt, b * out.img_stride + view_offset(out, e), v);
    }
}

// Fast path: both views are a set of contiguous rows of `row` elements (the inner
// dimension has stride 1 on both sides), fp32 or bf16, copied 4 elements at a time.
__global__ void row_copy_kernel(TView in, TView out, int64_t row, int64_t rows_per_img, int64_t total_rows) {
    const int64_t vec = row / 4;
    const int64_t total = total_rows * vec;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / vec, q = i - r * vec;
        const int64_t b = r / rows_per_img, rr = r - b * rows_per_img;
        // offset of the row start: index rr*row over the view shape
        const int64_t oi = b * in.img_stride + view_offset(in, rr * row) + q * 4;
        const int64_t oo = b * out.img_stride + view_offset(out, rr * row) + q * 4;
        float v[4];
        if (in.dt == F32) {
            const float4 t = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(in.ptr) + oi);
            v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
        } else {
            const uint2 t = *reinterpret_cast<const uint2*>(reinterpret_cast<const __nv_bfloat16*>(in.ptr) + oi);
            const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&t.x);
            const __nv_bfloat162 c = *reinterpret_cast<const __nv_bfloat162*>(&t.y);
            v[0] = __low2float(a); v[1] = __high2float(a); v[2] = __low2float(c); v[3] = __high2float(c);
        }
        if (out.dt == F32) {
            *reinterpret_cast<float4*>(reinterpret_cast<float*>(const_cast<void*>(out.ptr)) + oo) =
                make_float4(v[0], v[1], v[2], v[3]);
        } else {
            __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]);
            __nv_bfloat162 c = __floats2bfloat162_rn(v[2], v[3]);
            uint2 t;
            t.x = *reinterpret_cast<uint32_t*>(&a);
            t.y = *reinterpret_cast<uint32_t*>(&c);
            *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(const_cast<void*>(out.ptr)) + oo) = t;
        }
    }
}

__global__ void binary_kernel(int op, TView a, TView b, TView out, int64_t per_img, int64_t total) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t n = i / per_img, e = i - n * per_img;
        const float x = ld_elem(a.ptr, a.dt, n * a.img_stride + view_offset(a, e));
        const float y = ld_elem(b.ptr, b.dt, n * b.img_stride + view_offset(b, e));
        float r;
        switch (op) {
            case BIN_ADD: r = __fadd_rn(x, y); break;
            case BIN_SUB: r = __fsub_rn(x, y); break;
            case BIN_MUL: r = __fmul_rn(x, y); break;
            default: r = __fdiv_rn(x, y); break;
        }
        st_elem(const_cast<void*>(out.ptr), out.dt, n * out.img_stride + view_offset(out, e), r);
    }
}

__global__ void unary_kernel(int kind, TView in, TView out, int64_t per_img, int64_t total, float p0, float p1) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t n = i / per_img, e = i - n * per_img;
        const float x = ld_elem(in.ptr, in.dt, n * in.img_stride + view_offset(in, e));
        st_elem(const_cast<void*>(out.ptr), out.dt, n * out.img_stride + view_offset(out, e),
                apply_act(x, kind, p0, p1));
    }
}

// One thread per (image, outer, inner) column: max, exp-sum, normalise.
__global__ void softmax_kernel(const float* in, float* out, int64_t outer, int64_t axis_len,
                               int64_t inner, int64_t img_elems, int64_t total) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t per = outer * inner;
        const int64_t b = i / per, r = i - b * per;
        const int64_t o = r / inner, k = r - o * inner;
        const float* src = in + b * img_elems + o * axis_len * inner + k;
        float* dst = out + b * img_elems + o * axis_len * inner + k;
        float mx = -1e30f;
        for (int64_t a = 0; a < axis_len; ++a) mx = fmaxf(mx, src[a * inner]);
        float sum = 0.0f;
        for (int64_t a = 0; a < axis_len; ++a) {
            const float e = expf(src[a * inner] - mx);
            dst[a * inner] = e;
            sum += e;
        }
        const float inv = sum > 0.0f ? 1.0f / sum : 0.0f;
        for (int64_t a = 0; a < axis_len; ++a) dst[a * inner] *= inv;
    }
}

// NHWC pooling, one thread per output element. Max pooling skips padded taps
// (pooling.cpp:35-101: init -FLT_MAX, out-of-range taps ignored).
__global__ void pool2d_kernel(Pool2dArgs a, int64_t total) {
    const int64_t H = a.in.shape[1], W = a.in.shape[2], C = a.in.shape[3];
    const int64_t Ho = a.out.shape[1], Wo = a.out.shape[2];
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        int64_t t = i;
        const int64_t c = t % C; t /= C;
        const int64_t wo = t % Wo; t /= Wo;
        const int64_t ho = t % Ho;
        const int64_t b = t / Ho;
        const int64_t base = b * a.in.img_stride + c * a.in.stride[3];
        float acc;
        if (a.mode >= 2) {
            acc = a.mode == 2 ? -FLT_MAX : 0.0f;
            for (int64_t h = 0; h < H; ++h)
                for (int64_t w = 0; w < W; ++w) {
                    const float v = ld_elem(a.in.ptr, a.in.dt, base + h * a.in.stride[1] + w * a.in.stride[2]);
                    acc = a.mode == 2 ? (v > acc ? v : acc) : acc + v;
                }
            if (a.mode == 3) acc = acc / (float)(H * W);
        } else {
            const int64_t h0 = ho * a.sh - a.ph, w0 = wo * a.sw - a.pw;
            acc = a.mode == 0 ? -FLT_MAX : 0.0f;
            int cnt = 0;
            for (int kh = 0; kh < a.kh; ++kh) {
                const int64_t h = h0 + kh;
                if (h < 0 || h >= H) continue;
                for (int kw = 0; kw < a.kw; ++kw) {
                    const int64_t w = w0 + kw;
                    if (w < 0 || w >= W) continue;
                    const float v = ld_elem(a.in.ptr, a.in.dt, base + h * a.in.stride[1] + w * a.in.stride[2]);
                    if (a.mode == 0) { if (v > acc) acc = v; }
                    else { acc += v; ++cnt; }
                }
            }
            if (a.mode == 1) acc = cnt ? acc / (float)cnt : 0.0f;
        }
        st_elem(const_cast<void*>(a.out.ptr), a.out.dt,
                b * a.out.img_stride + ho * a.out.stride[1] + wo * a.out.stride[2] + c * a.out.stride[3], acc);
    }
}

__global__ void resize_nearest_kernel(TView in, TView out, int64_t total, float sy, float sx) {
    const int64_t Hi = in.shape[1], Wi = in.shape[2], C = in.shape[3];
    const int64_t Ho = out.shape[1], Wo = out.shape[2];
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        int64_t t = i;
        const int64_t c = t % C; t /= C;
        const int64_t wo = t % Wo; t /= Wo;
        const int64_t ho = t % Ho;
        const int64_t b = t / Ho;
        int64_t hi = (int64_t)((float)ho * sy); if (hi > Hi - 1) hi = Hi - 1;
        int64_t wi = (int64_t)((float)wo * sx); if (wi > Wi - 1) wi = Wi - 1;
        const float v = ld_elem(in.ptr, in.dt, b * in.img_stride + hi * in.stride[1] + wi * in.stride[2] + c * in.stride[3]);
        st_elem(const_cast<void*>(out.ptr), out.dt,
                b * out.img_stride + ho * out.stride[1] + wo * out.stride[2] + c * out.stride[3], v);
    }
}

__global__ void reduce_kernel(int mode, const float* in, void* out, int64_t outer, int64_t axis_len,
                              int64_t inner) {
    const int64_t total = outer * inner;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total;
         t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t o = t / inner, i = t - o * inner;
        const float* base = in + o * axis_len * inner + i;
        if (mode == 3) {
            float best = base[0];
            int32_t bi = 0;
            for (int64_t k = 1; k < axis_len; ++k)
                if (base[k * inner] > best) { best = base[k * inner]; bi = (int32_t)k; }
            reinterpret_cast<int32_t*>(out)[t] = bi;
        } else if (mode == 0) {
            float mx = -3.4e38f;
            for (int64_t k = 0; k < axis_len; ++k) if (base[k * inner] > mx) mx = base[k * inner];
            reinterpret_cast<float*>(out)[t] = mx;
        } else {
            float s = 0.0f;
            for (int64_t k = 0; k < axis_len; ++k) s += base[k * inner];
            if (mode == 2) s = s / (float)axis_len;
            reinterpret_cast<float*>(out)[t] = s;
        }
    }
}

__global__ void gather_kernel(const float* data, const int64_t* idx, float* out, int64_t outer, int64_t ax_dim,
                              int64_t n_idx, int64_t inner) {
    const int64_t total = outer * n_idx * inner;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total;
         t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = t % inner;
        const int64_t j = (t / inner) % n_idx;
        const int64_t o = t / (inner * n_idx);
        int64_t g = idx[j];
        if (g < 0) g += ax_dim;
        if (g < 0 || g >= ax_dim) g = 0;
        out[t] = data[(o * ax_dim + g) * inner + i];
    }
}

// 16-byte vector paths for NHWC views whose channels are contiguous: one thread
// moves one pixel's group of 16 bytes (8 bf16 or 4 fp32 channels).
bool nhwc_vec16(const TView& v) {
    const int esz = v.dt == BF16 ? 2 : 4;
    const int64_t vec = 16 / esz;
    if (v.rank != 4 || v.stride[3] != 1 || v.shape[3] % vec) return false;
    if (((uintptr_t)v.ptr) % 16) return false;
    return (v.stride[2] % vec) == 0 && (v.stride[1] % vec) == 0 && (v.img_stride % vec) == 0;
}

__global__ void resize_nearest_vec_kernel(TView in, TView out, int64_t total, float sy, float sx, int vec) {
    const int64_t Hi = in.shape[1], Wi = in.shape[2], G = in.shape[3] / vec;
    const int64_t Ho = out.shape[1], Wo = out.shape[2];
    const int esz = in.dt == BF16 ? 2 : 4;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        int64_t t = i;
        const int64_t g = t % G; t /= G;
        const int64_t wo = t % Wo; t /= Wo;
        const int64_t ho = t % Ho;
        const int64_t b = t / Ho;
        int64_t hi = (int64_t)((float)ho * sy); if (hi > Hi - 1) hi = Hi - 1;
        int64_t wi = (int64_t)((float)wo * sx); if (wi > Wi - 1) wi = Wi - 1;
        const char* src = static_cast<const char*>(in.ptr) +
                          (b * in.img_stride + hi * in.stride[1] + wi * in.stride[2] + g * vec) * esz;
        char* dst = static_cast<char*>(const_cast<void*>(out.ptr)) +
                    (b * out.img_stride + ho * out.stride[1] + wo * out.stride[2] + g * vec) * esz;
        *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
    }
}

// Max pooling over 16-byte channel groups (bf16 compared as float; the result is one
// of the inputs, so no rounding happens).
__global__ void maxpool_vec_kernel(Pool2dArgs a, int64_t total, int vec) {
    const int64_t H = a.in.shape[1], W = a.in.shape[2], G = a.in.shape[3] / vec;
    const int64_t Ho = a.out.shape[1], Wo = a.out.shape[2];
    const bool bf = a.in.dt == BF16;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        int64_t t = i;
        const int64_t g = t % G; t /= G;
        const int64_t wo = t % Wo; t /= Wo;
        const int64_t ho = t % Ho;
        const int64_t b = t / Ho;
        float best[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) best[j] = -FLT_MAX;
        const int64_t h0 = ho * a.sh - a.ph, w0 = wo * a.sw - a.pw;
        for (int kh = 0; kh < a.kh; ++kh) {
            const int64_t h = h0 + kh;
            if (h < 0 || h >= H) continue;
            for (int kw = 0; kw < a.kw; ++kw) {
                const int64_t w = w0 + kw;
                if (w < 0 || w >= W) continue;
                const int64_t off = b * a.in.img_stride + h * a.in.stride[1] + w * a.in.stride[2] + g * vec;
                if (bf) {
                    const uint4 q = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(a.in.ptr) + off);
                    const uint32_t u[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const __nv_bfloat162 h2 = *reinterpret_cast<const __nv_bfloat162*>(&u[j]);
                        const float lo = __low2float(h2), hi = __high2float(h2);
                        if (lo > best[2 * j]) best[2 * j] = lo;
                        if (hi > best[2 * j + 1]) best[2 * j + 1] = hi;
                    }
                } else {
                    const float4 q = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(a.in.ptr) + off);
                    if (q.x > best[0]) best[0] = q.x;
                    if (q.y > best[1]) best[1] = q.y;
                    if (q.z > best[2]) best[2] = q.z;
                    if (q.w > best[3]) best[3] = q.w;
                }
            }
        }
        const int64_t oo = b * a.out.img_stride + ho * a.out.stride[1] + wo * a.out.stride[2] + g * vec;
        if (bf) {
            uint32_t u[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                __nv_bfloat162 h2 = __floats2bfloat162_rn(best[2 * j], best[2 * j + 1]);
                u[j] = *reinterpret_cast<uint32_t*>(&h2);
            }
            *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(const_cast<void*>(a.out.ptr)) + oo) =
                make_uint4(u[0], u[1], u[2], u[3]);
        } else {
            *reinterpret_cast<float4*>(reinterpret_cast<float*>(const_cast<void*>(a.out.ptr)) + oo) =
                make_float4(best[0], best[1], best[2], best[3]);
        }
    }
}

// Stride-1 max pooling of one image's channel slice held in shared memory
// (SPPF: 5x5, pad 2, on 20x20 maps): a row pass then a column pass over 16-byte
// channel cells. Every window keeps at least one in-image tap (pad < k), so the
// separable result is the 2-D window maximum exactly; values compare as float with
// the reference's -FLT_MAX start (pooling.cpp:35-101), and are stored in the source
// type (a maximum is one of its inputs, so nothing rounds).
template <bool BF>
__device__ __forceinline__ void cell_max(float* best, uint4 q) {
    if (BF) {
        const uint32_t u[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const __nv_bfloat162 h2 = *reinterpret_cast<const __nv_bfloat162*>(&u[j]);
            const float lo = __low2float(h2), hi = __high2float(h2);
            if (lo > best[2 * j]) best[2 * j] = lo;
            if (hi > best[2 * j + 1]) best[2 * j + 1] = hi;
        }
    } else {
        const float f[4] = {__uint_as_float(q.x), __uint_as_float(q.y), __uint_as_float(q.z), __uint_as_float(q.w)};
#pragma unroll
        for (int j = 0; j < 4; ++j)
            if (f[j] > best[j]) best[j] = f[j];
    }
}

template <bool BF>
__device__ __forceinline__ uint4 cell_pack(const float* best) {
    if (BF) {
        uint32_t u[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            __nv_bfloat162 h2 = __floats2bfloat162_rn(best[2 * j], best[2 * j + 1]);
            u[j] = *reinterpret_cast<uint32_t*>(&h2);
        }
        return make_uint4(u[0], u[1], u[2], u[3]);
    }
    return make_uint4(__float_as_uint(best[0]), __float_as_uint(best[1]), __float_as_uint(best[2]),
                      __float_as_uint(best[3]));
}

template <bool BF>
__global__ void __launch_bounds__(256) maxpool_s1_tile_kernel(Pool2dArgs a, int gc) {
    extern __shared__ uint4 cells[];        // [H][W][gc] input, then [H][Wo][gc] row maxima
    constexpr int kVec = BF ? 8 : 4;
    constexpr int kEsz = BF ? 2 : 4;
    const int H = (int)a.in.shape[1], W = (int)a.in.shape[2];
    const int Ho = (int)a.out.shape[1], Wo = (int)a.out.shape[2];
    uint4* const rows = cells + H * W * gc;
    const int64_t b = blockIdx.y;
    const int g0 = blockIdx.x * gc;
    const char* const in = static_cast<const char*>(a.in.ptr) + (b * a.in.img_stride + (int64_t)g0 * kVec) * kEsz;
    char* const out = static_cast<char*>(const_cast<void*>(a.out.ptr)) + (b * a.out.img_stride + (int64_t)g0 * kVec) * kEsz;
    for (int i = threadIdx.x; i < H * W * gc; i += blockDim.x) {
        const int c = i % gc, pix = i / gc, h = pix / W, w = pix - h * W;
        cells[i] = *reinterpret_cast<const uint4*>(in + (h * a.in.stride[1] + w * a.in.stride[2] + c * kVec) * kEsz);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < H * Wo * gc; i += blockDim.x) {
        const int c = i % gc, pix = i / gc, h = pix / Wo, wo = pix - h * Wo;
        float best[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) best[j] = -FLT_MAX;
        const int w0 = wo - a.pw;
        for (int k = 0; k < a.kw; ++k) {
            const int w = w0 + k;
            if (w >= 0 && w < W) cell_max<BF>(best, cells[(h * W + w) * gc + c]);
        }
        rows[i] = cell_pack<BF>(best);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < Ho * Wo * gc; i += blockDim.x) {
        const int c = i % gc, pix = i / gc, ho = pix / Wo, wo = pix - ho * Wo;
        float best[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) best[j] = -FLT_MAX;
        const int h0 = ho - a.ph;
        for (int k = 0; k < a.kh; ++k) {
            const int h = h0 + k;
            if (h >= 0 && h < H) cell_max<BF>(best, rows[(h * Wo + wo) * gc + c]);
        }
        *reinterpret_cast<uint4*>(out + (ho * a.out.stride[1] + wo * a.out.stride[2] + c * kVec) * kEsz) =
            cell_pack<BF>(best);
    }
}

// Chained stride-1 'same' max pools (SPPF) of one image's slice of gc channel cells:
// the input is loaded once into shared memory, then each pool of the chain runs a row
// pass into `rows` and a column pass back into `cells`, storing its result. Indices are
// split by shifts (gc is a power of two) and a multiply-shift by W (exact for the
// pixel counts allowed here: pix < 2^16), so no integer division runs per element.
struct PoolChainArgs {
    Pool2dArgs a;
    TView out[3];
    int n, gc_log2;
    uint32_t w_magic;        // ceil(2^16 / W): pix / W == (pix * w_magic) >> 16 (see launch_maxpool_chain)
};

template <bool BF>
__global__ void __launch_bounds__(256) maxpool_chain_kernel(PoolChainArgs P) {
    extern __shared__ uint4 cells[];        // [H][W][gc] current map, then [H][W][gc] row maxima
    constexpr int kVec = BF ? 8 : 4;
    constexpr int kEsz = BF ? 2 : 4;
    const Pool2dArgs& a = P.a;
    const int H = (int)a.in.shape[1], W = (int)a.in.shape[2];
    const int gc = 1 << P.gc_log2, gmask = gc - 1;
    const int HW = H * W, total = HW * gc;
    uint4* const rows = cells + total;
    const int64_t b = blockIdx.y;
    const int g0 = blockIdx.x * gc;
    const char* const in = static_cast<const char*>(a.in.ptr) + (b * a.in.img_stride + (int64_t)g0 * kVec) * kEsz;
    for (int i = threadIdx.x; i < total; i += blockDim.x) {
        const int c = i & gmask, pix = i >> P.gc_log2;
        const int h = (int)((uint32_t)pix * P.w_magic >> 16), w = pix - h * W;
        cells[i] = *reinterpret_cast<const uint4*>(in + (h * a.in.stride[1] + w * a.in.stride[2] + c * kVec) * kEsz);
    }
    for (int k = 0; k < P.n; ++k) {
        __syncthreads();
        for (int i = threadIdx.x; i < total; i += blockDim.x) {
            const int c = i & gmask, pix = i >> P.gc_log2;
            const int h = (int)((uint32_t)pix * P.w_magic >> 16), w = pix - h * W;
            float best[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) best[j] = -FLT_MAX;
            for (int t = 0; t < a.kw; ++t) {
                const int ww = w - a.pw + t;
                if (ww >= 0 && ww < W) cell_max<BF>(best, cells[((h * W + ww) << P.gc_log2) + c]);
            }
            rows[i] = cell_pack<BF>(best);
        }
        __syncthreads();
        const TView& o = P.out[k];
        char* const out = static_cast<char*>(const_cast<void*>(o.ptr)) + (b * o.img_stride + (int64_t)g0 * kVec) * kEsz;
        for (int i = threadIdx.x; i < total; i += blockDim.x) {
            const int c = i & gmask, pix = i >> P.gc_log2;
            const int h = (int)((uint32_t)pix * P.w_magic >> 16), w = pix - h * W;
            float best[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) best[j] = -FLT_MAX;
            for (int t = 0; t < a.kh; ++t) {
                const int hh = h - a.ph + t;
                if (hh >= 0 && hh < H) cell_max<BF>(best, rows[((hh * W + w) << P.gc_log2) + c]);
            }
            const uint4 v = cell_pack<BF>(best);
            cells[i] = v;                    // the next pool's input (rows only are read above)
            *reinterpret_cast<uint4*>(out + (h * o.stride[1] + w * o.stride[2] + c * kVec) * kEsz) = v;
        }
    }
}

// Nearest 2x upsample (out(h, w) = in(h / 2, w / 2), the reference's floor(h * Hin / H)
// for an exact factor of two): one thread reads one 16-byte channel cell and writes
// it to its four output pixels.
__global__ void resize_nearest_2x_kernel(TView in, TView out, int cells, int G, int Wi, int Hi, int esz, int vec) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < cells; i += gridDim.x * blockDim.x) {
        const int g = i % G;
        int t = i / G;
        const int wi = t % Wi;
        t /= Wi;
        const int hi = t % Hi;
        const int64_t b = t / Hi;
        const uint4 q = *reinterpret_cast<const uint4*>(static_cast<const char*>(in.ptr) +
            (b * in.img_stride + hi * in.stride[1] + wi * in.stride[2] + (int64_t)g * vec) * esz);
        char* const o = static_cast<char*>(const_cast<void*>(out.ptr)) +
                        (b * out.img_stride + (int64_t)(2 * hi) * out.stride[1] + (int64_t)(2 * wi) * out.stride[2] +
                         (int64_t)g * vec) * esz;
        *reinterpret_cast<uint4*>(o) = q;
        *reinterpret_cast<uint4*>(o + out.stride[2] * esz) = q;
        *reinterpret_cast<uint4*>(o + out.stride[1] * esz) = q;
        *reinterpret_cast<uint4*>(o + (out.stride[1] + out.stride[2]) * esz) = q;
    }
}

bool rows_vectorisable(const TView& in, const TView& out, int64_t* row) {
    if (in.rank < 1 || in.stride[in.rank - 1] != 1 || out.stride[out.rank - 1] != 1) return false;
    const int64_t r = in.shape[in.rank - 1];
    if (r % 4) return false;
    auto aligned = [](const TView& v) {
        const int esz = v.dt == F32 ? 4 : 2;
        if (((uintptr_t)v.ptr) % (4 * esz)) return false;
        if (v.img_stride % 4) return false;
        for (int d = 0; d < v.rank - 1; ++d) if (v.stride[d] % 4) return false;
        return true;
    };
    if (!aligned(in) || !aligned(out)) return false;
    *row = r;
    return true;
}

}  // namespace

void launch_strided_copy(const TView& in, const TView& out, int64_t batch, cudaStream_t s) {
    const int64_t per = view_numel(out);
    const int64_t total = per * batch;
    if (total == 0) return;
    int64_t row = 0;
    if (rows_vectorisable(in, out, &row)) {
        const int64_t rows_per_img = per / row;
        const int64_t n = rows_per_img * batch * (row / 4);
        row_copy_kernel<<<grid_for(n, 256), 256, 0, s>>>(in, out, row, rows_per_img, rows_per_img * batch);
    } else {
        strided_copy_kernel<<<grid_for(total, 256), 256, 0, s>>>(in, out, per, total);
    }
    PB_CUDA(cudaGetLastError());
}

void launch_binary(int op, const TView& a, const TView& b, const TView& out, int64_t batch, cudaStream_t s) {
    const int64_t per = view_numel(out), total = per * batch;
    if (!total) return;
    binary_kernel<<<grid_for(total, 256), 256, 0, s>>>(op, a, b, out, per, total);
    PB_CUDA(cudaGetLastError());
}

void launch_unary(int kind, const TView& in, const TView& out, int64_t batch, float p0, float p1, cudaStream_t s) {
    const int64_t per = view_numel(out), total = per * batch;
    if (!total) return;
    unary_kernel<<<grid_for(total, 256), 256, 0, s>>>(kind, in, out, per, total, p0, p1);
    PB_CUDA(cudaGetLastError());
}

void launch_softmax(const float* in, float* out, int64_t outer, int64_t axis_len, int64_t inner,
                    int64_t img_elems, int64_t batch, cudaStream_t s) {
    const int64_t total = outer * inner * batch;
    if (!total) return;
    softmax_kernel<<<grid_for(total, 256), 256, 0, s>>>(in, out, outer, axis_len, inner, img_elems, total);
    PB_CUDA(cudaGetLastError());
}

void launch_reduce(int mode, const float* in, void* out, int64_t outer, int64_t axis_len, int64_t inner,
                   cudaStream_t s) {
    const int64_t total = outer * inner;
    if (!total) return;
    reduce_kernel<<<grid_for(total, 256), 256, 0, s>>>(mode, in, out, outer, axis_len, inner);
    PB_CUDA(cudaGetLastError());
}

void launch_gather(const float* data, const int64_t* idx, float* out, int64_t outer, int64_t ax_dim,
                   int64_t n_idx, int64_t inner, cudaStream_t s) {
    const int64_t total = outer * n_idx * inner;
    if (!total) return;
    gather_kernel<<<grid_for(total, 256), 256, 0, s>>>(data, idx, out, outer, ax_dim, n_idx, inner);
    PB_CUDA(cudaGetLastError());
}

void launch_pool2d(const Pool2dArgs& a, cudaStream_t s) {
    const int64_t total = a.out.shape[1] * a.out.shape[2] * a.out.shape[3] * a.batch;
    if (!total) return;
    if (a.mode == 0 && a.in.dt == a.out.dt && nhwc_vec16(a.in) && nhwc_vec16(a.out) && a.sh == 1 && a.sw == 1 &&
        a.ph < a.kh && a.pw < a.kw && a.batch <= 65535) {
        // one CTA per image and slice of gc channel cells, both passes in shared memory
        const int vec = a.in.dt == BF16 ? 8 : 4;
        const int G = (int)(a.in.shape[3] / vec);
        const int64_t per_cell = (a.in.shape[1] * a.in.shape[2] + a.in.shape[1] * a.out.shape[2]) * 16;
        int gc = 0;
        for (int d = G; d >= 1; --d)
            if (G % d == 0 && per_cell * d <= 48 * 1024) { gc = d; break; }
        // keep at least two CTAs per SM busy
        while (gc > 1 && (G / gc) * a.batch < 296) {
            int d = gc - 1;
            while (d > 1 && G % d) --d;
            gc = d;
        }
        if (gc > 0) {
            const dim3 grid((unsigned)(G / gc), (unsigned)a.batch);
            const size_t smem = (size_t)per_cell * gc;
            if (a.in.dt == BF16) maxpool_s1_tile_kernel<true><<<grid, 256, smem, s>>>(a, gc);
            else maxpool_s1_tile_kernel<false><<<grid, 256, smem, s>>>(a, gc);
            PB_CUDA(cudaGetLastError());
            return;
        }
    }
    if (a.mode == 0 && a.in.dt == a.out.dt && nhwc_vec16(a.in) && nhwc_vec16(a.out)) {
        const int vec = a.in.dt == BF16 ? 8 : 4;
        maxpool_vec_kernel<<<grid_for(total / vec, 256), 256, 0, s>>>(a, total / vec, vec);
        PB_CUDA(cudaGetLastError());
        return;
    }
    pool2d_kernel<<<grid_for(total, 256), 256, 0, s>>>(a, total);
    PB_CUDA(cudaGetLastError());
}

// The chain kernel's configuration (log2 of the channel cells per CTA), or -1 when the
// shapes or layouts do not allow it.
static int maxpool_chain_cells_log2(const Pool2dArgs& a, const TView* out, int n) {
    if (n < 1 || n > 3 || a.mode != 0 || a.sh != 1 || a.sw != 1 || a.batch > 65535 || a.batch < 1) return -1;
    const int64_t H = a.in.shape[1], W = a.in.shape[2];
    // 'same' pooling (the output is the next pool's input) with an in-image tap in every window
    if (a.kh != 2 * a.ph + 1 || a.kw != 2 * a.pw + 1 || H * W >= 4096 || W < 1) return -1;
    // pix * w_magic / 2^16 = pix / W + d with w_magic = 2^16 / W + e, 0 <= e < 1, so
    // 0 <= d < pix / 2^16 < H * W / 2^16; the floor stays pix / W while d < 1 / W, i.e.
    // for H * W * W <= 2^16 (SPPF's 20 x 20 maps: 8000)
    if (H * W * W > 65536) return -1;
    if (!nhwc_vec16(a.in)) return -1;
    for (int k = 0; k < n; ++k)
        if (out[k].dt != a.in.dt || !nhwc_vec16(out[k]) || out[k].shape[1] != H || out[k].shape[2] != W ||
            out[k].shape[3] != a.in.shape[3])
            return -1;
    const int vec = a.in.dt == BF16 ? 8 : 4;
    const int G = (int)(a.in.shape[3] / vec);
    const int64_t per_cell = 2 * H * W * 16;
    int lg = -1;
    for (int l = 4; l >= 0; --l)
        if (G % (1 << l) == 0 && per_cell * (1 << l) <= 48 * 1024) { lg = l; break; }
    // keep at least two CTAs per SM busy
    while (lg > 0 && (G >> lg) * a.batch < 296) --lg;
    return lg;
}

bool maxpool_chain_supported(const Pool2dArgs& a, const TView* out, int n) {
    return maxpool_chain_cells_log2(a, out, n) >= 0;
}

bool launch_maxpool_chain(const Pool2dArgs& a, const TView* out, int n, cudaStream_t s) {
    const int lg = maxpool_chain_cells_log2(a, out, n);
    if (lg < 0) return false;
    const int64_t H = a.in.shape[1], W = a.in.shape[2];
    const int G = (int)(a.in.shape[3] / (a.in.dt == BF16 ? 8 : 4));
    const int64_t per_cell = 2 * H * W * 16;
    PoolChainArgs P;
    P.a = a;
    for (int k = 0; k < n; ++k) P.out[k] = out[k];
    P.n = n;
    P.gc_log2 = lg;
    P.w_magic = (uint32_t)((65536 + W - 1) / W);
    const dim3 grid((unsigned)(G >> lg), (unsigned)a.batch);
    const size_t smem = (size_t)per_cell << lg;
    if (a.in.dt == BF16) maxpool_chain_kernel<true><<<grid, 256, smem, s>>>(P);
    else maxpool_chain_kernel<false><<<grid, 256, smem, s>>>(P);
    PB_CUDA(cudaGetLastError());
    return true;
}

void launch_resize_nearest(const TView& in, const TView& out, int64_t batch, cudaStream_t s) {
    const int64_t total = out.shape[1] * out.shape[2] * out.shape[3] * batch;
    if (!total) return;
    const float sy = (float)in.shape[1] / (float)out.shape[1];
    const float sx = (float)in.shape[2] / (float)out.shape[2];
    if (in.dt == out.dt && nhwc_vec16(in) && nhwc_vec16(out) && out.shape[1] == 2 * in.shape[1] &&
        out.shape[2] == 2 * in.shape[2] && in.shape[1] * in.shape[2] * in.shape[3] * batch < (int64_t(1) << 31)) {
        const int vec = in.dt == BF16 ? 8 : 4;
        const int G = (int)(in.shape[3] / vec);
        const int cells = (int)(in.shape[1] * in.shape[2] * G * batch);
        resize_nearest_2x_kernel<<<grid_for(cells, 256), 256, 0, s>>>(in, out, cells, G, (int)in.shape[2],
                                                                       (int)in.shape[1], in.dt == BF16 ? 2 : 4, vec);
        PB_CUDA(cudaGetLastError());
        return;
    }
    if (in.dt == out.dt && nhwc_vec16(in) && nhwc_vec16(out)) {
        const int vec = in.dt == BF16 ? 8 : 4;
        resize_nearest_vec_kernel<<<grid_for(total / vec, 256), 256, 0, s>>>(in, out, total / vec, sy, sx, vec);
        PB_CUDA(cudaGetLastError());
        return;
    }
    resize_nearest_kernel<<<grid_for(total, 256), 256, 0, s>>>(in, out, total, sy, sx);
    PB_CUDA(cudaGetLastError());
}

}  // namespace pb
