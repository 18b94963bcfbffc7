// TopK and GatherElements on the GPU (the YOLOv10 end-to-end tail), with the
// reference's semantics (PDEFA1.0/src/core/session_parts/session_ops_math.inc:321-433):
//
//   TopK(x, k, axis): along `axis` of each (outer, inner) slice, the k largest values in
//   descending order and their positions along the axis (k <= 0 or k > the axis length
//   means the whole axis; the largest flag is ignored, as in the reference). The
//   reference orders equal values as std::partial_sort leaves them, which the C++
//   standard does not specify; here equal values come lowest position first, so the
//   two agree whenever the k selected values are distinct.
//   GatherElements(data, idx, axis): out[o, a, i] = data[o, idx[o, a, i], i] with a
//   negative index counted from the end and an index still outside [0, L) read as 0.
//
// TopK: one CTA per slice. Every element becomes a 64-bit key, (order-flipped value
// bits << 32) | position, so ascending keys are values descending, positions ascending,
// and all keys differ. A most-significant-digit radix select (8 passes of 8 bits,
// shared-memory histograms, keys recomputed from the input on each pass: the slice is
// read 9 times, from L2 after the first) finds the k-th smallest key; the k keys up to
// it are gathered into shared memory, sorted by a bitonic network and written out.
#include <algorithm>
#include <climits>
#include <cstdint>

#include "common.h"
#include "device_common.cuh"

namespace pb {
namespace {

constexpr int kTopkThreads = 1024;
constexpr int kTopkMaxK = 4096;

__device__ __forceinline__ uint64_t topk_key(float v, uint32_t pos) {
    // float -> uint32 that sorts like the float (negatives flipped), then inverted so
    // that larger values give smaller keys
    uint32_t u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((uint64_t)(~u) << 32) | pos;
}

struct TopkArgs {
    const float* in;
    float* values;
    float* indices;        // positions, stored as exact float integers
    int64_t slices, L, inner, k;
};

__global__ void __launch_bounds__(kTopkThreads) topk_kernel(TopkArgs a) {
    __shared__ uint32_t hist[256];
    __shared__ uint64_t s_prefix, s_mask;
    __shared__ int64_t s_rank;
    __shared__ int s_count;
    extern __shared__ uint64_t sel[];      // kPow2 >= k keys
    const int64_t slice = blockIdx.x;
    const int64_t o = slice / a.inner, i = slice - o * a.inner;
    const float* base = a.in + o * a.L * a.inner + i;
    const int tid = threadIdx.x;
    if (tid == 0) { s_prefix = 0; s_mask = 0; s_rank = a.k; s_count = 0; }
    __syncthreads();
    // radix select: the k-th smallest key, 8 bits at a time from the top
    for (int shift = 56; shift >= 0; shift -= 8) {
        for (int b = tid; b < 256; b += kTopkThreads) hist[b] = 0;
        __syncthreads();
        const uint64_t prefix = s_prefix, mask = s_mask;
        for (int64_t p = tid; p < a.L; p += kTopkThreads) {
            const uint64_t key = topk_key(base[p * a.inner], (uint32_t)p);
            if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 0xFF], 1u);
        }
        __syncthreads();
        if (tid == 0) {
            int64_t r = s_rank;
            int b = 0;
            for (; b < 256; ++b) {
                if (r <= (int64_t)hist[b]) break;
                r -= hist[b];
            }
            s_prefix = prefix | ((uint64_t)b << shift);
            s_mask = mask | ((uint64_t)0xFF << shift);
            s_rank = r;
        }
        __syncthreads();
    }
    const uint64_t kth = s_prefix;
    // the k keys <= kth (keys are distinct, so exactly k)
    int n2 = 1;
    while (n2 < a.k) n2 <<= 1;
    for (int64_t p = tid; p < a.L; p += kTopkThreads) {
        const uint64_t key = topk_key(base[p * a.inner], (uint32_t)p);
        if (key <= kth) {
            const int q = atomicAdd(&s_count, 1);
            if (q < n2) sel[q] = key;
        }
    }
    __syncthreads();
    for (int q = s_count + tid; q < n2; q += kTopkThreads) sel[q] = ~0ull;
    __syncthreads();
    // bitonic sort, ascending
    for (int size = 2; size <= n2; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int t = tid; t < (n2 >> 1); t += kTopkThreads) {
                const int lo = 2 * t - (t & (stride - 1));
                const int hi = lo + stride;
                const bool up = (lo & size) == 0;
                const uint64_t x = sel[lo], y = sel[hi];
                if ((x > y) == up) { sel[lo] = y; sel[hi] = x; }
            }
            __syncthreads();
        }
    }
    float* vout = a.values + o * a.k * a.inner + i;
    float* iout = a.indices ? a.indices + o * a.k * a.inner + i : nullptr;
    for (int64_t j = tid; j < a.k; j += kTopkThreads) {
        const uint32_t pos = (uint32_t)(sel[j] & 0xFFFFFFFFu);
        vout[j * a.inner] = base[(int64_t)pos * a.inner];
        if (iout) iout[j * a.inner] = (float)pos;
    }
}

struct GatherElArgs {
    const float* data;
    const float* idx;      // exact float integers
    float* out;
    int64_t n, K, L, inner;
};

__global__ void gather_elements_kernel(GatherElArgs a) {
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < a.n; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = e % a.inner;
        const int64_t o = e / (a.inner * a.K);
        int64_t gi = (int64_t)a.idx[e];
        if (gi < 0) gi += a.L;
        if (gi < 0 || gi >= a.L) gi = 0;
        a.out[e] = a.data[(o * a.L + gi) * a.inner + i];
    }
}

}  // namespace

void launch_topk(const float* in, float* values, float* indices, int64_t outer, int64_t L, int64_t inner, int64_t k,
                 cudaStream_t s) {
    if (k < 1 || k > L) fail(ENGINE_ERR_INVALID_ARG, "topk: k out of range");
    if (k > kTopkMaxK) fail(ENGINE_ERR_NOT_IMPL, "topk: k above 4096");
    if (L > (int64_t)UINT32_MAX || outer * inner > (int64_t)INT_MAX) fail(ENGINE_ERR_NOT_IMPL, "topk: too large");
    const int64_t slices = outer * inner;
    if (slices == 0) return;
    int n2 = 1;
    while (n2 < k) n2 <<= 1;
    TopkArgs a{in, values, indices, slices, L, inner, k};
    topk_kernel<<<(unsigned)slices, kTopkThreads, (size_t)n2 * 8, s>>>(a);
    PB_CUDA(cudaGetLastError());
}

void launch_gather_elements(const float* data, const float* idx, float* out, int64_t outer, int64_t K, int64_t L,
                            int64_t inner, cudaStream_t s) {
    const int64_t n = outer * K * inner;
    if (n == 0) return;
    GatherElArgs a{data, idx, out, n, K, L, inner};
    const int64_t blocks = std::min<int64_t>((n + 255) / 256, 148 * 16);
    gather_elements_kernel<<<(unsigned)blocks, 256, 0, s>>>(a);
    PB_CUDA(cudaGetLastError());
}

}  // namespace pb
