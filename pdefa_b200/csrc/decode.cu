// Batched YOLO decode + class-wise greedy NMS, bit-exact with the reference's
// pure-Python decode_yolo / _nms / _iou (pdefa/python/src/pdefa/_bindings.py:1095-1212).
//
// A grid-wide pass evaluates every anchor, then one CTA per image (512 threads, two
// CTAs per SM, when its keys fit half an SM's shared memory; else 1024 threads):
//  1. candidates in anchor order: class argmax (strict '>', first maximum wins),
//     skip when best < conf; box (cx - w*0.5, cy - h*0.5, cx + w*0.5, cy + h*0.5) in
//     float64; optional letterbox unmap (v - pad) * (1.0 / ratio) clamped to
//     [0, orig] -- all with round-to-nearest float64 intrinsics, no contraction.
//     Order-preserving compaction uses warp ballots and a block scan.
//  2. class groups are ranked by the position of their first candidate (the
//     insertion order of the reference's defaultdict).
//  3. keys (conf desc, group, candidate index) are bitonic-sorted in shared memory:
//     the order of the reference's final stable sort of keep_all, which within a
//     class is also its per-class stable sort by confidence.
//  4. one greedy pass in that order keeps a box unless a kept box of its class has
//     IoU not <= iou_thres with it (IoU = inter / (area_a + area_b - inter + 1e-9),
//     0 when the overlap is empty) and stops after max_det kept boxes.
// Limit: at most 16384 anchors per image (keys live in shared memory).
#include <cfloat>
#include <atomic>
#include <climits>
#include <cstddef>

#include <mutex>

#include "../../include/pdefa_b200_ext.h"
#include "common.h"
#include "device_common.cuh"
#include "runtime.h"

namespace pb {

namespace {

constexpr int kMaxKeys = 16384;
constexpr int kMaxClasses = 1024;

// Shapes of the per-image NMS CTA. Both give the same output (the greedy pass is
// exact for any sub-block size); the small one takes 512 threads and about half the
// shared memory, so two CTAs share an SM and a batch of up to 2 x 148 images runs in
// one wave.
//   NT   threads (the kept test takes four per box, so SUB = NT / 4)
//   SUB  boxes settled per greedy sub-block
//   KEPT kept boxes mirrored in shared memory (float bounds + class)
//   TAB  entries of the per-class lists of mirrored kept boxes
template <int NT_, int KEPT_, int TAB_>
struct NmsShape {
    static constexpr int NT = NT_, NW = NT_ / 32, SUB = NT_ / 4, KEPT = KEPT_, TAB = TAB_;
    // dynamic shared memory after the keys and the class arrays: raw chunk (SUB) +
    // pending survivors (2 SUB) Det records | kept bounds + areas + classes (KEPT) |
    // survivor flags (SUB) | class lists
    static constexpr size_t kFixedSmem = 3 * SUB * 48 + KEPT * 44 + SUB * 4 + TAB * 4;
};
using NmsBig = NmsShape<1024, 512, 4096>;
using NmsSmall = NmsShape<512, 320, 2048>;

// keys (key_cap) | class first/group (2 ncp) | the shape's fixed part
template <class S>
constexpr size_t nms_smem(int64_t key_cap, int64_t ncp) {
    return (size_t)key_cap * 8 + (size_t)ncp * 8 + S::kFixedSmem;
}

// Size R of the sorted prefix (segment 0) of the greedy order: max_det * 8, at least
// 3968 (a little under a power of two: the sort pads to one), capped so that the
// product cannot overflow. It only splits the work; the output does not depend on it.
__host__ __device__ inline int nms_prefix_rank(int max_det) {
    if (max_det > (1 << 20)) return 1 << 23;
    return max_det * 8 > 3968 ? max_det * 8 : 3968;
}

struct Det {
    double x1, y1, x2, y2;
    float conf;
    int32_t cls;
    int32_t anchor;
    int32_t reserved;
};
static_assert(sizeof(Det) == 48, "Det must match PdefaDetection");
// a kept box's bounds and area, mirrored in shared memory for the kept test
struct Box {
    double x1, y1, x2, y2, area;
};
// the NMS reads a record's tail (conf, cls, anchor, reserved) as one 16-byte load
static_assert(offsetof(Det, conf) == 32 && offsetof(Det, cls) == 36 && offsetof(Det, anchor) == 40 &&
                  offsetof(Det, reserved) == 44,
              "Det tail layout");

__device__ __forceinline__ uint32_t desc_key(float f) {
    uint32_t u = __float_as_uint(f == 0.0f ? 0.0f : f);       // -0.0 orders as +0.0
    const uint32_t asc = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ~asc;
}

// Whether the reference's IoU (_bindings.py _iou: inter / (area_a + area_b - inter +
// 1e-9) in float64, 0 without overlap) is NOT <= thr, decided exactly but with the
// float64 division only where needed. With D the reference's rounded denominator and
// q the exact quotient inter / D, the reference's IoU is rn(q). e = fma(-thr, D, inter) has the sign of
// q - thr (one rounding keeps a nonzero sign). e <= 0: q <= thr, so rn(q) <= thr (thr is
// a double and rounding is monotone). e > 2 ulp(thr) D: q - thr > ulp(thr) even after
// e's rounding, so rn(q) > thr. Only q within ~2 ulp above thr (and odd inputs:
// thr outside (0,1), D <= 0 or NaN) take the division.
__device__ __forceinline__ double box_area(double x1, double y1, double x2, double y2) {
    return __dmul_rn(__dsub_rn(x2, x1), __dsub_rn(y2, y1));
}
template <class B>
__device__ __forceinline__ double box_area(const B& b) {
    return box_area(b.x1, b.y1, b.x2, b.y2);
}

// area_a and area_b are box_area(a) and box_area(b), passed in so that a box tested
// against many others computes its own once.
template <class BA, class BB>
__device__ __forceinline__ bool iou_exceeds(const BA& a, double area_a, const BB& b, double area_b, double thr,
                                            double two_ulp_thr) {
    const double x1 = a.x1 > b.x1 ? a.x1 : b.x1;
    const double y1 = a.y1 > b.y1 ? a.y1 : b.y1;
    const double x2 = a.x2 < b.x2 ? a.x2 : b.x2;
    const double y2 = a.y2 < b.y2 ? a.y2 : b.y2;
    const double w = __dsub_rn(x2, x1);
    const double h = __dsub_rn(y2, y1);
    if (w <= 0.0 || h <= 0.0) return !(0.0 <= thr);
    const double inter = __dmul_rn(w, h);
    const double D = __dadd_rn(__dsub_rn(__dadd_rn(area_a, area_b), inter), 1e-9);
    if (thr > 0.0 && thr < 1.0 && D > 0.0) {
        const double e = __fma_rn(-thr, D, inter);
        if (e <= 0.0) return false;
        if (e > __dmul_rn(two_ulp_thr, D)) return true;
    }
    return !(__ddiv_rn(inter, D) <= thr);
}

__device__ __forceinline__ double clamp_ref(double v, double hi) {
    return v < 0.0 ? 0.0 : (v > hi ? hi : v);
}

// Bitonic sort of np (a power of two) keys, ascending. Strides of 128 and more run
// in shared memory with a barrier per pass (every thread takes whole compare-exchange
// pairs); the strides below 128 of every stage run in registers: warp w holds
// 128-key groups g = w, w + kWarps, ... with key g*128 + 32*r + lane in register r of
// its lane (r = 0..3), so every warp load and store of the group touches consecutive
// keys (no bank conflicts: the sort moves its keys through shared memory once per
// stage and is bound by that bandwidth); strides 32 and 64 pair registers of one
// lane, strides 1 ... 16 pair lanes by shuffles, with one barrier per stage.
__device__ __forceinline__ void cmp_swap_reg(unsigned long long& lo, unsigned long long& hi, bool asc) {
    if ((lo > hi) == asc) { const unsigned long long t = lo; lo = hi; hi = t; }
}

template <int kThreads>
__device__ void bitonic_sort(unsigned long long* keys, int np) {
    constexpr int kWarps = kThreads / 32;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (np < 128) {
        const int half = np >> 1;
        for (int k = 2; k <= np; k <<= 1) {
            for (int j = k >> 1; j > 0; j >>= 1) {
                for (int t = threadIdx.x; t < half; t += kThreads) {
                    const int i = ((t & ~(j - 1)) << 1) | (t & (j - 1));
                    const int ixj = i | j;
                    const unsigned long long a = keys[i], b = keys[ixj];
                    const bool asc = (i & k) == 0;
                    if ((a > b) == asc) { keys[i] = b; keys[ixj] = a; }
                }
                __syncthreads();
            }
        }
        return;
    }
    const int half = np >> 1;
    // stage k (sequence length): register passes for strides min(k/2, 64) ... 1
    auto reg_passes = [&](int k) {
        for (int g = warp; g < (np >> 7); g += kWarps) {
            unsigned long long* const base = keys + g * 128 + lane;
            unsigned long long v0 = base[0], v1 = base[32], v2 = base[64], v3 = base[96];
            const int e0 = g * 128 + lane;       // key index of v0; v_r is e0 + 32 r
            for (int j = (k >> 1) < 64 ? (k >> 1) : 64; j > 0; j >>= 1) {
                if (j == 64) {
                    // pairs (v0, v2), (v1, v3); k >= 128, so bit k is shared by all four
                    const bool asc = (e0 & k) == 0;
                    cmp_swap_reg(v0, v2, asc);
                    cmp_swap_reg(v1, v3, asc);
                } else if (j == 32) {
                    cmp_swap_reg(v0, v1, (e0 & k) == 0);
                    cmp_swap_reg(v2, v3, ((e0 + 64) & k) == 0);
                } else {
                    // partner lane ^ j holds the other key of each pair
                    const bool lower = (lane & j) == 0;
                    // the lower element keeps the smaller key when ascending
                    auto step = [&](unsigned long long x, int e) {
                        const unsigned long long o = __shfl_xor_sync(0xffffffffu, x, j);
                        return (lower == ((e & k) == 0)) ? (o < x ? o : x) : (o > x ? o : x);
                    };
                    v0 = step(v0, e0);
                    v1 = step(v1, e0 + 32);
                    v2 = step(v2, e0 + 64);
                    v3 = step(v3, e0 + 96);
                }
            }
            base[0] = v0; base[32] = v1; base[64] = v2; base[96] = v3;
        }
        __syncthreads();
    };
    for (int k = 2; k <= np; k <<= 1) {
        for (int j = k >> 1; j >= 128; j >>= 1) {
            for (int t = threadIdx.x; t < half; t += kThreads) {
                const int i = ((t & ~(j - 1)) << 1) | (t & (j - 1));
                const int ixj = i | j;
                const unsigned long long a = keys[i], b = keys[ixj];
                const bool asc = (i & k) == 0;
                if ((a > b) == asc) { keys[i] = b; keys[ixj] = a; }
            }
            __syncthreads();
        }
        reg_passes(k);
    }
}

// Per anchor (all images, whole grid): class argmax (strict '>', first maximum),
// the conf test, the float64 box and the optional letterbox unmap. The record goes
// to the anchor's slot of the work area with `reserved` = 1 when it is a candidate.
__global__ void decode_candidates_kernel(DecodeArgs p) {
    const int64_t A = p.anchors, total = p.batch * A;
    const int nc = (int)p.channels - 4;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total;
         t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t b = t / A, a = t - b * A;
        const float* pr = p.preds + b * p.channels * A;
        float best = pr[4 * A + a];
        int best_c = 0;
        for (int c = 1; c < nc; ++c) {
            const float s = pr[(4 + c) * A + a];
            if (s > best) { best = s; best_c = c; }
        }
        Det d;
        d.x1 = d.y1 = d.x2 = d.y2 = 0.0;
        const bool flag = !((double)best < p.conf);
        if (flag) {
            const double cx = pr[a], cy = pr[A + a], w = pr[2 * A + a], h = pr[3 * A + a];
            const double hw = __dmul_rn(w, 0.5), hh = __dmul_rn(h, 0.5);
            d.x1 = __dsub_rn(cx, hw); d.y1 = __dsub_rn(cy, hh);
            d.x2 = __dadd_rn(cx, hw); d.y2 = __dadd_rn(cy, hh);
            if (p.meta) {
                const int32_t* m = p.meta + b * 9;
                const double ow = (double)m[2], oh = (double)m[3], px = (double)m[4], py = (double)m[5];
                const double scale = __ddiv_rn(1.0, (double)__int_as_float(m[8]));
                d.x1 = clamp_ref(__dmul_rn(__dsub_rn(d.x1, px), scale), ow);
                d.y1 = clamp_ref(__dmul_rn(__dsub_rn(d.y1, py), scale), oh);
                d.x2 = clamp_ref(__dmul_rn(__dsub_rn(d.x2, px), scale), ow);
                d.y2 = clamp_ref(__dmul_rn(__dsub_rn(d.y2, py), scale), oh);
            }
        }
        d.conf = best; d.cls = best_c; d.anchor = (int32_t)a; d.reserved = flag ? 1 : 0;
        reinterpret_cast<Det*>(p.work)[t] = d;
    }
}

// key_cap: capacity of the key array (>= anchors; 16384 for the big shape); ncp: length
// of each class array (>= the class count, even, so that the records after them stay
// 16-byte aligned).
template <class S>
__global__ void __launch_bounds__(S::NT, 1024 / S::NT) decode_nms_kernel(DecodeArgs p, int key_cap, int ncp) {
    constexpr int kThreads = S::NT, kWarps = S::NW, kSub = S::SUB, kKeptSmem = S::KEPT, kClsTab = S::TAB;
    extern __shared__ unsigned long long keys[];                       // key_cap
    int* first = reinterpret_cast<int*>(keys + key_cap);               // ncp
    int* grp = first + ncp;                  // ncp: group ranks
    __shared__ int warp_tot[32];
    __shared__ int s_n, s_kept;

    const int b = blockIdx.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t A = p.anchors;
    const int nc = (int)p.channels - 4;
    Det* cand = reinterpret_cast<Det*>(p.work) + (int64_t)b * A;
    Det* out = reinterpret_cast<Det*>(p.dets) + (int64_t)b * p.max_det;

    for (int c = tid; c < ncp; c += kThreads) first[c] = INT_MAX;
    if (tid == 0) { s_n = 0; s_kept = 0; }
    __syncthreads();

    // ---- 1. the candidates marked by decode_candidates_kernel, in anchor order ----
    // keys[k] = anchor of candidate k (records stay at their anchor slots). Every
    // thread reads the 16-byte tails (conf, cls, anchor, flag) of kChunks records of a
    // round before one block scan of all their flags, so a round costs one record
    // latency and three barriers for kChunks * kThreads anchors. The first call also
    // records each class's first candidate.
    constexpr int kChunks = 4;
    __shared__ int chunk_tot[kChunks * kWarps];
    auto compact = [&](bool classes) {
        if (tid == 0) s_n = 0;
        __syncthreads();
        for (int64_t a0 = 0; a0 < A; a0 += (int64_t)kChunks * kThreads) {
            bool flag[kChunks];
            int cls[kChunks];
            unsigned bal[kChunks];
#pragma unroll
            for (int c = 0; c < kChunks; ++c) {
                const int64_t a = a0 + c * kThreads + tid;
                flag[c] = false;
                cls[c] = 0;
                if (a < A) {
                    const int4 tail = *reinterpret_cast<const int4*>(reinterpret_cast<const char*>(cand + a) + 32);
                    flag[c] = tail.w != 0;        // reserved
                    cls[c] = tail.y;
                }
            }
#pragma unroll
            for (int c = 0; c < kChunks; ++c) {
                bal[c] = __ballot_sync(0xffffffffu, flag[c]);
                if (lane == 0) chunk_tot[c * kWarps + warp] = __popc(bal[c]);
            }
            __syncthreads();
            if (warp == 0) {
                // inclusive scan over (chunk, warp) in anchor order, kChunks * kWarps <= 64 counts
                constexpr int kPer = (kChunks * kWarps + 31) / 32;
                int v[kPer], tot = 0;
#pragma unroll
                for (int q = 0; q < kPer; ++q) {
                    const int e = lane * kPer + q;
                    v[q] = e < kChunks * kWarps ? chunk_tot[e] : 0;
                    tot += v[q];
                }
                int incl = tot;
                for (int o = 1; o < 32; o <<= 1) {
                    const int t = __shfl_up_sync(0xffffffffu, incl, o);
                    if (lane >= o) incl += t;
                }
                int run = incl - tot;
#pragma unroll
                for (int q = 0; q < kPer; ++q) {
                    const int e = lane * kPer + q;
                    run += v[q];
                    if (e < kChunks * kWarps) chunk_tot[e] = run;
                }
            }
            __syncthreads();
            const int base = s_n;
#pragma unroll
            for (int c = 0; c < kChunks; ++c) {
                if (flag[c]) {
                    const int e = c * kWarps + warp;
                    const int k = base + (e ? chunk_tot[e - 1] : 0) + __popc(bal[c] & ((1u << lane) - 1u));
                    if (k < key_cap) {
                        keys[k] = (unsigned long long)(a0 + c * kThreads + tid);
                        if (classes) atomicMin(&first[cls[c]], k);
                    }
                }
            }
            __syncthreads();
            if (tid == 0) s_n = base + chunk_tot[kChunks * kWarps - 1];
            __syncthreads();
        }
    };
    compact(true);
    const int n = s_n;
    if (n > key_cap) {
        if (tid == 0) p.counts[b] = -1;
        return;
    }

    // ---- 2. class group rank = order of first appearance ----
    for (int c = tid; c < nc; c += kThreads) {
        int g = -1;
        const int f = first[c];
        if (f != INT_MAX) {
            g = 0;
            for (int c2 = 0; c2 < nc; ++c2) g += first[c2] < f;
        }
        grp[c] = g;
    }
    __syncthreads();
    // the class-first array becomes the per-class kept counts (all zero)
    for (int c = tid; c < ncp; c += kThreads) first[c] = 0;
    __syncthreads();

    // ---- 3. the output order: (conf desc, class group, index) ----
    // The greedy pass below settles boxes in this order and stops at max_det kept, so
    // with many candidates it usually needs only a prefix of the order: segment 0 is
    // the prefix {key <= T}, T the R-th smallest key (radix select over the whole
    // keys, which are distinct: exactly R boxes, however many confidences tie); only
    // when the pass runs out of it before max_det boxes are kept is segment 1, the
    // rest, sorted and the pass continued on it. Without selection segment 0 is all n
    // boxes.
    __shared__ int hist[256];
    __shared__ unsigned long long s_prefix;
    __shared__ int s_rem, s_sel;
    const int R = nms_prefix_rank(p.max_det);
    const bool select = n > R && R <= key_cap / 2;
    unsigned long long T = ~0ull;
    // ---- 4. one greedy pass in output order ----
    // A box's same-class predecessors in the reference's per-class order all come
    // before it in this order, so deciding boxes in this order keeps exactly the
    // boxes the per-class greedy keeps, and the first max_det kept are the output.
    // Rounds: (a) raw chunks of kSub boxes in order are tested against every box kept
    // so far and the survivors appended, in order, to a pending list until it holds
    // kSub boxes or the order is exhausted; (b) the pending boxes (< 2 kSub, one thread
    // each) are decided in order: the first one still alive is kept, every later one
    // of its class with IoU not <= thres dies, and so on, one barrier per kept box.
    // With heavy suppression most boxes die in (a), against earlier rounds' kept boxes.
    Det* raw = reinterpret_cast<Det*>(grp + ncp);                      // kSub
    Det* sub = raw + kSub;                                             // 2 * kSub pending
    Box* kept_b = reinterpret_cast<Box*>(sub + 2 * kSub);              // kKeptSmem kept boxes
    int* kept_c = reinterpret_cast<int*>(kept_b + kKeptSmem);          // kKeptSmem classes
    int* flag = kept_c + kKeptSmem;                                    // kSub
    // kept boxes below kKeptSmem listed by class: cls_tab[cls * cap + e], e < cls_cnt[cls]
    // (the class-first array, free once the group ranks exist); a class with more than
    // cap of them is scanned instead
    int* cls_tab = flag + kSub;                                        // kClsTab
    int* cls_cnt = first;
    const int cap = kClsTab / (nc > 64 ? nc : 64) < 64 ? kClsTab / (nc > 64 ? nc : 64) : 64;
    __shared__ uint32_t s_words[2 * (kSub / 16)];
    __shared__ int s_np;
    // 2 ulp(thr) for thr in (0, 1) (used only there)
    const double two_ulp = p.iou > 0.0 && p.iou < 1.0
        ? 2.0 * (__longlong_as_double(__double_as_longlong(p.iou) + 1) - p.iou) : 0.0;
    // flag[j] = 1 when box j of `list` (cnt <= kSub boxes) is suppressed by a kept box in
    // [k0, k1). Kept boxes below kKeptSmem: four threads per box (consecutive lanes)
    // split its class's list (or, for a class past its list's capacity, the mirrored
    // kept range), newest first (the latest kept boxes of a class lie nearest in the
    // order, so they are the likeliest suppressors), and the four stop together at the
    // first suppressor any of them finds. Kept boxes from kKeptSmem on (max_det above
    // the mirror): lanes take the boxes (32 per warp) and the warps sharing a group of
    // 32 split that kept range, so every kept box is read by all lanes at once.
    auto test_kept = [&](const Det* list, int cnt, int k0, int k1) {
        {
            const int j = tid >> 2, q = tid & 3;
            const unsigned quad = 0xFu << (lane & ~3);
            const int lim = k1 < kKeptSmem ? k1 : kKeptSmem;
            bool live = j < cnt && k0 < lim, sup = false, listed = false;
            Det c;
            double area_c = 0.0;
            const int* tab = cls_tab;
            int e = 0, e_end = 0;
            if (live) {
                c = list[j];
                area_c = box_area(c);
                const int nk = cls_cnt[c.cls];
                listed = nk <= cap;
                tab = cls_tab + c.cls * cap;
                e = (listed ? nk : lim) - 1 - q;
                e_end = listed ? 0 : k0;
                live = e >= e_end;
            }
            while (__any_sync(0xffffffffu, live)) {
                bool hit = false;
                if (live) {
                    const int r = listed ? tab[e] : e;
                    hit = (listed ? r >= k0 && r < lim : kept_c[r] == c.cls) &&
                          iou_exceeds(kept_b[r], kept_b[r].area, c, area_c, p.iou, two_ulp);
                }
                if (__ballot_sync(0xffffffffu, hit) & quad) { sup = true; live = false; }
                e -= 4;
                if (e < e_end) live = false;
            }
            if (q == 0 && j < cnt) flag[j] = sup ? 1 : 0;
        }
        const int s0 = k0 > kKeptSmem ? k0 : kKeptSmem;
        if (k1 > s0) __syncthreads();           // the scan below adds to the results above
        const int groups = k1 > s0 ? (cnt + 31) >> 5 : 0;
        if (groups > 0) {
            const int slices = kWarps / groups;
            const int gsel = warp % groups, slice = warp / groups;
            const int j = gsel * 32 + lane;
            const bool valid = j < cnt && slice < slices;
            Det c;
            double area_c = 0.0;
            if (valid) { c = list[j]; area_c = box_area(c); }
            bool sup = !valid;
            if (slice < slices) {
                for (int r = s0 + slice; r < k1; r += slices) {
                    if (!sup) {
                        const Det& o = out[r];
                        if (o.cls == c.cls && iou_exceeds(o, box_area(o), c, area_c, p.iou, two_ulp)) sup = true;
                    }
                    if (((r - s0) & 7) == 7 && __all_sync(0xffffffffu, sup)) break;
                }
            }
            if (valid && sup) flag[j] = 1;
        }
        __syncthreads();
    };
    // appends the unflagged boxes of list[0..cnt) to sub[dst..], in order (cnt <= kThreads)
    auto append_survivors = [&](const Det* list, int cnt, int dst) {
        const bool keep = tid < cnt && !flag[tid];
        Det d;
        if (keep) d = list[tid];
        const unsigned bal = __ballot_sync(0xffffffffu, keep);
        if (lane == 0) warp_tot[warp] = __popc(bal);
        __syncthreads();
        if (warp == 0) {
            int v = lane < kWarps ? warp_tot[lane] : 0;
            for (int o = 1; o < 32; o <<= 1) {
                const int t2 = __shfl_up_sync(0xffffffffu, v, o);
                if (lane >= o) v += t2;
            }
            if (lane < kWarps) warp_tot[lane] = v;
        }
        __syncthreads();
        if (keep) sub[dst + (warp ? warp_tot[warp - 1] : 0) + __popc(bal & ((1u << lane) - 1u))] = d;
        if (tid == 0) s_np = dst + warp_tot[kWarps - 1];
        __syncthreads();
    };
    for (int seg = 0; seg < 2; ++seg) {
    // key of candidate i: (conf desc, class group, anchor); the anchor (< 2^14) orders
    // like the candidate index and locates the record
    if (seg == 1) compact(false);           // segment 0's sort overwrote the anchor list
    for (int i = tid; i < n; i += kThreads) {
        const int a = (int)keys[i];
        const int2 cc = *reinterpret_cast<const int2*>(reinterpret_cast<const char*>(cand + a) + 32);   // conf, cls
        keys[i] = ((unsigned long long)desc_key(__int_as_float(cc.x)) << 26) |
                  ((unsigned long long)grp[cc.y] << 16) | (unsigned long long)a;
    }
    __syncthreads();
    if (select && seg == 0) {
        if (tid == 0) { s_prefix = 0; s_rem = R; }
        __syncthreads();
        // keys < 2^58: eight 8-bit digits from bit 56 down. Lanes with the same bin add
        // once per warp (many confidences tie, and a bin hit by a whole warp would
        // otherwise take 32 serialised atomics).
        for (int shift = 56; shift >= 0; shift -= 8) {
            for (int i = tid; i < 256; i += kThreads) hist[i] = 0;
            __syncthreads();
            const unsigned long long pre_k = s_prefix;
            for (int i0 = 0; i0 < n; i0 += kThreads) {
                const int i = i0 + tid;
                const unsigned long long key = i < n ? keys[i] : 0ull;
                const bool in = i < n && (shift == 56 || (key >> (shift + 8)) == pre_k);
                const int bin = in ? (int)((key >> shift) & 255) : -1;
                const unsigned peers = __match_any_sync(0xffffffffu, bin);
                if (in && __ffs(peers) - 1 == lane) atomicAdd(&hist[bin], __popc(peers));
            }
            __syncthreads();
            if (warp == 0) {
                // the bin holding the s_rem-th key; lane l owns bins 8l .. 8l+7
                int v[8], tot = 0;
#pragma unroll
                for (int q = 0; q < 8; ++q) { v[q] = hist[lane * 8 + q]; tot += v[q]; }
                int incl = tot;
                for (int o = 1; o < 32; o <<= 1) {
                    const int t2 = __shfl_up_sync(0xffffffffu, incl, o);
                    if (lane >= o) incl += t2;
                }
                const int rem = s_rem;
                int excl = incl - tot;
                if (excl < rem && rem <= incl) {
                    int q = 0;
                    while (excl + v[q] < rem) { excl += v[q]; ++q; }
                    s_prefix = (pre_k << 8) | (unsigned long long)(lane * 8 + q);
                    s_rem = rem - excl;
                }
            }
            __syncthreads();
        }
        T = s_prefix;
    }
    int ns = n;
    if (select) {
        // keep segment seg's keys: gathered into registers, then written to keys[0 .. ns)
        unsigned long long mine[kMaxKeys / kThreads];
        int cnt_mine = 0;
        for (int i = tid; i < n; i += kThreads) {
            const bool in0 = keys[i] <= T;
            if (in0 == (seg == 0)) mine[cnt_mine++] = keys[i];
        }
        if (tid == 0) s_sel = 0;
        __syncthreads();
        const int pos = cnt_mine ? atomicAdd(&s_sel, cnt_mine) : 0;
        for (int q = 0; q < cnt_mine; ++q) keys[pos + q] = mine[q];
        __syncthreads();
        ns = s_sel;
    }
    int np = 1;
    while (np < ns) np <<= 1;
    for (int i = ns + tid; i < np; i += kThreads) keys[i] = ~0ull;
    __syncthreads();
    bitonic_sort<kThreads>(keys, np);

    if (tid == 0) s_np = 0;
    __syncthreads();
    int cursor = 0;
    while (s_kept < p.max_det && cursor < ns) {
        // (a) fill the pending list
        while (s_np < kSub && cursor < ns) {
            const int cnt = ns - cursor < kSub ? ns - cursor : kSub;
            for (int i = tid; i < cnt; i += kThreads) {
                Det d = cand[keys[cursor + i] & 0xFFFF];
                d.reserved = 0;                  // the candidate flag is not part of the output
                raw[i] = d;
            }
            __syncthreads();
            test_kept(raw, cnt, 0, s_kept);
            append_survivors(raw, cnt, s_np);
            cursor += cnt;
        }
        // (b) decide the pending boxes in order (threads below 2 kSub, one box each; a
        //     named barrier over them): per step the warps post their alive boxes, all
        //     find the first one, its thread keeps it and the later ones test against
        //     it. The boxes stay in shared memory (few registers live across the steps).
        if (tid < 2 * kSub) {
            const int np = s_np;
            bool alive = tid < np;
            const int my_cls = alive ? sub[tid].cls : -1;
            int k = s_kept;
            for (int step = 0; k < p.max_det; ++step) {
                uint32_t* words = s_words + (step & 1) * (kSub / 16);
                const unsigned bal = __ballot_sync(0xffffffffu, alive);
                if (lane == 0) words[warp] = bal;
                asm volatile("bar.sync 1, %0;" ::"r"(2 * kSub) : "memory");
                const unsigned v = lane < kSub / 16 ? words[lane] : 0u;
                const unsigned nz = __ballot_sync(0xffffffffu, v != 0u);
                if (!nz) break;
                const int w0 = __ffs(nz) - 1;
                const int j0 = w0 * 32 + __ffs(__shfl_sync(0xffffffffu, v, w0)) - 1;
                if (tid == j0) {
                    alive = false;
                    const Det& me = sub[tid];
                    out[k] = me;
                    if (k < kKeptSmem) {
                        kept_b[k] = Box{me.x1, me.y1, me.x2, me.y2, box_area(me)};
                        kept_c[k] = my_cls;
                        const int slot = cls_cnt[my_cls]++;
                        if (slot < cap) cls_tab[my_cls * cap + slot] = k;
                    }
                } else if (alive && sub[j0].cls == my_cls) {
                    const Det& o = sub[j0];
                    const Det& me = sub[tid];
                    if (iou_exceeds(o, box_area(o), me, box_area(me), p.iou, two_ulp)) alive = false;
                }
                ++k;
            }
            if (tid == 0) s_kept = k;
        }
        __syncthreads();
        if (tid == 0) s_np = 0;
        __syncthreads();
    }
    if (!select || s_kept >= p.max_det) break;
    __syncthreads();
    }
    if (tid == 0) p.counts[b] = s_kept;
}

}  // namespace

size_t decode_work_bytes(int64_t batch, int64_t anchors) {
    // SIZE_MAX when batch * anchors * sizeof(Det) does not fit in size_t, so a size
    // check against it can never pass by wrapping around
    if (batch <= 0 || anchors <= 0) return 0;
    if ((uint64_t)batch > SIZE_MAX / sizeof(Det) / (uint64_t)anchors) return SIZE_MAX;
    return (size_t)batch * (size_t)anchors * sizeof(Det);
}

namespace {

std::once_flag g_nms_once[64];
int g_nms_small_budget[64];

// Once per device (the opt-in shared-memory sizes are per-device function attributes;
// runner threads of several devices may get here at the same time): the big shape's
// opt-in size, and the dynamic shared memory the small shape may take with two CTAs
// on an SM (half the SM's shared memory less the per-CTA reservation and the
// kernel's static part), returned.
int nms_setup(int dev) {
    if (dev < 0 || dev >= 64) fail(ENGINE_ERR_INVALID_ARG, "decode: device index out of range");
    std::call_once(g_nms_once[dev], [dev] {
        PB_CUDA(cudaFuncSetAttribute(decode_nms_kernel<NmsBig>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)nms_smem<NmsBig>(kMaxKeys, kMaxClasses)));
        int per_sm = 0, reserved = 0;
        PB_CUDA(cudaDeviceGetAttribute(&per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev));
        PB_CUDA(cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev));
        cudaFuncAttributes fa{};
        PB_CUDA(cudaFuncGetAttributes(&fa, decode_nms_kernel<NmsSmall>));
        int budget = (per_sm / 2 - reserved - (int)fa.sharedSizeBytes) & ~15;
        if (budget > 0) {
            PB_CUDA(cudaFuncSetAttribute(decode_nms_kernel<NmsSmall>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         budget));
            PB_CUDA(cudaFuncSetAttribute(decode_nms_kernel<NmsSmall>,
                                         cudaFuncAttributePreferredSharedMemoryCarveout, 100));
        }
        g_nms_small_budget[dev] = budget > 0 ? budget : 0;
    });
    return g_nms_small_budget[dev];
}

}  // namespace

void launch_decode_nms(const DecodeArgs& a, cudaStream_t s) {
    if (a.anchors > kMaxKeys) fail(ENGINE_ERR_NOT_IMPL, "decode: more than 16384 anchors per image");
    if (a.channels - 4 > kMaxClasses || a.channels < 5) fail(ENGINE_ERR_INVALID_SHAPE, "decode: bad channel count");
    if (a.max_det < 0) fail(ENGINE_ERR_INVALID_ARG, "decode: max_det must be >= 0");
    if (a.batch < 0 || a.batch > INT_MAX) fail(ENGINE_ERR_INVALID_ARG, "decode: batch must be in [0, 2^31)");
    if (a.batch == 0) return;
    if ((uintptr_t)a.work % 16 || (a.max_det > 0 && (uintptr_t)a.dets % 8))
        fail(ENGINE_ERR_INVALID_ARG, "decode: work must be 16-byte and dets 8-byte aligned");
    int dev = 0;
    PB_CUDA(cudaGetDevice(&dev));
    const int small_budget = nms_setup(dev);
    const int ncp = ((int)a.channels - 4 + 1) & ~1;
    // The small shape's key array must hold every candidate (<= anchors), the padded
    // sort of segment 0 (< 2 R) and of segment 1 (the power of two >= anchors - R), and
    // R <= key_cap / 2 so that more than R candidates always take the select.
    const int64_t R = nms_prefix_rank(a.max_det);
    int64_t cap = a.anchors > 2 * R ? a.anchors : 2 * R;
    if (a.anchors > R) {
        int64_t q = 1;
        while (q < a.anchors - R) q <<= 1;
        if (q > cap) cap = q;
    }
    cap = (cap + 1) & ~int64_t(1);
    int64_t cblocks = (a.batch * a.anchors + 255) / 256;
    if (cblocks > 148 * 16) cblocks = 148 * 16;
    if (cblocks > 0) decode_candidates_kernel<<<(unsigned)cblocks, 256, 0, s>>>(a);
    if (cap <= kMaxKeys && nms_smem<NmsSmall>(cap, ncp) <= (size_t)small_budget) {
        decode_nms_kernel<NmsSmall><<<(unsigned)a.batch, NmsSmall::NT, nms_smem<NmsSmall>(cap, ncp), s>>>(
            a, (int)cap, ncp);
    } else {
        decode_nms_kernel<NmsBig><<<(unsigned)a.batch, NmsBig::NT, nms_smem<NmsBig>(kMaxKeys, ncp), s>>>(
            a, kMaxKeys, ncp);
    }
    PB_CUDA(cudaGetLastError());
}

}  // namespace pb

// ---------------------------------------------------------------------------
// Allocation-free decode (pdefa_decode_yolo_noalloc).
//
// Some callers cannot allocate device memory at the moment they decode: code that
// runs under a framework's caching allocator it must not bypass, inference servers
// that forbid cudaMalloc after start-up (allocation there can stall every stream on
// the device), and plugin hosts that hand out only their own input/output buffers.
// For them the candidate scratch of the decode kernel lives in a fixed file-scope
// device array, kNoAllocScratchBytes per GPU, held by every GPU that loads this
// library until the process exits.
// ---------------------------------------------------------------------------
namespace pb {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;   // 8 MiB = 174762 candidate records
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[64] = {};

// Device address of g_noalloc_scratch on the current device. In host code the
// array's name is only a host-side stand-in, so the address is looked up once per
// device (with that device current) and cached.
void* noalloc_scratch_address(int device) {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (device < 0 || device >= 64) fail(ENGINE_ERR_INVALID_ARG, "device index out of range");
    if (!g_noalloc_ptr[device]) {
        void* ptr = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
        if (e != cudaSuccess || !ptr) {
            cudaGetLastError();
            fail(ENGINE_ERR_RUNTIME, std::string("cudaGetSymbolAddress(decode scratch) failed: ") + cudaGetErrorString(e));
        }
        g_noalloc_ptr[device] = ptr;
    }
    return g_noalloc_ptr[device];
}

}  // namespace
}  // namespace pb

extern "C" ENGINE_API EngineStatus pdefa_decode_yolo_noalloc(const float* d_preds, int64_t batch, int64_t channels,
                                                            int64_t anchors, const PdefaPreprocessMeta* d_metas,
                                                            double conf_thres, double iou_thres, int32_t max_det,
                                                            int32_t* d_counts, PdefaDetection* d_dets,
                                                            void* stream) {
    using namespace pb;
    if (!d_preds || !d_counts || (!d_dets && max_det > 0)) return ENGINE_ERR_NULL_PTR;
    return guarded([&]() -> EngineStatus {
        clear_error();
        if (batch < 0 || channels < 5 || anchors < 0) { set_error("decode_noalloc: bad shape"); return ENGINE_ERR_INVALID_SHAPE; }
        if (max_det < 0) { set_error("decode_noalloc: max_det must be >= 0"); return ENGINE_ERR_INVALID_ARG; }
        // batch * anchors candidate records must fit the built-in scratch; checked by
        // division so that huge arguments cannot wrap the product around
        constexpr uint64_t kSlots = kNoAllocScratchBytes / sizeof(Det);
        if (anchors > 0 && (uint64_t)batch > kSlots / (uint64_t)anchors) {
            set_error("decode_noalloc: batch * anchors = " + std::to_string(batch) + " * " + std::to_string(anchors) +
                      " candidate slots exceed the built-in scratch of " + std::to_string(kSlots) +
                      " (8 MiB); decode fewer images per call or use pdefa_decode_yolo_device");
            return ENGINE_ERR_INVALID_ARG;
        }
        int dev = 0;
        PB_CUDA(cudaGetDevice(&dev));
        // The scratch address is the current device's; a stream of another device
        // would run the kernels there against this device's array.
        if (stream) {
            int sdev = -1;
            PB_CUDA(cudaStreamGetDevice(static_cast<cudaStream_t>(stream), &sdev));
            if (sdev != dev) {
                set_error("decode_noalloc: stream belongs to device " + std::to_string(sdev) +
                          " but the current device is " + std::to_string(dev));
                return ENGINE_ERR_INVALID_ARG;
            }
        }
        DecodeArgs a;
        a.preds = d_preds;
        a.batch = batch; a.channels = channels; a.anchors = anchors;
        a.meta = reinterpret_cast<const int32_t*>(d_metas);
        a.conf = conf_thres; a.iou = iou_thres; a.max_det = max_det;
        a.counts = d_counts; a.dets = d_dets;
        // Every candidate record is written before it is read, so the shared scratch
        // needs no clearing between calls.
        a.work = noalloc_scratch_address(dev);
        a.err = nullptr;
        launch_decode_nms(a, static_cast<cudaStream_t>(stream));
        return ENGINE_OK;
    });
}
