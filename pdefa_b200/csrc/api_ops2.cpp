// engine_ops_* part 2 and engine_random_* (engine_c_api.h:166-229), semantics of
// PDEFA1.0/src/api/engine_api.cpp:1085-1673: reductions with keepdims (rank-0
// results become [1]), argmax to I32 (first maximum), gather with wrapped/clamped
// indices, reshape with one -1, transpose by perm, concat along an axis, stack on a
// new axis. Data movement and reductions run as device kernels; random tensors are
// generated on the host with std::mt19937_64 and std::normal/uniform_real
// distributions, the reference's generator (engine_api.cpp:1085-1122).
#include <random>

#include "kernels.h"
#include "runtime.h"

using namespace pb;

namespace {

bool tok(const EngineTensor* t) { return t && t->magic == kMagicTensor; }

struct Dev {
    int device;
    cudaStream_t stream = nullptr;
    std::vector<void*> bufs;
    Dev() : device(default_device()) {
        require_device(device);
        PB_CUDA(cudaSetDevice(device));
        PB_CUDA(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
    }
    ~Dev() {
        cudaSetDevice(device);
        cudaStreamSynchronize(stream);
        for (void* p : bufs) cudaFree(p);
        cudaStreamDestroy(stream);
    }
    void* alloc(size_t n) {
        void* p = nullptr;
        if (cudaMalloc(&p, std::max<size_t>(n, 16)) != cudaSuccess) {
            cudaGetLastError();
            fail(ENGINE_ERR_OUT_OF_MEMORY, "device allocation failed");
        }
        bufs.push_back(p);
        return p;
    }
    void* up(TensorStore& t) {
        t.sync_to_host();
        void* d = alloc(t.nbytes);
        PB_CUDA(cudaMemcpyAsync(d, t.host, t.nbytes, cudaMemcpyHostToDevice, stream));
        return d;
    }
    void* up_bytes(const void* h, size_t n) {
        void* d = alloc(n);
        PB_CUDA(cudaMemcpyAsync(d, h, n, cudaMemcpyHostToDevice, stream));
        return d;
    }
    void down(TensorStore& t, const void* d) {
        PB_CUDA(cudaMemcpyAsync(t.host, d, t.nbytes, cudaMemcpyDeviceToHost, stream));
        PB_CUDA(cudaStreamSynchronize(stream));
    }
};

EngineTensor* make(std::vector<int64_t> shape, EngineDType dt) {
    auto* t = new EngineTensor();
    t->owned = std::make_shared<TensorStore>(std::move(shape), dt);
    return t;
}

TView dense(const void* p, const std::vector<int64_t>& s) {
    TView v;
    v.ptr = p;
    v.rank = std::max<int>(1, (int)s.size());
    int64_t st = 1;
    if (s.empty()) { v.shape[0] = 1; v.stride[0] = 1; }
    for (int d = (int)s.size() - 1; d >= 0; --d) { v.shape[d] = s[d]; v.stride[d] = st; st *= s[d]; }
    v.img_stride = st;
    return v;
}

EngineStatus reduce_impl(const EngineTensor* a, int32_t axis, int32_t keepdims, EngineTensor** out, int mode) {
    if (!tok(a)) return ENGINE_ERR_INVALID_HANDLE;
    if (!out) return ENGINE_ERR_NULL_PTR;
    *out = nullptr;
    return guarded([&]() -> EngineStatus {
        clear_error();
        TensorStore& in = *a->ptr();
        const char* what = mode == 3 ? "argmax" : "reduce";
        if (in.dtype != ENGINE_F32) { set_error(std::string(what) + ": only F32 supported"); return ENGINE_ERR_INVALID_ARG; }
        const int32_t rank = (int32_t)in.shape.size();
        int32_t ax = axis < 0 ? axis + rank : axis;
        if (ax < 0 || ax >= rank) { set_error(std::string(what) + ": axis out of range"); return ENGINE_ERR_INVALID_ARG; }
        int64_t outer = 1, inner = 1;
        for (int32_t d = 0; d < ax; ++d) outer *= in.shape[d];
        for (int32_t d = ax + 1; d < rank; ++d) inner *= in.shape[d];
        std::vector<int64_t> od;
        for (int32_t d = 0; d < rank; ++d) {
            if (d == ax) { if (keepdims) od.push_back(1); }
            else od.push_back(in.shape[d]);
        }
        if (od.empty()) od.push_back(1);
        std::unique_ptr<EngineTensor> r(make(od, mode == 3 ? ENGINE_I32 : ENGINE_F32));
        if (r->ptr()->nbytes) {
            Dev dv;
            const float* di = static_cast<const float*>(dv.up(in));
            void* dout = dv.alloc(r->ptr()->nbytes);
            launch_reduce(mode, di, dout, outer, in.shape[ax], inner, dv.stream);
            dv.down(*r->ptr(), dout);
        }
        *out = r.release();
        return ENGINE_OK;
    });
}

EngineStatus copy_into_new(TensorStore& in, const TView& src_view_host_shape, std::vector<int64_t> oshape, EngineTensor** out) {
    std::unique_ptr<EngineTensor> r(make(std::move(oshape), ENGINE_F32));
    if (r->ptr()->nbytes) {
        Dev dv;
        const void* di = dv.up(in);
        void* dout = dv.alloc(r->ptr()->nbytes);
        TView src = src_view_host_shape;
        src.ptr = di;
        TView dst = dense(dout, r->ptr()->shape);
        // the destination walks the same logical index space as src
        dst.rank = src.rank;
        int64_t st = 1;
        for (int d = src.rank - 1; d >= 0; --d) { dst.shape[d] = src.shape[d]; dst.stride[d] = st; st *= src.shape[d]; }
        launch_strided_copy(src, dst, 1, dv.stream);
        dv.down(*r->ptr(), dout);
    }
    *out = r.release();
    return ENGINE_OK;
}

}  // namespace

extern "C" {

ENGINE_API EngineStatus engine_ops_reduce_max(const EngineTensor* a, int32_t axis, int32_t keepdims, EngineTensor** out) { return reduce_impl(a, axis, keepdims, out, 0); }
ENGINE_API EngineStatus engine_ops_reduce_sum(const EngineTensor* a, int32_t axis, int32_t keepdims, EngineTensor** out) { return reduce_impl(a, axis, keepdims, out, 1); }
ENGINE_API EngineStatus engine_ops_reduce_mean(const EngineTensor* a, int32_t axis, int32_t keepdims, EngineTensor** out) { return reduce_impl(a, axis, keepdims, out, 2); }
ENGINE_API EngineStatus engine_ops_argmax(const EngineTensor* a, int32_t axis, int32_t keepdims, EngineTensor** out) { return reduce_impl(a, axis, keepdims, out, 3); }

ENGINE_API EngineStatus engine_ops_gather(const EngineTensor* a, const EngineTensor* indices, int32_t axis, EngineTensor** out) {
    if (!tok(a) || !tok(indices)) return ENGINE_ERR_INVALID_HANDLE;
    if (!out) return ENGINE_ERR_NULL_PTR;
    *out = nullptr;
    return guarded([&]() -> EngineStatus {
        clear_error();
        TensorStore& d = *a->ptr();
        TensorStore& ix = *indices->ptr();
        if (d.dtype != ENGINE_F32) { set_error("gather: only F32 data supported"); return ENGINE_ERR_INVALID_ARG; }
        const int32_t rank = (int32_t)d.shape.size();
        int32_t ax = axis < 0 ? axis + rank : axis;
        if (ax < 0 || ax >= rank) { set_error("gather: axis out of range"); return ENGINE_ERR_INVALID_ARG; }
        ix.sync_to_host();
        const int64_t n = ix.numel();
        std::vector<int64_t> idx(n);
        for (int64_t i = 0; i < n; ++i) {
            switch (ix.dtype) {
                case ENGINE_I64: idx[i] = static_cast<const int64_t*>(ix.host)[i]; break;
                case ENGINE_I32: idx[i] = static_cast<const int32_t*>(ix.host)[i]; break;
                default: idx[i] = (int64_t) static_cast<const float*>(ix.host)[i]; break;
            }
        }
        std::vector<int64_t> od;
        for (int32_t q = 0; q < ax; ++q) od.push_back(d.shape[q]);
        od.push_back(n);
        for (int32_t q = ax + 1; q < rank; ++q) od.push_back(d.shape[q]);
        int64_t outer = 1, inner = 1;
        for (int32_t q = 0; q < ax; ++q) outer *= d.shape[q];
        for (int32_t q = ax + 1; q < rank; ++q) inner *= d.shape[q];
        std::unique_ptr<EngineTensor> r(make(od, ENGINE_F32));
        if (r->ptr()->nbytes) {
            Dev dv;
            const float* dd = static_cast<const float*>(dv.up(d));
            const int64_t* di = static_cast<const int64_t*>(dv.up_bytes(idx.data(), idx.size() * 8));
            float* dout = static_cast<float*>(dv.alloc(r->ptr()->nbytes));
            launch_gather(dd, di, dout, outer, d.shape[ax], n, inner, dv.stream);
            dv.down(*r->ptr(), dout);
        }
        *out = r.release();
        return ENGINE_OK;
    });
}

ENGINE_API EngineStatus engine_ops_reshape(const EngineTensor* a, const int64_t* shape, int32_t rank, EngineTensor** out) {
    if (!tok(a)) return ENGINE_ERR_INVALID_HANDLE;
    if (!shape || !out) return ENGINE_ERR_NULL_PTR;
    if (rank < 0 || rank > 8) return ENGINE_ERR_INVALID_SHAPE;
    *out = nullptr;
    return guarded([&]() -> EngineStatus {
        clear_error();
        TensorStore& in = *a->ptr();
        if (in.dtype != ENGINE_F32) { set_error("reshape: only F32 supported"); return ENGINE_ERR_INVALID_ARG; }
        std::vector<int64_t> d(shape, shape + rank);
        int64_t known = 1; int neg = -1;
        for (int32_t i = 0; i < rank; ++i) { if (d[i] == -1) neg = i; else if (d[i] > 0) known *= d[i]; }
        if (neg >= 0) d[neg] = known > 0 ? in.numel() / known : 0;
        int64_t tot = 1;
        for (auto v : d) tot *= v;
        if (tot != in.numel()) { set_error("reshape: numel mismatch"); return ENGINE_ERR_INVALID_SHAPE; }
        TView src = dense(nullptr, {in.numel()});
        return copy_into_new(in, src, d, out);
    });
}

ENGINE_API EngineStatus engine_ops_transpose(const EngineTensor* a, const int32_t* perm, int32_t rank, EngineTensor** out) {
    if (!tok(a)) return ENGINE_ERR_INVALID_HANDLE;
    if (!perm || !out) return ENGINE_ERR_NULL_PTR;
    *out = nullptr;
    return guarded([&]() -> EngineStatus {
        clear_error();
        TensorStore& in = *a->ptr();
        if (in.dtype != ENGINE_F32) { set_error("transpose: only F32 supported"); return ENGINE_ERR_INVALID_ARG; }
        if (rank != (int32_t)in.shape.size()) { set_error("transpose: perm rank mismatch"); return ENGINE_ERR_INVALID_SHAPE; }
        std::vector<int64_t> od(rank);
        TView base = dense(nullptr, in.shape), src = base;
        for (int32_t i = 0; i < rank; ++i) {
            int32_t p = perm[i] < 0 ? perm[i] + rank : perm[i];
            if (p < 0 || p >= rank) { set_error("transpose: invalid perm"); return ENGINE_ERR_INVALID_ARG; }
            od[i] = in.shape[p];
            src.shape[i] = base.shape[p];
            src.stride[i] = base.stride[p];
        }
        return copy_into_new(in, src, od, out);
    });
}

ENGINE_API EngineStatus engine_ops_concat(const EngineTensor* const* inputs, int32_t n, int32_t axis, EngineTensor** out) {
    if (!inputs || n < 1 || !out) return ENGINE_ERR_NULL_PTR;
    *out = nullptr;
    return guarded([&]() -> EngineStatus {
        clear_error();
        for (int32_t i = 0; i < n; ++i) if (!tok(inputs[i])) return ENGINE_ERR_INVALID_HANDLE;
        const TensorStore& t0 = *inputs[0]->ptr();
        const int32_t rank = (int32_t)t0.shape.size();
        int32_t ax = axis < 0 ? axis + rank : axis;
        if (ax < 0 || ax >= rank) { set_error("concat: axis out of range"); return ENGINE_ERR_INVALID_ARG; }
        std::vector<int64_t> od = t0.shape;
        od[ax] = 0;
        for (int32_t i = 0; i < n; ++i) {
            const TensorStore& ti = *inputs[i]->ptr();
            if ((int32_t)ti.shape.size() != rank) { set_error("concat: rank mismatch"); return ENGINE_ERR_INVALID_SHAPE; }
            for (int32_t d = 0; d < rank; ++d)
                if (d != ax && ti.shape[d] != t0.shape[d]) { set_error("concat: non-axis dim mismatch"); return ENGINE_ERR_INVALID_SHAPE; }
            od[ax] += ti.shape[ax];
        }
        std::unique_ptr<EngineTensor> r(make(od, ENGINE_F32));
        if (r->ptr()->nbytes) {
            Dev dv;
            float* dout = static_cast<float*>(dv.alloc(r->ptr()->nbytes));
            const TView ov = dense(dout, od);
            int64_t off = 0;
            for (int32_t i = 0; i < n; ++i) {
                TensorStore& ti = *inputs[i]->ptr();
                if (ti.numel() == 0) continue;
                TView src = dense(dv.up(ti), ti.shape);
                TView dst = ov;
                for (int32_t d = 0; d < rank; ++d) dst.shape[d] = ti.shape[d];
                dst.ptr = dout + off * ov.stride[ax];
                launch_strided_copy(src, dst, 1, dv.stream);
                off += ti.shape[ax];
            }
            dv.down(*r->ptr(), dout);
        }
        *out = r.release();
        return ENGINE_OK;
    });
}

ENGINE_API EngineStatus engine_ops_stack(const EngineTensor* const* inputs, int32_t n, int32_t axis, EngineTensor** out) {
    if (!inputs || n < 1 || !out) return ENGINE_ERR_NULL_PTR;
    *out = nullptr;
    return guarded([&]() -> EngineStatus {
        clear_error();
        for (int32_t i = 0; i < n; ++i) if (!tok(inputs[i])) return ENGINE_ERR_INVALID_HANDLE;
        const TensorStore& t0 = *inputs[0]->ptr();
        const int32_t rank = (int32_t)t0.shape.size(), nr = rank + 1;
        int32_t ax = axis < 0 ? axis + nr : axis;
        if (ax < 0 || ax >= nr) { set_error("stack: axis out of range"); return ENGINE_ERR_INVALID_ARG; }
        for (int32_t i = 1; i < n; ++i) {
            const TensorStore& ti = *inputs[i]->ptr();
            if ((int32_t)ti.shape.size() != rank) { set_error("stack: rank mismatch"); return ENGINE_ERR_INVALID_SHAPE; }
            if (ti.shape != t0.shape) { set_error("stack: shape mismatch"); return ENGINE_ERR_INVALID_SHAPE; }
        }
        std::vector<int64_t> od;
        int32_t j = 0;
        for (int32_t d = 0; d < nr; ++d) od.push_back(d == ax ? n : t0.shape[j++]);
        std::unique_ptr<EngineTensor> r(make(od, ENGINE_F32));
        if (r->ptr()->nbytes) {
            Dev dv;
            float* dout = static_cast<float*>(dv.alloc(r->ptr()->nbytes));
            const TView ov = dense(dout, od);
            for (int32_t i = 0; i < n; ++i) {
                TensorStore& ti = *inputs[i]->ptr();
                TView src = dense(dv.up(ti), ti.shape);
                // destination: the new axis fixed at i, other axes as in the input
                TView dst;
                dst.ptr = dout + i * ov.stride[ax];
                dst.rank = std::max(1, rank);
                int q = 0;
                for (int32_t d = 0; d < nr; ++d) {
                    if (d == ax) continue;
                    dst.shape[q] = od[d];
                    dst.stride[q] = ov.stride[d];
                    ++q;
                }
                if (rank == 0) { dst.shape[0] = 1; dst.stride[0] = 1; }
                launch_strided_copy(src, dst, 1, dv.stream);
            }
            dv.down(*r->ptr(), dout);
        }
        *out = r.release();
        return ENGINE_OK;
    });
}

static EngineStatus random_impl(const int64_t* shape, int32_t rank, uint64_t seed, EngineTensor** out, bool normal) {
    if (!shape || !out) return ENGINE_ERR_NULL_PTR;
    if (rank < 0 || rank > 8) return ENGINE_ERR_INVALID_SHAPE;
    *out = nullptr;
    return guarded([&]() -> EngineStatus {
        clear_error();
        std::unique_ptr<EngineTensor> r(make(std::vector<int64_t>(shape, shape + rank), ENGINE_F32));
        float* p = static_cast<float*>(r->ptr()->host);
        const int64_t n = r->ptr()->numel();
        std::mt19937_64 rng(seed);
        if (normal) {
            std::normal_distribution<float> dist(0.0f, 1.0f);
            for (int64_t i = 0; i < n; ++i) p[i] = dist(rng);
        } else {
            std::uniform_real_distribution<float> dist(0.0f, 1.0f);
            for (int64_t i = 0; i < n; ++i) p[i] = dist(rng);
        }
        *out = r.release();
        return ENGINE_OK;
    });
}
ENGINE_API EngineStatus engine_random_randn(const int64_t* shape, int32_t rank, uint64_t seed, EngineTensor** out) { return random_impl(shape, rank, seed, out, true); }
ENGINE_API EngineStatus engine_random_rand(const int64_t* shape, int32_t rank, uint64_t seed, EngineTensor** out) { return random_impl(shape, rank, seed, out, false); }

}  // extern "C"
