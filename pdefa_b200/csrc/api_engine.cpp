// engine_* C ABI (PDEFA1.0/include/engine/engine_c_api.h:64-234) on the GPU runtime.
//
// Behaviour kept from the reference implementation (PDEFA1.0/src/api/engine_api.cpp):
// magic-checked handles, thread-local last error, exceptions mapped to status codes,
// owned vs borrowed tensors (borrowed: destroy is a no-op, writes are rejected),
// ops_matmul writing into a pre-allocated output and returning OK without touching
// it when shapes do not line up (engine_api.cpp:898-914 -> ops/matmul.cpp:107-135).
// Differences: session outputs are per-session borrowed wrappers (not one per thread),
// and every compute call runs on a CUDA device; without one it fails with
// ENGINE_ERR_RUNTIME instead of computing on the CPU.
#include <algorithm>
#if defined(__x86_64__) || defined(__i386__)
#include <cpuid.h>
#endif
#include <cmath>
#include <cstdlib>
#include <map>
#include <random>
#include <thread>

#include "../../include/pdefa_b200_ext.h"
#include "kernels.h"
#include "runtime.h"

namespace pb {

namespace {
thread_local std::string g_last_error;
}
void set_error(const std::string& m) { try { g_last_error = m; } catch (...) {} }
void clear_error() { try { g_last_error.clear(); } catch (...) {} }
const char* last_error_cstr() { return g_last_error.c_str(); }

int default_device() {
    const char* e = std::getenv("PDEFA_DEVICE");
    return (e && *e) ? std::atoi(e) : 0;
}

TensorStore::TensorStore(std::vector<int64_t> s, EngineDType dt) : shape(std::move(s)), dtype(dt) {
    int64_t n = 1;
    for (auto d : shape) {
        if (d < 0) fail(ENGINE_ERR_INVALID_SHAPE, "negative dimension");
        n *= d;
    }
    nbytes = (size_t)n * engine_dtype_bytes(dt);
    const size_t alloc = std::max<size_t>(nbytes, 64);
    if (device_count() > 0 && cudaHostAlloc(&host, alloc, cudaHostAllocPortable) == cudaSuccess) {
        pinned = true;
    } else {
        cudaGetLastError();
        host = nullptr;
        if (posix_memalign(&host, 64, alloc) != 0) host = nullptr;
    }
    if (!host) throw std::bad_alloc();
    std::memset(host, 0, alloc);
}

TensorStore::~TensorStore() {
    if (pinned) cudaFreeHost(host);
    else std::free(host);
}

int64_t TensorStore::numel() const {
    int64_t n = 1;
    for (auto d : shape) n *= d;
    return n;
}

void TensorStore::sync_to_host() {
    std::lock_guard<std::mutex> lk(mu);
    if (host_valid || !dev) return;
    int prev = 0;
    PB_CUDA(cudaGetDevice(&prev));
    PB_CUDA(cudaSetDevice(dev_id));
    PB_CUDA(cudaStreamSynchronize(dev_stream));
    PB_CUDA(cudaMemcpy(host, dev, nbytes, cudaMemcpyDeviceToHost));
    PB_CUDA(cudaSetDevice(prev));
    host_valid = true;
}

}  // namespace pb

using namespace pb;

// ---------------------------------------------------------------------------
// Session internals
// ---------------------------------------------------------------------------
pb::Plan& EngineSession::plan_for(int64_t batch, const std::vector<int64_t>& in_shape) {
    const auto key = std::make_pair(batch, in_shape);
    auto it = plans.find(key);
    if (it != plans.end()) return *it->second;
    // keep at most two plans alive (device memory is sized per batch)
    if (plans.size() >= 2) plans.erase(plans.begin());
    auto p = std::make_unique<pb::Plan>(graph, batch, precision, device, keep, in_shape);
    pb::Plan& ref = *p;
    plans[key] = std::move(p);
    return ref;
}

void EngineSession::run() {
    const auto t0 = std::chrono::high_resolution_clock::now();
    if (inputs.empty() || !inputs[0]) fail(ENGINE_ERR_INVALID_ARG, "input 0 is not set");
    PB_CUDA(cudaSetDevice(device));
    const TensorStore& x = *inputs[0]->ptr();
    if (x.dtype != ENGINE_F32) fail(ENGINE_ERR_INVALID_ARG, "input must be F32");
    const auto& info = graph->input_infos.empty() ? std::vector<int64_t>{} : graph->input_infos[0].shape;
    if (x.shape.empty()) fail(ENGINE_ERR_INVALID_SHAPE, "input has rank 0");
    // Like the reference interpreter, which runs the graph on whatever input it is
    // given (session.cpp:181-215), an input whose image size differs from the
    // declared one gets a plan lowered for its own shape; the rank must match.
    std::vector<int64_t> own;
    if (!info.empty()) {
        if (x.shape.size() != info.size()) fail(ENGINE_ERR_INVALID_SHAPE, "input rank differs from the model input");
        for (size_t d = 1; d < info.size(); ++d)
            if (info[d] > 0 && x.shape[d] != info[d]) own.assign(x.shape.begin(), x.shape.end());
        if (!own.empty()) own[0] = 1;
    }
    const int64_t batch = x.shape[0];
    pb::Plan& p = plan_for(batch, own);
    for (size_t i = 0; i < inputs.size() && i < graph->inputs.size(); ++i) {
        if (!inputs[i]) fail(ENGINE_ERR_INVALID_ARG, "input " + std::to_string(i) + " is not set");
        TensorStore& t = *inputs[i]->ptr();
        if (t.nbytes != p.input_bytes((int)i)) fail(ENGINE_ERR_INVALID_SHAPE, "input byte size mismatch");
        t.sync_to_host();
        PB_CUDA(cudaMemcpyAsync(p.input_buffer((int)i), t.host, t.nbytes, cudaMemcpyHostToDevice, stream));
    }
    if (profile_fn) {
        cudaEvent_t a, b;
        PB_CUDA(cudaEventCreate(&a));
        PB_CUDA(cudaEventCreate(&b));
        int64_t k = 0;
        for (auto& st : p.steps()) {
            PB_CUDA(cudaEventRecord(a, stream));
            st.run(stream);
            PB_CUDA(cudaEventRecord(b, stream));
            PB_CUDA(cudaEventSynchronize(b));
            float ms = 0;
            PB_CUDA(cudaEventElapsedTime(&ms, a, b));
            const std::string label = "node_" + std::to_string(k++) + " '" + st.name + "'";
            profile_fn(label.c_str(), (double)ms, profile_user);
        }
        cudaEventDestroy(a);
        cudaEventDestroy(b);
        p.enqueue_error_copy(stream);
    } else {
        p.run(stream);
    }
    PB_CUDA(cudaStreamSynchronize(stream));
    const int derr = p.take_error();
    if (derr) fail(ENGINE_ERR_RUNTIME, "device-side wait timed out (code " + std::to_string(derr) + ")");
    last = &p;
    outputs.resize(p.num_outputs());
    out_handles.resize(p.num_outputs());
    for (int k = 0; k < p.num_outputs(); ++k) {
        auto& o = outputs[k];
        if (!o || o->shape != p.output_shape(k)) o = std::make_shared<TensorStore>(p.output_shape(k), ENGINE_F32);
        std::lock_guard<std::mutex> lk(o->mu);
        o->dev = p.output_buffer(k);
        o->dev_id = device;
        o->dev_stream = stream;
        o->host_valid = false;
        out_handles[k].magic = kMagicTensor;
        out_handles[k].owned.reset();
        out_handles[k].borrowed = o.get();
    }
    const auto t1 = std::chrono::high_resolution_clock::now();
    last_run_ms = std::chrono::duration<double, std::milli>(t1 - t0).count();
    ++runs;
}

namespace {

bool tensor_ok(const EngineTensor* t) { return t && t->magic == kMagicTensor; }

EngineTensor* new_tensor(std::vector<int64_t> shape, EngineDType dt) {
    auto* t = new EngineTensor();
    t->owned = std::make_shared<TensorStore>(std::move(shape), dt);
    return t;
}

// Device scratch on the default device for the stateless ops.
// Per-thread, per-device resources of the direct ops (engine_ops_*): one non-blocking
// stream and a workspace that grows to the largest op seen and is reused, so a call
// makes no cudaMalloc/cudaFree and creates no stream once warm (the reference's ops run
// in the caller's thread too, ops/matmul.cpp:107-135). Freed when the thread exits.
struct OpCache {
    int device = -1;
    cudaStream_t stream = nullptr;
    std::vector<std::pair<void*, size_t>> chunks;   // device workspace pieces, kept across calls
    ~OpCache() {
        if (device < 0) return;
        if (cudaSetDevice(device) != cudaSuccess) return;
        if (stream) cudaStreamSynchronize(stream);
        for (auto& c : chunks) cudaFree(c.first);
        if (stream) cudaStreamDestroy(stream);
    }
};

OpCache& op_cache(int dev) {
    static thread_local std::map<int, OpCache> caches;
    OpCache& c = caches[dev];
    if (c.device < 0) {
        PB_CUDA(cudaSetDevice(dev));
        PB_CUDA(cudaStreamCreateWithFlags(&c.stream, cudaStreamNonBlocking));
        c.device = dev;
    }
    return c;
}

// One direct op: bump allocations from the thread's workspace on its stream; the
// destructor waits for the stream, so workspace and host copies are settled when the
// op returns.
struct OpDevice {
    int device = -1;
    cudaStream_t stream = nullptr;
    OpCache* cache = nullptr;
    size_t chunk = 0, used = 0;
    explicit OpDevice(int dev) : device(dev) {
        require_device(dev);
        PB_CUDA(cudaSetDevice(dev));
        cache = &op_cache(dev);
        stream = cache->stream;
    }
    ~OpDevice() {
        cudaSetDevice(device);
        if (stream) cudaStreamSynchronize(stream);
    }
    void* alloc(size_t n) {
        n = (std::max<size_t>(n, 16) + 255) & ~size_t(255);
        auto& cs = cache->chunks;
        while (chunk < cs.size() && used + n > cs[chunk].second) { ++chunk; used = 0; }
        if (chunk == cs.size()) {
            // a new piece; earlier pieces may still be in use by this op's queued work
            const size_t sz = std::max<size_t>(n, cs.empty() ? (size_t)4 << 20 : cs.back().second * 2);
            void* p = nullptr;
            if (cudaMalloc(&p, sz) != cudaSuccess) {
                cudaGetLastError();
                fail(ENGINE_ERR_OUT_OF_MEMORY, "device allocation failed");
            }
            cs.push_back({p, sz});
            used = 0;
        }
        void* p = static_cast<char*>(cs[chunk].first) + used;
        used += n;
        return p;
    }
    void* upload(TensorStore& t) {
        t.sync_to_host();
        void* d = alloc(t.nbytes);
        PB_CUDA(cudaMemcpyAsync(d, t.host, t.nbytes, cudaMemcpyHostToDevice, stream));
        return d;
    }
    void download(TensorStore& t, const void* d) {
        PB_CUDA(cudaMemcpyAsync(t.host, d, t.nbytes, cudaMemcpyDeviceToHost, stream));
        PB_CUDA(cudaStreamSynchronize(stream));
        t.host_valid = true;
        t.dev = nullptr;
    }
};

TView dense_view(const void* p, const std::vector<int64_t>& shape) {
    TView v;
    v.ptr = p;
    v.dt = F32;
    v.rank = (int)shape.size();
    int64_t st = 1;
    for (int d = v.rank - 1; d >= 0; --d) { v.shape[d] = shape[d]; v.stride[d] = st; st *= shape[d]; }
    if (v.rank == 0) { v.rank = 1; v.shape[0] = 1; v.stride[0] = 1; }
    v.img_stride = st;
    return v;
}

EngineStatus unary_op(EngineTensor* t, int kind, float p0 = 0, float p1 = 0) {
    if (!tensor_ok(t)) return ENGINE_ERR_INVALID_HANDLE;
    if (t->is_borrowed()) { set_error("cannot modify borrowed tensor"); return ENGINE_ERR_INVALID_ARG; }
    if (t->ptr()->dtype != ENGINE_F32) { set_error("only F32 supported"); return ENGINE_ERR_INVALID_ARG; }
    return guarded([&]() -> EngineStatus {
        clear_error();
        TensorStore& s = *t->ptr();
        if (s.numel() == 0) return ENGINE_OK;
        OpDevice od(default_device());
        void* d = od.upload(s);
        TView v = dense_view(d, s.shape);
        launch_unary(kind, v, v, 1, p0, p1, od.stream);
        od.download(s, d);
        return ENGINE_OK;
    });
}

EngineStatus binary_op(const EngineTensor* a, const EngineTensor* b, EngineTensor** out, int op) {
    if (!tensor_ok(a) || !tensor_ok(b)) return ENGINE_ERR_INVALID_HANDLE;
    if (!out) return ENGINE_ERR_NULL_PTR;
    *out = nullptr;
    return guarded([&]() -> EngineStatus {
        clear_error();
        TensorStore& A = *a->ptr();
        TensorStore& Bt = *b->ptr();
        const size_t r = std::max(A.shape.size(), Bt.shape.size());
        if (r > 8) { set_error("broadcast shape mismatch"); return ENGINE_ERR_INVALID_SHAPE; }
        std::vector<int64_t> o(r);
        for (size_t d = 0; d < r; ++d) {
            const int64_t da = d < r - A.shape.size() ? 1 : A.shape[d - (r - A.shape.size())];
            const int64_t db = d < r - Bt.shape.size() ? 1 : Bt.shape[d - (r - Bt.shape.size())];
            if (da != db && da != 1 && db != 1) { set_error("broadcast shape mismatch"); return ENGINE_ERR_INVALID_SHAPE; }
            o[d] = std::max(da, db);
        }
        std::unique_ptr<EngineTensor> res(new_tensor(o, ENGINE_F32));
        TensorStore& R = *res->ptr();
        if (R.numel() > 0) {
            OpDevice od(default_device());
            void* da = od.upload(A);
            void* db = od.upload(Bt);
            void* dr = od.alloc(R.nbytes);
            TView vo = dense_view(dr, o);
            auto aligned = [&](const void* p, const std::vector<int64_t>& s) {
                TView t = dense_view(p, s);
                TView u = vo;
                u.ptr = p;
                const int ra = (int)s.size();
                for (int d = 0; d < (int)r; ++d) {
                    const int sd = d - ((int)r - ra);
                    u.stride[d] = (sd < 0 || s[sd] == 1) ? 0 : t.stride[sd];
                }
                return u;
            };
            launch_binary(op, aligned(da, A.shape), aligned(db, Bt.shape), vo, 1, od.stream);
            od.download(R, dr);
        }
        *out = res.release();
        return ENGINE_OK;
    });
}

}  // namespace

extern "C" {

// ---------------------------------------------------------------------------
// META
// ---------------------------------------------------------------------------
ENGINE_API const char* engine_version(void) { return "1.0.3-b200"; }
ENGINE_API const char* engine_last_error(void) { return pb::last_error_cstr(); }
ENGINE_API const char* engine_status_string(EngineStatus s) {
    switch (s) {
        case ENGINE_OK: return "OK";
        case ENGINE_ERR_NULL_PTR: return "null pointer";
        case ENGINE_ERR_INVALID_HANDLE: return "invalid handle";
        case ENGINE_ERR_OUT_OF_MEMORY: return "out of memory";
        case ENGINE_ERR_FILE_NOT_FOUND: return "file not found";
        case ENGINE_ERR_INVALID_FORMAT: return "invalid format";
        case ENGINE_ERR_INVALID_SHAPE: return "invalid shape";
        case ENGINE_ERR_INVALID_ARG: return "invalid argument";
        case ENGINE_ERR_RUNTIME: return "runtime error";
        case ENGINE_ERR_NOT_IMPL: return "not implemented";
        default: return "unknown";
    }
}
ENGINE_API size_t engine_dtype_size(EngineDType dt) { return pb::engine_dtype_bytes(dt); }
// Host introspection keeps the reference's meaning (PDEFA1.0/src/api/engine_api.cpp:
// simd level, CPU brand and the AVX flags describe the host CPU), so callers that
// branch on them see the same answers; the compute device is reported by
// engine_device_count / engine_context_get_device (pdefa_b200_ext.h).
ENGINE_API const char* engine_simd_level(void) {
#if defined(__x86_64__) || defined(__i386__)
    __builtin_cpu_init();
    if (__builtin_cpu_supports("avx512f")) return "AVX-512";
    if (__builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma")) return "AVX2";
    if (__builtin_cpu_supports("sse2")) return "SSE";
#endif
    return "SCALAR";
}
ENGINE_API const char* engine_cpu_brand(void) {
    static std::string name;
    static std::once_flag once;
    std::call_once(once, [] {
#if defined(__x86_64__) || defined(__i386__)
        unsigned int r[12] = {};
        if (__get_cpuid_max(0x80000000u, nullptr) >= 0x80000004u) {
            for (unsigned int i = 0; i < 3; ++i)
                __get_cpuid(0x80000002u + i, &r[4 * i], &r[4 * i + 1], &r[4 * i + 2], &r[4 * i + 3]);
            name.assign(reinterpret_cast<const char*>(r), sizeof(r));
            name = name.c_str();                                   // up to the first NUL
            const size_t a = name.find_first_not_of(' '), b = name.find_last_not_of(' ');
            name = a == std::string::npos ? std::string() : name.substr(a, b - a + 1);
        }
#endif
        if (name.empty()) name = "unknown";
    });
    return name.c_str();
}

// ---------------------------------------------------------------------------
// CONTEXT
// ---------------------------------------------------------------------------
ENGINE_API EngineStatus engine_context_create(EngineContext** out_ctx) {
    if (!out_ctx) { set_error("out_ctx is null"); return ENGINE_ERR_NULL_PTR; }
    *out_ctx = nullptr;
    return guarded([&]() -> EngineStatus {
        clear_error();
        auto* c = new EngineContext();
        c->num_threads = (int32_t)std::max(1u, std::thread::hardware_concurrency());
        c->device = default_device();
        const char* p = std::getenv("PDEFA_PRECISION");
        if (p && *p) {
            const std::string s(p);
            c->precision = s == "bf16" ? PREC_BF16 : s == "tf32" ? PREC_TF32 : PREC_FP32;
        }
        *out_ctx = c;
        return ENGINE_OK;
    });
}
ENGINE_API void engine_context_destroy(EngineContext* ctx) {
    if (!ctx || ctx->magic != kMagicContext) return;
    ctx->magic = 0;
    delete ctx;
}
ENGINE_API EngineStatus engine_context_set_num_threads(EngineContext* ctx, int32_t n) {
    if (!ctx || ctx->magic != kMagicContext) return ENGINE_ERR_INVALID_HANDLE;
    if (n <= 0) return ENGINE_ERR_INVALID_ARG;
    ctx->num_threads = n;
    return ENGINE_OK;
}
ENGINE_API int32_t engine_context_get_num_threads(const EngineContext* ctx) {
    if (!ctx || ctx->magic != kMagicContext) return 0;
    return ctx->num_threads;
}
ENGINE_API int32_t engine_context_num_physical_cores(void) {
    return (int32_t)std::max(1u, std::thread::hardware_concurrency());
}
ENGINE_API int32_t engine_context_has_avx2(void) {
#if defined(__x86_64__) || defined(__i386__)
    __builtin_cpu_init();
    return __builtin_cpu_supports("avx2") ? 1 : 0;
#else
    return 0;
#endif
}
ENGINE_API int32_t engine_context_has_avx512(void) {
#if defined(__x86_64__) || defined(__i386__)
    __builtin_cpu_init();
    return __builtin_cpu_supports("avx512f") ? 1 : 0;
#else
    return 0;
#endif
}

// ---------------------------------------------------------------------------
// TENSOR
// ---------------------------------------------------------------------------
ENGINE_API EngineStatus engine_tensor_create(EngineTensor** out_t, const int64_t* shape, int32_t ndim,
                                             EngineDType dtype) {
    if (!out_t || !shape) { set_error("null argument"); return ENGINE_ERR_NULL_PTR; }
    *out_t = nullptr;
    return guarded([&]() -> EngineStatus {
        clear_error();
        if (ndim < 0 || ndim > 8) { set_error("rank must be 0..8"); return ENGINE_ERR_INVALID_SHAPE; }
        if (pb::engine_dtype_bytes(dtype) == 0) { set_error("unknown dtype"); return ENGINE_ERR_INVALID_ARG; }
        *out_t = new_tensor(std::vector<int64_t>(shape, shape + ndim), dtype);
        return ENGINE_OK;
    });
}
ENGINE_API EngineStatus engine_tensor_create_from_data(EngineTensor** out_t, const int64_t* shape, int32_t ndim,
                                                       EngineDType dtype, const void* data, size_t bytes) {
    if (!out_t || !shape || !data) { set_error("null argument"); return ENGINE_ERR_NULL_PTR; }
    *out_t = nullptr;
    return guarded([&]() -> EngineStatus {
        clear_error();
        if (ndim < 0 || ndim > 8) { set_error("rank must be 0..8"); return ENGINE_ERR_INVALID_SHAPE; }
        if (pb::engine_dtype_bytes(dtype) == 0) { set_error("unknown dtype"); return ENGINE_ERR_INVALID_ARG; }
        std::unique_ptr<EngineTensor> t(new_tensor(std::vector<int64_t>(shape, shape + ndim), dtype));
        if (bytes > t->ptr()->nbytes) { set_error("data too large"); return ENGINE_ERR_INVALID_ARG; }
        std::memcpy(t->ptr()->host, data, bytes);
        *out_t = t.release();
        return ENGINE_OK;
    });
}
ENGINE_API EngineStatus engine_tensor_data(EngineTensor* t, void** out_data, size_t* out_bytes) {
    if (!tensor_ok(t)) return ENGINE_ERR_INVALID_HANDLE;
    if (!out_data) return ENGINE_ERR_NULL_PTR;
    return guarded([&]() -> EngineStatus {
        TensorStore& s = *t->ptr();
        s.sync_to_host();
        *out_data = s.host;
        if (out_bytes) *out_bytes = s.nbytes;
        return ENGINE_OK;
    });
}
ENGINE_API EngineStatus engine_tensor_shape(const EngineTensor* t, int64_t* out_shape, int32_t* out_ndim) {
    if (!tensor_ok(t)) return ENGINE_ERR_INVALID_HANDLE;
    const TensorStore& s = *t->ptr();
    if (out_shape) for (size_t i = 0; i < s.shape.size(); ++i) out_shape[i] = s.shape[i];
    if (out_ndim) *out_ndim = (int32_t)s.shape.size();
    return ENGINE_OK;
}
ENGINE_API EngineStatus engine_tensor_copy_from(EngineTensor* t, const void* src, size_t bytes) {
    if (!tensor_ok(t)) return ENGINE_ERR_INVALID_HANDLE;
    if (!src) return ENGINE_ERR_NULL_PTR;
    if (t->is_borrowed()) { set_error("cannot write to borrowed tensor"); return ENGINE_ERR_INVALID_ARG; }
    TensorStore& s = *t->ptr();
    if (bytes > s.nbytes) return ENGINE_ERR_INVALID_ARG;
    return guarded([&]() -> EngineStatus {
        s.sync_to_host();
        std::memcpy(s.host, src, bytes);
        return ENGINE_OK;
    });
}
ENGINE_API EngineStatus engine_tensor_copy_to(const EngineTensor* t, void* dst, size_t bytes) {
    if (!tensor_ok(t)) return ENGINE_ERR_INVALID_HANDLE;
    if (!dst) return ENGINE_ERR_NULL_PTR;
    TensorStore& s = *t->ptr();
    if (bytes > s.nbytes) return ENGINE_ERR_INVALID_ARG;
    return guarded([&]() -> EngineStatus {
        s.sync_to_host();
        std::memcpy(dst, s.host, bytes);
        return ENGINE_OK;
    });
}
ENGINE_API int64_t engine_tensor_numel(const EngineTensor* t) { return tensor_ok(t) ? t->ptr()->numel() : 0; }
ENGINE_API EngineDType engine_tensor_dtype(const EngineTensor* t) { return tensor_ok(t) ? t->ptr()->dtype : ENGINE_F32; }
ENGINE_API int32_t engine_tensor_rank(const EngineTensor* t) { return tensor_ok(t) ? (int32_t)t->ptr()->shape.size() : 0; }
ENGINE_API void engine_tensor_destroy(EngineTensor* t) {
    if (!tensor_ok(t)) return;
    if (t->is_borrowed()) return;     // session-owned wrapper: no-op (engine_api.cpp:555-567)
    t->magic = 0;
    delete t;
}

// ---------------------------------------------------------------------------
// MODEL
// ---------------------------------------------------------------------------
ENGINE_API EngineStatus engine_model_load(EngineContext* ctx, const char* path, EngineModel** out_model) {
    (void)ctx;
    if (!out_model || !path) { set_error("null argument"); return ENGINE_ERR_NULL_PTR; }
    *out_model = nullptr;
    return guarded([&]() -> EngineStatus {
        clear_error();
        auto m = std::make_unique<EngineModel>();
        m->graph = load_engine_file(path);
        *out_model = m.release();
        return ENGINE_OK;
    });
}
ENGINE_API EngineStatus engine_model_input_count(const EngineModel* m, int32_t* out_n) {
    if (!m || m->magic != kMagicModel) return ENGINE_ERR_INVALID_HANDLE;
    if (out_n) *out_n = (int32_t)m->graph->inputs.size();
    return ENGINE_OK;
}
ENGINE_API EngineStatus engine_model_output_count(const EngineModel* m, int32_t* out_n) {
    if (!m || m->magic != kMagicModel) return ENGINE_ERR_INVALID_HANDLE;
    if (out_n) *out_n = (int32_t)m->graph->outputs.size();
    return ENGINE_OK;
}
ENGINE_API EngineStatus engine_model_name(const EngineModel* m, const char** out_name) {
    if (!m || m->magic != kMagicModel) return ENGINE_ERR_INVALID_HANDLE;
    if (!out_name) return ENGINE_ERR_NULL_PTR;
    *out_name = m->graph->name.c_str();
    return ENGINE_OK;
}
ENGINE_API void engine_model_destroy(EngineModel* m) {
    if (!m || m->magic != kMagicModel) return;
    m->magic = 0;
    delete m;
}

static EngineStatus model_info(const EngineModel* m, int32_t idx, bool input, const char** out_name,
                               int64_t* out_shape, int32_t* out_ndim, EngineDType* out_dtype) {
    if (!m || m->magic != kMagicModel) return ENGINE_ERR_INVALID_HANDLE;
    const auto& infos = input ? m->graph->input_infos : m->graph->output_infos;
    if (idx < 0 || idx >= (int32_t)infos.size()) { set_error("info index out of range"); return ENGINE_ERR_INVALID_ARG; }
    const TensorInfo& t = infos[idx];
    if (out_name) *out_name = t.name.c_str();
    if (out_shape) for (size_t i = 0; i < t.shape.size(); ++i) out_shape[i] = t.shape[i];
    if (out_ndim) *out_ndim = (int32_t)t.shape.size();
    if (out_dtype) {
        switch (t.dtype) {
            case DT_F16: *out_dtype = ENGINE_F16; break;
            case DT_BF16: *out_dtype = ENGINE_BF16; break;
            case DT_I8: *out_dtype = ENGINE_I8; break;
            case DT_U8: *out_dtype = ENGINE_U8; break;
            case DT_I32: *out_dtype = ENGINE_I32; break;
            case DT_I64: *out_dtype = ENGINE_I64; break;
            case DT_BOOL: *out_dtype = ENGINE_BOOL; break;
            default: *out_dtype = ENGINE_F32; break;
        }
    }
    return ENGINE_OK;
}
ENGINE_API EngineStatus engine_model_input_info(const EngineModel* m, int32_t idx, const char** out_name,
                                                int64_t* out_shape, int32_t* out_ndim, EngineDType* out_dtype) {
    return model_info(m, idx, true, out_name, out_shape, out_ndim, out_dtype);
}
ENGINE_API EngineStatus engine_model_output_info(const EngineModel* m, int32_t idx, const char** out_name,
                                                 int64_t* out_shape, int32_t* out_ndim, EngineDType* out_dtype) {
    return model_info(m, idx, false, out_name, out_shape, out_ndim, out_dtype);
}

// ---------------------------------------------------------------------------
// SESSION
// ---------------------------------------------------------------------------
ENGINE_API EngineStatus engine_session_create(EngineContext* ctx, EngineModel* model, EngineSession** out_sess) {
    if (!out_sess) return ENGINE_ERR_NULL_PTR;
    *out_sess = nullptr;
    if (!model || model->magic != kMagicModel) return ENGINE_ERR_INVALID_HANDLE;
    return guarded([&]() -> EngineStatus {
        clear_error();
        auto s = std::make_unique<EngineSession>();
        s->graph = model->graph;
        if (ctx && ctx->magic == kMagicContext) { s->device = ctx->device; s->precision = ctx->precision; }
        else {
            s->device = default_device();
            const char* p = std::getenv("PDEFA_PRECISION");
            if (p && *p) s->precision = std::string(p) == "bf16" ? PREC_BF16 : std::string(p) == "tf32" ? PREC_TF32 : PREC_FP32;
        }
        require_device(s->device);
        PB_CUDA(cudaSetDevice(s->device));
        PB_CUDA(cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking));
        s->inputs.assign(std::max<size_t>(1, model->graph->inputs.size()), nullptr);
        *out_sess = s.release();
        return ENGINE_OK;
    });
}
ENGINE_API EngineStatus engine_session_set_input(EngineSession* sess, int32_t index, const EngineTensor* input) {
    if (!sess || sess->magic != kMagicSession) return ENGINE_ERR_INVALID_HANDLE;
    if (!tensor_ok(input)) return ENGINE_ERR_INVALID_HANDLE;
    if (index < 0 || index >= (int32_t)sess->inputs.size()) return ENGINE_OK;   // session.cpp:156-159 ignores
    sess->inputs[index] = input;
    return ENGINE_OK;
}
ENGINE_API EngineStatus engine_session_run(EngineSession* sess) {
    if (!sess || sess->magic != kMagicSession) return ENGINE_ERR_INVALID_HANDLE;
    return guarded([&]() -> EngineStatus {
        std::lock_guard<std::mutex> lk(sess->mu);
        clear_error();
        sess->run();
        return ENGINE_OK;
    });
}
ENGINE_API EngineStatus engine_session_get_output(const EngineSession* sess, int32_t index, const EngineTensor** out_t) {
    if (!out_t) return ENGINE_ERR_NULL_PTR;
    *out_t = nullptr;
    if (!sess || sess->magic != kMagicSession) return ENGINE_ERR_INVALID_HANDLE;
    if (index < 0 || index >= (int32_t)sess->out_handles.size()) { set_error("output not available"); return ENGINE_ERR_INVALID_ARG; }
    *out_t = &sess->out_handles[index];
    return ENGINE_OK;
}
ENGINE_API void engine_session_destroy(EngineSession* sess) {
    if (!sess || sess->magic != kMagicSession) return;
    sess->magic = 0;
    if (sess->stream) { cudaSetDevice(sess->device); cudaStreamSynchronize(sess->stream); }
    for (auto& o : sess->outputs) {
        // outputs handed out earlier keep their last host copy
        if (o) try { o->sync_to_host(); } catch (...) {}
        if (o) o->dev = nullptr;
    }
    sess->plans.clear();
    if (sess->debug_buf) cudaFree(sess->debug_buf);
    if (sess->stream) cudaStreamDestroy(sess->stream);
    delete sess;
}
// Reference: PDEFA1.0/src/api/engine_api.cpp:876-892 -> Session::debug_intermediate. After
// a run the reference still holds the intermediates no node consumed (the others are
// freed by their last consumer); this session keeps those too, plus the indices named
// by engine_session_keep_intermediate. The tensor is borrowed (valid until the next
// call for the same index or the session's destruction), fp32, in the engine's
// internal (NHWC for rank 4) layout with the batch in dimension 0.
ENGINE_API EngineStatus engine_session_debug_intermediate(const EngineSession* csess, int32_t idx,
                                                          const EngineTensor** out_t) {
    if (!out_t) return ENGINE_ERR_NULL_PTR;
    *out_t = nullptr;
    if (!csess || csess->magic != kMagicSession) return ENGINE_ERR_INVALID_HANDLE;
    auto* sess = const_cast<EngineSession*>(csess);
    return guarded([&]() -> EngineStatus {
        clear_error();
        std::lock_guard<std::mutex> lk(sess->mu);
        const pb::TView* v = sess->last ? sess->last->debug_view(idx) : nullptr;
        if (!v) { set_error("intermediate not available"); return ENGINE_ERR_INVALID_ARG; }
        PB_CUDA(cudaSetDevice(sess->device));
        const int64_t B = sess->last->batch();
        std::vector<int64_t> shape(v->shape, v->shape + v->rank);
        int64_t per = 1;
        for (int64_t d : shape) per *= d;
        if (!shape.empty()) shape[0] *= B;
        const size_t bytes = (size_t)std::max<int64_t>(per * B, 1) * 4;
        if (sess->debug_cap < bytes) {
            if (sess->debug_buf) cudaFree(sess->debug_buf);
            sess->debug_buf = nullptr;
            sess->debug_cap = 0;
            PB_CUDA(cudaMalloc(&sess->debug_buf, bytes));
            sess->debug_cap = bytes;
        }
        pb::TView dst = *v;
        dst.ptr = sess->debug_buf;
        dst.dt = pb::F32;
        int64_t st = 1;
        for (int d = dst.rank - 1; d >= 0; --d) { dst.stride[d] = st; st *= dst.shape[d]; }
        dst.img_stride = per;
        pb::launch_strided_copy(*v, dst, B, sess->stream);
        auto& slot = sess->debug_out[idx];
        if (!slot.store || slot.store->shape != shape) slot.store = std::make_shared<TensorStore>(shape, ENGINE_F32);
        PB_CUDA(cudaMemcpyAsync(slot.store->host, sess->debug_buf, slot.store->nbytes, cudaMemcpyDeviceToHost,
                                sess->stream));
        PB_CUDA(cudaStreamSynchronize(sess->stream));
        slot.store->host_valid = true;
        slot.store->dev = nullptr;
        slot.handle.magic = pb::kMagicTensor;
        slot.handle.owned.reset();
        slot.handle.borrowed = slot.store.get();
        *out_t = &slot.handle;
        return ENGINE_OK;
    });
}
ENGINE_API EngineStatus engine_session_get_stats(const EngineSession* sess, EngineSessionStats* out_stats) {
    if (!sess || sess->magic != kMagicSession) return ENGINE_ERR_INVALID_HANDLE;
    if (!out_stats) return ENGINE_ERR_NULL_PTR;
    out_stats->last_run_ms = sess->last_run_ms;
    out_stats->runs = sess->runs;
    return ENGINE_OK;
}
ENGINE_API EngineStatus engine_session_set_profile_callback(EngineSession* sess, EngineProfileFn fn, void* user) {
    if (!sess || sess->magic != kMagicSession) return ENGINE_ERR_INVALID_HANDLE;
    sess->profile_fn = fn;
    sess->profile_user = user;
    return ENGINE_OK;
}
ENGINE_API EngineStatus engine_session_clear_profile_callback(EngineSession* sess) {
    if (!sess || sess->magic != kMagicSession) return ENGINE_ERR_INVALID_HANDLE;
    sess->profile_fn = nullptr;
    sess->profile_user = nullptr;
    return ENGINE_OK;
}
ENGINE_API EngineStatus engine_run_simple(const char* model_path, const EngineTensor* const* inputs, int32_t num_inputs,
                                          EngineTensor** outputs, int32_t num_outputs) {
    if (!model_path || !inputs || !outputs) return ENGINE_ERR_NULL_PTR;
    return guarded([&]() -> EngineStatus {
        clear_error();
        EngineModel* m = nullptr;
        EngineStatus st = engine_model_load(nullptr, model_path, &m);
        if (st != ENGINE_OK) return st;
        std::unique_ptr<EngineModel, void (*)(EngineModel*)> mg(m, engine_model_destroy);
        EngineSession* s = nullptr;
        st = engine_session_create(nullptr, m, &s);
        if (st != ENGINE_OK) return st;
        std::unique_ptr<EngineSession, void (*)(EngineSession*)> sg(s, engine_session_destroy);
        for (int32_t i = 0; i < num_inputs; ++i) engine_session_set_input(s, i, inputs[i]);
        std::lock_guard<std::mutex> lk(s->mu);
        s->run();
        for (int32_t i = 0; i < num_outputs; ++i) {
            outputs[i] = nullptr;
            if (i >= (int32_t)s->outputs.size()) continue;
            TensorStore& o = *s->outputs[i];
            o.sync_to_host();
            std::unique_ptr<EngineTensor> t(new_tensor(o.shape, ENGINE_F32));
            std::memcpy(t->ptr()->host, o.host, o.nbytes);
            outputs[i] = t.release();
        }
        return ENGINE_OK;
    });
}

// ---------------------------------------------------------------------------
// OPS
// ---------------------------------------------------------------------------
ENGINE_API EngineStatus engine_ops_add(const EngineTensor* a, const EngineTensor* b, EngineTensor** out) { return binary_op(a, b, out, BIN_ADD); }
ENGINE_API EngineStatus engine_ops_sub(const EngineTensor* a, const EngineTensor* b, EngineTensor** out) { return binary_op(a, b, out, BIN_SUB); }
ENGINE_API EngineStatus engine_ops_mul(const EngineTensor* a, const EngineTensor* b, EngineTensor** out) { return binary_op(a, b, out, BIN_MUL); }
ENGINE_API EngineStatus engine_ops_div(const EngineTensor* a, const EngineTensor* b, EngineTensor** out) { return binary_op(a, b, out, BIN_DIV); }

ENGINE_API EngineStatus engine_ops_matmul_ex(const EngineTensor* a, const EngineTensor* b, EngineTensor* out, int32_t precision) {
    if (!tensor_ok(a) || !tensor_ok(b) || !tensor_ok(out)) return ENGINE_ERR_INVALID_HANDLE;
    if (out->is_borrowed()) { set_error("cannot write to borrowed tensor"); return ENGINE_ERR_INVALID_ARG; }
    return guarded([&]() -> EngineStatus {
        clear_error();
        TensorStore& A = *a->ptr();
        TensorStore& Bt = *b->ptr();
        TensorStore& C = *out->ptr();
        // ops/matmul.cpp:107-135: silently leave `out` untouched on anything but F32 rank-2 [M,K]x[K,N]->[M,N]
        if (A.dtype != ENGINE_F32 || Bt.dtype != ENGINE_F32 || C.dtype != ENGINE_F32) return ENGINE_OK;
        if (A.shape.size() != 2 || Bt.shape.size() != 2 || C.shape.size() != 2) return ENGINE_OK;
        const int64_t M = A.shape[0], K = A.shape[1], N = Bt.shape[1];
        if (Bt.shape[0] != K || C.shape[0] != M || C.shape[1] != N) return ENGINE_OK;
        if (M == 0 || N == 0) return ENGINE_OK;
        OpDevice od(default_device());
        const float* da = static_cast<const float*>(od.upload(A));
        const float* db = static_cast<const float*>(od.upload(Bt));
        float* dc = static_cast<float*>(od.alloc(C.nbytes));
        const size_t sb = gemm_device_scratch_bytes(M, N, K, precision);
        gemm_device(da, db, dc, M, N, K, precision, sb ? od.alloc(sb) : nullptr, od.stream);
        od.download(C, dc);
        return ENGINE_OK;
    });
}
ENGINE_API EngineStatus engine_ops_matmul(const EngineTensor* a, const EngineTensor* b, EngineTensor* out) {
    int prec = PREC_FP32;
    const char* p = std::getenv("PDEFA_MATMUL_PRECISION");
    if (p && *p) prec = std::string(p) == "bf16" ? PREC_BF16 : std::string(p) == "tf32" ? PREC_TF32 : PREC_FP32;
    return engine_ops_matmul_ex(a, b, out, prec);
}

ENGINE_API EngineStatus engine_ops_relu(EngineTensor* t) {
    if (!tensor_ok(t)) return ENGINE_ERR_INVALID_HANDLE;
    if (t->is_borrowed()) return ENGINE_ERR_INVALID_ARG;
    if (t->ptr()->dtype != ENGINE_F32) return ENGINE_OK;   // activation.cpp: non-F32 is a no-op
    return unary_op(t, ACT_RELU);
}
ENGINE_API EngineStatus engine_ops_silu(EngineTensor* t) {
    if (!tensor_ok(t)) return ENGINE_ERR_INVALID_HANDLE;
    if (t->is_borrowed()) return ENGINE_ERR_INVALID_ARG;
    if (t->ptr()->dtype != ENGINE_F32) return ENGINE_OK;
    return unary_op(t, ACT_SILU);
}
ENGINE_API EngineStatus engine_ops_sigmoid(EngineTensor* t) { return unary_op(t, ACT_SIGMOID); }
ENGINE_API EngineStatus engine_ops_tanh(EngineTensor* t) { return unary_op(t, UN_TANH); }
ENGINE_API EngineStatus engine_ops_gelu(EngineTensor* t) { return unary_op(t, ACT_GELU_TANH); }
ENGINE_API EngineStatus engine_ops_clip(EngineTensor* t, float lo, float hi) {
    if (!tensor_ok(t)) return ENGINE_ERR_INVALID_HANDLE;
    if (t->is_borrowed()) { set_error("cannot modify borrowed tensor"); return ENGINE_ERR_INVALID_ARG; }
    if (t->ptr()->dtype != ENGINE_F32) { set_error("only F32 supported"); return ENGINE_ERR_INVALID_ARG; }
    if (lo > hi) { set_error("clip: lo > hi"); return ENGINE_ERR_INVALID_ARG; }
    return unary_op(t, UN_CLIP, lo, hi);
}
ENGINE_API EngineStatus engine_ops_softmax(EngineTensor* t, int32_t axis) {
    if (!tensor_ok(t)) return ENGINE_ERR_INVALID_HANDLE;
    if (t->is_borrowed()) { set_error("cannot modify borrowed tensor"); return ENGINE_ERR_INVALID_ARG; }
    if (t->ptr()->dtype != ENGINE_F32) { set_error("only F32 supported"); return ENGINE_ERR_INVALID_ARG; }
    return guarded([&]() -> EngineStatus {
        clear_error();
        TensorStore& s = *t->ptr();
        const int32_t rank = (int32_t)s.shape.size();
        int32_t ax = axis < 0 ? axis + rank : axis;
        if (ax < 0 || ax >= rank) { set_error("softmax: axis out of range"); return ENGINE_ERR_INVALID_ARG; }
        int64_t outer = 1, inner = 1;
        for (int32_t d = 0; d < ax; ++d) outer *= s.shape[d];
        for (int32_t d = ax + 1; d < rank; ++d) inner *= s.shape[d];
        if (s.numel() == 0) return ENGINE_OK;
        OpDevice od(default_device());
        float* d = static_cast<float*>(od.upload(s));
        launch_softmax(d, d, outer, s.shape[ax], inner, s.numel(), 1, od.stream);
        od.download(s, d);
        return ENGINE_OK;
    });
}

}  // extern "C"
