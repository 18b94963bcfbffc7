// Additive entry points (include/pdefa_b200_ext.h): precision/device selection,
// device-pointer execution, tensor-core GEMM, batched GPU decode/NMS and the
// multi-GPU batch runner (one replica per device, contiguous shards, no collective).
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <set>
#include <thread>

#include "../../include/pdefa_b200_ext.h"
#include "kernels.h"
#include "runtime.h"

using namespace pb;

namespace {

struct DeviceBuffer {
    void* p = nullptr;
    explicit DeviceBuffer(size_t n) {
        if (cudaMalloc(&p, std::max<size_t>(n, 16)) != cudaSuccess) {
            cudaGetLastError();
            fail(ENGINE_ERR_OUT_OF_MEMORY, "device allocation failed");
        }
    }
    ~DeviceBuffer() { if (p) cudaFree(p); }
};

void decode_on_device(const float* d_preds, int64_t batch, int64_t channels, int64_t anchors,
                      const PdefaPreprocessMeta* metas, double conf, double iou, int32_t max_det,
                      int32_t* d_counts, void* d_dets, void* d_work, int32_t* d_meta, int* err, cudaStream_t s) {
    if (metas) PB_CUDA(cudaMemcpyAsync(d_meta, metas, (size_t)batch * sizeof(PdefaPreprocessMeta), cudaMemcpyHostToDevice, s));
    DecodeArgs a;
    a.preds = d_preds;
    a.batch = batch; a.channels = channels; a.anchors = anchors;
    a.meta = metas ? d_meta : nullptr;
    a.conf = conf; a.iou = iou; a.max_det = max_det;
    a.counts = d_counts; a.dets = d_dets; a.work = d_work; a.err = err;
    launch_decode_nms(a, s);
}

}  // namespace

struct PdefaBatchRunner {
    // One of two ping-pong pipeline lanes of a replica: its own plans (input and
    // activation buffers), decode buffers and pinned host copies of the results, so
    // that the copy of micro-batch i+1 onto the GPU overlaps the inference of i.
    struct Lane {
        std::map<int64_t, std::unique_ptr<Plan>> plans;
        // plans whose stem reads the 8-bit frames itself (identity letterbox fused)
        std::map<int64_t, std::unique_ptr<Plan>> plans_u8;
        void* counts = nullptr;      // device [max_per_device]
        void* dets = nullptr;        // device [max_per_device * max_det]
        void* work = nullptr;
        void* meta = nullptr;
        int32_t* h_counts = nullptr; // pinned host mirrors
        PdefaDetection* h_dets = nullptr;
        PdefaPreprocessMeta* h_meta = nullptr;   // pinned staging of the micro-batch's meta records
        size_t dets_cap = 0;
        cudaEvent_t h2d = nullptr, done = nullptr;
        cudaStream_t compute = nullptr;  // letterbox + inference of this lane's micro-batches
        bool busy = false;           // results of (c0, nb) pending
        int64_t c0 = 0, nb = 0;
        // where the pending results go: the arrays of the call (ticket) that queued them
        int64_t ticket = 0;
        int32_t* dst_counts = nullptr;
        PdefaDetection* dst_dets = nullptr;
        int32_t dst_max_det = 0;
        void* pixels = nullptr;      // device copy of an 8-bit micro-batch (pdefa_batch_run_u8)
        size_t pixels_cap = 0;
        Plan* plan = nullptr;        // plan of the pending micro-batch (its error word)
    };
    struct Replica {
        int device = 0;
        cudaStream_t stream = nullptr;   // letterbox, inference, decode, result copies (both lanes)
        cudaStream_t copy = nullptr;     // image copies onto the GPU (overlap the inference)
        Lane lanes[2];
        int64_t next_lane = 0;           // lanes alternate across calls too
        bool u8_unfused = false;         // the graph cannot take 8-bit frames at its stem
    };
    std::shared_ptr<const Graph> graph;
    int precision = PREC_BF16;
    int64_t max_per_device = 1;
    std::vector<Replica> reps;
    int64_t tickets = 0;                 // calls queued so far (pdefa_batch_submit_u8 returns the number)
    // Earlier calls whose pending micro-batches were lost when a later call failed on a
    // device; pdefa_batch_wait reports them instead of returning unwritten arrays.
    std::mutex failed_mu;
    std::set<int64_t> failed_tickets;
};

namespace {

void free_lane(PdefaBatchRunner::Lane& l) {
    if (l.counts) { cudaFree(l.counts); cudaFree(l.dets); cudaFree(l.work); cudaFree(l.meta); }
    if (l.h_counts) { cudaFreeHost(l.h_counts); cudaFreeHost(l.h_dets); cudaFreeHost(l.h_meta); }
    if (l.pixels) cudaFree(l.pixels);
    l.pixels = nullptr;
    l.pixels_cap = 0;
    l.counts = l.dets = l.work = l.meta = nullptr;
    l.h_counts = nullptr;
    l.h_dets = nullptr;
    l.h_meta = nullptr;
    l.dets_cap = 0;
}

// A lane's finished micro-batch -> the arrays of the call that queued it.
void retire_lane(PdefaBatchRunner::Lane& l) {
    if (!l.busy) return;
    l.busy = false;
    PB_CUDA(cudaEventSynchronize(l.done));
    if (l.plan) {
        const int e = l.plan->take_error();
        if (e) fail(ENGINE_ERR_RUNTIME, "device-side wait timed out (code " + std::to_string(e) + ")");
    }
    std::memcpy(l.dst_counts + l.c0, l.h_counts, (size_t)l.nb * 4);
    if (l.dst_max_det > 0)
        std::memcpy(l.dst_dets + l.c0 * l.dst_max_det, l.h_dets, (size_t)l.nb * l.dst_max_det * sizeof(PdefaDetection));
}

}  // namespace

extern "C" {

ENGINE_API EngineStatus engine_context_set_precision(EngineContext* ctx, int32_t precision) {
    if (!ctx || ctx->magic != kMagicContext) return ENGINE_ERR_INVALID_HANDLE;
    if (precision < PREC_FP32 || precision > PREC_BF16) return ENGINE_ERR_INVALID_ARG;
    ctx->precision = precision;
    return ENGINE_OK;
}
ENGINE_API int32_t engine_context_get_precision(const EngineContext* ctx) {
    return (ctx && ctx->magic == kMagicContext) ? ctx->precision : -1;
}
ENGINE_API EngineStatus engine_context_set_device(EngineContext* ctx, int32_t device) {
    if (!ctx || ctx->magic != kMagicContext) return ENGINE_ERR_INVALID_HANDLE;
    if (device < 0) return ENGINE_ERR_INVALID_ARG;
    ctx->device = device;
    return ENGINE_OK;
}
ENGINE_API int32_t engine_context_get_device(const EngineContext* ctx) {
    return (ctx && ctx->magic == kMagicContext) ? ctx->device : -1;
}
ENGINE_API int32_t engine_device_count(void) { return pb::device_count(); }
ENGINE_API int32_t engine_device_error(int32_t device) {
    try { return read_device_error(device); } catch (...) { return -1; }
}
ENGINE_API int32_t engine_session_device_error(EngineSession* sess, int64_t batch) {
    if (!sess || sess->magic != kMagicSession) return -1;
    try {
        std::lock_guard<std::mutex> lk(sess->mu);
        return sess->plan_for(batch).take_error();
    } catch (...) {
        return -1;
    }
}

ENGINE_API EngineStatus engine_session_run_device(EngineSession* sess, const float* d_input, int64_t batch,
                                                  float* d_output, void* stream) {
    if (!sess || sess->magic != kMagicSession) return ENGINE_ERR_INVALID_HANDLE;
    if (!d_input) return ENGINE_ERR_NULL_PTR;
    return guarded([&]() -> EngineStatus {
        std::lock_guard<std::mutex> lk(sess->mu);
        clear_error();
        PB_CUDA(cudaSetDevice(sess->device));
        cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : sess->stream;
        Plan& p = sess->plan_for(batch);
        p.run(s, d_input, nullptr);
        if (d_output && d_output != p.output_buffer(0))
            PB_CUDA(cudaMemcpyAsync(d_output, p.output_buffer(0), p.output_bytes(0), cudaMemcpyDeviceToDevice, s));
        return ENGINE_OK;
    });
}
ENGINE_API EngineStatus engine_session_device_output(EngineSession* sess, int32_t index, int64_t batch, void** out_ptr) {
    if (!sess || sess->magic != kMagicSession) return ENGINE_ERR_INVALID_HANDLE;
    if (!out_ptr) return ENGINE_ERR_NULL_PTR;
    return guarded([&]() -> EngineStatus {
        std::lock_guard<std::mutex> lk(sess->mu);
        PB_CUDA(cudaSetDevice(sess->device));
        Plan& p = sess->plan_for(batch);
        if (index < 0 || index >= p.num_outputs()) return ENGINE_ERR_INVALID_ARG;
        *out_ptr = p.output_buffer(index);
        return ENGINE_OK;
    });
}
ENGINE_API EngineStatus engine_session_output_shape(const EngineSession* sess, int32_t index, int64_t batch,
                                                    int64_t* out_shape, int32_t* out_ndim) {
    if (!sess || sess->magic != kMagicSession) return ENGINE_ERR_INVALID_HANDLE;
    return guarded([&]() -> EngineStatus {
        Plan& p = const_cast<EngineSession*>(sess)->plan_for(batch);
        if (index < 0 || index >= p.num_outputs()) return ENGINE_ERR_INVALID_ARG;
        const auto& s = p.output_shape(index);
        if (out_shape) for (size_t i = 0; i < s.size(); ++i) out_shape[i] = s[i];
        if (out_ndim) *out_ndim = (int32_t)s.size();
        return ENGINE_OK;
    });
}
ENGINE_API EngineStatus engine_model_plan_summary(const EngineModel* model, int32_t precision, int64_t batch,
                                                  char* buf, size_t buf_len, int64_t* out_launches) {
    if (!model || model->magic != kMagicModel) return ENGINE_ERR_INVALID_HANDLE;
    return guarded([&]() -> EngineStatus {
        clear_error();
        auto plan = Plan::dry_run(model->graph, batch, precision);
        const std::string s = plan->summary();
        if (buf && buf_len) {
            const size_t n = std::min(buf_len - 1, s.size());
            std::memcpy(buf, s.data(), n);
            buf[n] = 0;
        }
        if (out_launches) *out_launches = plan->launch_count();
        return ENGINE_OK;
    });
}

ENGINE_API EngineStatus engine_session_keep_intermediate(EngineSession* sess, int32_t idx) {
    if (!sess || sess->magic != kMagicSession) return ENGINE_ERR_INVALID_HANDLE;
    return guarded([&]() -> EngineStatus {
        clear_error();
        if (idx < 0) { set_error("keep_intermediate: negative tensor index"); return ENGINE_ERR_INVALID_ARG; }
        std::lock_guard<std::mutex> lk(sess->mu);
        if (std::find(sess->keep.begin(), sess->keep.end(), idx) == sess->keep.end()) {
            sess->keep.push_back(idx);
            // plans are lowered again, with the value's storage reserved, at the next run
            PB_CUDA(cudaSetDevice(sess->device));
            if (sess->stream) PB_CUDA(cudaStreamSynchronize(sess->stream));
            sess->last = nullptr;
            sess->plans.clear();
        }
        return ENGINE_OK;
    });
}

ENGINE_API EngineStatus engine_model_memory_plan(const EngineModel* model, int32_t precision, int64_t batch,
                                                 size_t* out_packed_bytes, size_t* out_unpacked_bytes) {
    if (!model || model->magic != kMagicModel) return ENGINE_ERR_INVALID_HANDLE;
    return guarded([&]() -> EngineStatus {
        clear_error();
        auto plan = Plan::dry_run(model->graph, batch, precision);
        size_t packed = 0;
        pack_arena(plan->root_bytes(), plan->root_first(), plan->root_last(), &packed);
        if (out_packed_bytes) *out_packed_bytes = packed;
        if (out_unpacked_bytes) *out_unpacked_bytes = plan->activation_bytes();
        return ENGINE_OK;
    });
}

ENGINE_API EngineStatus engine_session_step_timing(EngineSession* sess, int64_t batch, int32_t enable) {
    if (!sess || sess->magic != kMagicSession) return ENGINE_ERR_INVALID_HANDLE;
    return guarded([&]() -> EngineStatus {
        std::lock_guard<std::mutex> lk(sess->mu);
        PB_CUDA(cudaSetDevice(sess->device));
        Plan& p = sess->plan_for(batch);
        p.collect_step_ms();
        p.set_step_timing(enable != 0);
        return ENGINE_OK;
    });
}
ENGINE_API int64_t engine_session_step_times(EngineSession* sess, int64_t batch, double* out_ms, int64_t n_steps) {
    if (!sess || sess->magic != kMagicSession) return -1;
    try {
        std::lock_guard<std::mutex> lk(sess->mu);
        PB_CUDA(cudaSetDevice(sess->device));
        Plan& p = sess->plan_for(batch);
        const auto ms = p.collect_step_ms();
        for (int64_t i = 0; i < n_steps && i < (int64_t)ms.size(); ++i) out_ms[i] = ms[i];
        return (int64_t)ms.size();
    } catch (const std::exception& e) {
        set_error(e.what());
        return -1;
    }
}

ENGINE_API size_t pdefa_decode_work_bytes(int64_t batch, int64_t anchors) { return decode_work_bytes(batch, anchors); }

ENGINE_API EngineStatus pdefa_decode_yolo_device(const float* d_preds, int64_t batch, int64_t channels, int64_t anchors,
                                                 const PdefaPreprocessMeta* d_metas, double conf_thres, double iou_thres,
                                                 int32_t max_det, int32_t* d_counts, PdefaDetection* d_dets, void* d_work,
                                                 size_t work_bytes, void* stream) {
    if (!d_preds || !d_counts || !d_work || (!d_dets && max_det > 0)) return ENGINE_ERR_NULL_PTR;
    return guarded([&]() -> EngineStatus {
        clear_error();
        if (batch < 0 || channels < 5 || anchors < 0) { set_error("decode: bad shape"); return ENGINE_ERR_INVALID_SHAPE; }
        if (max_det < 0) { set_error("decode: max_det must be >= 0"); return ENGINE_ERR_INVALID_ARG; }
        if (work_bytes < decode_work_bytes(batch, anchors)) { set_error("decode: work buffer too small"); return ENGINE_ERR_INVALID_ARG; }
        int dev = 0;
        PB_CUDA(cudaGetDevice(&dev));
        DecodeArgs a;
        a.preds = d_preds;
        a.batch = batch; a.channels = channels; a.anchors = anchors;
        a.meta = reinterpret_cast<const int32_t*>(d_metas);
        a.conf = conf_thres; a.iou = iou_thres; a.max_det = max_det;
        a.counts = d_counts; a.dets = d_dets; a.work = d_work; a.err = device_error_word(dev);
        launch_decode_nms(a, static_cast<cudaStream_t>(stream));
        return ENGINE_OK;
    });
}

ENGINE_API int64_t engine_session_launch_count(const EngineSession* sess, int64_t batch) {
    if (!sess || sess->magic != kMagicSession) return -1;
    try {
        return const_cast<EngineSession*>(sess)->plan_for(batch).launch_count();
    } catch (...) {
        return -1;
    }
}

}  // extern "C"

namespace pb {
size_t gemm_device_scratch_bytes(int64_t m, int64_t n, int64_t k, int precision) {
    if (precision == PREC_FP32) return 0;
    const int esz = precision == PREC_BF16 ? 2 : 4;
    return ((size_t)m * k + (size_t)n * k) * esz + 512;
}

// C[m,n] = A[m,k] B[k,n] on `s`; tensor-core precisions stage their operands in
// `scratch` (gemm_device_scratch_bytes), which must stay untouched until the GEMM ran.
void gemm_device(const float* d_a, const float* d_b, float* d_c, int64_t m, int64_t n, int64_t k, int precision,
                 void* scratch, cudaStream_t s) {
    int dev = 0;
    PB_CUDA(cudaGetDevice(&dev));
    if (precision != PREC_FP32) {
        const int op_dt = precision == PREC_BF16 ? BF16 : F32;
        const bool ok = n % 16 == 0 && k % (op_dt == BF16 ? 16 : 8) == 0 && ((uintptr_t)d_c % 16) == 0;
        if (ok) {
            launch_gemm_tc(d_a, d_b, d_c, m, n, k, op_dt, scratch, device_error_word(dev), s);
            return;
        }
    }
    launch_gemm_f32(d_a, d_b, d_c, nullptr, m, n, k, k, n, n, 1, 0, 0, 0, s);
}
}  // namespace pb

extern "C" {

ENGINE_API EngineStatus engine_gemm_f32_device(const float* d_a, const float* d_b, float* d_c, int64_t m, int64_t n,
                                               int64_t k, int32_t precision, void* stream) {
    if (!d_a || !d_b || !d_c) return ENGINE_ERR_NULL_PTR;
    return guarded([&]() -> EngineStatus {
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        // Operand staging comes from the stream-ordered pool: calls on different
        // streams never share it, and a warm pool makes no cudaMalloc.
        void* sc = nullptr;
        const size_t sb = gemm_device_scratch_bytes(m, n, k, precision);
        if (sb) PB_CUDA(cudaMallocAsync(&sc, sb, s));
        try {
            gemm_device(d_a, d_b, d_c, m, n, k, precision, sc, s);
        } catch (...) {
            if (sc) cudaFreeAsync(sc, s);
            throw;
        }
        if (sc) PB_CUDA(cudaFreeAsync(sc, s));
        return ENGINE_OK;
    });
}

ENGINE_API EngineStatus pdefa_decode_yolo(const float* preds, int32_t preds_on_device, int64_t batch, int64_t channels,
                                          int64_t anchors, const PdefaPreprocessMeta* metas, double conf_thres,
                                          double iou_thres, int32_t max_det, int32_t* out_counts,
                                          PdefaDetection* out_dets, int32_t device) {
    if (!preds || !out_counts || (!out_dets && max_det > 0)) return ENGINE_ERR_NULL_PTR;
    return guarded([&]() -> EngineStatus {
        clear_error();
        if (batch < 0 || channels < 5 || anchors < 0) { set_error("decode: bad shape"); return ENGINE_ERR_INVALID_SHAPE; }
        if (max_det < 0) { set_error("decode: max_det must be >= 0"); return ENGINE_ERR_INVALID_ARG; }
        if (batch == 0) return ENGINE_OK;
        require_device(device);
        PB_CUDA(cudaSetDevice(device));
        cudaStream_t s;
        PB_CUDA(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
        struct SG { cudaStream_t s; ~SG() { cudaStreamSynchronize(s); cudaStreamDestroy(s); } } sg{s};
        const size_t pbytes = (size_t)batch * channels * anchors * 4;
        std::unique_ptr<DeviceBuffer> dpred;
        const float* dp = preds;
        if (!preds_on_device) {
            dpred = std::make_unique<DeviceBuffer>(pbytes);
            PB_CUDA(cudaMemcpyAsync(dpred->p, preds, pbytes, cudaMemcpyHostToDevice, s));
            dp = static_cast<const float*>(dpred->p);
        }
        DeviceBuffer counts((size_t)batch * 4), dets((size_t)batch * std::max(1, max_det) * sizeof(PdefaDetection));
        DeviceBuffer work(decode_work_bytes(batch, anchors)), meta((size_t)batch * sizeof(PdefaPreprocessMeta));
        int* err = device_error_word(device);
        decode_on_device(dp, batch, channels, anchors, metas, conf_thres, iou_thres, max_det,
                         static_cast<int32_t*>(counts.p), dets.p, work.p, static_cast<int32_t*>(meta.p), err, s);
        PB_CUDA(cudaMemcpyAsync(out_counts, counts.p, (size_t)batch * 4, cudaMemcpyDeviceToHost, s));
        if (max_det > 0)
            PB_CUDA(cudaMemcpyAsync(out_dets, dets.p, (size_t)batch * max_det * sizeof(PdefaDetection),
                                    cudaMemcpyDeviceToHost, s));
        PB_CUDA(cudaStreamSynchronize(s));
        for (int64_t b = 0; b < batch; ++b)
            if (out_counts[b] < 0) { set_error("decode: more than 16384 candidates in one image"); return ENGINE_ERR_NOT_IMPL; }
        return ENGINE_OK;
    });
}

ENGINE_API EngineStatus pdefa_batch_create(EngineModel* model, int32_t n_devices, const int32_t* devices,
                                           int32_t precision, int64_t max_images_per_device,
                                           PdefaBatchRunner** out_runner) {
    if (!out_runner) return ENGINE_ERR_NULL_PTR;
    *out_runner = nullptr;
    if (!model || model->magic != kMagicModel) return ENGINE_ERR_INVALID_HANDLE;
    return guarded([&]() -> EngineStatus {
        clear_error();
        if (n_devices < 1 || max_images_per_device < 1) return ENGINE_ERR_INVALID_ARG;
        auto r = std::make_unique<PdefaBatchRunner>();
        r->graph = model->graph;
        r->precision = precision;
        r->max_per_device = max_images_per_device;
        r->reps.resize(n_devices);
        for (int i = 0; i < n_devices; ++i) {
            auto& rp = r->reps[i];
            rp.device = devices ? devices[i] : i;
            require_device(rp.device);
            PB_CUDA(cudaSetDevice(rp.device));
            PB_CUDA(cudaStreamCreateWithFlags(&rp.stream, cudaStreamNonBlocking));
            PB_CUDA(cudaStreamCreateWithFlags(&rp.copy, cudaStreamNonBlocking));
            // All GPU work of both lanes on one stream: a lane's own compute stream, or the
            // decode on a third stream, put kernels beside the convolutions that slowed them
            // more than they overlapped (pipelined e2e 29.3k against 30.9k images/s)
            rp.lanes[0].compute = rp.stream;
            rp.lanes[1].compute = rp.stream;
            for (auto& l : rp.lanes) {
                PB_CUDA(cudaEventCreateWithFlags(&l.h2d, cudaEventDisableTiming));
                PB_CUDA(cudaEventCreateWithFlags(&l.done, cudaEventDisableTiming));
            }
        }
        *out_runner = r.release();
        return ENGINE_OK;
    });
}

}  // extern "C"

namespace {

// What pdefa_batch_run / pdefa_batch_run_u8 feed the runner: float32 model inputs, or
// 8-bit images letterboxed on the GPU.
struct BatchInput {
    const float* f32 = nullptr;
    const uint8_t* u8 = nullptr;
    int channels = 0;
    LetterboxGeom geo{};
};

PdefaPreprocessMeta meta_of(const LetterboxGeom& g) {
    PdefaPreprocessMeta m;
    m.target_w = g.W; m.target_h = g.H;
    m.orig_w = g.src_w; m.orig_h = g.src_h;
    m.pad_x = g.px; m.pad_y = g.py;
    m.scaled_w = g.sw; m.scaled_h = g.sh;
    m.ratio = g.ratio;
    return m;
}

// drain = true: the call returns with its results in out_counts / out_dets. drain =
// false (pdefa_batch_submit_u8): the call returns once its work is queued; its last
// micro-batches finish later and are copied out when their lane is reused, by a later
// call, or by pdefa_batch_wait. Either way, results of earlier calls still pending in
// a lane are copied to those calls' arrays before the lane is reused, and every
// earlier call is complete when this one returns.
EngineStatus run_batch(PdefaBatchRunner* r, const BatchInput& in, int64_t n_images, const PdefaPreprocessMeta* metas,
                       double conf_thres, double iou_thres, int32_t max_det, int32_t* out_counts,
                       PdefaDetection* out_dets, bool drain = true, int64_t* out_ticket = nullptr) {
    return guarded([&]() -> EngineStatus {
        clear_error();
        if (max_det < 0) return ENGINE_ERR_INVALID_ARG;
        const int64_t ticket = ++r->tickets;
        if (out_ticket) *out_ticket = ticket;
        const int nd = (int)r->reps.size();
        const int64_t per = (n_images + nd - 1) / nd;
        std::vector<std::string> errs(nd);
        std::vector<std::thread> th;
        for (int d = 0; d < nd; ++d) {
            th.emplace_back([&, d] {
                auto& rp = r->reps[d];
                auto retire = [](PdefaBatchRunner::Lane& l) { retire_lane(l); };
                try {
                    PB_CUDA(cudaSetDevice(rp.device));
                    const int64_t lo = std::min(n_images, d * per), hi = std::min(n_images, lo + per);
                    // Micro-batches of at most max_per_device images alternate between the two
                    // lanes: the copy stream brings micro-batch i+1 onto the GPU while the
                    // compute stream runs inference + decode of micro-batch i.
                    // The first micro-batch of a shard is a quarter of the others, so the
                    // pipeline fills after a short copy; then full micro-batches.
                    const int64_t mfull = r->max_per_device;
                    const int64_t mfirst = (hi - lo > mfull && mfull >= 8) ? mfull / 4 : mfull;
                    int64_t i = 0;
                    for (int64_t c0 = lo, nb = 0; c0 < hi; c0 += nb, ++i) {
                        nb = std::min(i == 0 ? mfirst : mfull, hi - c0);
                        auto& l = rp.lanes[rp.next_lane++ & 1];
                        retire(l);    // the lane's buffers are free once its previous micro-batch is done
                        // Frames already at the model size with scale-only preprocessing go
                        // straight to a plan whose stem conv reads the 8-bit pixels (pixel *
                        // scale, bit for bit the letterbox's value); other geometries, and
                        // graphs whose stem cannot take them, letterbox into a float32 input.
                        const LetterboxGeom& gm = in.geo;
                        const bool fuse = !in.f32 && !rp.u8_unfused && in.channels == 3 && gm.ratio == 1.0f &&
                                          gm.inv == 1.0f && gm.src_w == gm.W && gm.src_h == gm.H && gm.sw == gm.W &&
                                          gm.sh == gm.H && gm.px == 0 && gm.py == 0 && gm.W % 4 == 0 &&
                                          gm.scale > 0.0f && r->precision == PREC_BF16;
                        Plan* pp = nullptr;
                        if (fuse) {
                            auto fit = l.plans_u8.find(nb);
                            if (fit != l.plans_u8.end() && fit->second->u8_scale() != gm.scale) {
                                l.plans_u8.erase(fit);
                                fit = l.plans_u8.end();
                            }
                            if (fit == l.plans_u8.end()) {
                                try {
                                    fit = l.plans_u8.emplace(nb, std::make_unique<Plan>(r->graph, nb, r->precision,
                                                                                        rp.device, std::vector<int32_t>{},
                                                                                        std::vector<int64_t>{}, gm.scale))
                                              .first;
                                    if (verbose())
                                        std::fprintf(stderr, "[pdefa-b200] batch runner: 8-bit frames read by the stem "
                                                     "(batch %lld)\n", (long long)nb);
                                } catch (const Error& e) {
                                    if (e.status != ENGINE_ERR_NOT_IMPL) throw;
                                    if (verbose())
                                        std::fprintf(stderr, "[pdefa-b200] batch runner: letterbox kept (%s)\n", e.what());
                                    rp.u8_unfused = true;
                                }
                            }
                            if (fit != l.plans_u8.end()) pp = fit->second.get();
                        }
                        if (!pp) {
                            auto it = l.plans.find(nb);
                            if (it == l.plans.end())
                                it = l.plans.emplace(nb, std::make_unique<Plan>(r->graph, nb, r->precision, rp.device))
                                         .first;
                            pp = it->second.get();
                        }
                        Plan& p = *pp;
                        const bool fused = p.u8_scale() > 0.0f;
                        const auto& os = p.output_shape(0);
                        if (os.size() != 3) fail(ENGINE_ERR_INVALID_SHAPE, "batch runner expects a [B, 4+nc, A] output");
                        const int64_t ch = os[1], A = os[2];
                        const size_t need = (size_t)r->max_per_device * std::max(1, max_det) * sizeof(PdefaDetection);
                        if (l.dets_cap < need || !l.work) {
                            free_lane(l);
                            const int64_t cap_imgs = r->max_per_device;
                            PB_CUDA(cudaMalloc(&l.counts, cap_imgs * 4));
                            PB_CUDA(cudaMalloc(&l.dets, need));
                            PB_CUDA(cudaMalloc(&l.work, decode_work_bytes(cap_imgs, A)));
                            PB_CUDA(cudaMalloc(&l.meta, cap_imgs * sizeof(PdefaPreprocessMeta)));
                            PB_CUDA(cudaMallocHost(reinterpret_cast<void**>(&l.h_counts), cap_imgs * 4));
                            PB_CUDA(cudaMallocHost(reinterpret_cast<void**>(&l.h_dets), need));
                            PB_CUDA(cudaMallocHost(reinterpret_cast<void**>(&l.h_meta),
                                                   cap_imgs * sizeof(PdefaPreprocessMeta)));
                            l.dets_cap = need;
                        }
                        const size_t ibytes = p.input_bytes(0);
                        if (in.f32) {
                            PB_CUDA(cudaMemcpyAsync(p.input_buffer(0), in.f32 + c0 * (ibytes / 4 / nb), ibytes,
                                                    cudaMemcpyHostToDevice, rp.copy));
                            PB_CUDA(cudaEventRecord(l.h2d, rp.copy));
                            PB_CUDA(cudaStreamWaitEvent(l.compute, l.h2d, 0));
                        } else {
                            // 8-bit pixels cross PCIe (a quarter of the float32 bytes for RGB) and
                            // are letterboxed into the plan's input on the GPU
                            if (ibytes != (size_t)nb * 3 * in.geo.H * in.geo.W * (fused ? 1 : sizeof(float)))
                                fail(ENGINE_ERR_INVALID_SHAPE, "batch_run_u8: the model input is not [B, 3, target_h, target_w]");
                            const size_t pb_img = (size_t)in.geo.src_h * in.geo.src_w * in.channels;
                            if (fused) {
                                PB_CUDA(cudaMemcpyAsync(p.input_buffer(0), in.u8 + c0 * pb_img, pb_img * nb,
                                                        cudaMemcpyHostToDevice, rp.copy));
                                PB_CUDA(cudaEventRecord(l.h2d, rp.copy));
                                PB_CUDA(cudaStreamWaitEvent(l.compute, l.h2d, 0));
                            } else {
                            if (l.pixels_cap < pb_img * r->max_per_device) {
                                if (l.pixels) cudaFree(l.pixels);
                                l.pixels = nullptr;
                                l.pixels_cap = 0;
                                PB_CUDA(cudaMalloc(&l.pixels, pb_img * r->max_per_device));
                                l.pixels_cap = pb_img * r->max_per_device;
                            }
                            PB_CUDA(cudaMemcpyAsync(l.pixels, in.u8 + c0 * pb_img, pb_img * nb, cudaMemcpyHostToDevice,
                                                    rp.copy));
                            PB_CUDA(cudaEventRecord(l.h2d, rp.copy));
                            PB_CUDA(cudaStreamWaitEvent(l.compute, l.h2d, 0));
                            launch_letterbox_u8(static_cast<const uint8_t*>(l.pixels), nb, in.channels, in.geo,
                                                p.input_buffer(0), l.compute);
                            }
                        }
                        p.run(l.compute);
                        // decode right after the inference, on the same stream
                        const cudaStream_t post = l.compute;
                        // meta records via pinned staging: the copy needs no wait for the
                        // decode stream (a pageable source would make the host wait for it)
                        if (metas) std::memcpy(l.h_meta, metas + c0, (size_t)nb * sizeof(PdefaPreprocessMeta));
                        decode_on_device(p.output_buffer(0), nb, ch, A, metas ? l.h_meta : nullptr, conf_thres,
                                         iou_thres, max_det, static_cast<int32_t*>(l.counts), l.dets, l.work,
                                         static_cast<int32_t*>(l.meta), device_error_word(rp.device), post);
                        PB_CUDA(cudaMemcpyAsync(l.h_counts, l.counts, nb * 4, cudaMemcpyDeviceToHost, post));
                        if (max_det > 0)
                            PB_CUDA(cudaMemcpyAsync(l.h_dets, l.dets, (size_t)nb * max_det * sizeof(PdefaDetection),
                                                    cudaMemcpyDeviceToHost, post));
                        PB_CUDA(cudaEventRecord(l.done, post));
                        l.busy = true;
                        l.plan = &p;
                        l.c0 = c0;
                        l.nb = nb;
                        l.ticket = ticket;
                        l.dst_counts = out_counts;
                        l.dst_dets = out_dets;
                        l.dst_max_det = max_det;
                    }
                    // oldest lane first; a submit leaves its own micro-batches pending
                    for (int k = 0; k < 2; ++k) {
                        auto& l = rp.lanes[(rp.next_lane + k) & 1];
                        if (drain || l.ticket < ticket) retire(l);
                    }
                    if (drain && read_device_error(rp.device)) fail(ENGINE_ERR_RUNTIME, "device-side wait timed out");
                } catch (const std::exception& e) {
                    errs[d] = e.what();
                    // Leave no lane pending: its buffers may be reused by the next call.
                    // A lane still holding an earlier call's micro-batch hands its results
                    // over if they finished; otherwise that call is marked failed, so its
                    // pdefa_batch_wait reports the loss.
                    for (auto& l : rp.lanes) {
                        if (!l.busy) continue;
                        l.busy = false;
                        const bool done = cudaEventSynchronize(l.done) == cudaSuccess;
                        if (l.ticket < ticket && done) {
                            std::memcpy(l.dst_counts + l.c0, l.h_counts, (size_t)l.nb * 4);
                            if (l.dst_max_det > 0)
                                std::memcpy(l.dst_dets + l.c0 * l.dst_max_det, l.h_dets,
                                            (size_t)l.nb * l.dst_max_det * sizeof(PdefaDetection));
                        } else if (l.ticket < ticket) {
                            std::lock_guard<std::mutex> lk(r->failed_mu);
                            r->failed_tickets.insert(l.ticket);
                        }
                    }
                    cudaStreamSynchronize(rp.copy);
                    cudaStreamSynchronize(rp.stream);
                }
            });
        }
        for (auto& t : th) t.join();
        for (int d = 0; d < nd; ++d)
            if (!errs[d].empty()) { set_error("device " + std::to_string(r->reps[d].device) + ": " + errs[d]); return ENGINE_ERR_RUNTIME; }
        return ENGINE_OK;
    });
}


}  // namespace

namespace {

EngineStatus batch_u8(PdefaBatchRunner* r, const uint8_t* images, int64_t n_images, int32_t src_h, int32_t src_w,
                      int32_t channels, const PdefaPreprocessConfig* cfg, double conf_thres, double iou_thres,
                      int32_t max_det, int32_t* out_counts, PdefaDetection* out_dets, PdefaPreprocessMeta* out_meta,
                      bool drain, int64_t* out_ticket) {
    if (!r || !images || !cfg || !out_counts || (!out_dets && max_det > 0)) return ENGINE_ERR_NULL_PTR;
    return guarded([&]() -> EngineStatus {
        clear_error();
        if (src_h <= 0 || src_w <= 0 || cfg->target_w <= 0 || cfg->target_h <= 0 ||
            (channels != 1 && channels != 3 && channels != 4)) {
            set_error("batch_run_u8: bad image size, target or channel count");
            return ENGINE_ERR_INVALID_ARG;
        }
        BatchInput in;
        in.u8 = images;
        in.channels = channels;
        in.geo = letterbox_geometry(src_w, src_h, cfg->target_w, cfg->target_h, cfg->scale, cfg->pad_value);
        const PdefaPreprocessMeta m = meta_of(in.geo);
        if (out_meta) *out_meta = m;
        // boxes come back in original-image coordinates, as decode_yolo(out, meta) gives them
        std::vector<PdefaPreprocessMeta> metas((size_t)std::max<int64_t>(n_images, 1), m);
        return run_batch(r, in, n_images, metas.data(), conf_thres, iou_thres, max_det, out_counts, out_dets, drain,
                         out_ticket);
    });
}

}  // namespace

extern "C" {

ENGINE_API EngineStatus pdefa_batch_run(PdefaBatchRunner* r, const float* images, int64_t n_images,
                                        const PdefaPreprocessMeta* metas, double conf_thres, double iou_thres,
                                        int32_t max_det, int32_t* out_counts, PdefaDetection* out_dets) {
    if (!r || !images || !out_counts || (!out_dets && max_det > 0)) return ENGINE_ERR_NULL_PTR;
    BatchInput in;
    in.f32 = images;
    return run_batch(r, in, n_images, metas, conf_thres, iou_thres, max_det, out_counts, out_dets);
}

ENGINE_API EngineStatus pdefa_batch_run_u8(PdefaBatchRunner* r, const uint8_t* images, int64_t n_images, int32_t src_h,
                                           int32_t src_w, int32_t channels, const PdefaPreprocessConfig* cfg,
                                           double conf_thres, double iou_thres, int32_t max_det, int32_t* out_counts,
                                           PdefaDetection* out_dets, PdefaPreprocessMeta* out_meta) {
    return batch_u8(r, images, n_images, src_h, src_w, channels, cfg, conf_thres, iou_thres, max_det, out_counts,
                    out_dets, out_meta, true, nullptr);
}

ENGINE_API EngineStatus pdefa_batch_submit_u8(PdefaBatchRunner* r, const uint8_t* images, int64_t n_images,
                                              int32_t src_h, int32_t src_w, int32_t channels,
                                              const PdefaPreprocessConfig* cfg, double conf_thres, double iou_thres,
                                              int32_t max_det, int32_t* out_counts, PdefaDetection* out_dets,
                                              PdefaPreprocessMeta* out_meta, int64_t* out_ticket) {
    if (!out_ticket) return ENGINE_ERR_NULL_PTR;
    return batch_u8(r, images, n_images, src_h, src_w, channels, cfg, conf_thres, iou_thres, max_det, out_counts,
                    out_dets, out_meta, false, out_ticket);
}

ENGINE_API EngineStatus pdefa_batch_wait(PdefaBatchRunner* r, int64_t ticket) {
    if (!r) return ENGINE_ERR_NULL_PTR;
    return guarded([&]() -> EngineStatus {
        clear_error();
        const int64_t upto = ticket > 0 ? ticket : r->tickets;
        {
            std::lock_guard<std::mutex> lk(r->failed_mu);
            auto it = r->failed_tickets.begin();
            if (it != r->failed_tickets.end() && *it <= upto) {
                const int64_t t = *it;
                r->failed_tickets.erase(r->failed_tickets.begin(), r->failed_tickets.upper_bound(upto));
                set_error("call " + std::to_string(t) + " lost its pending results when a later call failed");
                return ENGINE_ERR_RUNTIME;
            }
        }
        for (auto& rp : r->reps) {
            PB_CUDA(cudaSetDevice(rp.device));
            for (int k = 0; k < 2; ++k) {
                auto& l = rp.lanes[(rp.next_lane + k) & 1];    // oldest first
                if (l.busy && l.ticket <= upto) retire_lane(l);
            }
            if (read_device_error(rp.device)) fail(ENGINE_ERR_RUNTIME, "device-side wait timed out");
        }
        return ENGINE_OK;
    });
}

ENGINE_API EngineStatus pdefa_letterbox_meta(int32_t src_w, int32_t src_h, const PdefaPreprocessConfig* cfg,
                                             PdefaPreprocessMeta* out_meta) {
    if (!cfg || !out_meta) return ENGINE_ERR_NULL_PTR;
    if (src_w <= 0 || src_h <= 0 || cfg->target_w <= 0 || cfg->target_h <= 0) return ENGINE_ERR_INVALID_ARG;
    *out_meta = meta_of(letterbox_geometry(src_w, src_h, cfg->target_w, cfg->target_h, cfg->scale, cfg->pad_value));
    return ENGINE_OK;
}

ENGINE_API EngineStatus pdefa_letterbox_device(const uint8_t* d_images, int64_t n, int32_t src_h, int32_t src_w,
                                               int32_t channels, const PdefaPreprocessConfig* cfg, float* d_out,
                                               void* stream) {
    if (!d_images || !cfg || !d_out) return ENGINE_ERR_NULL_PTR;
    return guarded([&]() -> EngineStatus {
        clear_error();
        if (n < 0 || src_h <= 0 || src_w <= 0 || cfg->target_w <= 0 || cfg->target_h <= 0 ||
            (channels != 1 && channels != 3 && channels != 4)) {
            set_error("letterbox: bad image size, target or channel count");
            return ENGINE_ERR_INVALID_ARG;
        }
        const LetterboxGeom g = letterbox_geometry(src_w, src_h, cfg->target_w, cfg->target_h, cfg->scale,
                                                   cfg->pad_value);
        for (int64_t b0 = 0; b0 < n; b0 += 65535)
            launch_letterbox_u8(d_images + (size_t)b0 * src_h * src_w * channels, std::min<int64_t>(65535, n - b0),
                                channels, g, d_out + (size_t)b0 * 3 * g.H * g.W, static_cast<cudaStream_t>(stream));
        return ENGINE_OK;
    });
}

ENGINE_API EngineStatus pdefa_letterbox(const uint8_t* images, int64_t n, int32_t src_h, int32_t src_w,
                                        int32_t channels, const PdefaPreprocessConfig* cfg, float* out,
                                        PdefaPreprocessMeta* out_meta, int32_t device) {
    if (!images || !cfg || !out) return ENGINE_ERR_NULL_PTR;
    return guarded([&]() -> EngineStatus {
        clear_error();
        if (n < 0 || src_h <= 0 || src_w <= 0 || cfg->target_w <= 0 || cfg->target_h <= 0 ||
            (channels != 1 && channels != 3 && channels != 4)) {
            set_error("letterbox: bad image size, target or channel count");
            return ENGINE_ERR_INVALID_ARG;
        }
        const LetterboxGeom g = letterbox_geometry(src_w, src_h, cfg->target_w, cfg->target_h, cfg->scale,
                                                   cfg->pad_value);
        if (out_meta) *out_meta = meta_of(g);
        if (n == 0) return ENGINE_OK;
        require_device(device);
        PB_CUDA(cudaSetDevice(device));
        cudaStream_t s;
        PB_CUDA(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
        struct SG { cudaStream_t s; ~SG() { cudaStreamSynchronize(s); cudaStreamDestroy(s); } } sg{s};
        const size_t ib = (size_t)n * src_h * src_w * channels, ob = (size_t)n * 3 * g.H * g.W * sizeof(float);
        DeviceBuffer din(ib), dout(ob);
        PB_CUDA(cudaMemcpyAsync(din.p, images, ib, cudaMemcpyHostToDevice, s));
        for (int64_t b0 = 0; b0 < n; b0 += 65535)
            launch_letterbox_u8(static_cast<const uint8_t*>(din.p) + (size_t)b0 * src_h * src_w * channels,
                                std::min<int64_t>(65535, n - b0), channels, g,
                                static_cast<float*>(dout.p) + (size_t)b0 * 3 * g.H * g.W, s);
        PB_CUDA(cudaMemcpyAsync(out, dout.p, ob, cudaMemcpyDeviceToHost, s));
        PB_CUDA(cudaStreamSynchronize(s));
        return ENGINE_OK;
    });
}

ENGINE_API void pdefa_batch_destroy(PdefaBatchRunner* r) {
    if (!r) return;
    for (auto& rp : r->reps) {
        cudaSetDevice(rp.device);
        if (rp.stream) cudaStreamSynchronize(rp.stream);
        if (rp.copy) cudaStreamSynchronize(rp.copy);
        for (auto& l : rp.lanes) {
            l.plans.clear();
            l.plans_u8.clear();
            free_lane(l);
            if (l.h2d) cudaEventDestroy(l.h2d);
            if (l.done) cudaEventDestroy(l.done);
        }
        if (rp.stream) cudaStreamDestroy(rp.stream);
        if (rp.copy) cudaStreamDestroy(rp.copy);
    }
    delete r;
}

}  // extern "C"
