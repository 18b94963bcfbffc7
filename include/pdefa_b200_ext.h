/* pdefa_b200_ext.h - additive entry points of the B200 build of libpdefa_native.so.
 *
 * These have no counterpart in the reference ABI (pdefa/pdefa.def); they are extra
 * exports, so the reference ctypes layer is unaffected. They expose what a GPU
 * engine needs beyond the CPU engine's surface: precision and device selection,
 * device-pointer execution, the batched YOLO decode/NMS that replaces the
 * reference's pure-Python decode_yolo (pdefa/python/src/pdefa/_bindings.py:1095-1212),
 * and the multi-GPU batch runner behind BatchInference (pdefa/python/src/pdefa/batch.py:13-70).
 * All pointers are plain host or device pointers; no framework types cross the ABI.
 */
#ifndef PDEFA_B200_EXT_H
#define PDEFA_B200_EXT_H

#include <stdint.h>
#include "engine_c_api.h"
#include "pdefa_c_api.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Arithmetic used by sessions created from a context.
 * FP32: strict fp32 SIMT kernels (parity <= 1e-5 with the reference engine).
 * TF32 / BF16: tcgen05 tensor-core kernels with fp32 accumulation (<= 1e-2). */
typedef enum {
    PDEFA_PREC_FP32 = 0,
    PDEFA_PREC_TF32 = 1,
    PDEFA_PREC_BF16 = 2
} PdefaPrecision;

ENGINE_API EngineStatus engine_context_set_precision(EngineContext* ctx, int32_t precision);
ENGINE_API int32_t      engine_context_get_precision(const EngineContext* ctx);
ENGINE_API EngineStatus engine_context_set_device(EngineContext* ctx, int32_t device);
ENGINE_API int32_t      engine_context_get_device(const EngineContext* ctx);
/* Number of visible CUDA devices (0 without a GPU). */
ENGINE_API int32_t      engine_device_count(void);
/* Device-wide error word of the kernels that run outside a session's plan (GPU
 * decode, engine_gemm_f32_device): set by bounded waits that timed out (0 = none),
 * cleared when read. Plans have their own word (engine_session_device_error). */
ENGINE_API int32_t      engine_device_error(int32_t device);
/* Error code the kernels of `sess`'s plan for `batch` recorded in their last
 * engine_session_run_device call (0: none; a bounded wait that ran out), read once the
 * caller has synchronized that call's stream; the code is cleared when read. Each plan
 * has its own word, so one session's timeout never affects another's kernels. */
ENGINE_API int32_t      engine_session_device_error(EngineSession* sess, int64_t batch);

/* Run a session on device buffers already resident on the session's GPU.
 * d_input: [batch, C, H, W] fp32 NCHW; d_output: graph output 0 for `batch` images
 * (shape from engine_session_output_shape). stream: cudaStream_t or NULL for the
 * session's own stream. Returns after the work is enqueued (asynchronous). */
ENGINE_API EngineStatus engine_session_run_device(EngineSession* sess, const float* d_input,
                                                  int64_t batch, float* d_output, void* stream);
/* Device address of the session's own output buffer `index` for `batch` images
 * (valid until the session is destroyed; engine_session_run_device with
 * d_output == NULL leaves the result there without an extra copy). */
ENGINE_API EngineStatus engine_session_device_output(EngineSession* sess, int32_t index, int64_t batch,
                                                     void** out_ptr);
ENGINE_API EngineStatus engine_session_output_shape(const EngineSession* sess, int32_t index,
                                                    int64_t batch, int64_t* out_shape,
                                                    int32_t* out_ndim);
/* Lowers `model` for `batch` images at `precision` without touching a GPU and
 * reports whether it is supported (status + message as usual). On success
 * writes one line per launch ("<kernel kind> <node name>") into buf (truncated to
 * buf_len, NUL-terminated) and the launch count into *out_launches. */
ENGINE_API EngineStatus engine_model_plan_summary(const EngineModel* model, int32_t precision, int64_t batch,
                                                  char* buf, size_t buf_len, int64_t* out_launches);
/* Keeps intermediate tensor `idx` (an index of the .engine graph's tensors) readable
 * after each run, for engine_session_debug_intermediate. The reference keeps only the
 * intermediates no node consumes (PDEFA1.0/src/core/session.cpp:322-337); the memory
 * planner of this library reuses the storage of the others, so a caller that wants one
 * of them names it here first. The session's plans are lowered again at the next run
 * (the value's storage then stays reserved). No counterpart in the reference. */
ENGINE_API EngineStatus engine_session_keep_intermediate(EngineSession* sess, int32_t idx);
/* Device memory plan of `model` for `batch` images at `precision`, computed without a
 * GPU: *out_packed_bytes = the activation arena a session allocates (values whose live
 * ranges do not overlap share bytes, as PDEFA1.0/src/memory/memory_plan.cpp:105-137
 * plans the reference's buffers); *out_unpacked_bytes = one buffer per value.
 * Weights, the input and the output buffers are extra. Either pointer may be NULL. */
ENGINE_API EngineStatus engine_model_memory_plan(const EngineModel* model, int32_t precision, int64_t batch,
                                                 size_t* out_packed_bytes, size_t* out_unpacked_bytes);
/* Per-launch CUDA-event timing of the plan for `batch` (enable != 0 turns it on).
 * engine_session_step_times waits for the recorded events and writes, per launch in
 * engine_model_plan_summary order, the total milliseconds accumulated since timing
 * was enabled (n_steps entries at most); returns the number of launches. */
ENGINE_API EngineStatus engine_session_step_timing(EngineSession* sess, int64_t batch, int32_t enable);
ENGINE_API int64_t      engine_session_step_times(EngineSession* sess, int64_t batch, double* out_ms, int64_t n_steps);
/* Number of kernel launches one engine_session_run_device call issues. */
ENGINE_API int64_t      engine_session_launch_count(const EngineSession* sess, int64_t batch);

/* C[M,N] = A[M,K] * B[K,N], row-major fp32 device pointers on the current device. */
ENGINE_API EngineStatus engine_gemm_f32_device(const float* d_a, const float* d_b, float* d_c,
                                               int64_t m, int64_t n, int64_t k,
                                               int32_t precision, void* stream);
/* engine_ops_matmul with an explicit precision (PdefaPrecision). */
ENGINE_API EngineStatus engine_ops_matmul_ex(const EngineTensor* a, const EngineTensor* b,
                                             EngineTensor* out, int32_t precision);

/* One kept detection; boxes are float64 exactly as the reference decode computes them. */
typedef struct {
    double  x1, y1, x2, y2;
    float   conf;
    int32_t cls;
    int32_t anchor;
    int32_t reserved;
} PdefaDetection;

/* Batched decode_yolo + class-wise NMS on the GPU.
 * preds: [batch, channels, anchors] fp32 (host pointer, or device pointer on
 * `device` when preds_on_device != 0). metas: NULL or `batch` letterbox records.
 * out_counts[batch] and out_dets[batch * max_det] are host arrays. */
ENGINE_API EngineStatus pdefa_decode_yolo(const float* preds, int32_t preds_on_device,
                                          int64_t batch, int64_t channels, int64_t anchors,
                                          const PdefaPreprocessMeta* metas,
                                          double conf_thres, double iou_thres, int32_t max_det,
                                          int32_t* out_counts, PdefaDetection* out_dets,
                                          int32_t device);

/* Device-side variant of pdefa_decode_yolo for callers that manage memory: all
 * pointers are device pointers on the current device (d_metas may be NULL), work is
 * caller-provided scratch of pdefa_decode_work_bytes(batch, anchors) bytes (16-byte
 * aligned, as cudaMalloc returns; d_dets 8-byte aligned, else ENGINE_ERR_INVALID_ARG),
 * and the call only enqueues one kernel on `stream` (no allocation, no
 * synchronisation). */
ENGINE_API size_t       pdefa_decode_work_bytes(int64_t batch, int64_t anchors);
ENGINE_API EngineStatus pdefa_decode_yolo_device(const float* d_preds, int64_t batch, int64_t channels,
                                                 int64_t anchors, const PdefaPreprocessMeta* d_metas,
                                                 double conf_thres, double iou_thres, int32_t max_det,
                                                 int32_t* d_counts, PdefaDetection* d_dets, void* d_work,
                                                 size_t work_bytes, void* stream);

/* Allocation-free decode. No counterpart in the reference (its decode is Python).
 * For callers that cannot allocate device memory when they decode (a caching
 * allocator they must not bypass, a server that forbids cudaMalloc after start-up,
 * a plugin host that only provides input/output buffers): same inputs, outputs and
 * results as pdefa_decode_yolo_device, but the candidate scratch is a built-in
 * 8 MiB device array per GPU (kept until the process exits), so at most
 * batch * anchors <= 174762 per call (e.g. 20 images of 8400 anchors); larger calls
 * fail with ENGINE_ERR_INVALID_ARG. The first call on a device looks up the array's
 * device address (make it before any stream capture). Calls share the array: calls
 * that overlap on the GPU (other streams, other threads) race and must be ordered
 * by the caller. The array used is the current device's: a non-NULL `stream` must
 * belong to the current device (ENGINE_ERR_INVALID_ARG otherwise). Allocates
 * nothing, no cudaMalloc or cudaFree. */
ENGINE_API EngineStatus pdefa_decode_yolo_noalloc(const float* d_preds, int64_t batch, int64_t channels,
                                                  int64_t anchors, const PdefaPreprocessMeta* d_metas,
                                                  double conf_thres, double iou_thres, int32_t max_det,
                                                  int32_t* d_counts, PdefaDetection* d_dets, void* stream);

/* Multi-GPU batch runner: one replica of `model` per device, contiguous shards, no
 * collective. Each device runs its shard's inference and decode and returns only
 * detections. */
typedef struct PdefaBatchRunner PdefaBatchRunner;
ENGINE_API EngineStatus pdefa_batch_create(EngineModel* model, int32_t n_devices,
                                           const int32_t* devices, int32_t precision,
                                           int64_t max_images_per_device,
                                           PdefaBatchRunner** out_runner);
/* images: [n_images, C, H, W] fp32 host array. */
ENGINE_API EngineStatus pdefa_batch_run(PdefaBatchRunner* runner, const float* images,
                                        int64_t n_images, const PdefaPreprocessMeta* metas,
                                        double conf_thres, double iou_thres, int32_t max_det,
                                        int32_t* out_counts, PdefaDetection* out_dets);
ENGINE_API void         pdefa_batch_destroy(PdefaBatchRunner* runner);

/* GPU letterbox preprocess for images already decoded to 8-bit pixels. Replaces the
 * host letterbox of pdefa_preprocess_letterbox (pdefa/src/pdefa_c_api.cpp:83-126 ->
 * imageloader/src/preprocess.cpp:15-147) with the same arithmetic: the float32 NCHW
 * output and the meta record are bit-identical to the reference's.
 * images: [n, src_h, src_w, channels] uint8, channels 1 (gray), 3 (RGB) or 4 (RGBA,
 * alpha dropped); out: [n, 3, cfg->target_h, cfg->target_w] float32. The n images
 * share one size, so one meta record describes them all. */
ENGINE_API EngineStatus pdefa_letterbox_meta(int32_t src_w, int32_t src_h, const PdefaPreprocessConfig* cfg,
                                             PdefaPreprocessMeta* out_meta);
/* Device pointers on the current device; enqueues on `stream`, no allocation. */
ENGINE_API EngineStatus pdefa_letterbox_device(const uint8_t* d_images, int64_t n, int32_t src_h, int32_t src_w,
                                               int32_t channels, const PdefaPreprocessConfig* cfg, float* d_out,
                                               void* stream);
/* Host arrays; runs on `device` and returns when `out` is written. */
ENGINE_API EngineStatus pdefa_letterbox(const uint8_t* images, int64_t n, int32_t src_h, int32_t src_w,
                                        int32_t channels, const PdefaPreprocessConfig* cfg, float* out,
                                        PdefaPreprocessMeta* out_meta, int32_t device);
/* pdefa_batch_run from 8-bit images: each GPU receives its shard's pixels (a quarter
 * of the float32 bytes for RGB), letterboxes them into the model input, runs
 * inference and decode, and returns detections in original-image coordinates (the
 * decode unmaps boxes with the letterbox meta, as decode_yolo(out, meta) does).
 * The model input must be [B, 3, cfg->target_h, cfg->target_w]. out_meta (may be
 * NULL) receives the shared meta record. RGB images already at the target size
 * (width a multiple of 4) on a BF16 runner skip the letterbox kernel: the stem conv
 * reads the 8-bit pixels and applies pixel * cfg->scale itself (the letterbox's
 * value for that geometry, bit for bit), when the stem is a 3x3 stride-2 conv and
 * the input's only consumer; otherwise the letterbox runs as above. */
ENGINE_API EngineStatus pdefa_batch_run_u8(PdefaBatchRunner* runner, const uint8_t* images, int64_t n_images,
                                           int32_t src_h, int32_t src_w, int32_t channels,
                                           const PdefaPreprocessConfig* cfg, double conf_thres, double iou_thres,
                                           int32_t max_det, int32_t* out_counts, PdefaDetection* out_dets,
                                           PdefaPreprocessMeta* out_meta);
/* Pipelined form of pdefa_batch_run_u8 (no counterpart in the reference, whose
 * BatchInference.run in pdefa/python/src/pdefa/batch.py:45-60 blocks per call). The
 * call returns once its copies, letterbox, inference and decode are queued, so the
 * next call's image copies overlap this call's last micro-batches. *out_ticket
 * numbers the call. Its results are in out_counts / out_dets once
 * pdefa_batch_wait(runner, ticket) returns, or once a later submit or run on the same
 * runner returns. Until then, images, out_counts and out_dets must stay allocated and
 * unchanged. out_meta is written before the call returns. pdefa_batch_destroy
 * drops results that are still pending. */
ENGINE_API EngineStatus pdefa_batch_submit_u8(PdefaBatchRunner* runner, const uint8_t* images, int64_t n_images,
                                              int32_t src_h, int32_t src_w, int32_t channels,
                                              const PdefaPreprocessConfig* cfg, double conf_thres,
                                              double iou_thres, int32_t max_det, int32_t* out_counts,
                                              PdefaDetection* out_dets, PdefaPreprocessMeta* out_meta,
                                              int64_t* out_ticket);
/* Completes every queued call up to and including `ticket` (all of them when
 * ticket <= 0): their results land in the arrays they were given. If a later call
 * failed on a device before an earlier call's pending micro-batches finished there,
 * those results are lost and the wait covering that earlier call returns
 * ENGINE_ERR_RUNTIME (once) instead of leaving its arrays silently unwritten. */
ENGINE_API EngineStatus pdefa_batch_wait(PdefaBatchRunner* runner, int64_t ticket);

#ifdef __cplusplus
}
#endif
#endif /* PDEFA_B200_EXT_H */
