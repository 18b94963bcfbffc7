// Lowering of a .engine graph into a fixed sequence of GPU launches for a given
// batch size and precision ("plan"), and its execution on a CUDA stream.
//
// Semantics follow the reference CPU interpreter (PDEFA1.0/src/core/session.cpp
// and session_parts/*.inc): rank-4 activations are NHWC ("motor" shapes), ONNX axes
// are remapped exactly as the reference does, conv+activation fusion uses the
// reference's rule, and a batch of B images computes B independent batch-1 passes.
#pragma once

#include <functional>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "common.h"
#include "kernels.h"

namespace pb {

enum Precision : int { PREC_FP32 = 0, PREC_TF32 = 1, PREC_BF16 = 2 };

// Physical description of one graph value for the whole batch.
struct Value {
    std::vector<int64_t> shape;      // per-image motor shape (as the reference sees it at N = 1)
    std::vector<int64_t> stride;     // per-image strides, elements
    int64_t img_stride = 0;          // elements between images (0 = shared across images)
    int dt = F32;
    int buf = -1;                    // owning buffer (after allocation)
    int64_t off = 0;                 // element offset inside the buffer
    bool known = false;              // shape inferred
    // placement (decided before allocation)
    int alias_of = -1;               // value id this one views (slice / reshape views)
    int64_t alias_off = 0;           // element offset added to the aliased value's offset
    int place_in = -1;               // concat value this one is stored inside
    int64_t place_ch = 0;            // channel offset inside that concat
    bool dense_required = false;
    int weight = -1;                 // weight index when this value is a constant
    bool external = false;           // graph input
    int producer = -1;               // node index
};

struct PlanStep {
    std::string name;
    std::function<void(cudaStream_t)> run;
    int launches = 1;
    std::string kind;                // kernel family, for plan summaries
};

// PDEFA_VERBOSE set (and not "0"): lowering and runner decisions are printed to stderr.
bool verbose();

class Plan {
public:
    // keep: engine tensor indices whose values stay readable after a run (see
    // debug_view); values no node consumes are always kept, as in the reference.
    // in_shape: shape of one image of input 0 when it differs from the declared one
    // (empty: the declared shape).
    // in_u8_scale > 0: input 0 is given as 8-bit RGB frames [batch, H, W, 3] at the model
    // size, read by the stem conv as pixel * in_u8_scale (the identity letterbox, fused);
    // lowering fails unless the stem is input 0's only consumer.
    Plan(std::shared_ptr<const Graph> g, int64_t batch, int precision, int device,
         std::vector<int32_t> keep = {}, std::vector<int64_t> in_shape = {}, float in_u8_scale = 0.0f);
    // Device-free lowering: every pass runs and every launch is recorded, but nothing
    // is allocated or copied (addresses are placeholders). Used to validate a model
    // and to inspect its launch list without a GPU.
    static std::unique_ptr<Plan> dry_run(std::shared_ptr<const Graph> g, int64_t batch, int precision);
    // One line per launch: "<kind> <name>".
    std::string summary() const;
    ~Plan();
    Plan(const Plan&) = delete;
    Plan& operator=(const Plan&) = delete;

    // Input i: device buffer the caller fills with [batch, C, H, W] (NCHW fp32) data.
    float* input_buffer(int i) const { return inputs_.at(i); }
    size_t input_bytes(int i) const { return input_bytes_.at(i); }
    // > 0: input 0 holds 8-bit RGB frames [batch, H, W, 3] read as pixel * u8_scale()
    float u8_scale() const { return u8_scale_; }
    // Output i: dense fp32 device buffer in the reference's output layout.
    float* output_buffer(int i) const { return outputs_.at(i); }
    const std::vector<int64_t>& output_shape(int i) const { return out_shapes_.at(i); }
    size_t output_bytes(int i) const { return out_bytes_.at(i); }
    int num_outputs() const { return (int)outputs_.size(); }

    // Enqueue all steps on `s` (optionally redirecting input/output buffers).
    void run(cudaStream_t s, const float* in_override = nullptr, float* out_override = nullptr);
    const std::vector<PlanStep>& steps() const { return steps_; }
    int64_t launch_count() const;
    // Per-step CUDA-event timing: while enabled, run() brackets every step with
    // events on the launching stream; collect_step_ms() waits for them and adds the
    // elapsed times to per-step totals (one entry per step, summary() order).
    void set_step_timing(bool on) { timing_ = on; }
    std::vector<double> collect_step_ms();
    int64_t batch() const { return batch_; }
    // After the stream of the last run() was synchronized: the error code its kernels
    // recorded (0: none); the word is cleared, so the next run starts clean.
    int take_error();
    // Enqueues the copy of the error word to the host (Plan::run does it after its
    // launches; callers that launch the steps themselves call it).
    void enqueue_error_copy(cudaStream_t s);
    // Device bytes of the activations: packed in the arena, and what one buffer per
    // value would take.
    size_t activation_bytes() const { return activation_bytes_; }
    size_t unpacked_activation_bytes() const { return unpacked_bytes_; }
    const std::vector<size_t>& root_bytes() const { return root_bytes_; }
    const std::vector<int>& root_first() const { return root_first_; }
    const std::vector<int>& root_last() const { return root_last_; }
    // Device view of intermediate tensor `idx` after a run: values no node consumes
    // (PDEFA1.0/src/core/session.cpp:322-337 frees every other intermediate once its
    // last consumer ran) and the indices passed as `keep`. nullptr if not kept.
    const TView* debug_view(int32_t idx) const {
        auto it = debug_.find(idx);
        return it == debug_.end() ? nullptr : &it->second;
    }
    int precision() const { return prec_; }
    int device() const { return device_; }

private:
    void build();
    void* alloc(size_t bytes);

    struct DryTag {};
    Plan(DryTag, std::shared_ptr<const Graph> g, int64_t batch, int precision, std::vector<int32_t> keep = {},
         std::vector<int64_t> in_shape = {}, float in_u8_scale = 0.0f);
    std::vector<int32_t> keep_;
    std::vector<int64_t> in_shape_;
    float u8_scale_ = 0.0f;
    std::map<int32_t, TView> debug_;
    std::shared_ptr<const Graph> g_;
    bool dry_ = false;
    uintptr_t dry_next_ = 0x10000000;
    int64_t batch_;
    int prec_;
    int device_;
    std::vector<void*> allocs_;
    std::vector<float*> inputs_;
    std::vector<size_t> input_bytes_;
    std::vector<float*> outputs_;
    std::vector<size_t> out_bytes_;
    std::vector<std::vector<int64_t>> out_shapes_;
    std::vector<PlanStep> steps_;
    bool timing_ = false;
    // CUDA graph of the launch sequence: captured on the second untimed run (the
    // first, eager one makes every lazy allocation and attribute call) and replayed
    // while the input buffer stays the same.
    bool graphs_ = true;
    int eager_runs_ = 0;
    cudaGraphExec_t gexec_ = nullptr;
    const float* g_in_ = nullptr;
    void run_steps(cudaStream_t s);
    void run_launches(cudaStream_t s, const float* in_override);
    std::vector<cudaEvent_t> ev_pool_;
    std::vector<std::pair<int, std::pair<cudaEvent_t, cudaEvent_t>>> pending_;
    std::vector<double> step_ms_;
    cudaEvent_t take_event();
    const float* cur_in_ = nullptr;   // overrides valid during run()
    float* cur_out_ = nullptr;
    // memory plan: per value id, bytes of an arena root (0: not a root) and the range
    // of node indices that touch it (filled by every lowering)
    std::vector<size_t> root_bytes_;
    std::vector<int> root_first_, root_last_;
    size_t activation_bytes_ = 0, unpacked_bytes_ = 0;
    // Error word of this plan's kernels (a bounded wait that ran out records a code and
    // the plan's later CTAs skip their work), copied to pinned host memory at the end
    // of every run, so one plan's timeout never blanks another plan's work.
    int* err_ = nullptr;
    int* err_host_ = nullptr;
    long long wait_limit_ = 0;   // PDEFA_WAIT_LIMIT_CYCLES at lowering (0: kernel default)
    friend struct PlanBuilder;
};

// Arena offsets (bytes) of the activation roots: largest first, each at the lowest
// aligned offset free of every placed root whose node range intersects its own;
// SIZE_MAX for values that are not roots. *total: arena size.
std::vector<size_t> pack_arena(const std::vector<size_t>& bytes, const std::vector<int>& first,
                               const std::vector<int>& last, size_t* total);

// Kernel the reference dispatcher picks for a batch-1 NHWC conv
// (PDEFA1.0/src/ops/conv2d.cpp:602-642): 0 direct (Cin <= 16, not pure 1x1),
// 1 Winograd F(2,3) (3x3 s1 d1, Cin <= 512), 2 GEMM. Decides the SiLU flavour.
int reference_conv_path(int64_t cin, int64_t kh, int64_t kw, const OpParams& p);

}  // namespace pb
