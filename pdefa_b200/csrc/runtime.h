// Runtime objects behind the C ABI handles: tensors with a host mirror and a
// device copy, contexts, models and sessions.
#pragma once

#include <chrono>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "common.h"
#include "graph_plan.h"

namespace pb {

// Handle magics (same scheme as PDEFA1.0/src/api/engine_api.cpp:36-39).
constexpr uint32_t kMagicContext = 0xE0C0DE01u;
constexpr uint32_t kMagicModel = 0xE0C0DE02u;
constexpr uint32_t kMagicSession = 0xE0C0DE03u;
constexpr uint32_t kMagicTensor = 0xE0C0DE04u;

// Tensor storage: host memory is always present (engine_tensor_data returns a
// host pointer that Python reads directly); a device copy is attached when a
// session produces or consumes the tensor. Exactly one side is authoritative
// when they differ.
struct TensorStore {
    std::vector<int64_t> shape;
    EngineDType dtype = ENGINE_F32;
    size_t nbytes = 0;
    void* host = nullptr;
    bool pinned = false;
    const void* dev = nullptr;   // device data (not owned; session output buffers)
    int dev_id = -1;
    cudaStream_t dev_stream = nullptr;
    bool host_valid = true;
    std::mutex mu;

    TensorStore(std::vector<int64_t> s, EngineDType dt);
    ~TensorStore();
    int64_t numel() const;
    void sync_to_host();              // makes host authoritative
};

}  // namespace pb

struct EngineTensor {
    uint32_t magic = pb::kMagicTensor;
    std::shared_ptr<pb::TensorStore> owned;
    pb::TensorStore* borrowed = nullptr;
    pb::TensorStore* ptr() const { return owned ? owned.get() : borrowed; }
    bool is_borrowed() const { return !owned && borrowed != nullptr; }
};

struct EngineContext {
    uint32_t magic = pb::kMagicContext;
    int32_t num_threads = 1;
    int32_t precision = pb::PREC_FP32;
    int32_t device = 0;
};

struct EngineModel {
    uint32_t magic = pb::kMagicModel;
    std::shared_ptr<pb::Graph> graph;
};

struct EngineSession {
    uint32_t magic = pb::kMagicSession;
    std::shared_ptr<const pb::Graph> graph;
    int device = 0;
    int precision = pb::PREC_FP32;
    cudaStream_t stream = nullptr;
    std::vector<const EngineTensor*> inputs;
    // by (batch, input 0 shape of one image; empty = the model's declared shape)
    std::map<std::pair<int64_t, std::vector<int64_t>>, std::unique_ptr<pb::Plan>> plans;
    pb::Plan* last = nullptr;
    std::vector<std::shared_ptr<pb::TensorStore>> outputs;
    std::vector<EngineTensor> out_handles;
    double last_run_ms = 0.0;
    uint64_t runs = 0;
    EngineProfileFn profile_fn = nullptr;
    void* profile_user = nullptr;
    std::mutex mu;
    // intermediates: indices kept readable after a run (besides the unconsumed
    // ones), and the host tensors engine_session_debug_intermediate hands out
    std::vector<int32_t> keep;
    struct Debug {
        std::shared_ptr<pb::TensorStore> store;
        EngineTensor handle;
    };
    std::map<int32_t, Debug> debug_out;
    void* debug_buf = nullptr;       // dense fp32 staging on the device
    size_t debug_cap = 0;

    pb::Plan& plan_for(int64_t batch, const std::vector<int64_t>& in_shape = {});
    void run();
};

namespace pb {
void set_error(const std::string& m);
void clear_error();
// Runs fn, converting exceptions into status codes and the thread-local error text.
template <class Fn>
EngineStatus guarded(Fn&& fn) noexcept {
    try {
        return fn();
    } catch (const Error& e) {
        set_error(e.what());
        return e.status;
    } catch (const std::bad_alloc&) {
        set_error("out of memory");
        return ENGINE_ERR_OUT_OF_MEMORY;
    } catch (const std::exception& e) {
        set_error(e.what());
        return ENGINE_ERR_RUNTIME;
    } catch (...) {
        set_error("unknown exception");
        return ENGINE_ERR_UNKNOWN;
    }
}
int default_device();
}  // namespace pb
