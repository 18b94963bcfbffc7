// Shared definitions for the B200 engine: status/error plumbing, CUDA checks,
// the graph IR (same on-disk meaning as the reference .engine format) and small
// utilities. Host-only header (no device code).
#pragma once

#include <cstdint>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "../../include/engine_c_api.h"

namespace pb {

// Exception carrying an EngineStatus; converted to a status code at the C ABI.
struct Error : std::runtime_error {
    EngineStatus status;
    Error(EngineStatus s, const std::string& m) : std::runtime_error(m), status(s) {}
};

[[noreturn]] inline void fail(EngineStatus s, const std::string& m) { throw Error(s, m); }

#define PB_CUDA(call)                                                                   \
    do {                                                                                \
        cudaError_t _e = (call);                                                        \
        if (_e != cudaSuccess)                                                          \
            ::pb::fail(ENGINE_ERR_RUNTIME, std::string("CUDA error: ") +               \
                       cudaGetErrorString(_e) + " at " + __FILE__ + ":" +               \
                       std::to_string(__LINE__));                                       \
    } while (0)

// ---------------------------------------------------------------------------
// Graph IR. Op ids: PDEFA1.0/include/engine/graph.hpp:20-75.
// ---------------------------------------------------------------------------
enum class Op : uint8_t {
    Unknown = 0, Conv2d = 1, MatMul = 2, Add = 3, Mul = 4, Sub = 5, Div = 6,
    ReLU = 10, LeakyReLU = 11, Sigmoid = 12, Tanh = 13, SiLU = 14, GELU = 15,
    HardSwish = 16, HardSigmoid = 17,
    MaxPool2d = 20, AvgPool2d = 21, BatchNorm2d = 22, LayerNorm = 23,
    Softmax = 30, Concat = 31, Upsample = 32, Resize = 33, Input = 40, Output = 41,
    Reshape = 42, Transpose = 43, Slice = 44, Gather = 45, Shape = 46, Expand = 47,
    Unsqueeze = 48, Squeeze = 49, TopK = 50, GatherElements = 51, Mod = 52,
    ReduceMax = 53, ReduceMin = 54, ReduceProd = 55, NonZero = 56, ConstantOfShape = 57,
    Tile = 58, Range = 59, Equal = 60, Greater = 61, Exp = 62, Min = 63, Max = 64,
    ReduceSum = 65, Clip = 66, ArgMax = 67, Stack = 68,
};
const char* op_name(Op op);

// The 128-byte parameter record stored per node (graph.hpp:77-94, natural alignment).
struct OpParams {
    int64_t stride_h = 1, stride_w = 1;
    int64_t pad_h = 0, pad_w = 0;
    int64_t dil_h = 1, dil_w = 1;
    int64_t groups = 1;
    int64_t kernel_h = 2, kernel_w = 2;
    int32_t axis = -1;
    int32_t pad0_ = 0;
    int64_t scale_h = 2, scale_w = 2;
    int64_t target_h = 0, target_w = 0;
    uint8_t upsample_mode = 0;
    uint8_t pad1_[3] = {0, 0, 0};
    float eps = 1e-5f;
    uint8_t fused_activation = 0;
    uint8_t pad2_[3] = {0, 0, 0};
    float leaky_slope = 0.01f;
};
static_assert(sizeof(OpParams) == 128, "OpParams must match the on-disk record");

struct Node {
    Op op = Op::Unknown;
    std::string name;
    std::vector<int32_t> inputs, outputs;
    OpParams params;
};

// Internal dtype codes as stored in .engine (PDEFA1.0/include/engine/dtype.hpp:36-60).
enum : uint8_t { DT_BOOL = 1, DT_I8 = 2, DT_U8 = 3, DT_I32 = 6, DT_I64 = 8,
                 DT_F16 = 10, DT_BF16 = 11, DT_F32 = 12, DT_F64 = 13 };

struct Weight {
    std::string name;
    uint8_t dtype = DT_F32;
    std::vector<int64_t> shape;
    std::vector<uint8_t> bytes;
    int64_t numel() const { int64_t n = 1; for (auto d : shape) n *= d; return n; }
    double value(int64_t i) const;          // element i widened to double
    const float* f32() const { return dtype == DT_F32 ? reinterpret_cast<const float*>(bytes.data()) : nullptr; }
};

struct TensorInfo {
    std::string name;
    std::vector<int64_t> shape;
    uint8_t dtype = DT_F32;
};

struct Graph {
    std::string name;
    std::vector<Weight> weights;
    std::vector<Node> nodes;
    std::vector<int32_t> inputs, outputs;
    std::vector<TensorInfo> input_infos, output_infos;
};

// Parses a .engine v1/v2 file (layout of PDEFA1.0/src/loader/custom_loader.cpp:62-214).
std::shared_ptr<Graph> load_engine_file(const std::string& path);

// EngineDType <-> byte size.
size_t engine_dtype_bytes(EngineDType dt);

// Device helpers.
int device_count();
void require_device(int device);            // throws if no usable CUDA device
int* device_error_word(int device);         // sticky error word for bounded waits
int read_device_error(int device);

}  // namespace pb
