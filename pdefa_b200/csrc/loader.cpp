// .engine v1/v2 reader and small shared utilities.
//
// File layout (PDEFA1.0/src/loader/custom_loader.cpp:62-214, writer
// pdefa/tools/onnx_to_engine.py:747-818): header (magic "ENGN", version, counts,
// 64-byte brand), weight table, nodes with their 128-byte OpParams, graph I/O
// indices, v2 tensor infos, then the weight data blob (offsets relative to its start).
#include <cstdio>
#include <mutex>

#include "common.h"

namespace pb {

namespace {
constexpr uint32_t kMagic = 0x4E474E45u;  // "ENGN"
constexpr int kMaxNdim = 8;               // PDEFA1.0/include/engine/shape.hpp:16

struct Reader {
    std::FILE* f;
    template <class T> void pod(T& v) {
        if (std::fread(&v, sizeof(T), 1, f) != 1) fail(ENGINE_ERR_INVALID_FORMAT, "truncated .engine file");
    }
    void bytes(void* p, size_t n) {
        if (n && std::fread(p, 1, n, f) != n) fail(ENGINE_ERR_INVALID_FORMAT, "truncated .engine file");
    }
    std::string str(uint32_t max_len = 4096) {
        uint32_t n = 0;
        pod(n);
        if (n > max_len) fail(ENGINE_ERR_INVALID_FORMAT, "name too long in .engine file");
        std::string s(n, '\0');
        bytes(s.data(), n);
        return s;
    }
};

size_t dtype_bytes_internal(uint8_t dt) {
    switch (dt) {
        case DT_BOOL: case DT_I8: case DT_U8: return 1;
        case DT_F16: case DT_BF16: return 2;
        case DT_I32: case DT_F32: return 4;
        case DT_I64: case DT_F64: return 8;
        default: return 4;
    }
}
}  // namespace

double Weight::value(int64_t i) const {
    switch (dtype) {
        case DT_F32: return reinterpret_cast<const float*>(bytes.data())[i];
        case DT_F64: return reinterpret_cast<const double*>(bytes.data())[i];
        case DT_I64: return (double)reinterpret_cast<const int64_t*>(bytes.data())[i];
        case DT_I32: return reinterpret_cast<const int32_t*>(bytes.data())[i];
        case DT_I8: return reinterpret_cast<const int8_t*>(bytes.data())[i];
        case DT_U8: case DT_BOOL: return bytes[i];
        default: return 0.0;
    }
}

std::shared_ptr<Graph> load_engine_file(const std::string& path) {
    std::FILE* f = std::fopen(path.c_str(), "rb");
    if (!f) fail(ENGINE_ERR_INVALID_FORMAT, "failed to load model file");
    struct Closer { std::FILE* f; ~Closer() { std::fclose(f); } } closer{f};
    Reader r{f};
    uint32_t magic = 0, version = 0, nw = 0, nn = 0, ni = 0, no = 0;
    r.pod(magic); r.pod(version);
    if (magic != kMagic || (version != 1 && version != 2))
        fail(ENGINE_ERR_INVALID_FORMAT, "failed to load model file");
    r.pod(nw); r.pod(nn); r.pod(ni); r.pod(no);
    char brand[64];
    r.bytes(brand, sizeof brand);

    auto g = std::make_shared<Graph>();
    g->name = path;
    struct WMeta { uint64_t off, size; };
    std::vector<WMeta> wm(nw);
    g->weights.resize(nw);
    for (uint32_t i = 0; i < nw; ++i) {
        Weight& w = g->weights[i];
        w.name = r.str();
        uint8_t rank = 0;
        r.pod(w.dtype); r.pod(rank);
        if (rank > kMaxNdim) fail(ENGINE_ERR_INVALID_FORMAT, "weight rank > 8");
        w.shape.resize(rank);
        for (auto& d : w.shape) r.pod(d);
        r.pod(wm[i].off); r.pod(wm[i].size);
    }
    g->nodes.resize(nn);
    for (uint32_t i = 0; i < nn; ++i) {
        Node& n = g->nodes[i];
        uint8_t op = 0;
        r.pod(op);
        n.op = static_cast<Op>(op);
        n.name = r.str();
        uint16_t nin = 0, nout = 0;
        r.pod(nin); r.pod(nout);
        if (nin > 64 || nout > 64) fail(ENGINE_ERR_INVALID_FORMAT, "node arity > 64");
        n.inputs.resize(nin); n.outputs.resize(nout);
        for (auto& v : n.inputs) r.pod(v);
        for (auto& v : n.outputs) r.pod(v);
        r.bytes(&n.params, sizeof(OpParams));
    }
    g->inputs.resize(ni); g->outputs.resize(no);
    for (auto& v : g->inputs) r.pod(v);
    for (auto& v : g->outputs) r.pod(v);
    if (version >= 2) {
        auto info = [&](TensorInfo& t) {
            t.name = r.str();
            uint8_t nd = 0;
            r.pod(nd);
            if (nd > kMaxNdim) fail(ENGINE_ERR_INVALID_FORMAT, "tensor info rank > 8");
            t.shape.resize(nd);
            for (auto& d : t.shape) r.pod(d);
            r.pod(t.dtype);
        };
        g->input_infos.resize(ni); g->output_infos.resize(no);
        for (auto& t : g->input_infos) info(t);
        for (auto& t : g->output_infos) info(t);
    }
    const long base = std::ftell(f);
    for (uint32_t i = 0; i < nw; ++i) {
        Weight& w = g->weights[i];
        const size_t expect = (size_t)w.numel() * dtype_bytes_internal(w.dtype);
        if (wm[i].size < expect) fail(ENGINE_ERR_INVALID_FORMAT, "weight blob smaller than its shape");
        if (std::fseek(f, base + (long)wm[i].off, SEEK_SET) != 0)
            fail(ENGINE_ERR_INVALID_FORMAT, "bad weight offset");
        w.bytes.resize(expect);
        r.bytes(w.bytes.data(), expect);
    }
    return g;
}

size_t engine_dtype_bytes(EngineDType dt) {
    switch (dt) {
        case ENGINE_F32: case ENGINE_I32: return 4;
        case ENGINE_F16: case ENGINE_BF16: return 2;
        case ENGINE_I8: case ENGINE_U8: case ENGINE_BOOL: return 1;
        case ENGINE_I64: return 8;
    }
    return 0;
}

const char* op_name(Op op) {
    switch (op) {
        case Op::Conv2d: return "Conv2d"; case Op::MatMul: return "MatMul";
        case Op::Add: return "Add"; case Op::Mul: return "Mul"; case Op::Sub: return "Sub";
        case Op::Div: return "Div"; case Op::ReLU: return "ReLU"; case Op::LeakyReLU: return "LeakyReLU";
        case Op::Sigmoid: return "Sigmoid"; case Op::Tanh: return "Tanh"; case Op::SiLU: return "SiLU";
        case Op::GELU: return "GELU"; case Op::HardSwish: return "HardSwish";
        case Op::HardSigmoid: return "HardSigmoid"; case Op::MaxPool2d: return "MaxPool2d";
        case Op::AvgPool2d: return "AvgPool2d"; case Op::BatchNorm2d: return "BatchNorm2d";
        case Op::Softmax: return "Softmax"; case Op::Concat: return "Concat";
        case Op::Upsample: return "Upsample"; case Op::Resize: return "Resize";
        case Op::Reshape: return "Reshape"; case Op::Transpose: return "Transpose";
        case Op::Slice: return "Slice"; case Op::Gather: return "Gather"; case Op::Shape: return "Shape";
        case Op::Clip: return "Clip"; case Op::Input: return "Input"; case Op::Output: return "Output";
        default: return "Unknown";
    }
}

// ---------------------------------------------------------------------------
// Devices and the sticky error word used by bounded device-side waits.
// ---------------------------------------------------------------------------
int device_count() {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) { cudaGetLastError(); return 0; }
    return n;
}

void require_device(int device) {
    const int n = device_count();
    if (n == 0) fail(ENGINE_ERR_RUNTIME, "no CUDA device available: this engine runs on the GPU only");
    if (device < 0 || device >= n) fail(ENGINE_ERR_INVALID_ARG, "CUDA device index out of range");
}

namespace {
std::mutex g_err_mu;
int* g_err_words[64] = {};
}

int* device_error_word(int device) {
    std::lock_guard<std::mutex> lk(g_err_mu);
    if (device < 0 || device >= 64) fail(ENGINE_ERR_INVALID_ARG, "device index out of range");
    if (!g_err_words[device]) {
        int prev = 0;
        PB_CUDA(cudaGetDevice(&prev));
        PB_CUDA(cudaSetDevice(device));
        int* p = nullptr;
        PB_CUDA(cudaMalloc(&p, sizeof(int)));
        PB_CUDA(cudaMemset(p, 0, sizeof(int)));
        PB_CUDA(cudaSetDevice(prev));
        g_err_words[device] = p;
    }
    return g_err_words[device];
}

int read_device_error(int device) {
    // Reports a timeout once: the word is cleared after it has been read.
    int* p = device_error_word(device);
    int v = 0;
    PB_CUDA(cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost));
    if (v) PB_CUDA(cudaMemset(p, 0, sizeof(int)));
    return v;
}

}  // namespace pb
