// Graph lowering: reference shape semantics -> fusion -> placement -> launches.
//
// Passes:
//  1. activation fusion with the reference rule (session_fusion.inc:10-109);
//  2. shape inference with the reference's NHWC rules (session_ops_*.inc);
//  3. YOLOv8 Detect-tail match (replaced by one fused head kernel);
//  4. residual fusion: Add(x, conv(...)) becomes the conv's epilogue;
//  5. placement: channel slices become views, rank-4 channel concats become
//     zero-copy (producers write straight into their channel slice);
//  6. allocation and emission of one closure per launch.
#include "graph_plan.h"

#include <climits>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <map>
#include <unordered_map>

namespace pb {

int reference_conv_path(int64_t cin, int64_t kh, int64_t kw, const OpParams& p) {
    const bool pure_1x1 = kh == 1 && kw == 1 && p.pad_h == 0 && p.pad_w == 0 && p.stride_h == 1 &&
                          p.stride_w == 1 && p.dil_h == 1 && p.dil_w == 1;
    const int64_t groups = p.groups > 0 ? p.groups : 1;
    if (!pure_1x1 && cin <= 16 && groups == 1 && kh <= 7 && kw <= 7) return 0;
    if (kh == 3 && kw == 3 && p.stride_h == 1 && p.stride_w == 1 && p.dil_h == 1 && p.dil_w == 1 &&
        groups == 1 && cin <= 512)
        return 1;
    return 2;
}

bool verbose() {
    static int v = -1;
    if (v < 0) { const char* e = std::getenv("PDEFA_VERBOSE"); v = (e && *e && *e != '0') ? 1 : 0; }
    return v == 1;
}

namespace {

int64_t numel_of(const std::vector<int64_t>& s) {
    int64_t n = 1;
    for (auto d : s) n *= d;
    return n;
}

std::vector<int64_t> dense_strides(const std::vector<int64_t>& s) {
    std::vector<int64_t> st(s.size(), 1);
    for (int d = (int)s.size() - 2; d >= 0; --d) st[d] = st[d + 1] * s[d + 1];
    return st;
}

uint16_t f2bf(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x7FFFFFu)) return 0x7FC0;
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

std::string shape_str(const std::vector<int64_t>& s) {
    std::string r = "[";
    for (size_t i = 0; i < s.size(); ++i) r += (i ? "," : "") + std::to_string(s[i]);
    return r + "]";
}

}  // namespace

struct PlanBuilder {
    Plan& P;
    const Graph& g;
    int64_t B;
    int prec;
    int act_dt;
    std::vector<Node> nodes;            // working copy (fusion rewrites outputs)
    std::vector<char> skip;
    std::vector<int> conv_act;          // fused activation code per node
    std::vector<float> conv_slope;
    std::vector<int> conv_res;          // residual value id per conv node
    std::vector<Value> V;
    std::unordered_map<int32_t, int> vid;
    std::unordered_map<int32_t, int> consumers;
    std::vector<int> out_vids;
    // head
    bool head = false;
    int head_at = -1;                   // node index where the head step is emitted
    int head_out = -1;
    int head_levels[3] = {-1, -1, -1};
    int head_anchor_w = -1, head_stride_w = -1, head_dfl_w = -1, head_reg = 16, head_nc = 80;
    // per-node lowering notes
    struct Note {
        int mode = 0;
        std::vector<int64_t> a, b, c;   // mode-specific integer payloads
        bool dfl_fix = false;
        float scale = 1.0f;             // MatMul mode 2: scalar Mul folded into the product
    };
    std::unordered_map<int, int> folded_transpose;   // value read through permuted strides -> Transpose node
    std::vector<Note> note;
    std::unordered_map<int, void*> wdev;        // weight index -> device fp32 copy

    PlanBuilder(Plan& p, const Graph& graph)
        : P(p), g(graph), B(p.batch_), prec(p.prec_), act_dt(p.prec_ == PREC_BF16 ? BF16 : F32) {}

    // -------------------------------------------------------------------
    int new_value() { V.emplace_back(); return (int)V.size() - 1; }

    int value_for(int32_t idx) {
        auto it = vid.find(idx);
        if (it != vid.end()) return it->second;
        const int v = new_value();
        vid[idx] = v;
        if (idx <= -1000) {
            const int w = -idx - 1000;
            if (w >= (int)g.weights.size()) fail(ENGINE_ERR_INVALID_FORMAT, "weight index out of range");
            V[v].weight = w;
            V[v].shape = g.weights[w].shape;
            V[v].known = true;
        }
        return v;
    }

    int input_vid(const Node& n, size_t k) {
        int32_t idx = n.inputs[k];
        if (!n.outputs.empty() && idx == n.outputs[0] && idx > 0) idx -= 1;  // session.cpp:396-399
        const int v = value_for(idx);
        if (!V[v].known) fail(ENGINE_ERR_RUNTIME, "node '" + n.name + "' reads a value that is not produced");
        return v;
    }

    const Weight& wt(int v) {
        if (V[v].weight < 0) fail(ENGINE_ERR_NOT_IMPL, "shape/index tensor computed at run time is not supported");
        return g.weights[V[v].weight];
    }
    int64_t get_int(int v, int64_t i) {   // session_helpers.inc: get_tensor_int (float truncates)
        const Weight& w = wt(v);
        if (i < 0 || i >= w.numel()) return 0;
        return (int64_t)w.value(i);
    }
    double get_float(int v, int64_t i) {
        const Weight& w = wt(v);
        if (i < 0 || i >= w.numel()) return 0.0;
        return w.value(i);
    }

    // -------------------------------------------------------------------
    // 1. fusion (session_fusion.inc:10-109)
    void fuse() {
        nodes = g.nodes;
        skip.assign(nodes.size(), 0);
        conv_act.assign(nodes.size(), 0);
        conv_slope.assign(nodes.size(), 0.01f);
        conv_res.assign(nodes.size(), -1);
        auto count_consumers = [&](int32_t t, size_t self) {
            int c = 0;
            for (size_t k = 0; k < nodes.size(); ++k) {
                if (k == self) continue;
                for (int32_t in : nodes[k].inputs) c += in == t;
            }
            for (int32_t o : g.outputs) c += o == t;
            return c;
        };
        for (size_t i = 0; i < nodes.size(); ++i) {
            Node& conv = nodes[i];
            if (conv.op != Op::Conv2d || conv.outputs.empty() || conv.outputs[0] < 0) continue;
            const int32_t co = conv.outputs[0];
            const int cc = count_consumers(co, i);
            if (cc == 2) {
                int sig = -1, mul = -1;
                for (size_t j = i + 1; j < nodes.size(); ++j) {
                    if (nodes[j].op == Op::Sigmoid && nodes[j].inputs.size() == 1 && nodes[j].inputs[0] == co) {
                        if (nodes[j].outputs.empty() || nodes[j].outputs[0] < 0) break;
                        if (count_consumers(nodes[j].outputs[0], j) != 1) break;
                        sig = (int)j;
                        break;
                    }
                }
                if (sig >= 0) {
                    const int32_t so = nodes[sig].outputs[0];
                    for (size_t j = i + 1; j < nodes.size(); ++j) {
                        const Node& m = nodes[j];
                        if (m.op == Op::Mul && m.inputs.size() == 2 &&
                            ((m.inputs[0] == co && m.inputs[1] == so) || (m.inputs[1] == co && m.inputs[0] == so))) {
                            mul = (int)j;
                            break;
                        }
                    }
                }
                if (sig >= 0 && mul >= 0) {
                    conv_act[i] = ACT_SILU;
                    conv.outputs[0] = nodes[mul].outputs[0];
                    nodes[sig].op = Op::Input;
                    nodes[mul].op = Op::Input;
                    continue;
                }
            }
            if (cc != 1) continue;
            for (size_t j = i + 1; j < nodes.size(); ++j) {
                Node& a = nodes[j];
                if (a.inputs.size() == 1 && a.inputs[0] == co &&
                    (a.op == Op::ReLU || a.op == Op::LeakyReLU || a.op == Op::Sigmoid || a.op == Op::Tanh)) {
                    conv_act[i] = a.op == Op::ReLU ? ACT_RELU : a.op == Op::LeakyReLU ? ACT_LEAKY
                                : a.op == Op::Sigmoid ? ACT_SIGMOID : ACT_GELU_TANH;
                    if (a.op == Op::Tanh) conv_act[i] = 100;  // tanh: unary after conv (see emit)
                    conv_slope[i] = a.params.leaky_slope;
                    conv.outputs[0] = a.outputs[0];
                    a.op = Op::Input;
                    break;
                }
            }
        }
        for (size_t i = 0; i < nodes.size(); ++i)
            if (nodes[i].op == Op::Input || nodes[i].op == Op::Output) skip[i] = 1;
        consumers.clear();
        for (size_t i = 0; i < nodes.size(); ++i) {
            if (skip[i]) continue;
            for (int32_t in : nodes[i].inputs) consumers[in]++;
        }
        for (int32_t o : g.outputs) consumers[o]++;
    }

    // -------------------------------------------------------------------
    // 2. shapes
    void set_out(const Node& n, int k, std::vector<int64_t> shape, int dt, int node_idx) {
        const int v = value_for(n.outputs[k]);
        V[v].shape = std::move(shape);
        V[v].dt = dt;
        V[v].known = true;
        V[v].producer = node_idx;
    }

    int dt_for(const std::vector<int64_t>& shape) const { return shape.size() == 4 ? act_dt : F32; }

    void infer() {
        note.assign(nodes.size(), Note{});
        // external inputs: rank-4 F32 become NHWC motor views of the NCHW buffer (session.cpp:199-215)
        for (size_t i = 0; i < g.inputs.size(); ++i) {
            const int v = value_for(g.inputs[i]);
            Value& x = V[v];
            x.external = true;
            x.known = true;
            x.dt = F32;
            std::vector<int64_t> s = i < g.input_infos.size() ? g.input_infos[i].shape : std::vector<int64_t>{};
            if (i == 0 && !P.in_shape_.empty()) s = P.in_shape_;
            if (s.empty()) fail(ENGINE_ERR_INVALID_FORMAT, "model has no input shape information (v1 file)");
            for (auto& d : s) if (d <= 0) d = 1;
            s[0] = 1;
            x.shape = s.size() == 4 ? std::vector<int64_t>{1, s[2], s[3], s[1]} : s;
        }
        for (size_t i = 0; i < nodes.size(); ++i) {
            if (skip[i]) continue;
            infer_node((int)i);
        }
    }

    void infer_node(int ni) {
        const Node& n = nodes[ni];
        Note& nt = note[ni];
        const size_t nin = n.inputs.size();
        auto need = [&](size_t k) { if (nin < k) fail(ENGINE_ERR_INVALID_FORMAT, "node '" + n.name + "' has too few inputs"); };
        if (n.outputs.empty()) return;
        switch (n.op) {
        case Op::Conv2d: {
            need(2);
            const int x = input_vid(n, 0), w = input_vid(n, 1);
            auto is = V[x].shape;
            const auto ws = V[w].shape;
            if (is.size() != 4 || ws.size() != 4) fail(ENGINE_ERR_INVALID_SHAPE, "conv '" + n.name + "': rank != 4");
            const int64_t ci_w = ws[1];
            if (is[3] != ci_w && is[2] == ci_w) {   // session_ops_nn.inc:10-33
                nt.dfl_fix = true;
                std::swap(is[2], is[3]);
            }
            const int64_t groups = n.params.groups > 0 ? n.params.groups : 1;
            if (ws[2] == 1 && ws[3] == 1 && groups == 1 && is[1] == ci_w && ci_w != is[3]) {
                nt.mode = 1;   // channel-major 1x1 (conv2d.cpp:464-468, 518-571)
                set_out(n, 0, {is[0], ws[0], is[2], is[3]}, F32, ni);
                return;
            }
            if (groups != 1 && (is[3] != ci_w * groups || ws[0] % groups))
                fail(ENGINE_ERR_INVALID_SHAPE, "conv '" + n.name + "': channels do not match the groups");
            if (groups == 1 && is[3] != ci_w) fail(ENGINE_ERR_INVALID_SHAPE, "conv '" + n.name + "': channel mismatch");
            auto osz = [](int64_t in, int64_t k, int64_t s, int64_t p, int64_t d) {
                return (in + 2 * p - ((k - 1) * d + 1)) / s + 1;
            };
            const int64_t ho = osz(is[1], ws[2], n.params.stride_h, n.params.pad_h, n.params.dil_h);
            const int64_t wo = osz(is[2], ws[3], n.params.stride_w, n.params.pad_w, n.params.dil_w);
            if (ho <= 0 || wo <= 0) fail(ENGINE_ERR_INVALID_SHAPE, "conv '" + n.name + "': empty output");
            set_out(n, 0, {is[0], ho, wo, ws[0]}, act_dt, ni);
            return;
        }
        case Op::MatMul: {
            need(2);
            const auto a = V[input_vid(n, 0)].shape;
            const auto b = V[input_vid(n, 1)].shape;
            if (a.size() == 4 && b.size() == 4 && b[0] == a[0] && b[1] == a[2] && b[3] == a[3]) {
                nt.mode = 2;   // head-batched attention product (session_ops_nn.inc:75-108)
                set_out(n, 0, {a[0], a[1], b[2], a[3]}, F32, ni);
            } else if (a.size() == 4 && b.size() == 2 && a[3] == b[0]) {
                nt.mode = 1;
                set_out(n, 0, {a[0], a[1], a[2], b[1]}, act_dt, ni);
            } else if (a.size() == 2 && b.size() == 2 && a[1] == b[0]) {
                nt.mode = 0;
                set_out(n, 0, {a[0], b[1]}, F32, ni);
            } else {
                fail(ENGINE_ERR_NOT_IMPL, "MatMul '" + n.name + "': only the 2-D, 4-D x 2-D and head-batched 4-D x 4-D forms are supported");
            }
            return;
        }
        case Op::ReLU: case Op::LeakyReLU: case Op::Sigmoid: case Op::Tanh: case Op::SiLU: case Op::GELU:
        case Op::HardSwish: case Op::HardSigmoid: case Op::Clip: {
            need(1);
            const auto s = V[input_vid(n, 0)].shape;
            set_out(n, 0, s, dt_for(s), ni);
            return;
        }
        case Op::Add: case Op::Sub: case Op::Mul: case Op::Div: {
            need(2);
            const auto a = V[input_vid(n, 0)].shape;
            const auto b = V[input_vid(n, 1)].shape;
            const size_t r = std::max(a.size(), b.size());
            std::vector<int64_t> o(r);
            for (size_t d = 0; d < r; ++d) {
                const int64_t da = d < r - a.size() ? 1 : a[d - (r - a.size())];
                const int64_t db = d < r - b.size() ? 1 : b[d - (r - b.size())];
                if (da != db && da != 1 && db != 1) fail(ENGINE_ERR_INVALID_SHAPE, "broadcast mismatch in '" + n.name + "'");
                o[d] = std::max(da, db);
            }
            // bf16 activations stay bf16; fp32 operands (attention scores) stay fp32
            const bool any_bf16 = V[input_vid(n, 0)].dt == BF16 || V[input_vid(n, 1)].dt == BF16;
            set_out(n, 0, o, any_bf16 ? dt_for(o) : F32, ni);
            return;
        }
        case Op::Concat: {
            need(1);
            const auto s0 = V[input_vid(n, 0)].shape;
            const int r = (int)s0.size();
            int ax = n.params.axis < 0 ? n.params.axis + r : n.params.axis;
            if (r == 4 && ax == 1) ax = 3;   // session_ops_shape.inc:73-75
            if (ax < 0 || ax >= r)
                fail(ENGINE_ERR_INVALID_SHAPE, "concat '" + n.name + "': axis " + std::to_string(n.params.axis) +
                                                   " out of range for input shape " + shape_str(s0));
            auto o = s0;
            o[ax] = 0;
            for (size_t k = 0; k < nin; ++k) {
                const auto s = V[input_vid(n, k)].shape;
                if ((int)s.size() != r) fail(ENGINE_ERR_INVALID_SHAPE, "concat rank mismatch");
                o[ax] += s[ax];
            }
            nt.mode = ax;
            set_out(n, 0, o, dt_for(o), ni);
            return;
        }
        case Op::Upsample: case Op::Resize: {
            need(1);
            const auto s = V[input_vid(n, 0)].shape;
            if (s.size() != 4) fail(ENGINE_ERR_INVALID_SHAPE, "resize needs a rank-4 input");
            int64_t H = 0, W = 0;
            const OpParams& p = n.params;
            if (n.op == Op::Upsample) { H = s[1] * p.scale_h; W = s[2] * p.scale_w; }
            else {   // session_ops_shape.inc:111-167
                H = p.target_h; W = p.target_w;
                if ((H <= 0 || W <= 0) && p.scale_h > 1 && p.scale_w > 1) { H = s[1] * p.scale_h; W = s[2] * p.scale_w; }
                if (H <= 0 || W <= 0) {
                    for (size_t k = 1; k < nin && k < 4; ++k) {
                        const int t = input_vid(n, k);
                        const int64_t ne = numel_of(V[t].shape);
                        if (ne == 4 || ne == 2) {
                            const int o = ne == 4 ? 2 : 0;
                            const float a = (float)get_float(t, o), b = (float)get_float(t, o + 1);
                            if (a > 8.0f && b > 8.0f) { H = (int64_t)(a + 0.5f); W = (int64_t)(b + 0.5f); }
                            else { H = (int64_t)((float)s[1] * a + 0.5f); W = (int64_t)((float)s[2] * b + 0.5f); }
                            break;
                        }
                    }
                }
                if (H <= 0 || W <= 0) { H = s[1] * 2; W = s[2] * 2; }
            }
            if (H <= 0 || W <= 0) fail(ENGINE_ERR_INVALID_SHAPE, "resize to an empty shape");
            set_out(n, 0, {s[0], H, W, s[3]}, act_dt, ni);
            return;
        }
        case Op::MaxPool2d: case Op::AvgPool2d: {
            need(1);
            const auto s = V[input_vid(n, 0)].shape;
            if (s.size() != 4) fail(ENGINE_ERR_INVALID_SHAPE, "pool needs a rank-4 input");
            const OpParams& p = n.params;
            if (p.kernel_h <= 0 || p.kernel_w <= 0) { nt.mode = 1; set_out(n, 0, {s[0], 1, 1, s[3]}, act_dt, ni); return; }
            const int64_t ho = (s[1] + 2 * p.pad_h - p.kernel_h) / p.stride_h + 1;
            const int64_t wo = (s[2] + 2 * p.pad_w - p.kernel_w) / p.stride_w + 1;
            set_out(n, 0, {s[0], ho, wo, s[3]}, act_dt, ni);
            return;
        }
        case Op::Reshape: infer_reshape(ni); return;
        case Op::Transpose: infer_transpose(ni); return;
        case Op::Slice: infer_slice(ni); return;
        case Op::Softmax: {
            need(1);
            const auto s = V[input_vid(n, 0)].shape;
            int64_t ax = n.params.axis < 0 ? n.params.axis + (int64_t)s.size() : n.params.axis;
            if (s.size() == 4) { static const int64_t remap[4] = {0, 2, 3, 1}; if (ax >= 0 && ax < 4) ax = remap[ax]; }
            if (ax < 0 || ax >= (int64_t)s.size()) fail(ENGINE_ERR_INVALID_SHAPE, "softmax axis");
            nt.mode = (int)ax;
            set_out(n, 0, s, F32, ni);
            return;
        }
        case Op::TopK: {
            // session_ops_math.inc:321-391: the axis indexes the tensor as stored (no
            // NHWC remap), k comes from the second input, k <= 0 or > the axis: all
            need(2);
            const auto s = V[input_vid(n, 0)].shape;
            int64_t ax = n.params.axis < 0 ? n.params.axis + (int64_t)s.size() : n.params.axis;
            if (ax < 0 || ax >= (int64_t)s.size()) fail(ENGINE_ERR_INVALID_SHAPE, "TopK '" + n.name + "': axis");
            std::vector<double> kv;
            if (!weight_values(n.inputs[1], kv) || kv.empty())
                fail(ENGINE_ERR_NOT_IMPL, "TopK '" + n.name + "': k computed at run time is not supported");
            int64_t k = (int64_t)kv[0];
            if (k <= 0 || k > s[ax]) k = s[ax];
            auto os = s;
            os[ax] = k;
            nt.mode = (int)ax;
            nt.a = {k};
            set_out(n, 0, os, F32, ni);
            if (n.outputs.size() > 1 && n.outputs[1] >= 0) set_out(n, 1, os, F32, ni);   // positions as exact floats
            return;
        }
        case Op::GatherElements: {
            // session_ops_math.inc:393-433: output shaped like the indices
            need(2);
            const auto ds = V[input_vid(n, 0)].shape, is = V[input_vid(n, 1)].shape;
            int64_t ax = n.params.axis < 0 ? n.params.axis + (int64_t)ds.size() : n.params.axis;
            if (ax < 0 || ax >= (int64_t)ds.size() || is.size() != ds.size())
                fail(ENGINE_ERR_INVALID_SHAPE, "GatherElements '" + n.name + "': axis or rank");
            for (size_t d = 0; d < ds.size(); ++d)
                if ((int64_t)d != ax && is[d] != ds[d])
                    fail(ENGINE_ERR_NOT_IMPL, "GatherElements '" + n.name + "': indices must match the data off the axis");
            nt.mode = (int)ax;
            set_out(n, 0, is, F32, ni);
            return;
        }
        default:
            fail(ENGINE_ERR_NOT_IMPL, std::string("op ") + op_name(n.op) + " (id " + std::to_string((int)n.op) +
                                          ") in node '" + n.name + "' is not supported by this build");
        }
    }

    // Reshape (session_ops_shape.inc:512-733). Modes: 0 flat reinterpretation,
    // 1 NCHW-order 4D->4D remap, 2 DFL 4D->3D permute, 3 NHWC->NCHW then flat.
    void infer_reshape(int ni) {
        const Node& n = nodes[ni];
        Note& nt = note[ni];
        const int x = input_vid(n, 0);
        const auto in = V[x].shape;
        const size_t nin = n.inputs.size();
        if (in.size() == 4 && nin >= 2 && numel_of(V[input_vid(n, 1)].shape) == 5) {
            const int t = input_vid(n, 1);
            int64_t tg[5];
            for (int i = 0; i < 5; ++i) tg[i] = get_int(t, i);
            if (in[0] == tg[0] && in[1] == tg[3] && in[2] == tg[4] && tg[1] * tg[2] == in[3]) {
                nt.mode = 0;
                set_out(n, 0, {tg[0], tg[3], tg[4], tg[1], tg[2]}, V[x].dt, ni);
                return;
            }
        }
        if (in.size() == 5 && nin >= 2 && numel_of(V[input_vid(n, 1)].shape) == 4) {
            const int t = input_vid(n, 1);
            int64_t tg[4];
            for (int i = 0; i < 4; ++i) tg[i] = get_int(t, i);
            if (in[0] == tg[0] && in[1] == tg[2] && in[2] == tg[3] && in[3] * in[4] == tg[1]) {
                nt.mode = 0;
                set_out(n, 0, {tg[0], tg[2], tg[3], tg[1]}, V[x].dt, ni);
                return;
            }
        }
        std::vector<int64_t> nd;
        if (nin >= 2) {
            const int t = input_vid(n, 1);
            const int64_t cnt = numel_of(V[t].shape);
            if (cnt < 1 || cnt > 8) fail(ENGINE_ERR_INVALID_SHAPE, "reshape target rank");
            nd.resize(cnt);
            for (int64_t d = 0; d < cnt; ++d) {
                int64_t s = get_int(t, d);
                if (s == 0) s = d < (int64_t)in.size() ? in[d] : 0;
                nd[d] = s;
            }
            int64_t known = 1; int neg = -1;
            for (int i = 0; i < (int)cnt; ++i) { if (nd[i] == -1) neg = i; else known *= nd[i]; }
            if (neg >= 0) nd[neg] = known > 0 ? numel_of(in) / known : 0;
        } else {
            nd = {in[0], numel_of(in) / std::max<int64_t>(in[0], 1)};
        }
        if (numel_of(nd) != numel_of(in)) fail(ENGINE_ERR_INVALID_SHAPE, "reshape changes the element count");
        if (in.size() == 4 && nd.size() == 4) {
            nt.mode = 1;
            set_out(n, 0, {nd[0], nd[2], nd[3], nd[1]}, V[x].dt, ni);
            return;
        }
        if (in.size() == 4 && nd.size() == 3 && in[3] == 1 && in[0] == nd[0] && in[2] == nd[1] && in[1] == nd[2]) {
            nt.mode = 2;
            set_out(n, 0, nd, F32, ni);
            return;
        }
        bool convert = false;
        if (in.size() == 4 && nd.size() != 4) {
            const int64_t c = in[3], h = in[1], w = in[2];
            if (nd.size() == 2 && nd[1] == c * h * w) convert = true;
            else if (nd.size() >= 2 && nd[1] == c) {
                int64_t ts = 1;
                for (size_t d = 2; d < nd.size(); ++d) ts *= nd[d];
                if (h * w == ts) convert = true;
            }
        }
        nt.mode = convert ? 3 : 0;
        set_out(n, 0, nd, nd.size() == 4 ? V[x].dt : F32, ni);
    }

    // Transpose (session_ops_shape.inc:946-1096). Mode 0 identity, 1 permute (perm in note.a).
    void infer_transpose(int ni) {
        const Node& n = nodes[ni];
        Note& nt = note[ni];
        if (n.inputs.size() < 2) fail(ENGINE_ERR_INVALID_FORMAT, "transpose without perm");
        const int x = input_vid(n, 0), pt = input_vid(n, 1);
        const auto s = V[x].shape;
        const int64_t r = (int64_t)s.size();
        if (numel_of(V[pt].shape) != r) fail(ENGINE_ERR_INVALID_SHAPE, "transpose perm length");
        std::vector<int64_t> perm(r);
        if (r == 4) {
            int64_t op[4];
            for (int d = 0; d < 4; ++d) { int64_t p = get_int(pt, d); if (p < 0) p += 4; op[d] = p; }
            const bool id1 = op[0] == 0 && op[1] == 2 && op[2] == 3 && op[3] == 1;
            const bool id2 = op[0] == 0 && op[1] == 3 && op[2] == 1 && op[3] == 2;
            if (id1 || id2) { nt.mode = 0; set_out(n, 0, s, V[x].dt, ni); return; }
            static const int64_t o2m[4] = {0, 3, 1, 2}, m2o[4] = {0, 2, 3, 1};
            for (int d = 0; d < 4; ++d) perm[d] = o2m[op[m2o[d]]];
        } else if (r == 5) {
            int64_t op[5];
            for (int d = 0; d < 5; ++d) { int64_t p = get_int(pt, d); if (p < 0) p += 5; op[d] = p; }
            static const int64_t m5[5] = {0, 3, 4, 1, 2};
            for (int d = 0; d < 5; ++d) perm[d] = m5[op[m5[d]]];
        } else {
            for (int64_t d = 0; d < r; ++d) { int64_t p = get_int(pt, d); if (p < 0) p += r; perm[d] = p; }
        }
        std::vector<int64_t> o(r);
        for (int64_t d = 0; d < r; ++d) o[d] = s[perm[d]];
        nt.mode = 1;
        nt.a = perm;
        set_out(n, 0, o, r == 4 ? V[x].dt : F32, ni);
    }

    // Slice (session_ops_shape.inc:754-889): note.a = starts, note.b = steps per axis.
    void infer_slice(int ni) {
        const Node& n = nodes[ni];
        Note& nt = note[ni];
        if (n.inputs.size() < 3) fail(ENGINE_ERR_INVALID_FORMAT, "slice needs starts and ends");
        const int x = input_vid(n, 0), st = input_vid(n, 1), en = input_vid(n, 2);
        int ax_v = -1, sp_v = -1;
        if (n.inputs.size() > 3) { ax_v = input_vid(n, 3); if (numel_of(V[ax_v].shape) == 0) ax_v = -1; }
        if (n.inputs.size() > 4) { sp_v = input_vid(n, 4); if (numel_of(V[sp_v].shape) == 0) sp_v = -1; }
        const auto s = V[x].shape;
        const int64_t r = (int64_t)s.size();
        const int64_t ns = numel_of(V[st].shape);
        std::vector<int64_t> od = s, sv(r, 0), stv(r, 1);
        for (int64_t k = 0; k < ns; ++k) {
            int64_t ax = ax_v >= 0 ? get_int(ax_v, k) : k;
            if (ax < 0) ax += r;
            const int64_t ax_orig = ax;
            if (r == 4) { if (ax == 1) ax = 3; else if (ax == 2) ax = 1; else if (ax == 3) ax = 2; }
            int64_t b = get_int(st, k), e = get_int(en, k);
            if (ax != ax_orig && r == 4) {
                if (e > s[ax] * 2 && e <= s[ax_orig]) ax = ax_orig;
            }
            if (ax < 0 || ax >= r) continue;
            int64_t step = sp_v >= 0 ? get_int(sp_v, k) : 1;
            if (step == 0) step = 1;
            const int64_t len = s[ax];
            if (b < 0) b += len;
            if (e < 0) e += len;
            b = std::clamp<int64_t>(b, 0, len);
            e = std::clamp<int64_t>(e, 0, len);
            if (e < b) e = b;
            sv[ax] = b;
            stv[ax] = step;
            od[ax] = step > 0 ? (e - b + step - 1) / step : 0;
        }
        nt.a = sv;
        nt.b = stv;
        int sliced = -1, cnt = 0;
        bool unit = true;
        for (int64_t d = 0; d < r; ++d)
            if (od[d] != s[d] || sv[d] != 0 || stv[d] != 1) { sliced = (int)d; ++cnt; unit &= stv[d] == 1; }
        nt.mode = (r == 4 && cnt == 1 && sliced == 3 && unit) ? 1 : 0;   // 1 = channel view
        set_out(n, 0, od, V[x].dt, ni);
    }

    // -------------------------------------------------------------------
    // 3. YOLOv8 Detect tail
    int producer_node(int32_t t) {
        for (size_t i = 0; i < nodes.size(); ++i)
            if (!skip[i] && !nodes[i].outputs.empty() && nodes[i].outputs[0] == t) return (int)i;
        return -1;
    }
    int single_consumer(int32_t t) {
        if (consumers[t] != 1) return -1;
        for (size_t i = 0; i < nodes.size(); ++i) {
            if (skip[i]) continue;
            for (int32_t in : nodes[i].inputs) if (in == t) return (int)i;
        }
        return -1;
    }
    bool weight_values(int32_t idx, std::vector<double>& out) {
        if (idx > -1000) return false;
        const Weight& w = g.weights[-idx - 1000];
        out.resize(w.numel());
        for (int64_t i = 0; i < w.numel(); ++i) out[i] = w.value(i);
        return true;
    }

    void match_head() {
        if (g.outputs.size() != 1) return;
        const char* off = std::getenv("PDEFA_NO_HEAD_FUSION");
        if (off && *off && *off != '0') return;
        std::vector<int> covered;
        auto at = [&](int32_t t) { return producer_node(t); };
        const int fin = at(g.outputs[0]);
        if (fin < 0 || nodes[fin].op != Op::Concat || nodes[fin].inputs.size() != 2) return;
        const Value& fo = V[vid[nodes[fin].outputs[0]]];
        if (fo.shape.size() != 3) return;
        const int mul = at(nodes[fin].inputs[0]), sig = at(nodes[fin].inputs[1]);
        if (mul < 0 || sig < 0 || nodes[mul].op != Op::Mul || nodes[sig].op != Op::Sigmoid) return;
        const int cat4 = at(nodes[mul].inputs[0]);
        const int32_t stride_w = nodes[mul].inputs[1];
        if (cat4 < 0 || nodes[cat4].op != Op::Concat || nodes[cat4].inputs.size() != 2 || stride_w > -1000) return;
        const int div = at(nodes[cat4].inputs[0]), sub1 = at(nodes[cat4].inputs[1]);
        if (div < 0 || sub1 < 0 || nodes[div].op != Op::Div || nodes[sub1].op != Op::Sub) return;
        std::vector<double> two;
        if (!weight_values(nodes[div].inputs[1], two) || two.size() != 1 || two[0] != 2.0) return;
        const int add2 = at(nodes[div].inputs[0]);
        if (add2 < 0 || nodes[add2].op != Op::Add) return;
        const int subA = at(nodes[add2].inputs[0]), addA = at(nodes[add2].inputs[1]);
        if (subA < 0 || addA < 0 || nodes[subA].op != Op::Sub || nodes[addA].op != Op::Add) return;
        if (at(nodes[sub1].inputs[0]) != addA || at(nodes[sub1].inputs[1]) != subA) return;
        const int32_t anc = nodes[subA].inputs[0];
        if (anc > -1000 || nodes[addA].inputs[0] != anc) return;
        const int slt = at(nodes[subA].inputs[1]), srb = at(nodes[addA].inputs[1]);
        if (slt < 0 || srb < 0 || nodes[slt].op != Op::Slice || nodes[srb].op != Op::Slice) return;
        if (nodes[slt].inputs[0] != nodes[srb].inputs[0]) return;
        const int rs1 = at(nodes[slt].inputs[0]);
        if (rs1 < 0 || nodes[rs1].op != Op::Reshape) return;
        const int conv = at(nodes[rs1].inputs[0]);
        if (conv < 0 || nodes[conv].op != Op::Conv2d || nodes[conv].inputs.size() != 2 || conv_act[conv]) return;
        const int32_t dflw = nodes[conv].inputs[1];
        const int smx = at(nodes[conv].inputs[0]);
        if (smx < 0 || nodes[smx].op != Op::Softmax) return;
        const int tr = at(nodes[smx].inputs[0]);
        if (tr < 0 || nodes[tr].op != Op::Transpose) return;
        const int rs0 = at(nodes[tr].inputs[0]);
        if (rs0 < 0 || nodes[rs0].op != Op::Reshape) return;
        const int sbox = at(nodes[rs0].inputs[0]), scls = at(nodes[sig].inputs[0]);
        if (sbox < 0 || scls < 0 || nodes[sbox].op != Op::Slice || nodes[scls].op != Op::Slice) return;
        if (nodes[sbox].inputs[0] != nodes[scls].inputs[0]) return;
        const int cat3 = at(nodes[sbox].inputs[0]);
        if (cat3 < 0 || nodes[cat3].op != Op::Concat || nodes[cat3].inputs.size() != 3) return;
        // expected value shapes
        const Value& x3 = V[vid[nodes[cat3].outputs[0]]];
        if (x3.shape.size() != 3) return;
        const int64_t no = x3.shape[1], A = x3.shape[2];
        const Value& wv = V[vid[dflw]];
        if (wv.shape.size() != 4 || wv.shape[0] != 1 || wv.shape[2] != 1 || wv.shape[3] != 1) return;
        const int64_t reg = wv.shape[1];
        const int64_t nc = no - 4 * reg;
        if (nc <= 0 || fo.shape[1] != 4 + nc || fo.shape[2] != A || reg > 32) return;
        // slice bounds: box [0, 4reg), cls [4reg, no), lt [0,2), rb [2,4) on axis 1
        auto slice_is = [&](int sn, int64_t b, int64_t len) {
            const auto& sv = note[sn].a;
            const Value& o = V[vid[nodes[sn].outputs[0]]];
            return sv.size() == 3 && sv[1] == b && sv[0] == 0 && sv[2] == 0 && o.shape.size() == 3 && o.shape[1] == len;
        };
        if (!slice_is(sbox, 0, 4 * reg) || !slice_is(scls, 4 * reg, nc) || !slice_is(slt, 0, 2) || !slice_is(srb, 2, 2)) return;
        if (note[tr].a != std::vector<int64_t>{0, 3, 2, 1} || note[smx].mode != 2 || note[rs1].mode != 2) return;
        std::vector<double> av, sv;
        if (!weight_values(anc, av) || (int64_t)av.size() != 2 * A) return;
        if (!weight_values(stride_w, sv) || (int64_t)sv.size() != A) return;
        int levels[3];
        int64_t tot = 0;
        for (int l = 0; l < 3; ++l) {
            const int rs = at(nodes[cat3].inputs[l]);
            if (rs < 0 || nodes[rs].op != Op::Reshape || note[rs].mode != 3) return;
            const Value& lv = V[vid[nodes[rs].inputs[0]]];
            if (lv.shape.size() != 4 || lv.shape[3] != no) return;
            levels[l] = vid[nodes[rs].inputs[0]];
            tot += lv.shape[1] * lv.shape[2];
            covered.push_back(rs);
        }
        if (tot != A) return;
        const int chain[] = {fin, mul, sig, cat4, div, sub1, add2, subA, addA, slt, srb, rs1, conv, smx, tr, rs0, sbox, scls, cat3};
        // every intermediate of the chain must stay internal to it
        for (int c : chain) {
            if (c == fin) continue;
            const int32_t o = nodes[c].outputs[0];
            for (int32_t go : g.outputs) if (go == o) return;
            for (size_t i = 0; i < nodes.size(); ++i) {
                if (skip[i]) continue;
                bool inside = std::find(std::begin(chain), std::end(chain), (int)i) != std::end(chain) ||
                              std::find(covered.begin(), covered.end(), (int)i) != covered.end();
                if (inside) continue;
                for (int32_t in : nodes[i].inputs) if (in == o) return;
            }
        }
        for (int c : covered) {
            const int32_t o = nodes[c].outputs[0];
            if (consumers[o] != 1) return;
        }
        for (int c : chain) skip[c] = 2;
        for (int c : covered) skip[c] = 2;
        skip[fin] = 3;                 // emit the head here
        head = true;
        head_at = fin;
        head_out = vid[g.outputs[0]];
        for (int l = 0; l < 3; ++l) head_levels[l] = levels[l];
        head_anchor_w = -anc - 1000;
        head_stride_w = -stride_w - 1000;
        head_dfl_w = -dflw - 1000;
        head_reg = (int)reg;
        head_nc = (int)nc;
        if (verbose()) std::fprintf(stderr, "[pdefa-b200] fused YOLO head: A=%lld reg=%lld nc=%lld\n",
                                    (long long)A, (long long)reg, (long long)nc);
    }

    // -------------------------------------------------------------------
    // 4. residual fusion: Add(x, conv_out) -> conv epilogue adds x.
    void fuse_residuals() {
        const char* off = std::getenv("PDEFA_NO_RESIDUAL_FUSION");
        if (off && *off && *off != '0') return;
        for (size_t i = 0; i < nodes.size(); ++i) {
            if (skip[i] || nodes[i].op != Op::Add || nodes[i].inputs.size() != 2) continue;
            const Node& a = nodes[i];
            for (int side = 1; side >= 0; --side) {
                const int32_t ct = a.inputs[side], xt = a.inputs[1 - side];
                if (ct == xt || consumers[ct] != 1) continue;
                const int cn = producer_node(ct);
                if (cn < 0 || nodes[cn].op != Op::Conv2d || note[cn].mode != 0 || conv_res[cn] >= 0) continue;
                if (conv_act[cn] == 100) continue;
                const int cv = vid[ct], xv = vid[xt], ov = vid[a.outputs[0]];
                if (V[cv].shape.size() != 4 || V[cv].shape != V[xv].shape || V[ov].shape != V[cv].shape) continue;
                const int xp = V[xv].producer;
                if (!V[xv].external && V[xv].weight < 0 && xp >= cn) continue;
                if (V[xv].weight >= 0) continue;
                conv_res[cn] = xv;
                nodes[cn].outputs[0] = a.outputs[0];
                V[ov].producer = cn;
                skip[i] = 1;
                break;
            }
        }
    }

    // Attention products (MatMul mode 2): a Transpose whose only reader is the product
    // is not materialised (the product reads its input through permuted strides), and
    // a Mul by a scalar constant that is the product's only reader is applied to the
    // product's sums (out = sum * s, the reference's separate Mul rounding once the
    // same way).
    void fold_attention() {
        for (size_t i = 0; i < nodes.size(); ++i) {
            if (skip[i] || nodes[i].op != Op::MatMul || note[i].mode != 2) continue;
            for (int side = 0; side < 2; ++side) {
                const int32_t t = nodes[i].inputs[side];
                if (consumers[t] != 1) continue;
                const int k = producer_node(t);
                if (k < 0 || nodes[k].op != Op::Transpose || note[k].mode != 1) continue;
                if (V[input_vid(nodes[k], 0)].shape.size() != 4) continue;
                skip[k] = 1;
                folded_transpose[vid[t]] = k;
            }
            const int32_t ot = nodes[i].outputs[0];
            if (consumers[ot] != 1) continue;
            for (size_t m = i + 1; m < nodes.size(); ++m) {
                const Node& mn = nodes[m];
                if (skip[m] || mn.op != Op::Mul || mn.inputs.size() != 2) continue;
                const int side = mn.inputs[0] == ot ? 0 : (mn.inputs[1] == ot ? 1 : -1);
                if (side < 0) continue;
                const int sv = vid[mn.inputs[1 - side]];
                const int mo = vid[mn.outputs[0]];
                if (V[sv].weight >= 0 && numel_of(V[sv].shape) == 1 && V[mo].shape == V[vid[ot]].shape &&
                    V[mo].dt == F32) {
                    note[i].scale = (float)g.weights[V[sv].weight].value(0);
                    nodes[i].outputs[0] = mn.outputs[0];
                    V[mo].producer = (int)i;
                    skip[m] = 1;
                }
                break;
            }
        }
    }

    // Tensor-core convs need Cout % 16 == 0 and >= 32-byte channel rows. A conv with
    // a narrow output (e.g. the 8-channel bottleneck of a YOLO11n C3k2) whose only
    // readers are convs gets its output stored with Cout rounded up to 16 (zero
    // weights and bias in the extra channels, whose activation is then exactly 0) and
    // each reader gets zero weights for those channels: both run on tcgen05 instead of
    // the SIMT kernels, with the same values (an exact 0 adds nothing to a sum).
    // FP32 plans keep the strict SIMT path and are not padded.
    void pad_narrow_channels() {
        if (prec == PREC_FP32) return;
        const char* off = std::getenv("PDEFA_NO_CHANNEL_PAD");
        if (off && *off && *off != '0') return;
        auto conv_reader = [&](size_t k, int32_t t) {
            const Node& c = nodes[k];
            if (c.op != Op::Conv2d || skip[k] || note[k].mode != 0 || note[k].dfl_fix) return false;
            if ((c.params.groups > 0 ? c.params.groups : 1) != 1) return false;
            for (size_t j = 1; j < c.inputs.size(); ++j) if (c.inputs[j] == t) return false;
            return c.inputs[0] == t;
        };
        for (size_t i = 0; i < nodes.size(); ++i) {
            const Node& n = nodes[i];
            if (n.op != Op::Conv2d || skip[i] || note[i].mode != 0 || note[i].dfl_fix || conv_res[i] >= 0) continue;
            if ((n.params.groups > 0 ? n.params.groups : 1) != 1) continue;
            const int act = conv_act[i];
            if (act != ACT_NONE && act != ACT_RELU && act != ACT_LEAKY && act != ACT_SILU) continue;
            const int32_t t = n.outputs[0];
            const int o = vid[t];
            auto& sh = V[o].shape;
            if (sh.size() != 4 || sh[3] % 16 == 0 || sh[3] > 256 || is_graph_output(o)) continue;
            int readers = 0;
            bool ok = true;
            for (size_t k = 0; k < nodes.size() && ok; ++k) {
                if (k == i || nodes[k].op == Op::Input) continue;
                bool reads = false;
                for (int32_t in : nodes[k].inputs) reads |= in == t;
                if (!reads) continue;
                if (conv_reader(k, t)) ++readers;
                else ok = false;
            }
            if (ok && readers > 0) sh[3] = (sh[3] + 15) / 16 * 16;
        }
    }

    // -------------------------------------------------------------------
    // 5. placement
    bool is_graph_output(int v) {
        for (int32_t o : g.outputs) if (vid.count(o) && vid[o] == v) return true;
        return false;
    }
    bool writer(int v) {
        const Value& x = V[v];
        if (x.external || x.weight >= 0 || x.alias_of >= 0 || x.place_in >= 0 || x.producer < 0) return false;
        if (is_graph_output(v)) return false;
        const Node& n = nodes[x.producer];
        switch (n.op) {
            case Op::Conv2d: return note[x.producer].mode == 0 && conv_act[x.producer] != 100;
            case Op::MaxPool2d: case Op::AvgPool2d: case Op::Upsample: case Op::Resize:
            case Op::Add: case Op::Sub: case Op::Mul: case Op::Div:
            case Op::ReLU: case Op::LeakyReLU: case Op::Sigmoid: case Op::Tanh: case Op::SiLU: case Op::GELU:
            case Op::HardSwish: case Op::HardSigmoid: case Op::Clip: case Op::Concat:
                return true;
            default: return false;
        }
    }

    void place() {
        // channel-slice views
        for (size_t i = 0; i < nodes.size(); ++i) {
            if (skip[i] || nodes[i].op != Op::Slice || note[i].mode != 1) continue;
            const int src = vid[nodes[i].inputs[0]];
            const int dst = vid[nodes[i].outputs[0]];
            if (V[src].external || V[src].weight >= 0) continue;
            V[dst].alias_of = src;
            V[dst].alias_off = note[i].a[3];
            note[i].mode = 2;   // realised as a view
        }
        // zero-copy concats (rank 4, channel axis)
        for (size_t i = 0; i < nodes.size(); ++i) {
            if (skip[i] || nodes[i].op != Op::Concat || note[i].mode != 3) continue;
            const Node& n = nodes[i];
            const int C = vid[n.outputs[0]];
            if (V[C].shape.size() != 4) continue;
            int64_t off = 0;
            for (size_t k = 0; k < n.inputs.size();) {
                const int v = vid[n.inputs[k]];
                const int64_t len = V[v].shape[3];
                // run of channel views covering one value in order
                if (V[v].alias_of >= 0 && V[v].alias_off == 0 && V[V[v].alias_of].shape.size() == 4) {
                    const int base = V[v].alias_of;
                    int64_t covered = 0;
                    size_t j = k;
                    while (j < n.inputs.size()) {
                        const int u = vid[n.inputs[j]];
                        if (V[u].alias_of != base || V[u].alias_off != covered) break;
                        covered += V[u].shape[3];
                        ++j;
                        if (covered == V[base].shape[3]) break;
                    }
                    if (covered == V[base].shape[3] && writer(base) && V[base].dt == V[C].dt) {
                        V[base].place_in = C;
                        V[base].place_ch = off;
                        off += covered;
                        k = j;
                        continue;
                    }
                }
                if (writer(v) && v != C && V[v].dt == V[C].dt) {
                    bool dup = false;
                    for (size_t j = 0; j < k; ++j) dup |= vid[n.inputs[j]] == v;
                    if (!dup) { V[v].place_in = C; V[v].place_ch = off; }
                }
                off += len;
                ++k;
            }
        }
    }

    // -------------------------------------------------------------------
    // 6. allocation
    // Activations that own their storage ("roots": not a view, not placed inside a
    // concat, not a weight or graph input) live in one arena. A dry lowering records
    // each root's byte size and the range of nodes that touch it (any view of the
    // root, its slices or its concat members); pack_arena() then gives roots whose
    // node ranges do not intersect the same bytes, and the real lowering places each
    // root at its offset (PDEFA1.0/src/memory/memory_plan.cpp:105-137 plans the
    // reference's CPU buffers the same way, by live ranges).
    std::vector<void*> bufs;
    int cur_node = -1;                       // node being emitted; nodes.size() for the outputs
    bool u8_stem = false;                    // the stem reads 8-bit input frames (Plan::u8_scale_)
    const std::vector<size_t>* arena_off = nullptr;   // real lowering: byte offset per value id
    char* arena = nullptr;

    int root_of(int v) const {
        while (V[v].alias_of >= 0 || V[v].place_in >= 0) v = V[v].alias_of >= 0 ? V[v].alias_of : V[v].place_in;
        return v;
    }
    void touch(int v) {
        const int r = root_of(v);
        if ((size_t)r >= P.root_first_.size()) {
            P.root_first_.resize(V.size(), INT_MAX);
            P.root_last_.resize(V.size(), -1);
            P.root_bytes_.resize(V.size(), 0);
        }
        const int n = std::max(cur_node, 0);
        P.root_first_[r] = std::min(P.root_first_[r], n);
        P.root_last_[r] = std::max(P.root_last_[r], n);
    }
    void finalize(int v) {
        Value& x = V[v];
        if (x.buf >= 0 || !x.known) return;
        if (x.alias_of >= 0) {
            finalize(x.alias_of);
            const Value& s = V[x.alias_of];
            x.buf = s.buf; x.off = s.off + x.alias_off; x.stride = s.stride; x.img_stride = s.img_stride; x.dt = s.dt;
            return;
        }
        if (x.place_in >= 0) {
            finalize(x.place_in);
            const Value& c = V[x.place_in];
            x.buf = c.buf; x.off = c.off + x.place_ch; x.stride = c.stride; x.img_stride = c.img_stride;
            return;
        }
        x.stride = dense_strides(x.shape);
        if (x.weight >= 0) {
            x.buf = (int)bufs.size();
            bufs.push_back(weight_f32(x.weight));
            x.img_stride = 0;
            return;
        }
        x.img_stride = numel_of(x.shape);
        const size_t bytes = (size_t)x.img_stride * B * (x.dt == BF16 ? 2 : 4);
        x.buf = (int)bufs.size();
        if ((size_t)v >= P.root_bytes_.size()) {
            P.root_first_.resize(V.size(), INT_MAX);
            P.root_last_.resize(V.size(), -1);
            P.root_bytes_.resize(V.size(), 0);
        }
        P.root_bytes_[v] = std::max<size_t>(bytes, 16);
        if (arena_off && (size_t)v < arena_off->size() && (*arena_off)[v] != SIZE_MAX)
            bufs.push_back(arena + (*arena_off)[v]);
        else
            bufs.push_back(P.alloc(bytes > 0 ? bytes : 16));
    }

    void* weight_f32(int w) {
        auto it = wdev.find(w);
        if (it != wdev.end()) return it->second;
        const Weight& W = g.weights[w];
        std::vector<float> h(W.numel());
        for (int64_t i = 0; i < W.numel(); ++i) h[i] = (float)W.value(i);
        void* d = P.alloc(std::max<size_t>(h.size() * 4, 16));
        if (!P.dry_) PB_CUDA(cudaMemcpy(d, h.data(), h.size() * 4, cudaMemcpyHostToDevice));
        wdev[w] = d;
        return d;
    }

    TView view(int v) {
        finalize(v);
        touch(v);
        const Value& x = V[v];
        TView t;
        t.ptr = static_cast<char*>(bufs[x.buf]) + x.off * (x.dt == BF16 ? 2 : 4);
        t.dt = x.dt;
        t.rank = (int)x.shape.size();
        for (int d = 0; d < t.rank; ++d) { t.shape[d] = x.shape[d]; t.stride[d] = x.stride[d]; }
        t.img_stride = x.img_stride;
        return t;
    }

    bool dense(int v) {
        finalize(v);
        touch(v);
        const Value& x = V[v];
        return x.stride == dense_strides(x.shape) && (x.img_stride == numel_of(x.shape) || x.img_stride == 0);
    }

    // A dense fp32 copy of v (or v itself when already dense fp32).
    TView dense_f32(int v, const std::string& name) {
        TView src = view(v);
        if (dense(v) && V[v].dt == F32) return src;
        TView dst = src;
        const auto st = dense_strides(V[v].shape);
        dst.dt = F32;
        for (int d = 0; d < dst.rank; ++d) dst.stride[d] = st[d];
        dst.img_stride = numel_of(V[v].shape);
        dst.ptr = P.alloc(std::max<size_t>((size_t)dst.img_stride * B * 4, 16));
        add_copy(src, dst, name + "/densify");
        return dst;
    }

    // -------------------------------------------------------------------
    // 7. emission
    int external_of(const TView& t) {
        for (size_t i = 0; i < P.inputs_.size(); ++i) if (t.ptr == P.inputs_[i]) return (int)i;
        return -1;
    }

    std::string next_kind = "kernel";
    void add_step(const std::string& name, std::function<void(cudaStream_t)> fn, int launches = 1) {
        P.steps_.push_back(PlanStep{name, std::move(fn), launches, next_kind});
        next_kind = "kernel";
    }
    void kind(const char* k) { next_kind = k; }

    void add_copy(TView src, TView dst, const std::string& name) {
        const int64_t b = B;
        const bool ext = external_of(src) == 0;
        Plan* pp = &P;
        kind("copy");
        add_step(name, [src, dst, b, ext, pp](cudaStream_t s) mutable {
            if (ext && pp->cur_in_) src.ptr = pp->cur_in_;
            launch_strided_copy(src, dst, b, s);
        });
    }

    void emit() {
        // inputs
        for (size_t i = 0; i < g.inputs.size(); ++i) {
            const int v = vid[g.inputs[i]];
            Value& x = V[v];
            const auto& s = x.shape;   // motor [1,H,W,C] for rank 4
            const int64_t per = numel_of(s);
            // 8-bit frames: one byte per element, read only by the stem (checked below)
            const size_t ibytes = (size_t)per * B * (i == 0 && P.u8_scale_ > 0.0f ? 1 : 4);
            float* d = static_cast<float*>(P.alloc(std::max<size_t>(ibytes, 16)));
            P.inputs_.push_back(d);
            P.input_bytes_.push_back(ibytes);
            x.buf = (int)bufs.size();
            bufs.push_back(d);
            x.off = 0;
            x.img_stride = per;
            if (s.size() == 4) {     // NCHW memory seen through NHWC motor dims
                const int64_t H = s[1], W = s[2], C = s[3];
                x.stride = {C * H * W, W, 1, H * W};
            } else {
                x.stride = dense_strides(s);
            }
        }
        for (size_t i = 0; i < nodes.size(); ++i) {
            cur_node = (int)i;
            if (skip[i] == 3) { emit_head(); continue; }
            if (skip[i]) continue;
            emit_node((int)i);
        }
        cur_node = (int)nodes.size();
        if (P.u8_scale_ > 0.0f && (!u8_stem || consumers[g.inputs[0]] != 1))
            fail(ENGINE_ERR_NOT_IMPL, "8-bit input: the stem conv must be the graph input's only consumer");
        // outputs: dense fp32, rank-4 converted to NCHW (session.cpp:347-361)
        for (size_t k = 0; k < g.outputs.size(); ++k) {
            const int v = vid[g.outputs[k]];
            if (!V[v].known) fail(ENGINE_ERR_RUNTIME, "graph output is never produced");
            TView src = view(v);
            std::vector<int64_t> oshape = V[v].shape;
            TView dst = src;
            dst.dt = F32;
            if (oshape.size() == 4) {
                // destination NCHW buffer viewed with motor dims (n,h,w,c)
                const int64_t H = oshape[1], W = oshape[2], C = oshape[3];
                dst.stride[0] = C * H * W; dst.stride[1] = W; dst.stride[2] = 1; dst.stride[3] = H * W;
                dst.img_stride = C * H * W;
                oshape = {1, C, H, W};
            } else {
                const auto st = dense_strides(oshape);
                for (int d = 0; d < dst.rank; ++d) dst.stride[d] = st[d];
                dst.img_stride = numel_of(oshape);
            }
            const size_t bytes = (size_t)numel_of(oshape) * B * 4;
            float* obuf;
            if (head && v == head_out) {
                obuf = static_cast<float*>(const_cast<void*>(src.ptr));
            } else {
                obuf = static_cast<float*>(P.alloc(std::max<size_t>(bytes, 16)));
                dst.ptr = obuf;
                add_copy(src, dst, "output" + std::to_string(k));
            }
            std::vector<int64_t> bshape = oshape;
            if (!bshape.empty()) bshape[0] *= B;
            P.outputs_.push_back(obuf);
            P.out_bytes_.push_back(bytes);
            P.out_shapes_.push_back(bshape);
        }
        // Intermediates readable after a run: values produced by an emitted node that
        // no node consumes, and the requested ones; their storage stays reserved past
        // the last node, so no later launch reuses it.
        cur_node = (int)nodes.size() + 1;
        std::vector<int32_t> want;
        for (size_t i = 0; i < nodes.size(); ++i) {
            if (skip[i]) continue;     // fused away or inside the fused head: never written
            for (int32_t o : nodes[i].outputs) {
                if (o < 0) continue;
                const bool asked = std::find(P.keep_.begin(), P.keep_.end(), o) != P.keep_.end();
                if (asked || consumers[o] == 0) want.push_back(o);
            }
        }
        for (int32_t idx : want) {
            auto it = vid.find(idx);
            if (it == vid.end() || !V[it->second].known || V[it->second].weight >= 0) continue;
            P.debug_[idx] = view(it->second);
        }
    }

    void emit_head() {
        YoloHeadArgs a;
        for (int l = 0; l < 3; ++l) {
            a.level[l] = view(head_levels[l]);
            a.level_anchors[l] = V[head_levels[l]].shape[1] * V[head_levels[l]].shape[2];
        }
        a.nlevels = 3;
        a.reg_max = head_reg;
        a.nc = head_nc;
        a.anchors = static_cast<const float*>(weight_f32(head_anchor_w));
        a.strides = static_cast<const float*>(weight_f32(head_stride_w));
        a.dfl_w = static_cast<const float*>(weight_f32(head_dfl_w));
        const TView o = view(head_out);
        a.out = static_cast<float*>(const_cast<void*>(o.ptr));
        a.A = V[head_out].shape[2];
        a.batch = B;
        kind("yolo_head");
        add_step("yolo_head", [a](cudaStream_t s) { launch_yolo_head(a, s); });
    }

    void emit_node(int ni) {
        const Node& n = nodes[ni];
        const Note& nt = note[ni];
        switch (n.op) {
        case Op::Conv2d: emit_conv(ni); return;
        case Op::MatMul: emit_matmul(ni); return;
        case Op::ReLU: case Op::LeakyReLU: case Op::Sigmoid: case Op::Tanh: case Op::SiLU: case Op::GELU:
        case Op::HardSwish: case Op::HardSigmoid: case Op::Clip: {
            int kind = 0; float p0 = 0, p1 = 0;
            switch (n.op) {
                case Op::ReLU: kind = ACT_RELU; break;
                case Op::LeakyReLU: kind = ACT_LEAKY; p0 = n.params.leaky_slope; break;
                case Op::Sigmoid: kind = ACT_SIGMOID; break;
                case Op::Tanh: kind = UN_TANH; break;
                case Op::SiLU: kind = ACT_SILU; break;
                case Op::GELU: kind = ACT_GELU_TANH; break;
                case Op::HardSwish: kind = UN_HARDSWISH; break;
                case Op::HardSigmoid: kind = UN_HARDSIGMOID; break;
                default: kind = UN_CLIP; p0 = n.params.eps; p1 = n.params.leaky_slope; break;   // session_ops_nn.inc:503-529
            }
            TView in = view(input_vid(n, 0)), out = view(vid[n.outputs[0]]);
            const int64_t b = B;
            const bool ext = external_of(in) == 0;
            Plan* pp = &P;
            this->kind("unary");
            add_step(n.name, [=](cudaStream_t s) mutable {
                if (ext && pp->cur_in_) in.ptr = pp->cur_in_;
                launch_unary(kind, in, out, b, p0, p1, s);
            });
            return;
        }
        case Op::Add: case Op::Sub: case Op::Mul: case Op::Div: {
            const int op = n.op == Op::Add ? BIN_ADD : n.op == Op::Sub ? BIN_SUB : n.op == Op::Mul ? BIN_MUL : BIN_DIV;
            const int ov = vid[n.outputs[0]];
            TView out = view(ov);
            auto aligned = [&](int v) {
                TView t = view(v);
                const int r = out.rank, ra = t.rank;
                TView u = t;
                u.rank = r;
                for (int d = 0; d < r; ++d) {
                    const int sd = d - (r - ra);
                    if (sd < 0) { u.shape[d] = out.shape[d]; u.stride[d] = 0; }
                    else { u.shape[d] = out.shape[d]; u.stride[d] = t.shape[sd] == 1 ? 0 : t.stride[sd]; }
                }
                return u;
            };
            TView a = aligned(input_vid(n, 0)), bb = aligned(input_vid(n, 1));
            const int64_t b = B;
            kind("binary");
            add_step(n.name, [=](cudaStream_t s) { launch_binary(op, a, bb, out, b, s); });
            return;
        }
        case Op::Concat: {
            const int C = vid[n.outputs[0]];
            const int ax = nt.mode;
            TView out = view(C);
            int64_t off = 0;
            for (size_t k = 0; k < n.inputs.size(); ++k) {
                const int v = input_vid(n, k);
                const int64_t len = V[v].shape[ax];
                bool placed = false;
                if (V[v].place_in == C) placed = true;
                if (V[v].alias_of >= 0 && V[V[v].alias_of].place_in == C) placed = true;
                if (!placed) {
                    TView src = view(v);
                    TView dst = out;
                    for (int d = 0; d < dst.rank; ++d) dst.shape[d] = src.shape[d];
                    dst.ptr = static_cast<const char*>(out.ptr) + off * out.stride[ax] * (out.dt == BF16 ? 2 : 4);
                    add_copy(src, dst, n.name + "/in" + std::to_string(k));
                }
                off += len;
            }
            return;
        }
        case Op::Upsample: case Op::Resize: {
            TView in = view(input_vid(n, 0)), out = view(vid[n.outputs[0]]);
            const int64_t b = B;
            kind("resize");
            add_step(n.name, [=](cudaStream_t s) { launch_resize_nearest(in, out, b, s); });
            return;
        }
        case Op::MaxPool2d: case Op::AvgPool2d: {
            Pool2dArgs a;
            a.in = view(input_vid(n, 0));
            a.out = view(vid[n.outputs[0]]);
            a.kh = (int)n.params.kernel_h; a.kw = (int)n.params.kernel_w;
            a.sh = (int)n.params.stride_h; a.sw = (int)n.params.stride_w;
            a.ph = (int)n.params.pad_h; a.pw = (int)n.params.pad_w;
            a.mode = (n.op == Op::MaxPool2d ? 0 : 1) + (nt.mode == 1 ? 2 : 0);
            a.batch = B;
            kind("pool");
            // SPPF: the next two max pools with the same parameters that each read the
            // previous one's output run in the same launch (the input is read once); they
            // are not emitted again
            std::vector<int> chain;
            if (a.mode == 0) {
                int cur = ni;
                for (size_t j = (size_t)ni + 1; j < nodes.size() && chain.size() < 2; ++j) {
                    const Node& m = nodes[j];
                    if (skip[j] || m.op != Op::MaxPool2d || note[j].mode != 0 || m.inputs.empty() ||
                        m.inputs[0] != nodes[cur].outputs[0] || m.params.kernel_h != n.params.kernel_h ||
                        m.params.kernel_w != n.params.kernel_w || m.params.stride_h != n.params.stride_h ||
                        m.params.stride_w != n.params.stride_w || m.params.pad_h != n.params.pad_h ||
                        m.params.pad_w != n.params.pad_w)
                        continue;
                    chain.push_back((int)j);
                    cur = (int)j;
                }
            }
            if (!chain.empty()) {
                TView outs[3];
                outs[0] = a.out;
                for (size_t k = 0; k < chain.size(); ++k) outs[k + 1] = view(vid[nodes[chain[k]].outputs[0]]);
                const int cnt = 1 + (int)chain.size();
                if (maxpool_chain_supported(a, outs, cnt)) {
                    for (int j : chain) skip[j] = 1;
                    add_step(n.name, [a, outs, cnt](cudaStream_t s) {
                        if (!launch_maxpool_chain(a, outs, cnt, s)) fail(ENGINE_ERR_RUNTIME, "max pool chain: layout changed");
                    });
                    return;
                }
            }
            add_step(n.name, [a](cudaStream_t s) { launch_pool2d(a, s); });
            return;
        }
        case Op::Reshape: emit_reshape(ni); return;
        case Op::Transpose: {
            const int x = input_vid(n, 0), o = vid[n.outputs[0]];
            TView src = view(x), dst = view(o);
            if (nt.mode == 1) {
                TView p = src;
                for (int d = 0; d < p.rank; ++d) { p.shape[d] = src.shape[nt.a[d]]; p.stride[d] = src.stride[nt.a[d]]; }
                src = p;
            }
            add_copy(src, dst, n.name);
            return;
        }
        case Op::Slice: {
            if (nt.mode == 2) return;   // view
            const int x = input_vid(n, 0), o = vid[n.outputs[0]];
            TView src = view(x), dst = view(o);
            const char* base = static_cast<const char*>(src.ptr);
            int64_t off = 0;
            for (int d = 0; d < src.rank; ++d) {
                off += nt.a[d] * src.stride[d];
                src.stride[d] *= nt.b[d];
                src.shape[d] = V[o].shape[d];
            }
            src.ptr = base + off * (src.dt == BF16 ? 2 : 4);
            add_copy(src, dst, n.name);
            return;
        }
        case Op::Softmax: {
            const int x = input_vid(n, 0), o = vid[n.outputs[0]];
            TView in = dense_f32(x, n.name);
            TView out = view(o);
            const auto s = V[x].shape;
            const int ax = nt.mode;
            int64_t outer = 1, inner = 1;
            for (int d = 0; d < ax; ++d) outer *= s[d];
            for (size_t d = ax + 1; d < s.size(); ++d) inner *= s[d];
            const int64_t axl = s[ax], per = numel_of(s), b = B;
            const float* ip = static_cast<const float*>(in.ptr);
            float* op = static_cast<float*>(const_cast<void*>(out.ptr));
            kind("softmax");
            add_step(n.name, [=](cudaStream_t st) { launch_softmax(ip, op, outer, axl, inner, per, b, st); });
            return;
        }
        case Op::TopK: {
            const int x = input_vid(n, 0);
            TView in = dense_f32(x, n.name);
            const auto s = V[x].shape;
            const int ax = nt.mode;
            const int64_t k = nt.a[0];
            int64_t outer = B, inner = 1;        // images are consecutive slices of dense values
            for (int d = 0; d < ax; ++d) outer *= s[d];
            for (size_t d = ax + 1; d < s.size(); ++d) inner *= s[d];
            const int64_t L = s[ax];
            TView vo = view(vid[n.outputs[0]]);
            float* ip_out = nullptr;
            if (n.outputs.size() > 1 && n.outputs[1] >= 0 && vid.count(n.outputs[1]))
                ip_out = static_cast<float*>(const_cast<void*>(view(vid[n.outputs[1]]).ptr));
            const float* ip = static_cast<const float*>(in.ptr);
            float* vp = static_cast<float*>(const_cast<void*>(vo.ptr));
            kind("topk");
            add_step(n.name, [=](cudaStream_t st) { launch_topk(ip, vp, ip_out, outer, L, inner, k, st); });
            return;
        }
        case Op::GatherElements: {
            const int x = input_vid(n, 0), ix = input_vid(n, 1);
            TView data = dense_f32(x, n.name + "/data");
            TView idx = dense_f32(ix, n.name + "/indices");
            const auto ds = V[x].shape, is = V[ix].shape;
            const int ax = nt.mode;
            int64_t outer = B, inner = 1;
            for (int d = 0; d < ax; ++d) outer *= ds[d];
            for (size_t d = ax + 1; d < ds.size(); ++d) inner *= ds[d];
            const int64_t L = ds[ax], K = is[ax];
            TView out = view(vid[n.outputs[0]]);
            const float* dp = static_cast<const float*>(data.ptr);
            const float* xp = static_cast<const float*>(idx.ptr);
            float* op = static_cast<float*>(const_cast<void*>(out.ptr));
            kind("gather_elements");
            add_step(n.name, [=](cudaStream_t st) { launch_gather_elements(dp, xp, op, outer, K, L, inner, st); });
            return;
        }
        default:
            fail(ENGINE_ERR_NOT_IMPL, std::string("op ") + op_name(n.op) + " not supported");
        }
    }

    void emit_reshape(int ni) {
        const Node& n = nodes[ni];
        const int x = input_vid(n, 0), o = vid[n.outputs[0]];
        const int mode = note[ni].mode;
        const auto is = V[x].shape;
        if (mode == 0) {
            TView src = view(x);
            // flat reinterpretation: copy the logical row-major order into the new shape
            TView flat_src = src, dst = view(o);
            if (dense(x)) {
                flat_src.rank = 1; flat_src.shape[0] = numel_of(is); flat_src.stride[0] = 1;
                TView flat_dst = dst; flat_dst.rank = 1; flat_dst.shape[0] = numel_of(is); flat_dst.stride[0] = 1;
                add_copy(flat_src, flat_dst, n.name);
            } else {
                // element order of a strided view = its logical order; copy through a dense staging view
                TView staged = dense_f32(x, n.name);
                staged.rank = 1; staged.shape[0] = numel_of(is); staged.stride[0] = 1;
                TView flat_dst = dst; flat_dst.rank = 1; flat_dst.shape[0] = numel_of(is); flat_dst.stride[0] = 1;
                add_copy(staged, flat_dst, n.name);
            }
            return;
        }
        TView src = view(x), dst = view(o);
        if (mode == 3) {
            // NHWC -> NCHW order, then flat into the target (session_ops_shape.inc:698-721)
            TView p = src;
            p.rank = 4;
            const int perm[4] = {0, 3, 1, 2};
            for (int d = 0; d < 4; ++d) { p.shape[d] = src.shape[perm[d]]; p.stride[d] = src.stride[perm[d]]; }
            TView d4 = dst;
            d4.rank = 4;
            const auto st = dense_strides({p.shape[0], p.shape[1], p.shape[2], p.shape[3]});
            for (int d = 0; d < 4; ++d) { d4.shape[d] = p.shape[d]; d4.stride[d] = st[d]; }
            add_copy(p, d4, n.name);
            return;
        }
        if (mode == 2) {
            // DFL: out[w * S + h] = in[h * W + w]  (session_ops_shape.inc:653-693)
            TView p = src;
            p.rank = 3;
            p.shape[0] = 1; p.shape[1] = is[2]; p.shape[2] = is[1];
            p.stride[0] = src.stride[0]; p.stride[1] = src.stride[2]; p.stride[2] = src.stride[1];
            add_copy(p, dst, n.name);
            return;
        }
        // mode 1: 4D -> 4D NCHW-order remap via a dense NCHW staging buffer
        const int64_t N = is[0], H = is[1], W = is[2], C = is[3];
        TView nchw = src;
        nchw.rank = 4;
        const int perm[4] = {0, 3, 1, 2};
        for (int d = 0; d < 4; ++d) { nchw.shape[d] = src.shape[perm[d]]; nchw.stride[d] = src.stride[perm[d]]; }
        TView stage = nchw;
        stage.dt = src.dt;
        const auto st = dense_strides({N, C, H, W});
        for (int d = 0; d < 4; ++d) stage.stride[d] = st[d];
        stage.img_stride = N * C * H * W;
        stage.ptr = P.alloc(std::max<size_t>((size_t)stage.img_stride * B * (src.dt == BF16 ? 2 : 4), 16));
        add_copy(nchw, stage, n.name + "/nchw");
        const auto od = V[o].shape;   // motor [N', H', W', C'] of ONNX target [N', C', H', W']
        TView in2 = stage;
        in2.shape[0] = od[0]; in2.shape[1] = od[1]; in2.shape[2] = od[2]; in2.shape[3] = od[3];
        const int64_t Ho = od[1], Wo = od[2], Co = od[3];
        in2.stride[0] = Co * Ho * Wo; in2.stride[1] = Wo; in2.stride[2] = 1; in2.stride[3] = Ho * Wo;
        add_copy(in2, dst, n.name);
    }

    void emit_conv(int ni) {
        const Node& n = nodes[ni];
        const Note& nt = note[ni];
        const int x = input_vid(n, 0), w = input_vid(n, 1);
        const int bv = n.inputs.size() > 2 ? input_vid(n, 2) : -1;
        const int o = vid[n.outputs[0]];
        const Weight& W = wt(w);
        const auto& ws = W.shape;
        int64_t Co = ws[0], Ci = ws[1];
        const int64_t KH = ws[2], KW = ws[3];
        const float* bias = nullptr;
        if (bv >= 0) {
            const Weight& bw = wt(bv);
            if (bw.numel() < Co) fail(ENGINE_ERR_INVALID_SHAPE, "conv bias shorter than Cout");
            bias = static_cast<const float*>(weight_f32(V[bv].weight));
        }
        TView in = view(x);
        if (nt.dfl_fix) {
            std::swap(in.shape[2], in.shape[3]);
            std::swap(in.stride[2], in.stride[3]);
        }
        int act = conv_act[ni];
        bool tanh_after = false;
        if (act == 100) { act = ACT_NONE; tanh_after = true; }
        if (act == ACT_SILU && reference_conv_path(Ci, KH, KW, n.params) == 1) act = ACT_SILU_WINO;
        const char* exact = std::getenv("PDEFA_EXACT_SILU");
        if (act == ACT_SILU_WINO && exact && *exact && *exact != '0') act = ACT_SILU;
        const TView out = view(o);
        const bool ext = external_of(in) == 0;
        Plan* pp = &P;
        if (nt.mode == 1) {
            // channel-major 1x1: out[co][t] = sum_ci w[co][ci] * in[ci][t] (conv2d.cpp:518-571)
            TView src = dense_f32(x, n.name);
            const int64_t HWt = numel_of(V[x].shape) / Ci;
            const float* wp = static_cast<const float*>(weight_f32(V[w].weight));
            float* op = static_cast<float*>(const_cast<void*>(out.ptr));
            const float* ip = static_cast<const float*>(src.ptr);
            const int64_t b = B, per_in = numel_of(V[x].shape), per_out = numel_of(V[o].shape);
            kind("gemm_f32");
            add_step(n.name, [=](cudaStream_t s) {
                launch_gemm_f32(wp, ip, op, nullptr, Co, HWt, Ci, Ci, HWt, HWt, b, 0, per_in, per_out, s);
            });
            if (bias || act != ACT_NONE) {
                // bias per output channel (dim 1 of the channel-major output) then activation
                TView ov = out;
                TView bb = ov; bb.ptr = bias; bb.dt = F32; bb.img_stride = 0;
                for (int d = 0; d < 4; ++d) bb.stride[d] = d == 1 ? 1 : 0;
                const int64_t bt = B;
                if (bias) add_step(n.name + "/bias", [=](cudaStream_t s) { launch_binary(BIN_ADD, ov, bb, ov, bt, s); });
                const float sl = conv_slope[ni];
                if (act != ACT_NONE) add_step(n.name + "/act", [=](cudaStream_t s) { launch_unary(act, ov, ov, bt, sl, 0, s); });
            }
            return;
        }
        ConvArgs a;
        a.in = in;
        a.out = out;
        if (conv_res[ni] >= 0) a.res = view(conv_res[ni]);
        a.bias = bias;
        a.cin = (int)Ci; a.cout = (int)Co; a.kh = (int)KH; a.kw = (int)KW;
        const int64_t groups = n.params.groups > 0 ? n.params.groups : 1;
        if (groups > 1) {
            // grouped / depthwise (conv2d.cpp:164-393): fp32 weights [Cout][kh][kw][Cin/groups]
            a.cin = (int)(Ci * groups);
            a.sh = (int)n.params.stride_h; a.sw = (int)n.params.stride_w;
            a.ph = (int)n.params.pad_h; a.pw = (int)n.params.pad_w;
            a.dh = (int)n.params.dil_h; a.dw = (int)n.params.dil_w;
            a.act = act == ACT_SILU_WINO ? ACT_SILU : act;
            a.slope = conv_slope[ni];
            a.batch = B;
            const float* wf0 = W.f32();
            std::vector<float> w0;
            if (!wf0) { w0.resize(W.numel()); for (int64_t i = 0; i < W.numel(); ++i) w0[i] = (float)W.value(i); wf0 = w0.data(); }
            std::vector<float> h((size_t)Co * KH * KW * Ci);
            for (int64_t co = 0; co < Co; ++co)
                for (int64_t ci = 0; ci < Ci; ++ci)
                    for (int64_t r = 0; r < KH; ++r)
                        for (int64_t s2 = 0; s2 < KW; ++s2)
                            h[((size_t)(co * KH + r) * KW + s2) * Ci + ci] = wf0[((co * Ci + ci) * KH + r) * KW + s2];
            void* d = P.alloc(h.size() * 4);
            if (!P.dry_) PB_CUDA(cudaMemcpy(d, h.data(), h.size() * 4, cudaMemcpyHostToDevice));
            a.weight = d;
            const int g = (int)groups;
            kind("conv_grouped");
            add_step(n.name, [a, g, ext, pp](cudaStream_t s) mutable {
                if (ext && pp->cur_in_) a.in.ptr = pp->cur_in_;
                launch_conv_grouped(a, g, s);
            });
            if (tanh_after) {
                const TView ov = out;
                const int64_t bt = B;
                add_step(n.name + "/tanh", [=](cudaStream_t s) { launch_unary(UN_TANH, ov, ov, bt, 0.0f, 0, s); });
            }
            return;
        }
        a.sh = (int)n.params.stride_h; a.sw = (int)n.params.stride_w;
        a.ph = (int)n.params.pad_h; a.pw = (int)n.params.pad_w;
        a.dh = (int)n.params.dil_h; a.dw = (int)n.params.dil_w;
        a.act = act; a.slope = conv_slope[ni];
        a.batch = B;
        const float* wf = W.f32();
        std::vector<float> wtmp;
        if (!wf) { wtmp.resize(W.numel()); for (int64_t i = 0; i < W.numel(); ++i) wtmp[i] = (float)W.value(i); wf = wtmp.data(); }
        // channels padded by pad_narrow_channels: zero weights (and bias) for them
        const int64_t Co_e = (nt.mode == 0 && !nt.dfl_fix && V[o].shape.size() == 4) ? V[o].shape[3] : Co;
        const int64_t Ci_e = (nt.mode == 0 && !nt.dfl_fix && V[x].shape.size() == 4) ? V[x].shape[3] : Ci;
        std::vector<float> wpad;
        if ((Co_e > Co || Ci_e > Ci) && Co_e >= Co && Ci_e >= Ci) {
            wpad.assign((size_t)Co_e * Ci_e * KH * KW, 0.0f);
            for (int64_t co = 0; co < Co; ++co)
                for (int64_t ci = 0; ci < Ci; ++ci)
                    for (int64_t r = 0; r < KH * KW; ++r)
                        wpad[((size_t)co * Ci_e + ci) * KH * KW + r] = wf[((size_t)co * Ci + ci) * KH * KW + r];
            if (bias && Co_e > Co) {
                std::vector<float> bp((size_t)Co_e, 0.0f);
                const Weight& bw = wt(bv);
                for (int64_t c = 0; c < Co; ++c) bp[c] = (float)bw.value(c);
                void* db = P.alloc(bp.size() * 4);
                if (!P.dry_) PB_CUDA(cudaMemcpy(db, bp.data(), bp.size() * 4, cudaMemcpyHostToDevice));
                a.bias = static_cast<const float*>(db);
            }
            wf = wpad.data();
            Co = Co_e;
            Ci = Ci_e;
            a.cin = (int)Ci; a.cout = (int)Co;
        }
        bool tc = false;
        const char* why = "fp32 precision";
        const int op_dt = prec == PREC_BF16 ? BF16 : F32;
        if (prec != PREC_FP32 && !ext) {
            a.weight = reinterpret_cast<const void*>(16);   // placeholder for the alignment check
            tc = conv_tc_supported(a, op_dt, &why);
        }
        if (prec != PREC_FP32 && !tc && Ci > 8) {
            // The input is not in the operand layout (a graph input in fp32 NCHW, or a
            // view with a channel stride): stage it once into a dense NHWC buffer of the
            // operand type and run the tensor-core path on that.
            ConvArgs t = a;
            t.weight = reinterpret_cast<const void*>(16);
            t.in.dt = op_dt;
            const int64_t H = in.shape[1], Wd = in.shape[2];
            t.in.rank = 4;
            t.in.stride[3] = 1; t.in.stride[2] = Ci; t.in.stride[1] = Wd * Ci; t.in.stride[0] = H * Wd * Ci;
            t.in.img_stride = H * Wd * Ci;
            t.in.ptr = reinterpret_cast<const void*>(256);
            const char* why2 = nullptr;
            if (conv_tc_supported(t, op_dt, &why2)) {
                t.in.ptr = P.alloc(std::max<size_t>((size_t)t.in.img_stride * B * (op_dt == BF16 ? 2 : 4), 16));
                add_copy(in, t.in, n.name + "/stage");
                a = t;
                tc = true;
            }
        }
        if (tc) {
            const int64_t K = KH * KW * Ci;
            void* d = P.alloc((size_t)Co * K * (op_dt == BF16 ? 2 : 4));
            if (op_dt == BF16) {
                std::vector<uint16_t> h((size_t)Co * K);
                for (int64_t co = 0; co < Co; ++co)
                    for (int64_t r = 0; r < KH; ++r)
                        for (int64_t s = 0; s < KW; ++s)
                            for (int64_t ci = 0; ci < Ci; ++ci)
                                h[(size_t)co * K + (r * KW + s) * Ci + ci] = f2bf(wf[((co * Ci + ci) * KH + r) * KW + s]);
                if (!P.dry_) PB_CUDA(cudaMemcpy(d, h.data(), h.size() * 2, cudaMemcpyHostToDevice));
            } else {
                std::vector<float> h((size_t)Co * K);
                for (int64_t co = 0; co < Co; ++co)
                    for (int64_t r = 0; r < KH; ++r)
                        for (int64_t s = 0; s < KW; ++s)
                            for (int64_t ci = 0; ci < Ci; ++ci)
                                h[(size_t)co * K + (r * KW + s) * Ci + ci] = wf[((co * Ci + ci) * KH + r) * KW + s];
                if (!P.dry_) PB_CUDA(cudaMemcpy(d, h.data(), h.size() * 4, cudaMemcpyHostToDevice));
            }
            a.weight = d;
            int* err = P.err_;
            a.wait_limit = P.wait_limit_;
            kind(op_dt == BF16 ? "conv_tc_bf16" : "conv_tc_tf32");
            add_step(n.name, [a, op_dt, err](cudaStream_t s) { launch_conv_tc(a, op_dt, err, s); });
        } else {
            if (verbose() && prec != PREC_FP32)
                std::fprintf(stderr, "[pdefa-b200] conv '%s' on SIMT path: %s\n", n.name.c_str(), why);
            std::vector<float> h((size_t)KH * KW * Ci * Co);
            for (int64_t co = 0; co < Co; ++co)
                for (int64_t ci = 0; ci < Ci; ++ci)
                    for (int64_t r = 0; r < KH; ++r)
                        for (int64_t s = 0; s < KW; ++s)
                            h[((size_t)(r * KW + s) * Ci + ci) * Co + co] = wf[((co * Ci + ci) * KH + r) * KW + s];
            void* d = P.alloc(h.size() * 4);
            if (!P.dry_) PB_CUDA(cudaMemcpy(d, h.data(), h.size() * 4, cudaMemcpyHostToDevice));
            a.weight = d;
            if (prec == PREC_BF16 && conv_stem_tc_supported(a)) {
                int* err = P.err_;
                const bool u8 = ext && P.u8_scale_ > 0.0f;
                if (u8 && !(a.kh == 3 && a.kw == 3 && a.cin == 3 && a.sh == 2 && a.sw == 2 && a.ph == 1 && a.pw == 1 &&
                            a.dh == 1 && a.dw == 1 && a.in.shape[2] % 4 == 0))
                    fail(ENGINE_ERR_NOT_IMPL, "8-bit input needs a 3x3 stride-2 RGB stem with width % 4 == 0");
                if (u8) {
                    a.in_u8 = reinterpret_cast<const uint8_t*>(P.inputs_[0]);
                    a.in_u8_scale = P.u8_scale_;
                    u8_stem = true;
                }
                kind("conv_stem_tc");
                add_step(n.name, [a, ext, u8, pp, err](cudaStream_t s) mutable {
                    if (ext && pp->cur_in_) {
                        if (u8) a.in_u8 = reinterpret_cast<const uint8_t*>(pp->cur_in_);
                        else a.in.ptr = pp->cur_in_;
                    }
                    launch_conv_stem_tc(a, err, s);
                });
            } else if (conv_direct_supported(a)) {
                kind("conv_direct");
                add_step(n.name, [a, ext, pp](cudaStream_t s) mutable {
                    if (ext && pp->cur_in_) a.in.ptr = pp->cur_in_;
                    launch_conv_direct(a, s);
                });
            } else {
                kind("conv_simt");
                add_step(n.name, [a, ext, pp](cudaStream_t s) mutable {
                    if (ext && pp->cur_in_) a.in.ptr = pp->cur_in_;
                    launch_conv_simt(a, s);
                });
            }
        }
        if (tanh_after) {
            const int64_t bt = B;
            add_step(n.name + "/tanh", [out, bt](cudaStream_t s) { launch_unary(UN_TANH, out, out, bt, 0, 0, s); });
        }
    }

    void emit_matmul(int ni) {
        const Node& n = nodes[ni];
        const int a = input_vid(n, 0), w = input_vid(n, 1), o = vid[n.outputs[0]];
        const int bv = n.inputs.size() > 2 ? input_vid(n, 2) : -1;
        TView O = view(o);
        const auto as = V[a].shape;
        const auto wsh = V[w].shape;
        if (note[ni].mode == 2) {
            const int64_t M = as[1], K = as[2], N = wsh[2], H = as[3];
            if (as[0] != 1) fail(ENGINE_ERR_NOT_IMPL, "MatMul '" + n.name + "': batched 4-D product with a leading dimension > 1");
            const bool odense = dense(o) && V[o].dt == F32;
            float* op = static_cast<float*>(const_cast<void*>(O.ptr));
            float* tmp = odense ? op : static_cast<float*>(P.alloc(std::max<size_t>((size_t)B * M * N * H * 4, 16)));
            // operand views: the value itself, or the input of a folded Transpose with its
            // dimensions permuted
            auto operand = [&](int v) {
                TView t;
                auto it = folded_transpose.find(v);
                if (it != folded_transpose.end()) {
                    const Node& tn = nodes[it->second];
                    const TView src = view(input_vid(tn, 0));
                    t = src;
                    for (int d = 0; d < 4; ++d) { t.shape[d] = src.shape[note[it->second].a[d]]; t.stride[d] = src.stride[note[it->second].a[d]]; }
                } else {
                    t = view(v);
                }
                HeadOperand h;
                h.p = t.ptr;
                h.bf = t.dt == BF16;
                h.s1 = t.stride[1]; h.s2 = t.stride[2]; h.s3 = t.stride[3];
                h.sb = t.img_stride;
                return h;
            };
            const HeadOperand ha = operand(a), hb = operand(w);
            const float scale = note[ni].scale;
            const int64_t nb = B;
            kind("matmul_heads");
            add_step(n.name, [=](cudaStream_t s) {
                launch_matmul_heads(ha, hb, tmp, nb, M, K, N, H, scale, M * N * H, s);
            });
            if (!odense) {
                TView src = O;
                src.ptr = tmp; src.dt = F32;
                const auto st = dense_strides(V[o].shape);
                for (int d = 0; d < src.rank; ++d) src.stride[d] = st[d];
                src.img_stride = numel_of(V[o].shape);
                add_copy(src, O, n.name + "/store");
            }
            return;
        }
        TView A = dense_f32(a, n.name + "/a");
        TView Wt = dense_f32(w, n.name + "/b");
        int64_t M, K = wsh[0], N = wsh[1];
        if (note[ni].mode == 1) M = as[0] * as[1] * as[2]; else M = as[0];
        const float* bias = nullptr;
        if (bv >= 0 && numel_of(V[bv].shape) == N) bias = static_cast<const float*>(weight_f32(V[bv].weight));
        const bool odense = dense(o) && V[o].dt == F32;
        float* op = static_cast<float*>(const_cast<void*>(O.ptr));
        float* tmp = op;
        if (!odense) tmp = static_cast<float*>(P.alloc(std::max<size_t>((size_t)M * N * B * 4, 16)));
        const float* ap = static_cast<const float*>(A.ptr);
        const float* bp = static_cast<const float*>(Wt.ptr);
        const int64_t b = B, sa = A.img_stride, sb = Wt.img_stride;
        kind("gemm_f32");
        add_step(n.name, [=](cudaStream_t s) { launch_gemm_f32(ap, bp, tmp, bias, M, N, K, K, N, N, b, sa, sb, M * N, s); });
        if (!odense) {
            TView src = O;
            src.ptr = tmp; src.dt = F32;
            const auto st = dense_strides(V[o].shape);
            for (int d = 0; d < src.rank; ++d) src.stride[d] = st[d];
            src.img_stride = numel_of(V[o].shape);
            add_copy(src, O, n.name + "/store");
        }
    }

    void build() {
        // Value slots are reserved up front: references into V must stay valid while
        // later values are created.
        size_t slots = g.weights.size() + g.inputs.size() + 16;
        for (const Node& n : g.nodes) slots += n.outputs.size() + n.inputs.size();
        V.reserve(slots);
        fuse();
        infer();
        match_head();
        fuse_residuals();
        fold_attention();
        pad_narrow_channels();
        place();
        emit();
        if (verbose()) {
            std::fprintf(stderr, "[pdefa-b200] plan: batch=%lld precision=%d steps=%zu\n", (long long)B, prec,
                         P.steps_.size());
            for (size_t i = 0; i < V.size(); ++i) {
                if (!V[i].known || V[i].weight >= 0) continue;
                std::fprintf(stderr, "  v%zu %s dt=%d alias=%d place=%d+%lld\n", i, shape_str(V[i].shape).c_str(),
                             V[i].dt, V[i].alias_of, V[i].place_in, (long long)V[i].place_ch);
            }
        }
    }
};

Plan::Plan(std::shared_ptr<const Graph> g, int64_t batch, int precision, int device, std::vector<int32_t> keep,
           std::vector<int64_t> in_shape, float in_u8_scale)
    : g_(std::move(g)), batch_(batch), prec_(precision), device_(device), keep_(std::move(keep)),
      in_shape_(std::move(in_shape)), u8_scale_(in_u8_scale) {
    require_device(device);
    if (batch < 1) fail(ENGINE_ERR_INVALID_ARG, "batch must be >= 1");
    PB_CUDA(cudaSetDevice(device));
    try {
        build();
    } catch (...) {
        for (void* p : allocs_) cudaFree(p);
        allocs_.clear();
        throw;
    }
}

Plan::Plan(DryTag, std::shared_ptr<const Graph> g, int64_t batch, int precision, std::vector<int32_t> keep,
           std::vector<int64_t> in_shape, float in_u8_scale)
    : g_(std::move(g)), dry_(true), batch_(batch), prec_(precision), device_(0), keep_(std::move(keep)),
      in_shape_(std::move(in_shape)), u8_scale_(in_u8_scale) {
    if (batch < 1) fail(ENGINE_ERR_INVALID_ARG, "batch must be >= 1");
    build();
}

std::unique_ptr<Plan> Plan::dry_run(std::shared_ptr<const Graph> g, int64_t batch, int precision) {
    return std::unique_ptr<Plan>(new Plan(DryTag{}, std::move(g), batch, precision));
}

std::string Plan::summary() const {
    std::string r;
    for (const auto& s : steps_) r += s.kind + " " + s.name + "\n";
    return r;
}

Plan::~Plan() {
    if (dry_) return;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(device_);
    for (auto& p : pending_) { cudaEventDestroy(p.second.first); cudaEventDestroy(p.second.second); }
    for (auto e : ev_pool_) cudaEventDestroy(e);
    if (gexec_) cudaGraphExecDestroy(gexec_);
    for (void* p : allocs_) cudaFree(p);
    if (err_host_) cudaFreeHost(err_host_);
    cudaSetDevice(prev);
}

int Plan::take_error() {
    if (dry_ || !err_host_) return 0;
    const int v = *reinterpret_cast<volatile int*>(err_host_);
    if (v) {
        PB_CUDA(cudaSetDevice(device_));
        PB_CUDA(cudaMemset(err_, 0, sizeof(int)));
        *err_host_ = 0;
    }
    return v;
}

void* Plan::alloc(size_t bytes) {
    if (dry_) {
        void* p = reinterpret_cast<void*>(dry_next_);
        dry_next_ += (bytes + 1023) & ~size_t(1023);
        return p;
    }
    void* p = nullptr;
    const cudaError_t e = cudaMalloc(&p, (bytes + 255) & ~size_t(255));
    if (e != cudaSuccess) {
        cudaGetLastError();
        fail(ENGINE_ERR_OUT_OF_MEMORY, std::string("device allocation failed: ") + cudaGetErrorString(e));
    }
    allocs_.push_back(p);
    return p;
}

// Offsets of the arena roots: largest first, each at the lowest 256-byte aligned
// offset that overlaps no already placed root whose node range intersects its own.
// first/last: node range per value id; bytes: 0 for values that are not roots.
std::vector<size_t> pack_arena(const std::vector<size_t>& bytes, const std::vector<int>& first,
                               const std::vector<int>& last, size_t* total) {
    std::vector<size_t> off(bytes.size(), SIZE_MAX);
    std::vector<int> ids;
    for (size_t v = 0; v < bytes.size(); ++v)
        if (bytes[v] > 0 && v < first.size() && first[v] <= last[v]) ids.push_back((int)v);
    std::stable_sort(ids.begin(), ids.end(), [&](int a, int b) {
        return bytes[a] != bytes[b] ? bytes[a] > bytes[b] : first[a] < first[b];
    });
    struct Placed { size_t lo, hi; int first, last; };
    std::vector<Placed> placed;
    size_t top = 0;
    for (int v : ids) {
        const size_t need = (bytes[v] + 255) & ~size_t(255);
        std::vector<std::pair<size_t, size_t>> busy;
        for (const Placed& p : placed)
            if (p.first <= last[v] && first[v] <= p.last) busy.push_back({p.lo, p.hi});
        std::sort(busy.begin(), busy.end());
        size_t at = 0;
        for (const auto& b : busy) {
            if (at + need <= b.first) break;
            at = std::max(at, b.second);
        }
        off[v] = at;
        placed.push_back({at, at + need, first[v], last[v]});
        top = std::max(top, at + need);
    }
    // self-check: roots live at the same time never share a byte
    for (size_t i = 0; i < placed.size(); ++i)
        for (size_t j = i + 1; j < placed.size(); ++j) {
            const Placed& a = placed[i];
            const Placed& b = placed[j];
            if (a.first <= b.last && b.first <= a.last && a.lo < b.hi && b.lo < a.hi)
                fail(ENGINE_ERR_RUNTIME, "memory plan: overlapping live buffers");
        }
    *total = top;
    return off;
}

void Plan::build() {
    if (!dry_) {
        if (const char* w = std::getenv("PDEFA_WAIT_LIMIT_CYCLES")) wait_limit_ = std::atoll(w);
        err_ = static_cast<int*>(alloc(sizeof(int)));
        PB_CUDA(cudaMemset(err_, 0, sizeof(int)));
        PB_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&err_host_), sizeof(int), cudaHostAllocDefault));
        *err_host_ = 0;
    }
    if (dry_ || std::getenv("PDEFA_NO_ARENA") != nullptr) {
        PlanBuilder b(*this, *g_);
        b.build();
        if (!dry_) activation_bytes_ = 0;
        for (size_t v = 0; v < root_bytes_.size(); ++v) activation_bytes_ += root_bytes_[v];
        return;
    }
    // A dry lowering of the same graph records every root's size and node range; the
    // real lowering then places the roots in one arena at packed offsets.
    Plan probe(DryTag{}, g_, batch_, prec_, keep_, in_shape_, u8_scale_);
    size_t total = 0;
    const std::vector<size_t> off = pack_arena(probe.root_bytes_, probe.root_first_, probe.root_last_, &total);
    char* base = static_cast<char*>(alloc(std::max<size_t>(total, 256)));
    PlanBuilder b(*this, *g_);
    b.arena_off = &off;
    b.arena = base;
    b.build();
    activation_bytes_ = total;
    unpacked_bytes_ = probe.activation_bytes_;
}

void Plan::run_steps(cudaStream_t s) {
    for (size_t i = 0; i < steps_.size(); ++i) {
        if (timing_) {
            cudaEvent_t a = take_event(), b = take_event();
            PB_CUDA(cudaEventRecord(a, s));
            steps_[i].run(s);
            PB_CUDA(cudaEventRecord(b, s));
            pending_.push_back({(int)i, {a, b}});
        } else {
            steps_[i].run(s);
        }
    }
}

void Plan::run(cudaStream_t s, const float* in_override, float* out_override) {
    (void)out_override;
    run_launches(s, in_override);
    enqueue_error_copy(s);
}

void Plan::enqueue_error_copy(cudaStream_t s) {
    // the plan's error word reaches the host with the stream's other results
    if (err_host_) PB_CUDA(cudaMemcpyAsync(err_host_, err_, sizeof(int), cudaMemcpyDeviceToHost, s));
}

void Plan::run_launches(cudaStream_t s, const float* in_override) {
    cur_in_ = in_override;
    struct Reset { const float*& p; ~Reset() { p = nullptr; } } reset{cur_in_};
    // Eager: timed runs, the legacy default stream (cannot be captured), the first run.
    if (timing_ || !graphs_ || s == nullptr || eager_runs_ < 1) {
        run_steps(s);
        if (!timing_) ++eager_runs_;
        return;
    }
    if (gexec_ && g_in_ == in_override) {
        PB_CUDA(cudaGraphLaunch(gexec_, s));
        return;
    }
    if (gexec_) {
        cudaGraphExecDestroy(gexec_);
        gexec_ = nullptr;
    }
    // Capture the launch sequence (kernel parameters, tensor maps included, are
    // copied into the graph), then replay it. Any failure falls back to eager runs.
    cudaGraph_t graph = nullptr;
    if (cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
        cudaGetLastError();
        graphs_ = false;
        run_steps(s);
        return;
    }
    try {
        run_steps(s);
    } catch (...) {
        cudaStreamEndCapture(s, &graph);
        if (graph) cudaGraphDestroy(graph);
        cudaGetLastError();
        throw;
    }
    cudaError_t e = cudaStreamEndCapture(s, &graph);
    if (e == cudaSuccess) e = cudaGraphInstantiate(&gexec_, graph, 0);
    if (graph) cudaGraphDestroy(graph);
    if (e != cudaSuccess) {
        cudaGetLastError();
        gexec_ = nullptr;
        graphs_ = false;
        run_steps(s);
        return;
    }
    g_in_ = in_override;
    PB_CUDA(cudaGraphLaunch(gexec_, s));
}

cudaEvent_t Plan::take_event() {
    if (ev_pool_.empty()) {
        cudaEvent_t e;
        PB_CUDA(cudaEventCreate(&e));
        return e;
    }
    cudaEvent_t e = ev_pool_.back();
    ev_pool_.pop_back();
    return e;
}

std::vector<double> Plan::collect_step_ms() {
    step_ms_.resize(steps_.size(), 0.0);
    for (auto& p : pending_) {
        PB_CUDA(cudaEventSynchronize(p.second.second));
        float ms = 0.0f;
        PB_CUDA(cudaEventElapsedTime(&ms, p.second.first, p.second.second));
        step_ms_[p.first] += ms;
        ev_pool_.push_back(p.second.first);
        ev_pool_.push_back(p.second.second);
    }
    pending_.clear();
    return step_ms_;
}

int64_t Plan::launch_count() const {
    int64_t n = 0;
    for (auto& s : steps_) n += s.launches;
    return n;
}

}  // namespace pb
