"""Synthetic YOLOv8 ``.engine`` graphs with seeded random weights.

The graphs use the node patterns that ``pdefa/tools/onnx_to_engine.py`` emits for
an Ultralytics YOLOv8 ONNX export, so the reference CPU engine and this library
run the same file:

* ``Conv`` (BN folded into the bias) -> ``Sigmoid`` -> ``Mul``: the SiLU pattern
  the reference fuses (``PDEFA1.0/src/core/session_parts/session_fusion.inc:33-81``);
* C2f ``chunk(2)`` as two ``Slice`` nodes with float32 starts/ends/axes weights
  (the converter's Split rewrite, ``onnx_to_engine.py:216-268``);
* ``Resize`` nearest x2 with a 4-element scales constant;
* head: per level ``Concat``, ``Reshape [1,no,-1]``, ``Concat axis 2``, ``Slice``
  split, DFL ``Reshape -> Transpose(0,2,1,3) + perm weight -> Softmax(1) ->
  Conv 1x1 (arange weights) -> Reshape``, anchor decode ``Sub/Add/Add/Div/Sub``,
  ``Concat``, ``Mul`` by strides, cls ``Sigmoid``, final ``Concat`` -> [1,84,A].

Architecture: Ultralytics yolov8.yaml with depth/width/max-channel scales;
weights He-normal (std sqrt(2/fan_in)), biases N(0, 0.1), one numpy
``default_rng([seed, weight_index])`` stream per tensor.
"""
from __future__ import annotations

import math
from typing import Dict, List, Tuple

import numpy as np

from .engine_file import EngineGraph, TensorInfo, write_engine

SCALES = {  # depth, width, max_channels
    'n': (0.33, 0.25, 1024), 's': (0.33, 0.50, 1024), 'm': (0.67, 0.75, 768),
    'l': (1.00, 1.00, 512), 'x': (1.00, 1.25, 512),
}


def _make_div(x: float, d: int = 8) -> int:
    return int(math.ceil(x / d) * d)


class _Builder:
    def __init__(self, seed: int):
        self.g = EngineGraph()
        self.seed = seed
        self.n_rand = 0
        self.convs: List[Tuple] = []   # (name, cin, cout, k, s, hin, win) for FLOP accounting
        self.groups: Dict[str, int] = {}

    def rand_weight(self, name, shape, std):
        rng = np.random.default_rng([self.seed, self.n_rand])
        self.n_rand += 1
        return self.g.add_weight(name, rng.standard_normal(shape) * std)

    def const(self, name, arr):
        return self.g.add_weight(name, np.asarray(arr, dtype=np.float32))

    # -- layers ---------------------------------------------------------
    def conv(self, x, shp, cout, k, s, name, act=True, bias=True, groups=1):
        cin, h, w = shp
        p = k // 2
        cg = cin // groups
        wi = self.rand_weight(f"{name}.weight", (cout, cg, k, k), math.sqrt(2.0 / (cg * k * k)))
        ins = [x, wi]
        if bias:
            ins.append(self.rand_weight(f"{name}.bias", (cout,), 0.1))
        (y,) = self.g.add_node('Conv2d', f"/{name}/conv/Conv", ins,
                               stride_h=s, stride_w=s, pad_h=p, pad_w=p, groups=groups)
        ho, wo = (h + 2 * p - k) // s + 1, (w + 2 * p - k) // s + 1
        self.convs.append((name, cin, cout, k, s, h, w))
        if groups != 1:
            self.groups[name] = groups
        if act:
            (sg,) = self.g.add_node('Sigmoid', f"/{name}/act/Sigmoid", [y])
            (y,) = self.g.add_node('Mul', f"/{name}/act/Mul", [y, sg])
        return y, (cout, ho, wo)

    def slice(self, x, start, end, axis, name):
        ins = [x, self.const(f"{name}_start", [start]), self.const(f"{name}_end", [end]),
               self.const(f"{name}_axis", [axis])]
        (y,) = self.g.add_node('Slice', name, ins)
        return y

    def concat(self, xs, axis, name):
        (y,) = self.g.add_node('Concat', name, xs, axis=axis)
        return y

    def c2f(self, x, shp, c2, n, shortcut, name):
        c = int(c2 * 0.5)
        y, s1 = self.conv(x, shp, 2 * c, 1, 1, f"{name}/cv1")
        _, h, w = s1
        ys = [self.slice(y, 0, c, 1, f"/{name}/Split_slice_0"),
              self.slice(y, c, 2 * c, 1, f"/{name}/Split_slice_1")]
        for i in range(n):
            src = ys[-1]
            t, ts = self.conv(src, (c, h, w), c, 3, 1, f"{name}/m.{i}/cv1")
            t, ts = self.conv(t, ts, c, 3, 1, f"{name}/m.{i}/cv2")
            if shortcut:
                (t,) = self.g.add_node('Add', f"/{name}/m.{i}/Add", [src, t])
            ys.append(t)
        cat = self.concat(ys, 1, f"/{name}/Concat")
        return self.conv(cat, ((2 + n) * c, h, w), c2, 1, 1, f"{name}/cv2")

    def sppf(self, x, shp, c2, k, name):
        c_ = shp[0] // 2
        y, s1 = self.conv(x, shp, c_, 1, 1, f"{name}/cv1")
        outs = [y]
        for i in range(3):
            (m,) = self.g.add_node('MaxPool2d', f"/{name}/m_{i}/MaxPool", [outs[-1]],
                                   kernel_h=k, kernel_w=k, stride_h=1, stride_w=1,
                                   pad_h=k // 2, pad_w=k // 2)
            outs.append(m)
        cat = self.concat(outs, 1, f"/{name}/Concat")
        return self.conv(cat, (4 * c_, s1[1], s1[2]), c2, 1, 1, f"{name}/cv2")

    # -- YOLO11 blocks (ultralytics/nn/modules/block.py: C3k2, C3k, C2PSA, PSABlock, Attention)
    def bottleneck(self, x, shp, c2, shortcut, e, name):
        c_ = int(c2 * e)
        t, ts = self.conv(x, shp, c_, 3, 1, f"{name}/cv1")
        t, ts = self.conv(t, ts, c2, 3, 1, f"{name}/cv2")
        if shortcut and shp[0] == c2:
            (t,) = self.g.add_node('Add', f"/{name}/Add", [x, t])
        return t, ts

    def c3k(self, x, shp, c2, n, shortcut, name, e=0.5):
        c_ = int(c2 * e)
        a, sa = self.conv(x, shp, c_, 1, 1, f"{name}/cv1")
        for i in range(n):
            a, sa = self.bottleneck(a, sa, c_, shortcut, 1.0, f"{name}/m/m.{i}")
        bb, _ = self.conv(x, shp, c_, 1, 1, f"{name}/cv2")
        cat = self.concat([a, bb], 1, f"/{name}/Concat")
        return self.conv(cat, (2 * c_, sa[1], sa[2]), c2, 1, 1, f"{name}/cv3")

    def c3k2(self, x, shp, c2, n, c3k, e, name, shortcut=True):
        c = int(c2 * e)
        y, s1 = self.conv(x, shp, 2 * c, 1, 1, f"{name}/cv1")
        _, h, w = s1
        ys = [self.slice(y, 0, c, 1, f"/{name}/Split_slice_0"),
              self.slice(y, c, 2 * c, 1, f"/{name}/Split_slice_1")]
        for i in range(n):
            if c3k:
                t, _ = self.c3k(ys[-1], (c, h, w), c, 2, shortcut, f"{name}/m.{i}")
            else:
                t, _ = self.bottleneck(ys[-1], (c, h, w), c, shortcut, 0.5, f"{name}/m.{i}")
            ys.append(t)
        cat = self.concat(ys, 1, f"/{name}/Concat")
        return self.conv(cat, ((2 + n) * c, h, w), c2, 1, 1, f"{name}/cv2")

    def attention(self, x, shp, num_heads, attn_ratio, name):
        """Attention.forward as exported: Reshape [1, nh, 2kd+hd, N], Split on axis 2,
        Transpose(0,1,3,2), MatMul, Mul(scale), Softmax(-1), Transpose, MatMul,
        Reshape [1, C, H, W] + pe(depthwise 3x3 of v) -> proj."""
        c, h, w = shp
        hd = c // num_heads
        kd = int(hd * attn_ratio)
        nn_ = h * w
        qkv, _ = self.conv(x, shp, c + 2 * kd * num_heads, 1, 1, f"{name}/qkv", act=False)
        g = self.g
        (r,) = g.add_node('Reshape', f"/{name}/Reshape", [qkv, self.const(f"/{name}/Reshape_shape",
                                                                          [1, num_heads, 2 * kd + hd, nn_])])
        q = self.slice(r, 0, kd, 2, f"/{name}/Split_slice_0")
        k = self.slice(r, kd, 2 * kd, 2, f"/{name}/Split_slice_1")
        v = self.slice(r, 2 * kd, 2 * kd + hd, 2, f"/{name}/Split_slice_2")
        perm = lambda t: self.const(f"/{name}/{t}::perm", [0, 1, 3, 2])   # noqa: E731
        (qt,) = g.add_node('Transpose', f"/{name}/Transpose", [q, perm("Transpose")])
        (a,) = g.add_node('MatMul', f"/{name}/MatMul", [qt, k])
        (a,) = g.add_node('Mul', f"/{name}/Mul", [a, self.const(f"/{name}/Constant_scale", [kd ** -0.5])])
        (a,) = g.add_node('Softmax', f"/{name}/Softmax", [a], axis=-1)
        (at,) = g.add_node('Transpose', f"/{name}/Transpose_1", [a, perm("Transpose_1")])
        (o,) = g.add_node('MatMul', f"/{name}/MatMul_1", [v, at])
        (o,) = g.add_node('Reshape', f"/{name}/Reshape_1", [o, self.const(f"/{name}/Reshape_1_shape", [1, c, h, w])])
        (vr,) = g.add_node('Reshape', f"/{name}/Reshape_2", [v, self.const(f"/{name}/Reshape_2_shape", [1, c, h, w])])
        pe, _ = self.conv(vr, shp, c, 3, 1, f"{name}/pe", act=False, groups=c)
        (o,) = g.add_node('Add', f"/{name}/Add", [o, pe])
        return self.conv(o, shp, c, 1, 1, f"{name}/proj", act=False)

    def c2psa(self, x, shp, c2, n, name, e=0.5):
        c = int(shp[0] * e)
        y, s1 = self.conv(x, shp, 2 * c, 1, 1, f"{name}/cv1")
        _, h, w = s1
        a = self.slice(y, 0, c, 1, f"/{name}/Split_slice_0")
        t = self.slice(y, c, 2 * c, 1, f"/{name}/Split_slice_1")
        for i in range(n):
            blk = f"{name}/m/m.{i}"
            at, _ = self.attention(t, (c, h, w), max(c // 64, 1), 0.5, f"{blk}/attn")
            (t,) = self.g.add_node('Add', f"/{blk}/Add", [t, at])
            f1, fs = self.conv(t, (c, h, w), 2 * c, 1, 1, f"{blk}/ffn/ffn.0")
            f2, _ = self.conv(f1, fs, c, 1, 1, f"{blk}/ffn/ffn.1", act=False)
            (t,) = self.g.add_node('Add', f"/{blk}/Add_1", [t, f2])
        cat = self.concat([a, t], 1, f"/{name}/Concat")
        return self.conv(cat, (2 * c, h, w), shp[0], 1, 1, f"{name}/cv2")

    def upsample(self, x, shp, name):
        sc = self.const(f"{name}_scales", [1.0, 1.0, 2.0, 2.0])
        (y,) = self.g.add_node('Resize', f"/{name}/Resize", [x, sc])
        return y, (shp[0], shp[1] * 2, shp[2] * 2)


def build_yolov8(scale: str = 'n', imgsz: int = 640, nc: int = 80, seed: int = 0,
                 reg_max: int = 16) -> Tuple[EngineGraph, Dict]:
    """Return (graph, info) for a random-init YOLOv8 of the given scale.

    ``info`` holds the conv list (for FLOP/byte accounting), the anchor count and
    the output shape.
    """
    if imgsz % 32:
        raise ValueError("imgsz must be a multiple of 32")
    depth, width, mc = SCALES[scale]
    ch = lambda c: _make_div(min(c, mc) * width, 8)      # noqa: E731
    dp = lambda n: max(round(n * depth), 1)              # noqa: E731
    b = _Builder(seed)
    g = b.g
    x = -1
    g.graph_inputs = [-1]
    g.input_infos = [TensorInfo("images", [1, 3, imgsz, imgsz])]
    s = (3, imgsz, imgsz)
    x0, s = b.conv(x, s, ch(64), 3, 2, "model.0")
    x1, s = b.conv(x0, s, ch(128), 3, 2, "model.1")
    x2, s = b.c2f(x1, s, ch(128), dp(3), True, "model.2")
    x3, s = b.conv(x2, s, ch(256), 3, 2, "model.3")
    x4, s4 = b.c2f(x3, s, ch(256), dp(6), True, "model.4")
    x5, s = b.conv(x4, s4, ch(512), 3, 2, "model.5")
    x6, s6 = b.c2f(x5, s, ch(512), dp(6), True, "model.6")
    x7, s = b.conv(x6, s6, ch(1024), 3, 2, "model.7")
    x8, s = b.c2f(x7, s, ch(1024), dp(3), True, "model.8")
    x9, s9 = b.sppf(x8, s, ch(1024), 5, "model.9")
    x10, s = b.upsample(x9, s9, "model.10")
    x11 = b.concat([x10, x6], 1, "/model.11/Concat")
    x12, s12 = b.c2f(x11, (s[0] + s6[0], s[1], s[2]), ch(512), dp(3), False, "model.12")
    x13, s = b.upsample(x12, s12, "model.13")
    x14 = b.concat([x13, x4], 1, "/model.14/Concat")
    x15, s15 = b.c2f(x14, (s[0] + s4[0], s[1], s[2]), ch(256), dp(3), False, "model.15")
    x16, s = b.conv(x15, s15, ch(256), 3, 2, "model.16")
    x17 = b.concat([x16, x12], 1, "/model.17/Concat")
    x18, s18 = b.c2f(x17, (s[0] + s12[0], s[1], s[2]), ch(512), dp(3), False, "model.18")
    x19, s = b.conv(x18, s18, ch(512), 3, 2, "model.19")
    x20 = b.concat([x19, x9], 1, "/model.20/Concat")
    x21, s21 = b.c2f(x20, (s[0] + s9[0], s[1], s[2]), ch(1024), dp(3), False, "model.21")

    levels = [(x15, s15, 8), (x18, s18, 16), (x21, s21, 32)]
    out, A = _detect(b, levels, nc, reg_max, dw_cls=False)
    info = dict(convs=b.convs, anchors=A, nc=nc, reg_max=reg_max, scale=scale, imgsz=imgsz,
                levels=[(si[1], si[2], st) for _, si, st in levels])
    return g, info


SCALES_11 = {  # depth, width, max_channels (yolo11.yaml)
    'n': (0.50, 0.25, 1024), 's': (0.50, 0.50, 1024), 'm': (0.50, 1.00, 512),
    'l': (1.00, 1.00, 512), 'x': (1.00, 1.50, 512),
}


def build_yolo11(scale: str = 'n', imgsz: int = 640, nc: int = 80, seed: int = 0,
                 reg_max: int = 16) -> Tuple[EngineGraph, Dict]:
    """(graph, info) for a random-init YOLO11 (Ultralytics yolo11.yaml): C3k2 blocks,
    SPPF, C2PSA attention at P5, and the Detect head with depthwise class branches.
    C3k2 uses C3k inner blocks where the yaml says so (and for every C3k2 of the
    m/l/x scales), as the Ultralytics model parser does."""
    if imgsz % 32:
        raise ValueError("imgsz must be a multiple of 32")
    depth, width, mc = SCALES_11[scale]
    ch = lambda c: _make_div(min(c, mc) * width, 8)      # noqa: E731
    dp = lambda n: max(round(n * depth), 1)              # noqa: E731
    big = scale in "mlx"
    b = _Builder(seed)
    g = b.g
    g.graph_inputs = [-1]
    g.input_infos = [TensorInfo("images", [1, 3, imgsz, imgsz])]
    s = (3, imgsz, imgsz)
    x0, s = b.conv(-1, s, ch(64), 3, 2, "model.0")
    x1, s = b.conv(x0, s, ch(128), 3, 2, "model.1")
    x2, s = b.c3k2(x1, s, ch(256), dp(2), big, 0.25, "model.2")
    x3, s = b.conv(x2, s, ch(256), 3, 2, "model.3")
    x4, s4 = b.c3k2(x3, s, ch(512), dp(2), big, 0.25, "model.4")
    x5, s = b.conv(x4, s4, ch(512), 3, 2, "model.5")
    x6, s6 = b.c3k2(x5, s, ch(512), dp(2), True, 0.5, "model.6")
    x7, s = b.conv(x6, s6, ch(1024), 3, 2, "model.7")
    x8, s = b.c3k2(x7, s, ch(1024), dp(2), True, 0.5, "model.8")
    x9, s = b.sppf(x8, s, ch(1024), 5, "model.9")
    x10, s10 = b.c2psa(x9, s, ch(1024), dp(2), "model.10")
    x11, s = b.upsample(x10, s10, "model.11")
    x12 = b.concat([x11, x6], 1, "/model.12/Concat")
    x13, s13 = b.c3k2(x12, (s[0] + s6[0], s[1], s[2]), ch(512), dp(2), big, 0.5, "model.13")
    x14, s = b.upsample(x13, s13, "model.14")
    x15 = b.concat([x14, x4], 1, "/model.15/Concat")
    x16, s16 = b.c3k2(x15, (s[0] + s4[0], s[1], s[2]), ch(256), dp(2), big, 0.5, "model.16")
    x17, s = b.conv(x16, s16, ch(256), 3, 2, "model.17")
    x18 = b.concat([x17, x13], 1, "/model.18/Concat")
    x19, s19 = b.c3k2(x18, (s[0] + s13[0], s[1], s[2]), ch(512), dp(2), big, 0.5, "model.19")
    x20, s = b.conv(x19, s19, ch(512), 3, 2, "model.20")
    x21 = b.concat([x20, x10], 1, "/model.21/Concat")
    x22, s22 = b.c3k2(x21, (s[0] + s10[0], s[1], s[2]), ch(1024), dp(2), True, 0.5, "model.22")
    levels = [(x16, s16, 8), (x19, s19, 16), (x22, s22, 32)]
    out, A = _detect(b, levels, nc, reg_max, dw_cls=True, m="model.23")
    info = dict(convs=b.convs, groups=b.groups, anchors=A, nc=nc, reg_max=reg_max, scale=scale, imgsz=imgsz,
                levels=[(si[1], si[2], st) for _, si, st in levels])
    return g, info


def build_c2psa(c: int = 128, hw: int = 20, seed: int = 0) -> Tuple[EngineGraph, Dict]:
    """One C2PSA block (cv1 -> split -> PSABlock(attention + FFN) -> concat -> cv2) on a
    [1, c, hw, hw] input: the attention subgraph of YOLO11 on its own."""
    b = _Builder(seed)
    g = b.g
    g.graph_inputs = [-1]
    g.input_infos = [TensorInfo("images", [1, c, hw, hw])]
    y, shp = b.c2psa(-1, (c, hw, hw), c, 1, "model.10")
    g.graph_outputs = [y]
    g.output_infos = [TensorInfo("output0", [1, c, hw, hw])]
    return g, dict(convs=b.convs, groups=b.groups)


def build_single_conv(cin: int = 3, cout: int = 16, k: int = 3, s: int = 2, hw: int = 640,
                      seed: int = 0, act: bool = True, groups: int = 1) -> Tuple[EngineGraph, Dict]:
    """Conv-BN-SiLU stem layer as a 3-node graph (Conv -> Sigmoid -> Mul); groups > 1
    makes it a grouped (groups = cin = cout: depthwise) convolution."""
    b = _Builder(seed)
    g = b.g
    g.graph_inputs = [-1]
    g.input_infos = [TensorInfo("images", [1, cin, hw, hw])]
    y, shp = b.conv(-1, (cin, hw, hw), cout, k, s, "model.0", act=act, groups=groups)
    g.graph_outputs = [y]
    g.output_infos = [TensorInfo("output0", [1, cout, shp[1], shp[2]])]
    return g, dict(convs=b.convs)


def conv_flops(info: Dict) -> int:
    """2 * MACs over every conv in the graph, per image (DFL 1x1 excluded)."""
    tot = 0
    groups = info.get('groups', {})
    for name, cin, cout, k, s, h, w in info['convs']:
        p = k // 2
        ho, wo = (h + 2 * p - k) // s + 1, (w + 2 * p - k) // s + 1
        tot += 2 * (cin // groups.get(name, 1)) * cout * k * k * ho * wo
    return tot


def write_yolov8(path: str, **kw) -> Dict:
    g, info = build_yolov8(**kw)
    write_engine(path, g)
    return info


def _detect(b: "_Builder", levels, nc: int, reg_max: int, dw_cls: bool, m: str = "model.22"):
    """Detect head + the exported decode tail -> (output value id, anchor count).
    dw_cls selects the YOLO11 class branch (depthwise 3x3 + pointwise pairs)."""
    g = b.g
    c2 = max(16, levels[0][1][0] // 4, reg_max * 4)
    c3 = max(levels[0][1][0], min(nc, 100))
    no = nc + reg_max * 4
    flat = []
    for i, (xi, si, _) in enumerate(levels):
        t, ts = b.conv(xi, si, c2, 3, 1, f"{m}/cv2.{i}/cv2.{i}.0")
        t, ts = b.conv(t, ts, c2, 3, 1, f"{m}/cv2.{i}/cv2.{i}.1")
        bx, _ = b.conv(t, ts, 4 * reg_max, 1, 1, f"{m}/cv2.{i}/cv2.{i}.2", act=False)
        if dw_cls:   # DWConv(x, x, 3) -> Conv(x, c3, 1) -> DWConv(c3, c3, 3) -> Conv(c3, c3, 1)
            t, ts = b.conv(xi, si, si[0], 3, 1, f"{m}/cv3.{i}/cv3.{i}.0/cv3.{i}.0.0", groups=si[0])
            t, ts = b.conv(t, ts, c3, 1, 1, f"{m}/cv3.{i}/cv3.{i}.0/cv3.{i}.0.1")
            t, ts = b.conv(t, ts, c3, 3, 1, f"{m}/cv3.{i}/cv3.{i}.1/cv3.{i}.1.0", groups=c3)
            t, ts = b.conv(t, ts, c3, 1, 1, f"{m}/cv3.{i}/cv3.{i}.1/cv3.{i}.1.1")
        else:
            t, ts = b.conv(xi, si, c3, 3, 1, f"{m}/cv3.{i}/cv3.{i}.0")
            t, ts = b.conv(t, ts, c3, 3, 1, f"{m}/cv3.{i}/cv3.{i}.1")
        cl, _ = b.conv(t, ts, nc, 1, 1, f"{m}/cv3.{i}/cv3.{i}.2", act=False)
        cat = b.concat([bx, cl], 1, f"/{m}/Concat_{i}")
        shp = b.const(f"/{m}/Reshape_{i}_shape", [1, no, -1])
        (r,) = g.add_node('Reshape', f"/{m}/Reshape_{i}", [cat, shp])
        flat.append(r)
    xcat = b.concat(flat, 2, f"/{m}/Concat_3")
    box = b.slice(xcat, 0, 4 * reg_max, 1, f"/{m}/Split_slice_0")
    cls = b.slice(xcat, 4 * reg_max, no, 1, f"/{m}/Split_slice_1")

    # anchors / strides (make_anchors with grid offset 0.5)
    pts, strs = [], []
    for _, si, st in levels:
        h, w = si[1], si[2]
        sy, sx = np.meshgrid(np.arange(h) + 0.5, np.arange(w) + 0.5, indexing='ij')
        pts.append(np.stack([sx.ravel(), sy.ravel()], 0))
        strs.append(np.full((h * w,), float(st)))
    anchors = np.concatenate(pts, 1)[None].astype(np.float32)      # [1,2,A]
    strides = np.concatenate(strs)[None].astype(np.float32)        # [1,A]
    A = anchors.shape[2]

    # DFL
    s1 = b.const(f"/{m}/dfl/Reshape_shape", [1, 4, reg_max, A])
    (d,) = g.add_node('Reshape', f"/{m}/dfl/Reshape", [box, s1])
    perm = b.const(f"/{m}/dfl/Transpose::perm", [0, 2, 1, 3])
    (d,) = g.add_node('Transpose', f"/{m}/dfl/Transpose", [d, perm])
    (d,) = g.add_node('Softmax', f"/{m}/dfl/Softmax", [d], axis=1)
    wdfl = b.const(f"{m}.dfl.conv.weight", np.arange(reg_max, dtype=np.float32).reshape(1, reg_max, 1, 1))
    (d,) = g.add_node('Conv2d', f"/{m}/dfl/conv/Conv", [d, wdfl])
    s2 = b.const(f"/{m}/dfl/Reshape_1_shape", [1, 4, A])
    (d,) = g.add_node('Reshape', f"/{m}/dfl/Reshape_1", [d, s2])
    lt = b.slice(d, 0, 2, 1, f"/{m}/Split_1_slice_0")
    rb = b.slice(d, 2, 4, 1, f"/{m}/Split_1_slice_1")
    anc = b.const(f"/{m}/anchors", anchors)
    (x1y1,) = g.add_node('Sub', f"/{m}/Sub", [anc, lt])
    (x2y2,) = g.add_node('Add', f"/{m}/Add_1", [anc, rb])
    (cxy,) = g.add_node('Add', f"/{m}/Add_2", [x1y1, x2y2])
    two = b.const(f"/{m}/Constant_2", [2.0])
    (cxy,) = g.add_node('Div', f"/{m}/Div_1", [cxy, two])
    (wh,) = g.add_node('Sub', f"/{m}/Sub_1", [x2y2, x1y1])
    dbox = b.concat([cxy, wh], 1, f"/{m}/Concat_4")
    stc = b.const(f"/{m}/strides", strides)
    (dbox,) = g.add_node('Mul', f"/{m}/Mul_2", [dbox, stc])
    (sig,) = g.add_node('Sigmoid', f"/{m}/Sigmoid", [cls])
    out = b.concat([dbox, sig], 1, f"/{m}/Concat_5")
    g.graph_outputs = [out]
    g.output_infos = [TensorInfo("output0", [1, 4 + nc, A])]
    return out, A
