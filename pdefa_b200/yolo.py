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

    # ---- Detect head ----
    levels = [(x15, s15, 8), (x18, s18, 16), (x21, s21, 32)]
    c2 = max(16, levels[0][1][0] // 4, reg_max * 4)
    c3 = max(levels[0][1][0], min(nc, 100))
    no = nc + reg_max * 4
    flat = []
    for i, (xi, si, _) in enumerate(levels):
        t, ts = b.conv(xi, si, c2, 3, 1, f"model.22/cv2.{i}/cv2.{i}.0")
        t, ts = b.conv(t, ts, c2, 3, 1, f"model.22/cv2.{i}/cv2.{i}.1")
        bx, _ = b.conv(t, ts, 4 * reg_max, 1, 1, f"model.22/cv2.{i}/cv2.{i}.2", act=False)
        t, ts = b.conv(xi, si, c3, 3, 1, f"model.22/cv3.{i}/cv3.{i}.0")
        t, ts = b.conv(t, ts, c3, 3, 1, f"model.22/cv3.{i}/cv3.{i}.1")
        cl, _ = b.conv(t, ts, nc, 1, 1, f"model.22/cv3.{i}/cv3.{i}.2", act=False)
        cat = b.concat([bx, cl], 1, f"/model.22/Concat_{i}")
        shp = b.const(f"/model.22/Reshape_{i}_shape", [1, no, -1])
        (r,) = g.add_node('Reshape', f"/model.22/Reshape_{i}", [cat, shp])
        flat.append(r)
    xcat = b.concat(flat, 2, "/model.22/Concat_3")
    box = b.slice(xcat, 0, 4 * reg_max, 1, "/model.22/Split_slice_0")
    cls = b.slice(xcat, 4 * reg_max, no, 1, "/model.22/Split_slice_1")

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
    s1 = b.const("/model.22/dfl/Reshape_shape", [1, 4, reg_max, A])
    (d,) = g.add_node('Reshape', "/model.22/dfl/Reshape", [box, s1])
    perm = b.const("/model.22/dfl/Transpose::perm", [0, 2, 1, 3])
    (d,) = g.add_node('Transpose', "/model.22/dfl/Transpose", [d, perm])
    (d,) = g.add_node('Softmax', "/model.22/dfl/Softmax", [d], axis=1)
    wdfl = b.const("model.22.dfl.conv.weight", np.arange(reg_max, dtype=np.float32).reshape(1, reg_max, 1, 1))
    (d,) = g.add_node('Conv2d', "/model.22/dfl/conv/Conv", [d, wdfl])
    s2 = b.const("/model.22/dfl/Reshape_1_shape", [1, 4, A])
    (d,) = g.add_node('Reshape', "/model.22/dfl/Reshape_1", [d, s2])
    lt = b.slice(d, 0, 2, 1, "/model.22/Split_1_slice_0")
    rb = b.slice(d, 2, 4, 1, "/model.22/Split_1_slice_1")
    anc = b.const("/model.22/anchors", anchors)
    (x1y1,) = g.add_node('Sub', "/model.22/Sub", [anc, lt])
    (x2y2,) = g.add_node('Add', "/model.22/Add_1", [anc, rb])
    (cxy,) = g.add_node('Add', "/model.22/Add_2", [x1y1, x2y2])
    two = b.const("/model.22/Constant_2", [2.0])
    (cxy,) = g.add_node('Div', "/model.22/Div_1", [cxy, two])
    (wh,) = g.add_node('Sub', "/model.22/Sub_1", [x2y2, x1y1])
    dbox = b.concat([cxy, wh], 1, "/model.22/Concat_4")
    stc = b.const("/model.22/strides", strides)
    (dbox,) = g.add_node('Mul', "/model.22/Mul_2", [dbox, stc])
    (sig,) = g.add_node('Sigmoid', "/model.22/Sigmoid", [cls])
    out = b.concat([dbox, sig], 1, "/model.22/Concat_5")
    g.graph_outputs = [out]
    g.output_infos = [TensorInfo("output0", [1, 4 + nc, A])]
    info = dict(convs=b.convs, anchors=A, nc=nc, reg_max=reg_max, scale=scale, imgsz=imgsz,
                levels=[(si[1], si[2], st) for _, si, st in levels])
    return g, info


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
    for _, cin, cout, k, s, h, w in info['convs']:
        p = k // 2
        ho, wo = (h + 2 * p - k) // s + 1, (w + 2 * p - k) // s + 1
        tot += 2 * cin * cout * k * k * ho * wo
    return tot


def write_yolov8(path: str, **kw) -> Dict:
    g, info = build_yolov8(**kw)
    write_engine(path, g)
    return info
