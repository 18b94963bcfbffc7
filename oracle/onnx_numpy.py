"""Plain-ONNX (NCHW) numpy interpreter for ``.engine`` graphs.

TEST INFRASTRUCTURE ONLY. An independent restatement of what each node means in
ONNX terms, used to check that the reference engine's NHWC heuristics
(``PDEFA1.0/src/core/session_parts/session_ops_shape.inc``, ``session_ops_math.inc``)
compute the intended graph on the synthetic YOLOv8 files, and as a second opinion
on small cases. It computes in float64 by default.

Per-op meaning (ONNX operator definitions):
Conv (pads symmetric, groups 1), Sigmoid, Add/Sub/Mul/Div (numpy broadcasting),
Slice (starts/ends/axes), Concat, MaxPool (padding ignored), Resize nearest with
integer scales, Reshape (0 = copy, -1 = infer), Transpose, Softmax.
"""
from __future__ import annotations

import numpy as np

from pdefa_b200.engine_file import EngineGraph, OP_NAME


def conv2d_nchw(x, w, b, stride, pad, groups=1):
    """ONNX Conv (dilation 1); groups > 1 splits input and output channels into
    `groups` independent convolutions (the reference's depthwise / grouped paths,
    PDEFA1.0/src/ops/conv2d.cpp:164-393)."""
    if groups > 1:
        xs = np.split(x, groups, axis=1)
        ws = np.split(w, groups, axis=0)
        bs = np.split(b, groups) if b is not None else [None] * groups
        return np.concatenate([conv2d_nchw(xs[i], ws[i], bs[i], stride, pad) for i in range(groups)], axis=1)
    n, c, h, wd = x.shape
    co, ci, kh, kw = w.shape
    xp = np.pad(x, ((0, 0), (0, 0), (pad[0], pad[0]), (pad[1], pad[1])))
    ho = (h + 2 * pad[0] - kh) // stride[0] + 1
    wo = (wd + 2 * pad[1] - kw) // stride[1] + 1
    out = np.zeros((n, co, ho, wo), dtype=x.dtype)
    for r in range(kh):
        for s in range(kw):
            patch = xp[:, :, r:r + stride[0] * ho:stride[0], s:s + stride[1] * wo:stride[1]]
            out += np.einsum('nchw,oc->nohw', patch, w[:, :, r, s], optimize=True)
    if b is not None:
        out += b.reshape(1, -1, 1, 1)
    return out


def maxpool_nchw(x, k, stride, pad):
    n, c, h, w = x.shape
    xp = np.pad(x, ((0, 0), (0, 0), (pad[0], pad[0]), (pad[1], pad[1])), constant_values=-np.inf)
    ho = (h + 2 * pad[0] - k[0]) // stride[0] + 1
    wo = (w + 2 * pad[1] - k[1]) // stride[1] + 1
    out = np.full((n, c, ho, wo), -np.inf, dtype=x.dtype)
    for r in range(k[0]):
        for s in range(k[1]):
            out = np.maximum(out, xp[:, :, r:r + stride[0] * ho:stride[0], s:s + stride[1] * wo:stride[1]])
    return out


def ref_conv_path(cin, kh, kw, sh, sw, ph, pw, dh, dw, groups):
    """Kernel the reference dispatcher picks for a batch-1 NHWC conv.

    Follows ``PDEFA1.0/src/ops/conv2d.cpp:602-642``: direct NHWC for Cin <= 16
    (not a pure 1x1), Winograd F(2,3) for 3x3 s1 d1 with Cin <= 512, else GEMM.
    """
    pure_1x1 = kh == 1 and kw == 1 and ph == 0 and pw == 0 and sh == 1 and sw == 1 and dh == 1 and dw == 1
    if not pure_1x1 and cin <= 16 and groups == 1 and kh <= 7 and kw <= 7:
        return 'direct'
    if kh == 3 and kw == 3 and sh == 1 and sw == 1 and dh == 1 and dw == 1 and groups == 1 and cin <= 512:
        return 'winograd'
    return 'gemm'


def silu_winograd_flavor(x):
    """SiLU as the reference's Winograd epilogue evaluates it
    (``PDEFA1.0/src/kernels/simd/avx2/conv2d_winograd.cpp:81-101``), in float32.

    exp(-x) is formed as 2**n * q(f) with n = round(-x*log2 e), f the remaining
    log2 fraction and q(f) = 1 + f/2 + f^2/6 + ... (the Taylor series of
    (e^f - 1)/f, degree 6); the result is x / (1 + q(f) * 2**n).
    """
    x = np.asarray(x, dtype=np.float32)
    nx = -x
    fx = (nx * np.float32(1.44269504088896341)).astype(np.float32)
    n = np.where(fx >= 0, np.floor(fx + np.float32(0.5)), np.ceil(fx - np.float32(0.5))).astype(np.float32)
    f = (fx - n).astype(np.float32)
    p = np.float32(1.9875691500e-4)
    for c in (1.3981999507e-3, 8.3334519073e-3, 4.1665795894e-2, 1.6666665459e-1, 5.0000001201e-1, 1.0):
        p = (p * f + np.float32(c)).astype(np.float32)
    scale = np.ldexp(np.float32(1.0), np.clip(n, -126, 127).astype(np.int32)).astype(np.float32)
    y = (x / (np.float32(1.0) + p * scale)).astype(np.float32)
    y = np.where(nx < np.float32(-88.37626), x, y)
    y = np.where(nx > np.float32(88.37626), np.float32(0.0), y)
    return y


def fused_silu_convs(g: EngineGraph):
    """Conv -> Sigmoid -> Mul triples the reference fuses (session_fusion.inc:33-81).

    Returns {conv_node_index: (sigmoid_index, mul_index)}.
    """
    cons = {}
    for k, n in enumerate(g.nodes):
        for i in n.inputs:
            cons[i] = cons.get(i, 0) + 1
    for o in g.graph_outputs:
        cons[o] = cons.get(o, 0) + 1
    out = {}
    for i, n in enumerate(g.nodes):
        if OP_NAME[n.op] != 'Conv2d' or cons.get(n.outputs[0], 0) != 2:
            continue
        co = n.outputs[0]
        sig = next((j for j in range(i + 1, len(g.nodes)) if OP_NAME[g.nodes[j].op] == 'Sigmoid'
                    and g.nodes[j].inputs == [co]), None)
        if sig is None or cons.get(g.nodes[sig].outputs[0], 0) != 1:
            continue
        so = g.nodes[sig].outputs[0]
        mul = next((j for j in range(i + 1, len(g.nodes)) if OP_NAME[g.nodes[j].op] == 'Mul'
                    and sorted(g.nodes[j].inputs) == sorted([co, so])), None)
        if mul is not None:
            out[i] = (sig, mul)
    return out


def run(g: EngineGraph, inputs, dtype=np.float64, reference_silu=True):
    """Evaluate ``g``. With ``reference_silu`` the fused Conv-SiLU layers that the
    reference sends through its Winograd kernel use that kernel's SiLU flavour."""
    fused = fused_silu_convs(g) if reference_silu else {}
    skip = set()
    vals = {}
    for i, x in enumerate(inputs):
        vals[-1 - i] = np.asarray(x, dtype=dtype)

    def get(idx):
        if idx <= -1000:
            return g.weight(idx).astype(dtype)
        return vals[idx]

    for k, n in enumerate(g.nodes):
        if k in skip:
            continue
        op = OP_NAME[n.op]
        p = n.params
        ins = [get(i) for i in n.inputs]
        if op == 'Conv2d':
            y = conv2d_nchw(ins[0], ins[1], ins[2] if len(ins) > 2 else None,
                            (p['stride_h'], p['stride_w']), (p['pad_h'], p['pad_w']), max(1, p['groups']))
            if k in fused:
                w = ins[1]
                path = ref_conv_path(w.shape[1], w.shape[2], w.shape[3], p['stride_h'], p['stride_w'],
                                     p['pad_h'], p['pad_w'], p['dil_h'], p['dil_w'], p['groups'])
                if path == 'winograd':
                    y = silu_winograd_flavor(y).astype(dtype)
                else:
                    y = y / (1.0 + np.exp(-y))
                sig, mul = fused[k]
                skip.update((sig, mul))
                vals[g.nodes[mul].outputs[0]] = np.ascontiguousarray(y)
                continue
        elif op == 'Sigmoid':
            y = 1.0 / (1.0 + np.exp(-ins[0]))
        elif op == 'Add':
            y = ins[0] + ins[1]
        elif op == 'Sub':
            y = ins[0] - ins[1]
        elif op == 'Mul':
            y = ins[0] * ins[1]
        elif op == 'Div':
            y = ins[0] / ins[1]
        elif op == 'Slice':
            x = ins[0]
            sl = [slice(None)] * x.ndim
            axes = ins[3].astype(int) if len(ins) > 3 else range(len(ins[1]))
            for st, en, ax in zip(ins[1].astype(int), ins[2].astype(int), axes):
                sl[ax] = slice(st, en)
            y = x[tuple(sl)]
        elif op == 'Concat':
            y = np.concatenate(ins, axis=p['axis'])
        elif op == 'MaxPool2d':
            y = maxpool_nchw(ins[0], (p['kernel_h'], p['kernel_w']), (p['stride_h'], p['stride_w']),
                             (p['pad_h'], p['pad_w']))
        elif op == 'Resize':
            sc = ins[1].astype(int)
            y = ins[0].repeat(sc[2], axis=2).repeat(sc[3], axis=3)
        elif op == 'Reshape':
            shape = [int(v) for v in ins[1]]
            shape = [ins[0].shape[i] if v == 0 else v for i, v in enumerate(shape)]
            y = ins[0].reshape(shape)
        elif op == 'Transpose':
            y = np.transpose(ins[0], [int(v) for v in ins[1]])
        elif op == 'Softmax':
            x = ins[0]
            e = np.exp(x - x.max(axis=p['axis'], keepdims=True))
            y = e / e.sum(axis=p['axis'], keepdims=True)
        else:
            raise NotImplementedError(op)
        vals[n.outputs[0]] = np.ascontiguousarray(y)
    return [vals[o] for o in g.graph_outputs]
