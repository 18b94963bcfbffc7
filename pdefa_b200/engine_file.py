"""Reader and writer for pdefa's ``.engine`` graph files (format v1 and v2).

The byte layout is fixed by the reference loader and converter, so it is kept
identical here:

* header: magic ``0x4E474E45`` ("ENGN"), version (1|2), counts of weights,
  nodes, inputs, outputs, then a 64-byte brand string
  (``PDEFA1.0/src/loader/custom_loader.cpp:70-78``,
  ``pdefa/tools/onnx_to_engine.py:755-762``);
* weight table: name, dtype (internal ``DType`` code, F32 = 12), rank, dims,
  data offset, byte size (``custom_loader.cpp:83-107``);
* nodes: op id, name, input/output index lists, and the 128-byte ``OpParams``
  blob (``custom_loader.cpp:118-143``; layout ``PDEFA1.0/include/engine/graph.hpp:77-94``,
  packer ``onnx_to_engine.py:312-333``);
* graph input/output indices, v2 tensor infos (``custom_loader.cpp:145-170``);
* weight data blob.

Tensor index convention (``PDEFA1.0/src/core/session_parts/session_helpers.inc:6-25``):
``idx >= 0`` intermediate, ``idx <= -1000`` weight ``-idx-1000``, otherwise
external input ``-idx-1``.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence

import numpy as np

MAGIC = 0x4E474E45
PARAMS_SIZE = 128

# Op ids (graph.hpp:20-75 / onnx_to_engine.py:28-78)
OP = dict(
    Conv2d=1, MatMul=2, Add=3, Mul=4, Sub=5, Div=6,
    ReLU=10, LeakyReLU=11, Sigmoid=12, Tanh=13, SiLU=14, GELU=15,
    HardSwish=16, HardSigmoid=17,
    MaxPool2d=20, AvgPool2d=21, BatchNorm2d=22, LayerNorm=23,
    Softmax=30, Concat=31, Upsample=32, Resize=33, Input=40, Output=41,
    Reshape=42, Transpose=43, Slice=44, Gather=45, Shape=46, Expand=47,
    Unsqueeze=48, Squeeze=49, TopK=50, GatherElements=51, Mod=52,
    ReduceMax=53, ReduceMin=54, ReduceProd=55, NonZero=56,
    ConstantOfShape=57, Tile=58, Range=59, Equal=60, Greater=61, Exp=62,
    Min=63, Max=64, ReduceSum=65, Clip=66, ArgMax=67, Stack=68,
)
OP_NAME = {v: k for k, v in OP.items()}

# Internal dtype codes (PDEFA1.0/include/engine/dtype.hpp:36-60)
DT_F32 = 12
DT_I8 = 2
_DT_NP = {12: np.float32, 13: np.float64, 2: np.int8, 3: np.uint8, 6: np.int32,
          8: np.int64, 10: np.float16, 1: np.bool_}

_PARAM_DEFAULTS = dict(
    stride_h=1, stride_w=1, pad_h=0, pad_w=0, dil_h=1, dil_w=1, groups=1,
    kernel_h=0, kernel_w=0, axis=-1, scale_h=0, scale_w=0, target_h=0, target_w=0,
    upsample_mode=0, eps=1e-5, fused_activation=0, leaky_slope=0.01,
)


def pack_params(**kw) -> bytes:
    """Pack an ``OpParams`` record into its 128-byte on-disk form.

    Field order and padding follow ``graph.hpp:77-94`` (natural C++ alignment):
    9 x int64, int32 axis (+4 pad), 4 x int64, u8 upsample_mode (+3 pad),
    f32 eps, u8 fused_activation (+3 pad), f32 leaky_slope, zero padding.
    Unset fields take the converter's defaults (``onnx_to_engine.py:312-317``).
    """
    p = dict(_PARAM_DEFAULTS)
    for k, v in kw.items():
        if k not in p:
            raise KeyError(f"unknown OpParams field {k!r}")
        p[k] = v
    buf = struct.pack('<9q', p['stride_h'], p['stride_w'], p['pad_h'], p['pad_w'],
                      p['dil_h'], p['dil_w'], p['groups'], p['kernel_h'], p['kernel_w'])
    buf += struct.pack('<i4x', p['axis'])
    buf += struct.pack('<4q', p['scale_h'], p['scale_w'], p['target_h'], p['target_w'])
    buf += struct.pack('<B3xf', p['upsample_mode'], p['eps'])
    buf += struct.pack('<B3xf', p['fused_activation'], p['leaky_slope'])
    return buf.ljust(PARAMS_SIZE, b'\x00')


def unpack_params(blob: bytes) -> Dict[str, float]:
    v = struct.unpack_from('<9q', blob, 0)
    keys = ['stride_h', 'stride_w', 'pad_h', 'pad_w', 'dil_h', 'dil_w', 'groups',
            'kernel_h', 'kernel_w']
    p = dict(zip(keys, v))
    p['axis'], = struct.unpack_from('<i', blob, 72)
    p['scale_h'], p['scale_w'], p['target_h'], p['target_w'] = struct.unpack_from('<4q', blob, 80)
    p['upsample_mode'], p['eps'] = struct.unpack_from('<B3xf', blob, 112)
    p['fused_activation'], p['leaky_slope'] = struct.unpack_from('<B3xf', blob, 120)
    return p


@dataclass
class TensorInfo:
    name: str
    shape: List[int]
    dtype: int = DT_F32


@dataclass
class Node:
    op: int
    name: str
    inputs: List[int]
    outputs: List[int]
    params: Dict[str, float] = field(default_factory=dict)


@dataclass
class EngineGraph:
    """In-memory ``.engine`` contents: weights, nodes, graph I/O."""
    weights: List[tuple] = field(default_factory=list)     # (name, np.ndarray)
    nodes: List[Node] = field(default_factory=list)
    graph_inputs: List[int] = field(default_factory=list)
    graph_outputs: List[int] = field(default_factory=list)
    input_infos: List[TensorInfo] = field(default_factory=list)
    output_infos: List[TensorInfo] = field(default_factory=list)
    version: int = 2
    brand: bytes = b"engine-ai"
    _next_inter: int = 0

    # ---- builder helpers -------------------------------------------------
    def add_weight(self, name: str, arr) -> int:
        """Append a weight; returns its tensor index (``-1000 - w``)."""
        a = np.ascontiguousarray(np.asarray(arr, dtype=np.float32))
        self.weights.append((name, a))
        return -1000 - (len(self.weights) - 1)

    def new_tensor(self) -> int:
        i = self._next_inter
        self._next_inter += 1
        return i

    def add_node(self, op: str, name: str, inputs: Sequence[int], n_out: int = 1,
                 **params) -> List[int]:
        outs = [self.new_tensor() for _ in range(n_out)]
        full = dict(_PARAM_DEFAULTS)
        full.update(params)
        self.nodes.append(Node(OP[op], name, list(inputs), outs, full))
        return outs

    def weight(self, idx: int) -> np.ndarray:
        return self.weights[-idx - 1000][1]


def write_engine(path: str, g: EngineGraph) -> None:
    """Serialise ``g`` with the layout of ``onnx_to_engine.py:747-818``."""
    with open(path, 'wb') as f:
        f.write(struct.pack('<6I', MAGIC, g.version, len(g.weights), len(g.nodes),
                            len(g.graph_inputs), len(g.graph_outputs)))
        f.write(g.brand[:63].ljust(64, b'\x00'))
        cursor = 0
        for name, arr in g.weights:
            nb = name.encode()
            f.write(struct.pack('<I', len(nb)) + nb)
            f.write(struct.pack('<BB', DT_F32, arr.ndim))
            for d in arr.shape:
                f.write(struct.pack('<q', int(d)))
            f.write(struct.pack('<QQ', cursor, arr.nbytes))
            cursor += arr.nbytes
        for n in g.nodes:
            nb = n.name.encode()
            f.write(struct.pack('<BI', n.op, len(nb)) + nb)
            f.write(struct.pack('<HH', len(n.inputs), len(n.outputs)))
            for i in n.inputs:
                f.write(struct.pack('<i', i))
            for o in n.outputs:
                f.write(struct.pack('<i', o))
            f.write(pack_params(**n.params))
        for i in g.graph_inputs:
            f.write(struct.pack('<i', i))
        for o in g.graph_outputs:
            f.write(struct.pack('<i', o))
        if g.version >= 2:
            for info in list(g.input_infos) + list(g.output_infos):
                nb = info.name.encode()
                f.write(struct.pack('<I', len(nb)) + nb)
                f.write(struct.pack('<B', len(info.shape)))
                for d in info.shape:
                    f.write(struct.pack('<q', int(d)))
                f.write(struct.pack('<B', int(info.dtype)))
        for _, arr in g.weights:
            f.write(arr.tobytes())


def read_engine(path: str) -> EngineGraph:
    """Parse a ``.engine`` file (v1 or v2), mirroring ``custom_loader.cpp:62-214``."""
    data = open(path, 'rb').read()
    off = 0

    def take(fmt):
        nonlocal off
        v = struct.unpack_from(fmt, data, off)
        off += struct.calcsize(fmt)
        return v

    magic, version, nw, nn, ni, no = take('<6I')
    if magic != MAGIC or version not in (1, 2):
        raise ValueError(f"{path}: not an .engine file (magic {magic:#x}, v{version})")
    brand = data[off:off + 64].rstrip(b'\x00')
    off += 64
    g = EngineGraph(version=version, brand=brand)
    wmeta = []
    for _ in range(nw):
        (ln,) = take('<I')
        name = data[off:off + ln].decode()
        off += ln
        dt, rank = take('<BB')
        dims = take(f'<{rank}q') if rank else ()
        o, sz = take('<QQ')
        wmeta.append((name, dt, dims, o, sz))
    for _ in range(nn):
        op, ln = take('<BI')
        name = data[off:off + ln].decode()
        off += ln
        nin, nout = take('<HH')
        ins = list(take(f'<{nin}i')) if nin else []
        outs = list(take(f'<{nout}i')) if nout else []
        params = unpack_params(data[off:off + PARAMS_SIZE])
        off += PARAMS_SIZE
        g.nodes.append(Node(op, name, ins, outs, params))
    g.graph_inputs = list(take(f'<{ni}i')) if ni else []
    g.graph_outputs = list(take(f'<{no}i')) if no else []
    if version >= 2:
        for k in range(ni + no):
            (ln,) = take('<I')
            name = data[off:off + ln].decode()
            off += ln
            (rank,) = take('<B')
            dims = list(take(f'<{rank}q')) if rank else []
            (dt,) = take('<B')
            (g.input_infos if k < ni else g.output_infos).append(TensorInfo(name, dims, dt))
    base = off
    for name, dt, dims, o, sz in wmeta:
        npdt = _DT_NP.get(dt, np.float32)
        arr = np.frombuffer(data, dtype=npdt, count=sz // np.dtype(npdt).itemsize,
                            offset=base + o).reshape(dims)
        g.weights.append((name, arr))
    outs = [o for n in g.nodes for o in n.outputs]
    g._next_inter = (max(outs) + 1) if outs else 0
    return g
