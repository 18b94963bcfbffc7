"""Python API of the B200 engine, mirroring pdefa's public surface
(pdefa/python/src/pdefa/__init__.py:45-139): Context, Model, Session, Tensor,
ops_*, decode_yolo, load/EngineModel. Names, argument meaning and error behaviour
follow the reference; compute runs on the GPU through libpdefa_native.so.

Differences from the reference:
* decode_yolo on a Tensor or an ndarray runs the batched GPU decode/NMS
  (pdefa_decode_yolo) and returns the reference's list of dicts; for a
  [B, 4+nc, A] output with B > 1 it returns one list per image;
* Context.set_precision / set_device select strict FP32, TF32 or BF16 arithmetic
  and the GPU; Session.run_device runs on device pointers;
* image files: PNG and baseline JPEG are decoded on the host (the reference's
  pixels); letterboxing runs on the GPU (bit-identical to the reference's
  preprocess_letterbox), also for decoded 8-bit arrays (letterbox_u8) and inside
  BatchInference.detect_u8.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple

from . import _native as N

FP32, TF32, BF16 = 0, 1, 2
_DT_SIZE = {0: 4, 1: 2, 2: 2, 3: 1, 4: 1, 5: 4, 6: 8, 7: 1}


class PdefaError(RuntimeError):
    """Raised when a native call returns a non-zero status (_bindings.py:476-487)."""


def _check(rc: int, what: str = "") -> None:
    if rc != 0:
        L = N.lib()
        msg = (L.pdefa_last_error() or b"").decode(errors="replace")
        status = (L.engine_status_string(rc) or b"").decode()
        raise PdefaError(f"{what} failed: [{rc}] {status}" + (f" - {msg}" if msg else ""))


def version() -> str:
    return N.lib().pdefa_version().decode()


def simd_level() -> str:
    return N.lib().engine_simd_level().decode()


def cpu_brand() -> str:
    return N.lib().engine_cpu_brand().decode()


def device_count() -> int:
    return int(N.lib().engine_device_count())


@dataclass
class PreprocessMeta:
    target_w: int = 640
    target_h: int = 640
    orig_w: int = 640
    orig_h: int = 640
    pad_x: int = 0
    pad_y: int = 0
    scaled_w: int = 640
    scaled_h: int = 640
    ratio: float = 1.0

    def to_c(self) -> N.PreMeta:
        return N.PreMeta(self.target_w, self.target_h, self.orig_w, self.orig_h, self.pad_x, self.pad_y,
                         self.scaled_w, self.scaled_h, self.ratio)

    @classmethod
    def from_c(cls, c: N.PreMeta) -> "PreprocessMeta":
        return cls(c.target_w, c.target_h, c.orig_w, c.orig_h, c.pad_x, c.pad_y, c.scaled_w, c.scaled_h, c.ratio)


@dataclass
class Box:
    x1: float
    y1: float
    x2: float
    y2: float


@dataclass
class TensorInfo:
    name: str
    shape: Tuple[int, ...]
    dtype: int


# ----------------------------------------------------------------------------
# Tensor
# ----------------------------------------------------------------------------
def _reshape_list(flat, shape):
    if not shape:
        return flat[0] if flat else 0.0
    if len(shape) == 1:
        return list(flat)
    step = 1
    for d in shape[1:]:
        step *= d
    return [_reshape_list(flat[i * step:(i + 1) * step], shape[1:]) for i in range(shape[0])]


def _flatten_list(data):
    shape = []
    x = data
    while isinstance(x, (list, tuple)):
        shape.append(len(x))
        x = x[0] if x else None
    flat = []

    def rec(v, depth):
        if depth == len(shape):
            flat.append(float(v))
            return
        if not isinstance(v, (list, tuple)) or len(v) != shape[depth]:
            raise PdefaError("ragged nested list")
        for e in v:
            rec(e, depth + 1)

    rec(data, 0)
    return flat, shape


class Tensor:
    """Handle to an engine tensor (owned, or borrowed from a Session)."""

    def __init__(self, handle, owns: bool = True):
        self._handle = handle
        self._owns = owns

    def __del__(self):
        h = getattr(self, "_handle", None)
        if h and self._owns and N._lib is not None:
            N._lib.engine_tensor_destroy(h)
            self._handle = None

    @property
    def raw(self):
        return self._handle

    @property
    def numel(self) -> int:
        return int(N.lib().engine_tensor_numel(self._handle))

    @property
    def ndim(self) -> int:
        return int(N.lib().engine_tensor_rank(self._handle))

    @property
    def dtype(self) -> int:
        return int(N.lib().engine_tensor_dtype(self._handle))

    @property
    def shape(self) -> Tuple[int, ...]:
        n = self.ndim
        buf = (N.i64 * max(n, 1))()
        nd = N.i32(0)
        _check(N.lib().engine_tensor_shape(self._handle, buf, C.byref(nd)), "tensor_shape")
        return tuple(int(buf[i]) for i in range(nd.value))

    def _data(self):
        ptr, size = C.c_void_p(), C.c_size_t()
        _check(N.lib().engine_tensor_data(self._handle, C.byref(ptr), C.byref(size)), "tensor_data")
        return ptr.value, size.value

    def tolist(self):
        ptr, size = self._data()
        ctype = {5: C.c_int32, 6: C.c_int64, 3: C.c_int8, 4: C.c_uint8}.get(self.dtype, C.c_float)
        n = size // C.sizeof(ctype)
        flat = list((ctype * n).from_address(ptr)) if n else []
        return _reshape_list(flat, self.shape)

    def to_numpy(self):
        import numpy as np
        ptr, size = self._data()
        npdt = {5: np.int32, 6: np.int64, 3: np.int8, 4: np.uint8}.get(self.dtype, np.float32)
        buf = (C.c_uint8 * size).from_address(ptr) if size else b""
        return np.frombuffer(bytes(buf), dtype=npdt).reshape(self.shape)

    numpy = to_numpy

    @classmethod
    def from_numpy(cls, arr) -> "Tensor":
        import numpy as np
        a = np.ascontiguousarray(arr, dtype=np.float32)
        shp = (N.i64 * max(a.ndim, 1))(*a.shape)
        h = C.c_void_p()
        _check(N.lib().engine_tensor_create_from_data(C.byref(h), shp, a.ndim, 0, a.ctypes.data, a.nbytes),
               "tensor_create_from_data")
        return cls(h)

    def fill(self, value: float) -> "Tensor":
        n = self.numel
        arr = (C.c_float * n)(*([float(value)] * n))
        _check(N.lib().engine_tensor_copy_from(self._handle, arr, n * 4), "fill")
        return self

    def copy_from_list(self, data) -> "Tensor":
        flat, shape = _flatten_list(data)
        if tuple(shape) != self.shape:
            raise PdefaError(f"shape mismatch: {tuple(shape)} != {self.shape}")
        arr = (C.c_float * len(flat))(*flat)
        _check(N.lib().engine_tensor_copy_from(self._handle, arr, len(flat) * 4), "copy_from_list")
        return self

    def __add__(self, o): return ops_add(self, o if isinstance(o, Tensor) else _scalar(o))
    def __sub__(self, o): return ops_sub(self, o if isinstance(o, Tensor) else _scalar(o))
    def __mul__(self, o): return ops_mul(self, o if isinstance(o, Tensor) else _scalar(o))
    def __truediv__(self, o): return ops_div(self, o if isinstance(o, Tensor) else _scalar(o))
    def __neg__(self): return ops_mul(self, _scalar(-1.0))

    def __matmul__(self, other):
        if not isinstance(other, Tensor):
            raise TypeError("matmul requires Tensor")
        sa, sb = self.shape, other.shape
        if len(sa) != 2 or len(sb) != 2:
            raise PdefaError("matmul: 2D tensors required")
        if sa[1] != sb[0]:
            raise PdefaError(f"matmul: inner dims mismatch {sa} @ {sb}")
        return ops_matmul(self, other)

    def __repr__(self):
        return f"Tensor(shape={self.shape}, dtype={self.dtype})"


def tensor_empty(shape, dtype: int = 0) -> Tensor:
    shape = list(shape)
    shp = (N.i64 * max(len(shape), 1))(*shape)
    h = C.c_void_p()
    _check(N.lib().engine_tensor_create(C.byref(h), shp, len(shape), dtype), "tensor_create")
    return Tensor(h)


def _scalar(v: float) -> Tensor:
    return from_list([float(v)])


def from_list(data) -> Tensor:
    flat, shape = _flatten_list(data)
    if not shape:
        shape = [1]
    arr = (C.c_float * max(len(flat), 1))(*flat)
    shp = (N.i64 * len(shape))(*shape)
    h = C.c_void_p()
    _check(N.lib().engine_tensor_create_from_data(C.byref(h), shp, len(shape), 0, arr, len(flat) * 4),
           "tensor_create_from_data")
    return Tensor(h)


def zeros(*shape) -> Tensor:
    return tensor_empty(shape)


def ones(*shape) -> Tensor:
    return tensor_empty(shape).fill(1.0)


def empty(*shape) -> Tensor:
    return tensor_empty(shape)


def random_randn(shape, seed: int = 0) -> Tensor:
    shape = list(shape)
    h = C.c_void_p()
    _check(N.lib().engine_random_randn((N.i64 * max(len(shape), 1))(*shape), len(shape), seed, C.byref(h)), "randn")
    return Tensor(h)


def random_rand(shape, seed: int = 0) -> Tensor:
    shape = list(shape)
    h = C.c_void_p()
    _check(N.lib().engine_random_rand((N.i64 * max(len(shape), 1))(*shape), len(shape), seed, C.byref(h)), "rand")
    return Tensor(h)


def randn(*shape, seed=0) -> Tensor:
    return random_randn(shape, seed)


def rand(*shape, seed=0) -> Tensor:
    return random_rand(shape, seed)


# ----------------------------------------------------------------------------
# Ops
# ----------------------------------------------------------------------------
def _binary(a, b, fn, what) -> Tensor:
    h = C.c_void_p()
    _check(fn(a.raw, b.raw, C.byref(h)), what)
    return Tensor(h)


def ops_add(a, b): return _binary(a, b, N.lib().engine_ops_add, "ops_add")
def ops_sub(a, b): return _binary(a, b, N.lib().engine_ops_sub, "ops_sub")
def ops_mul(a, b): return _binary(a, b, N.lib().engine_ops_mul, "ops_mul")
def ops_div(a, b): return _binary(a, b, N.lib().engine_ops_div, "ops_div")


def ops_matmul(a: Tensor, b: Tensor, out: Optional[Tensor] = None, precision: Optional[int] = None) -> Tensor:
    """out = a @ b (engine_ops_matmul; out is allocated [M, N] when not given)."""
    if out is None:
        out = tensor_empty([a.shape[0], b.shape[1]])
    if precision is None:
        _check(N.lib().engine_ops_matmul(a.raw, b.raw, out.raw), "ops_matmul")
    else:
        _check(N.lib().engine_ops_matmul_ex(a.raw, b.raw, out.raw, int(precision)), "ops_matmul")
    return out


def _unary(t, fn, what, *args):
    _check(fn(t.raw, *args), what)
    return t


def ops_relu(t): return _unary(t, N.lib().engine_ops_relu, "ops_relu")
def ops_silu(t): return _unary(t, N.lib().engine_ops_silu, "ops_silu")
def ops_sigmoid(t): return _unary(t, N.lib().engine_ops_sigmoid, "ops_sigmoid")
def ops_tanh(t): return _unary(t, N.lib().engine_ops_tanh, "ops_tanh")
def ops_gelu(t): return _unary(t, N.lib().engine_ops_gelu, "ops_gelu")
def ops_clip(t, lo, hi): return _unary(t, N.lib().engine_ops_clip, "ops_clip", float(lo), float(hi))
def ops_softmax(t, axis=-1): return _unary(t, N.lib().engine_ops_softmax, "ops_softmax", int(axis))


def _reduce(a, axis, keepdims, fn, what):
    h = C.c_void_p()
    _check(fn(a.raw, int(axis), 1 if keepdims else 0, C.byref(h)), what)
    return Tensor(h)


def ops_reduce_max(a, axis=-1, keepdims=False): return _reduce(a, axis, keepdims, N.lib().engine_ops_reduce_max, "reduce_max")
def ops_reduce_sum(a, axis=-1, keepdims=False): return _reduce(a, axis, keepdims, N.lib().engine_ops_reduce_sum, "reduce_sum")
def ops_reduce_mean(a, axis=-1, keepdims=False): return _reduce(a, axis, keepdims, N.lib().engine_ops_reduce_mean, "reduce_mean")
def ops_argmax(a, axis=-1, keepdims=False): return _reduce(a, axis, keepdims, N.lib().engine_ops_argmax, "argmax")


def ops_gather(a, indices, axis=0):
    h = C.c_void_p()
    _check(N.lib().engine_ops_gather(a.raw, indices.raw, int(axis), C.byref(h)), "gather")
    return Tensor(h)


def ops_reshape(a, shape):
    shape = list(shape)
    h = C.c_void_p()
    _check(N.lib().engine_ops_reshape(a.raw, (N.i64 * max(len(shape), 1))(*shape), len(shape), C.byref(h)), "reshape")
    return Tensor(h)


def ops_transpose(a, perm):
    perm = list(perm)
    h = C.c_void_p()
    _check(N.lib().engine_ops_transpose(a.raw, (N.i32 * max(len(perm), 1))(*perm), len(perm), C.byref(h)), "transpose")
    return Tensor(h)


def ops_concat(inputs, axis=0):
    arr = (C.c_void_p * len(inputs))(*[t.raw for t in inputs])
    h = C.c_void_p()
    _check(N.lib().engine_ops_concat(arr, len(inputs), int(axis), C.byref(h)), "concat")
    return Tensor(h)


def ops_stack(inputs, axis=0):
    arr = (C.c_void_p * len(inputs))(*[t.raw for t in inputs])
    h = C.c_void_p()
    _check(N.lib().engine_ops_stack(arr, len(inputs), int(axis), C.byref(h)), "stack")
    return Tensor(h)


# ----------------------------------------------------------------------------
# Context / Model / Session
# ----------------------------------------------------------------------------
class Context:
    def __init__(self, precision: Optional[int] = None, device: Optional[int] = None):
        h = C.c_void_p()
        _check(N.lib().engine_context_create(C.byref(h)), "context_create")
        self._handle = h
        if precision is not None:
            self.set_precision(precision)
        if device is not None:
            self.set_device(device)

    def __del__(self):
        if getattr(self, "_handle", None) and N._lib is not None:
            N._lib.engine_context_destroy(self._handle)
            self._handle = None

    @property
    def raw(self):
        return self._handle

    def set_num_threads(self, n: int):
        _check(N.lib().engine_context_set_num_threads(self._handle, int(n)), "set_num_threads")
        return self

    def get_num_threads(self) -> int:
        return int(N.lib().engine_context_get_num_threads(self._handle))

    def set_precision(self, p: int):
        _check(N.lib().engine_context_set_precision(self._handle, int(p)), "set_precision")
        return self

    def get_precision(self) -> int:
        return int(N.lib().engine_context_get_precision(self._handle))

    def set_device(self, d: int):
        _check(N.lib().engine_context_set_device(self._handle, int(d)), "set_device")
        return self

    def get_device(self) -> int:
        return int(N.lib().engine_context_get_device(self._handle))


def _info(handle, idx, fn) -> TensorInfo:
    name = C.c_char_p()
    shp = (N.i64 * 8)()
    nd = N.i32()
    dt = C.c_int()
    _check(fn(handle, int(idx), C.byref(name), shp, C.byref(nd), C.byref(dt)), "model_info")
    return TensorInfo((name.value or b"").decode(), tuple(int(shp[i]) for i in range(nd.value)), int(dt.value))


class Model:
    def __init__(self, ctx: Context, path: str):
        self._ctx = ctx
        h = C.c_void_p()
        _check(N.lib().engine_model_load(ctx.raw if ctx else None, str(path).encode(), C.byref(h)), "model_load")
        self._handle = h

    def __del__(self):
        if getattr(self, "_handle", None) and N._lib is not None:
            N._lib.engine_model_destroy(self._handle)
            self._handle = None

    @property
    def raw(self):
        return self._handle

    @property
    def name(self) -> str:
        s = C.c_char_p()
        _check(N.lib().engine_model_name(self._handle, C.byref(s)), "model_name")
        return (s.value or b"").decode()

    @property
    def num_inputs(self) -> int:
        n = N.i32()
        _check(N.lib().engine_model_input_count(self._handle, C.byref(n)), "input_count")
        return n.value

    @property
    def num_outputs(self) -> int:
        n = N.i32()
        _check(N.lib().engine_model_output_count(self._handle, C.byref(n)), "output_count")
        return n.value

    def input_info(self, idx: int) -> TensorInfo:
        return _info(self._handle, idx, N.lib().engine_model_input_info)

    def plan_summary(self, precision: int = FP32, batch: int = 1) -> List[Tuple[str, str]]:
        """(kernel kind, node name) per launch, from a device-free lowering."""
        buf = C.create_string_buffer(1 << 20)
        n = N.i64()
        _check(N.lib().engine_model_plan_summary(self._handle, int(precision), int(batch), buf, len(buf),
                                                 C.byref(n)), "plan_summary")
        lines = [l for l in buf.value.decode().splitlines() if l]
        return [tuple(l.split(" ", 1)) for l in lines]

    def memory_plan(self, precision: int = FP32, batch: int = 1) -> Tuple[int, int]:
        """(arena bytes with live-range reuse, bytes with one buffer per value) of the
        activations, from a device-free lowering."""
        packed, unpacked = N.sz(), N.sz()
        _check(N.lib().engine_model_memory_plan(self._handle, int(precision), int(batch), C.byref(packed),
                                                C.byref(unpacked)), "memory_plan")
        return int(packed.value), int(unpacked.value)

    def output_info(self, idx: int) -> TensorInfo:
        return _info(self._handle, idx, N.lib().engine_model_output_info)


class Session:
    def __init__(self, ctx: Context, model: Model):
        self._ctx, self._model = ctx, model
        h = C.c_void_p()
        _check(N.lib().engine_session_create(ctx.raw if ctx else None, model.raw, C.byref(h)), "session_create")
        self._handle = h
        self._inputs = {}
        self._cb = None

    def __del__(self):
        if getattr(self, "_handle", None) and N._lib is not None:
            N._lib.engine_session_destroy(self._handle)
            self._handle = None

    @property
    def raw(self):
        return self._handle

    def set_input(self, index: int, tensor: Tensor):
        self._inputs[index] = tensor        # keep the tensor alive (the session borrows it)
        _check(N.lib().engine_session_set_input(self._handle, int(index), tensor.raw), "set_input")
        return self

    def run(self):
        _check(N.lib().engine_session_run(self._handle), "session_run")
        return self

    def output(self, index: int = 0) -> Tensor:
        h = C.c_void_p()
        _check(N.lib().engine_session_get_output(self._handle, int(index), C.byref(h)), "get_output")
        return Tensor(h, owns=False)

    def run_and_decode(self, meta: Optional[PreprocessMeta] = None, conf_thres=0.25, iou_thres=0.45, max_det=300):
        self.run()
        return decode_yolo(self.output(0), meta, conf_thres, iou_thres, max_det)

    def stats(self) -> dict:
        s = N.SessionStats()
        _check(N.lib().engine_session_get_stats(self._handle, C.byref(s)), "get_stats")
        return {"last_run_ms": s.last_run_ms, "runs": int(s.runs)}

    def keep_intermediate(self, idx: int) -> None:
        """Keep tensor `idx` of the graph readable after runs (debug_intermediate)."""
        _check(N.lib().engine_session_keep_intermediate(self._handle, int(idx)), "keep_intermediate")

    def debug_intermediate(self, idx: int) -> Tensor:
        h = C.c_void_p()
        _check(N.lib().engine_session_debug_intermediate(self._handle, int(idx), C.byref(h)), "debug_intermediate")
        return Tensor(h, owns=False)

    def set_profile_callback(self, fn):
        self._cb = N.PROFILE_FN(lambda name, ms, user: fn(name.decode(), ms))
        _check(N.lib().engine_session_set_profile_callback(self._handle, self._cb, None), "set_profile_callback")

    def clear_profile_callback(self):
        _check(N.lib().engine_session_clear_profile_callback(self._handle), "clear_profile_callback")
        self._cb = None

    # -- device-pointer execution (additive) --
    def output_shape(self, batch: int, index: int = 0) -> Tuple[int, ...]:
        shp = (N.i64 * 8)()
        nd = N.i32()
        _check(N.lib().engine_session_output_shape(self._handle, index, batch, shp, C.byref(nd)), "output_shape")
        return tuple(int(shp[i]) for i in range(nd.value))

    def run_device(self, d_input: int, batch: int, d_output: Optional[int] = None, stream: Optional[int] = None):
        _check(N.lib().engine_session_run_device(self._handle, d_input, batch, d_output, stream), "run_device")

    def device_output(self, batch: int, index: int = 0) -> int:
        """Device address of the session-owned output buffer for `batch` images."""
        ptr = C.c_void_p()
        _check(N.lib().engine_session_device_output(self._handle, index, batch, C.byref(ptr)), "device_output")
        return int(ptr.value)

    def set_step_timing(self, batch: int, enable: bool = True):
        _check(N.lib().engine_session_step_timing(self._handle, batch, 1 if enable else 0), "step_timing")

    def step_times(self, batch: int) -> List[float]:
        n = self.launch_count(batch)
        buf = (C.c_double * max(n, 1))()
        got = N.lib().engine_session_step_times(self._handle, batch, buf, n)
        if got < 0:
            _check(8, "step_times")
        return [buf[i] for i in range(got)]

    def launch_count(self, batch: int) -> int:
        return int(N.lib().engine_session_launch_count(self._handle, batch))


# ----------------------------------------------------------------------------
# Images (outside this library) and box mapping
# ----------------------------------------------------------------------------
class Image:
    """Decoded image (pdefa/python/src/pdefa/_bindings.py:693-733): width, height,
    channels, format (PdefaPixelFormat: 0 GRAY8, 1 RGB8, 2 RGBA8, 3 GRAY16) and the
    tightly packed row-major pixel bytes."""

    def __init__(self, handle):
        self._handle = handle

    def __del__(self):
        h = getattr(self, "_handle", None)
        if h and N._lib is not None:
            N._lib.pdefa_image_free(h)
            self._handle = None

    @property
    def width(self) -> int:
        return int(N.lib().pdefa_image_width(self._handle))

    @property
    def height(self) -> int:
        return int(N.lib().pdefa_image_height(self._handle))

    @property
    def channels(self) -> int:
        return int(N.lib().pdefa_image_channels(self._handle))

    @property
    def format(self) -> int:
        return int(N.lib().pdefa_image_format(self._handle))

    def pixels_bytes(self) -> bytes:
        n = C.c_size_t(0)
        ptr = N.lib().pdefa_image_pixels(self._handle, C.byref(n))
        return C.string_at(ptr, n.value) if ptr and n.value else b""

    def to_numpy(self):
        """uint8 [h, w, C] (GRAY16: [h, w, 2] big-endian byte pairs)."""
        import numpy as np
        a = np.frombuffer(self.pixels_bytes(), np.uint8)
        per = 2 if self.format == 3 else self.channels
        return a.reshape(self.height, self.width, per)


def load_image(path: str) -> Image:
    """Decode a PNG or baseline JPEG file to the reference's pixels (imageloader/src/loader.cpp:60-67)."""
    h = N.lib().pdefa_image_load(path.encode("utf-8"))
    if not h:
        raise PdefaError(f"load_image({path}): {(N.lib().pdefa_last_error() or b'').decode()}")
    return Image(h)


def preprocess_letterbox(img: Image, target_w: int = 640, target_h: int = 640, scale: float = 1.0 / 255.0,
                         pad_value: float = 0.0) -> Tuple["Tensor", PreprocessMeta]:
    """Letterbox on the GPU -> ([1, 3, H, W] fp32 Tensor, meta), bit-identical to the
    reference's preprocess_letterbox (imageloader/src/preprocess.cpp:15-147)."""
    t = C.c_void_p()
    m = N.PreMeta()
    _check(N.lib().pdefa_preprocess_letterbox(img._handle, C.byref(N.PreConfig(target_w, target_h, scale, pad_value)),
                                              C.byref(t), C.byref(m)), "preprocess_letterbox")
    return Tensor(t, owns=True), PreprocessMeta.from_c(m)


def prepare_for_engine(path: str, target_w: int = 640, target_h: int = 640, scale: float = 1.0 / 255.0,
                       pad_value: float = 0.0) -> Tuple["Tensor", PreprocessMeta]:
    """Image file -> letterboxed [1, 3, H, W] fp32 Tensor + meta."""
    t = C.c_void_p()
    m = N.PreMeta()
    _check(N.lib().pdefa_prepare_for_engine(path.encode("utf-8"), target_w, target_h, scale, pad_value,
                                            C.byref(t), C.byref(m)), "prepare_for_engine")
    return Tensor(t, owns=True), PreprocessMeta.from_c(m)


def load_image_as_tensor(path: str, target_w: int = 640, target_h: int = 640) -> "Tensor":
    t = C.c_void_p()
    _check(N.lib().pdefa_load_image_as_tensor(path.encode("utf-8"), target_w, target_h, C.byref(t)),
           "load_image_as_tensor")
    return Tensor(t, owns=True)


def _u8_batch(images):
    """[h, w] (gray), [h, w, C], [N, h, w] (gray) or [N, h, w, C] uint8 ->
    ([N, h, w, C] array, C); a 3-D array whose last extent is 1, 3 or 4 is one image."""
    import numpy as np
    a = np.ascontiguousarray(images, dtype=np.uint8)
    if a.ndim == 2:
        a = a[None, :, :, None]
    elif a.ndim == 3:
        a = a[None] if a.shape[2] in (1, 3, 4) else a[..., None]
    if a.ndim != 4 or a.shape[3] not in (1, 3, 4):
        raise PdefaError("letterbox: images must be uint8 [h, w], [h, w, C] or [N, h, w, C] with C = 1, 3 or 4")
    return np.ascontiguousarray(a), int(a.shape[3])


def letterbox_meta(src_w: int, src_h: int, target_w: int = 640, target_h: int = 640, scale: float = 1.0 / 255.0,
                   pad_value: float = 0.0) -> PreprocessMeta:
    """Letterbox geometry of a src_w x src_h image (imageloader/src/preprocess.cpp:22-41)."""
    m = N.PreMeta()
    _check(N.lib().pdefa_letterbox_meta(int(src_w), int(src_h), C.byref(N.PreConfig(target_w, target_h, scale,
                                                                                        pad_value)), C.byref(m)),
           "letterbox_meta")
    return PreprocessMeta.from_c(m)


def letterbox_u8(images, target_w: int = 640, target_h: int = 640, scale: float = 1.0 / 255.0,
                 pad_value: float = 0.0, device: int = 0):
    """GPU letterbox of decoded 8-bit images -> (float32 [N, 3, target_h, target_w]
    numpy array, PreprocessMeta). images: [h, w] gray, [h, w, C] or [N, h, w, C]
    uint8 with C = 1, 3 or 4 (RGBA drops alpha). Bit-identical to the reference's
    preprocess_letterbox (imageloader/src/preprocess.cpp:15-147)."""
    import numpy as np
    a, ch = _u8_batch(images)
    n, h, w = a.shape[:3]
    out = np.empty((n, 3, target_h, target_w), np.float32)
    m = N.PreMeta()
    _check(N.lib().pdefa_letterbox(a.ctypes.data, n, h, w, ch, C.byref(N.PreConfig(target_w, target_h, scale,
                                                                                     pad_value)),
                                   out.ctypes.data, C.byref(m), int(device)), "letterbox")
    return out, PreprocessMeta.from_c(m)


def map_box_to_original(box: Box, meta: PreprocessMeta) -> Box:
    i = (C.c_float * 4)(box.x1, box.y1, box.x2, box.y2)
    o = (C.c_float * 4)()
    m = meta.to_c()
    _check(N.lib().pdefa_map_box_to_original(i, C.byref(m), o), "map_box_to_original")
    return Box(o[0], o[1], o[2], o[3])


def map_point_to_original(x: float, y: float, meta: PreprocessMeta) -> Tuple[float, float]:
    cx, cy = C.c_float(x), C.c_float(y)
    m = meta.to_c()
    _check(N.lib().pdefa_map_point_to_original(C.byref(cx), C.byref(cy), C.byref(m)), "map_point_to_original")
    return cx.value, cy.value


# ----------------------------------------------------------------------------
# YOLO decode (GPU)
# ----------------------------------------------------------------------------
def _det_dict(d: N.Detection) -> dict:
    return {"x1": d.x1, "y1": d.y1, "x2": d.x2, "y2": d.y2, "conf": float(d.conf), "cls": int(d.cls)}


def decode_yolo_arrays(preds, metas=None, conf_thres=0.25, iou_thres=0.45, max_det=300, device=0):
    """GPU decode of a [B, 4+nc, A] float32 array (numpy); returns per-image
    lists of PdefaDetection records (with the anchor index)."""
    import numpy as np
    p = np.ascontiguousarray(preds, dtype=np.float32)
    if p.ndim == 2:
        p = p[None]
    B, ch, A = p.shape
    counts = (N.i32 * B)()
    md = max(int(max_det), 0)
    dets = (N.Detection * max(B * md, 1))()
    marr = None
    if metas is not None:
        ms = metas if isinstance(metas, (list, tuple)) else [metas] * B
        marr = (N.PreMeta * B)(*[m.to_c() for m in ms])
    _check(N.lib().pdefa_decode_yolo(p.ctypes.data, 0, B, ch, A, marr, float(conf_thres), float(iou_thres), md,
                                     counts, dets, int(device)), "decode_yolo")
    return [[dets[b * md + i] for i in range(counts[b])] for b in range(B)]


def decode_yolo(output, meta=None, conf_thres=0.25, iou_thres=0.45, max_det=300):
    """YOLOv8 raw output -> [{'x1','y1','x2','y2','conf','cls'}, ...]
    (same fields, order and values as _bindings.py:1095-1175)."""
    import numpy as np
    if isinstance(output, Tensor):
        arr = output.to_numpy()
    elif isinstance(output, np.ndarray):
        arr = output
    else:
        arr = np.asarray(output, dtype=np.float32)
    arr = np.asarray(arr, dtype=np.float32)
    while arr.ndim > 2 and arr.shape[0] == 1:
        arr = arr[0]
    if arr.ndim == 2:
        if arr.shape[0] < 5:
            raise PdefaError(f"decode_yolo: unexpected shape {arr.shape}")
        dets = decode_yolo_arrays(arr[None], meta, conf_thres, iou_thres, max_det)[0]
        return [_det_dict(d) for d in dets]
    if arr.ndim == 3:
        res = decode_yolo_arrays(arr, meta, conf_thres, iou_thres, max_det)
        return [[_det_dict(d) for d in r] for r in res]
    raise PdefaError(f"decode_yolo: unexpected shape {arr.shape}")


def _model_input_shape(model: Model, idx: int = 0):
    return model.input_info(idx).shape


def prepare_for_model(model: Model, path: str, input_idx: int = 0, scale: float = 1.0 / 255.0,
                      pad_value: float = 0.0):
    shape = _model_input_shape(model, input_idx)
    if len(shape) != 4:
        raise PdefaError(f"prepare_for_model: expected 4D input, got {shape}")
    _, _, H, W = shape
    return prepare_for_engine(path, W, H, scale, pad_value)


class EngineModel:
    """One-line inference (_bindings.py:1250-1282)."""

    def __init__(self, ctx: Context, model: Model, session: Session):
        self.ctx, self.model, self.session = ctx, model, session

    def __call__(self, image, conf_thres: float = 0.25, iou_thres: float = 0.45):
        if isinstance(image, str):
            tensor, meta = prepare_for_model(self.model, image)
        else:
            tensor, meta = (image if isinstance(image, Tensor) else Tensor.from_numpy(image)), None
        self.session.set_input(0, tensor)
        self.session.run()
        return decode_yolo(self.session.output(0), meta, conf_thres, iou_thres)

    def set_num_threads(self, n: int):
        self.ctx.set_num_threads(n)
        return self


def load(engine_path: str, precision: Optional[int] = None) -> EngineModel:
    ctx = Context(precision=precision)
    model = Model(ctx, engine_path)
    return EngineModel(ctx, model, Session(ctx, model))
