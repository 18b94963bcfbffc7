"""ctypes driver for the compiled reference engine (``oracle/_ref/libpdefa_ref.so``).

TEST INFRASTRUCTURE ONLY. This module runs the reference pdefa CPU engine, built
from its own sources by ``oracle/ref.mk``, as the parity checker and as the timed
CPU baseline. The product (``pdefa_b200``) never imports it.

Entry points used (signatures from ``PDEFA1.0/include/engine/engine_c_api.h:64-234``):
context/model/session lifecycle, ``engine_session_run``, ``engine_ops_matmul``.
"""
from __future__ import annotations

import ctypes
import os
import time
from typing import Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_ref", "libpdefa_ref.so")

_lib = None
vp = ctypes.c_void_p


def available() -> bool:
    return os.path.isfile(LIB_PATH)


def lib():
    global _lib
    if _lib is None:
        if not available():
            raise RuntimeError(f"reference engine not built: {LIB_PATH} (run make -f oracle/ref.mk)")
        L = ctypes.CDLL(LIB_PATH)
        i64p = ctypes.POINTER(ctypes.c_int64)
        L.engine_context_create.argtypes = [ctypes.POINTER(vp)]
        L.engine_context_set_num_threads.argtypes = [vp, ctypes.c_int32]
        L.engine_context_destroy.argtypes = [vp]
        L.engine_model_load.argtypes = [vp, ctypes.c_char_p, ctypes.POINTER(vp)]
        L.engine_model_destroy.argtypes = [vp]
        L.engine_session_create.argtypes = [vp, vp, ctypes.POINTER(vp)]
        L.engine_session_destroy.argtypes = [vp]
        L.engine_session_set_input.argtypes = [vp, ctypes.c_int32, vp]
        L.engine_session_run.argtypes = [vp]
        L.engine_session_get_output.argtypes = [vp, ctypes.c_int32, ctypes.POINTER(vp)]
        L.engine_tensor_create_from_data.argtypes = [ctypes.POINTER(vp), i64p, ctypes.c_int32,
                                                     ctypes.c_int, vp, ctypes.c_size_t]
        L.engine_tensor_create.argtypes = [ctypes.POINTER(vp), i64p, ctypes.c_int32, ctypes.c_int]
        L.engine_tensor_destroy.argtypes = [vp]
        L.engine_tensor_data.argtypes = [vp, ctypes.POINTER(vp), ctypes.POINTER(ctypes.c_size_t)]
        L.engine_tensor_shape.argtypes = [vp, i64p, ctypes.POINTER(ctypes.c_int32)]
        L.engine_ops_matmul.argtypes = [vp, vp, vp]
        L.engine_last_error.restype = ctypes.c_char_p
        _lib = L
    return _lib


def _check(rc, what):
    if rc != 0:
        raise RuntimeError(f"reference {what} failed rc={rc}: {lib().engine_last_error().decode()}")


def _tensor_from(arr: np.ndarray):
    arr = np.ascontiguousarray(arr, dtype=np.float32)
    shp = (ctypes.c_int64 * arr.ndim)(*arr.shape)
    t = vp()
    _check(lib().engine_tensor_create_from_data(ctypes.byref(t), shp, arr.ndim, 0,
                                                arr.ctypes.data_as(vp), arr.nbytes), "tensor_create")
    return t


def _to_numpy(t) -> np.ndarray:
    L = lib()
    shp = (ctypes.c_int64 * 8)()
    nd = ctypes.c_int32()
    _check(L.engine_tensor_shape(t, shp, ctypes.byref(nd)), "tensor_shape")
    ptr, nb = vp(), ctypes.c_size_t()
    _check(L.engine_tensor_data(t, ctypes.byref(ptr), ctypes.byref(nb)), "tensor_data")
    buf = (ctypes.c_uint8 * nb.value).from_address(ptr.value)
    return np.frombuffer(bytes(buf), dtype=np.float32).reshape([shp[i] for i in range(nd.value)]).copy()


class RefContext:
    def __init__(self, threads: Optional[int] = None):
        self.h = vp()
        _check(lib().engine_context_create(ctypes.byref(self.h)), "context_create")
        if threads:
            _check(lib().engine_context_set_num_threads(self.h, int(threads)), "set_num_threads")

    def __del__(self):
        if getattr(self, 'h', None) and _lib is not None:
            _lib.engine_context_destroy(self.h)


class RefSession:
    """Loads an ``.engine`` file and runs batch-1 inference on the reference engine."""

    def __init__(self, path: str, threads: Optional[int] = None):
        self.ctx = RefContext(threads)
        L = lib()
        self.model = vp()
        _check(L.engine_model_load(self.ctx.h, path.encode(), ctypes.byref(self.model)), "model_load")
        self.sess = vp()
        _check(L.engine_session_create(self.ctx.h, self.model, ctypes.byref(self.sess)), "session_create")

    def run(self, x: np.ndarray) -> np.ndarray:
        L = lib()
        t = _tensor_from(x)
        try:
            _check(L.engine_session_set_input(self.sess, 0, t), "set_input")
            _check(L.engine_session_run(self.sess), "session_run")
            out = vp()
            _check(L.engine_session_get_output(self.sess, 0, ctypes.byref(out)), "get_output")
            return _to_numpy(out)
        finally:
            L.engine_tensor_destroy(t)

    def run_all(self, x: np.ndarray, n_outputs: int):
        """Outputs 0..n_outputs-1 of one batch-1 run (float32 outputs only)."""
        L = lib()
        t = _tensor_from(x)
        try:
            _check(L.engine_session_set_input(self.sess, 0, t), "set_input")
            _check(L.engine_session_run(self.sess), "session_run")
            res = []
            for i in range(n_outputs):
                out = vp()
                _check(L.engine_session_get_output(self.sess, i, ctypes.byref(out)), "get_output")
                res.append(_to_numpy(out))
            return res
        finally:
            L.engine_tensor_destroy(t)

    def run_batch(self, xs: np.ndarray) -> np.ndarray:
        """Image-by-image, as the reference's BatchInference does (batch.py:45-60)."""
        return np.stack([self.run(xs[i:i + 1])[0] for i in range(xs.shape[0])])

    def time_run(self, x: np.ndarray, iters: int) -> float:
        """Median wall seconds of ``iters`` runs."""
        L = lib()
        t = _tensor_from(x)
        try:
            _check(L.engine_session_set_input(self.sess, 0, t), "set_input")
            ts = []
            for _ in range(iters):
                t0 = time.perf_counter()
                _check(L.engine_session_run(self.sess), "session_run")
                ts.append(time.perf_counter() - t0)
            return float(np.median(ts))
        finally:
            L.engine_tensor_destroy(t)

    def __del__(self):
        if _lib is not None:
            if getattr(self, 'sess', None):
                _lib.engine_session_destroy(self.sess)
            if getattr(self, 'model', None):
                _lib.engine_model_destroy(self.model)


def matmul(a: np.ndarray, b: np.ndarray, threads: Optional[int] = None) -> np.ndarray:
    """C = A @ B through ``engine_ops_matmul`` (AVX2 sgemm, matmul_avx2.cpp:538)."""
    ctx = RefContext(threads)  # noqa: F841  (sets the global pool size)
    L = lib()
    ta, tb = _tensor_from(a), _tensor_from(b)
    shp = (ctypes.c_int64 * 2)(a.shape[0], b.shape[1])
    tc = vp()
    _check(L.engine_tensor_create(ctypes.byref(tc), shp, 2, 0), "tensor_create")
    try:
        _check(L.engine_ops_matmul(ta, tb, tc), "ops_matmul")
        return _to_numpy(tc)
    finally:
        for t in (ta, tb, tc):
            L.engine_tensor_destroy(t)


def time_matmul(a: np.ndarray, b: np.ndarray, iters: int, threads: Optional[int] = None) -> float:
    ctx = RefContext(threads)  # noqa: F841
    L = lib()
    ta, tb = _tensor_from(a), _tensor_from(b)
    shp = (ctypes.c_int64 * 2)(a.shape[0], b.shape[1])
    tc = vp()
    _check(L.engine_tensor_create(ctypes.byref(tc), shp, 2, 0), "tensor_create")
    try:
        ts = []
        for _ in range(iters):
            t0 = time.perf_counter()
            _check(L.engine_ops_matmul(ta, tb, tc), "ops_matmul")
            ts.append(time.perf_counter() - t0)
        return float(np.median(ts))
    finally:
        for t in (ta, tb, tc):
            L.engine_tensor_destroy(t)
