"""ctypes driver for the C letterbox restatement (``oracle/letterbox_ref.c``).

TEST INFRASTRUCTURE ONLY: the parity checker of the GPU letterbox kernel. The product
(``pdefa_b200``) never imports it. The shared object is built by ``__graft_entry__.build``
into ``oracle/_lib/`` (and on first use here if it is missing).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "letterbox_ref.c")
LIB = os.path.join(HERE, "_lib", "libletterbox_ref.so")
_lib = None


def build() -> str:
    os.makedirs(os.path.dirname(LIB), exist_ok=True)
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < os.path.getmtime(SRC):
        subprocess.run(["gcc", "-O2", "-ffp-contract=off", "-fPIC", "-shared", SRC, "-o", LIB, "-lm"], check=True)
    return LIB


def lib():
    global _lib
    if _lib is None:
        _lib = C.CDLL(build())
        _lib.letterbox_ref.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float, C.c_float,
                                       C.c_void_p, C.c_void_p, C.POINTER(C.c_float)]
        _lib.letterbox_ref.restype = C.c_int
    return _lib


def letterbox(img: np.ndarray, target_w: int = 640, target_h: int = 640, scale: float = 1.0 / 255.0,
              pad_value: float = 0.0):
    """img: [h, w] or [h, w, C] uint8 (C = 1, 3, 4) -> (out [3, H, W] float32,
    meta dict with the PdefaPreprocessMeta fields)."""
    a = np.ascontiguousarray(img, dtype=np.uint8)
    h, w = a.shape[:2]
    ch = 1 if a.ndim == 2 else a.shape[2]
    out = np.empty((3, target_h, target_w), np.float32)
    meta = np.zeros(8, np.int32)
    ratio = C.c_float()
    rc = lib().letterbox_ref(a.ctypes.data, h, w, ch, target_w, target_h, scale, pad_value, out.ctypes.data,
                             meta.ctypes.data, C.byref(ratio))
    if rc != 0:
        raise ValueError("letterbox_ref: invalid image or target")
    names = ("target_w", "target_h", "orig_w", "orig_h", "pad_x", "pad_y", "scaled_w", "scaled_h")
    m = {k: int(v) for k, v in zip(names, meta)}
    m["ratio"] = ratio.value
    return out, m
