"""Generates tests/golden/letterbox_ref.npz from the reference letterbox preprocess.

Runs the reference library built from its own sources (oracle/ref.mk ->
oracle/_ref/libpdefa_ref.so) through its public C API: each seeded uint8 image is
written as a PNG (colour types 0, 2, 6), read back with pdefa_image_load
(pdefa/src/pdefa_c_api.cpp) and letterboxed with pdefa_preprocess_letterbox
(pdefa_c_api.cpp:83-126 -> imageloader/src/preprocess.cpp:15-147). The fixture keeps
the pixels, the config, the float32 NCHW output and the meta record of every case.

    python tests/golden/make_letterbox_golden.py
"""
from __future__ import annotations

import ctypes as C
import os
import struct
import sys
import tempfile
import zlib

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
OUT = os.path.join(ROOT, "tests", "golden", "letterbox_ref.npz")

# (h, w, channels, target_w, target_h, scale, pad_value)
CASES = [
    (37, 53, 3, 64, 64, 1 / 255, 0.0),      # upscale, rows padded
    (64, 48, 3, 64, 64, 1 / 255, 0.0),      # ratio 1, columns padded
    (20, 20, 1, 64, 64, 1 / 255, 0.0),      # gray, upscale 3.2
    (31, 17, 4, 64, 64, 1 / 255, 0.0),      # RGBA (alpha dropped)
    (97, 131, 3, 48, 40, 1 / 255, 0.0),     # downscale into a non-square target
    (1, 7, 3, 16, 16, 1 / 255, 0.0),        # one row
    (5, 1, 3, 16, 16, 1 / 255, 0.0),        # one column
    (40, 40, 3, 40, 40, 1 / 255, 114 / 255),  # identity, YOLO grey padding
    (23, 29, 3, 32, 32, 1.0, 0.5),          # unnormalised, other pad value
    (200, 120, 3, 56, 56, 1 / 255, 0.0),    # downscale 0.28, columns padded
]


class Cfg(C.Structure):
    _fields_ = [("target_w", C.c_int32), ("target_h", C.c_int32), ("scale", C.c_float), ("pad_value", C.c_float)]


class Meta(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("target_w", "target_h", "orig_w", "orig_h", "pad_x", "pad_y",
                                         "scaled_w", "scaled_h")] + [("ratio", C.c_float)]


def write_png(path: str, a: np.ndarray) -> None:
    h, w = a.shape[:2]
    ch = 1 if a.ndim == 2 else a.shape[2]
    raw = b"".join(b"\x00" + a[y].tobytes() for y in range(h))

    def chunk(t: bytes, d: bytes) -> bytes:
        return struct.pack(">I", len(d)) + t + d + struct.pack(">I", zlib.crc32(t + d) & 0xFFFFFFFF)

    ihdr = struct.pack(">IIBBBBB", w, h, 8, {1: 0, 3: 2, 4: 6}[ch], 0, 0, 0)
    with open(path, "wb") as f:
        f.write(b"\x89PNG\r\n\x1a\n" + chunk(b"IHDR", ihdr) + chunk(b"IDAT", zlib.compress(raw)) + chunk(b"IEND", b""))


def reference_letterbox(L, png: str, tw: int, th: int, scale: float, pad: float):
    img = L.pdefa_image_load(png.encode())
    if not img:
        raise RuntimeError(L.pdefa_last_error())
    t, m = C.c_void_p(), Meta()
    cfg = Cfg(tw, th, scale, pad)
    rc = L.pdefa_preprocess_letterbox(img, C.byref(cfg), C.byref(t), C.byref(m))
    if rc != 0:
        raise RuntimeError(L.pdefa_last_error())
    d, nb = C.c_void_p(), C.c_size_t()
    L.engine_tensor_data(t, C.byref(d), C.byref(nb))
    out = np.ctypeslib.as_array((C.c_float * (3 * th * tw)).from_address(d.value)).copy().reshape(3, th, tw)
    L.engine_tensor_destroy(t)
    L.pdefa_image_free(img)
    meta = np.array([m.target_w, m.target_h, m.orig_w, m.orig_h, m.pad_x, m.pad_y, m.scaled_w, m.scaled_h], np.int32)
    return out, meta, np.float32(m.ratio)


def main() -> None:
    L = C.CDLL(os.path.join(ROOT, "oracle", "_ref", "libpdefa_ref.so"))
    L.pdefa_image_load.restype = C.c_void_p
    L.pdefa_image_load.argtypes = [C.c_char_p]
    L.pdefa_image_free.argtypes = [C.c_void_p]
    L.pdefa_preprocess_letterbox.argtypes = [C.c_void_p, C.POINTER(Cfg), C.POINTER(C.c_void_p), C.POINTER(Meta)]
    L.engine_tensor_data.argtypes = [C.c_void_p, C.POINTER(C.c_void_p), C.POINTER(C.c_size_t)]
    L.engine_tensor_destroy.argtypes = [C.c_void_p]
    L.pdefa_last_error.restype = C.c_char_p
    rng = np.random.default_rng(2024)
    arrays = {}
    with tempfile.TemporaryDirectory() as tmp:
        for i, (h, w, ch, tw, th, scale, pad) in enumerate(CASES):
            img = rng.integers(0, 256, (h, w) if ch == 1 else (h, w, ch), dtype=np.uint8)
            png = os.path.join(tmp, f"c{i}.png")
            write_png(png, img)
            out, meta, ratio = reference_letterbox(L, png, tw, th, scale, pad)
            arrays[f"c{i}_img"] = img
            arrays[f"c{i}_cfg"] = np.array([tw, th, scale, pad], np.float64)
            arrays[f"c{i}_out"] = out
            arrays[f"c{i}_meta"] = meta
            arrays[f"c{i}_ratio"] = np.array(ratio, np.float32)
    arrays["n_cases"] = np.array(len(CASES))
    np.savez_compressed(OUT, **arrays)
    print(f"wrote {OUT} ({os.path.getsize(OUT)} bytes, {len(CASES)} cases)")


if __name__ == "__main__":
    sys.exit(main())
