"""Writes tests/golden/jpeg_ref.npz: a few seeded JPEG files (Pillow / libjpeg)
and the pixels the reference decoder gives for them.

The reference is the pdefa C library built from its own sources by
oracle/ref.mk (oracle/_ref/libpdefa_ref.so, pdefa_image_load ->
imageloader/src/jpeg/jpeg_decoder.cpp:157-179). The JPEG bytes are stored
as well, so the fixture does not depend on the encoder's version.

Usage: python tests/golden/make_jpeg_golden.py
"""
import ctypes as C
import io
import os
import tempfile

import numpy as np
from PIL import Image

HERE = os.path.dirname(os.path.abspath(__file__))
REF_LIB = os.path.join(HERE, "..", "..", "oracle", "_ref", "libpdefa_ref.so")


def content(rng, h, w, ch):
    y, x = np.mgrid[0:h, 0:w].astype(np.float32)
    a = np.stack([128 + 90 * np.sin(rng.uniform(0.05, 0.5) * x) * np.cos(rng.uniform(0.05, 0.5) * y)
                  for _ in range(ch)], -1)
    a += rng.normal(0, 10, a.shape)
    return np.clip(a, 0, 255).astype(np.uint8)


CASES = [
    ("rgb444_q95", 16, 24, "RGB", dict(quality=95, subsampling=0)),
    ("rgb420_q75_odd", 21, 35, "RGB", dict(quality=75, subsampling=2)),
    ("rgb422_rst", 24, 40, "RGB", dict(quality=85, subsampling=1, restart_marker_blocks=2)),
    ("gray_q90", 19, 23, "L", dict(quality=90)),
    ("rgb420_optimized", 32, 32, "RGB", dict(quality=60, optimize=True)),
]


def ref_decode(L, data):
    with tempfile.NamedTemporaryFile(suffix=".jpg", delete=False) as f:
        f.write(data)
        path = f.name
    try:
        img = L.pdefa_image_load(path.encode())
        assert img, L.pdefa_last_error()
        n = C.c_size_t()
        ptr = L.pdefa_image_pixels(img, C.byref(n))
        out = (L.pdefa_image_width(img), L.pdefa_image_height(img), L.pdefa_image_format(img),
               C.string_at(ptr, n.value))
        L.pdefa_image_free(img)
        return out
    finally:
        os.unlink(path)


def main():
    L = C.CDLL(REF_LIB)
    L.pdefa_image_load.restype = C.c_void_p
    L.pdefa_image_load.argtypes = [C.c_char_p]
    L.pdefa_last_error.restype = C.c_char_p
    for f in ("pdefa_image_width", "pdefa_image_height", "pdefa_image_format"):
        getattr(L, f).argtypes = [C.c_void_p]
        getattr(L, f).restype = C.c_int32
    L.pdefa_image_pixels.argtypes = [C.c_void_p, C.POINTER(C.c_size_t)]
    L.pdefa_image_pixels.restype = C.c_void_p
    L.pdefa_image_free.argtypes = [C.c_void_p]
    out = {"names": np.array([c[0] for c in CASES])}
    for i, (name, h, w, mode, kw) in enumerate(CASES):
        rng = np.random.default_rng(900 + i)
        a = content(rng, h, w, 1 if mode == "L" else 3)
        b = io.BytesIO()
        Image.fromarray(a[..., 0] if mode == "L" else a, mode=mode).save(b, "JPEG", **kw)
        data = b.getvalue()
        W, H, fmt, px = ref_decode(L, data)
        out[f"{name}.jpg"] = np.frombuffer(data, np.uint8)
        out[f"{name}.whf"] = np.array([W, H, fmt], np.int32)
        out[f"{name}.rgb"] = np.frombuffer(px, np.uint8)
    np.savez_compressed(os.path.join(HERE, "jpeg_ref.npz"), **out)


if __name__ == "__main__":
    main()
