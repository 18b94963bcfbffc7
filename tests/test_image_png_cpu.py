"""PNG decoding (pdefa_image_load, csrc/image_png.cpp) against the reference decoder.

Seeded images of every PNG colour type and bit depth, with and without tRNS, Adam7
interlacing and all five row filters, are written by a small encoder here and
decoded by both this library and the reference library built from its sources
(imageloader/src/png/*.cpp through pdefa_image_load); width, height, pixel format
and every pixel byte must agree. Malformed files must fail in both.
"""
import ctypes as C
import os
import struct
import zlib

import numpy as np
import pytest

import pdefa_b200 as pb

REF_LIB = os.path.join(os.path.dirname(os.path.dirname(__file__)), "oracle", "_ref", "libpdefa_ref.so")
ADAM7 = [(0, 0, 8, 8), (4, 0, 8, 8), (0, 4, 4, 8), (2, 0, 4, 4), (0, 2, 2, 4), (1, 0, 2, 2), (0, 1, 1, 2)]
CHANNELS = {0: 1, 2: 3, 3: 1, 4: 2, 6: 4}


def _pack_row(samples, bd):
    if bd == 8:
        return bytes(samples.astype(np.uint8))
    if bd == 16:
        return samples.astype(">u2").tobytes()
    per = 8 // bd
    out = bytearray((len(samples) + per - 1) // per)
    for i, v in enumerate(samples):
        out[i // per] |= int(v) << (8 - bd * (i % per + 1))
    return bytes(out)


def _paeth(a, b, c):
    p = a + b - c
    pa, pb_, pc = abs(p - a), abs(p - b), abs(p - c)
    return a if pa <= pb_ and pa <= pc else (b if pb_ <= pc else c)


def _filter_rows(rows, bpp, rng):
    out = bytearray()
    prev = bytes(len(rows[0])) if rows else b""
    for row in rows:
        f = int(rng.integers(0, 5))
        enc = bytearray(len(row))
        for i in range(len(row)):
            a = row[i - bpp] if i >= bpp else 0
            b = prev[i]
            c = prev[i - bpp] if i >= bpp else 0
            pred = [0, a, b, (a + b) // 2, _paeth(a, b, c)][f]
            enc[i] = (row[i] - pred) & 0xFF
        out += bytes([f]) + enc
        prev = row
    return bytes(out)


def write_png(path, samples, ct, bd, palette=None, trns=None, interlace=False, seed=0, crc_ok=True):
    """samples: [h, w, channels] integer array of raw PNG samples."""
    rng = np.random.default_rng(seed)
    h, w, ch = samples.shape
    bpp = max(1, (bd * ch + 7) // 8)
    passes = ADAM7 if interlace else [(0, 0, 1, 1)]
    raw = b""
    for x0, y0, dx, dy in passes:
        sub = samples[y0::dy, x0::dx]
        if sub.size == 0:
            continue
        rows = [_pack_row(sub[y].reshape(-1), bd) for y in range(sub.shape[0])]
        raw += _filter_rows(rows, bpp, rng)

    def chunk(t, d, good=True):
        crc = zlib.crc32(t + d) & 0xFFFFFFFF
        return struct.pack(">I", len(d)) + t + d + struct.pack(">I", crc if good else crc ^ 1)

    body = chunk(b"IHDR", struct.pack(">IIBBBBB", w, h, bd, ct, 0, 0, 1 if interlace else 0))
    if palette is not None:
        body += chunk(b"PLTE", bytes(palette.astype(np.uint8).reshape(-1)))
    if trns is not None:
        body += chunk(b"tRNS", bytes(trns))
    body += chunk(b"IDAT", zlib.compress(raw), crc_ok) + chunk(b"IEND", b"")
    with open(path, "wb") as f:
        f.write(b"\x89PNG\r\n\x1a\n" + body)


def _cases():
    cases = []
    for interlace in (False, True):
        for bd in (1, 2, 4, 8, 16):
            cases.append((0, bd, False, interlace))
        cases.append((0, 8, True, interlace))
        cases.append((0, 16, True, interlace))
        for bd in (8, 16):
            cases += [(2, bd, False, interlace), (2, bd, True, interlace), (4, bd, False, interlace),
                      (6, bd, False, interlace)]
        for bd in (1, 2, 4, 8):
            cases += [(3, bd, False, interlace), (3, bd, True, interlace)]
    return cases


def _make(tmp_path, k, ct, bd, with_trns, interlace):
    rng = np.random.default_rng(100 + k)
    h, w = int(rng.integers(1, 23)), int(rng.integers(1, 29))
    ch = CHANNELS[ct]
    top = (1 << bd) - 1
    palette = trns = None
    if ct == 3:
        npal = int(rng.integers(1, min(256, 1 << bd) + 1))
        samples = rng.integers(0, npal, (h, w, 1))
        palette = rng.integers(0, 256, (npal, 3))
        if with_trns:
            trns = rng.integers(0, 256, int(rng.integers(1, npal + 1))).astype(np.uint8).tobytes()
    else:
        samples = rng.integers(0, top + 1, (h, w, ch))
        if with_trns:
            key = samples[0, 0]
            vals = [int(key[0])] if ct == 0 else [int(v) for v in key]
            trns = b"".join(struct.pack(">H", v) for v in vals)
    p = str(tmp_path / f"c{k}.png")
    write_png(p, samples, ct, bd, palette, trns, interlace, seed=k)
    return p


def _ref_decode(path):
    L = C.CDLL(REF_LIB)
    L.pdefa_image_load.restype = C.c_void_p
    L.pdefa_image_load.argtypes = [C.c_char_p]
    for f in ("pdefa_image_width", "pdefa_image_height", "pdefa_image_format"):
        getattr(L, f).argtypes = [C.c_void_p]
        getattr(L, f).restype = C.c_int32
    L.pdefa_image_pixels.argtypes = [C.c_void_p, C.POINTER(C.c_size_t)]
    L.pdefa_image_pixels.restype = C.c_void_p
    L.pdefa_image_free.argtypes = [C.c_void_p]
    img = L.pdefa_image_load(path.encode())
    if not img:
        return None
    n = C.c_size_t()
    ptr = L.pdefa_image_pixels(img, C.byref(n))
    out = (L.pdefa_image_width(img), L.pdefa_image_height(img), L.pdefa_image_format(img), C.string_at(ptr, n.value))
    L.pdefa_image_free(img)
    return out


@pytest.mark.parametrize("k", range(len(_cases())))
def test_png_matches_reference_decoder(tmp_path, k):
    if not os.path.exists(REF_LIB):
        pytest.skip("reference library not built")
    ct, bd, with_trns, interlace = _cases()[k]
    p = _make(tmp_path, k, ct, bd, with_trns, interlace)
    ref = _ref_decode(p)
    assert ref is not None
    img = pb.load_image(p)
    assert (img.width, img.height, img.format) == ref[:3]
    assert img.pixels_bytes() == ref[3]


def test_png_known_pixels(tmp_path):
    """Without the reference: 8-bit RGB and 4-bit gray decode to the written samples."""
    rng = np.random.default_rng(3)
    a = rng.integers(0, 256, (9, 14, 3))
    p = str(tmp_path / "rgb.png")
    write_png(p, a, 2, 8, interlace=True, seed=1)
    img = pb.load_image(p)
    assert img.format == 1 and img.channels == 3
    np.testing.assert_array_equal(img.to_numpy(), a.astype(np.uint8))
    g = rng.integers(0, 16, (5, 7, 1))
    p = str(tmp_path / "g4.png")
    write_png(p, g, 0, 4, seed=2)
    np.testing.assert_array_equal(pb.load_image(p).to_numpy()[..., 0], ((g[..., 0] * 255 + 7) // 15).astype(np.uint8))


def test_png_malformed_files_fail(tmp_path):
    a = np.zeros((4, 4, 3), np.int64)
    bad_crc = str(tmp_path / "crc.png")
    write_png(bad_crc, a, 2, 8, crc_ok=False)
    trunc = str(tmp_path / "trunc.png")
    write_png(trunc, a, 2, 8)
    data = open(trunc, "rb").read()
    open(trunc, "wb").write(data[:len(data) - 20])
    for p in (bad_crc, trunc, str(tmp_path / "missing.png")):
        with pytest.raises(pb.PdefaError):
            pb.load_image(p)
        if os.path.exists(REF_LIB):
            assert _ref_decode(p) is None
