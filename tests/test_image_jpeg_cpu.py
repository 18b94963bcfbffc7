"""Baseline JPEG decoding (pdefa_image_load, csrc/image_jpeg.cpp) against the
reference decoder (imageloader/src/jpeg/*.cpp, built from its sources into
oracle/_ref through pdefa_image_load).

Seeded images are encoded by Pillow and OpenCV (libjpeg) with every chroma
subsampling they offer (4:4:4, 4:2:2, 4:2:0, 4:1:1, 4:4:0), greyscale and CMYK,
standard, optimised and custom quantisation/Huffman tables, restart intervals,
and sizes that are not multiples of the MCU. Width, height, pixel format and
every pixel byte must agree with the reference; progressive, truncated and
corrupted files must fail, or decode to the same pixels, in both. The committed
fixture tests/golden/jpeg_ref.npz (made by tests/golden/make_jpeg_golden.py from
the reference decoder) pins the pixels where the reference library is absent.
"""
import ctypes as C
import io
import os

import numpy as np
import pytest

import pdefa_b200 as pb
from pdefa_b200 import _native as N

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_LIB = os.path.join(ROOT, "oracle", "_ref", "libpdefa_ref.so")
GOLDEN = os.path.join(ROOT, "tests", "golden", "jpeg_ref.npz")
# the reference checkout (PDEFA_REFERENCE) holds its own JPEG fixture
REF_FIXTURE = os.path.join(os.environ.get("PDEFA_REFERENCE", ""), "pdefa", "tests", "data", "cat.jpg")

PIL = pytest.importorskip("PIL.Image")
cv2 = pytest.importorskip("cv2")


def _ref_lib():
    if not os.path.exists(REF_LIB):
        pytest.skip("reference library not built (oracle/ref.mk)")
    L = C.CDLL(REF_LIB)
    L.pdefa_image_load.restype = C.c_void_p
    L.pdefa_image_load.argtypes = [C.c_char_p]
    for f in ("pdefa_image_width", "pdefa_image_height", "pdefa_image_format"):
        getattr(L, f).argtypes = [C.c_void_p]
        getattr(L, f).restype = C.c_int32
    L.pdefa_image_pixels.argtypes = [C.c_void_p, C.POINTER(C.c_size_t)]
    L.pdefa_image_pixels.restype = C.c_void_p
    L.pdefa_image_free.argtypes = [C.c_void_p]
    return L


def _decode(L, path):
    """(width, height, format, pixel bytes) from a pdefa_image_load ABI, or None."""
    img = L.pdefa_image_load(path.encode())
    if not img:
        return None
    n = C.c_size_t()
    ptr = L.pdefa_image_pixels(img, C.byref(n))
    out = (L.pdefa_image_width(img), L.pdefa_image_height(img), L.pdefa_image_format(img),
           C.string_at(ptr, n.value))
    L.pdefa_image_free(img)
    return out


def _ours(path):
    return _decode(N.lib(), path)


def _content(rng, h, w, ch):
    """Smooth gradients + texture + flat patches (DC-only blocks) + noise."""
    y, x = np.mgrid[0:h, 0:w].astype(np.float32)
    base = []
    for c in range(ch):
        fx, fy, ph = rng.uniform(0.02, 0.4), rng.uniform(0.02, 0.4), rng.uniform(0, 6.3)
        base.append(128 + 90 * np.sin(fx * x + ph) * np.cos(fy * y - ph))
    a = np.stack(base, -1)
    a += rng.normal(0, 12, a.shape)
    if h >= 16 and w >= 16:
        a[: h // 2, : w // 2] = rng.integers(0, 256, ch)
    return np.clip(a, 0, 255).astype(np.uint8)


def _pil(rng, h, w, mode="RGB", **kw):
    ch = {"RGB": 3, "L": 1, "CMYK": 4}[mode]
    a = _content(rng, h, w, ch)
    b = io.BytesIO()
    PIL.fromarray(a[..., 0] if ch == 1 else a, mode=mode).save(b, "JPEG", **kw)
    return b.getvalue()


def _cv(rng, h, w, gray=False, **params):
    a = _content(rng, h, w, 1 if gray else 3)
    flags = []
    for k, v in params.items():
        flags += [getattr(cv2, k), v]
    ok, buf = cv2.imencode(".jpg", a[..., 0] if gray else a, flags)
    assert ok
    return buf.tobytes()


SIZES = [(1, 1), (8, 8), (16, 16), (7, 13), (29, 37), (64, 64), (75, 100), (3, 257), (120, 33)]


def _cases():
    cs = []
    for i, (h, w) in enumerate(SIZES):
        for sub in (0, 1, 2):
            cs.append((f"pil_s{sub}_{h}x{w}", "pil", dict(h=h, w=w, subsampling=sub, quality=(95, 75, 30)[i % 3])))
        cs.append((f"pil_gray_{h}x{w}", "pil", dict(h=h, w=w, mode="L", quality=90)))
    cs += [
        ("pil_q100", "pil", dict(h=40, w=56, quality=100, subsampling=0)),
        ("pil_q5", "pil", dict(h=40, w=56, quality=5, subsampling=2)),
        ("pil_optimize", "pil", dict(h=48, w=72, quality=85, optimize=True)),
        ("pil_rst_blocks1", "pil", dict(h=33, w=47, quality=80, restart_marker_blocks=1)),
        ("pil_rst_blocks5", "pil", dict(h=64, w=90, quality=80, restart_marker_blocks=5, subsampling=2)),
        ("pil_rst_rows", "pil", dict(h=70, w=50, quality=70, restart_marker_rows=1, subsampling=1)),
        ("pil_rst_gray", "pil", dict(h=40, w=40, mode="L", quality=70, restart_marker_blocks=2)),
        ("pil_cmyk", "pil", dict(h=24, w=40, mode="CMYK", quality=90)),
        ("pil_qtables", "pil", dict(h=32, w=48, subsampling=0,
                                    qtables=[[1 + (i * 7) % 50 for i in range(64)],
                                             [2 + (i * 11) % 90 for i in range(64)]])),
        ("cv_411", "cv", dict(h=40, w=70, IMWRITE_JPEG_SAMPLING_FACTOR=cv2.IMWRITE_JPEG_SAMPLING_FACTOR_411)),
        ("cv_440", "cv", dict(h=50, w=30, IMWRITE_JPEG_SAMPLING_FACTOR=cv2.IMWRITE_JPEG_SAMPLING_FACTOR_440)),
        ("cv_420_rst", "cv", dict(h=77, w=91, IMWRITE_JPEG_RST_INTERVAL=3,
                                  IMWRITE_JPEG_SAMPLING_FACTOR=cv2.IMWRITE_JPEG_SAMPLING_FACTOR_420)),
        ("cv_opt_gray", "cv", dict(h=45, w=61, gray=True, IMWRITE_JPEG_OPTIMIZE=1, IMWRITE_JPEG_QUALITY=60)),
        ("cv_luma_chroma", "cv", dict(h=36, w=36, IMWRITE_JPEG_LUMA_QUALITY=90, IMWRITE_JPEG_CHROMA_QUALITY=20)),
    ]
    return cs


CASES = _cases()


def _encode(kind, kw, seed):
    rng = np.random.default_rng(seed)
    kw = dict(kw)
    h, w = kw.pop("h"), kw.pop("w")
    return _pil(rng, h, w, **kw) if kind == "pil" else _cv(rng, h, w, **kw)


@pytest.mark.parametrize("k", range(len(CASES)), ids=[c[0] for c in CASES])
def test_jpeg_matches_reference_decoder(tmp_path, k):
    L = _ref_lib()
    name, kind, kw = CASES[k]
    p = str(tmp_path / f"{name}.jpg")
    with open(p, "wb") as f:
        f.write(_encode(kind, kw, 500 + k))
    ref = _decode(L, p)
    assert ref is not None, name
    got = _ours(p)
    assert got is not None, N.lib().pdefa_last_error()
    assert got[:3] == ref[:3]
    assert got[3] == ref[3], f"{name}: {sum(a != b for a, b in zip(got[3], ref[3]))} bytes differ"


def test_jpeg_golden_fixture(tmp_path):
    z = np.load(GOLDEN)
    for name in z["names"]:
        p = str(tmp_path / f"{name}.jpg")
        with open(p, "wb") as f:
            f.write(z[f"{name}.jpg"].tobytes())
        got = _ours(p)
        assert got is not None, (name, N.lib().pdefa_last_error())
        w, h, fmt = (int(v) for v in z[f"{name}.whf"])
        assert got[:3] == (w, h, fmt)
        assert got[3] == z[f"{name}.rgb"].tobytes(), name


def test_jpeg_reference_fixture_file():
    if not os.path.exists(REF_FIXTURE):
        pytest.skip("reference test data not present")
    L = _ref_lib()
    ref = _decode(L, REF_FIXTURE)
    got = _ours(REF_FIXTURE)
    assert ref is not None and got is not None
    assert got[:3] == ref[:3] and got[3] == ref[3]


def test_jpeg_known_pixels(tmp_path):
    """A flat 16x16 grey JPEG decodes to one value within JPEG rounding, as RGB8."""
    b = io.BytesIO()
    PIL.fromarray(np.full((16, 16), 77, np.uint8), mode="L").save(b, "JPEG", quality=95)
    p = str(tmp_path / "g.jpg")
    open(p, "wb").write(b.getvalue())
    img = pb.load_image(p)
    assert (img.width, img.height, img.channels, img.format) == (16, 16, 3, 1)
    a = img.to_numpy()
    assert a.shape == (16, 16, 3) and np.all(np.abs(a.astype(int) - 77) <= 1)
    assert np.all(a == a[0, 0])


def _both(L, p):
    return _decode(L, p), _ours(p)


def test_jpeg_truncated_and_corrupted_files(tmp_path):
    """Cut files and flipped entropy-coded bytes: same pixels, or both fail."""
    L = _ref_lib()
    rng = np.random.default_rng(7)
    data = _encode("pil", dict(h=48, w=64, quality=80, subsampling=2, restart_marker_blocks=4), 11)
    sos = data.find(b"\xff\xda")
    start = sos + 2 + int.from_bytes(data[sos + 2:sos + 4], "big")
    cuts = [len(data) - 2, len(data) - 50, start + 10, start + 1, start, sos + 3, 300, 100, 3, 2]
    variants = [data[:c] for c in cuts if c > 0]
    for _ in range(40):
        d = bytearray(data)
        for _ in range(int(rng.integers(1, 6))):
            i = int(rng.integers(start, len(data) - 2))
            d[i] = int(rng.integers(0, 256))
        variants.append(bytes(d))
    for i, v in enumerate(variants):
        p = str(tmp_path / f"v{i}.jpg")
        open(p, "wb").write(v)
        ref, got = _both(L, p)
        assert (ref is None) == (got is None), (i, N.lib().pdefa_last_error())
        if ref is not None:
            assert got == ref, i


def test_jpeg_unsupported_forms_fail(tmp_path):
    L = _ref_lib()
    good = _encode("pil", dict(h=24, w=24, quality=80), 3)
    prog = _encode("pil", dict(h=24, w=24, quality=80, progressive=True), 3)
    sof0 = good.find(b"\xff\xc0")
    twelve = bytearray(good)
    twelve[sof0 + 4] = 12                                   # 12-bit precision
    dqt = good.find(b"\xff\xdb")
    q16 = bytearray(good)
    q16[dqt + 4] = 0x10                                     # 16-bit DQT entries
    no_sos = good[: good.find(b"\xff\xda")] + b"\xff\xd9"
    no_soi = b"\xff\xd9\xff" + good[3:]
    sof1 = bytearray(good)
    sof1[sof0 + 1] = 0xC1                                   # extended sequential: skipped -> no SOF0
    for i, v in enumerate([prog, bytes(twelve), bytes(q16), no_sos, no_soi, bytes(sof1), good[:3]]):
        p = str(tmp_path / f"u{i}.jpg")
        open(p, "wb").write(v)
        ref, got = _both(L, p)
        assert ref is None and got is None, i
        assert N.lib().pdefa_last_error()


def test_jpeg_through_prepare_for_engine_path(tmp_path):
    """load_image -> the host letterbox geometry the reference computes for it."""
    data = _encode("pil", dict(h=30, w=50, quality=90), 5)
    p = str(tmp_path / "a.jpg")
    open(p, "wb").write(data)
    img = pb.load_image(p)
    assert (img.width, img.height) == (50, 30)
    meta = pb.letterbox_meta(img.width, img.height, 64, 64)
    assert (meta.orig_w, meta.orig_h, meta.scaled_w) == (50, 30, 64)
