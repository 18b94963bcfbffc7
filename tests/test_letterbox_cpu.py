"""Letterbox preprocess oracle (oracle/letterbox_ref.c) against the reference.

The restatement must equal, bit for bit, the outputs of the reference library built
from its sources (imageloader/src/preprocess.cpp:15-147 through the pdefa C API),
kept as golden fixtures in tests/golden/letterbox_ref.npz, and, when that library is
built here, fresh random cases run through it.
"""
import os

import numpy as np
import pytest

from oracle import letterbox_ref

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "letterbox_ref.npz")


def _cases():
    d = np.load(GOLDEN)
    for i in range(int(d["n_cases"])):
        tw, th, scale, pad = d[f"c{i}_cfg"]
        yield i, d[f"c{i}_img"], int(tw), int(th), float(scale), float(pad), d[f"c{i}_out"], d[f"c{i}_meta"], \
            d[f"c{i}_ratio"]


@pytest.mark.parametrize("case", list(range(10)))
def test_oracle_matches_reference_golden(case):
    i, img, tw, th, scale, pad, out, meta, ratio = list(_cases())[case]
    got, m = letterbox_ref.letterbox(img, tw, th, scale, pad)
    np.testing.assert_array_equal(got, out)
    assert [m[k] for k in ("target_w", "target_h", "orig_w", "orig_h", "pad_x", "pad_y", "scaled_w", "scaled_h")] \
        == meta.tolist()
    assert np.float32(m["ratio"]) == ratio


def test_oracle_rejects_bad_input():
    with pytest.raises(ValueError):
        letterbox_ref.letterbox(np.zeros((4, 4, 2), np.uint8), 8, 8)
    with pytest.raises(ValueError):
        letterbox_ref.letterbox(np.zeros((4, 4, 3), np.uint8), 0, 8)


def test_oracle_matches_live_reference():
    """More random sizes through the compiled reference, when it is built here."""
    ref_lib = os.path.join(os.path.dirname(os.path.dirname(__file__)), "oracle", "_ref", "libpdefa_ref.so")
    if not os.path.exists(ref_lib):
        pytest.skip("reference library not built")
    import tempfile

    from tests.golden import make_letterbox_golden as g
    import ctypes as C
    L = C.CDLL(ref_lib)
    L.pdefa_image_load.restype = C.c_void_p
    L.pdefa_image_load.argtypes = [C.c_char_p]
    L.pdefa_image_free.argtypes = [C.c_void_p]
    L.pdefa_preprocess_letterbox.argtypes = [C.c_void_p, C.POINTER(g.Cfg), C.POINTER(C.c_void_p), C.POINTER(g.Meta)]
    L.engine_tensor_data.argtypes = [C.c_void_p, C.POINTER(C.c_void_p), C.POINTER(C.c_size_t)]
    L.engine_tensor_destroy.argtypes = [C.c_void_p]
    L.pdefa_last_error.restype = C.c_char_p
    rng = np.random.default_rng(77)
    with tempfile.TemporaryDirectory() as tmp:
        for k in range(12):
            h, w = int(rng.integers(1, 300)), int(rng.integers(1, 300))
            ch = int(rng.choice([1, 3, 4]))
            tw, th = int(rng.integers(8, 160)), int(rng.integers(8, 160))
            img = rng.integers(0, 256, (h, w) if ch == 1 else (h, w, ch), dtype=np.uint8)
            png = os.path.join(tmp, f"r{k}.png")
            g.write_png(png, img)
            out, meta, ratio = g.reference_letterbox(L, png, tw, th, 1 / 255, 114 / 255)
            got, m = letterbox_ref.letterbox(img, tw, th, 1 / 255, 114 / 255)
            np.testing.assert_array_equal(got, out, err_msg=f"{(h, w, ch, tw, th)}")
            assert m["pad_x"] == meta[4] and m["pad_y"] == meta[5] and m["scaled_w"] == meta[6]
