"""The CPU oracle is pinned against the reference's own outputs (golden fixtures
made by tests/golden/make_golden.py from the compiled reference engine and the
reference's Python decode_yolo)."""
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN, normwise
from oracle import decode_ref, onnx_numpy
from pdefa_b200.yolo import build_single_conv, build_yolov8


def _cases():
    with open(os.path.join(GOLDEN, "decode_expected.json")) as f:
        return json.load(f)


@pytest.mark.parametrize("case", _cases(), ids=lambda c: c["name"])
def test_decode_restatement_matches_reference_python(case, golden):
    preds = golden("decode_inputs.npz")[case["input"]]
    got = decode_ref.decode(preds, case["meta"], case["conf"], case["iou"], case["max_det"])
    exp = case["dets"]
    assert len(got) == len(exp)
    for g, e in zip(got, exp):
        for k in ("x1", "y1", "x2", "y2", "conf"):
            assert g[k] == e[k], (k, g, e)          # bit-exact float64
        assert g["cls"] == e["cls"]


def test_numpy_yolov8_matches_reference_engine(golden):
    d = golden("yolov8n_128.npz")
    g, _ = build_yolov8("n", imgsz=128, seed=0)
    y = onnx_numpy.run(g, [d["x"]])[0]
    assert y.shape == d["y"].shape
    assert normwise(y, d["y"]) < 1e-5


def test_numpy_yolov8_without_reference_silu_flavour_differs(golden):
    """The reference's Winograd path evaluates SiLU with its own polynomial; exact
    SiLU alone does not reproduce the reference (documents why the flavour exists)."""
    d = golden("yolov8n_128.npz")
    g, _ = build_yolov8("n", imgsz=128, seed=0)
    y = onnx_numpy.run(g, [d["x"]], reference_silu=False)[0]
    assert normwise(y, d["y"]) > 1e-4


def test_numpy_stem_matches_reference_engine(golden):
    d = golden("stem_64.npz")
    g, _ = build_single_conv(cin=3, cout=16, k=3, s=2, hw=64, seed=1)
    y = onnx_numpy.run(g, [d["x"]])[0]
    assert normwise(y, d["y"]) < 1e-6


def test_matmul_golden_against_fp64(golden):
    d = golden("matmul_96x80x64.npz")
    ref = d["a"].astype(np.float64) @ d["b"].astype(np.float64)
    assert normwise(d["c"], ref) < 1e-6


def test_silu_winograd_flavour_is_not_exact_silu():
    x = np.linspace(-8, 8, 2001, dtype=np.float32)
    exact = x / (1 + np.exp(-x.astype(np.float64)))
    flav = onnx_numpy.silu_winograd_flavor(x)
    err = np.abs(flav - exact).max()
    assert 1e-3 < err < 0.2
    # integral log2 points (f == 0) are exact up to float rounding
    xi = np.array([0.0, -np.log(2) * 3], dtype=np.float32)
    np.testing.assert_allclose(onnx_numpy.silu_winograd_flavor(xi), xi / (1 + np.exp(-xi)), rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("cin,cout,k,s,groups,hw", [(16, 16, 3, 1, 16, 12), (32, 64, 3, 2, 4, 13),
                                                    (24, 24, 5, 2, 24, 11)])
def test_numpy_grouped_conv_matches_reference_engine(tmp_path, cin, cout, k, s, groups, hw):
    """Grouped and depthwise convs (conv2d.cpp:164-393) in the numpy restatement agree
    with the compiled reference engine, when it is built on this host."""
    from oracle import ref_engine as R
    from pdefa_b200.engine_file import write_engine
    if not R.available():
        pytest.skip("reference engine not built on this host")
    g, _ = build_single_conv(cin=cin, cout=cout, k=k, s=s, hw=hw, seed=4, groups=groups)
    p = str(tmp_path / "grouped.engine")
    write_engine(p, g)
    x = np.random.default_rng(1).random((1, cin, hw, hw), dtype=np.float32) - 0.5
    ref = R.RefSession(p).run(x)
    y = onnx_numpy.run(g, [x])[0]
    assert normwise(y, ref) <= 1e-6


def test_yolo11_graphs_flops_and_reference_engine(tmp_path):
    """YOLO11 builders: conv FLOPs equal the published 6.5 / 21.5 / 68.0 / 86.9 GFLOPs
    (n/s/m/l at 640), and the reference engine runs the C2PSA attention graph."""
    from oracle import ref_engine as R
    from pdefa_b200.engine_file import write_engine
    from pdefa_b200.yolo import build_c2psa, build_yolo11, conv_flops
    for sc, gf in (("n", 6.5), ("s", 21.5), ("m", 68.0), ("l", 86.9)):
        _, info = build_yolo11(sc, imgsz=640)
        assert abs(conv_flops(info) / 1e9 - gf) < 0.06, sc
    if not R.available():
        pytest.skip("reference engine not built on this host")
    g, _ = build_c2psa(c=128, hw=8, seed=1)
    p = str(tmp_path / "c2psa.engine")
    write_engine(p, g)
    y = R.RefSession(p).run(np.random.default_rng(0).random((1, 128, 8, 8), dtype=np.float32))
    assert y.shape == (1, 128, 8, 8) and np.isfinite(y).all()
