"""YOLO11 graphs (C3k2, C2PSA attention, depthwise class branches) on the GPU
against the reference engine: golden outputs (tests/golden/make_yolo11_golden.py)
and the reference engine itself (oracle/_ref) run on this host.

The attention block exercises the head-batched 4-D x 4-D MatMul
(session_ops_nn.inc:68-108), the NCHW-order 4-D Reshape, the Split-as-Slice on
axis 2, Transpose(0,1,3,2), Mul by a scalar and Softmax with the reference's
axis remapping. Tolerances as in test_gpu_parity: strict FP32 <= 1e-5, TF32/BF16
<= 1e-2 (normwise).
"""
import numpy as np
import pytest

import pdefa_b200 as pb
from conftest import normwise
from oracle import ref_engine as R
from pdefa_b200.engine_file import write_engine
from pdefa_b200.yolo import build_c2psa, build_yolo11
from test_gpu_parity import PRECS, TOL, run_engine

pytestmark = pytest.mark.gpu


def _engine(engine_dir, name, g):
    p = str(engine_dir / name)
    write_engine(p, g)
    return p


def _x(seed, shape):
    return np.random.default_rng(seed).random(shape, dtype=np.float32)


@pytest.mark.parametrize("prec", PRECS)
def test_c2psa_golden(golden, engine_dir, prec):
    d = golden("c2psa_12.npz")
    p = _engine(engine_dir, "c2psa_12.engine", build_c2psa(c=128, hw=12, seed=0)[0])
    y = run_engine(p, _x(int(d["seed"]), (1, 128, 12, 12)), prec)
    assert y.shape == d["y"].shape == (1, 128, 12, 12)
    assert normwise(y, d["y"]) <= TOL[prec]


@pytest.mark.parametrize("prec", PRECS)
def test_c2psa_p5_size_against_reference_engine(engine_dir, prec):
    """The C2PSA block at YOLO11n-640's P5 size: 400 tokens, 2 heads, key 32, value 64."""
    if not R.available():
        pytest.skip("reference engine not built on this host")
    p = _engine(engine_dir, "c2psa_20.engine", build_c2psa(c=128, hw=20, seed=3)[0])
    x = _x(5, (1, 128, 20, 20))
    ref = R.RefSession(p).run(x)
    y = run_engine(p, x, prec)
    assert normwise(y, ref) <= TOL[prec]


@pytest.mark.parametrize("prec", PRECS)
def test_yolo11n_96_golden(golden, engine_dir, prec):
    d = golden("yolo11n_96.npz")
    p = _engine(engine_dir, "y11n_96.engine", build_yolo11("n", imgsz=96, seed=0)[0])
    y = run_engine(p, _x(int(d["seed"]), (1, 3, 96, 96)), prec)
    assert y.shape == d["y"].shape == (1, 84, 189)
    assert normwise(y, d["y"]) <= TOL[prec]
    assert np.abs(y[0, 4:] - d["y"][0, 4:]).max() <= (5e-6 if prec == pb.FP32 else 2e-2)


@pytest.mark.parametrize("prec", PRECS)
def test_yolo11n_640_against_reference_engine(engine_dir, prec):
    if not R.available():
        pytest.skip("reference engine not built on this host")
    p = _engine(engine_dir, "y11n_640.engine", build_yolo11("n", imgsz=640, seed=0)[0])
    x = _x(1, (1, 3, 640, 640))
    ref = R.RefSession(p).run(x)
    y = run_engine(p, x, prec)
    assert y.shape == (1, 84, 8400)
    assert normwise(y, ref) <= TOL[prec]


@pytest.mark.parametrize("prec", [pb.FP32, pb.BF16])
def test_yolo11n_batch_equals_per_image(engine_dir, prec):
    p = _engine(engine_dir, "y11n_128.engine", build_yolo11("n", imgsz=128, seed=0)[0])
    x = _x(3, (3, 3, 128, 128))
    yb = run_engine(p, x, prec)
    for i in range(3):
        yi = run_engine(p, x[i:i + 1], prec)
        if prec == pb.FP32:
            np.testing.assert_array_equal(yb[i], yi[0])
        else:
            assert normwise(yb[i], yi[0]) <= 1e-6


def test_yolo11n_batch_inference_detect(engine_dir):
    """The batch runner (CUDA graphs, GPU decode) on a YOLO11n engine gives the
    detections of decode_yolo on the session output of the same batch."""
    p = _engine(engine_dir, "y11n_160.engine", build_yolo11("n", imgsz=160, seed=0)[0])
    ctx = pb.Context(precision=pb.BF16)
    m = pb.Model(ctx, p)
    x = _x(7, (4, 3, 160, 160))
    with pb.BatchInference(ctx, m, batch_size=4, devices=[0]) as bi:
        dets = bi.detect(x, conf_thres=0.25, iou_thres=0.45)
    y = run_engine(p, x, pb.BF16)
    for i in range(4):
        ref = pb.decode_yolo(y[i:i + 1], conf_thres=0.25, iou_thres=0.45)
        assert len(dets[i]) == len(ref) > 0
        for a, b in zip(dets[i], ref):
            assert a["cls"] == b["cls"]
            np.testing.assert_allclose([a[k] for k in ("x1", "y1", "x2", "y2", "conf")],
                                       [b[k] for k in ("x1", "y1", "x2", "y2", "conf")], rtol=1e-6, atol=1e-4)


@pytest.mark.parametrize("prec", [pb.TF32, pb.BF16])
def test_yolo11n_channel_padding_and_folds_keep_results(engine_dir, prec):
    """Padding the 8-channel convs to 16 for tcgen05 changes only the accumulation
    blocking: the outputs stay within the tensor-core tolerance of the unpadded plan."""
    p = _engine(engine_dir, "y11n_128p.engine", build_yolo11("n", imgsz=128, seed=0)[0])
    x = _x(4, (2, 3, 128, 128))
    padded = run_engine(p, x, prec)
    plain = run_engine(p, x, prec, env={"PDEFA_NO_CHANNEL_PAD": "1"})
    assert normwise(padded, plain) <= 5e-3
