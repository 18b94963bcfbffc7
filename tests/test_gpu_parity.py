"""GPU parity tests through the C ABI (libpdefa_native.so via the Python mirror).

Tolerances (normwise max|y - ref| / max|ref|): strict FP32 path <= 1e-5, TF32/BF16
tensor-core paths <= 1e-2. Decode/NMS: exact equality of kept boxes (float64),
confidences and classes. References: golden fixtures made from the reference
engine, and the reference engine itself (oracle/_ref) run on this host for the
full-size configurations.
"""
import json
import os

import numpy as np
import pytest

import pdefa_b200 as pb
from conftest import GOLDEN, normwise
from oracle import ref_engine as R
from pdefa_b200.engine_file import write_engine
from pdefa_b200.yolo import build_single_conv, build_yolov8

pytestmark = pytest.mark.gpu

TOL = {pb.FP32: 1e-5, pb.TF32: 1e-2, pb.BF16: 1e-2}
PRECS = [pb.FP32, pb.TF32, pb.BF16]


def run_engine(path, x, precision, env=None):
    old = {}
    for k, v in (env or {}).items():
        old[k] = os.environ.get(k)
        os.environ[k] = v
    try:
        ctx = pb.Context(precision=precision)
        m = pb.Model(ctx, path)
        s = pb.Session(ctx, m)
        s.set_input(0, pb.Tensor.from_numpy(x))
        s.run()
        return s.output(0).to_numpy()
    finally:
        for k, v in old.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v


@pytest.fixture(scope="module")
def y8n_128(engine_dir):
    g, _ = build_yolov8("n", imgsz=128, seed=0)
    p = str(engine_dir / "y8n_128.engine")
    write_engine(p, g)
    return p


@pytest.fixture(scope="module")
def y8n_640(engine_dir):
    g, _ = build_yolov8("n", imgsz=640, seed=0)
    p = str(engine_dir / "y8n_640.engine")
    write_engine(p, g)
    return p


# ---------------------------------------------------------------- matmul (cfg1)
@pytest.mark.parametrize("prec", PRECS)
def test_matmul_golden(golden, prec):
    d = golden("matmul_96x80x64.npz")
    a, b = pb.Tensor.from_numpy(d["a"]), pb.Tensor.from_numpy(d["b"])
    c = pb.ops_matmul(a, b, precision=prec).to_numpy()
    assert normwise(c, d["c"]) <= TOL[prec]


@pytest.mark.parametrize("prec", PRECS)
def test_matmul_cfg1_512(prec):
    rng = np.random.default_rng(42)
    A = rng.standard_normal((512, 512)).astype(np.float32)
    B = rng.standard_normal((512, 512)).astype(np.float32)
    ref = R.matmul(A, B) if R.available() else (A.astype(np.float64) @ B)
    c = pb.ops_matmul(pb.Tensor.from_numpy(A), pb.Tensor.from_numpy(B), precision=prec).to_numpy()
    assert normwise(c, ref) <= TOL[prec]


def test_matmul_default_is_strict_and_shape_mismatch_is_noop():
    a = pb.Tensor.from_numpy(np.ones((3, 5), np.float32))
    b = pb.Tensor.from_numpy(np.ones((4, 2), np.float32))
    out = pb.tensor_empty([3, 2]).fill(7.0)
    pb.api._check(pb._native.lib().engine_ops_matmul(a.raw, b.raw, out.raw))   # ops/matmul.cpp: silent no-op
    assert (out.to_numpy() == 7.0).all()
    m = (np.arange(12, dtype=np.float32).reshape(3, 4) - 5) / 3
    e = np.eye(4, dtype=np.float32)
    np.testing.assert_array_equal((pb.Tensor.from_numpy(m) @ pb.Tensor.from_numpy(e)).to_numpy(), m)


# ---------------------------------------------------------------- stem conv (cfg2)
@pytest.mark.parametrize("prec", PRECS)
def test_stem_golden(golden, engine_dir, prec):
    d = golden("stem_64.npz")
    g, _ = build_single_conv(cin=3, cout=16, k=3, s=2, hw=64, seed=1)
    p = str(engine_dir / "stem64.engine")
    write_engine(p, g)
    y = run_engine(p, d["x"], prec)
    assert y.shape == d["y"].shape
    assert normwise(y, d["y"]) <= TOL[prec]


@pytest.mark.parametrize("prec", [pb.FP32, pb.BF16])
def test_stem_cfg2_640(engine_dir, prec):
    g, _ = build_single_conv(cin=3, cout=16, k=3, s=2, hw=640, seed=1)
    p = str(engine_dir / "stem640.engine")
    write_engine(p, g)
    x = np.random.default_rng(0).random((1, 3, 640, 640), dtype=np.float32)
    y = run_engine(p, x, prec)
    if not R.available():
        pytest.skip("reference engine not built on this host")
    ref = R.RefSession(p).run(x)
    assert normwise(y, ref) <= TOL[prec]


@pytest.mark.parametrize("prec", [pb.FP32, pb.BF16])
@pytest.mark.parametrize("cout,hw,s", [(16, 37, 2), (32, 53, 2), (48, 33, 1), (16, 20, 1)])
def test_stem_rows_kernel_batched(engine_dir, prec, cout, hw, s):
    """Cin=3 convs on the fp32 NCHW input (row-tiled direct kernel in FP32, tcgen05 stem
    kernel in BF16): odd sizes, batch 3, each Cout tile width, against the fp64 oracle."""
    from oracle import onnx_numpy
    g, _ = build_single_conv(cin=3, cout=cout, k=3, s=s, hw=hw, seed=4)
    p = str(engine_dir / f"stem_rows_{cout}_{hw}_{s}.engine")
    write_engine(p, g)
    first = [kd for kd, _ in pb.Model(pb.Context(), p).plan_summary(prec, 3)][0]
    assert first == ("conv_stem_tc" if prec == pb.BF16 else "conv_direct")
    x = np.random.default_rng(6).random((3, 3, hw, hw), dtype=np.float32)
    y = run_engine(p, x, prec)
    ref = onnx_numpy.run(g, [x])[0]
    assert y.shape == ref.shape
    assert normwise(y, ref) <= TOL[prec]


# ------------------------------------------------- tensor-core conv on a staged graph input
@pytest.mark.parametrize("prec", [pb.TF32, pb.BF16])
@pytest.mark.parametrize("cin,cout,k,s,hw", [(64, 64, 3, 1, 20), (16, 48, 3, 2, 33), (80, 80, 1, 1, 12),
                                             (80, 80, 3, 1, 20), (48, 32, 1, 1, 24), (80, 64, 3, 2, 21),
                                             (112, 32, 3, 1, 9), (16, 16, 3, 1, 40), (32, 32, 3, 1, 37),
                                             (16, 32, 3, 1, 61), (144, 48, 3, 1, 13), (144, 32, 1, 1, 19)])
def test_single_conv_staged_input(engine_dir, prec, cin, cout, k, s, hw):
    """A conv fed directly by the fp32 NCHW graph input: the plan stages the input into
    the operand layout and runs the tensor-core kernel (no SIMT fallback). In BF16,
    multi-tap convs with Cin = 80 and 144 run as full 64-channel chunks plus a 16-channel
    tail chunk (own 32-byte-swizzle maps); 1x1 convs with those Cin and Cin = 48 and 112
    run as zero-padded 64-channel chunks; the 16- and 32-channel
    3x3 cases run in window mode (zero-padded row windows, taps as shifted windows)
    at sizes whose last tile is partial.

    The 3x3 stride-1 case takes the reference's Winograd SiLU, which jumps by up to
    ~0.04 where round(-x*log2 e) changes; a BF16/TF32 pre-activation on the other
    side of a jump is still a correct result. So each output is compared with the
    activation evaluated anywhere within +-1e-2 * max|z| of the exact fp64
    pre-activation z, and the smallest difference must stay within the tolerance.
    """
    from oracle import onnx_numpy
    g, _ = build_single_conv(cin=cin, cout=cout, k=k, s=s, hw=hw, seed=3)
    p = str(engine_dir / f"single_{cin}_{cout}_{k}_{s}_{hw}.engine")
    write_engine(p, g)
    kinds = [kd for kd, _ in pb.Model(pb.Context(), p).plan_summary(prec, 2)]
    assert kinds[:2] == ["copy", "conv_tc_bf16" if prec == pb.BF16 else "conv_tc_tf32"]
    x = np.random.default_rng(5).random((2, cin, hw, hw), dtype=np.float32) - 0.5
    y = run_engine(p, x, prec).astype(np.float64)
    ref = onnx_numpy.run(g, [x])[0]
    assert y.shape == ref.shape
    conv = g.nodes[0]
    z = onnx_numpy.conv2d_nchw(x.astype(np.float64), g.weight(conv.inputs[1]).astype(np.float64),
                               g.weight(conv.inputs[2]).astype(np.float64), (s, s), (k // 2, k // 2))
    wino = onnx_numpy.ref_conv_path(cin, k, k, s, s, k // 2, k // 2, 1, 1, 1) == "winograd"
    act = onnx_numpy.silu_winograd_flavor if wino else (lambda v: v / (1.0 + np.exp(-v)))
    np.testing.assert_allclose(act(z), ref, rtol=0, atol=1e-12)
    eps = TOL[prec] * np.abs(z).max()
    best = np.full(y.shape, np.inf)
    for t in np.linspace(-1.0, 1.0, 81):
        best = np.minimum(best, np.abs(y - act(z + t * eps)))
    assert best.max() / np.abs(ref).max() <= TOL[prec]
    if not wino:
        assert normwise(y, ref) <= TOL[prec]


def check_head(y, ref, prec, ref64=None):
    """[B, 4+nc, A] head outputs, channel groups checked apart: the box channels
    (pixels, up to the image size) normwise over the boxes, the class scores (in [0, 1])
    absolutely, so loose boxes cannot hide behind the scores or the other way round.
    BF16/TF32: both against the compiled reference at 1e-2. FP32: boxes against it at
    1e-5; the scores at 1e-5 against ref64, the float64 restatement of the same graph
    semantics (oracle/onnx_numpy.py), and at 1e-2 against the compiled reference, whose
    Winograd SiLU flavour is discontinuous at the points where its rounded exponent
    changes: its own float rounding puts single activations on the other side of such a
    jump (on YOLOv8n-640 seed 1: one 3x3 block of anchors, 1.7e-3 on one score, while
    the boxes agree to 2e-7)."""
    tol = TOL[prec]
    bx, rb = y[..., :4, :], ref[..., :4, :]
    assert normwise(bx, rb) <= tol, ("boxes", normwise(bx, rb))
    err = float(np.abs(y[..., 4:, :] - ref[..., 4:, :]).max())
    assert err <= max(tol, 1e-2), ("class scores", err)
    if ref64 is not None:
        err64 = float(np.abs(y[..., 4:, :] - ref64[..., 4:, :]).max())
        assert err64 <= tol, ("class scores vs float64", err64)


# ---------------------------------------------------------------- YOLOv8n (cfg3/cfg4 numerics)
@pytest.mark.parametrize("prec", PRECS)
def test_yolov8n_128_golden(golden, y8n_128, prec):
    d = golden("yolov8n_128.npz")
    y = run_engine(y8n_128, d["x"], prec)
    assert y.shape == (1, 84, 336)
    assert normwise(y, d["y"]) <= TOL[prec]
    # class scores separately (they are ~0.5 while boxes reach hundreds of pixels)
    assert np.abs(y[0, 4:] - d["y"][0, 4:]).max() <= (5e-6 if prec == pb.FP32 else 2e-2)


def test_yolov8n_128_unfused_head_and_residual_match(golden, y8n_128):
    d = golden("yolov8n_128.npz")
    y0 = run_engine(y8n_128, d["x"], pb.FP32)
    y1 = run_engine(y8n_128, d["x"], pb.FP32, env={"PDEFA_NO_HEAD_FUSION": "1", "PDEFA_NO_RESIDUAL_FUSION": "1"})
    assert normwise(y1, d["y"]) <= 1e-5
    assert normwise(y0, y1) <= 1e-6


@pytest.mark.parametrize("prec", [pb.FP32, pb.BF16])
def test_yolov8n_batch_equals_per_image(y8n_128, prec):
    rng = np.random.default_rng(3)
    x = rng.random((5, 3, 128, 128), dtype=np.float32)
    yb = run_engine(y8n_128, x, prec)
    assert yb.shape == (5, 84, 336)
    for i in range(5):
        yi = run_engine(y8n_128, x[i:i + 1], prec)
        if prec == pb.FP32:
            np.testing.assert_array_equal(yb[i], yi[0])
        else:
            assert normwise(yb[i], yi[0]) <= 1e-6


@pytest.mark.parametrize("prec", PRECS)
def test_yolov8n_640_against_reference_engine(y8n_640, prec):
    if not R.available():
        pytest.skip("reference engine not built on this host")
    x = np.random.default_rng(1).random((1, 3, 640, 640), dtype=np.float32)
    ref = R.RefSession(y8n_640).run(x)
    y = run_engine(y8n_640, x, prec)
    assert normwise(y, ref) <= TOL[prec]
    ref64 = None
    if prec == pb.FP32:
        from oracle import onnx_numpy
        g, _ = build_yolov8("n", imgsz=640, seed=0)
        ref64 = np.asarray(onnx_numpy.run(g, [x.astype(np.float64)])[0], dtype=np.float64)
    check_head(y, ref, prec, ref64)


@pytest.mark.parametrize("prec", [pb.TF32, pb.BF16])
def test_yolov8m_640_against_reference_engine(engine_dir, prec):
    """YOLOv8m (width 0.75, depth 0.67; convs up to 768 channels, K up to
    5184) on the tensor-core paths, batch 2, each image against the reference engine."""
    if not R.available():
        pytest.skip("reference engine not built on this host")
    g, _ = build_yolov8("m", imgsz=640, seed=0)
    p = str(engine_dir / "y8m_640.engine")
    write_engine(p, g)
    x = np.random.default_rng(2).random((2, 3, 640, 640), dtype=np.float32)
    y = run_engine(p, x, prec)
    sess = R.RefSession(p)
    for i in range(2):
        ref = sess.run(x[i:i + 1])[0]
        assert normwise(y[i], ref) <= TOL[prec]
        check_head(y[i], ref, prec)


def test_tiny_classifier_graph(golden, engine_dir):
    import tests.golden.make_golden as mg
    d = golden("tiny.npz")
    p = str(engine_dir / "tiny.engine")
    write_engine(p, mg.build_tiny())
    y = run_engine(p, d["x"], pb.FP32)
    assert y.shape == (1, 4)
    assert normwise(y, d["y"]) <= 1e-5


def test_input_size_other_than_declared(engine_dir):
    """The reference interpreter runs a graph on whatever image size it is given (its
    BatchInference feeds 640x640 images to a model declared at 64x64); a session here
    lowers a plan for the input's own size and matches the reference engine on it."""
    import tests.golden.make_golden as mg
    from oracle import ref_engine as R
    if not R.available():
        pytest.skip("compiled reference engine (oracle/_ref) not built")
    p = str(engine_dir / "tiny_any.engine")
    write_engine(p, mg.build_tiny())
    for h, w in ((96, 80), (64, 64), (130, 47)):
        x = np.random.default_rng(h * w).random((1, 3, h, w), dtype=np.float32)
        y = run_engine(p, x, pb.FP32)
        ref = R.RefSession(p, threads=4).run(x)
        assert y.shape == (1, 4)
        assert normwise(y, ref) <= 1e-5, (h, w)


# ---------------------------------------------------------------- decode / NMS
def _cases():
    with open(os.path.join(GOLDEN, "decode_expected.json")) as f:
        return json.load(f)


@pytest.mark.parametrize("case", _cases(), ids=lambda c: c["name"])
def test_gpu_decode_bit_exact(golden, case):
    preds = golden("decode_inputs.npz")[case["input"]]
    meta = pb.PreprocessMeta(**case["meta"]) if case["meta"] else None
    got = pb.decode_yolo(preds[None], meta, case["conf"], case["iou"], case["max_det"])
    exp = case["dets"]
    assert len(got) == len(exp)
    for g, e in zip(got, exp):
        for k in ("x1", "y1", "x2", "y2", "conf"):
            assert g[k] == e[k], (k, g, e)
        assert g["cls"] == e["cls"]


def test_gpu_decode_batched_matches_single(golden):
    d = golden("decode_inputs.npz")
    stack = np.stack([d["adversarial"], d["adversarial"][:, ::-1].copy()])
    both = pb.decode_yolo_arrays(stack, conf_thres=0.3, iou_thres=0.5, max_det=50)
    for b in range(2):
        one = pb.decode_yolo_arrays(stack[b:b + 1], conf_thres=0.3, iou_thres=0.5, max_det=50)[0]
        assert [(x.anchor, x.cls, x.x1, x.y2) for x in both[b]] == [(x.anchor, x.cls, x.x1, x.y2) for x in one]


@pytest.mark.parametrize("max_det,iou,conf", [(300, 0.45, 0.25), (1000, 0.45, 0.25), (2000, 0.7, 0.1),
                                               (5, 0.45, 0.25), (300, 0.0, 0.25)])
def test_gpu_decode_full_size_against_restatement(y8n_640, max_det, iou, conf):
    """8400 anchors, every one a candidate (random-init head): heavy same-class
    suppression, kept lists past the shared-memory mirror (max_det > 512), IoU 0."""
    from oracle import decode_ref
    x = np.random.default_rng(2).random((1, 3, 640, 640), dtype=np.float32)
    y = run_engine(y8n_640, x, pb.BF16)
    got = pb.decode_yolo(y, conf_thres=conf, iou_thres=iou, max_det=max_det)
    exp = decode_ref.decode(y[0], conf_thres=conf, iou_thres=iou, max_det=max_det)
    assert len(got) == len(exp)
    if (max_det, iou) == (300, 0.45):
        assert len(exp) == 300
    for g, e in zip(got, exp):
        assert (g["x1"], g["y1"], g["x2"], g["y2"], g["conf"], g["cls"]) == \
               (e["x1"], e["y1"], e["x2"], e["y2"], e["conf"], e["cls"])


def test_gpu_decode_iou_near_threshold():
    """Same-class box pairs whose IoU sweeps across iou_thres in steps of ~3e-8: the
    NMS decides most pairs from float bounds and must leave every close call (within
    ~1e-6 of the threshold) to the float64 test, so the kept lists equal the restated
    reference's bit for bit on both sides of the threshold."""
    from oracle import decode_ref
    P, thr = 512, 0.45
    A = 2 * P
    w = (100.0 + (np.arange(P) - P // 2) * 7.62939453125e-06).astype(np.float32)   # float32 steps near 100
    d = np.float32(37.93103)                                                      # IoU ~ (w - d) / (w + d) = 0.45
    cls = np.arange(P) % 80
    cell = np.arange(P) // 80
    cx = (60.0 + cell * 300.0).astype(np.float32)
    cy = (60.0 + (np.arange(P) % 80) * 3.0).astype(np.float32)    # classes differ, so overlap across classes is harmless
    preds = np.zeros((84, A), np.float32)
    preds[0, 0::2], preds[0, 1::2] = cx, cx + d
    preds[1, 0::2], preds[1, 1::2] = cy, cy
    preds[2, 0::2], preds[2, 1::2] = w, w
    preds[3, 0::2], preds[3, 1::2] = w, w
    preds[4 + cls, 2 * np.arange(P)] = 0.9
    preds[4 + cls, 2 * np.arange(P) + 1] = 0.8
    # the reference's float64 IoU of each pair: the sweep must straddle the threshold closely
    x1a, x2a = cx.astype(np.float64) - w * 0.5, cx.astype(np.float64) + w * 0.5
    cxb = (cx + d).astype(np.float64)
    x1b, x2b = cxb - w * 0.5, cxb + w * 0.5
    y1, y2 = cy.astype(np.float64) - w * 0.5, cy.astype(np.float64) + w * 0.5
    inter = (np.minimum(x2a, x2b) - np.maximum(x1a, x1b)) * (y2 - y1)
    area = (x2a - x1a) * (y2 - y1)
    iou = inter / (area + area - inter + 1e-9)
    assert ((iou > thr) & (iou < thr + 1e-6)).sum() >= 10 and ((iou <= thr) & (iou > thr - 1e-6)).sum() >= 10
    got = pb.decode_yolo(preds[None], None, 0.25, thr, A)
    exp = decode_ref.decode(preds, conf_thres=0.25, iou_thres=thr, max_det=A)
    assert P < len(exp) < A
    assert len(got) == len(exp)
    for g, e in zip(got, exp):
        assert (g["x1"], g["y1"], g["x2"], g["y2"], g["conf"], g["cls"]) == \
               (e["x1"], e["y1"], e["x2"], e["y2"], e["conf"], e["cls"])


# ---------------------------------------------------------------- ops
def test_elementwise_and_shape_ops():
    rng = np.random.default_rng(4)
    a = rng.standard_normal((2, 3, 4)).astype(np.float32)
    b = rng.standard_normal((3, 1)).astype(np.float32)
    A, Bt = pb.Tensor.from_numpy(a), pb.Tensor.from_numpy(b)
    np.testing.assert_allclose((A + Bt).to_numpy(), a + b, rtol=0, atol=0)
    np.testing.assert_allclose((A * Bt).to_numpy(), a * b, rtol=0, atol=0)
    np.testing.assert_allclose((A / Bt).to_numpy(), a / b, rtol=1e-7)
    t = pb.Tensor.from_numpy(a)
    pb.ops_sigmoid(t)
    np.testing.assert_allclose(t.to_numpy(), 1 / (1 + np.exp(-a.astype(np.float64))), rtol=1e-6)
    t = pb.Tensor.from_numpy(a)
    pb.ops_softmax(t, axis=1)
    e = np.exp(a - a.max(1, keepdims=True))
    np.testing.assert_allclose(t.to_numpy(), e / e.sum(1, keepdims=True), rtol=1e-6)
    np.testing.assert_allclose(pb.ops_reduce_sum(A, 2).to_numpy(), a.sum(2), rtol=1e-6)
    np.testing.assert_allclose(pb.ops_reduce_mean(A, 0, True).to_numpy(), a.mean(0, keepdims=True), rtol=1e-6)
    np.testing.assert_array_equal(pb.ops_reduce_max(A, -1).to_numpy(), a.max(-1))
    np.testing.assert_array_equal(pb.ops_argmax(A, 1).to_numpy(), a.argmax(1))
    np.testing.assert_array_equal(pb.ops_transpose(A, [2, 0, 1]).to_numpy(), a.transpose(2, 0, 1))
    np.testing.assert_array_equal(pb.ops_reshape(A, [4, -1]).to_numpy(), a.reshape(4, -1))
    np.testing.assert_array_equal(pb.ops_concat([A, A], 1).to_numpy(), np.concatenate([a, a], 1))
    np.testing.assert_array_equal(pb.ops_stack([A, A], 1).to_numpy(), np.stack([a, a], 1))
    idx = pb.Tensor.from_numpy(np.array([2, -1, 0], np.float32))
    np.testing.assert_array_equal(pb.ops_gather(A, idx, 2).to_numpy(), a[:, :, [2, 3, 0]])
    t = pb.Tensor.from_numpy(a)
    pb.ops_clip(t, -0.5, 0.5)
    np.testing.assert_array_equal(t.to_numpy(), np.clip(a, -0.5, 0.5))


# ---------------------------------------------------------------- BatchInference
def test_batch_inference_matches_session_decode(y8n_128):
    ctx = pb.Context(precision=pb.BF16)
    m = pb.Model(ctx, y8n_128)
    x = np.random.default_rng(9).random((6, 3, 128, 128), dtype=np.float32)
    with pb.BatchInference(ctx, m, batch_size=4) as bi:
        got = bi.detect(x, conf_thres=0.25, iou_thres=0.45, max_det=100)
    y = run_engine(y8n_128, x, pb.BF16)
    for i in range(6):
        exp = pb.decode_yolo(y[i], None, 0.25, 0.45, 100)
        assert got[i] == exp


def test_batch_inference_pipelined_micro_batches(y8n_128):
    """Micro-batches alternate between the runner's two pipeline lanes (copy of one
    overlapping inference of the other); results equal one single-batch pass, also
    when the runner is reused and the last micro-batch is short."""
    ctx = pb.Context(precision=pb.BF16)
    m = pb.Model(ctx, y8n_128)
    x = np.random.default_rng(11).random((7, 3, 128, 128), dtype=np.float32)
    with pb.BatchInference(ctx, m, batch_size=7, devices=[0]) as bi:
        c_ref, d_ref = bi.detect_arrays(x, conf_thres=0.2, iou_thres=0.5, max_det=50)
    assert c_ref.shape == (7,) and d_ref.shape == (7, 50)
    with pb.BatchInference(ctx, m, batch_size=2, devices=[0]) as bi:
        for _ in range(2):
            c, d = bi.detect_arrays(x, conf_thres=0.2, iou_thres=0.5, max_det=50)
            np.testing.assert_array_equal(c, c_ref)
            for b in range(7):
                np.testing.assert_array_equal(d[b, :c[b]], d_ref[b, :c_ref[b]])
        lists = bi.detect(x[:3], conf_thres=0.2, iou_thres=0.5, max_det=50)
    for b in range(3):
        assert [(e["x1"], e["y1"], e["x2"], e["y2"], e["conf"], e["cls"]) for e in lists[b]] == \
            [(r["x1"], r["y1"], r["x2"], r["y2"], float(r["conf"]), int(r["cls"])) for r in d_ref[b, :c_ref[b]]]


def test_batch_inference_shards_across_devices(y8n_128):
    """The batch split over every visible GPU (one replica and one native thread per
    device, contiguous shards, no collective) returns, image for image, what one GPU
    returns. Needs two or more GPUs."""
    n = pb.device_count()
    if n < 2:
        pytest.skip("needs two or more GPUs")
    ctx = pb.Context(precision=pb.BF16)
    m = pb.Model(ctx, y8n_128)
    x = np.random.default_rng(13).random((2 * n + 1, 3, 128, 128), dtype=np.float32)
    with pb.BatchInference(ctx, m, batch_size=2, devices=[0]) as bi:
        c_ref, d_ref = bi.detect_arrays(x, conf_thres=0.2, iou_thres=0.5, max_det=50)
    with pb.BatchInference(ctx, m, batch_size=2, devices=list(range(n))) as bi:
        c, d = bi.detect_arrays(x, conf_thres=0.2, iou_thres=0.5, max_det=50)
    np.testing.assert_array_equal(c, c_ref)
    for b in range(len(x)):
        np.testing.assert_array_equal(d[b, :c[b]], d_ref[b, :c_ref[b]])


# ------------------------------------------------------------- grouped / depthwise conv
@pytest.mark.parametrize("prec", PRECS)
@pytest.mark.parametrize("cin,cout,k,s,groups,hw", [(16, 16, 3, 1, 16, 40), (64, 64, 3, 2, 64, 33),
                                                    (32, 64, 3, 2, 4, 29), (24, 24, 5, 1, 24, 17)])
def test_grouped_conv_against_reference_engine(engine_dir, prec, cin, cout, k, s, groups, hw):
    """Depthwise and grouped convs (the reference's conv2d.cpp:164-393 paths) with the
    fused SiLU, against the compiled reference engine and the numpy restatement."""
    from oracle import onnx_numpy
    g, _ = build_single_conv(cin=cin, cout=cout, k=k, s=s, hw=hw, seed=6, groups=groups)
    p = str(engine_dir / f"grouped_{cin}_{cout}_{k}_{s}_{groups}_{hw}.engine")
    write_engine(p, g)
    x = np.random.default_rng(8).random((3, cin, hw, hw), dtype=np.float32) - 0.5
    y = run_engine(p, x, prec)
    ref = onnx_numpy.run(g, [x])[0]
    assert normwise(y, ref) <= TOL[prec]
    if R.available():
        for i in range(3):
            r = R.RefSession(p).run(x[i:i + 1])
            assert normwise(y[i:i + 1], r) <= TOL[prec]


@pytest.mark.parametrize("prec", [pb.FP32, pb.BF16])
def test_depthwise3x3_kernel_equals_generic(engine_dir, prec):
    """The depthwise 3x3 kernel (two channels x four rows per thread) sums each output
    in the generic grouped kernel's order: identical bits, stride 1 and 2, odd sizes,
    fused SiLU and a residual."""
    from pdefa_b200.engine_file import TensorInfo
    from pdefa_b200.yolo import _Builder
    b = _Builder(4)
    g = b.g
    g.graph_inputs = [-1]
    g.input_infos = [TensorInfo("images", [1, 8, 37, 29])]
    y, s = b.conv(-1, (8, 37, 29), 48, 1, 1, "m.0")
    z, s = b.conv(y, s, 48, 3, 1, "m.1", groups=48)
    (z,) = g.add_node('Add', "/m.1/Add", [y, z])
    z, s = b.conv(z, s, 48, 3, 2, "m.2", groups=48)
    z, s = b.conv(z, s, 48, 3, 1, "m.3", groups=48, act=False)
    g.graph_outputs = [z]
    g.output_infos = [TensorInfo("output0", [1, 48, s[1], s[2]])]
    p = str(engine_dir / "dw_chain.engine")
    write_engine(p, g)
    x = np.random.default_rng(9).random((3, 8, 37, 29), dtype=np.float32) - 0.5
    fast = run_engine(p, x, prec)
    generic = run_engine(p, x, prec, env={"PDEFA_NO_DW3": "1"})
    np.testing.assert_array_equal(fast, generic)
    if R.available():
        for i in range(3):
            assert normwise(fast[i:i + 1], R.RefSession(p).run(x[i:i + 1])) <= TOL[prec]
