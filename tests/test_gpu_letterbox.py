"""GPU letterbox preprocess (pdefa_letterbox*, letterbox.cu) and the 8-bit batch path.

Parity bar: bit-exact. The kernel must equal the reference's preprocess_letterbox
outputs kept in tests/golden/letterbox_ref.npz, and the C restatement
(oracle/letterbox_ref.c, itself pinned to those fixtures) on larger random images.
"""
import os

import numpy as np
import pytest

import pdefa_b200 as pb
from oracle import letterbox_ref
from pdefa_b200.engine_file import write_engine
from pdefa_b200.yolo import build_yolov8

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "letterbox_ref.npz")
META_FIELDS = ("target_w", "target_h", "orig_w", "orig_h", "pad_x", "pad_y", "scaled_w", "scaled_h")


def test_letterbox_matches_reference_golden():
    d = np.load(GOLDEN)
    for i in range(int(d["n_cases"])):
        tw, th, scale, pad = d[f"c{i}_cfg"]
        out, meta = pb.letterbox_u8(d[f"c{i}_img"], int(tw), int(th), float(scale), float(pad))
        np.testing.assert_array_equal(out[0], d[f"c{i}_out"], err_msg=f"case {i}")
        assert [getattr(meta, k) for k in META_FIELDS] == d[f"c{i}_meta"].tolist()
        assert np.float32(meta.ratio) == d[f"c{i}_ratio"]


@pytest.mark.parametrize("n,h,w,ch,tw,th", [(3, 480, 640, 3, 640, 640), (2, 1080, 1920, 3, 640, 640),
                                            (4, 300, 200, 1, 320, 320), (2, 333, 517, 4, 416, 416),
                                            (1, 17, 1, 3, 63, 61), (5, 64, 64, 3, 64, 64)])
def test_letterbox_matches_oracle(n, h, w, ch, tw, th):
    rng = np.random.default_rng(n * 1000 + h)
    imgs = rng.integers(0, 256, (n, h, w, ch), dtype=np.uint8)
    out, meta = pb.letterbox_u8(imgs, tw, th, 1 / 255, 114 / 255)
    assert out.shape == (n, 3, th, tw)
    for b in range(n):
        exp, m = letterbox_ref.letterbox(imgs[b] if ch > 1 else imgs[b, :, :, 0], tw, th, 1 / 255, 114 / 255)
        np.testing.assert_array_equal(out[b], exp)
    assert [getattr(meta, k) for k in META_FIELDS] == [m[k] for k in META_FIELDS]
    assert pb.letterbox_meta(w, h, tw, th) == meta


def test_letterbox_device_entry_point():
    import ctypes as C

    import torch
    from pdefa_b200 import _native as N
    rng = np.random.default_rng(3)
    imgs = rng.integers(0, 256, (3, 90, 70, 3), dtype=np.uint8)
    d_in = torch.from_numpy(imgs).cuda()
    d_out = torch.full((3, 3, 96, 96), -1.0, device="cuda")
    cfg = N.PreConfig(96, 96, 1 / 255, 0.25)
    rc = N.lib().pdefa_letterbox_device(d_in.data_ptr(), 3, 90, 70, 3, C.byref(cfg), d_out.data_ptr(),
                                        torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    host, _ = pb.letterbox_u8(imgs, 96, 96, 1 / 255, 0.25)
    np.testing.assert_array_equal(d_out.cpu().numpy(), host)
    assert N.lib().pdefa_letterbox_device(d_in.data_ptr(), 3, 90, 70, 2, C.byref(cfg), d_out.data_ptr(), None) != 0


def test_detect_u8_matches_letterbox_session_decode(engine_dir):
    """detect_u8 = letterbox on the GPU + inference + decode with the letterbox meta;
    the same pieces run one by one give the same detections."""
    g, _ = build_yolov8("n", imgsz=128, seed=0)
    p = str(engine_dir / "y8n_128_u8.engine")
    write_engine(p, g)
    ctx = pb.Context(precision=pb.BF16)
    m = pb.Model(ctx, p)
    rng = np.random.default_rng(21)
    imgs = rng.integers(0, 256, (5, 96, 150, 3), dtype=np.uint8)
    with pb.BatchInference(ctx, m, batch_size=2, devices=[0]) as bi:
        counts, dets, meta = bi.detect_u8(imgs, 128, 128, conf_thres=0.2, iou_thres=0.5, max_det=40)
    x, meta2 = pb.letterbox_u8(imgs, 128, 128)
    assert meta == meta2 and meta.pad_y > 0
    s = pb.Session(ctx, m)
    s.set_input(0, pb.Tensor.from_numpy(x))
    s.run()
    y = s.output(0).to_numpy()
    for b in range(5):
        exp = pb.decode_yolo(y[b], meta, 0.2, 0.5, 40)
        got = dets[b, :counts[b]]
        assert len(exp) == counts[b]
        assert [(e["x1"], e["y1"], e["x2"], e["y2"], e["cls"]) for e in exp] == \
            [(r["x1"], r["y1"], r["x2"], r["y2"], int(r["cls"])) for r in got]
