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
                                            (1, 17, 1, 3, 63, 61), (5, 64, 64, 3, 64, 64),
                                            # identity geometry (the identity kernel): RGB, gray, RGBA
                                            (3, 640, 640, 3, 640, 640), (2, 96, 128, 1, 128, 96),
                                            (2, 40, 72, 4, 72, 40)])
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


def _ref_prepare(path, tw, th, scale, pad):
    """The reference's pdefa_prepare_for_engine (compiled from its sources)."""
    import ctypes as C
    from tests.golden import make_letterbox_golden as g
    L = C.CDLL(os.path.join(os.path.dirname(os.path.dirname(__file__)), "oracle", "_ref", "libpdefa_ref.so"))
    L.pdefa_prepare_for_engine.argtypes = [C.c_char_p, C.c_int32, C.c_int32, C.c_float, C.c_float,
                                           C.POINTER(C.c_void_p), C.POINTER(g.Meta)]
    L.engine_tensor_data.argtypes = [C.c_void_p, C.POINTER(C.c_void_p), C.POINTER(C.c_size_t)]
    L.engine_tensor_destroy.argtypes = [C.c_void_p]
    t, m = C.c_void_p(), g.Meta()
    assert L.pdefa_prepare_for_engine(path.encode(), tw, th, scale, pad, C.byref(t), C.byref(m)) == 0
    d, nb = C.c_void_p(), C.c_size_t()
    L.engine_tensor_data(t, C.byref(d), C.byref(nb))
    out = np.ctypeslib.as_array((C.c_float * (3 * th * tw)).from_address(d.value)).copy().reshape(1, 3, th, tw)
    L.engine_tensor_destroy(t)
    return out, [m.target_w, m.target_h, m.orig_w, m.orig_h, m.pad_x, m.pad_y, m.scaled_w, m.scaled_h], m.ratio


@pytest.mark.parametrize("ct,bd,hw,target", [(2, 8, (48, 64), 96), (6, 8, (33, 20), 64), (0, 16, (17, 23), 40),
                                             (3, 4, (29, 31), 56), (0, 8, (50, 41), 64)])
def test_prepare_for_engine_png_matches_reference(tmp_path, ct, bd, hw, target):
    """PNG file -> letterboxed tensor: decode on the host + letterbox on the GPU equal the
    reference's prepare_for_engine bit for bit (16-bit gray included, which the
    reference letterboxes one byte per sample)."""
    from tests.test_image_png_cpu import CHANNELS, write_png
    ref_lib = os.path.join(os.path.dirname(os.path.dirname(__file__)), "oracle", "_ref", "libpdefa_ref.so")
    rng = np.random.default_rng(ct * 100 + bd)
    palette = None
    if ct == 3:
        palette = rng.integers(0, 256, (16, 3))
        samples = rng.integers(0, 16, hw + (1,))
    else:
        samples = rng.integers(0, 1 << bd, hw + (CHANNELS[ct],))
    p = str(tmp_path / "img.png")
    write_png(p, samples, ct, bd, palette, seed=5)
    t, meta = pb.prepare_for_engine(p, target, target, 1 / 255, 114 / 255)
    y = t.to_numpy()
    assert y.shape == (1, 3, target, target)
    assert meta.orig_w == hw[1] and meta.orig_h == hw[0]
    if os.path.exists(ref_lib):
        ref, m, ratio = _ref_prepare(p, target, target, 1 / 255, 114 / 255)
        np.testing.assert_array_equal(y, ref)
        assert [getattr(meta, k) for k in META_FIELDS] == m and np.float32(meta.ratio) == np.float32(ratio)
    img = pb.load_image(p)
    t2, meta2 = pb.preprocess_letterbox(img, target, target, 1 / 255, 114 / 255)
    np.testing.assert_array_equal(t2.to_numpy(), y)
    assert meta2 == meta


def test_batch_inference_run_on_png_files(tmp_path, engine_dir):
    """BatchInference.run(paths), the reference's image-file signature, gives each file's
    raw model output and letterbox meta."""
    from tests.test_image_png_cpu import write_png
    g, _ = build_yolov8("n", imgsz=128, seed=0)
    p = str(engine_dir / "y8n_128_run.engine")
    write_engine(p, g)
    ctx = pb.Context(precision=pb.BF16)
    m = pb.Model(ctx, p)
    rng = np.random.default_rng(4)
    paths = []
    for i, hw in enumerate([(96, 128), (128, 100)]):
        f = str(tmp_path / f"f{i}.png")
        write_png(f, rng.integers(0, 256, hw + (3,)), 2, 8, seed=i)
        paths.append(f)
    with pb.BatchInference(ctx, m, batch_size=2, devices=[0]) as bi:
        res = bi.run(paths, 128, 128)
    for f, (out, meta) in zip(paths, res):
        x, meta2 = pb.prepare_for_engine(f, 128, 128)
        s = pb.Session(ctx, m)
        s.set_input(0, x)
        s.run()
        np.testing.assert_array_equal(out.to_numpy(), s.output(0).to_numpy())
        assert meta == meta2


@pytest.mark.parametrize("name", ["rgb420_q75_odd", "gray_q90", "rgb422_rst"])
def test_prepare_for_engine_jpeg_matches_reference(tmp_path, name):
    """JPEG file -> letterboxed tensor equals the reference's prepare_for_engine, and
    the GPU letterbox of the pinned reference pixels (tests/golden/jpeg_ref.npz)."""
    ref_lib = os.path.join(os.path.dirname(os.path.dirname(__file__)), "oracle", "_ref", "libpdefa_ref.so")
    z = np.load(os.path.join(os.path.dirname(__file__), "golden", "jpeg_ref.npz"))
    p = str(tmp_path / f"{name}.jpg")
    with open(p, "wb") as f:
        f.write(z[f"{name}.jpg"].tobytes())
    w, h, _ = (int(v) for v in z[f"{name}.whf"])
    t, meta = pb.prepare_for_engine(p, 64, 64, 1 / 255, 114 / 255)
    y = t.to_numpy()
    assert (meta.orig_w, meta.orig_h) == (w, h)
    pixels = z[f"{name}.rgb"].reshape(h, w, 3)
    y2, meta2 = pb.letterbox_u8(pixels, 64, 64, 1 / 255, 114 / 255)
    np.testing.assert_array_equal(np.asarray(y2)[0], y[0])
    if os.path.exists(ref_lib):
        ref, m, ratio = _ref_prepare(p, 64, 64, 1 / 255, 114 / 255)
        np.testing.assert_array_equal(y, ref)
        assert [getattr(meta, k) for k in META_FIELDS] == m


def test_batch_submit_u8_matches_detect_u8(engine_dir):
    """Pipelined submits (pdefa_batch_submit_u8 / pdefa_batch_wait): each call's
    results, collected after later calls were queued (and after a synchronous call on
    the same runner), equal what detect_u8 returns for the same frames."""
    g, _ = build_yolov8("n", imgsz=128, seed=0)
    p = str(engine_dir / "y8n_128_submit.engine")
    write_engine(p, g)
    ctx = pb.Context(precision=pb.BF16)
    m = pb.Model(ctx, p)
    rng = np.random.default_rng(21)
    frames = [rng.integers(0, 256, (n, 96, 120, 3), dtype=np.uint8) for n in (7, 3, 9, 1)]
    kw = dict(target_w=128, target_h=128, conf_thres=0.2, iou_thres=0.5, max_det=40)
    with pb.BatchInference(ctx, m, batch_size=4, devices=[0]) as bi:
        want = [bi.detect_u8(f, **kw) for f in frames]
        pend = [bi.submit_u8(frames[0], **kw), bi.submit_u8(frames[1], **kw)]
        mid = bi.detect_u8(frames[2], **kw)        # a synchronous call between submits
        pend += [bi.submit_u8(frames[2], **kw), bi.submit_u8(frames[3], **kw)]
        got = [q.result() for q in pend]
        again = bi.submit_u8(frames[0], **kw)
        bi.wait()
        got.append(again.result())
    for (c, d, meta), (cw, dw, mw) in zip(got[:4] + [mid, got[4]], want + [want[2], want[0]]):
        np.testing.assert_array_equal(c, cw)
        for b in range(len(c)):
            np.testing.assert_array_equal(d[b, :c[b]], dw[b, :cw[b]])
        assert meta == mw


_FUSED_SCRIPT = r"""
import sys
import numpy as np
import pdefa_b200 as pb
path, out, prec = sys.argv[1], sys.argv[2], sys.argv[3]
ctx = pb.Context(precision=pb.BF16 if prec == "bf16" else pb.FP32)
m = pb.Model(ctx, path)
rng = np.random.default_rng(33)
ident = rng.integers(0, 256, (5, 128, 128, 3), dtype=np.uint8)
other = rng.integers(0, 256, (3, 96, 150, 3), dtype=np.uint8)
kw = dict(conf_thres=0.2, iou_thres=0.5, max_det=40)
res = {}
with pb.BatchInference(ctx, m, batch_size=2, devices=[0]) as bi:
    for tag, f in (("a", ident), ("b", other), ("c", ident[::-1].copy())):
        c, d, meta = bi.detect_u8(f, 128, 128, **kw)
        res["counts_" + tag], res["dets_" + tag] = c, d
np.savez(out, **res)
"""


def _session_dets(ctx, m, imgs, kw):
    x, meta = pb.letterbox_u8(imgs, 128, 128)
    s = pb.Session(ctx, m)
    s.set_input(0, pb.Tensor.from_numpy(x))
    s.run()
    y = s.output(0).to_numpy()
    return [pb.decode_yolo(y[b], meta, kw["conf_thres"], kw["iou_thres"], kw["max_det"]) for b in range(len(imgs))]


@pytest.mark.parametrize("prec", ["bf16", "fp32"])
def test_detect_u8_fused_stem_matches_letterbox_path(engine_dir, tmp_path, prec):
    """Frames already at the model size with scale-only preprocessing skip the letterbox
    kernel: the runner lowers a plan whose stem conv reads the 8-bit pixels itself
    (pixel * scale, the identity letterbox's value). Its detections equal the letterbox
    + session + decode pieces run one by one, on the same runner as calls with other
    geometries (which keep the letterbox). PDEFA_VERBOSE shows which path ran: BF16
    fuses, FP32 (no tcgen05 stem) keeps the letterbox."""
    import subprocess
    import sys
    g, _ = build_yolov8("n", imgsz=128, seed=0)
    p = str(engine_dir / "y8n_128_fused.engine")
    write_engine(p, g)
    out = str(tmp_path / "fused.npz")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, PDEFA_VERBOSE="1", PYTHONPATH=root + os.pathsep + os.environ.get("PYTHONPATH", ""))
    r = subprocess.run([sys.executable, "-c", _FUSED_SCRIPT, p, out, prec], capture_output=True, text=True,
                       timeout=600, env=env, cwd=root)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    fused = "8-bit frames read by the stem" in r.stderr
    assert fused == (prec == "bf16"), r.stderr[-3000:]
    d = np.load(out)
    ctx = pb.Context(precision=pb.BF16 if prec == "bf16" else pb.FP32)
    m = pb.Model(ctx, p)
    rng = np.random.default_rng(33)
    ident = rng.integers(0, 256, (5, 128, 128, 3), dtype=np.uint8)
    other = rng.integers(0, 256, (3, 96, 150, 3), dtype=np.uint8)
    kw = dict(conf_thres=0.2, iou_thres=0.5, max_det=40)
    total = 0
    for tag, f in (("a", ident), ("b", other), ("c", ident[::-1].copy())):
        exp = _session_dets(ctx, m, f, kw)
        counts, dets = d["counts_" + tag], d["dets_" + tag]
        for b in range(len(f)):
            got = dets[b, :counts[b]]
            assert len(exp[b]) == counts[b], (tag, b)
            assert [(e["x1"], e["y1"], e["x2"], e["y2"], e["conf"], e["cls"]) for e in exp[b]] == \
                [(r["x1"], r["y1"], r["x2"], r["y2"], r["conf"], int(r["cls"])) for r in got], (tag, b)
            total += int(counts[b])
    assert total > 0
