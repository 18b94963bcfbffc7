"""Generates the committed golden fixtures under tests/golden/.

Run here (where the reference sources exist), never on the GPU box:
    make -f oracle/ref.mk -j8 && python tests/golden/make_golden.py

Every expected output comes from the reference itself:
* engine outputs from the reference CPU engine compiled from its sources
  (oracle/_ref/libpdefa_ref.so, driven through its C ABI by oracle/ref_engine.py);
* decode outputs from the reference's own Python decode_yolo
  (pdefa/python/src/pdefa/_bindings.py:1095-1212), imported from a temporary copy
  of the reference package whose native library is the compiled oracle (the
  temporary copy adds `from __future__ import annotations` so it imports on
  Python 3.12; the reference source tree is not modified).
Inputs are seeded numpy arrays or graphs built by pdefa_b200.yolo, so only
small arrays are stored.
"""
from __future__ import annotations

import json
import os
import shutil
import sys
import tempfile

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
OUT = os.path.dirname(os.path.abspath(__file__))
REF = os.environ.get("PDEFA_REFERENCE", "")   # the pdefa reference checkout (needed to make the decode goldens)

from oracle import ref_engine as R  # noqa: E402
from pdefa_b200.engine_file import EngineGraph, TensorInfo, write_engine  # noqa: E402
from pdefa_b200.yolo import build_single_conv, build_yolov8  # noqa: E402


def build_tiny(seed: int = 3) -> EngineGraph:
    """Conv3x3 3->8 -> global mean -> Reshape [1,8] -> MatMul [8,4] (classifier-style)."""
    rng = np.random.default_rng(seed)
    g = EngineGraph()
    g.graph_inputs = [-1]
    g.input_infos = [TensorInfo("input", [1, 3, 64, 64])]
    w = g.add_weight("conv.weight", rng.standard_normal((8, 3, 3, 3)) * 0.3)
    b = g.add_weight("conv.bias", rng.standard_normal(8) * 0.1)
    (y,) = g.add_node('Conv2d', "/conv/Conv", [-1, w, b], stride_h=1, stride_w=1, pad_h=1, pad_w=1)
    (y,) = g.add_node('AvgPool2d', "/ReduceMean", [y], kernel_h=0, kernel_w=0)
    s = g.add_weight("/Reshape_shape", [1, 8])
    (y,) = g.add_node('Reshape', "/Reshape", [y, s])
    fc = g.add_weight("fc.weight_T", rng.standard_normal((8, 4)) * 0.5)
    (y,) = g.add_node('MatMul', "/fc/MatMul", [y, fc])
    g.graph_outputs = [y]
    g.output_infos = [TensorInfo("output", [1, 4])]
    return g


def reference_python_decode():
    """Import the reference decode_yolo from a temporary copy of its package."""
    tmp = tempfile.mkdtemp(prefix="pdefa_refpy_")
    pkg = os.path.join(tmp, "pdefa")
    if not REF:
        sys.exit("set PDEFA_REFERENCE to the pdefa reference checkout")
    src = os.path.join(REF, "pdefa", "python", "src", "pdefa")
    os.makedirs(os.path.join(pkg, "lib"))
    for f in ("__init__.py", "batch.py"):
        shutil.copy(os.path.join(src, f), os.path.join(pkg, f))
    with open(os.path.join(src, "_bindings.py")) as fi, open(os.path.join(pkg, "_bindings.py"), "w") as fo:
        fo.write("from __future__ import annotations\n" + fi.read())
    open(os.path.join(pkg, "lib", "__init__.py"), "w").close()
    os.symlink(R.LIB_PATH, os.path.join(pkg, "lib", "libpdefa_native.so"))
    sys.path.insert(0, tmp)
    import pdefa  # noqa: F401
    return pdefa


def dets_json(dets):
    return [{k: (float(v) if k != "cls" else int(v)) for k, v in d.items()} for d in dets]


def main():
    if not R.available():
        raise SystemExit("build the reference engine first: make -f oracle/ref.mk")
    tmp = tempfile.mkdtemp()

    # a) ops_matmul, small
    rng = np.random.default_rng(7)
    A = rng.standard_normal((96, 80)).astype(np.float32)
    B = rng.standard_normal((80, 64)).astype(np.float32)
    np.savez_compressed(os.path.join(OUT, "matmul_96x80x64.npz"), a=A, b=B, c=R.matmul(A, B, threads=4))

    # b) stem conv (cfg2 layer at 64x64)
    g, _ = build_single_conv(cin=3, cout=16, k=3, s=2, hw=64, seed=1)
    p = os.path.join(tmp, "stem.engine")
    write_engine(p, g)
    x = np.random.default_rng(0).random((1, 3, 64, 64), dtype=np.float32)
    np.savez_compressed(os.path.join(OUT, "stem_64.npz"), x=x, y=R.RefSession(p, threads=4).run(x))

    # c) YOLOv8n at 128x128, batch 1
    g, info = build_yolov8("n", imgsz=128, seed=0)
    p = os.path.join(tmp, "y8n_128.engine")
    write_engine(p, g)
    x = np.random.default_rng(0).random((1, 3, 128, 128), dtype=np.float32)
    y = R.RefSession(p, threads=4).run(x)
    np.savez_compressed(os.path.join(OUT, "yolov8n_128.npz"), x=x, y=y)

    # d) tiny classifier graph
    g = build_tiny()
    p = os.path.join(tmp, "tiny.engine")
    write_engine(p, g)
    xt = np.random.default_rng(5).random((1, 3, 64, 64), dtype=np.float32)
    np.savez_compressed(os.path.join(OUT, "tiny.npz"), x=xt, y=R.RefSession(p, threads=4).run(xt))

    # e) decode: reference Python decode_yolo on reference engine output + adversarial cases
    pdefa = reference_python_decode()
    cases = []

    def add(name, key, preds, meta=None, conf=0.25, iou=0.45, max_det=300):
        m = None
        if meta is not None:
            m = pdefa.PreprocessMeta(**meta) if hasattr(pdefa, "PreprocessMeta") else None
        dets = pdefa.decode_yolo(preds.tolist(), m, conf, iou, max_det)
        cases.append({"name": name, "input": key, "meta": meta, "conf": conf, "iou": iou, "max_det": max_det,
                      "dets": dets_json(dets)})

    preds = {"y8n_128": y[0]}
    add("y8n_128", "y8n_128", y[0])
    meta = dict(target_w=128, target_h=128, orig_w=200, orig_h=150, pad_x=0, pad_y=16, scaled_w=128,
                scaled_h=96, ratio=float(np.float32(0.64)))  # ratio arrives as float32 from C
    add("y8n_128_meta", "y8n_128", y[0], meta=meta)
    add("y8n_128_conf55_iou30_det25", "y8n_128", y[0], conf=0.55, iou=0.30, max_det=25)

    r = np.random.default_rng(11)
    A_ = 700
    adv = np.zeros((84, A_), dtype=np.float32)
    centers = r.uniform(50, 590, size=(12, 2))
    k = r.integers(0, 12, size=A_)
    adv[0] = centers[k, 0] + r.normal(0, 6, A_)
    adv[1] = centers[k, 1] + r.normal(0, 6, A_)
    adv[2] = r.uniform(10, 120, A_)
    adv[3] = r.uniform(10, 120, A_)
    adv[4:] = np.round(r.uniform(0, 1, (80, A_)) ** 6 * 16) / 16     # coarse scores: many exact ties
    adv[4 + r.integers(0, 80, A_), np.arange(A_)] = np.round(r.uniform(0.2, 1.0, A_) * 8) / 8
    preds["adversarial"] = adv
    add("adversarial", "adversarial", adv)
    add("adversarial_meta", "adversarial", adv, meta=dict(target_w=640, target_h=640, orig_w=500, orig_h=333, pad_x=0,
                                           pad_y=106, scaled_w=640, scaled_h=426,
                                           ratio=float(np.float32(1.28))))
    add("adversarial_det7", "adversarial", adv, conf=0.3, iou=0.5, max_det=7)
    add("adversarial_iou0", "adversarial", adv, conf=0.5, iou=0.0)
    empty = np.zeros((84, 8400), dtype=np.float32)
    preds["zeros_8400"] = empty
    add("zeros_8400", "zeros_8400", empty)
    np.savez_compressed(os.path.join(OUT, "decode_inputs.npz"), **preds)
    with open(os.path.join(OUT, "decode_expected.json"), "w") as f:
        json.dump(cases, f, indent=0)
    print("golden fixtures written to", OUT)


if __name__ == "__main__":
    main()
