"""Runs the reference's own Python layer (package `pdefa`, its files unchanged) on top of
this repository's libpdefa_native.so and saves what it returns, for
tests/test_gpu_reference_python.py to check against the oracle and the GPU decode.

Usage: python reference_python_driver.py <dir holding the pdefa package> <repo root>
                                         <images dir> <out.npz>

The reference's `_bindings.py` annotates `_ops_binary(...) -> Tensor` before `Tensor`
is defined (pdefa/python/src/pdefa/_bindings.py:306), which raises NameError at import
on every Python version. The caller predefines `Tensor` in builtins (a placeholder the
module's own class then shadows) instead of editing the file.
"""
import builtins
import json
import os
import sys
import tempfile

import numpy as np

pkg_dir, repo, images, out_path = sys.argv[1:5]
sys.path.insert(0, pkg_dir)
builtins.Tensor = object
import pdefa  # noqa: E402  (the reference package)
del builtins.Tensor

sys.path.insert(1, repo)
from pdefa_b200.engine_file import write_engine  # noqa: E402  (writes the .engine files only)
from pdefa_b200.yolo import build_yolov8  # noqa: E402

res = {}
lib_path = os.path.realpath(os.path.join(os.path.dirname(pdefa.__file__), "lib", "libpdefa_native.so"))
res["lib"] = np.array(lib_path)

ctx = pdefa.Context()
ctx.set_num_threads(3)
res["threads"] = np.array(ctx.get_num_threads())
tmp = tempfile.mkdtemp()

# Context / Model / Session.run / output().tolist() on the YOLOv8n-128 golden input
g = np.load(os.path.join(repo, "tests", "golden", "yolov8n_128.npz"))
graph, _ = build_yolov8("n", imgsz=128, seed=0)
p128 = os.path.join(tmp, "y8n_128.engine")
write_engine(p128, graph)
model = pdefa.Model(ctx, p128)
info = model.input_info(0)
res["input_shape"] = np.array(list(info.shape) if hasattr(info, "shape") else [])
sess = pdefa.Session(ctx, model)
x = pdefa.from_list(g["x"].tolist())
sess.set_input(0, x)
sess.run()
out = sess.output(0)
res["y128"] = np.array(out.tolist(), dtype=np.float32)
res["y128_shape"] = np.array(out.shape)
st = sess.stats()
res["stats_runs"] = np.array(st["runs"] if isinstance(st, dict) else getattr(st, "runs", -1))

# decode_yolo (the reference's Python decode) on that output
dets = pdefa.decode_yolo(out, None, 0.25, 0.45, 300)
res["dets128"] = np.array(json.dumps([{k: (float(v) if k != "cls" else int(v)) for k, v in d.items()}
                                      for d in dets]))

# ops_matmul on the golden operands
m = np.load(os.path.join(repo, "tests", "golden", "matmul_96x80x64.npz"))
c = pdefa.ops_matmul(pdefa.from_list(m["a"].tolist()), pdefa.from_list(m["b"].tolist()))
res["matmul"] = np.array(c.tolist(), dtype=np.float32)

# BatchInference.run on image files at 640 (batch_size >= images: each image keeps its
# own session's output, as the reference's borrowed outputs require)
graph640, _ = build_yolov8("n", imgsz=640, seed=0)
p640 = os.path.join(tmp, "y8n_640.engine")
write_engine(p640, graph640)
model640 = pdefa.Model(ctx, p640)
paths = [os.path.join(images, f) for f in ("bus.png", "cat.jpg")]
with pdefa.BatchInference(ctx, model640, batch_size=len(paths), num_threads=2) as bi:
    outs = bi.run(paths, 640, 640)
    res["batch_y"] = np.stack([np.array(t.tolist(), dtype=np.float32) for t, _ in outs])
    res["batch_meta"] = np.array([[m_.target_w, m_.target_h, m_.orig_w, m_.orig_h, m_.pad_x, m_.pad_y,
                                   m_.scaled_w, m_.scaled_h, m_.ratio] for _, m_ in outs], dtype=np.float64)
np.savez(out_path, **res)
print("ok")
