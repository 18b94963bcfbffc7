"""The drop-in claim, tested through the reference's own Python layer: the package
`pdefa` (pdefa/python/src/pdefa: _bindings.py, batch.py, __init__.py, byte-identical
to the reference's, installed by tests/install_reference_python.sh into baseline/_ref)
loads this repository's libpdefa_native.so by the file name it looks for
(_bindings.py:13-23) and drives it through its ctypes declarations.

* test_reference_python_layer_results: Context / Model / Session.run /
  output().tolist() / stats, ops_matmul, the reference's pure-Python decode_yolo and
  BatchInference.run on image files, checked against the compiled reference engine's
  goldens (FP32 path: normwise <= 1e-5) and, for decode, bit for bit against this
  library's GPU decode of the same output.
* test_reference_suite_passes: the reference's own pytest suite (pdefa/tests, 86
  tests) run unchanged against the library.

The only help the layer gets: `Tensor` is predefined in builtins while `_bindings.py`
is imported, because its annotation `-> Tensor` at line 306 precedes the class and
raises NameError on every Python version (the module's own class then shadows it).
"""
import json
import os
import re
import shutil
import subprocess
import sys

import numpy as np
import pytest

import pdefa_b200 as pb

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_PKG = os.path.join(ROOT, "baseline", "_ref", "pdefa")
REF_TESTS = os.path.join(ROOT, "baseline", "_ref", "pdefa_tests")
LIB = os.path.join(ROOT, "pdefa_b200", "lib", "libpdefa_native.so")
PLUGIN = "import builtins\nbuiltins.Tensor = object   # see tests/test_gpu_reference_python.py\n"


def _package(tmp):
    """Copy of the reference package whose lib/ holds only this repository's library."""
    if not os.path.isfile(os.path.join(REF_PKG, "_bindings.py")):
        pytest.skip("reference Python layer not installed (PDEFA_REFERENCE=... sh tests/install_reference_python.sh)")
    dst = os.path.join(tmp, "pdefa")
    os.makedirs(os.path.join(dst, "lib"))
    for f in ("__init__.py", "_bindings.py", "batch.py", "py.typed"):
        if os.path.exists(os.path.join(REF_PKG, f)):
            shutil.copy(os.path.join(REF_PKG, f), os.path.join(dst, f))
    shutil.copy(os.path.join(REF_PKG, "lib", "__init__.py"), os.path.join(dst, "lib", "__init__.py"))
    os.symlink(LIB, os.path.join(dst, "lib", "libpdefa_native.so"))
    return tmp


def _normwise(y, ref):
    return float(np.abs(y - ref).max() / max(np.abs(ref).max(), 1e-30))


def test_reference_python_layer_results(tmp_path, golden):
    from oracle import ref_engine as R
    if not R.available():
        pytest.skip("compiled reference engine (oracle/_ref) not built")
    pkg = _package(str(tmp_path))
    images = os.path.join(REF_TESTS, "data")
    if not os.path.isdir(images):
        pytest.skip("reference test data not installed")
    out = os.path.join(str(tmp_path), "res.npz")
    env = dict(os.environ, PDEFA_PRECISION="")
    r = subprocess.run([sys.executable, os.path.join(ROOT, "tests", "reference_python_driver.py"), pkg, ROOT,
                        images, out], capture_output=True, text=True, timeout=600, env=env)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    d = np.load(out)
    # the reference layer loaded this repository's library, not another one
    assert os.path.realpath(str(d["lib"])) == os.path.realpath(LIB)
    assert int(d["threads"]) == 3

    g = golden("yolov8n_128.npz")
    y = d["y128"]
    assert tuple(d["y128_shape"]) == (1, 84, 336)
    assert _normwise(y, g["y"]) <= 1e-5
    assert int(d["stats_runs"]) == 1

    # the reference's Python decode_yolo on our output == our GPU decode of the same array
    ref_dets = json.loads(str(d["dets128"]))
    gpu_dets = pb.decode_yolo(y, None, 0.25, 0.45, 300)
    assert len(ref_dets) == len(gpu_dets) > 0
    for a, b in zip(ref_dets, gpu_dets):
        for k in ("x1", "y1", "x2", "y2", "conf"):
            assert a[k] == b[k], (k, a, b)
        assert a["cls"] == b["cls"]

    m = golden("matmul_96x80x64.npz")
    assert _normwise(d["matmul"], m["c"]) <= 1e-5

    # BatchInference outputs against the compiled reference engine on the same images
    from pdefa_b200.engine_file import write_engine
    from pdefa_b200.yolo import build_yolov8
    g640, _ = build_yolov8("n", imgsz=640, seed=0)
    p = os.path.join(str(tmp_path), "y8n_640.engine")
    write_engine(p, g640)
    ref = R.RefSession(p, threads=os.cpu_count() or 4)
    for i, name in enumerate(("bus.png", "cat.jpg")):
        t, meta = pb.prepare_for_engine(os.path.join(images, name), 640, 640)
        x = t.to_numpy()
        np.testing.assert_array_equal(
            d["batch_meta"][i], [meta.target_w, meta.target_h, meta.orig_w, meta.orig_h, meta.pad_x, meta.pad_y,
                                 meta.scaled_w, meta.scaled_h, meta.ratio])
        yr = ref.run(x)
        assert _normwise(d["batch_y"][i], yr[0] if yr.ndim == 3 else yr) <= 1e-5, name


def test_reference_suite_passes(tmp_path):
    pkg = _package(str(tmp_path))
    if not os.path.isfile(os.path.join(REF_TESTS, "conftest.py")):
        pytest.skip("reference test suite not installed (tests/install_reference_python.sh)")
    shutil.copytree(REF_TESTS, os.path.join(pkg, "tests"))
    with open(os.path.join(pkg, "_pdefa_forward_ref.py"), "w") as f:
        f.write(PLUGIN)
    env = dict(os.environ, PYTHONPATH=pkg, PDEFA_PRECISION="")
    r = subprocess.run([sys.executable, "-m", "pytest", "-p", "_pdefa_forward_ref", "-p", "no:cacheprovider", "-q",
                        "-rfE", "tests"], cwd=pkg, capture_output=True, text=True, timeout=900, env=env)
    tail = r.stdout[-6000:]
    m = re.search(r"(\d+) passed", tail)
    assert r.returncode == 0, tail + r.stderr[-2000:]
    assert m and int(m.group(1)) >= 80, tail
