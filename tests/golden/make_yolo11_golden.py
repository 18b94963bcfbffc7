"""Writes tests/golden/yolo11n_96.npz and tests/golden/c2psa_12.npz: the reference
engine's outputs for a random-init YOLO11n at 96x96 and for one C2PSA block
(128 channels, 12x12), on seeded inputs the tests regenerate.

The reference is the pdefa CPU engine built from its own sources by oracle/ref.mk
(oracle/_ref/libpdefa_ref.so), driven through its C API (oracle/ref_engine.py).
Inputs are not stored: they are np.random.default_rng(seed).random(shape, float32)
with the seeds below.

Usage: python tests/golden/make_yolo11_golden.py
"""
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", ".."))

from oracle import ref_engine as R                      # noqa: E402
from pdefa_b200.engine_file import write_engine           # noqa: E402
from pdefa_b200.yolo import build_c2psa, build_yolo11     # noqa: E402

CASES = {
    "yolo11n_96.npz": (lambda: build_yolo11("n", imgsz=96, seed=0)[0], (1, 3, 96, 96), 11),
    "c2psa_12.npz": (lambda: build_c2psa(c=128, hw=12, seed=0)[0], (1, 128, 12, 12), 12),
}


def main():
    tmp = tempfile.mkdtemp()
    for name, (make, shape, seed) in CASES.items():
        p = os.path.join(tmp, name + ".engine")
        write_engine(p, make())
        x = np.random.default_rng(seed).random(shape, dtype=np.float32)
        y = R.RefSession(p, threads=4).run(x)
        np.savez_compressed(os.path.join(HERE, name), y=y, seed=seed)


if __name__ == "__main__":
    main()
