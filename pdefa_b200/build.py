"""Builds pdefa_b200/lib/libpdefa_native.so from pdefa_b200/csrc with nvcc.

The library is built in-tree (objects under pdefa_b200/_build, the shared object
under pdefa_b200/lib) for sm_100a only. Only the C-ABI entry points are exported
(-fvisibility=hidden + explicit default visibility on the API declarations).

Usage: python -m pdefa_b200.build [--force] [--jobs N]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB_DIR = os.path.join(HERE, "lib")
LIB = os.path.join(LIB_DIR, "libpdefa_native.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(f for f in os.listdir(SRC) if f.endswith((".cu", ".cpp")))


def _newest_header() -> float:
    hs = [os.path.join(SRC, f) for f in os.listdir(SRC) if f.endswith((".h", ".cuh"))]
    inc = os.path.join(os.path.dirname(HERE), "include")
    hs += [os.path.join(inc, f) for f in os.listdir(inc)]
    return max(os.path.getmtime(h) for h in hs)


def compile_one(src: str, force: bool) -> str:
    obj = os.path.join(BUILD, src + ".o")
    path = os.path.join(SRC, src)
    if (not force and os.path.exists(obj) and os.path.getmtime(obj) >= os.path.getmtime(path)
            and os.path.getmtime(obj) >= _newest_header()):
        return obj
    cmd = [nvcc(), "-std=c++17", "-O3", *ARCH, "-lineinfo", "-Xcompiler", "-fPIC",
           "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr", "-c", path, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    return obj


def build(force: bool = False, jobs: int = 0) -> str:
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIB_DIR, exist_ok=True)
    srcs = sources()
    jobs = jobs or min(len(srcs), os.cpu_count() or 4)
    with cf.ThreadPoolExecutor(jobs) as ex:
        objs = list(ex.map(lambda s: compile_one(s, force), srcs))
    if (force or not os.path.exists(LIB)
            or max(os.path.getmtime(o) for o in objs) > os.path.getmtime(LIB)):
        cmd = [nvcc(), "-shared", *ARCH, "-cudart", "static", "-o", LIB + ".tmp", *objs, "-lpthread", "-ldl", "-lrt", "-lz"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(LIB + ".tmp", LIB)
    return LIB


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=0)
    a = ap.parse_args(argv)
    print(build(a.force, a.jobs))


if __name__ == "__main__":
    sys.exit(main())
