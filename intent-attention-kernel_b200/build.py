"""Build libiak_b200.so (sm_100a) in-tree with nvcc.

    python intent-attention-kernel_b200/build.py [--force] [--verbose-ptxas]

Each csrc/*.cu is compiled for ``-gencode arch=compute_100a,code=sm_100a`` with
``-lineinfo``; the objects are linked into
``intent-attention-kernel_b200/intent_attention/libiak_b200.so`` with the CUDA
runtime linked statically, so the library needs only the NVIDIA driver at run
time.  Rebuilds only what changed unless ``--force``.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
OBJ_DIR = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "intent_attention", "libiak_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
          "-I", INCLUDE, "-I", CSRC]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _deps_mtime() -> float:
    files = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(INCLUDE, "*.h"))
    return max((os.path.getmtime(f) for f in files), default=0.0)


def _compile(src: str, force: bool, ptxas_v: bool) -> str:
    obj = os.path.join(OBJ_DIR, os.path.basename(src) + ".o")
    if not force and os.path.exists(obj):
        if os.path.getmtime(obj) >= max(os.path.getmtime(src), _deps_mtime()):
            return obj
    cmd = [nvcc()] + ARCH + CFLAGS + (["-Xptxas", "-v"] if ptxas_v else []) + ["-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    if ptxas_v:
        sys.stderr.write(r.stderr)
    return obj


def build(force: bool = False, ptxas_v: bool = False) -> str:
    os.makedirs(OBJ_DIR, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, ptxas_v), srcs))
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        tmp = LIB + ".tmp"
        cmd = [nvcc()] + ARCH + ["-shared", "-cudart", "static", "-o", tmp] + objs
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose-ptxas", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.verbose_ptxas))
