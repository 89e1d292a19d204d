"""In-tree build of the four kernel libraries for sm_100a.

Each op compiles from csrc/<op>.cu into lib/<op>/libkernel.so, the layout the reference's Python wrappers load
(`$CKOPT_BUILD_DIR/libkernel.so`, e.g. rmsnorm/candidate.py:25): pointing CKOPT_BUILD_DIR at lib/<op> makes the
reference's own candidate.py drive these kernels. The CUDA runtime is linked statically (nvcc's default), so a
library needs only the driver at run time.
"""

import os
import shutil
import subprocess
from concurrent.futures import ThreadPoolExecutor

PKG_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REPO_ROOT = os.path.dirname(PKG_ROOT)
CSRC = os.path.join(PKG_ROOT, "csrc")
INCLUDE = os.path.join(REPO_ROOT, "include")
LIB_ROOT = os.path.join(PKG_ROOT, "lib")
OPS = ("softmax", "rmsnorm", "rope", "topk")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-shared", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-I", INCLUDE,
]


def nvcc_path():
    for cand in (os.environ.get("CUDA_HOME") and os.path.join(os.environ["CUDA_HOME"], "bin", "nvcc"),
                 "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("ckb200 build: nvcc not found (set CUDA_HOME)")


def lib_path(op):
    return os.path.join(LIB_ROOT, op, "libkernel.so")


def _sources(op):
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cuh")]
    return [os.path.join(CSRC, op + ".cu"), os.path.join(INCLUDE, f"ckb200_{op}.h")] + headers


def _stale(op):
    out = lib_path(op)
    if not os.path.exists(out):
        return True
    built = os.path.getmtime(out)
    return any(os.path.getmtime(s) > built for s in _sources(op))


def _compile(op, verbose):
    out = lib_path(op)
    os.makedirs(os.path.dirname(out), exist_ok=True)
    tmp = out + ".tmp"
    cmd = [nvcc_path(), *NVCC_FLAGS, "-o", tmp, os.path.join(CSRC, op + ".cu")]
    if verbose:
        print(" ".join(cmd), flush=True)
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"ckb200 build of {op} failed:\n{proc.stdout}\n{proc.stderr}")
    os.replace(tmp, out)
    return out


def build(force=False, verbose=False, ops=OPS):
    """Compiles every stale (or, with force, every) op library; returns the library paths."""
    todo = [op for op in ops if force or _stale(op)]
    with ThreadPoolExecutor(max_workers=len(todo) or 1) as pool:
        list(pool.map(lambda op: _compile(op, verbose), todo))
    return [lib_path(op) for op in ops]


if __name__ == "__main__":
    import sys
    for path in build(force="--force" in sys.argv, verbose=True):
        print(path)
