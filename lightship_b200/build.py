"""Builds the CUDA backend library ``lightship_b200/liblightship_cuda.so`` for sm_100a.

Every ``.cu`` / ``.cpp`` file under ``lightship_b200/csrc`` is compiled with nvcc
(``-gencode arch=compute_100a,code=sm_100a -lineinfo``) into ``lightship_b200/_build`` and
linked into one shared library next to this file, so the built library travels with the
source tree.  Objects are rebuilt only when a source or header is newer.

Floating point: no fast-math; host code is compiled with ``-ffp-contract=off`` so the
weight-prepack arithmetic (BN fold, per-channel quantization) rounds every operation, as
the reference's Rust code does.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD_DIR = os.path.join(PKG_DIR, "_build")
LIB_PATH = os.path.join(PKG_DIR, "liblightship_cuda.so")


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: set NVCC or install the CUDA toolkit")


ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler", "-fPIC",
    "-Xcompiler", "-ffp-contract=off",
    "--expt-relaxed-constexpr",
    "-I", INCLUDE,
    "-I", CSRC,
]


def _sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))


def _headers() -> list[str]:
    return sorted(
        glob.glob(os.path.join(CSRC, "*.cuh"))
        + glob.glob(os.path.join(CSRC, "*.h"))
        + glob.glob(os.path.join(INCLUDE, "*.h"))
    )


def _newest(paths: list[str]) -> float:
    return max((os.path.getmtime(p) for p in paths), default=0.0)


def _compile(src: str, obj: str, extra: list[str], verbose: bool) -> str:
    cmd = [nvcc_path(), *ARCH_FLAGS, *COMMON_FLAGS, *extra, "-c", src, "-o", obj]
    if src.endswith(".cpp"):
        cmd.insert(1, "-x")
        cmd.insert(2, "cu")
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{res.stdout}\n{res.stderr}")
    return res.stderr


def build(verbose: bool = False, jobs: int = 0, ptxas_verbose: bool = False) -> str:
    """Compiles the library if anything changed and returns its path."""
    os.makedirs(BUILD_DIR, exist_ok=True)
    srcs = _sources()
    hdr_time = _newest(_headers())
    extra = ["-Xptxas", "-v"] if ptxas_verbose else []
    todo = []
    objs = []
    for s in srcs:
        o = os.path.join(BUILD_DIR, os.path.basename(s) + ".o")
        objs.append(o)
        if ptxas_verbose or not os.path.exists(o) or os.path.getmtime(o) < max(os.path.getmtime(s), hdr_time):
            todo.append((s, o))
    if todo:
        workers = jobs or min(len(todo), os.cpu_count() or 4)
        with cf.ThreadPoolExecutor(max_workers=workers) as ex:
            futs = {ex.submit(_compile, s, o, extra, verbose): s for s, o in todo}
            for f in cf.as_completed(futs):
                log = f.result()
                if ptxas_verbose and log:
                    print(f"== {os.path.basename(futs[f])}\n{log}", flush=True)
    if todo or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < _newest(objs):
        tmp = LIB_PATH + ".tmp"
        cmd = [nvcc_path(), *ARCH_FLAGS, "-shared", "-o", tmp, *objs, "-lpthread"]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, ptxas_verbose="--ptxas" in sys.argv))
