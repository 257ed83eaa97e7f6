"""Build libb200gemm.so (the C-ABI library) and the per-experiment executables.

Every CUDA translation unit is compiled for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``), the B200 counterpart of the
reference's ``-gencode=arch=compute_90a,code=sm_90a`` (CMakeLists.txt:21).
Objects go to ``hopper-lab_b200/_build/``; the shared library to
``hopper-lab_b200/lib/`` (in-tree, so it travels with the repository snapshot).

Executables (one per reference experiment) go to ``hopper-lab_b200/bin/``.

Usage: python hopper-lab_b200/build.py [--force] [-j N] [--out DIR]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "lib"
BIN = PKG / "bin"

NVCC = os.environ.get("NVCC", shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVFLAGS = ARCH + [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC",
    f"-I{ROOT / 'include'}",
    f"-I{CSRC}",
]

LIB_SOURCES = ["b200gemm.cu", "inst_f16.cu", "inst_bf16.cu", "inst_e4m3.cu", "quant.cu", "noalloc.cu"]
HEADERS = ["sm100_ptx.cuh", "gemm_sm100.cuh", "gemm_launch.cuh", "gemm_internal.h"]


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.exists() and d.stat().st_mtime > t for d in deps)


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {cmd[-1]}")


def _headers() -> list[Path]:
    return [CSRC / h for h in HEADERS] + [ROOT / "include" / "b200gemm.h"]


def build_library(force: bool = False, jobs: int = 8, out: Path | None = None) -> Path:
    """lib/libb200gemm.so, or <out>/libb200gemm.so (objects in <out>/_build) for a second
    build with other compile-time options (nvcc reads extra ones from NVCC_APPEND_FLAGS)."""
    build = BUILD if out is None else out / "_build"
    lib = LIB if out is None else out
    build.mkdir(parents=True, exist_ok=True)
    lib.mkdir(parents=True, exist_ok=True)
    objs = []
    todo = []
    for src in LIB_SOURCES:
        s = CSRC / src
        o = build / (s.stem + ".o")
        objs.append(o)
        if force or _stale(o, [s] + _headers()):
            todo.append([NVCC, *NVFLAGS, "-c", str(s), "-o", str(o)])
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        list(ex.map(_run, todo))
    so = lib / "libb200gemm.so"
    if force or todo or _stale(so, objs):
        _run([NVCC, *ARCH, "-shared", "-cudart", "static", "-o", str(so), *map(str, objs)])
    return so


EXPERIMENTS = {
    # executable: extra link libraries
    "gemm_ws": [],
    "gemm_cluster": [],
    "gemm_fp8": [],
    "gemm_persistent": [],
    "peak_tcgen05": [],
    "cublaslt_ref": ["-lcublasLt"],
    "gemm_multi_gpu": ["-lnccl"],
    "umma_desc_sweep": [],
}


def build_experiments(force: bool = False, jobs: int = 8) -> list[Path]:
    """One executable per experiment (hopper-lab_b200/experiments/*.cu), linked
    against lib/libb200gemm.so with an $ORIGIN-relative rpath."""
    BIN.mkdir(exist_ok=True)
    exp = PKG / "experiments"
    so = LIB / "libb200gemm.so"
    deps_common = [exp / "exp_common.h", so] + _headers() + sorted((ROOT / "include" / "common").glob("*.h"))
    todo, outs = [], []
    for name, libs in EXPERIMENTS.items():
        src = exp / f"{name}.cu"
        out = BIN / name
        outs.append(out)
        if force or _stale(out, [src] + deps_common):
            todo.append([NVCC, *[f for f in NVFLAGS if f != "-std=c++17"], "-std=c++20", f"-I{exp}",
                         str(src), "-o", str(out), f"-L{LIB}", "-lb200gemm", *libs,
                         "-Xlinker", "-rpath", "-Xlinker", "$ORIGIN/../lib"])
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        list(ex.map(_run, todo))
    return outs


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=8)
    ap.add_argument("--out", type=Path, default=None,
                    help="build only the library, into this directory (e.g. an experimental build: "
                         "NVCC_APPEND_FLAGS=-DB200_EXPERIMENT_ENV)")
    a = ap.parse_args()
    so = build_library(force=a.force, jobs=a.j, out=a.out)
    print(so)
    if a.out is not None:
        return
    for b in build_experiments(force=a.force, jobs=a.j):
        print(b)


if __name__ == "__main__":
    main()
