"""Build ``dart_cuda_b200/lib/libmat_mul.so`` from ``csrc/*.cu`` with nvcc.

sm_100a only: ``-gencode arch=compute_100a,code=sm_100a``.  The library is
built in-tree so that it travels with the source tree; nothing is installed.

    python -m dart_cuda_b200.build [--force] [-v]
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
CSRC = PKG / "csrc"
OUT_DIR = PKG / "lib"
LIB = OUT_DIR / "libmat_mul.so"
OBJ_DIR = PKG / "_build"
INCLUDE = PKG.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall", "-Xcompiler", "-Wno-unused-function",
    f"-I{INCLUDE}",
]


def nvcc() -> str:
    p = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    return p


def _sources():
    return sorted(CSRC.glob("*.cu"))


def _headers():
    return sorted(list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h")))


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


# Test-only library for the bounded-wait test (tests/test_bounded_wait_gpu.py):
# the AFT kernels and the runtime helpers built with a short wait limit and
# DC_TEST_WITHHOLD, which adds dc_test_withhold_next(); never loaded by the
# product.
WAITTEST_LIB = OUT_DIR / "libmat_mul_waittest.so"
WAITTEST_SOURCES = ("aft.cu", "dc_common.cu")
WAITTEST_DEFINES = ["-DDC_TEST_WITHHOLD", "-DDC_WAIT_NS=50000000ull"]


def _compile(src: Path, verbose: bool, extra, obj_dir: Path = OBJ_DIR) -> Path:
    obj = obj_dir / (src.stem + ".o")
    if _stale(obj, [src, *_headers()]):
        cmd = [nvcc(), *NVCC_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout, r.stderr, flush=True)
    return obj


def build(force: bool = False, verbose: bool = False, extra=()) -> Path:
    OBJ_DIR.mkdir(exist_ok=True)
    OUT_DIR.mkdir(exist_ok=True)
    srcs = _sources()
    if force:
        for o in OBJ_DIR.glob("**/*.o"):
            o.unlink()
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose, list(extra)), srcs))
    _link(LIB, objs, force, verbose)
    # the bounded-wait test library
    wdir = OBJ_DIR / "waittest"
    wdir.mkdir(exist_ok=True)
    wsrcs = [CSRC / n for n in WAITTEST_SOURCES]
    with cf.ThreadPoolExecutor(max_workers=2) as ex:
        wobjs = list(ex.map(lambda s: _compile(s, verbose, list(extra) + WAITTEST_DEFINES, wdir), wsrcs))
    _link(WAITTEST_LIB, wobjs, force, verbose)
    return LIB


def _link(lib: Path, objs, force: bool, verbose: bool):
    if force or _stale(lib, objs):
        cmd = [nvcc(), *ARCH, "--shared", "-o", str(lib), *map(str, objs), "-lcudart_static",
               "-ldl", "-lrt", "-lpthread"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print register/smem usage")
    a = ap.parse_args(argv)
    extra = ["-Xptxas", "-v"] if a.ptxas_v else []
    lib = build(force=a.force or a.ptxas_v, verbose=a.verbose or a.ptxas_v, extra=extra)
    print(lib)


if __name__ == "__main__":
    sys.exit(main())
