"""Build libdop.so (the sm_100a CUDA library behind include/dop.h) in-tree.

    python dependent-optics_b200/build.py [--force] [--ptxas-v]

Each csrc/*.cu is compiled by nvcc for sm_100a into _build/ (in parallel,
skipped when the object is newer than every source and header), then linked
into dependent-optics_b200/libdop.so with the CUDA runtime linked statically,
so the library needs only the driver at run time.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libdop.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-Xcompiler", "-Wall", "-diag-suppress", "177"]


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + [ROOT / "include" / "dop.h"]


def _stale(obj: Path, src: Path) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(p.stat().st_mtime > t for p in [src, *_headers()])


def _compile(src: Path, force: bool, ptxas_v: bool) -> Path:
    obj = BUILD / (src.stem + ".o")
    if force or _stale(obj, src):
        cmd = [NVCC, *ARCH, *FLAGS, "-I", str(ROOT / "include"), "-c", str(src), "-o", str(obj)]
        if ptxas_v:
            cmd += ["-Xptxas", "-v"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
        if ptxas_v:
            sys.stderr.write(r.stderr)
    return obj


def build(force: bool = False, ptxas_v: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    with cf.ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, ptxas_v), srcs))
    if force or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-cudart", "static"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.ptxas_v))
