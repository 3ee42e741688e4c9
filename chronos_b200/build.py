"""Builds libchronos_b200.so (sm_100a only) in-tree with nvcc. Usable as `python -m chronos_b200.build`.

Every `.cu` file is compiled to its own object (in parallel, and only when it or a header changed), then the objects
are linked into the shared library. Objects live under `csrc/obj/` and are not part of the source tree.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OBJ = CSRC / "obj"
LIB = PKG / "libchronos_b200.so"
SOURCES = ("api.cu", "probe_kernels.cu", "router.cu", "plan.cu", "transform_kernels.cu", "bank_stream.cu", "bank_gemm.cu",
           "bank_fp4.cu", "healer_mma.cu", "tail.cu", "decode_fused.cu", "ep_kernels.cu", "shared_fp8.cu", "fused_healer.cu")
HEADERS = (CSRC / "common.cuh", CSRC / "fp4_mma.cuh", ROOT / "include" / "chronos_b200.h")
ARCH = ("-gencode", "arch=compute_100a,code=sm_100a")


def nvcc_path() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: set NVCC or put it on PATH")
    return cand


def _sources() -> list[Path]:
    return [CSRC / s for s in SOURCES if (CSRC / s).exists()]


def _headers() -> list[Path]:
    return [h for h in HEADERS if h.exists()]


def needs_build() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(d.stat().st_mtime > t for d in _sources() + _headers())


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not needs_build():
        return LIB
    nvcc = nvcc_path()
    OBJ.mkdir(exist_ok=True)
    hdr_time = max(h.stat().st_mtime for h in _headers())
    common = [nvcc, *ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-I", str(ROOT / "include"), "-I", str(CSRC)]
    if verbose:
        common += ["-Xptxas", "-v"]

    def compile_one(src: Path) -> Path:
        obj = OBJ / (src.stem + ".o")
        if force or verbose or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, hdr_time):
            subprocess.check_call(common + ["-c", str(src), "-o", str(obj)])
        return obj

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as pool:
        objs = list(pool.map(compile_one, _sources()))
    subprocess.check_call([nvcc, *ARCH, "-shared", "-o", str(LIB)] + [str(o) for o in objs])
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
