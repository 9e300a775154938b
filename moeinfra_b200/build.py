"""Build the sm_100a CUDA library ``moeinfra_b200/_lib/libmoe_b200.so`` in-tree.

``python -m moeinfra_b200.build`` (or ``__graft_entry__.build()``) compiles
every ``csrc/*.cu`` with nvcc for ``sm_100a`` only and links one shared
library exposing the C ABI declared in ``include/moe_b200.h``.  Objects are
rebuilt only when a source or header is newer than the object.
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
OUT_DIR = PKG / "_lib"
OBJ_DIR = ROOT / "_build" / "obj"
LIB = OUT_DIR / "libmoe_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-O2",
    "--expt-relaxed-constexpr", "-I", str(ROOT / "include"),
]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build moeinfra_b200")
    return cand


def _headers() -> list[Path]:
    return list(CSRC.glob("*.cuh")) + list((ROOT / "include").glob("*.h"))


def _stale(obj: Path, src: Path, deps: list[Path]) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(p.stat().st_mtime > t for p in [src, *deps])


def build(verbose: bool = False, extra_flags: list[str] | None = None) -> Path:
    nvcc = _nvcc()
    OUT_DIR.mkdir(parents=True, exist_ok=True)
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    deps = _headers()
    flags = NVCC_FLAGS + list(extra_flags or [])

    def compile_one(src: Path) -> Path:
        obj = OBJ_DIR / (src.stem + ".o")
        if _stale(obj, src, deps) or extra_flags:
            cmd = [nvcc, *flags, "-c", str(src), "-o", str(obj)]
            if verbose:
                print(" ".join(cmd))
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode != 0:
                raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
            if verbose and r.stderr.strip():
                print(r.stderr)
        return obj

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(compile_one, srcs))
    if not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        cmd = [nvcc, *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lcudart"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    v = "-v" in sys.argv
    extra = ["-Xptxas", "-v"] if "--ptxas" in sys.argv else None
    print(build(verbose=v, extra_flags=extra))
