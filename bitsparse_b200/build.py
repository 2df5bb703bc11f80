"""Build libbitsparse_b200.so (sm_100a) in-tree with nvcc.

    python -m bitsparse_b200.build            # build if sources are newer
    python -m bitsparse_b200.build --force    # always rebuild

The library is a plain C-ABI shared object (declarations in
include/bitsparse.h); it links only the CUDA runtime.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libbitsparse_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def sources():
    return sorted(CSRC.glob("*.cu"))


def _nvcc():
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put CUDA's bin on PATH")


def needs_build() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = sources() + list(CSRC.glob("*.cuh")) + [ROOT / "include" / "bitsparse.h"]
    return any(p.stat().st_mtime > t for p in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not needs_build():
        return LIB
    objs = []
    build_dir = PKG / "_build"
    build_dir.mkdir(exist_ok=True)
    nvcc = _nvcc()
    common = [nvcc, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
              "--expt-relaxed-constexpr", "-I", str(ROOT / "include")]
    if verbose:
        common += ["-Xptxas", "-v"]
    common += os.environ.get("BS_NVCC_EXTRA", "").split()
    from concurrent.futures import ThreadPoolExecutor

    def compile_one(src):
        obj = build_dir / (src.stem + ".o")
        subprocess.run(common + ["-c", str(src), "-o", str(obj)], check=True)
        return str(obj)

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(compile_one, sources()))
    tmp = LIB.with_suffix(".so.tmp")
    subprocess.run([nvcc, *ARCH, "-shared", "-o", str(tmp), *objs, "-lcudart"], check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
    sys.exit(0)
