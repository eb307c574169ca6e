"""Build the in-tree CUDA library ``edgeexpert_b200/libtfcuda.so`` for sm_100a.

Each ``csrc/*.cu`` file is compiled separately (in parallel) with
``-gencode arch=compute_100a,code=sm_100a`` and linked into one shared
library whose exported symbols are the C ABI of ``include/tfcuda.h``.
Usage: ``python -m edgeexpert_b200.build [--force] [--verbose]``.
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
OBJ = PKG / "_build"
LIB = PKG / "libtfcuda.so"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-fvisibility=hidden",
    "-I", str(ROOT / "include"),
    "-I", str(CSRC),
]
LINK_LIBS = ["--cudart", "static", "-lrt", "-lpthread", "-ldl"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libtfcuda.so")


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _deps_mtime() -> float:
    files = list(CSRC.glob("*")) + list((ROOT / "include").glob("*.h"))
    return max(f.stat().st_mtime for f in files)


def _compile(src: Path, verbose: bool, extra: list[str]) -> Path:
    out = OBJ / (src.stem + ".o")
    cmd = [_nvcc(), *NVCC_FLAGS, *extra, "-c", str(src), "-o", str(out)]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    if verbose and res.stderr.strip():
        print(res.stderr, flush=True)
    return out


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> Path:
    """Compile every csrc/*.cu for sm_100a and link libtfcuda.so (in-tree)."""
    extra = extra or []
    if LIB.exists() and not force and LIB.stat().st_mtime >= _deps_mtime():
        return LIB
    OBJ.mkdir(exist_ok=True)
    srcs = _sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose, extra), srcs))
    cmd = [_nvcc(), "-shared", "-gencode", "arch=compute_100a,code=sm_100a", *map(str, objs),
           "-o", str(LIB) + ".tmp", *LINK_LIBS]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(str(LIB) + ".tmp", LIB)
    return LIB


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true", help="pass -Xptxas -v (registers/spills)")
    a = ap.parse_args(argv)
    extra = ["-Xptxas", "-v"] if a.ptxas_verbose else []
    print(build(force=a.force or a.ptxas_verbose, verbose=a.verbose or a.ptxas_verbose, extra=extra))
    return 0


if __name__ == "__main__":
    sys.exit(main())
