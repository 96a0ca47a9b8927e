"""Build the sm_100a shared library ``libmvr_b200.so`` in-tree.

Compiles every ``csrc/*.cu`` / ``csrc/*.cpp`` with nvcc for sm_100a and
links them, with a static CUDA runtime, into
``ir_multivector_retrieval_b200/libmvr_b200.so``. The library's ABI is
``include/mvr.h`` (plain C, no torch types).

Floating point: ``-fmad=false`` and no fast-math, so device arithmetic is
IEEE round-to-nearest without contraction (the reference's strict float
mode); host code is built with ``-ffp-contract=off`` for the same reason.

Usage: ``python -m ir_multivector_retrieval_b200.build [--force] [--verbose]``
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD = PKG.parent / "_build" / "mvr_b200"
LIB = PKG / "libmvr_b200.so"
INCLUDE = PKG.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nccl_include() -> str:
    """Header directory of the NCCL that PyTorch ships (the library itself is
    loaded at run time), else the system one."""
    try:
        import nvidia.nccl as nn  # noqa: PLC0415

        for p in nn.__path__:
            inc = Path(p) / "include"
            if (inc / "nccl.h").exists():
                return str(inc)
    except Exception:
        pass
    return "/usr/include"


NVCC_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-fmad=false",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC,-ffp-contract=off,-O2",
    f"-I{INCLUDE}",
    f"-I{nccl_include()}",
]


def nvcc_path() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the B200 library cannot be built")
    return cand


def sources() -> list[Path]:
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cpp")))


def headers() -> list[Path]:
    return sorted(list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h")))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    nvcc = nvcc_path()
    BUILD.mkdir(parents=True, exist_ok=True)
    hdrs = headers()
    objs = []
    for src in sources():
        obj = BUILD / (src.name + ".o")
        objs.append(obj)
        if force or _stale(obj, [src, *hdrs, Path(__file__)]):
            cmd = [nvcc, *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
            if ptxas_verbose and src.suffix == ".cu":
                cmd.insert(1, "-Xptxas=-v")
            if verbose:
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)
    if force or _stale(LIB, objs):
        cmd = [nvcc, *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lpthread", "-ldl"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true")
    a = ap.parse_args(argv)
    lib = build(force=a.force, verbose=a.verbose, ptxas_verbose=a.ptxas_verbose)
    print(lib)
    return 0


if __name__ == "__main__":
    sys.exit(main())
