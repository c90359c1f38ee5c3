"""Build ``libngdn2.so`` (the C-ABI library) in-tree with nvcc for sm_100a.

    python -m nested_recurrent_memory_b200.build [--force] [--verbose]

Compiles every ``csrc/*.cu`` to an object and links a shared library next
to this file. Rebuilds only when a source or header is newer than the
library (or with ``--force``).
"""

from __future__ import annotations

import argparse
import os
import pathlib
import shutil
import subprocess
import sys

HERE = pathlib.Path(__file__).resolve().parent
CSRC = HERE / "csrc"
INCLUDE = HERE.parent / "include"
LIB = HERE / "libngdn2.so"
BUILD_DIR = HERE.parent / "_build"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr", "-I", str(INCLUDE),
]


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = pathlib.Path(cuda_home) / "bin" / "nvcc"
    if cand.exists():
        return str(cand)
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found (set CUDA_HOME)")
    return found


def _flags() -> list[str]:
    return list(NVCC_FLAGS)


def sources() -> list[pathlib.Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    return any(p.stat().st_mtime > t for p in deps)


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> pathlib.Path:
    """Compile and link; returns the library path."""
    if not force and not _stale():
        return LIB
    nvcc = _nvcc()
    BUILD_DIR.mkdir(exist_ok=True)
    objs = []
    for src in sources():
        obj = BUILD_DIR / (src.stem + ".o")
        cmd = [nvcc, *ARCH, *_flags(), "-c", str(src), "-o", str(obj)]
        if ptxas_verbose:
            cmd += ["-Xptxas", "-v"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        objs.append(str(obj))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH, "-shared", "-cudart", "shared", "-o", str(tmp), *objs]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true")
    args = ap.parse_args(argv)
    print(build(force=args.force, verbose=args.verbose, ptxas_verbose=args.ptxas_verbose))
    return 0


if __name__ == "__main__":
    sys.exit(main())
