"""Build the sm_100a kernel library ``lunara_b200/liblunara_b200.so`` in-tree.

Every ``csrc/*.cu`` translation unit is compiled by nvcc for
``-gencode arch=compute_100a,code=sm_100a`` only (no PTX for other targets, no
runtime dispatch) and linked into one shared library with the CUDA runtime
statically linked. The library is loaded with ctypes by
``lunara_b200.runtime._lib``; it does not link libcuda (the tensor-map encoder
is resolved through the runtime's driver entry point).

Usage: ``python -m lunara_b200.build [--verbose-ptxas] [--force]``
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
BUILD = PKG / "_build"
LIB = PKG / "liblunara_b200.so"
INCLUDE = PKG.parent / "include"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-O3", "-Xcompiler", "-Wall",
    "-I", str(INCLUDE),
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the sm_100a kernel library cannot be built")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _headers_mtime() -> float:
    hs = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def _compile(src: Path, verbose_ptxas: bool) -> tuple[Path, str]:
    obj = BUILD / (src.stem + ".o")
    cmd = [nvcc(), *ARCH_FLAGS, *COMMON_FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose_ptxas:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    return obj, r.stdout + r.stderr


def build(force: bool = False, verbose_ptxas: bool = False, jobs: int | None = None) -> Path:
    """Compile and link the library if any source is newer than it. Returns its path."""
    BUILD.mkdir(exist_ok=True)
    srcs = sources()
    newest = max([s.stat().st_mtime for s in srcs] + [_headers_mtime(), Path(__file__).stat().st_mtime])
    if not force and LIB.exists() and LIB.stat().st_mtime >= newest:
        return LIB
    jobs = jobs or min(len(srcs), os.cpu_count() or 4)
    logs = []
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        futs = [ex.submit(_compile, s, verbose_ptxas) for s in srcs]
        objs = []
        for f in futs:
            obj, log = f.result()
            objs.append(obj)
            logs.append(log)
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH_FLAGS, "-shared", "-Xcompiler", "-fPIC", "-cudart", "static",
           *map(str, objs), "-o", str(tmp)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    if verbose_ptxas:
        sys.stdout.write("".join(logs))
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose-ptxas", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose_ptxas=args.verbose_ptxas))


if __name__ == "__main__":
    main()
