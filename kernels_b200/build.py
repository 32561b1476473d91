"""Builds libcuda-graft.so (sm_100a) in-tree with nvcc.

    python -m kernels_b200.build            # build if sources are newer
    python -m kernels_b200.build --force    # always rebuild
    python -m kernels_b200.build --ptxas-v  # print per-kernel registers/spills

The library is plain CUDA C++ with an extern "C" ABI (include/cuda_graft.h): it
links the static CUDA runtime and the system NCCL, and never links PyTorch.
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIBDIR = PKG / "lib"
LIB = LIBDIR / "libcuda-graft.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O2",
    "--expt-relaxed-constexpr", "-Xfatbin", "-compress-all",
]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or "/usr/local/cuda/bin/nvcc"
    return cand if Path(cand).exists() else "nvcc"


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in sources() + headers() + [Path(__file__)])


def build(force: bool = False, ptxas_v: bool = False, verbose: bool = False) -> Path:
    if not force and not ptxas_v and up_to_date():
        return LIB
    LIBDIR.mkdir(exist_ok=True)
    objdir = LIBDIR / "obj"
    objdir.mkdir(exist_ok=True)

    def compile_one(src: Path) -> tuple[Path, subprocess.CompletedProcess]:
        obj = objdir / (src.stem + ".o")
        cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-I", str(INCLUDE), "-I", str(CSRC),
               "-c", str(src), "-o", str(obj)]
        if ptxas_v:
            cmd += ["-Xptxas", "-v"]
        if verbose:
            print(" ".join(cmd), flush=True)
        return obj, subprocess.run(cmd, capture_output=True, text=True)

    # translation units compile independently: one nvcc per source, in parallel
    with ThreadPoolExecutor(max_workers=min(len(sources()), os.cpu_count() or 1)) as ex:
        results = list(ex.map(compile_one, sources()))
    objs = []
    for src, (obj, r) in zip(sources(), results):
        if r.returncode != 0 or ptxas_v:
            sys.stderr.write(r.stdout + r.stderr)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}")
        objs.append(str(obj))
    tmp = LIB.with_suffix(".so.tmp")
    link = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *objs, "-lnccl", "-lpthread"]
    if verbose:
        print(" ".join(link), flush=True)
    r = subprocess.run(link, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("link of libcuda-graft.so failed")
    os.replace(tmp, LIB)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, ptxas_v=a.ptxas_v, verbose=a.verbose))


if __name__ == "__main__":
    main()
