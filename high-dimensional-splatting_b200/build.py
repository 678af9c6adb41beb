"""Builds libhds_b200.so (all CUDA kernels + the C ABI) for sm_100a with nvcc.

    python high-dimensional-splatting_b200/build.py [--force]

Objects go to high-dimensional-splatting_b200/_build/ and the library to
high-dimensional-splatting_b200/hds_b200/libhds_b200.so, both in-tree so the built library travels
with the repository snapshot.  Rebuilds only what changed (object older than its source or any
header).  nvcc cross-compiles, so no GPU is needed.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
from pathlib import Path

ROOT = Path(__file__).resolve().parent
CSRC = ROOT / "csrc"
INCLUDE = ROOT.parent / "include"
BUILD = ROOT / "_build"
LIB = ROOT / "hds_b200" / "libhds_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
# --fmad=false: a*b+c rounds twice unless the source writes fmaf(); with IEEE div/sqrt (no fast
# math) the forward kernels round exactly like the CPU oracle that checks them.
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--fmad=false", "-Xcompiler", "-fPIC", "-Xptxas", "-warn-spills",
              f"-I{INCLUDE}", f"-I{CSRC}"]


def nvcc() -> str:
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = Path(cuda) / "bin" / "nvcc"
    return str(path) if path.exists() else (shutil.which("nvcc") or "nvcc")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def stale(obj: Path, src: Path) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(dep.stat().st_mtime > t for dep in [src, *headers(), Path(__file__)])


def compile_one(src: Path, verbose: bool) -> Path:
    obj = BUILD / (src.stem + ".o")
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
    if res.stderr.strip() and verbose:
        print(res.stderr, flush=True)
    return obj


def build(force: bool = False, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    srcs = sources()
    todo = [s for s in srcs if force or stale(BUILD / (s.stem + ".o"), s)]
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as pool:
        list(pool.map(lambda s: compile_one(s, verbose), todo))
    objs = [BUILD / (s.stem + ".o") for s in srcs]
    if force or todo or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(f".{os.getpid()}.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs)]
        subprocess.run(cmd, check=True)
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    args = ap.parse_args()
    print(build(args.force, args.verbose))
