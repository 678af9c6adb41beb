"""Builds the reference's own CUDA extension into oracle/_ref/ (a checker, not part of the product).

The reference JIT-builds gaussian_splatting/rasterizer/{forward,backward,features,sh,projection,
ssim}.cu + bindings.cpp with torch.utils.cpp_extension (rasterizer/__init__.py:15-54, flags
-O3 --use_fast_math -std=c++17 -lineinfo).  This recipe compiles the same sources, where they lie in
the reference checkout, with the same flags for sm_100a, and writes only into oracle/_ref/.  The
built module (gaussian_rasterizer_ref*.so) travels with the repository snapshot; the GPU tests load
it to compare this library with the reference itself on identical inputs.

    python oracle/build_ref.py [/path/to/reference]
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
SOURCES = ["forward.cu", "backward.cu", "features.cu", "sh.cu", "projection.cu", "ssim.cu", "bindings.cpp"]
NAME = "gaussian_rasterizer_ref"


def built() -> Path | None:
    hits = sorted(OUT.glob(f"{NAME}*.so"))
    return hits[0] if hits else None


def build(reference: str | os.PathLike = "/root/reference") -> Path:
    src = Path(reference) / "gaussian_splatting" / "rasterizer"
    if not src.exists():
        raise FileNotFoundError(f"no reference rasterizer sources under {src}")
    if built() is not None:
        return built()
    OUT.mkdir(exist_ok=True)
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    from torch.utils.cpp_extension import load

    load(name=NAME, sources=[str(src / s) for s in SOURCES], build_directory=str(OUT),
         extra_cuda_cflags=["-O3", "--use_fast_math", "-std=c++17", "-lineinfo"],
         extra_cflags=["-O3", "-std=c++17"], verbose=False)
    return built()


def load_built():
    """Imports the built reference module (no compiler involved)."""
    import importlib.util

    import torch  # noqa: F401  (the extension links against torch)

    path = built()
    if path is None:
        raise FileNotFoundError("oracle/_ref holds no built reference extension; run oracle/build_ref.py")
    spec = importlib.util.spec_from_file_location(NAME, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    print(build(sys.argv[1] if len(sys.argv) > 1 else "/root/reference"))
