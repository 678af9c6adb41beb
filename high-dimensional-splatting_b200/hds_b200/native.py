"""ctypes binding of libhds_b200.so (include/hds_b200.h).

The library is the only compute path.  It is mapped on the first call of any entry point (so that
importing the package, e.g. for its scene generators, loads no native code); if it is missing or
fails to load, that first call raises ImportError instead of falling back to anything else.  Build
it with ``python high-dimensional-splatting_b200/build.py``.
"""
from __future__ import annotations

import ctypes
from ctypes import c_float, c_int, c_int64, c_size_t, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libhds_b200.so"
ABI_VERSION = 3

P = c_void_p  # device pointer
S = c_void_p  # cudaStream_t

# name -> argtypes (every entry point returns int status, except where restype is given below)
SIGNATURES = {
    "hds_project_forward": [c_int, P, P, P, P, P, c_float, c_float, c_float, c_float, c_int, c_int, c_float, c_float,
                            c_float, P, P, P, P, S],
    "hds_project_backward": [c_int, P, P, P, P, P, P, c_float, c_float, c_float, c_float, c_int, c_int, c_float,
                             c_float, c_float, P, P, P, S],
    "hds_project_forward_raw": [c_int, P, P, P, P, P, c_float, c_float, c_float, c_float, c_int, c_int, c_float,
                                c_float, c_float, P, P, P, P, P, S],
    "hds_project_backward_raw": [c_int, P, P, P, P, P, P, P, P, c_float, c_float, c_float, c_float, c_int, c_int,
                                 c_float, c_float, c_float, P, P, P, P, c_int, S],
    "hds_eval_sh_forward": [c_int, c_int, P, P, P, P, P, S],
    "hds_eval_sh_backward_adam": [c_int, c_int, P, P, P, P, P, P, P, P, P, P, P, c_float, c_float, c_float, c_float,
                                  c_float, c_float, c_float, P, S],
    "hds_eval_sh_backward": [c_int, c_int, P, P, P, P, P, P, P, P, S],
    "hds_eval_sh_backward_accumulate": [c_int, c_int, P, P, P, P, P, P, P, P, S],
    "hds_eval_sh_forward_view": [c_int, c_int, P, P, P, P, P, P, S],
    "hds_eval_sh_backward_view": [c_int, c_int, P, P, P, P, P, P, P, P, P, c_int, S],
    "hds_rasterize_prepare_scratch_bytes": [c_int],
    "hds_rasterize_prepare": [c_int, P, P, P, P, P, P, c_int, c_int, c_int, P, P, P, c_size_t, ctypes.POINTER(c_int64),
                              S],
    "hds_rasterize_sort_scratch_bytes": [c_int, c_int64, c_int, c_int],
    "hds_rasterize_sort": [c_int, c_int64, c_int, c_int, P, P, c_size_t, P, P, P, S],
    "hds_render_forward": [c_int, c_int, c_int, P, P, P, P, P, P, P, P, P, S],
    "hds_render_backward": [c_int, c_int, c_int, c_int, P, P, P, P, P, P, P, P, P, P, P, P, P, S],
    "hds_render_features_forward": [c_int, c_int, c_int, c_int, c_int, P, P, P, P, P, P, P, P, P, P, P, S],
    "hds_render_features_backward": [c_int, c_int, c_int, c_int, c_int, c_int, P, P, P, P, P, P, P, P, P, P, P, P, P,
                                     S],
    "hds_render_features_backward_accumulate": [c_int, c_int, c_int, c_int, c_int, c_int, P, P, P, P, P, P, P, P, P, P,
                                                P, P, P, S],
    "hds_render_backward_fused": [c_int, c_int, c_int, c_int, c_int, P, P, P, P, P, P, P, P, P, P, P, P, P, P, P, P,
                                  c_int, P, c_size_t, S],
    "hds_backward_workspace_bytes": [c_int64, c_int, c_int],
    "hds_ssim_forward": [c_int, c_int, P, P, P, P, P, P, S],
    "hds_ssim_backward": [c_int, c_int, P, P, P, P, P, P, P, S],
    "hds_adam_step": [c_int64, P, P, P, P, c_int, ctypes.POINTER(c_int64), ctypes.POINTER(c_float), c_float, c_float,
                      c_float, c_float, c_float, c_float, S],
    "hds_densify_stats": [c_int, P, P, c_int, c_int, P, P, P, S],
    "hds_densify_apply": [c_int, c_int, c_int, ctypes.POINTER(c_int), c_int, c_int, c_float, P, P, P, P, P, P, P, P,
                          P, S],
    "hds_device_status": [ctypes.POINTER(c_int), S],
    "hds_rasterize_bin_noalloc": [c_int, P, P, P, P, P, P, c_int, c_int, P, P, P, c_int64, P,
                                  ctypes.POINTER(c_int64), S],
    "hds_last_error": [],
    "hds_abi_version": [],
    "hds_launch_count": [],
}
RESTYPES = {
    "hds_rasterize_prepare_scratch_bytes": c_size_t,
    "hds_rasterize_sort_scratch_bytes": c_size_t,
    "hds_backward_workspace_bytes": c_size_t,
    "hds_last_error": ctypes.c_char_p,
    "hds_launch_count": ctypes.c_ulonglong,
}


def _load() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(f"{LIB_PATH} is not built; run python high-dimensional-splatting_b200/build.py")
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, args in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = RESTYPES.get(name, c_int)
    if lib.hds_abi_version() != ABI_VERSION:
        raise ImportError(f"{LIB_PATH} has ABI {lib.hds_abi_version()}, expected {ABI_VERSION}; rebuild it")
    return lib


class _LazyLib:
    """Stand-in for the ctypes library that loads it on first attribute access.  Attributes set on
    it (a wrapper installed by a profiler, say) take precedence over the library's own symbols."""

    def __init__(self):
        self._cdll = None

    def loaded(self) -> bool:
        return self._cdll is not None

    def __getattr__(self, name):
        if name.startswith("__"):
            raise AttributeError(name)
        if self._cdll is None:
            self._cdll = _load()
        return getattr(self._cdll, name)


lib = _LazyLib()


def check(rc: int) -> None:
    """Raises RuntimeError with the library's message for a non-zero status."""
    if rc != 0:
        raise RuntimeError(lib.hds_last_error().decode() or f"libhds_b200 call failed with status {rc}")


def ptr(t) -> int | None:
    """Device address of a tensor (None for None)."""
    return None if t is None else t.data_ptr()


def stream_of(device) -> int:
    import torch

    return torch.cuda.current_stream(device).cuda_stream


def device_status(device=None) -> int:
    """Reads and clears the device-side failure word (0 = no bounded wait ran out)."""
    out = c_int(0)
    check(lib.hds_device_status(ctypes.byref(out), stream_of(device)))
    return out.value
