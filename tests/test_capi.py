"""CPU checks of the C ABI: the library loads, exports every function include/*.h declares, and the
host-side argument checks reject bad calls before any device work (no GPU needed)."""
import ctypes
import re
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent


def declared_functions():
    names = []
    for header in (REPO / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
        names += re.findall(r"^\s*(?:const\s+)?[A-Za-z_][A-Za-z0-9_]*\s*\*?\s*(hds_[a-z0-9_]+)\s*\(", text, flags=re.M)
    return sorted(set(names))


def test_header_declares_the_entry_points():
    names = declared_functions()
    for required in ("hds_project_forward", "hds_project_backward", "hds_eval_sh_forward", "hds_eval_sh_backward_adam",
                     "hds_rasterize_prepare", "hds_rasterize_sort", "hds_render_forward", "hds_render_backward",
                     "hds_render_features_forward", "hds_render_features_backward", "hds_ssim_forward",
                     "hds_ssim_backward"):
        assert required in names


def test_library_exports_every_declared_symbol():
    from hds_b200 import native

    for name in declared_functions():
        assert hasattr(native.lib, name), f"{name} declared in include/ but not exported"
        assert name in native.SIGNATURES, f"{name} has no ctypes signature in native.py"


def test_abi_version_and_scratch_queries():
    from hds_b200 import native

    assert native.lib.hds_abi_version() == native.ABI_VERSION
    small = native.lib.hds_rasterize_prepare_scratch_bytes(10)
    big = native.lib.hds_rasterize_prepare_scratch_bytes(1_000_000)
    assert 0 < small < big and big % 256 == 0
    # 12 bytes per pair (two tile-key buffers, one value buffer) and 32 per gaussian (depth sort).
    assert native.lib.hds_rasterize_sort_scratch_bytes(10, 2_000_000, 979, 546) > 2_000_000 * 12
    assert native.lib.hds_rasterize_sort_scratch_bytes(1_000_000, 2_000_000, 979, 546) > 1_000_000 * 32 + 2_000_000 * 12


def test_bad_arguments_are_rejected_on_the_host():
    from hds_b200 import native

    rc = native.lib.hds_render_features_forward(10, 24, 16, 16, 0, None, None, None, None, None, None, None, None, None,
                                                None, None, None)
    assert rc == 2 and b"32, 64, 128, 256 or 512" in native.lib.hds_last_error()
    rc = native.lib.hds_render_features_backward(10, 256, 32, 16, 16, 0, *([None] * 14))
    assert rc == 2 and b"no feature backward for 256 channels in slices of 32" in native.lib.hds_last_error()
    rc = native.lib.hds_eval_sh_forward(10, 4, None, None, None, None, None, None)
    assert rc == 1 and b"degree" in native.lib.hds_last_error()
    out = ctypes.c_int64(0)
    rc = native.lib.hds_rasterize_prepare(10, *([None] * 6), 16, 16, 0, None, None, None, 0, ctypes.byref(out), None)
    assert rc == 4 and b"scratch" in native.lib.hds_last_error()
    with pytest.raises(RuntimeError, match="scratch"):
        native.check(rc)


def test_new_entry_points_reject_bad_arguments_on_the_host():
    """The view-direction SH, the SH accumulate and the raw-parameter projection validate their
    arguments before touching the device (no GPU needed)."""
    from hds_b200 import native

    lib = native.lib
    assert lib.hds_eval_sh_forward_view(10, 3, *([None] * 6), None) == 1
    assert b"camera_center" in lib.hds_last_error()
    assert lib.hds_eval_sh_backward_view(10, 3, *([None] * 9), 0, None) == 1
    assert b"camera_center" in lib.hds_last_error()
    assert lib.hds_eval_sh_forward_view(10, 5, *([None] * 6), None) == 1
    assert b"degree" in lib.hds_last_error()
    assert lib.hds_eval_sh_backward_accumulate(-1, 3, *([None] * 8), None) == 1
    assert b"n must be" in lib.hds_last_error()
    # quats 4 bytes off 16-byte alignment
    assert lib.hds_project_forward_raw(10, None, None, 4, None, None, 1.0, 1.0, 0.0, 0.0, 16, 16, 0.2, 0.3, 1.3,
                                       None, None, None, None, None, None) == 1
    assert b"16-byte" in lib.hds_last_error()
    assert lib.hds_project_backward_raw(10, *([None] * 8), 1.0, 1.0, 0.0, 0.0, 0, 16, 0.2, 0.3, 1.3,
                                        *([None] * 4), 0, None) == 1
    assert b"bad sizes" in lib.hds_last_error()
    # Zero gaussians is a valid empty call.
    assert lib.hds_project_forward_raw(0, None, None, None, None, None, 1.0, 1.0, 0.0, 0.0, 16, 16, 0.2, 0.3, 1.3,
                                       None, None, None, None, None, None) == 0


def test_adam_step_rejects_bad_tables_on_the_host():
    """hds_adam_step checks its segment table before any device work (no GPU needed); an empty
    buffer with a valid table is a no-op."""
    from hds_b200 import native

    lib = native.lib
    ends = (ctypes.c_int64 * 2)(5, 10)
    lrs = (ctypes.c_float * 2)(0.1, 0.2)
    args = (0.9, 0.999, 0.1, 0.001, 1e-15, None)
    assert lib.hds_adam_step(10, None, None, None, None, 0, ends, lrs, 1.0, *args) == 1
    assert b"segments" in lib.hds_last_error()
    assert lib.hds_adam_step(10, None, None, None, None, 17, ends, lrs, 1.0, *args) == 1
    assert lib.hds_adam_step(12, None, None, None, None, 2, ends, lrs, 1.0, *args) == 1
    assert b"not at n" in lib.hds_last_error()
    assert lib.hds_adam_step(10, None, None, None, None, 2, ends, lrs, 0.0, *args) == 1
    assert b"count from 1" in lib.hds_last_error()
    back = (ctypes.c_int64 * 2)(6, 5)
    assert lib.hds_adam_step(5, None, None, None, None, 2, back, lrs, 1.0, *args) == 1
    zero = (ctypes.c_int64 * 1)(0)
    assert lib.hds_adam_step(0, None, None, None, None, 1, zero, lrs, 1.0, *args) == 0


def test_densify_entry_points_reject_bad_arguments_on_the_host():
    from hds_b200 import native

    lib = native.lib
    widths = (ctypes.c_int * 2)(3, 3)
    assert lib.hds_densify_apply(10, 5, 0, widths, 0, 1, 1.6, *([None] * 10)) == 1
    assert b"segments" in lib.hds_last_error()
    assert lib.hds_densify_apply(10, 5, 2, widths, 0, 1, 0.0, *([None] * 10)) == 1
    bad = (ctypes.c_int * 2)(4, 3)
    assert lib.hds_densify_apply(10, 5, 2, bad, 0, 1, 1.6, *([None] * 10)) == 1
    assert b"means segment" in lib.hds_last_error()
    assert lib.hds_densify_apply(10, 0, 2, widths, 0, 1, 1.6, *([None] * 10)) == 0
    assert lib.hds_densify_stats(-1, None, None, 16, 16, None, None, None, None) == 1
