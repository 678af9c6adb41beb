"""The allocation-free binning entry point (hds_rasterize_bin_noalloc).

Some callers cannot allocate device memory where they bin a frame.  Examples: a renderer inside an
application whose GPU memory belongs to another allocator, a real-time loop that must not call
cudaMalloc (it can synchronise the device), or an FFI host that only hands over finished buffers.
For them the library keeps the binning scratch in a fixed 64 MiB device array.  This test calls that
entry point through the C ABI twice in a row, on two different scenes, and checks each result
bit-exactly (the tolerance every binning test uses) against the existing allocating path
(hds_rasterize_prepare + hds_rasterize_sort, through rasterize()).  The second call must not see the
first call's leftovers in the shared array.  It also checks that a request beyond the limits is
refused with a clear error.

This file is named so pytest collects it last.
"""
import ctypes

import numpy as np
import pytest

from scenes_np import config_scene, reference_scene

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

BACKGROUND = np.array([0.3, 0.5, 0.7], np.float32)


def cuda(*arrays):
    return [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in arrays]


def bin_noalloc(native, inputs, width, height, capacity):
    means2D, depths, radii, conics, colors, opacities = inputs
    n = means2D.shape[0]
    dev = means2D.device
    conic4 = torch.empty(n, 4, device=dev)
    color_opacity = torch.empty(n, 4, device=dev)
    values = torch.empty(max(capacity, 1), dtype=torch.int32, device=dev)
    tiles = ((width + 15) // 16) * ((height + 15) // 16)
    ranges = torch.empty(tiles, 2, dtype=torch.int32, device=dev)
    dups = ctypes.c_int64(-1)
    rc = native.lib.hds_rasterize_bin_noalloc(n, *(native.ptr(t) for t in inputs), width, height, native.ptr(conic4),
                                              native.ptr(color_opacity), native.ptr(values), capacity,
                                              native.ptr(ranges), ctypes.byref(dups),
                                              torch.cuda.current_stream().cuda_stream)
    return rc, conic4, color_opacity, values[:dups.value], ranges, dups.value


def test_no_alloc_binning_matches_the_allocating_path_on_two_calls_in_a_row():
    from hds_b200 import gaussian_rasterizer as ext
    from hds_b200 import native, scenes

    big, cam = config_scene(scenes.config1(0, n=20_000, channels=0))
    small = reference_scene(3, 3000, 17, 17)
    for inputs_np, w, h in ((big, cam.width, cam.height), (small, 17, 17)):
        inputs = cuda(*inputs_np)
        _, _, _, values, ranges, conic4, color_opacity = ext.rasterize(*inputs, cuda(BACKGROUND)[0], w, h)
        rc, g_conic4, g_co, g_values, g_ranges, dups = bin_noalloc(native, inputs, w, h, capacity=values.numel() + 7)
        assert rc == 0, native.lib.hds_last_error().decode()
        assert dups == values.numel()
        assert torch.equal(g_values, values), "sort order differs"
        assert torch.equal(g_ranges, ranges), "tile ranges differ"
        assert torch.equal(g_conic4, conic4) and torch.equal(g_co, color_opacity)


def test_no_alloc_binning_refuses_requests_beyond_its_limits():
    from hds_b200 import native, scenes

    inputs_np, cam = config_scene(scenes.config1(0, n=20_000, channels=0))
    inputs = cuda(*inputs_np)
    rc, *_ = bin_noalloc(native, inputs, cam.width, cam.height, capacity=10)
    assert rc == 5  # HDS_ERR_TOO_LARGE
    assert b"exceed values_sorted capacity" in native.lib.hds_last_error()
    huge = 5_000_000  # needs ~120 MB of prepare scratch, more than the fixed array
    z = torch.zeros(huge, 4, device="cuda")
    rc = native.lib.hds_rasterize_bin_noalloc(huge, *(native.ptr(z),) * 6, 64, 64, native.ptr(z), native.ptr(z),
                                              native.ptr(z), 1, native.ptr(z), ctypes.byref(ctypes.c_int64()),
                                              torch.cuda.current_stream().cuda_stream)
    assert rc == 5 and b"more than the fixed" in native.lib.hds_last_error()
