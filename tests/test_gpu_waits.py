"""Failure detection of the bounded device waits, without a GPU fault.

Every wait of the library's kernels on another CTA's word (the radix sort's
look-back) or on a barrier (the blend's record ring) polls at most
ns_set_wait_limit times, then records an error bit and lets the kernel finish.
Here a wait is made to run out on purpose: ns_wait_selftest waits, with the
sort's wait code, on a device word that nothing sets. The kernel must return
(no trap, no hang), ns_read_device_status must report NS_ERR_DEVICE, and the
context must stay usable for the next render and sort.
"""
import time

import numpy as np
import pytest
import torch

from helpers import api_inputs, small_scene
from nest_b200 import _lib, raster

pytestmark = pytest.mark.gpu
P = 16


def _stream():
    return _lib.stream_handle(torch.device("cuda"))


def test_wait_that_runs_out_reports_device_error():
    lib = _lib.load()
    geom = torch.zeros(lib.ns_geometry_scratch_bytes(P), dtype=torch.uint8, device="cuda")
    assert lib.ns_read_device_status(geom.data_ptr(), P, _stream()) == _lib.NS_OK
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    prev = lib.ns_set_wait_limit(1 << 14)
    try:
        t0 = time.perf_counter()
        assert lib.ns_wait_selftest(flag.data_ptr(), geom.data_ptr(), P, _stream()) == _lib.NS_OK
        assert lib.ns_read_device_status(geom.data_ptr(), P, _stream()) == _lib.NS_ERR_DEVICE
        assert time.perf_counter() - t0 < 5.0
        # the status word was cleared by the read; a word that is set ends the wait at once
        flag.fill_(1)
        assert lib.ns_wait_selftest(flag.data_ptr(), geom.data_ptr(), P, _stream()) == _lib.NS_OK
        assert lib.ns_read_device_status(geom.data_ptr(), P, _stream()) == _lib.NS_OK
    finally:
        assert lib.ns_set_wait_limit(prev) == 1 << 14
    # the context is still usable: a render and a sort run and report no error
    sc = small_scene(n=800, seed=31)
    inp = {k: v.cuda().contiguous() for k, v in api_inputs(sc).items()}
    g, cam = sc.grid, sc.camera
    cfg = raster.RasterConfig(image_height=cam.height, image_width=cam.width, tanfovx=cam.tanfovx,
                              tanfovy=cam.tanfovy, viewmatrix=cam.world_view_transform.cuda(),
                              projmatrix=cam.full_proj_transform.cuda(), levels=g.levels, S=g.S,
                              base_resolution=g.base_resolution, channels=g.channels, level_dim=g.level_dim)
    n, color, others, radii, _, _, scratch = raster.rasterize_forward(
        cfg, inp["means3D"], inp["scales"], inp["rotations"], inp["opacities"], inp["homotrans"],
        inp["ap_level"], g.table.cuda(), g.offsets.cuda(), g.gridrange.cuda())
    assert n > 0 and float(others[1].max()) > 0
    assert lib.ns_read_device_status(scratch.geom.data_ptr(), sc.P, _stream()) == _lib.NS_OK


def test_short_wait_limit_still_sorts():
    """The bound is a launch parameter of the sort's look-back: a short one
    (2^14 polls, far above what a running predecessor needs) leaves a large
    sort exact."""
    lib = _lib.load()
    rng = np.random.default_rng(3)
    n = 3_000_000
    keys = torch.from_numpy(rng.integers(0, 1 << 40, size=n, dtype=np.int64)).cuda()
    vals = torch.arange(n, dtype=torch.int32, device="cuda")
    prev = lib.ns_set_wait_limit(1 << 14)
    try:
        ko, vo = raster.radix_sort_pairs(keys, vals, end_bit=40)
    finally:
        lib.ns_set_wait_limit(prev)
    order = np.argsort(keys.cpu().numpy(), kind="stable")
    assert np.array_equal(vo.cpu().numpy(), order.astype(np.int32))
