"""The CUDA hash-grid lookups against the reference's own gridencoder kernels.

ns_grid_encode_forward / ns_grid_encode_backward (csrc/gridencode.cu) run the
blend kernel's lookup code (hashgrid.cuh: make_level, corner_rows,
lookup_issue, lookup_finish). tests/golden/gridencoder_ref.npz holds what the
reference's gridencoder.cu computed on a B200 for the same points and table
(tests/golden/make_gridencoder_golden.py). Both are nvcc-compiled float32 code
with the same operation order, so the forward outputs and dy_dx are expected to
be bit-identical; the table gradient is summed with float atomics in both, so
its rows must be the same and its values equal up to summation order.
"""
from __future__ import annotations

import pathlib
import sys

import numpy as np
import pytest
import torch

HERE = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(HERE / "golden"))

import gridenc_cases as gc  # noqa: E402
from nest_b200 import gridencode  # noqa: E402

pytestmark = pytest.mark.gpu
L, LD, D = gc.LEVELS, gc.LEVEL_DIM, 3


@pytest.fixture(scope="module")
def ref():
    return np.load(HERE / "golden" / "gridencoder_ref.npz")


@pytest.fixture(scope="module")
def tables():
    t = torch.from_numpy(gc.table()).cuda()
    return {"fp32": t, "fp16": t.half()}


def _forward(pts, table, align, interp, with_dydx=True):
    B = pts.shape[0]
    out = torch.empty(L, B, LD, device="cuda")
    dydx = torch.empty(B, L * D * LD, device="cuda") if with_dydx else None
    offs = torch.from_numpy(gc.offsets()).cuda()
    gridencode.grid_encode_forward(pts, table, offs, out, B, D, LD, L, gc.S, gc.BASE_RES, dydx, 0, align, interp)
    return out, dydx


@pytest.mark.parametrize("dtype", ["fp32", "fp16"])
@pytest.mark.parametrize("align,interp", gc.CASES)
def test_grid_encode_forward_bit_exact_vs_reference(ref, tables, dtype, align, interp):
    name = gc.case_name(align, interp)
    pts = torch.from_numpy(gc.points()).cuda()
    out, _ = _forward(pts, tables[dtype], align, interp, with_dydx=False)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), ref[f"{name}_out"])
    _, dydx = _forward(pts[: gc.N_BWD].contiguous(), tables[dtype], align, interp)
    assert np.array_equal(dydx.cpu().numpy(), ref[f"{name}_dydx"])


@pytest.mark.parametrize("dtype", ["fp32", "fp16"])
@pytest.mark.parametrize("align,interp", gc.CASES)
def test_grid_encode_backward_vs_reference(ref, tables, dtype, align, interp):
    name = gc.case_name(align, interp)
    B = gc.N_BWD
    pts = torch.from_numpy(gc.points()[:B]).cuda()
    table = tables[dtype]
    _, dydx = _forward(pts, table, align, interp)
    grad = torch.from_numpy(gc.grad_outputs()).cuda()
    gtab = torch.zeros(table.shape, dtype=torch.float32, device="cuda")
    gin = torch.empty(B, D, device="cuda")
    offs = torch.from_numpy(gc.offsets()).cuda()
    gridencode.grid_encode_backward(grad, pts, table, offs, gtab, B, D, LD, L, gc.S, gc.BASE_RES, dydx, gin, 0, align,
                                    interp)
    g = gtab.cpu().numpy()
    rows = ref[f"{name}_grad_rows"]
    assert np.array_equal(np.nonzero(np.any(g != 0, axis=1))[0], rows)
    vals = ref[f"{name}_grad_vals"]
    assert np.allclose(g[rows], vals, rtol=1e-5, atol=1e-6 * np.abs(vals).max())
    assert np.array_equal(gin.cpu().numpy(), ref[f"{name}_grad_inputs"])


def test_grid_encode_refuses_unbuilt_shapes(tables):
    pts = torch.rand(8, 3, device="cuda")
    offs = torch.from_numpy(gc.offsets()).cuda()
    out = torch.empty(L, 8, 4, device="cuda")
    with pytest.raises(RuntimeError):  # C = 4: not built (the reference builds 1, 2, 4, 8, 16)
        gridencode.grid_encode_forward(pts, tables["fp32"], offs, out, 8, D, 4, L, gc.S, gc.BASE_RES, None, 0,
                                       False, 0)
    with pytest.raises(RuntimeError):  # non-contiguous inputs (TORCH_CHECK in the reference)
        gridencode.grid_encode_forward(pts.t().contiguous().t(), tables["fp32"], offs, out[..., :2], 8, D, 2, L,
                                       gc.S, gc.BASE_RES, None, 0, False, 0)
