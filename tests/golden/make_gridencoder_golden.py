"""Writes tests/golden/gridencoder_ref.npz by running the reference's own
gridencoder CUDA kernels (gridencoder/src/gridencoder.cu) on a GPU.

The module is built from the unmodified reference sources by
oracle/build_ref.py into oracle/_ref/gridencoder/ (the build needs the
reference checkout; running it needs a CUDA device, not the checkout):

    python oracle/build_ref.py                              # build container
    python tests/golden/make_gridencoder_golden.py OUT.npz  # GPU box

For each case of gridenc_cases.CASES (align_corners x linear/smoothstep) on the
benchmark grid (16 levels x 2, 2^19 rows per level, H 16, scale 1.447) and the
U(-1, 1) fp16-valued table, it records, through the reference's pybind entry
points (gridencoder/src/bindings.cpp):
  * grid_encode_forward: outputs [L, B, 2] (kernel_grid, gridencoder.cu:88-242)
    and dy_dx [B, L*3*2] (the first N_BWD points);
  * grid_encode_backward with the seeded upstream gradient: the non-zero rows
    of grad_embeddings (kernel_grid_backward, :246-338) and grad_inputs [B, 3]
    (kernel_input_backward, :341-367).
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
sys.path.insert(0, str(HERE.parent.parent))

import gridenc_cases as gc  # noqa: E402
from oracle import build_ref  # noqa: E402


def main(out_path: str) -> None:
    assert torch.cuda.is_available(), "the reference gridencoder runs on a CUDA device"
    ref = build_ref.load_module()
    dev = torch.device("cuda:0")
    table = torch.from_numpy(gc.table()).to(dev)
    offs = torch.from_numpy(gc.offsets()).to(dev)
    pts = torch.from_numpy(gc.points()).to(dev)
    grad = torch.from_numpy(gc.grad_outputs()).to(dev)
    L, C, D, H, S = gc.LEVELS, gc.LEVEL_DIM, 3, gc.BASE_RES, float(gc.S)
    blob = {"points": gc.points(), "offsets": gc.offsets()}
    for align, interp in gc.CASES:
        name = gc.case_name(align, interp)
        B = gc.N_FWD
        out = torch.empty(L, B, C, device=dev)
        dydx = torch.empty(B, L * D * C, device=dev)
        ref.grid_encode_forward(pts, table, offs, out, B, D, C, L, S, H, dydx, 0, align, interp)
        torch.cuda.synchronize()
        blob[f"{name}_out"] = out.cpu().numpy()
        Bb = gc.N_BWD
        pb = pts[:Bb].contiguous()
        outb = torch.empty(L, Bb, C, device=dev)
        dydxb = torch.empty(Bb, L * D * C, device=dev)
        ref.grid_encode_forward(pb, table, offs, outb, Bb, D, C, L, S, H, dydxb, 0, align, interp)
        gtab = torch.zeros_like(table)
        gin = torch.zeros(Bb, D, device=dev)
        ref.grid_encode_backward(grad.contiguous(), pb, table, offs, gtab, Bb, D, C, L, S, H, dydxb, gin, 0,
                                 align, interp)
        torch.cuda.synchronize()
        g = gtab.cpu().numpy()
        rows = np.nonzero(np.any(g != 0, axis=1))[0].astype(np.int32)
        blob[f"{name}_dydx"] = dydxb.cpu().numpy()
        blob[f"{name}_grad_rows"] = rows
        blob[f"{name}_grad_vals"] = g[rows]
        blob[f"{name}_grad_inputs"] = gin.cpu().numpy()
    meta = {"gpu": torch.cuda.get_device_name(0), "torch": torch.__version__,
            "cuda": torch.version.cuda, "module": "gridencoder/src/gridencoder.cu (unmodified)",
            "levels": L, "level_dim": C, "log2_T": gc.LOG2_T, "base_resolution": H,
            "per_level_scale": gc.PER_LEVEL_SCALE, "S": S}
    blob["meta"] = np.array(json.dumps(meta))
    Path(out_path).parent.mkdir(parents=True, exist_ok=True)
    np.savez_compressed(out_path, **blob)
    print(f"wrote {out_path}: {json.dumps(meta)}")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else str(HERE / "gridencoder_ref.npz"))
