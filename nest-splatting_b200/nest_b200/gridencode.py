"""Hash-grid encoding entry points with the reference gridencoder's Python-facing
signatures (the functions its pybind module exports, gridencoder/src/bindings.cpp,
declared in gridencoder/src/gridencoder.h:9-10), on libnest_b200.so.

This module can stand in for the reference's `_backend` (gridencoder/grid.py:9-12):
`grid_encode_forward` / `grid_encode_backward` take the same tensors and scalars
in the same order and raise RuntimeError where the reference's TORCH_CHECKs and
shape switches raise. Supported: D = 3, C = 2, gridtype 0 (hash). The lookup is
computed in fp32 also for an fp16 table; half-precision `outputs` / `dy_dx` /
`grad_embeddings` tensors receive the fp32 results rounded once.
"""
from __future__ import annotations

import torch

from . import _lib


def _need(t: torch.Tensor, name: str, dtypes) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be a contiguous tensor")
    if t.dtype not in dtypes:
        raise RuntimeError(f"{name} has dtype {t.dtype}")


_FLOATS = (torch.float32, torch.float16)


def _fp32_view(t: torch.Tensor | None):
    """(fp32 tensor to write, tensor to copy it back into or None)."""
    if t is None or t.dtype == torch.float32:
        return t, None
    return torch.empty(t.shape, dtype=torch.float32, device=t.device), t


def grid_encode_forward(inputs, embeddings, offsets, outputs, B, D, C, L, S, H, dy_dx, gridtype, align_corners,
                        interp):
    """outputs [L, B, C] (and dy_dx [B, L*D*C] when given) for inputs [B, D] in [0, 1]."""
    _need(inputs, "inputs", (torch.float32,))
    _need(embeddings, "embeddings", _FLOATS)
    _need(offsets, "offsets", (torch.int32,))
    _need(outputs, "outputs", _FLOATS)
    out32, out_back = _fp32_view(outputs)
    dyd32, dyd_back = _fp32_view(dy_dx)
    lib = _lib.load()
    _lib.check("ns_grid_encode_forward", lib.ns_grid_encode_forward(
        inputs.data_ptr(), embeddings.data_ptr(), int(embeddings.dtype == torch.float16), offsets.data_ptr(),
        out32.data_ptr(), int(B), int(D), int(C), int(L), float(S), int(H), _lib.ptr(dyd32), int(gridtype),
        int(bool(align_corners)), int(interp), _lib.stream_handle(inputs.device)))
    if out_back is not None:
        out_back.copy_(out32)
    if dyd_back is not None:
        dyd_back.copy_(dyd32)


def grid_encode_backward(grad, inputs, embeddings, offsets, grad_embeddings, B, D, C, L, S, H, dy_dx, grad_inputs,
                         gridtype, align_corners, interp):
    """Accumulates grad_embeddings (zero it first) and writes grad_inputs from dy_dx."""
    _need(grad, "grad", _FLOATS)
    _need(inputs, "inputs", (torch.float32,))
    _need(embeddings, "embeddings", _FLOATS)
    _need(offsets, "offsets", (torch.int32,))
    _need(grad_embeddings, "grad_embeddings", _FLOATS)
    g32 = grad.float().contiguous()
    ge32, ge_back = _fp32_view(grad_embeddings)
    if ge_back is not None:
        ge32.copy_(ge_back)
    dyd32 = None if dy_dx is None else dy_dx.float().contiguous()
    gi32, gi_back = _fp32_view(grad_inputs)
    lib = _lib.load()
    _lib.check("ns_grid_encode_backward", lib.ns_grid_encode_backward(
        g32.data_ptr(), inputs.data_ptr(), embeddings.data_ptr(), int(embeddings.dtype == torch.float16),
        offsets.data_ptr(), ge32.data_ptr(), int(B), int(D), int(C), int(L), float(S), int(H), _lib.ptr(dyd32),
        _lib.ptr(gi32), int(gridtype), int(bool(align_corners)), int(interp), _lib.stream_handle(inputs.device)))
    if ge_back is not None:
        ge_back.copy_(ge32)
    if gi_back is not None:
        gi_back.copy_(gi32)
