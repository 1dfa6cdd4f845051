"""CPU oracle for the nest-splatting render path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
arm may import this module, and only as the checker (or the CPU baseline):
the product path (nest-splatting_b200) never calls it.

Contents:
  * ctypes wrapper of oracle/_build/libnest_oracle.so (nest_oracle.cpp, the C++
    restatement of preprocess / binning / mode-0 blend / hash query);
  * rvq_decode_np: numpy restatement of the RVQ decode (benchmark config 0);
  * rvq_decode_torch: the "reference PyTorch CPU path" timed as the RVQ baseline;
  * mlp_oracle: fp16 MLP restatement (tiny-cuda-nn is not vendored: parity of
    the MLP is unpinned, this fixes one definition);
  * forward / frame helpers chaining the above.

Parity status: pinned by the known-answer tests in tests/test_oracle.py and, for
the camera and homotrans inputs, by tests/golden (made by importing the
reference's own Python utilities). The reference CUDA rasterizer cannot be
built here (its glm dependency is absent), so the blend restatement itself is
"parity unpinned" against reference outputs.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "libnest_oracle.so"
KBLOCK = 16

_lib = None


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def load() -> C.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        build()
    lib = C.CDLL(str(LIB_PATH))
    vp, i32, u32, i64, f32 = C.c_void_p, C.c_int, C.c_uint32, C.c_int64, C.c_float
    lib.oracle_preprocess.argtypes = [i32, vp, vp, f32, vp, vp, vp, vp, i32, i32, vp, vp, vp, vp, vp, vp]
    lib.oracle_preprocess_precomp.argtypes = [i32, vp, vp, vp, vp, vp, i32, i32, vp, vp, vp, vp, vp, vp]
    lib.oracle_preprocess_backward_precomp.argtypes = [i32, vp, vp, i32, i32, f32, f32, vp, vp, vp, vp, vp, vp]
    lib.oracle_preprocess_backward_precomp_f64.argtypes = lib.oracle_preprocess_backward_precomp.argtypes
    lib.oracle_bin.restype = i64
    lib.oracle_bin.argtypes = [i32, vp, vp, vp, i32, i32, vp, vp, i64, vp]
    lib.oracle_render.argtypes = [i32, i32, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, i32, i32, u32, f32, u32,
                                  i32, u32, i32, f32, u32, i32, vp, vp, vp, vp, vp, vp, i32, i32, vp,
                                  i32, i32, i32, vp]
    lib.oracle_query.argtypes = [i32, vp, vp, vp, vp, f32, f32, i32, i32, u32, f32, u32, i32, u32, i32, vp, vp]
    lib.oracle_query_backward.argtypes = [i32, vp, vp, vp, vp, f32, f32, i32, i32, u32, f32, u32, i32, u32, i32,
                                          vp, vp, vp, vp]
    lib.oracle_sh_color.argtypes = [i32, i32, i32, vp, vp, vp, vp]
    lib.oracle_sh_color_backward.argtypes = [i32, i32, i32, vp, vp, vp, vp, vp, vp, vp]
    lib.oracle_sh_color_backward_f64.argtypes = [i32, i32, i32, vp, vp, vp, vp, vp, vp, vp]
    lib.oracle_grid_index.restype = u32
    lib.oracle_grid_index.argtypes = [i32, u32, u32, u32, u32, u32]
    lib.oracle_rvq_decode.argtypes = [i64, i32, i32, i32, vp, vp, vp]
    lib.oracle_num_threads.restype = i32
    lib.oracle_render_backward.argtypes = [i32, i32, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, i32, i32, u32, f32,
                                           u32, i32, u32, i32, f32, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp,
                                           i32, vp, vp, i32, i32, i32, vp, vp, i32]
    lib.oracle_preprocess_backward.argtypes = [i32, vp, vp, vp, vp, vp, vp, vp, i32, i32, f32, f32, vp, vp, vp,
                                               vp, vp, vp, vp]
    lib.oracle_render_backward_f64.argtypes = lib.oracle_render_backward.argtypes
    lib.oracle_preprocess_backward_f64.argtypes = lib.oracle_preprocess_backward.argtypes
    _lib = lib
    return lib


def _p(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p) if a is not None else None


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def preprocess(means3D, scales, rotations, opacities, viewmatrix, projmatrix, W, H, scale_modifier=1.0,
               transmat_precomp=None):
    """forward.cu:323-441 restated. Returns dict of per-surfel arrays. With
    transmat_precomp [P, 9] (columns Tu, Tv, Tw) the transforms are taken as
    given and scales / rotations are not read (forward.cu:366-380)."""
    lib = load()
    means3D = _f32(means3D)
    opacities = _f32(opacities).reshape(-1)
    vm, pm = _f32(viewmatrix).reshape(16), _f32(projmatrix).reshape(16)
    P = means3D.shape[0]
    out = dict(radii=np.zeros(P, np.int32), means2D=np.zeros((P, 2), np.float32), depths=np.zeros(P, np.float32),
               transMat=np.zeros((P, 9), np.float32), normal_opacity=np.zeros((P, 4), np.float32),
               tiles_touched=np.zeros(P, np.uint32))
    tail = (_p(out["radii"]), _p(out["means2D"]), _p(out["depths"]), _p(out["transMat"]),
            _p(out["normal_opacity"]), _p(out["tiles_touched"]))
    if transmat_precomp is not None:
        Ts = _f32(transmat_precomp).reshape(P, 9)
        lib.oracle_preprocess_precomp(P, _p(means3D), _p(Ts), _p(opacities), _p(vm), _p(pm), int(W), int(H), *tail)
        return out
    scales, rotations = _f32(scales), _f32(rotations)
    lib.oracle_preprocess(P, _p(means3D), _p(scales), float(scale_modifier), _p(rotations), _p(opacities), _p(vm),
                          _p(pm), int(W), int(H), *tail)
    return out


def bin_surfels(pre, W, H):
    """duplicateWithKeys + stable sort + identifyTileRanges. Returns (keys, vals, ranges [tiles,2])."""
    lib = load()
    P = pre["radii"].shape[0]
    tiles = ((W + KBLOCK - 1) // KBLOCK) * ((H + KBLOCK - 1) // KBLOCK)
    cap = int(pre["tiles_touched"].astype(np.int64).sum())
    keys = np.zeros(max(cap, 1), np.uint64)
    vals = np.zeros(max(cap, 1), np.uint32)
    ranges = np.zeros((tiles, 2), np.uint32)
    n = lib.oracle_bin(P, _p(pre["means2D"]), _p(pre["depths"]), _p(pre["radii"]), int(W), int(H), _p(keys),
                       _p(vals), cap, _p(ranges))
    assert n == cap, (n, cap)
    return keys[:n], vals[:n], ranges


def render(pre, vals, ranges, homotrans, ap_level, table_f32, offsets, gridrange, W, H, C_out, LD, L, S, Hres,
           align_corners=False, interp=0, contract=False, beta=0.0, max_intersections=0,
           record_transmittance=False, row_stride=1, kernel_type=0, shapes=None, render_mode=0,
           hybrid_levels=0, total_levels=0, gauss=None):
    """renderCUDAsurfelForward<C> restated. Returns dict of output images.
    kernel_type 1-3 (beta / flex / general splat kernels) read shapes [P].
    render_mode 4 / 12 / 14 (| 256 for the inference flag) combine per-surfel
    features `gauss` (colors_precomp rows) with the L hash levels at channel
    hybrid_levels * LD. Modes 8 / 9 / 10 read one 3-wide hash level (LD 3, L 1)
    and rows of 3 raw SH colours (48 SH coefficients for 9), hybrid_levels
    carrying the level word's decompose flag; mode 11 adds the rows' degree-3
    SH colour in out_others channels 14-16 (17 channels for that mode).

    row_stride > 1 renders only tile rows ty with ty % row_stride == 0 (a bounded
    sample for CPU timing); other pixels stay zero."""
    lib = load()
    HW = W * H
    P = pre["radii"].shape[0]
    n_others = 17 if (int(render_mode) & 0xFF) == 11 else 14
    out = dict(out_color=np.zeros((C_out, H, W), np.float32), out_others=np.zeros((n_others, H, W), np.float32),
               final_T=np.zeros((3, H, W), np.float32), n_contrib=np.zeros((2, H, W), np.uint32),
               cover_pixels=np.zeros(P, np.float32), trans_avg=np.zeros(P, np.float32))
    homotrans = _f32(homotrans).reshape(-1, 16)
    ap = _f32(ap_level).reshape(-1) if ap_level is not None else np.full(P, 1e9, np.float32)
    table = _f32(table_f32)
    offs = np.ascontiguousarray(np.asarray(offsets, dtype=np.int32))
    gr = _f32(gridrange).reshape(2)
    lib.oracle_render(int(W), int(H), _p(np.ascontiguousarray(ranges, np.uint32)),
                      _p(np.ascontiguousarray(vals, np.uint32)), _p(pre["means2D"]), _p(pre["transMat"]),
                      _p(pre["normal_opacity"]), _p(homotrans), _p(ap), _p(table), _p(offs), _p(gr), int(C_out),
                      int(LD), int(L), float(S), int(Hres), int(bool(align_corners)), int(interp),
                      int(bool(contract)), float(beta), int(max_intersections), int(bool(record_transmittance)),
                      _p(out["out_color"]), _p(out["out_others"]), _p(out["final_T"]), _p(out["n_contrib"]),
                      _p(out["cover_pixels"]), _p(out["trans_avg"]), int(row_stride), int(kernel_type),
                      _p(_f32(shapes).reshape(-1)) if shapes is not None else None, int(render_mode),
                      int(hybrid_levels), int(total_levels), _p(_f32(gauss).reshape(-1)) if gauss is not None else None)
    assert HW == W * H
    return out


def query(xyz, ap_level, table_f32, offsets, vmin, vmax, C_out, LD, L, S, Hres, align_corners=False, interp=0,
          contract=False, level_exp2=None):
    """hashgrid.h:53-212 per point -> [n, C_out]. level_exp2: optional [L] values of
    exp2f(l S) (e.g. the device's) in place of the host's."""
    lib = load()
    lexp = None if level_exp2 is None else _f32(level_exp2).reshape(-1)
    xyz = _f32(xyz).reshape(-1, 3)
    n = xyz.shape[0]
    ap = np.ascontiguousarray(np.asarray(ap_level, dtype=np.uint32).reshape(-1))
    out = np.zeros((n, C_out), np.float32)
    lib.oracle_query(n, _p(xyz), _p(ap), _p(_f32(table_f32)), _p(np.ascontiguousarray(offsets, np.int32)),
                     float(vmin), float(vmax), int(C_out), int(LD), int(L), float(S), int(Hres),
                     int(bool(align_corners)), int(interp), int(bool(contract)), _p(lexp), _p(out))
    return out


def sh_color(means3D, campos, shs, deg):
    """computeColorFromSH (forward.cu:21-74) of every surfel: shs [P, M, 3]
    (coefficient-major RGB triples), campos [3]; returns rgb [P, 3]."""
    lib = load()
    means3D, campos, shs = _f32(means3D).reshape(-1, 3), _f32(campos).reshape(3), _f32(shs)
    P = means3D.shape[0]
    M = shs.reshape(P, -1, 3).shape[1] if P else 1
    rgb = np.zeros((P, 3), np.float32)
    lib.oracle_sh_color(P, int(deg), int(M), _p(means3D), _p(campos), _p(shs), _p(rgb))
    return rgb


def sh_color_backward(means3D, campos, shs, deg, radii, dL_drgb, f64=False):
    """The SH colour's backward (backward.cu:21-140): returns (dL_dshs [P, M, 3],
    dL_dmeans [P, 3], the view-direction part), zero where radii <= 0."""
    lib = load()
    means3D, campos, shs = _f32(means3D).reshape(-1, 3), _f32(campos).reshape(3), _f32(shs)
    P = means3D.shape[0]
    M = shs.reshape(P, -1, 3).shape[1] if P else 1
    dt = np.float64 if f64 else np.float32
    g = np.ascontiguousarray(np.asarray(dL_drgb, dt).reshape(P, 3))
    dsh = np.zeros((P, M, 3), dt)
    dmean = np.zeros((P, 3), dt)
    fn = lib.oracle_sh_color_backward_f64 if f64 else lib.oracle_sh_color_backward
    fn(P, int(deg), int(M), _p(means3D), _p(campos), _p(shs),
       _p(np.ascontiguousarray(np.asarray(radii, np.int32))), _p(g), _p(dsh), _p(dmean))
    return dsh, dmean


def query_backward(xyz, ap_level, table_f32, offsets, vmin, vmax, C_out, LD, L, S, Hres, grad_feat,
                   align_corners=False, interp=0, contract=False, level_exp2=None):
    """hashgrid.h:106-299 per point: (dL_dtable [rows, LD], dL_dxyz [n, 3]) for grad_feat [n, C_out]."""
    lib = load()
    lexp = None if level_exp2 is None else _f32(level_exp2).reshape(-1)
    xyz = _f32(xyz).reshape(-1, 3)
    n = xyz.shape[0]
    ap = np.ascontiguousarray(np.asarray(ap_level, dtype=np.uint32).reshape(-1))
    table_f32 = _f32(table_f32)
    dtab = np.zeros_like(table_f32)
    dxyz = np.zeros((n, 3), np.float32)
    g = _f32(grad_feat).reshape(n, C_out)
    lib.oracle_query_backward(n, _p(xyz), _p(ap), _p(table_f32), _p(np.ascontiguousarray(offsets, np.int32)),
                              float(vmin), float(vmax), int(C_out), int(LD), int(L), float(S), int(Hres),
                              int(bool(align_corners)), int(interp), int(bool(contract)), _p(lexp), _p(g),
                              _p(dtab), _p(dxyz))
    return dtab, dxyz


def grid_index(align_corners, hashmap_size, res, x, y, z) -> int:
    return int(load().oracle_grid_index(int(bool(align_corners)), hashmap_size, res, x, y, z))


def rvq_decode_np(idx: np.ndarray, codebooks: np.ndarray) -> np.ndarray:
    """out[n] = (((0 + CB0[i0]) + CB1[i1]) + ...) in fp32, stage order."""
    idx = np.asarray(idx)
    cb = np.asarray(codebooks, dtype=np.float32)
    out = np.zeros((idx.shape[0], cb.shape[2]), np.float32)
    for k in range(cb.shape[0]):
        out += cb[k][idx[:, k].astype(np.int64)]
    return out


def rvq_decode_c(idx: np.ndarray, codebooks: np.ndarray) -> np.ndarray:
    """The same decode through the C++ oracle (OpenMP over surfels)."""
    lib = load()
    idx = np.ascontiguousarray(idx, dtype=np.uint8)
    cb = _f32(codebooks)
    K, E, D = cb.shape
    out = np.empty((idx.shape[0], D), np.float32)
    lib.oracle_rvq_decode(idx.shape[0], K, E, D, _p(idx), _p(cb), _p(out))
    return out


def rvq_decode_torch(idx, codebooks):
    """PyTorch CPU restatement (index_select + in-order adds): the timed CPU baseline."""
    import torch
    idx = idx.long()
    out = torch.zeros((idx.shape[0], codebooks.shape[2]), dtype=torch.float32)
    for k in range(codebooks.shape[0]):
        out += codebooks[k].index_select(0, idx[:, k])
    return out


def mlp_oracle(feat_np: np.ndarray, weights, alpha=None, bg=None) -> np.ndarray:
    """feat [C, ...] fp32 -> rgb [3, ...]: fp16 operands, fp32 accumulation, each layer
    (and the network output) rounded to fp16, sigmoid in fp32, x (alpha > 0), + (1-alpha) bg."""
    import torch
    shape = feat_np.shape[1:]
    x = torch.as_tensor(np.asarray(feat_np, np.float32)).reshape(feat_np.shape[0], -1).T
    h = x.half().float()
    ws = [torch.as_tensor(np.asarray(w)).half().float() for w in weights]
    for i, w in enumerate(ws):
        h = h @ w.T
        if i < len(ws) - 1:
            h = torch.clamp_min(h, 0.0)
        h = h.half().float()
    rgb = torch.sigmoid(h[:, :3]).T.reshape((3,) + tuple(shape)).numpy().astype(np.float32)
    if alpha is not None:
        a = np.asarray(alpha, np.float32).reshape(shape)
        rgb = rgb * (a > 0)
        if bg is not None and float(np.sum(bg)) > 0:
            rgb = rgb + (1.0 - a)[None] * np.asarray(bg, np.float32).reshape(3, *([1] * len(shape)))
    return rgb.astype(np.float32)


def forward(means3D, scales, rotations, opacities, homotrans, ap_level, table_f32, offsets, gridrange,
            viewmatrix, projmatrix, W, H, C_out, LD, L, S, Hres, **kw):
    """Full oracle forward: preprocess -> bin -> render. Returns (render dict, pre, num_rendered)."""
    pre = preprocess(means3D, scales, rotations, opacities, viewmatrix, projmatrix, W, H,
                     kw.pop("scale_modifier", 1.0), transmat_precomp=kw.pop("transmat_precomp", None))
    keys, vals, ranges = bin_surfels(pre, W, H)
    out = render(pre, vals, ranges, homotrans, ap_level, table_f32, offsets, gridrange, W, H, C_out, LD, L, S,
                 Hres, **kw)
    return out, pre, len(vals)


def render_backward(pre, vals, ranges, fwd, homotrans, ap_level, table_f32, offsets, gridrange, W, H, C_out, LD,
                    L, S, Hres, dL_dcolor, dL_dothers, align_corners=False, interp=0, contract=False, beta=0.0,
                    f64=False, kernel_type=0, shapes=None, render_mode=0, hybrid_levels=0, total_levels=0,
                    gauss=None, row_stride=1):
    """renderCUDAsurfelBackward<C> mode 0 restated (nest_oracle_bw.cpp). `fwd` is the
    dict returned by render(). Returns the render-pass gradients (reference layouts).
    f64=True evaluates the same formulas in double (float64 outputs). kernel_type
    1-3 take per-surfel `shapes` [P] and add dL_dshapes [P]. Render modes 4 / 12 /
    14 (and 6 / 7, and level 0: mode 0 with L = 0) take the per-surfel rows
    `gauss` and add dL_dcolors (same shape).
    row_stride > 1 walks only tile rows ty % row_stride == 0 (the upstream
    gradient must be zero on the others, e.g. after a sampled forward)."""
    lib = load()
    P = pre["radii"].shape[0]
    table = _f32(table_f32)
    dt = np.float64 if f64 else np.float32
    g = dict(dL_dtable=np.zeros(table.shape, dt), dL_dtransMat=np.zeros((P, 9), dt),
             dL_dhomoMat=np.zeros((P, 9), dt), dL_dmean2D=np.zeros((P, 3), dt),
             dL_dnormal=np.zeros((P, 3), dt), dL_dopacity=np.zeros(P, dt), dL_gradsum=np.zeros(P, dt),
             dL_dshapes=np.zeros(P, dt))
    rows = render_mode != 0 or int(L) == 0  # per-surfel rows: every mode but 0, and level 0
    if rows:
        if gauss is None:
            raise ValueError(f"render_mode {render_mode} with {L} levels needs the per-surfel rows (gauss)")
        gauss = _f32(gauss).reshape(P, -1)
        g["dL_dcolors"] = np.zeros(gauss.shape, dt)
    if kernel_type != 0:
        assert shapes is not None
        shapes = _f32(shapes).reshape(P)
    homotrans = _f32(homotrans).reshape(-1, 16)
    ap = _f32(ap_level).reshape(-1) if ap_level is not None else np.full(P, 1e9, np.float32)
    offs = np.ascontiguousarray(np.asarray(offsets, dtype=np.int32))
    gc, go = _f32(dL_dcolor), _f32(np.asarray(dL_dothers)[:14])  # channels 14-16 (mode 11) have no gradient
    assert gc.shape == (C_out, H, W) and go.shape == (14, H, W)
    fn = lib.oracle_render_backward_f64 if f64 else lib.oracle_render_backward
    fn(int(W), int(H), _p(np.ascontiguousarray(ranges, np.uint32)),
                               _p(np.ascontiguousarray(vals, np.uint32)), _p(pre["means2D"]), _p(pre["transMat"]),
                               _p(pre["normal_opacity"]), _p(homotrans), _p(ap), _p(table), _p(offs),
                               _p(_f32(gridrange).reshape(2)), int(C_out), int(LD), int(L), float(S), int(Hres),
                               int(bool(align_corners)), int(interp), int(bool(contract)), float(beta),
                               _p(fwd["final_T"]), _p(fwd["n_contrib"]), _p(gc), _p(go), _p(g["dL_dtable"]),
                               _p(g["dL_dtransMat"]), _p(g["dL_dhomoMat"]), _p(g["dL_dmean2D"]),
                               _p(g["dL_dnormal"]), _p(g["dL_dopacity"]), _p(g["dL_gradsum"]), int(kernel_type),
                               _p(shapes if kernel_type != 0 else None), _p(g["dL_dshapes"]), int(render_mode),
                               int(hybrid_levels), int(total_levels), _p(gauss if rows else None),
                               _p(g.get("dL_dcolors")), int(row_stride))
    return g


def preprocess_backward(means3D, scales, rotations, pre, g, viewmatrix, projmatrix, W, H, tanfovx, tanfovy,
                        f64=False, precomp=False):
    """preprocessCUDA backward + compute_transmat_aabb restated. Consumes the
    render-pass gradients `g` (from render_backward) and returns
    dL_dmeans3D [P,3], dL_dscales [P,2], dL_drots [P,4] and the densification
    statistic dL_dmean2D [P,3] (the rasterizer's means2D gradient). With
    precomp (the forward took transmat_precomp) also dL_dtransMat [P,9], the
    given transforms' gradient; means, scales and rotations get zeros."""
    lib = load()
    if precomp:
        P = pre["radii"].shape[0]
        dt = np.float64 if f64 else np.float32
        out = dict(dL_dmeans3D=np.zeros((P, 3), dt), dL_dscales=np.zeros((P, 2), dt),
                   dL_drots=np.zeros((P, 4), dt), dL_dmean2D=np.array(g["dL_dmean2D"], dt, copy=True),
                   dL_dtransMat=np.zeros((P, 9), dt))
        fn = lib.oracle_preprocess_backward_precomp_f64 if f64 else lib.oracle_preprocess_backward_precomp
        fn(P, _p(pre["radii"]), _p(pre["transMat"]), int(W), int(H), float(tanfovx), float(tanfovy),
           _p(out["dL_dmean2D"]), _p(np.ascontiguousarray(np.asarray(g["dL_dtransMat"], dt))),
           _p(out["dL_dtransMat"]), _p(out["dL_dmeans3D"]), _p(out["dL_dscales"]), _p(out["dL_drots"]))
        return out
    means3D, scales, rotations = _f32(means3D), _f32(scales), _f32(rotations)
    P = means3D.shape[0]
    dt = np.float64 if f64 else np.float32
    cast = lambda a: np.ascontiguousarray(np.asarray(a, dtype=dt))  # noqa: E731
    out = dict(dL_dmeans3D=np.zeros((P, 3), dt), dL_dscales=np.zeros((P, 2), dt),
               dL_drots=np.zeros((P, 4), dt), dL_dmean2D=np.array(g["dL_dmean2D"], dt, copy=True))
    fn = lib.oracle_preprocess_backward_f64 if f64 else lib.oracle_preprocess_backward
    fn(P, _p(means3D), _p(scales), _p(rotations), _p(pre["radii"]), _p(pre["transMat"]),
       _p(_f32(viewmatrix).reshape(16)), _p(_f32(projmatrix).reshape(16)), int(W), int(H), float(tanfovx),
       float(tanfovy), _p(out["dL_dmean2D"]), _p(cast(g["dL_dnormal"])), _p(cast(g["dL_dtransMat"])),
       _p(cast(g["dL_dhomoMat"])), _p(out["dL_dmeans3D"]), _p(out["dL_dscales"]), _p(out["dL_drots"]))
    return out


def num_threads() -> int:
    return int(load().oracle_num_threads())


def set_num_threads(n: int) -> int:
    """Sets the oracle's OpenMP thread count; returns the count now in effect."""
    lib = load()
    lib.oracle_set_num_threads.argtypes = [C.c_int]
    lib.oracle_set_num_threads(int(n))
    return num_threads()


if __name__ == "__main__":
    print(build(), os.cpu_count())
