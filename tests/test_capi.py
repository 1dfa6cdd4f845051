"""C-ABI checks that need no GPU: the library loads, exports every function the
header declares, the ctypes structures match the C layout, and the host-side
argument validation answers with status codes (no kernel is launched)."""
import ctypes as C
import pathlib
import re
import subprocess
import tempfile

import pytest

from nest_b200 import _lib

ROOT = pathlib.Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "nest_b200.h"


def _lib_or_build():
    if not _lib.LIB_PATH.exists():
        import importlib.util
        spec = importlib.util.spec_from_file_location("nsbuild", ROOT / "nest-splatting_b200" / "build.py")
        m = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(m)
        m.build()
    return _lib.load()


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ns_[a-z0-9_]+)\s*\(", text)))


def test_every_declared_symbol_is_exported():
    lib = _lib_or_build()
    decl = declared_functions()
    assert len(decl) >= 10
    for name in decl:
        assert hasattr(lib, name), name
    assert set(decl) == set(_lib.EXPORTED)


def test_struct_layout_matches_header():
    structs = {"ns_raster_settings": _lib.RasterSettings, "ns_surfels": _lib.Surfels,
               "ns_raster_outputs": _lib.RasterOutputs, "ns_frame_inputs": _lib.FrameInputs,
               "ns_frame_outputs": _lib.FrameOutputs, "ns_raster_grads_in": _lib.GradsIn,
               "ns_raster_grads_out": _lib.GradsOut}
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "nest_b200.h"', 'int main(void) {']
    for cname, py in structs.items():
        lines.append(f'printf("{cname} %zu\\n", sizeof({cname}));')
        for f, _ in py._fields_:
            lines.append(f'printf("{cname}.{f} %zu\\n", offsetof({cname}, {f}));')
    lines.append("return 0; }")
    with tempfile.TemporaryDirectory() as d:
        src = pathlib.Path(d) / "layout.c"
        src.write_text("\n".join(lines))
        exe = pathlib.Path(d) / "layout"
        subprocess.run(["gcc", "-I", str(ROOT / "include"), str(src), "-o", str(exe)], check=True)
        out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split("\n")
    got = dict(l.split() for l in out if l.strip())
    for cname, py in structs.items():
        assert int(got[cname]) == C.sizeof(py), cname
        for f, _ in py._fields_:
            assert int(got[f"{cname}.{f}"]) == getattr(py, f).offset, f"{cname}.{f}"


def test_status_strings_and_scratch_sizes():
    lib = _lib_or_build()
    assert lib.ns_status_string(0) == b"ok"
    assert b"too small" in lib.ns_status_string(_lib.NS_ERR_CAPACITY)
    assert lib.ns_geometry_scratch_bytes(1000) >= 1000 * (128 + 16 + 8)
    assert lib.ns_image_scratch_bytes(100, 70) >= 100 * 70 * 20
    a, b = lib.ns_binning_scratch_bytes(1000), lib.ns_binning_scratch_bytes(100000)
    assert b > a >= 1000 * 36
    assert lib.ns_radix_sort_temp_bytes(1 << 20) > 0
    assert lib.ns_backward_scratch_bytes(1000) >= 1000 * 18 * 4
    # deterministic mode: + a 64-bit fixed-point word per table entry and the scale word
    assert lib.ns_backward_scratch_bytes_deterministic(1000, 4096, 2) >= \
        lib.ns_backward_scratch_bytes(1000) + 4096 * 2 * 8 + 4
    assert lib.ns_normal_error_scratch_bytes(64, 48) >= 64 * 48 * 6 * 4
    assert lib.ns_normal_error_scratch_bytes(0, 48) == 0


def test_invalid_arguments_return_status_without_launching():
    lib = _lib_or_build()
    # null pointers and bad shapes are rejected on the host
    assert lib.ns_rvq_decode(None, None, None, 10, 6, 256, 59, None) == _lib.NS_ERR_INVALID
    assert lib.ns_rvq_decode(None, None, None, 10, 9, 256, 59, None) == _lib.NS_ERR_UNSUPPORTED
    assert lib.ns_rvq_decode(None, None, None, 0, 6, 256, 59, None) == _lib.NS_OK
    assert lib.ns_mlp_forward(None, 16, 10, None, 64, 3, None, None, None, None) == _lib.NS_ERR_UNSUPPORTED
    assert lib.ns_mlp_backward(None, 16, 10, None, 64, 3, None, None, None, None, None) == \
        _lib.NS_ERR_UNSUPPORTED
    assert lib.ns_mlp_backward(None, 32, 10, None, 64, 3, None, None, None, None, None) == _lib.NS_ERR_INVALID
    assert lib.ns_rasterize_forward(None, None, None, None, 0, None, 0, None, 0, None, 0, None) == \
        _lib.NS_ERR_INVALID
    assert lib.ns_mark_visible(-1, None, None, None, None, None) == _lib.NS_ERR_INVALID
    s = _lib.RasterSettings()
    s.image_width, s.image_height = 64, 48
    s.viewmatrix, s.projmatrix = 8, 8  # never dereferenced: validation fails first
    s.levels, s.level_dim, s.channels = 16, 2, 16  # 16 levels x 2 > 16 channels
    assert lib.ns_rasterize_forward(C.byref(s), None, None, None, 0, None, 0, None, 0, None, 0, None) == \
        _lib.NS_ERR_INVALID
    assert lib.ns_rasterize_backward(C.byref(s), None, None, None, None, 0, None, 0, None, 0, 0, None, 0,
                                     None) == _lib.NS_ERR_INVALID
    s.channels = 32
    surf = _lib.Surfels()
    surf.P = 10
    gi, go = _lib.GradsIn(), _lib.GradsOut()  # null gradient buffers
    assert lib.ns_rasterize_backward(C.byref(s), C.byref(surf), C.byref(gi), C.byref(go), None, 0, None, 0,
                                     None, 0, 0, None, 0, None) == _lib.NS_ERR_INVALID
    p = 1 << 20  # never dereferenced: every call below fails validation first
    assert lib.ns_normal_error(None, p, p, p, 4, 4, p, None) == _lib.NS_ERR_INVALID
    assert lib.ns_normal_error(p, p, p, p, -1, 4, p, None) == _lib.NS_ERR_INVALID
    assert lib.ns_normal_error(None, None, None, None, 0, 7, None, None) == _lib.NS_OK
    sb = lib.ns_normal_error_scratch_bytes(4, 4)
    assert lib.ns_normal_error_backward(p, p, p, p, 4, 4, p, -1, p, p, sb, None) == _lib.NS_ERR_INVALID
    assert lib.ns_normal_error_backward(p, p, p, p, 4, 4, p, 0, p, None, sb, None) == _lib.NS_ERR_INVALID
    assert lib.ns_normal_error_backward(p, p, p, p, 4, 4, p, 0, p, p, sb - 1, None) == _lib.NS_ERR_SCRATCH


def test_python_api_surface_matches_reference():
    import diff_surfel_rasterization as dsr
    assert dsr.GaussianRasterizationSettings._fields == (
        "image_height", "image_width", "tanfovx", "tanfovy", "bg", "scale_modifier", "viewmatrix",
        "projmatrix", "sh_degree", "campos", "prefiltered", "debug", "beta", "if_contract",
        "record_transmittance", "max_intersections")
    assert dsr.HashGridSettings._fields == ("L", "S", "H", "align_corners", "interpolation", "shape_dims")
    import inspect
    params = list(inspect.signature(dsr.GaussianRasterizer.forward).parameters)
    assert params == ["self", "means3D", "means2D", "opacities", "shs", "colors_precomp", "scales", "rotations",
                      "cov3D_precomp", "homotrans", "ap_level", "features", "offsets", "gridrange",
                      "features_diffuse", "offsets_diffuse", "gridrange_diffuse", "render_mode", "shapes",
                      "kernel_type"]
    for name in ("rasterize_gaussians", "GaussianRasterizer", "compute_relocation", "_RasterizeGaussians"):
        assert hasattr(dsr, name)


def test_gpu_calls_fail_loudly_without_device():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from nest_b200 import raster
    with pytest.raises(Exception):
        raster.rvq_decode(torch.zeros(4, 6, dtype=torch.uint8), torch.zeros(6, 256, 59))
