"""ctypes bindings of libnest_b200.so (include/nest_b200.h).

The library is loaded from the package directory (built in-tree by
nest-splatting_b200/build.py). There is no CPU or PyTorch fallback: when the
library or a CUDA device is missing, every call raises.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent.parent / "libnest_b200.so"

NS_OK, NS_ERR_INVALID, NS_ERR_UNSUPPORTED, NS_ERR_CAPACITY, NS_ERR_CUDA, NS_ERR_SCRATCH, NS_ERR_DEVICE = range(7)
NS_FLAG_DEVICE_COUNT = 1
NS_FLAG_SKIP_DECODE = 2
NS_FRAME_STAGES = 5
STAGE_NAMES = ("decode", "preprocess", "binning", "blend", "mlp")

EXPORTED = [
    "ns_status_string", "ns_kernel_launches", "ns_last_cuda_error", "ns_version",
    "ns_geometry_scratch_bytes", "ns_image_scratch_bytes", "ns_binning_scratch_bytes",
    "ns_rasterize_forward", "ns_read_device_status", "ns_mark_visible", "ns_mlp_forward",
    "ns_rvq_decode", "ns_radix_sort_temp_bytes", "ns_radix_sort_pairs", "ns_render_frame",
    "ns_radix_sort_pairs_noalloc", "ns_backward_scratch_bytes", "ns_backward_scratch_bytes_deterministic",
    "ns_rasterize_backward",
    "ns_normal_error", "ns_normal_error_scratch_bytes", "ns_normal_error_backward", "ns_mlp_backward",
    "ns_allmap_decode", "ns_grid_encode_forward", "ns_grid_encode_backward", "ns_read_binning",
    "ns_gather_probe", "ns_set_wait_limit", "ns_wait_selftest",
]


class RasterSettings(C.Structure):
    _fields_ = [
        ("image_height", C.c_int32), ("image_width", C.c_int32),
        ("tanfovx", C.c_float), ("tanfovy", C.c_float), ("scale_modifier", C.c_float),
        ("viewmatrix", C.c_void_p), ("projmatrix", C.c_void_p),
        ("beta", C.c_float), ("if_contract", C.c_int32), ("record_transmittance", C.c_int32),
        ("max_intersections", C.c_uint32), ("prefiltered", C.c_int32),
        ("levels", C.c_uint32), ("level_scale_log2", C.c_float), ("base_resolution", C.c_uint32),
        ("align_corners", C.c_int32), ("interpolation", C.c_uint32), ("channels", C.c_uint32),
        ("level_dim", C.c_uint32), ("table_fp16", C.c_int32), ("kernel_type", C.c_int32),
        ("deterministic", C.c_int32), ("render_mode", C.c_int32), ("hybrid_levels", C.c_uint32),
        ("total_levels", C.c_uint32), ("sh_degree", C.c_int32), ("campos", C.c_void_p),
    ]


class Surfels(C.Structure):
    _fields_ = [
        ("P", C.c_int32), ("means3D", C.c_void_p), ("scales", C.c_void_p),
        ("rotations", C.c_void_p), ("opacities", C.c_void_p), ("homotrans", C.c_void_p),
        ("ap_level", C.c_void_p), ("features", C.c_void_p), ("offsets", C.c_void_p),
        ("gridrange", C.c_void_p), ("shapes", C.c_void_p), ("colors_precomp", C.c_void_p),
        ("shs", C.c_void_p), ("sh_coeffs", C.c_int32), ("transmat_precomp", C.c_void_p),
    ]


class RasterOutputs(C.Structure):
    _fields_ = [
        ("out_color", C.c_void_p), ("out_others", C.c_void_p), ("radii", C.c_void_p),
        ("cover_pixels", C.c_void_p), ("trans_avg", C.c_void_p),
    ]


class FrameInputs(C.Structure):
    _fields_ = [
        ("P", C.c_int32), ("rvq_idx", C.c_void_p), ("codebooks", C.c_void_p),
        ("stages", C.c_int32), ("entries", C.c_int32), ("dims", C.c_int32),
        ("base", C.c_void_p), ("mix", C.c_float), ("decoded", C.c_void_p),
        ("ap_level", C.c_void_p), ("features", C.c_void_p), ("offsets", C.c_void_p),
        ("gridrange", C.c_void_p), ("mlp_weights", C.c_void_p), ("mlp_hidden", C.c_int32),
        ("bg_host", C.c_void_p), ("stage_events", C.c_void_p),
    ]


class FrameOutputs(C.Structure):
    _fields_ = [
        ("rgb", C.c_void_p), ("out_color", C.c_void_p), ("out_others", C.c_void_p),
        ("radii", C.c_void_p),
    ]


class GradsIn(C.Structure):
    _fields_ = [("dL_dout_color", C.c_void_p), ("dL_dout_others", C.c_void_p), ("radii", C.c_void_p)]


class GradsOut(C.Structure):
    _fields_ = [
        ("dL_dmeans3D", C.c_void_p), ("dL_dmean2D", C.c_void_p), ("dL_dopacity", C.c_void_p),
        ("dL_dscales", C.c_void_p), ("dL_drots", C.c_void_p), ("dL_dtable", C.c_void_p),
        ("table_rows", C.c_int64), ("dL_gradsum", C.c_void_p), ("dL_dshapes", C.c_void_p),
        ("dL_dcolors_precomp", C.c_void_p), ("dL_dshs", C.c_void_p), ("dL_dtransmat_precomp", C.c_void_p),
    ]


_lib = None


class NestError(RuntimeError):
    def __init__(self, fn: str, status: int):
        lib = load()
        msg = lib.ns_status_string(status).decode()
        if status == NS_ERR_CUDA:
            msg += f" (cudaError {lib.ns_last_cuda_error()})"
        super().__init__(f"{fn}: {msg} [status {status}]")
        self.status = status


def load() -> C.CDLL:
    """Loads the library once; raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(f"{LIB_PATH} is missing: run `python nest-splatting_b200/build.py` "
                           "(there is no CPU fallback)")
    lib = C.CDLL(str(LIB_PATH), mode=os.RTLD_NOW | os.RTLD_GLOBAL)
    vp, i32, i64, sz = C.c_void_p, C.c_int32, C.c_int64, C.c_size_t
    lib.ns_status_string.restype = C.c_char_p
    lib.ns_status_string.argtypes = [C.c_int]
    lib.ns_last_cuda_error.restype = C.c_int
    lib.ns_kernel_launches.restype = C.c_uint64
    lib.ns_version.restype = C.c_int
    lib.ns_geometry_scratch_bytes.restype = sz
    lib.ns_geometry_scratch_bytes.argtypes = [i32]
    lib.ns_image_scratch_bytes.restype = sz
    lib.ns_image_scratch_bytes.argtypes = [i32, i32]
    lib.ns_binning_scratch_bytes.restype = sz
    lib.ns_binning_scratch_bytes.argtypes = [i64]
    lib.ns_rasterize_forward.restype = C.c_int
    lib.ns_rasterize_forward.argtypes = [C.POINTER(RasterSettings), C.POINTER(Surfels),
                                         C.POINTER(RasterOutputs), vp, sz, vp, sz, vp, sz,
                                         C.POINTER(C.c_int64), C.c_int, vp]
    lib.ns_read_device_status.restype = C.c_int
    lib.ns_read_device_status.argtypes = [vp, i32, vp]
    lib.ns_mark_visible.restype = C.c_int
    lib.ns_mark_visible.argtypes = [i32, vp, vp, vp, vp, vp]
    lib.ns_mlp_forward.restype = C.c_int
    lib.ns_mlp_forward.argtypes = [vp, i32, i64, vp, i32, i32, vp, vp, vp, vp]
    lib.ns_rvq_decode.restype = C.c_int
    lib.ns_rvq_decode.argtypes = [vp, vp, vp, i64, i32, i32, i32, vp]
    lib.ns_radix_sort_temp_bytes.restype = sz
    lib.ns_radix_sort_temp_bytes.argtypes = [i64]
    lib.ns_radix_sort_pairs.restype = C.c_int
    lib.ns_radix_sort_pairs.argtypes = [vp, vp, vp, vp, vp, vp, i64, i32, vp, sz, vp]
    lib.ns_radix_sort_pairs_noalloc.restype = C.c_int
    lib.ns_radix_sort_pairs_noalloc.argtypes = [vp, vp, vp, vp, i64, i32, vp]
    lib.ns_render_frame.restype = C.c_int
    lib.ns_render_frame.argtypes = [C.POINTER(RasterSettings), C.POINTER(FrameInputs),
                                    C.POINTER(FrameOutputs), vp, sz, vp, sz, vp, sz,
                                    C.POINTER(C.c_int64), C.c_int, vp]
    lib.ns_backward_scratch_bytes.restype = sz
    lib.ns_backward_scratch_bytes.argtypes = [i32]
    lib.ns_backward_scratch_bytes_deterministic.restype = sz
    lib.ns_backward_scratch_bytes_deterministic.argtypes = [i32, C.c_int64, i32]
    lib.ns_rasterize_backward.restype = C.c_int
    lib.ns_rasterize_backward.argtypes = [C.POINTER(RasterSettings), C.POINTER(Surfels), C.POINTER(GradsIn),
                                          C.POINTER(GradsOut), vp, sz, vp, sz, vp, sz, i64, vp, sz, vp]
    lib.ns_mlp_backward.restype = C.c_int
    lib.ns_mlp_backward.argtypes = [vp, i32, i64, vp, i32, i32, vp, vp, vp, vp, vp]
    lib.ns_allmap_decode.restype = C.c_int
    lib.ns_allmap_decode.argtypes = [vp, vp, vp, vp, i32, i32, C.c_float, vp, vp]
    lib.ns_normal_error.restype = C.c_int
    lib.ns_normal_error.argtypes = [vp, vp, vp, vp, i32, i32, vp, vp]
    lib.ns_normal_error_scratch_bytes.restype = sz
    lib.ns_normal_error_scratch_bytes.argtypes = [i32, i32]
    lib.ns_normal_error_backward.restype = C.c_int
    lib.ns_normal_error_backward.argtypes = [vp, vp, vp, vp, i32, i32, vp, i64, vp, vp, sz, vp]
    lib.ns_read_binning.restype = C.c_int
    lib.ns_read_binning.argtypes = [vp, sz, i32, vp, sz, vp, sz, i32, i32, i64, vp, vp, vp, vp, vp, vp, vp]
    u32, f32 = C.c_uint32, C.c_float
    lib.ns_grid_encode_forward.restype = C.c_int
    lib.ns_grid_encode_forward.argtypes = [vp, vp, i32, vp, vp, u32, u32, u32, u32, f32, u32, vp, u32, i32, u32,
                                           vp]
    lib.ns_grid_encode_backward.restype = C.c_int
    lib.ns_grid_encode_backward.argtypes = [vp, vp, vp, i32, vp, vp, u32, u32, u32, u32, f32, u32, vp, vp, u32,
                                            i32, u32, vp]
    lib.ns_set_wait_limit.restype = C.c_uint32
    lib.ns_set_wait_limit.argtypes = [C.c_uint32]
    lib.ns_wait_selftest.restype = C.c_int
    lib.ns_wait_selftest.argtypes = [vp, vp, i32, vp]
    lib.ns_gather_probe.restype = C.c_int
    lib.ns_gather_probe.argtypes = [vp, i32, vp, u32, u32, f32, u32, u32, f32, i32, vp, vp]
    _lib = lib
    return lib


def check(fn: str, status: int) -> None:
    if status != NS_OK:
        raise NestError(fn, status)


def ptr(t) -> int | None:
    """Device pointer of a tensor (None for None)."""
    if t is None:
        return None
    return t.data_ptr()


def stream_handle(device=None) -> int:
    import torch
    return torch.cuda.current_stream(device).cuda_stream
