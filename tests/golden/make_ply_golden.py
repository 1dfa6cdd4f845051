"""Generates tests/golden/reference_ply.npz from the reference's own surfel
PLY code: scene/gaussian_model.py construct_list_of_attributes (:533-552),
save_ply (:554-589) and load_ply (:597-685), run unmodified.

Run in a container where the reference checkout is importable:
    python tests/golden/make_ply_golden.py /path/to/nest-splatting

What stands in for what is absent here (the arithmetic of the reference's
code is unchanged):
  * plyfile is not installed. A stand-in PlyElement / PlyData keeps the
    structured vertex array that save_ply builds (exactly the records it would
    write) and hands a recorded array back to load_ply through the same
    interface (`elements[0][name]`, `elements[0].properties[i].name`);
  * simple_knn._C (used only when creating a model from a point cloud) is an
    empty module;
  * device='cuda' in torch.tensor / zeros / ones / empty and Tensor.cuda()
    are redirected to the CPU for the duration of the calls;
  * GaussianModel.__init__ (optimiser and activation set-up) is skipped: the
    three methods only read and write the parameter tensors.
The fixture holds, per case, the model tensors save_ply was given, the field
names and float32 records it produced, and the tensors load_ply rebuilt from
those records. Tests never import the reference.
"""
from __future__ import annotations

import importlib.util
import sys
import tempfile
import types
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent / "reference_ply.npz"

CASES = [  # (surfels, SH degree, per-surfel feature width, beta shape present)
    (7, 3, 0, False),
    (5, 3, 8, True),
    (4, 0, 0, False),
]


class _Prop:
    def __init__(self, name):
        self.name = name


class _Element:
    def __init__(self, arr):
        self.data = arr
        self.properties = [_Prop(n) for n in arr.dtype.names]

    def __getitem__(self, name):
        return self.data[name]


class _PlyStub:
    written = None   # the structured array of the last save_ply
    to_read = None   # the structured array the next load_ply reads

    class PlyElement:
        @staticmethod
        def describe(arr, name):
            assert name == "vertex"
            return _Element(arr)

    class PlyData:
        def __init__(self, elements):
            self.elements = elements

        def write(self, path):
            _PlyStub.written = self.elements[0].data.copy()

        @staticmethod
        def read(path):
            return _PlyStub.PlyData([_Element(_PlyStub.to_read)])


def _cpu_device_shim():
    saved = {k: getattr(torch, k) for k in ("tensor", "zeros", "ones", "empty")}

    def drop_device(fn):
        def call(*a, **k):
            k.pop("device", None)
            return fn(*a, **k)
        return call

    for k, fn in saved.items():
        setattr(torch, k, drop_device(fn))
    real_cuda = torch.Tensor.cuda
    torch.Tensor.cuda = lambda self, *a, **k: self

    def undo():
        for k, fn in saved.items():
            setattr(torch, k, fn)
        torch.Tensor.cuda = real_cuda

    return undo


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    ply = types.ModuleType("plyfile")
    ply.PlyData, ply.PlyElement = _PlyStub.PlyData, _PlyStub.PlyElement
    sys.modules["plyfile"] = ply
    knn = types.ModuleType("simple_knn")
    knn._C = types.ModuleType("simple_knn._C")
    knn._C.distCUDA2 = None
    sys.modules["simple_knn"], sys.modules["simple_knn._C"] = knn, knn._C
    spec = importlib.util.spec_from_file_location("gaussian_model", Path(ref_root) / "scene" / "gaussian_model.py")
    gm = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(gm)

    class Model(gm.GaussianModel):
        def __init__(self, sh_degree):  # parameters only (see the module docstring)
            self.max_sh_degree = sh_degree
            self.env_map = None

    data = {}
    g = torch.Generator().manual_seed(2024)
    for c, (n, deg, gf, shape) in enumerate(CASES):
        r = lambda *s: torch.randn(*s, generator=g)  # noqa: E731
        m = Model(deg)
        m._xyz = r(n, 3)
        m._features_dc = r(n, 1, 3)
        m._features_rest = r(n, (deg + 1) ** 2 - 1, 3)
        m._opacity = r(n, 1)
        m._scaling = r(n, 2)
        m._rotation = r(n, 4)
        m._gaussian_feat_dim = gf
        m._gaussian_features = r(n, gf) if gf else torch.empty(0)
        m._shape = r(n, 1) if shape else torch.empty(0)
        undo = _cpu_device_shim()
        try:
            with tempfile.TemporaryDirectory() as d:
                m.save_ply(str(Path(d) / "point_cloud.ply"))
            rec = _PlyStub.written
            back = Model(deg)
            _PlyStub.to_read = rec
            back.load_ply("point_cloud.ply")
        finally:
            undo()
        data[f"case{c}_meta"] = np.array([n, deg, gf, int(shape)], np.int64)
        data[f"case{c}_names"] = np.array(rec.dtype.names)
        data[f"case{c}_records"] = np.stack([rec[k] for k in rec.dtype.names], 1).astype(np.float32)
        for k in ("_xyz", "_features_dc", "_features_rest", "_opacity", "_scaling", "_rotation"):
            data[f"case{c}_saved{k}"] = getattr(m, k).numpy()
            data[f"case{c}_loaded{k}"] = getattr(back, k).detach().numpy()
        if gf:
            data[f"case{c}_saved_gaussian_features"] = m._gaussian_features.numpy()
            data[f"case{c}_loaded_gaussian_features"] = back._gaussian_features.detach().numpy()
        if shape:
            data[f"case{c}_saved_shape"] = m._shape.numpy()
            data[f"case{c}_loaded_shape"] = back._shape.detach().numpy()
        data[f"case{c}_loaded_ap_level"] = back._appearance_level.detach().numpy()
    np.savez(OUT, **data)
    print("wrote", OUT)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python make_ply_golden.py <path to the reference repository checkout>")
    main(sys.argv[1])
