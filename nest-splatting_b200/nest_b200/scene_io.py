"""On-disk scenes of the reference: the surfel PLY and the INGP checkpoint.

PLY (scene/gaussian_model.py:533-552 construct_list_of_attributes, :554-589
save_ply, :597-677 load_ply): one `vertex` element of float32 properties
x y z, nx ny nz, f_dc_0..2, f_rest_0..(3 (d+1)^2 - 4), opacity (logit),
scale_0..1 (log), rot_0..3 (raw quaternion), then optional gf_* (per-surfel
features of the cat modes) and `shape` (beta kernel). load_ply sets every
surfel's appearance level to 6 (`init_level`, :664-666); it is not stored.

INGP checkpoint `ngp_{iteration}.pth` (hash_encoder/modules.py:740-755):
torch.save({'model_state_dict': INGP.state_dict()}). The hash table is
`hash_encoding.embeddings` [sum_l T_l, level_dim] with `hash_encoding.offsets`
[L + 1] (gridencoder/grid.py:120-138). The colour MLP is tiny-cuda-nn's
`mlp_rgb.params`, one flat array of the layer matrices; tiny-cuda-nn is not
vendored in the reference, so `ngp_mlp_weights` states the layout it assumes.

A plain binary / ASCII PLY reader and writer (no plyfile dependency).
"""
from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path

import numpy as np
import torch

_PLY_TYPES = {
    "char": "i1", "int8": "i1", "uchar": "u1", "uint8": "u1", "short": "i2", "int16": "i2",
    "ushort": "u2", "uint16": "u2", "int": "i4", "int32": "i4", "uint": "u4", "uint32": "u4",
    "float": "f4", "float32": "f4", "double": "f8", "float64": "f8",
}


def read_ply(path) -> dict:
    """All properties of the `vertex` element as numpy arrays (name -> [N]), in
    file order. Binary little/big endian and ASCII; list properties are not
    supported (the reference writes none)."""
    data = Path(path).read_bytes()
    end = data.find(b"end_header")
    if not data.startswith(b"ply") or end < 0:
        raise ValueError(f"{path}: not a PLY file")
    nl = data.find(b"\n", end)
    header = data[:nl].decode("ascii").splitlines()
    body = data[nl + 1:]
    fmt, elements, cur = None, [], None
    for line in header[1:]:
        tok = line.split()
        if not tok or tok[0] in ("comment", "obj_info", "end_header"):
            continue
        if tok[0] == "format":
            fmt = tok[1]
        elif tok[0] == "element":
            cur = {"name": tok[1], "count": int(tok[2]), "props": []}
            elements.append(cur)
        elif tok[0] == "property":
            if tok[1] == "list":
                raise ValueError(f"{path}: list properties are not supported")
            if cur is None or tok[1] not in _PLY_TYPES:
                raise ValueError(f"{path}: bad property line {line!r}")
            cur["props"].append((tok[2], _PLY_TYPES[tok[1]]))
    if fmt not in ("binary_little_endian", "binary_big_endian", "ascii"):
        raise ValueError(f"{path}: unsupported PLY format {fmt!r}")
    out = None
    offset = 0
    text_rows = body.decode("ascii").split("\n") if fmt == "ascii" else None
    row = 0
    for el in elements:
        if fmt == "ascii":
            vals = np.array([[float(v) for v in text_rows[row + i].split()] for i in range(el["count"])],
                            dtype=np.float64).reshape(el["count"], len(el["props"]))
            row += el["count"]
            arrays = {n: vals[:, j].astype(t) for j, (n, t) in enumerate(el["props"])}
        else:
            e = "<" if fmt == "binary_little_endian" else ">"
            dt = np.dtype([(n, e + t) for n, t in el["props"]])
            arr = np.frombuffer(body, dtype=dt, count=el["count"], offset=offset)
            offset += dt.itemsize * el["count"]
            arrays = {n: arr[n].astype(arr[n].dtype.newbyteorder("=")) for n, _ in el["props"]}
        if el["name"] == "vertex":
            out = arrays
    if out is None:
        raise ValueError(f"{path}: no vertex element")
    return out


def write_ply(path, props: dict) -> None:
    """Binary little-endian PLY with one `vertex` element of float32 properties
    (name -> [N] array), in the dict's order."""
    names = list(props)
    n = len(props[names[0]])
    dt = np.dtype([(k, "<f4") for k in names])
    arr = np.empty(n, dtype=dt)
    for k in names:
        v = np.asarray(props[k], np.float32).reshape(-1)
        if len(v) != n:
            raise ValueError(f"property {k} has {len(v)} values, expected {n}")
        arr[k] = v
    head = ["ply", "format binary_little_endian 1.0", f"element vertex {n}"]
    head += [f"property float {k}" for k in names]
    head.append("end_header")
    Path(path).parent.mkdir(parents=True, exist_ok=True)
    Path(path).write_bytes(("\n".join(head) + "\n").encode("ascii") + arr.tobytes())


def _indexed(props: dict, prefix: str) -> list:
    names = [k for k in props if k.startswith(prefix) and k[len(prefix):].isdigit()]
    return sorted(names, key=lambda k: int(k[len(prefix):]))


@dataclass
class SurfelPLY:
    """Raw (pre-activation) surfel parameters as the reference stores them."""
    xyz: np.ndarray          # [N, 3]
    f_dc: np.ndarray         # [N, 3]
    f_rest: np.ndarray       # [N, 3 ((d+1)^2 - 1)], channel-major as saved
    opacity: np.ndarray      # [N, 1] logit
    scale: np.ndarray        # [N, 2] log
    rotation: np.ndarray     # [N, 4] raw quaternion (w, x, y, z)
    gf: np.ndarray | None = None     # [N, F] per-surfel features (cat modes)
    shape: np.ndarray | None = None  # [N, 1] beta-kernel shape

    @property
    def P(self) -> int:
        return self.xyz.shape[0]


def load_surfel_ply(path, max_sh_degree: int | None = None) -> SurfelPLY:
    """scene/gaussian_model.py load_ply (:597-677), reading the same names."""
    p = read_ply(path)
    xyz = np.stack([p["x"], p["y"], p["z"]], 1).astype(np.float32)
    f_dc = np.stack([p[f"f_dc_{i}"] for i in range(3)], 1).astype(np.float32)
    rest = _indexed(p, "f_rest_")
    if max_sh_degree is not None and len(rest) != 3 * (max_sh_degree + 1) ** 2 - 3:
        raise ValueError(f"{path}: {len(rest)} f_rest properties, SH degree {max_sh_degree} needs "
                         f"{3 * (max_sh_degree + 1) ** 2 - 3}")
    f_rest = (np.stack([p[k] for k in rest], 1) if rest else np.zeros((len(xyz), 0))).astype(np.float32)
    scale = np.stack([p[k] for k in _indexed(p, "scale_")], 1).astype(np.float32)
    rot = np.stack([p[k] for k in _indexed(p, "rot_")], 1).astype(np.float32)
    gf_names = _indexed(p, "gf_")
    gf = np.stack([p[k] for k in gf_names], 1).astype(np.float32) if gf_names else None
    shape = p["shape"][:, None].astype(np.float32) if "shape" in p else None
    return SurfelPLY(xyz, f_dc, f_rest, p["opacity"][:, None].astype(np.float32), scale, rot, gf, shape)


def save_surfel_ply(path, s: SurfelPLY) -> None:
    """scene/gaussian_model.py save_ply (:554-589): the reference's property order,
    normals written as zeros."""
    props = {"x": s.xyz[:, 0], "y": s.xyz[:, 1], "z": s.xyz[:, 2]}
    for k in ("nx", "ny", "nz"):
        props[k] = np.zeros(s.P, np.float32)
    for i in range(s.f_dc.shape[1]):
        props[f"f_dc_{i}"] = s.f_dc[:, i]
    for i in range(s.f_rest.shape[1]):
        props[f"f_rest_{i}"] = s.f_rest[:, i]
    props["opacity"] = s.opacity[:, 0]
    for i in range(s.scale.shape[1]):
        props[f"scale_{i}"] = s.scale[:, i]
    for i in range(s.rotation.shape[1]):
        props[f"rot_{i}"] = s.rotation[:, i]
    if s.gf is not None:
        for i in range(s.gf.shape[1]):
            props[f"gf_{i}"] = s.gf[:, i]
    if s.shape is not None:
        props["shape"] = s.shape[:, 0]
    write_ply(path, props)


INIT_APPEARANCE_LEVEL = 6.0  # load_ply's init_level (gaussian_model.py:664-666)


def from_model_tensors(xyz, features_dc, features_rest, opacity, scaling, rotation,
                       gaussian_features=None, shape=None) -> SurfelPLY:
    """A SurfelPLY from GaussianModel's parameter tensors as save_ply
    (gaussian_model.py:557-584) flattens them: features_dc [N, 1, 3] and
    features_rest [N, (d+1)^2 - 1, 3] transposed to channel-major rows, empty
    gaussian_features / shape left out."""
    a = lambda t: (t.detach().cpu().numpy() if torch.is_tensor(t) else np.asarray(t)).astype(np.float32)  # noqa: E731
    n = a(xyz).shape[0]
    dc = a(features_dc).transpose(0, 2, 1).reshape(n, -1)
    rest = a(features_rest).transpose(0, 2, 1).reshape(n, -1)
    gf = a(gaussian_features) if gaussian_features is not None and np.size(a(gaussian_features)) else None
    sh = a(shape).reshape(n, 1) if shape is not None and np.size(a(shape)) else None
    return SurfelPLY(a(xyz), dc, rest, a(opacity).reshape(n, 1), a(scaling), a(rotation), gf, sh)


def model_tensors(s: SurfelPLY, device="cpu") -> dict:
    """GaussianModel's parameter tensors as load_ply (gaussian_model.py:601-666)
    rebuilds them: features_dc [N, 1, 3], features_rest [N, (d+1)^2 - 1, 3] from
    the channel-major rows, appearance_level at its initial value, and
    gaussian_features / shape when the file has them."""
    t = lambda x: torch.as_tensor(np.ascontiguousarray(x), dtype=torch.float32, device=device)  # noqa: E731
    n = s.P
    out = {"xyz": t(s.xyz), "features_dc": t(s.f_dc.reshape(n, 3, 1)).transpose(1, 2).contiguous(),
           "features_rest": t(s.f_rest.reshape(n, 3, -1)).transpose(1, 2).contiguous(),
           "opacity": t(s.opacity), "scaling": t(s.scale), "rotation": t(s.rotation),
           "appearance_level": torch.full((n, 1), INIT_APPEARANCE_LEVEL, device=device)}
    if s.gf is not None:
        out["gaussian_features"] = t(s.gf)
    if s.shape is not None:
        out["shape"] = t(s.shape)
    return out


def rasterizer_inputs(s: SurfelPLY, device="cuda", ap_level: float = INIT_APPEARANCE_LEVEL,
                      base_opacity: float = 0.0) -> dict:
    """Activated tensors for the rasterizer (gaussian_model.py:231-281): exp
    scales, normalised quaternions, sigmoid(opacity) * (1 - base) + base, and the
    appearance level load_ply assigns."""
    t = lambda a: torch.as_tensor(a, dtype=torch.float32, device=device)  # noqa: E731
    rot = t(s.rotation)
    rot = rot / rot.norm(dim=1, keepdim=True).clamp_min(1e-12)
    op = torch.sigmoid(t(s.opacity)) * (1.0 - base_opacity) + base_opacity
    return {"means3D": t(s.xyz).contiguous(), "scales": torch.exp(t(s.scale)).contiguous(),
            "rotations": rot.contiguous(), "opacities": op.contiguous(),
            "ap_level": torch.full((s.P, 1), float(ap_level), device=device)}


def load_ngp(path) -> dict:
    """hash table, offsets and the raw MLP parameter array of ngp_{it}.pth."""
    ck = torch.load(path, map_location="cpu", weights_only=False)
    sd = ck["model_state_dict"] if "model_state_dict" in ck else ck
    out = {"table": sd["hash_encoding.embeddings"].float().contiguous(),
           "offsets": sd["hash_encoding.offsets"].to(torch.int32).contiguous()}
    if "mlp_rgb.params" in sd:
        out["mlp_params"] = sd["mlp_rgb.params"].float().contiguous()
    return out


def ngp_mlp_weights(params: torch.Tensor, n_in: int = 32, hidden: int = 64, n_hidden_layers: int = 2,
                    n_out: int = 3, pad: int = 16) -> list:
    """Layer matrices [out, in] of a bias-free tiny-cuda-nn MLP from its flat
    parameter array, ASSUMING the layers are stored one after another, each
    row-major [out, in], with the output layer's rows padded to a multiple of
    `pad`. tiny-cuda-nn is not part of the reference, so this layout is not
    pinned by any file or test here."""
    widths = [n_in] + [hidden] * n_hidden_layers
    outs = [hidden] * n_hidden_layers + [-(-n_out // pad) * pad]
    need = sum(i * o for i, o in zip(widths, outs))
    if params.numel() != need:
        raise ValueError(f"MLP parameter count {params.numel()} != {need} for the assumed layout")
    mats, off = [], 0
    for i, o in zip(widths, outs):
        mats.append(params[off:off + o * i].reshape(o, i))
        off += o * i
    mats[-1] = mats[-1][:n_out]
    return mats
