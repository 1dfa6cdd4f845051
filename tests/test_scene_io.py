"""Scene files: the reference's surfel PLY (attribute names and order of
scene/gaussian_model.py:533-589) and the INGP checkpoint layout."""
import numpy as np
import pytest
import torch

from nest_b200 import scene_io


def make_surfels(n=50, sh_degree=3, gf=0, shape=False, seed=0):
    rng = np.random.default_rng(seed)
    f = lambda *s: rng.standard_normal(s).astype(np.float32)  # noqa: E731
    return scene_io.SurfelPLY(f(n, 3), f(n, 3), f(n, 3 * (sh_degree + 1) ** 2 - 3), f(n, 1), f(n, 2), f(n, 4),
                              f(n, gf) if gf else None, f(n, 1) if shape else None)


def reference_attribute_names(sh_degree, gf=0, shape=False):
    """construct_list_of_attributes (gaussian_model.py:533-552) for 2D surfels."""
    names = ["x", "y", "z", "nx", "ny", "nz"] + [f"f_dc_{i}" for i in range(3)]
    names += [f"f_rest_{i}" for i in range(3 * (sh_degree + 1) ** 2 - 3)]
    names += ["opacity", "scale_0", "scale_1"] + [f"rot_{i}" for i in range(4)]
    names += [f"gf_{i}" for i in range(gf)] + (["shape"] if shape else [])
    return names


@pytest.mark.parametrize("gf,shape", [(0, False), (8, True)])
def test_ply_roundtrip_in_reference_order(tmp_path, gf, shape):
    s = make_surfels(gf=gf, shape=shape)
    path = tmp_path / "point_cloud.ply"
    scene_io.save_surfel_ply(path, s)
    head = path.read_bytes().split(b"end_header")[0].decode()
    props = [line.split()[2] for line in head.splitlines() if line.startswith("property")]
    assert props == reference_attribute_names(3, gf, shape)
    assert "element vertex 50" in head and "binary_little_endian" in head
    r = scene_io.load_surfel_ply(path, max_sh_degree=3)
    for k in ("xyz", "f_dc", "f_rest", "opacity", "scale", "rotation"):
        assert np.array_equal(getattr(r, k), getattr(s, k)), k
    assert (r.gf is None) == (s.gf is None) and (r.shape is None) == (s.shape is None)
    if gf:
        assert np.array_equal(r.gf, s.gf) and np.array_equal(r.shape, s.shape)
    assert np.all(scene_io.read_ply(path)["nx"] == 0)


def test_ply_ascii_big_endian_and_property_order(tmp_path):
    names = ["rot_3", "x", "y", "z", "f_dc_0", "f_dc_1", "f_dc_2", "opacity", "scale_1", "scale_0",
             "rot_0", "rot_1", "rot_2", "extra"]
    rng = np.random.default_rng(1)
    vals = rng.standard_normal((4, len(names))).astype(np.float32)
    head = "ply\nformat {fmt} 1.0\ncomment made by a test\nelement vertex 4\n" + "".join(
        f"property float {n}\n" for n in names) + "end_header\n"
    (tmp_path / "a.ply").write_bytes(head.format(fmt="ascii").encode() +
                                     "\n".join(" ".join(repr(float(v)) for v in row) for row in vals).encode())
    (tmp_path / "b.ply").write_bytes(head.format(fmt="binary_big_endian").encode() + vals.astype(">f4").tobytes())
    for f in ("a.ply", "b.ply"):
        r = scene_io.load_surfel_ply(tmp_path / f)
        col = {n: vals[:, i] for i, n in enumerate(names)}
        assert np.allclose(r.scale, np.stack([col["scale_0"], col["scale_1"]], 1))
        assert np.allclose(r.rotation, np.stack([col[f"rot_{i}"] for i in range(4)], 1))
        assert r.f_rest.shape == (4, 0)


def test_ply_rejects_wrong_sh_degree_and_lists(tmp_path):
    s = make_surfels(sh_degree=1)
    scene_io.save_surfel_ply(tmp_path / "p.ply", s)
    with pytest.raises(ValueError):
        scene_io.load_surfel_ply(tmp_path / "p.ply", max_sh_degree=3)
    (tmp_path / "l.ply").write_bytes(b"ply\nformat ascii 1.0\nelement vertex 1\n"
                                     b"property list uchar int idx\nend_header\n1 0\n")
    with pytest.raises(ValueError):
        scene_io.read_ply(tmp_path / "l.ply")


def test_rasterizer_inputs_activations():
    s = make_surfels(n=10)
    t = scene_io.rasterizer_inputs(s, device="cpu", base_opacity=0.1)
    assert torch.allclose(t["scales"], torch.exp(torch.from_numpy(s.scale)))
    q = torch.from_numpy(s.rotation)
    assert torch.allclose(t["rotations"], q / q.norm(dim=1, keepdim=True))
    assert torch.allclose(t["opacities"], torch.sigmoid(torch.from_numpy(s.opacity)) * 0.9 + 0.1)
    assert torch.all(t["ap_level"] == scene_io.INIT_APPEARANCE_LEVEL)


def test_ngp_checkpoint_layout(tmp_path):
    table = torch.randn(100, 2)
    offsets = torch.tensor([0, 40, 100], dtype=torch.int32)
    w = [torch.randn(64, 32), torch.randn(64, 64), torch.randn(16, 64)]
    params = torch.cat([m.reshape(-1) for m in w]).half()
    torch.save({"model_state_dict": {"hash_encoding.embeddings": table, "hash_encoding.offsets": offsets,
                                     "mlp_rgb.params": params}}, tmp_path / "ngp_30000.pth")
    ck = scene_io.load_ngp(tmp_path / "ngp_30000.pth")
    assert torch.equal(ck["table"], table) and torch.equal(ck["offsets"], offsets)
    mats = scene_io.ngp_mlp_weights(ck["mlp_params"])
    assert [tuple(m.shape) for m in mats] == [(64, 32), (64, 64), (3, 64)]
    assert torch.equal(mats[2], w[2][:3].half().float())
    with pytest.raises(ValueError):
        scene_io.ngp_mlp_weights(ck["mlp_params"][:-1])


REF_PLY = np.load(__import__("pathlib").Path(__file__).resolve().parent / "golden" / "reference_ply.npz")


@pytest.mark.parametrize("case", [0, 1, 2])
def test_ply_writer_matches_reference_save_ply(tmp_path, case):
    """The reference's save_ply (run unmodified by tests/golden/make_ply_golden.py)
    on the same parameter tensors: same property names in the same order and
    the same float32 records, bit for bit."""
    g = lambda k: REF_PLY[f"case{case}_saved{k}"]  # noqa: E731
    _, _, gf, shape = REF_PLY[f"case{case}_meta"]
    s = scene_io.from_model_tensors(g("_xyz"), g("_features_dc"), g("_features_rest"), g("_opacity"),
                                    g("_scaling"), g("_rotation"), g("_gaussian_features") if gf else None,
                                    g("_shape") if shape else None)
    path = tmp_path / "point_cloud.ply"
    scene_io.save_surfel_ply(path, s)
    head, body = path.read_bytes().split(b"end_header\n", 1)
    props = [line.split()[2] for line in head.decode().splitlines() if line.startswith("property")]
    assert props == [str(n) for n in REF_PLY[f"case{case}_names"]]
    rec = np.frombuffer(body, "<f4").reshape(REF_PLY[f"case{case}_records"].shape)
    assert np.array_equal(rec, REF_PLY[f"case{case}_records"])


@pytest.mark.parametrize("case", [0, 1, 2])
def test_ply_reader_matches_reference_load_ply(tmp_path, case):
    """The reference's load_ply on the records its save_ply wrote: the same
    parameter tensors from load_surfel_ply + model_tensors, bit for bit."""
    names = [str(n) for n in REF_PLY[f"case{case}_names"]]
    recs = REF_PLY[f"case{case}_records"]
    head = (f"ply\nformat binary_little_endian 1.0\nelement vertex {recs.shape[0]}\n"
            + "".join(f"property float {n}\n" for n in names) + "end_header\n")
    path = tmp_path / "point_cloud.ply"
    path.write_bytes(head.encode() + recs.astype("<f4").tobytes())
    deg = int(REF_PLY[f"case{case}_meta"][1])
    m = scene_io.model_tensors(scene_io.load_surfel_ply(path, max_sh_degree=deg))
    ref = {"xyz": "_xyz", "features_dc": "_features_dc", "features_rest": "_features_rest",
           "opacity": "_opacity", "scaling": "_scaling", "rotation": "_rotation", "appearance_level": "_ap_level"}
    _, _, gf, shape = REF_PLY[f"case{case}_meta"]
    if gf:
        ref["gaussian_features"] = "_gaussian_features"
    if shape:
        ref["shape"] = "_shape"
    assert set(m) == set(ref)
    for k, rk in ref.items():
        want = REF_PLY[f"case{case}_loaded{rk}"]
        assert m[k].shape == want.shape, k
        assert np.array_equal(m[k].numpy(), want), k
