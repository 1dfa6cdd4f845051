"""GPU parity of the tensor-core MLP and of the fused RVQ frame
(decode -> activate -> rasterize -> MLP -> mask) against the CPU oracle chain."""
import numpy as np
import pytest
import torch

from helpers import api_inputs, oracle_render, psnr, raw_attributes, small_scene
from nest_b200 import raster, synth
from nest_b200.frame import FrameRenderer
from oracle import oracle

pytestmark = pytest.mark.gpu
TOL = 2e-3


@pytest.mark.parametrize("npix", [1, 15, 16, 1000, 77_777])
def test_mlp_matches_oracle(npix):
    g = torch.Generator().manual_seed(npix)
    ws = synth.xavier_mlp(g)
    feat = torch.randn(32, npix, generator=g) * 2.0
    alpha = torch.rand(npix, generator=g)
    alpha[::5] = 0.0
    rgb = raster.mlp_forward(feat.cuda(), raster.pack_mlp(ws).cuda(), alpha.cuda()).cpu().numpy()
    ref = oracle.mlp_oracle(feat.numpy(), ws, alpha.numpy())
    assert np.abs(rgb - ref).max() <= TOL
    assert np.all(rgb[:, ::5] == 0)


def test_mlp_background():
    g = torch.Generator().manual_seed(7)
    ws = synth.xavier_mlp(g)
    feat = torch.randn(32, 40, 30, generator=g)
    alpha = torch.rand(40, 30, generator=g)
    bg = np.array([0.2, 0.5, 1.0], np.float32)
    rgb = raster.mlp_forward(feat.cuda(), raster.pack_mlp(ws).cuda(), alpha.cuda(), bg=bg).cpu().numpy()
    ref = oracle.mlp_oracle(feat.numpy(), ws, alpha.numpy(), bg=bg)
    assert np.abs(rgb - ref).max() <= TOL


def frame_oracle(sc):
    decoded = torch.from_numpy(oracle.rvq_decode_np(sc.rvq_idx.numpy(), sc.codebooks.numpy()))
    raw = raw_attributes(sc, decoded)
    inp = api_inputs(sc, raw)
    out, pre, n = oracle_render(sc, inp)
    rgb = oracle.mlp_oracle(out["out_color"], sc.mlp, out["out_others"][1])
    return decoded.numpy(), out, pre, n, rgb


@pytest.mark.parametrize("table_range", [1e-4, 1.0])
def test_fused_frame_matches_oracle(table_range):
    sc = small_scene(n=2500, seed=21, rvq=True, table_range=table_range)
    decoded, out, pre, n, rgb_ref = frame_oracle(sc)
    fr = FrameRenderer(sc)
    rgb = fr.render(sc.camera)
    torch.cuda.synchronize()
    assert np.array_equal(fr.decoded.cpu().numpy().view(np.uint32), decoded.view(np.uint32))
    # Tile instances: the reference's rectangles minus the tiles the surfel's
    # alpha box (alpha >= 1/255) does not reach, so never more than the oracle's.
    assert 0 < fr.num_rendered <= n
    feats = fr.features.cpu().numpy()
    assert np.abs(feats - out["out_color"]).max() <= TOL
    others = fr.others.cpu().numpy()
    for ch in (0, 1, 2, 3, 4, 5):
        assert np.abs(others[ch] - out["out_others"][ch]).max() <= TOL * max(1.0, np.abs(out["out_others"][ch]).max())
    rgb = rgb.cpu().numpy()
    assert np.abs(rgb - rgb_ref).max() <= TOL
    assert psnr(rgb, rgb_ref) >= 60


def test_fused_frame_repeatable_and_index_upload():
    sc = small_scene(n=2000, seed=22, rvq=True)
    fr = FrameRenderer(sc)
    a = fr.render(sc.camera).clone()
    host = sc.rvq_idx.clone().pin_memory()
    fr.upload_indices(host)
    b = fr.render(sc.camera).clone()
    torch.cuda.synchronize()
    assert torch.equal(a, b)


@pytest.mark.parametrize("graphs", [False, True])
def test_frame_pipeline_sequence_matches_single_frames(graphs):
    """FramePipeline: every frame's image, copied back to the host, equals the same
    frame rendered alone (frames alternate between two index streams and cameras;
    graphs=True replays one captured frame per buffer set)."""
    from nest_b200.camera import orbit_camera
    from nest_b200.frame import FramePipeline

    sc = small_scene(n=3000, seed=23, rvq=True)
    fr = FrameRenderer(sc)
    W, H = sc.camera.width, sc.camera.height
    cams = [orbit_camera(W, H, 50.0, 4.0, az) for az in (0.0, 40.0)]
    g = torch.Generator().manual_seed(5)
    streams = [sc.rvq_idx.clone(), torch.randint(0, 256, sc.rvq_idx.shape, generator=g).to(torch.uint8)]
    ref = []
    for i in range(2):
        fr.upload_indices(streams[i].cuda())
        ref.append(fr.render(cams[i]).cpu())
    host_idx = [s.pin_memory() for s in streams]
    host_cam = [torch.stack([c.world_view_transform, c.full_proj_transform]).contiguous().pin_memory()
                for c in cams]
    n = 7
    host_rgb = [torch.empty((3, H, W)).pin_memory() for _ in range(n)]
    pipe = FramePipeline(fr, graphs=graphs)
    pipe.run(n, cams[0], lambda i: host_idx[i % 2], lambda i: host_cam[i % 2], lambda i: host_rgb[i])
    torch.cuda.synchronize()
    for i in range(n):
        assert torch.equal(host_rgb[i], ref[i % 2]), i


def test_frame_graph_replays_the_frame():
    """FrameGraph: the frame with the device-side instance count, captured as a
    CUDA graph, gives the same image bits as the host-count frame, also after
    new indices are uploaded into the captured buffer."""
    from nest_b200.frame import FrameGraph
    sc = small_scene(n=2500, seed=21, rvq=True)
    fr = FrameRenderer(sc)
    cam = sc.camera
    view = cam.world_view_transform.cuda().contiguous()
    proj = cam.full_proj_transform.cuda().contiguous()
    ref = fr.render(cam, view, proj).clone()
    graph = FrameGraph(fr, cam, view, proj)
    out = graph.replay().clone()
    torch.cuda.synchronize()
    assert graph.status() == 0
    assert torch.equal(out, ref) and ref.abs().sum() > 0
    g = torch.Generator().manual_seed(5)
    new_idx = torch.randint(0, sc.codebooks.shape[1], sc.rvq_idx.shape, generator=g).to(torch.uint8)
    fr.upload_indices(new_idx.cuda())
    out2 = graph.replay().clone()
    ref2 = fr.render(cam, view, proj).clone()
    torch.cuda.synchronize()
    assert torch.equal(out2, ref2) and not torch.equal(out2, ref)


def test_device_count_overflow_reports_error():
    """Device-count mode with binning buffers too small: the frame renders no
    instances and the device error word reports it (no host check in between)."""
    from nest_b200 import _lib
    sc = small_scene(n=2500, seed=21, rvq=True)
    fr = FrameRenderer(sc, capacity=100)
    cam = sc.camera
    fr._extra_flags = _lib.NS_FLAG_DEVICE_COUNT
    try:
        rgb = fr.render(cam).clone()
    finally:
        fr._extra_flags = 0
    lib = _lib.load()
    st = lib.ns_read_device_status(fr.scratch.geom.data_ptr(), fr.P, _lib.stream_handle(fr.device))
    assert st == _lib.NS_ERR_DEVICE
    assert not rgb.any()
    assert lib.ns_read_device_status(fr.scratch.geom.data_ptr(), fr.P, _lib.stream_handle(fr.device)) == 0
