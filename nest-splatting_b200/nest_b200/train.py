"""One training step of the baseline render mode (benchmark config 4), on torch
autograd around the library's kernels.

Forward: the drop-in rasterizer (ns_rasterize_forward) -> the fp16 MLP
(ns_mlp_forward) -> the losses, the depth-normal term fused into one kernel
(ns_normal_error). Backward: ns_normal_error_backward for that term,
ns_mlp_backward for the MLP (features and weights), ns_rasterize_backward for
the surfels and the hash table.

Restated from the reference: the allmap decode (gaussian_renderer/__init__.py
:763-797: alpha, view-to-world normal, expected depth = depth / alpha with NaN
-> 0, surf_normal = depth_to_normal(expected depth) * alpha.detach(),
depth_ratio 0), depth_to_normal / depths_to_points (utils/point_utils.py
:10-30, 48-60) and the losses of train.py:651-675 used by config 4:
L1(rgb, target) + lambda_normal * mean(1 - sum_c rend_normal * surf_normal).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

from . import raster


class _MLP(torch.autograd.Function):
    """rgb [3,H,W] = sigmoid(W3 relu(W2 relu(W1 feat)))[:3] * (alpha > 0) (+ (1 - alpha) bg).

    Forward on the library's tensor-core kernel (fp16 operands, fp32
    accumulation, each layer rounded to fp16). Backward on the library's fused
    kernel (ns_mlp_backward: the forward recomputed, the backward on TF32
    tensor cores in fp32 range -- the per-pixel gradients of a mean loss over
    megapixels are ~1e-7, below fp16's normal range -- and the weight
    gradients reduced on chip); the fp16 roundings are treated as identity.
    """

    @staticmethod
    def forward(ctx, feat, w1, w2, w3, alpha, bg):
        packed = raster.pack_mlp([w1.detach(), w2.detach(), w3.detach()])
        feat_c = feat.detach().contiguous()
        alpha_c = alpha.detach().contiguous()
        rgb = raster.mlp_forward(feat_c, packed, alpha=alpha_c, bg=bg, hidden=w1.shape[0])
        ctx.save_for_backward(feat_c, packed, alpha_c)
        ctx.shapes = (w1.shape, w2.shape, w3.shape, w1.dtype)
        ctx.bg = bg
        return rgb

    @staticmethod
    def backward(ctx, grgb):
        feat, packed, alpha = ctx.saved_tensors
        (s1, s2, s3, wdt) = ctx.shapes
        dfeat, dW = raster.mlp_backward(feat, packed, grgb, alpha=alpha, hidden=s1[0])
        n1, n2 = s1.numel(), s2.numel()
        dW1, dW2, dW3 = dW[:n1].view(s1), dW[n1:n1 + n2].view(s2), dW[n1 + n2:].view(s3)
        dalpha = None
        bg = ctx.bg
        if ctx.needs_input_grad[4]:
            dalpha = torch.zeros_like(alpha)
            if bg is not None and float(sum(float(b) for b in bg)) > 0:
                bgt = torch.as_tensor([float(b) for b in bg], device=grgb.device).view(3, *([1] * (grgb.dim() - 1)))
                dalpha = -(grgb.float() * bgt).sum(0).reshape(alpha.shape)
        return dfeat.to(feat.dtype), dW1.to(wdt), dW2.to(wdt), dW3.to(wdt), dalpha, None


def mlp(feat, w1, w2, w3, alpha, bg=None):
    return _MLP.apply(feat, w1, w2, w3, alpha, bg)


_RAYS = {}


def _camera_rays(cam, dev):
    """Per-pixel ray directions and origin of utils/point_utils.py:10-30, computed
    once per camera (the reference recomputes them, with a 3x3 inverse, per call)."""
    key = (id(cam), cam.width, cam.height, str(dev))
    hit = _RAYS.get(key)
    if hit is not None and hit[0] is cam:
        return hit[1], hit[2]
    W, H = cam.width, cam.height
    wv = cam.world_view_transform.to(dev)
    c2w = wv.T.inverse()
    ndc2pix = torch.tensor([[W / 2, 0, 0, W / 2], [0, H / 2, 0, H / 2], [0, 0, 0, 1]],
                           dtype=torch.float32, device=dev).T
    proj = c2w.T @ cam.full_proj_transform.to(dev)
    intrins = (proj @ ndc2pix)[:3, :3].T
    gx, gy = torch.meshgrid(torch.arange(W, device=dev).float(), torch.arange(H, device=dev).float(), indexing="xy")
    pts = torch.stack([gx, gy, torch.ones_like(gx)], dim=-1).reshape(-1, 3)
    rays_d = pts @ intrins.inverse().T @ c2w[:3, :3].T
    rays_o = c2w[:3, 3]
    if len(_RAYS) > 64:
        _RAYS.clear()
    _RAYS[key] = (cam, rays_d, rays_o)
    return rays_d, rays_o


def depths_to_points(cam, depthmap):
    """utils/point_utils.py:10-30: pixel rays scaled by depth (world points [H*W, 3])."""
    rays_d, rays_o = _camera_rays(cam, depthmap.device)
    return depthmap.reshape(-1, 1) * rays_d + rays_o


def depth_to_normal(cam, depth):
    """utils/point_utils.py:48-60: normals from central differences of the points."""
    pts = depths_to_points(cam, depth).reshape(*depth.shape[1:], 3)
    out = torch.zeros_like(pts)
    dx = pts[2:, 1:-1] - pts[:-2, 1:-1]
    dy = pts[1:-1, 2:] - pts[1:-1, :-2]
    out[1:-1, 1:-1, :] = F.normalize(torch.cross(dx, dy, dim=-1), dim=-1)
    return out


def decode_allmap(allmap, cam):
    """gaussian_renderer/__init__.py:763-797 (depth_ratio 0): alpha [1,H,W],
    world-space rend_normal [3,H,W], surf_normal [3,H,W], expected depth [1,H,W]."""
    alpha = allmap[1:2]
    wv = cam.world_view_transform.to(allmap.device)
    rend_normal = (allmap[2:5].permute(1, 2, 0) @ wv[:3, :3].T).permute(2, 0, 1)
    depth = torch.nan_to_num(allmap[0:1] / alpha, 0, 0)
    surf_normal = depth_to_normal(cam, depth).permute(2, 0, 1) * alpha.detach()
    return alpha, rend_normal, surf_normal, depth


class _NormalError(torch.autograd.Function):
    """normal_error [H, W] of train.py:674 from the allmap, on the library's kernels."""

    @staticmethod
    def forward(ctx, allmap, viewmatrix, rays_d, ray_o):
        allmap = allmap.detach().contiguous()
        ctx.save_for_backward(allmap, viewmatrix, rays_d, ray_o)
        return raster.normal_error(allmap, viewmatrix, rays_d, ray_o)

    @staticmethod
    def backward(ctx, gerr):
        allmap, viewmatrix, rays_d, ray_o = ctx.saved_tensors
        return raster.normal_error_backward(allmap, viewmatrix, rays_d, ray_o, gerr), None, None, None


def normal_error(allmap, cam):
    """1 - sum_c rend_normal * surf_normal per pixel ([H, W]); differentiable in allmap."""
    dev = allmap.device
    rays_d, rays_o = _camera_rays(cam, dev)
    vm = cam.world_view_transform.to(dev).float().contiguous()
    return _NormalError.apply(allmap, vm, rays_d.contiguous(), rays_o.contiguous())


def normal_error_torch(allmap, cam):
    """The same error from the torch restatement (decode_allmap), for comparison."""
    _, rend_normal, surf_normal, _ = decode_allmap(allmap, cam)
    return 1 - (rend_normal * surf_normal).sum(dim=0)


def config4_loss(rgb, allmap, cam, target, lambda_normal=0.05):
    """train.py:651, 674-675 with lambda_dssim 0: L1 + lambda_normal * normal error."""
    l1 = (rgb - target).abs().mean()
    return l1 + lambda_normal * normal_error(allmap, cam).mean()


@dataclass
class TrainState:
    """Leaves of config 4 and the fixed inputs of its step."""
    means3D: torch.Tensor
    scales: torch.Tensor
    rotations: torch.Tensor
    opacities: torch.Tensor
    table: torch.Tensor
    mlp: list
    ap_level: torch.Tensor
    offsets: torch.Tensor
    gridrange: torch.Tensor
    target: torch.Tensor
    extra: dict = field(default_factory=dict)

    def leaves(self):
        return [self.means3D, self.scales, self.rotations, self.opacities, self.table, *self.mlp]


def make_state(scene, target_seed: int = 4, device="cuda") -> TrainState:
    """Config-4 leaves from a synthetic scene: activated surfel tensors, the fp32
    hash table, fp32 MLP weights, and a U(0,1) target image."""
    from . import synth
    means, scales, rots, opac = synth.activate(scene.base)
    leaf = lambda t: t.detach().to(device).float().contiguous().requires_grad_(True)  # noqa: E731
    g = torch.Generator().manual_seed(target_seed)
    cam = scene.camera
    target = torch.rand(3, cam.height, cam.width, generator=g).to(device)
    return TrainState(leaf(means), leaf(scales), leaf(rots), leaf(opac), leaf(scene.grid.table.float()),
                      [leaf(w.float()) for w in scene.mlp], scene.ap_level.to(device).contiguous(),
                      scene.grid.offsets.to(device), scene.grid.gridrange.to(device), target)


def forward(state: TrainState, rasterizer, cam, bg=None, keep_upstream=False):
    """Rasterize + MLP + loss. Returns (loss, rgb, allmap). With keep_upstream the
    rasterizer outputs keep their gradients (state.extra["color"].grad and
    state.extra["allmap"].grad after backward), for tests."""
    P = state.means3D.shape[0]
    dev = state.means3D.device
    means2D = torch.zeros(P, 3, device=dev, requires_grad=True)
    color, radii, allmap, _, _ = rasterizer(
        means3D=state.means3D, means2D=means2D, opacities=state.opacities,
        shs=torch.zeros(P, 1, 3, device=dev), scales=state.scales, rotations=state.rotations,
        homotrans=None, ap_level=state.ap_level, features=state.table, offsets=state.offsets,
        gridrange=state.gridrange, render_mode=0)
    if keep_upstream:
        color.retain_grad()
        allmap.retain_grad()
        state.extra["color"], state.extra["allmap"] = color, allmap
    rgb = mlp(color, *state.mlp, allmap[1], bg)
    loss = config4_loss(rgb, allmap, cam, state.target)
    state.extra["means2D"] = means2D
    state.extra["radii"] = radii
    return loss, rgb, allmap


def step(state: TrainState, rasterizer, cam, bg=None):
    """Forward + backward; leaves' .grad hold the gradients afterwards."""
    for t in state.leaves():
        t.grad = None
    loss, rgb, allmap = forward(state, rasterizer, cam, bg)
    loss.backward()
    return loss
