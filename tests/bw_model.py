"""Float64 torch model of the mode-0 forward pass, differentiated by autograd.

Test infrastructure: it pins the CPU oracle's backward (oracle/nest_oracle_bw.cpp)
to true gradients. It is written independently of the oracle -- tensors over
the pixels of a tile, one step per list entry -- and reuses only the oracle's
discrete structure (per-tile lists from binning), so that both walk the same
surfels in the same order.

The reference's backward differs from the derivative of its forward in known
places; the model states them explicitly so the comparison covers the rest:
  * means2D: the forward centre uses compute_aabb's cutoff 4 (forward.cu:294-320,
    t = (16, 16, -1)); the backward pushes dL/dmeans2D into T with cutoff 3
    (backward.cu:2143, t = (9, 9, -1)). The model's centre has the cutoff-4 value
    and the cutoff-3 derivative.
  * rotations: quat_to_rotmat_vjp (auxiliary.h:243-287) is the derivative of the
    rotation formula on the quaternion as given, without the normalisation; the
    model feeds unit quaternions to that formula directly.
  * beta > 0 and the 0.99 alpha clamp are not modelled (the pin uses beta = 0 and
    opacities below 0.99).
  * splat kernel 1 (beta, (1 - rho)^shape): the reference's dG/ds factor
    -shape G / (1 - rho) (backward.cu:1965, :2025) is half of d/ds of its
    forward (rho = s.x^2 + s.y^2 gives 2 shape G / (1 - rho) s); the model's G
    has the forward's value, the full shape derivative and half the rho
    derivative.
"""
from __future__ import annotations

import numpy as np
import torch

NEAR, FAR = 0.2, 100.0
TILE = 16


def rotation_columns(q: torch.Tensor):
    w, x, y, z = q.unbind(1)
    r0 = torch.stack([1 - 2 * (y * y + z * z), 2 * (x * y + w * z), 2 * (x * z - w * y)], 1)
    r1 = torch.stack([2 * (x * y - w * z), 1 - 2 * (x * x + z * z), 2 * (y * z + w * x)], 1)
    r2 = torch.stack([2 * (x * z + w * y), 2 * (y * z - w * x), 1 - 2 * (x * x + y * y)], 1)
    return r0, r1, r2


def ndc_to_pixel(pm: np.ndarray, W: int, H: int) -> torch.Tensor:
    """P[c, r] = sum_k pm[4r + k] n[c][k]: world -> homogeneous pixel coordinates."""
    n = np.array([[W / 2, 0, 0, (W - 1) / 2], [0, H / 2, 0, (H - 1) / 2], [0, 0, 0, 1]], np.float64)
    M = np.asarray(pm, np.float64).reshape(4, 4)  # M[r, k] = pm[4r + k]
    return torch.tensor(n @ M.T)  # [3, 4]


def centre(Tu, Tv, Tw, cutoff: float):
    t0 = cutoff * cutoff
    d = t0 * Tw[:, 0] ** 2 + t0 * Tw[:, 1] ** 2 - Tw[:, 2] ** 2
    px = (t0 * Tu[:, 0] * Tw[:, 0] + t0 * Tu[:, 1] * Tw[:, 1] - Tu[:, 2] * Tw[:, 2]) / d
    py = (t0 * Tv[:, 0] * Tw[:, 0] + t0 * Tv[:, 1] * Tw[:, 1] - Tv[:, 2] * Tw[:, 2]) / d
    return torch.stack([px, py], 1)


def grid_index(g: torch.Tensor, hsize: int, res: int, align_corners: bool) -> torch.Tensor:
    stride, index = 1, torch.zeros_like(g[:, 0])
    for d in range(3):
        if stride > hsize:
            break
        index = index + g[:, d] * stride
        stride *= res if align_corners else res + 1
    if stride > hsize:
        m = 0xFFFFFFFF
        index = (g[:, 0] & m) ^ ((g[:, 1] * 2654435761) & m) ^ ((g[:, 2] * 805459861) & m)
    return index % hsize


def query(xyz, apl, table, offsets, L, LD, S, Hres, vmin, vmax, align_corners=False, interp=0):
    """Trilinear hash-grid features [n, L*LD] at xyz [n,3]; levels >= apl are zero."""
    inp = (xyz - vmin) / (vmax - vmin)
    oob = ((inp < 0) | (inp > 1)).any(1)
    feats = []
    for lv in range(L):
        hs = int(offsets[lv + 1] - offsets[lv])
        scale = float(np.float32(np.exp2(np.float32(lv * np.float32(S)))) * np.float32(Hres) - np.float32(1.0))
        res = int(np.ceil(np.float32(scale))) + 1
        pos = inp * scale + (0.0 if align_corners else 0.5)
        pg = torch.floor(pos.detach())
        frac = pos - pg
        if interp == 1:
            frac = frac * frac * (3.0 - 2.0 * frac)
        acc = 0
        for c in range(8):
            bits = [(c >> d) & 1 for d in range(3)]
            w = 1
            for d in range(3):
                w = w * (frac[:, d] if bits[d] else 1 - frac[:, d])
            g = pg.long() + torch.tensor(bits, dtype=torch.long)
            rows = int(offsets[lv]) + grid_index(g, hs, res, align_corners)
            acc = acc + w[:, None] * table[rows]
        on = torch.as_tensor(lv < apl, dtype=table.dtype)[:, None] * (~oob)[:, None].to(table.dtype)
        feats.append(acc * on)
    if not feats:  # no level (level 0)
        return xyz.new_zeros(xyz.shape[0], 0)
    return torch.cat(feats, 1)


def splat_value(rho, shape, kernel_type: int):
    """G of the splat kernels (forward.cu:864-902) and the kernel's own validity
    mask (kernel 1 stops at the unit circle). shape: 0-d tensor."""
    if kernel_type == 1:
        inside = (rho < 1.0).detach()
        base = torch.where(inside, 1.0 - rho, torch.ones_like(rho))
        f = lambda b, s: b ** s  # noqa: E731
        Gv = f(base, shape).detach()
        G = Gv + 0.5 * (f(base, shape.detach()) - Gv) + (f(base.detach(), shape) - Gv)
        return G, inside
    if kernel_type == 2:
        g = torch.exp(-0.5 * rho)
        if float(shape.detach()) > 0:
            g = (1.0 + shape) * g / (1.0 + shape * g)
        return g, torch.ones_like(rho, dtype=torch.bool)
    if kernel_type == 3:
        pt = torch.clamp_min(rho, 1e-8) ** (0.5 * shape)
        return torch.exp(-0.5 * pt), torch.ones_like(rho, dtype=torch.bool)
    return torch.exp(-0.5 * rho), torch.ones_like(rho, dtype=torch.bool)


SH_C0 = 0.28209479177387814
SH_C1 = 0.4886025119029199
SH_C2 = (1.0925484305920792, -1.0925484305920792, 0.31539156525252005, -1.0925484305920792, 0.5462742152960396)
SH_C3 = (-0.5900435899266435, 2.890611442640554, -0.4570457994644658, 0.3731763325901154, -0.4570457994644658,
         1.445305721320277, -0.5900435899266435)


def eval_sh_interleaved(sh, d, deg=3):
    """SH colour [n, 3] of coefficients read interleaved (coefficient k of
    channel c at 3 k + c; sh [3 M] shared by all rows or [n, 3 M]) along unit
    directions d [n, 3], degree `deg` terms, + 0.5 and clamped at 0
    (forward.cu:21-74 computeColorFromSH, :76-155 for render mode 11)."""
    x, y, z = d[:, 0:1], d[:, 1:2], d[:, 2:3]
    sh = sh[None, :] if sh.dim() == 1 else sh
    c = lambda k: sh[:, 3 * k:3 * k + 3]  # noqa: E731
    xx, yy, zz, xy, yz, xz = x * x, y * y, z * z, x * y, y * z, x * z
    r = SH_C0 * c(0)
    if deg > 0:
        r = r - SH_C1 * y * c(1) + SH_C1 * z * c(2) - SH_C1 * x * c(3)
    if deg > 1:
        r = (r + SH_C2[0] * xy * c(4) + SH_C2[1] * yz * c(5) + SH_C2[2] * (2 * zz - xx - yy) * c(6)
             + SH_C2[3] * xz * c(7) + SH_C2[4] * (xx - yy) * c(8))
    if deg > 2:
        r = (r + SH_C3[0] * y * (3 * xx - yy) * c(9) + SH_C3[1] * xy * z * c(10)
             + SH_C3[2] * y * (4 * zz - xx - yy) * c(11) + SH_C3[3] * z * (2 * zz - 3 * xx - 3 * yy) * c(12)
             + SH_C3[4] * x * (4 * zz - xx - yy) * c(13) + SH_C3[5] * z * (xx - yy) * c(14)
             + SH_C3[6] * x * (xx - 3 * yy) * c(15))
    return torch.clamp_min(r + 0.5, 0.0)


def sh_hybrid_feature(h, row, mode, decompose):
    """Features of render modes 8 / 9 / 10 (forward.cu:1378-1526) from the
    single-level 3-wide hash value h [n, 3] and the surfel's row (3 raw SH
    colours; 48 SH coefficients for mode 9). With decompose 1 (the surfel only)
    the grid is not queried (h = 0). Mode 8 keeps the reference backward's
    mask for every decompose flag: gradients pass only where
    clamp(row + 0.5) + sigmoid(h) lies in [0, 1], also when the forward used
    one of the two parts alone."""
    n = h.shape[0]
    if decompose == 1:
        h = torch.zeros_like(h)
    if mode == 8:
        gr = torch.clamp(row[:3] + 0.5, 0.0, 1.0).expand(n, 3)
        hr = torch.sigmoid(h)
        s = gr + hr
        if decompose == 0:
            return torch.clamp(s, 0.0, 1.0)
        mask = ((s >= 0) & (s <= 1)).detach().to(h.dtype)
        part = hr if decompose == 2 else gr
        return part.detach() + mask * (part - part.detach())
    if mode == 10:
        comb = h if decompose == 2 else (row[:3].expand(n, 3) if decompose == 1 else row[:3] + h)
        return torch.sigmoid(comb)
    feat = row[:48].expand(n, 48)
    dc = torch.zeros(n, 48, dtype=h.dtype)
    keep = torch.ones(48, dtype=h.dtype)
    if decompose != 1:
        for c in range(3):
            dc[:, 16 * c] = h[:, c]
            if decompose == 2:
                keep[16 * c] = 0.0
    return feat * keep + dc


def mode_feature(f_hash, row, mode, pg, td, C):
    """Feature vectors [n, C] of render modes 4 / 6 / 7 / 12 / 14
    (forward.cu:1218-1377, 1593-1790, training rules) and of level 0 (mode 0
    without hash levels, :1093-1096) from the hash features f_hash [n, L*LD]
    and the surfel's row of colors_precomp (blend weight last for 7 / 12 / 14)."""
    n, hd = f_hash.shape
    if mode == 0:  # level 0: the row is the colour
        return row[:C].expand(n, C)
    if mode in (6, 7):
        if mode == 6:  # uniform blend on the hash levels' channels
            feat = 0.5 * row[:hd].expand(n, hd) + 0.5 * f_hash
        else:  # weighted blend over total LD channels, hash zero past its levels
            wgt = row[td]
            hpad = torch.cat([f_hash, f_hash.new_zeros(n, td - hd)], 1)
            feat = wgt * row[:td].expand(n, td) + (1 - wgt) * hpad
        if feat.shape[1] < C:
            feat = torch.cat([feat, feat.new_zeros(n, C - feat.shape[1])], 1)
        return feat[:, :C]
    coarse = row[:pg].expand(n, pg)
    if mode == 4:
        fine = f_hash
    elif mode == 12:
        wgt = row[td]
        fine = wgt * row[pg:pg + hd].expand(n, hd) + (1 - wgt) * f_hash
    else:
        wgt = row[pg]
        fine = wgt * f_hash if float(wgt.detach()) > 1e-6 else torch.zeros_like(f_hash)
    feat = torch.cat([coarse, fine], 1)
    if feat.shape[1] < C:
        feat = torch.cat([feat, feat.new_zeros(n, C - feat.shape[1])], 1)
    return feat


def render(means, scales, rots, opac, table, cam, lists, grid, apl_int, W, H, kernel_type=0, shapes=None,
           modes=None, Ts=None, homo=None):
    """Forward pass over the oracle's tile lists. Returns (color [C,H,W], others [7,H,W], margins).

    Ts [P, 9] (columns Tu, Tv, Tw) replaces the transforms built from means,
    scales and rotations (the reference's transMat_precomp): the normal is then
    the view axis, flipped to face the camera, and the hit point is formed from
    the constant homotrans `homo` [P, 16] (its gradient is not returned).

    margins: the smallest relative distance of any decision (alpha >= 1/255, the
    rho3d/rho2d branch, near plane, termination) from its threshold, so a test can
    check that float32 and float64 take the same branches."""
    vm = np.asarray(cam["viewmatrix"], np.float64).reshape(4, 4)
    P = ndc_to_pixel(cam["projmatrix"], W, H)
    vmt = torch.tensor(vm)
    pk = means
    if Ts is not None:
        Tu, Tv, Tw = Ts[:, 0:3], Ts[:, 3:6], Ts[:, 6:9]
        h = torch.as_tensor(np.asarray(homo, np.float64)).reshape(-1, 4, 4)
        L0, L1, pk = h[:, :3, 0], h[:, :3, 1], h[:, :3, 3]
        n = torch.tensor([0.0, 0.0, 1.0], dtype=torch.float64).expand(Ts.shape[0], 3)
    else:
        r0, r1, r2 = rotation_columns(rots)
        L0, L1 = r0 * scales[:, 0:1], r1 * scales[:, 1:2]
        Tu = torch.stack([L0 @ P[0, :3], L1 @ P[0, :3], means @ P[0, :3] + P[0, 3]], 1)
        Tv = torch.stack([L0 @ P[1, :3], L1 @ P[1, :3], means @ P[1, :3] + P[1, 3]], 1)
        Tw = torch.stack([L0 @ P[2, :3], L1 @ P[2, :3], means @ P[2, :3] + P[2, 3]], 1)
        n = r2 @ vmt[:3, :3]
        n = n / n.norm(dim=1, keepdim=True)
    pv = means @ vmt[:3, :3] + vmt[3, :3]
    flip = torch.where(-(pv * n).sum(1) > 0, 1.0, -1.0).detach()
    n = n * flip[:, None]
    xy3 = centre(Tu, Tv, Tw, 3.0)
    xy = xy3 + (centre(Tu, Tv, Tw, 4.0) - xy3).detach()

    ranges, point_list = lists
    C = grid["L"] * grid["LD"] if modes is None else modes["C"]
    color = torch.zeros(C, H * W, dtype=torch.float64)
    others = torch.zeros(7, H * W, dtype=torch.float64)
    sh_map = torch.zeros(3, H * W, dtype=torch.float64)
    gx = (W + TILE - 1) // TILE
    margin = np.inf
    for t in range(ranges.shape[0]):
        tx, ty = t % gx, t // gx
        ys, xs = np.meshgrid(np.arange(ty * TILE, min(H, ty * TILE + TILE)),
                             np.arange(tx * TILE, min(W, tx * TILE + TILE)), indexing="ij")
        ys, xs = ys.reshape(-1), xs.reshape(-1)
        pid = torch.as_tensor(ys * W + xs)
        pxf = torch.as_tensor(xs, dtype=torch.float64)
        pyf = torch.as_tensor(ys, dtype=torch.float64)
        npx = len(xs)
        T = torch.ones(npx, dtype=torch.float64)
        done = torch.zeros(npx, dtype=torch.bool)
        D = torch.zeros(npx, dtype=torch.float64)
        M1, M2, dist, med = D.clone(), D.clone(), D.clone(), D.clone()
        N = torch.zeros(npx, 3, dtype=torch.float64)
        Cacc = torch.zeros(npx, C, dtype=torch.float64)
        SH = torch.zeros(npx, 3, dtype=torch.float64)
        for k in range(int(ranges[t, 0]), int(ranges[t, 1])):
            i = int(point_list[k])
            kk = pxf[:, None] * Tw[i] - Tu[i]
            ll = pyf[:, None] * Tw[i] - Tv[i]
            p = torch.linalg.cross(kk, ll, dim=1)
            sx, sy = p[:, 0] / p[:, 2], p[:, 1] / p[:, 2]
            rho3d = sx * sx + sy * sy
            dx, dy = xy[i, 0] - pxf, xy[i, 1] - pyf
            rho2d = 2.0 * (dx * dx + dy * dy)
            b3 = (rho3d <= rho2d).detach()
            rho = torch.where(b3, rho3d, rho2d)
            c_d = torch.where(b3, sx * Tw[i, 0] + sy * Tw[i, 1] + Tw[i, 2], Tw[i, 2].expand(npx))
            G, inside = splat_value(rho, shapes[i] if kernel_type else None, kernel_type)
            alpha = opac[i] * G
            valid = (~done) & (c_d.detach() >= NEAR) & (alpha.detach() >= 1.0 / 255.0) & inside
            test_T = T * (1 - alpha)
            stop = valid & (test_T.detach() < 1e-4)
            live = (~done)
            if live.any():
                a = alpha.detach()[live].numpy()
                gap = (rho3d - rho2d).detach().abs() / torch.maximum(rho3d, rho2d).detach().clamp_min(1e-300)
                m = [np.abs(a - 1 / 255) / np.maximum(a, 1e-300), gap[live].numpy(),
                     np.abs(c_d.detach()[live].numpy() - NEAR)]
                tt = test_T.detach()[live].numpy()
                m.append(np.abs(tt - 1e-4) / 1e-4)
                if kernel_type == 1:
                    m.append(np.abs(rho.detach()[live].numpy() - 1.0))
                margin = min(margin, *[float(np.min(x)) for x in m])
            done = done | stop
            valid = valid & ~stop
            vf = valid.to(torch.float64)
            w = alpha * T * vf
            A = 1 - T
            md = FAR / (FAR - NEAR) * (1 - NEAR / c_d)
            dist = dist + (md * md * A + M2 - 2 * md * M1) * w
            D = D + c_d * w
            M1 = M1 + md * w
            M2 = M2 + md * md * w
            med = torch.where(valid & (T.detach() > 0.5), c_d, med)
            N = N + n[i][None, :] * w[:, None]
            hit = torch.where(b3[:, None], sx[:, None] * L0[i] + sy[:, None] * L1[i] + pk[i], pk[i].expand(npx, 3))
            f = query(hit, np.full(npx, apl_int[i]), table, grid["offsets"], grid["L"], grid["LD"], grid["S"],
                      grid["H"], grid["vmin"], grid["vmax"], grid.get("align_corners", False),
                      grid.get("interp", 0))
            if modes is not None and modes["mode"] in (8, 9, 10):
                # the reference's cases 8-10 scale the row and hash gradients by
                # alpha T once more (backward.cu:1191-1371): same value, gradient
                # through f times the detached weight
                f = sh_hybrid_feature(f, modes["gauss"][i], modes["mode"], modes["decompose"])
                f = f.detach() + w.detach()[:, None] * (f - f.detach())
            elif modes is not None and modes["mode"] == 11:
                # hash levels from channel 0; the surfel's SH colour along hit - centre
                # goes to its own map (no gradient in the reference's backward)
                f = torch.cat([f, f.new_zeros(npx, C - f.shape[1])], 1) if f.shape[1] < C else f
                dvec = (hit - pk[i]).detach()
                rgb = eval_sh_interleaved(modes["gauss"][i].detach(), dvec / dvec.norm(dim=1, keepdim=True))
                rgb = torch.where(b3[:, None], torch.nan_to_num(rgb, nan=0.0), torch.zeros_like(rgb))
                SH = SH + rgb * w.detach()[:, None]
            elif modes is not None:
                f = mode_feature(f, modes["gauss"][i], modes["mode"], modes["pg"], modes["td"], C)
            Cacc = Cacc + f * w[:, None]
            T = torch.where(valid, test_T, T)
        color = color.index_copy(1, pid, Cacc.T)
        sh_map = sh_map.index_copy(1, pid, SH.T)
        others = others.index_copy(1, pid, torch.stack([D, 1 - T, N[:, 0], N[:, 1], N[:, 2], med, dist], 0))
    if modes is not None and modes["mode"] == 11:
        modes["sh_rgb"] = sh_map.reshape(3, H, W)
    return color.reshape(C, H, W), others.reshape(7, H, W), margin, xy
