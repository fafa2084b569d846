"""Torch fp32 restatements of the reference's own torch oracles (test infrastructure).

Each function follows a reference function line by line (paths inside
nbardy/fast-mac-gsplat); tests pin them to golden vectors made by the originals.
"""
from __future__ import annotations

import torch
from torch import Tensor


def _batched(*xs: Tensor):
    squeeze = xs[0].ndim == 2
    if squeeze:
        xs = tuple(x.unsqueeze(0) for x in xs)
    return squeeze, xs


def dense_reference(means2d, conics, colors, opacities, depths, H, W, bg=(0.0, 0.0, 0.0),
                    alpha_threshold=1.0 / 255.0, max_alpha=0.99):
    """No early stop. Restates benchmarks/benchmark_full_matrix.py:128-152 and
    variants/v8_project3d/tests/reference_check.py:15-50."""
    squeeze, (means2d, conics, colors, opacities, depths) = _batched(means2d, conics, colors, opacities, depths)
    dev, dt = means2d.device, means2d.dtype
    bg_t = torch.tensor(bg, dtype=dt, device=dev)
    ys = torch.arange(H, dtype=dt, device=dev) + 0.5
    xs = torch.arange(W, dtype=dt, device=dev) + 0.5
    yy, xx = torch.meshgrid(ys, xs, indexing="ij")
    outs = []
    for b in range(means2d.shape[0]):
        perm = torch.argsort(depths[b].detach(), stable=True)
        m, q, c, o = means2d[b][perm], conics[b][perm], colors[b][perm], opacities[b][perm]
        out = torch.zeros(H, W, 3, dtype=dt, device=dev)
        T = torch.ones(H, W, dtype=dt, device=dev)
        for i in range(m.shape[0]):
            dx = xx - m[i, 0]
            dy = yy - m[i, 1]
            power = -0.5 * (q[i, 0] * dx * dx + 2 * q[i, 1] * dx * dy + q[i, 2] * dy * dy)
            alpha = torch.clamp(o[i] * torch.exp(power), max=max_alpha)
            alpha = torch.where((power <= 0) & (alpha >= alpha_threshold), alpha, torch.zeros_like(alpha))
            out = out + (T * alpha)[..., None] * c[i]
            T = T * (1.0 - alpha)
        outs.append(out + T[..., None] * bg_t)
    out = torch.stack(outs, 0)
    return out[0] if squeeze else out


def saturating_reference(means2d, conics, colors, opacities, depths, H, W, bg=(0.0, 0.0, 0.0),
                         alpha_threshold=1.0 / 255.0, transmittance_threshold=1.0e-4, max_alpha=0.99,
                         pixel_mask: Tensor | None = None):
    """Early-stop oracle with the kernel's exact semantics. Restates
    variants/v8_project3d/tests/reference_check.py:53-104 (there `bg` defaults to
    white; here it is an explicit argument). `pixel_mask` [H,W] bool optionally
    restricts the evaluation to a subset of pixels (others render background and
    carry no gradient) for tile-sampled parity on large frames."""
    squeeze, (means2d, conics, colors, opacities, depths) = _batched(means2d, conics, colors, opacities, depths)
    dev, dt = means2d.device, means2d.dtype
    bg_t = torch.tensor(bg, dtype=dt, device=dev)
    ys = torch.arange(H, dtype=dt, device=dev) + 0.5
    xs = torch.arange(W, dtype=dt, device=dev) + 0.5
    yy, xx = torch.meshgrid(ys, xs, indexing="ij")
    if pixel_mask is not None:
        sel = pixel_mask.to(dev).reshape(-1)
        yy = yy.reshape(-1)[sel]
        xx = xx.reshape(-1)[sel]
        shape = (int(sel.sum()),)
    else:
        shape = (H, W)
    outs = []
    for b in range(means2d.shape[0]):
        perm = torch.argsort(depths[b].detach(), stable=True)
        m, q, c, o = means2d[b][perm], conics[b][perm], colors[b][perm], opacities[b][perm]
        out = torch.zeros(*shape, 3, dtype=dt, device=dev)
        T = torch.ones(*shape, dtype=dt, device=dev)
        for i in range(m.shape[0]):
            active = T > transmittance_threshold
            dx = xx - m[i, 0]
            dy = yy - m[i, 1]
            power = -0.5 * (q[i, 0] * dx * dx + 2 * q[i, 1] * dx * dy + q[i, 2] * dy * dy)
            alpha = torch.clamp(o[i] * torch.exp(power), max=max_alpha)
            alpha = torch.where((power <= 0) & (alpha >= alpha_threshold) & active, alpha, torch.zeros_like(alpha))
            out = out + (T * alpha)[..., None] * c[i]
            T = T * (1.0 - alpha)
        outs.append(out + T[..., None] * bg_t)
    out = torch.stack(outs, 0)
    return out[0] if squeeze else out


def project_pinhole(means3d_b, scales_b, quats_b, opacities_b, camera_to_world_b, camera_params, near_plane):
    """Restates _torch_project_pinhole_gaussians_batched
    (variants/v8_project3d/torch_gsplat_bridge_v8_project3d/rasterize.py:288-358)."""
    B, G = means3d_b.shape[:2]
    qr, qi, qj, qk = quats_b[..., 0], quats_b[..., 1], quats_b[..., 2], quats_b[..., 3]
    R = torch.stack(
        [
            torch.stack([1 - 2 * (qj * qj + qk * qk), 2 * (qi * qj - qr * qk), 2 * (qi * qk + qr * qj)], -1),
            torch.stack([2 * (qi * qj + qr * qk), 1 - 2 * (qi * qi + qk * qk), 2 * (qj * qk - qr * qi)], -1),
            torch.stack([2 * (qi * qk - qr * qj), 2 * (qj * qk + qr * qi), 1 - 2 * (qi * qi + qj * qj)], -1),
        ],
        -2,
    )
    M = R * scales_b[..., None, :]
    cov3d = M @ M.transpose(-1, -2)
    Rcw = camera_to_world_b[:, :3, :3]
    t = camera_to_world_b[:, :3, 3]
    mc = (means3d_b - t[:, None, :]) @ Rcw
    covc = Rcw.transpose(1, 2).unsqueeze(1) @ cov3d @ Rcw.unsqueeze(1)
    x, y, z = mc[..., 0], mc[..., 1], mc[..., 2]
    front = z > float(near_plane)
    zs = torch.where(front, torch.clamp(z, min=float(near_plane)), torch.ones_like(z))
    xp = torch.where(front, x, torch.zeros_like(x))
    yp = torch.where(front, y, torch.zeros_like(y))
    fx, fy, cx, cy = (camera_params[:, k : k + 1] for k in range(4))
    zero = torch.zeros_like(zs)
    J = torch.stack(
        [torch.stack([fx / zs, zero, -(fx * xp) / zs.square()], -1),
         torch.stack([zero, fy / zs, -(fy * yp) / zs.square()], -1)],
        -2,
    )
    cov2d = J @ covc @ J.transpose(-1, -2)
    c00 = cov2d[..., 0, 0] + 0.3
    c01 = cov2d[..., 0, 1]
    c11 = cov2d[..., 1, 1] + 0.3
    det = torch.clamp(c00 * c11 - c01 * c01, min=1.0e-6)
    conics = torch.stack([c11 / det, -c01 / det, c00 / det], -1)
    means2d = torch.stack([(fx * xp) / zs + cx, (fy * yp) / zs + cy], -1)
    opac = torch.where(front, opacities_b, torch.zeros_like(opacities_b))
    return means2d, conics, opac, z


def tiled_scan_work(tile_offsets: Tensor, *, height: int, width: int, tile_size: int = 16, batch: int = 1) -> int:
    """E = sum over tiles of valid_pixels(tile) * count(tile); restates
    variants/v7_tiled_capture/torch_gsplat_bridge_v72/reference.py:288-302 for a flat
    [B*tiles+1] offsets array."""
    off = tile_offsets.detach().to("cpu", torch.int64)
    tx = (width + tile_size - 1) // tile_size
    ty = (height + tile_size - 1) // tile_size
    counts = (off[1:] - off[:-1]).view(batch, ty, tx)
    h = torch.full((ty,), tile_size, dtype=torch.int64)
    h[-1] = height - (ty - 1) * tile_size
    w = torch.full((tx,), tile_size, dtype=torch.int64)
    w[-1] = width - (tx - 1) * tile_size
    return int((counts * (h[:, None] * w[None, :])[None]).sum())


def saturating_reference_pixels(means2d, conics, colors, opacities, depths, px, py, bg=(0.0, 0.0, 0.0),
                                alpha_threshold=1.0 / 255.0, transmittance_threshold=1.0e-4, max_alpha=0.99,
                                chunk=256):
    """saturating_reference (variants/v8_project3d/tests/reference_check.py:53-104) for
    one view, evaluated only at the pixel-centre samples (px+0.5, py+0.5), with the
    per-splat loop replaced by a cumulative product over the depth-sorted splats:
    T_before_i = prod_{j<i} (1 - alpha_j); active_i = T_before_i > T_thr. T is
    non-increasing, so once a pixel stops every later splat is inactive, exactly as
    in the loop. Splats are processed in chunks to bound memory. -> [N,3]."""
    dev, dt = means2d.device, means2d.dtype
    perm = torch.argsort(depths.detach(), stable=True)
    m, q, c, o = means2d[perm], conics[perm], colors[perm], opacities[perm]
    xs = px.to(dev, dt)[:, None] + 0.5
    ys = py.to(dev, dt)[:, None] + 0.5
    T = torch.ones(xs.shape[0], 1, dtype=dt, device=dev)
    out = torch.zeros(xs.shape[0], 3, dtype=dt, device=dev)
    for s in range(0, m.shape[0], chunk):
        e = min(m.shape[0], s + chunk)
        dx = xs - m[s:e, 0][None]
        dy = ys - m[s:e, 1][None]
        power = -0.5 * (q[s:e, 0][None] * dx * dx + 2 * q[s:e, 1][None] * dx * dy + q[s:e, 2][None] * dy * dy)
        alpha = torch.clamp(o[s:e][None] * torch.exp(power), max=max_alpha)
        alpha = torch.where((power <= 0) & (alpha >= alpha_threshold), alpha, torch.zeros_like(alpha))
        one_minus = 1.0 - alpha
        t_incl = T * torch.cumprod(one_minus, dim=1)
        t_before = torch.cat([T, t_incl[:, :-1]], dim=1)
        active = (t_before > transmittance_threshold).detach()
        a_eff = torch.where(active, alpha, torch.zeros_like(alpha))
        out = out + (t_before * a_eff) @ c[s:e]
        T = T * torch.prod(1.0 - a_eff, dim=1, keepdim=True)
    return out + T * torch.tensor(bg, dtype=dt, device=dev)


# ---------------------------------------------------------------------------
# Spherical-harmonic colours (no reference counterpart: the reference takes
# RGB). Real SH basis, degree <= 3, in the (y, z, x) ordering of the common
# 3D Gaussian splatting convention; each constant is
# sqrt((2l+1)/(4 pi) (l-|m|)!/(l+|m|)!) (times sqrt 2 for m != 0) with the
# Cartesian polynomial of Y_lm. Used as the fp32 reference of the CUDA kernel.
# ---------------------------------------------------------------------------
def sh_basis(dirs: Tensor, degree: int) -> Tensor:
    """dirs [..., 3] unit vectors -> basis [..., (degree+1)^2]."""
    x, y, z = dirs.unbind(-1)
    out = [torch.full_like(x, 0.28209479177387814)]
    if degree >= 1:
        c1 = 0.4886025119029199
        out += [-c1 * y, c1 * z, -c1 * x]
    if degree >= 2:
        xx, yy, zz = x * x, y * y, z * z
        out += [1.0925484305920792 * x * y, -1.0925484305920792 * y * z,
                0.31539156525252005 * (2 * zz - xx - yy), -1.0925484305920792 * x * z,
                0.5462742152960396 * (xx - yy)]
    if degree >= 3:
        out += [-0.5900435899266435 * y * (3 * xx - yy), 2.890611442640554 * x * y * z,
                -0.4570457994644658 * y * (4 * zz - xx - yy), 0.3731763325901154 * z * (2 * zz - 3 * xx - 3 * yy),
                -0.4570457994644658 * x * (4 * zz - xx - yy), 1.445305721320277 * z * (xx - yy),
                -0.5900435899266435 * x * (xx - 3 * yy)]
    return torch.stack(out, dim=-1)


def sh_colors_reference(sh: Tensor, means3d: Tensor, camera_to_world: Tensor, degree: int) -> Tensor:
    """sh [G,K,3], means3d [G,3], camera_to_world [B,4,4] -> colours [B,G,3]:
    max(0, 0.5 + sum_k sh_k Y_k(normalize(mean - centre)))."""
    centre = camera_to_world[:, :3, 3]
    d = means3d[None] - centre[:, None]
    d = d / torch.sqrt((d * d).sum(-1, keepdim=True).clamp_min(1e-24))
    Y = sh_basis(d, degree)
    K = Y.shape[-1]
    return torch.clamp_min((Y[..., None] * sh[None, :, :K]).sum(-2) + 0.5, 0.0)


# ---------------------------------------------------------------------------
# The reference benchmark harness's accuracy check (benchmarks/benchmark_full_matrix.py),
# so a renderer entry written for that harness can be driven here.
# ---------------------------------------------------------------------------
def clone_inputs(inputs, backward: bool):
    """benchmark_full_matrix.py:155-161: detached contiguous copies, the four
    differentiable inputs requiring grad when the mode has a backward."""
    out = []
    for i, t in enumerate(inputs):
        c = t.detach().clone().contiguous()
        c.requires_grad_(backward and i < 4)
        out.append(c)
    return tuple(out)


def harness_measure_accuracy(run_renderer, renderer: str, base_inputs, height: int, width: int,
                             mode: str = "forward_backward", max_work_items: int = 64_000_000):
    """measure_accuracy (benchmark_full_matrix.py:380-427) for one renderer: the
    renderer's image and (forward_backward) its gradients of out.square().mean()
    against the dense torch reference on clones of the same inputs."""
    B, G = base_inputs[0].shape[:2]
    work = B * height * width * G
    if work > max_work_items:
        return {"accuracy_status": "skipped",
                "accuracy_reason": f"work_items {work} exceeds accuracy limit {max_work_items}"}
    backward = mode == "forward_backward"
    run_inputs = clone_inputs(base_inputs, backward)
    ref_inputs = clone_inputs(base_inputs, backward)
    out = run_renderer(renderer, run_inputs, height, width)
    ref = dense_reference(*ref_inputs, height, width)
    err = (out - ref).detach().abs()
    result = {"accuracy_status": "ok", "image_max_abs_error": float(err.max().item()),
              "image_mean_abs_error": float(err.mean().item())}
    if backward:
        out.square().mean().backward()
        ref.square().mean().backward()
        worst = []
        for name, got, want in zip(("means2d", "conics", "colors", "opacities"), run_inputs[:4], ref_inputs[:4]):
            if got.grad is None or want.grad is None:
                continue
            e = (got.grad - want.grad).detach().abs()
            result[f"grad_{name}_max_abs_error"] = float(e.max().item())
            result[f"grad_{name}_mean_abs_error"] = float(e.mean().item())
            worst.append(float(e.max().item()))
        result["grad_max_abs_error"] = max(worst) if worst else 0.0
    return result
