"""GPU pinhole projection (forward + VJP) and the full 3D path through the C ABI,
against the reference's torch projection (golden vectors) and its restatement."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import torch_gsplat_bridge_fast as tgb
from helpers import GRAD_RTOL, IMAGE_ATOL, golden, max_abs, np_, rel_err, rel_err_finite
from oracle import oracle as O
from oracle import torch_ref as TR
from workloads import config_3d

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def test_projection_matches_reference_golden():
    c = golden("project_pinhole")
    m3, s3, q4, op = (torch.tensor(c[k], device=DEV, requires_grad=True) for k in
                      ("means3d", "scales", "quats", "opacities"))
    c2w = torch.tensor(c["c2w"], device=DEV, requires_grad=True)
    cam = torch.tensor(c["cam"], device=DEV, requires_grad=True)
    fx, fy, cx, cy = (cam[:, k] for k in range(4))
    outs = tgb.project_pinhole_gaussians(m3, s3, q4, op, fx, fy, cx, cy, camera_to_world=c2w,
                                         near_plane=float(c["near_plane"]))
    for o, key in zip(outs, ("means2d", "conics", "proj_opacities", "depths")):
        assert rel_err(np_(o), c[key]) <= 1e-5, key
    ups = [torch.tensor(c[k], device=DEV) for k in ("up_means2d", "up_conics", "up_opacities", "up_depths")]
    torch.autograd.backward(outs, ups)
    for t, key in zip((m3, s3, q4, op, c2w, cam), ("g_means3d", "g_scales", "g_quats", "g_opacities", "g_c2w",
                                                   "g_cam")):
        assert rel_err(np_(t.grad), c[key]) <= GRAD_RTOL, key


def test_projection_unbatched_and_defaults():
    g = torch.Generator().manual_seed(2)
    m3 = (torch.randn(100, 3, generator=g) + torch.tensor([0.0, 0.0, 6.0])).to(DEV)
    s3 = torch.exp(torch.randn(100, 3, generator=g) - 1).to(DEV)
    q4 = torch.randn(100, 4, generator=g).to(DEV)
    op = torch.rand(100, 1, generator=g).to(DEV)
    outs = tgb.project_pinhole_gaussians(m3, s3, q4, op, 200.0, 210.0, 32.0, 24.0)
    assert outs[0].shape == (100, 2) and outs[3].shape == (100,)
    ref = TR.project_pinhole(m3[None].cpu(), s3[None].cpu(), q4[None].cpu(), op[None, :, 0].cpu(),
                             torch.eye(4)[None], torch.tensor([[200.0, 210.0, 32.0, 24.0]]), 1e-4)
    for o, r in zip(outs, ref):
        assert rel_err(np_(o), np_(r[0])) <= 1e-5


def test_projection_c4_scale_matches_torch_restatement():
    """One view of the config-4 scene (2^20 Gaussians, camera on the radius-25
    sphere). Gaussians within 0.2 of the camera plane are left out: there the EWA
    Jacobian overflows fp32 (det -> inf) and the chain rule produces 0 * inf,
    which any two evaluation orders turn into different non-finite sums."""
    sc = config_3d(seed=0).to(DEV)
    c2w0 = sc.camera_to_world[:1]
    with torch.no_grad():
        z = TR.project_pinhole(sc.means3d[None], sc.scales[None], sc.quats[None], sc.opacities[None], c2w0,
                               sc.camera_params[:1], 1e-4)[3][0]
    keep = z.abs() > 0.2
    ins = [t[keep].clone().requires_grad_(True) for t in (sc.means3d, sc.scales, sc.quats, sc.opacities)]
    c2w = c2w0.clone().requires_grad_(True)
    cam = sc.camera_params[:1].clone().requires_grad_(True)
    outs = tgb.project_pinhole_gaussians(*(t[None] for t in ins), cam[:, 0], cam[:, 1], cam[:, 2], cam[:, 3],
                                         camera_to_world=c2w)
    ref_ins = [t.detach().clone().requires_grad_(True) for t in ins]
    rc2w = c2w.detach().clone().requires_grad_(True)
    rcam = cam.detach().clone().requires_grad_(True)
    refs = TR.project_pinhole(*(t[None] for t in ref_ins), rc2w, rcam, 1e-4)
    for o, r, name in zip(outs, refs, ("means2d", "conics", "opac", "depth")):
        assert rel_err_finite(np_(o), np_(r)) <= GRAD_RTOL, name
    gen = torch.Generator(device=DEV).manual_seed(3)
    ups = [torch.randn(o.shape, device=DEV, generator=gen) for o in outs]
    torch.autograd.backward(outs, ups)
    torch.autograd.backward(refs, ups)
    for a, b, name in zip(ins + [c2w, cam], ref_ins + [rc2w, rcam], ("m3", "s", "q", "o", "c2w", "cam")):
        assert rel_err_finite(np_(a.grad), np_(b.grad)) <= GRAD_RTOL, name


def test_full_pinhole_path_matches_torch_reference():
    """Project -> bin -> composite -> backward through projection, against the
    reference's torch projection followed by its early-stop compositing oracle."""
    g = torch.Generator().manual_seed(21)
    B, G, H, W = 2, 300, 40, 56
    m3 = torch.randn(B, G, 3, generator=g) * torch.tensor([1.5, 1.0, 0.5]) + torch.tensor([0.0, 0.0, 5.0])
    s3 = torch.exp(torch.randn(B, G, 3, generator=g) * 0.3 - 2.0)
    q4 = torch.randn(B, G, 4, generator=g)
    q4 = q4 / q4.norm(dim=-1, keepdim=True)
    op = torch.sigmoid(torch.randn(B, G, generator=g))
    col = torch.rand(B, G, 3, generator=g)
    gimg = torch.randn(B, H, W, 3, generator=g)
    cfg = tgb.RasterConfig(H, W)
    ins = [t.to(DEV).requires_grad_(True) for t in (m3, s3, q4, op, col)]
    out = tgb.rasterize_pinhole_gaussians(*ins[:4], ins[4], 60.0, 62.0, W / 2, H / 2, config=cfg)
    out.backward(gimg.to(DEV))
    ref_ins = [t.to(DEV).requires_grad_(True) for t in (m3, s3, q4, op, col)]
    cam = torch.tensor([[60.0, 62.0, W / 2, H / 2]] * B, device=DEV)
    m2, con, po, dep = TR.project_pinhole(*ref_ins[:4], torch.eye(4, device=DEV).expand(B, 4, 4), cam, 1e-4)
    ref = TR.saturating_reference(m2, con, ref_ins[4], po, dep, H, W)
    ref.backward(gimg.to(DEV))
    assert max_abs(np_(out), np_(ref)) <= IMAGE_ATOL
    for a, b, name in zip(ins, ref_ins, ("m3", "s", "q", "o", "rgb")):
        assert rel_err(np_(a.grad), np_(b.grad)) <= GRAD_RTOL, name


def _tile_candidates(m2, q2, o2, x0, y0, x1, y1, alpha_threshold=1.0 / 255.0):
    """Indices of the splats that can be visible at some pixel centre of the
    tile [x0, x1) x [y0, y1): the box of the support ellipse
    a dx^2 + 2b dx dy + c dy^2 <= tau, tau = -2 ln(alpha_thr / op) (outside it
    alpha < alpha_thr: the reference skips the splat), widened by one pixel
    against rounding, must reach the pixel-centre rectangle. Splats with a
    non-finite or degenerate conic are never visible in the kernel (their
    exponent is NaN or -inf) and are left out."""
    a, b, c = q2[:, 0], q2[:, 1], q2[:, 2]
    det = a * c - b * b
    ok = (o2 > alpha_threshold) & torch.isfinite(det) & (det > 0) & torch.isfinite(m2).all(-1)
    tau = -2.0 * torch.log(alpha_threshold / o2.clamp_min(1e-30))
    hx = torch.sqrt((tau * c / det).clamp_min(0)) + 1.0
    hy = torch.sqrt((tau * a / det).clamp_min(0)) + 1.0
    mx, my = m2[:, 0], m2[:, 1]
    ok &= (mx + hx >= x0 + 0.5) & (mx - hx <= x1 - 0.5) & (my + hy >= y0 + 0.5) & (my - hy <= y1 - 0.5)
    return torch.nonzero(ok).squeeze(1)


# The reference kernel's support box clamps the conic determinant at the meta
# eps (snugbox, …kernels.metal:537-546). For a splat whose projected conic has
# a smaller determinant (a Gaussian close to the camera, thousands of pixels
# wide) the box shrinks to a few pixels around the mean, so the reference
# kernel bins it into almost no tile, while the reference's dense torch oracle
# draws it across the frame. This renderer follows the kernel (binning is
# bit-exact against its restatement). In config 4, view 0, about 3,000 of the
# 2^20 Gaussians are such splats.
CONIC_DET_EPS = 1e-8


def _c4_view0(drop_degenerate: bool):
    """Config 4's scene and camera 0 on the device; with drop_degenerate, the
    Gaussians whose view-0 conic determinant is below CONIC_DET_EPS get zero
    opacity (they then take part nowhere, in the kernel or in the oracles)."""
    sc = config_3d(seed=0).to(DEV)
    if drop_degenerate:
        with torch.no_grad():
            _, q, _, _ = TR.project_pinhole(sc.means3d[None], sc.scales[None], sc.quats[None], sc.opacities[None],
                                            sc.camera_to_world[:1], sc.camera_params[:1], 1e-4)
            det = q[0, :, 0] * q[0, :, 2] - q[0, :, 1] ** 2
            sc.opacities[~(det >= CONIC_DET_EPS)] = 0.0
    return sc


def _c4_forward_backward(sc, n_busy=12, n_random=12):
    """The public 3D entry point's pieces (projection, then the rasterizer on the
    projected packet) on camera 0, with an N(0,1) upstream gradient on the
    n_busy busiest and n_random random tiles and zero elsewhere."""
    from torch_gsplat_bridge_fast.rasterize import _bin
    from workloads import grad_image

    H, W = sc.height, sc.width
    fx, fy, cx, cy = (float(v) for v in sc.camera_params[0])
    c2w = sc.camera_to_world[0]
    cfg = tgb.RasterConfig(H, W)
    params = [t.clone().requires_grad_(True) for t in (sc.means3d, sc.scales, sc.quats, sc.opacities, sc.colors)]
    m2, q2, o2, d2 = tgb.project_pinhole_gaussians(*params[:4], fx, fy, cx, cy, camera_to_world=c2w)
    for t in (m2, q2, o2):
        t.retain_grad()
    img = tgb.rasterize_projected_gaussians(m2, q2, params[4], o2, d2, cfg)
    with torch.no_grad():  # the one-call 3D entry point renders the same image
        img3 = tgb.rasterize_pinhole_gaussians(*(p.detach() for p in params), fx, fy, cx, cy, camera_to_world=c2w,
                                               config=cfg)
    assert torch.equal(img3, img.detach())
    tx, ty = (W + 15) // 16, (H + 15) // 16
    with torch.no_grad():
        st = _bin(cfg, m2[None].contiguous(), q2[None].contiguous(), params[4][None].detach().contiguous(),
                  o2[None].contiguous(), d2[None].contiguous())
    counts = (st.tile_offsets[1:] - st.tile_offsets[:-1]).cpu()
    assert int(counts.max()) > 2000, int(counts.max())
    gen = torch.Generator().manual_seed(7)
    busy = torch.argsort(counts, descending=True)[:n_busy]
    rnd = torch.randint(0, tx * ty, (n_random,), generator=gen)
    tiles = torch.unique(torch.cat([busy, rnd])).tolist()
    full = grad_image(1, H, W, seed=8)[0]
    gimg = torch.zeros(H, W, 3)
    for t in tiles:
        y0, x0 = (t // tx) * 16, (t % tx) * 16
        gimg[y0:y0 + 16, x0:x0 + 16] = full[y0:y0 + 16, x0:x0 + 16]
    img.backward(gimg.to(DEV))
    torch.cuda.synchronize()
    return dict(params=params, packet=(m2, q2, o2, d2), img=img, st=st, tiles=tiles, gimg=gimg, tx=tx, cfg=cfg)


def _tile_pixels(t, tx, H, W):
    y0, x0 = (t // tx) * 16, (t % tx) * 16
    yy, xx = torch.meshgrid(torch.arange(y0, min(y0 + 16, H)), torch.arange(x0, min(x0 + 16, W)), indexing="ij")
    return yy.reshape(-1), xx.reshape(-1)


def _check_projection_vjp(sc, params, packet):
    """The projection VJP at full scale against autograd through the reference's
    torch projection (_torch_project_pinhole_gaussians_batched), given the same
    2D gradients. As in test_projection_c4_scale_matches_torch_restatement,
    Gaussians within 0.2 of the camera plane are left out: there the EWA
    Jacobian overflows fp32 and the two evaluation orders give different
    non-finite values."""
    m2, q2, o2, d2 = packet
    r3 = [p.detach().clone().requires_grad_(True) for p in params[:4]]
    outs = TR.project_pinhole(*(t[None] for t in r3), sc.camera_to_world[:1], sc.camera_params[:1], 1e-4)
    torch.autograd.backward(outs[:3], [m2.grad[None], q2.grad[None], o2.grad[None]])
    keep = (d2.detach().abs() > 0.2).cpu().numpy()
    for a, b, name in zip(params[:4], r3, ("means3d", "scales", "quats", "opacities")):
        assert rel_err_finite(np_(a.grad)[keep], np_(b.grad)[keep]) <= GRAD_RTOL, name


def test_c4_scale_matches_kernel_restatement_and_oracle_on_its_lists():
    """Config 4 at full scale (2^20 Gaussians, one 1920x1080 camera, tiles of up
    to ~11,000 pairs: the long-tile CTA kernels and the reverse recurrence over
    long lists), with the reference kernel's semantics, degenerate conics
    included:
      * binning of the projected packet bit-exact against the C restatement of
        the reference's binning (permutation, keys, lists, ranges);
      * the full frame's image and the 2D gradients against the C oracle's
        forward and backward (upstream N(0,1) on 24 sampled tiles, 12 of them
        the busiest, zero elsewhere);
      * on those tiles, the reference's early-stop torch oracle
        (saturating_reference, float64) run on exactly the splats the
        reference kernel lists for the tile, image and 2D gradients;
      * the projection VJP against the reference's torch projection.
    Gates: image max-abs <= 1e-4, gradients <= 1e-3 relative."""
    sc = _c4_view0(drop_degenerate=False)
    r = _c4_forward_backward(sc)
    m2, q2, o2, d2 = r["packet"]
    H, W, tx, st = sc.height, sc.width, r["tx"], r["st"]
    G = m2.shape[0]
    cols = r["params"][4]
    host = [np_(t)[None].copy() for t in (m2, q2, cols, o2, d2)]
    meta = O.Meta(H, W, 1, G)
    perm, rec, off, P = O.bin_prepare(meta, *host)
    keys, ids, toff = O.bin_emit(meta, rec, off, P)
    assert st.P == P
    assert np.array_equal(np_(st.perm).reshape(-1), perm)
    assert np.array_equal(np_(st.tile_offsets), toff)
    assert np.array_equal(np_(st.binned_ids), ids)
    assert np.array_equal(np_(st.keys).view(np.uint64), keys)
    img_np = np_(r["img"])
    ref_img, _, _ = O.render_forward(meta, rec, toff, ids)
    assert max_abs(img_np, ref_img[0]) <= IMAGE_ATOL
    g_ref = O.unsort_grads(meta, perm, O.render_backward(meta, rec, toff, ids, r["gimg"][None].numpy()))
    for got, want, name in zip((m2.grad, q2.grad, cols.grad, o2.grad), g_ref, ("means2d", "conics", "colors", "opac")):
        assert rel_err(np_(got).reshape(want.shape), want) <= GRAD_RTOL, name

    ref = [t.detach().double().requires_grad_(i < 4) for i, t in enumerate((m2, q2, cols, o2, d2))]
    worst = 0.0
    for t in r["tiles"]:
        py, px = _tile_pixels(t, tx, H, W)
        listed = torch.from_numpy(perm[ids[toff[t]:toff[t + 1]]].astype(np.int64)).to(DEV)
        out_t = TR.saturating_reference_pixels(*(x[listed] for x in ref), px, py, chunk=2048)
        worst = max(worst, max_abs(img_np[py.numpy(), px.numpy()], np_(out_t)))
        (out_t * r["gimg"][py, px].to(DEV, torch.float64)).sum().backward()
    assert worst <= IMAGE_ATOL, worst
    # One Gaussian at the camera plane projects to a 2D mean near -9e6 px with
    # conic entries near 1e24; the kernel and the C oracle find it invisible
    # everywhere (zero gradient, checked above), while torch's autograd through
    # the oracle returns NaN for it. Entries that are finite on both sides are
    # compared; rel_err_finite allows at most 1e-5 of them to differ in that.
    for got, want, name in ((m2.grad, ref[0].grad, "means2d"), (q2.grad, ref[1].grad, "conics"),
                            (cols.grad, ref[2].grad, "colors"), (o2.grad, ref[3].grad, "opacities")):
        assert rel_err_finite(np_(got), np_(want)) <= GRAD_RTOL, name
    _check_projection_vjp(sc, r["params"], r["packet"])


def test_c4_scale_matches_dense_torch_oracle_without_degenerate_conics():
    """Config 4 at full scale against the reference's torch oracle with no
    binning at all: on each of 24 sampled tiles every splat whose support can
    reach the tile (_tile_candidates, a conservative superset) is composited by
    saturating_reference (float64), image and gradients of the same restricted
    loss. The Gaussians whose view-0 conic is degenerate (determinant below
    CONIC_DET_EPS, where the reference kernel and its torch oracle disagree)
    are given zero opacity first; everything else must agree."""
    sc = _c4_view0(drop_degenerate=True)
    r = _c4_forward_backward(sc)
    m2, q2, o2, d2 = r["packet"]
    H, W, tx = sc.height, sc.width, r["tx"]
    cols = r["params"][4]
    ref = [t.detach().double().requires_grad_(i < 4) for i, t in enumerate((m2, q2, cols, o2, d2))]
    img_np = np_(r["img"])
    worst = 0.0
    for t in r["tiles"]:
        py, px = _tile_pixels(t, tx, H, W)
        y0, x0 = (t // tx) * 16, (t % tx) * 16
        cand = _tile_candidates(ref[0].detach(), ref[1].detach(), ref[3].detach(), x0, y0, min(x0 + 16, W),
                                min(y0 + 16, H))
        out_t = TR.saturating_reference_pixels(*(x[cand] for x in ref), px, py, chunk=2048)
        worst = max(worst, max_abs(img_np[py.numpy(), px.numpy()], np_(out_t)))
        (out_t * r["gimg"][py, px].to(DEV, torch.float64)).sum().backward()
    assert worst <= IMAGE_ATOL, worst
    for got, want, name in ((m2.grad, ref[0].grad, "means2d"), (q2.grad, ref[1].grad, "conics"),
                            (cols.grad, ref[2].grad, "colors"), (o2.grad, ref[3].grad, "opacities")):
        assert rel_err(np_(got), np_(want)) <= GRAD_RTOL, name
    _check_projection_vjp(sc, r["params"], r["packet"])
