"""GPU pinhole projection (forward + VJP) and the full 3D path through the C ABI,
against the reference's torch projection (golden vectors) and its restatement."""
from __future__ import annotations

import pytest
import torch

import torch_gsplat_bridge_fast as tgb
from helpers import GRAD_RTOL, IMAGE_ATOL, golden, max_abs, np_, rel_err, rel_err_finite
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
