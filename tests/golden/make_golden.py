"""Generates the golden fixtures in tests/golden/ by running the reference's OWN
torch code (nbardy/fast-mac-gsplat) on CPU. Run where a checkout of the
reference is available, with its path in GSPLAT_REF_ROOT; the GPU box never
runs this.

    GSPLAT_REF_ROOT=<reference checkout> python tests/golden/make_golden.py

Reference functions executed:
  variants/v8_project3d/tests/reference_check.py: dense_reference (15-50),
      saturating_reference (53-104), and the check_case / check_saturated_many_splats
      fixtures (114-214)
  benchmarks/benchmark_full_matrix.py: dense_torch_reference (128-152)
  variants/v8_project3d/torch_gsplat_bridge_v8_project3d/rasterize.py:
      _torch_project_pinhole_gaussians_batched (288-358)
  variants/v7_tiled_capture/torch_gsplat_bridge_v72/reference.py: tiled_scan_work (288-302)
"""
from __future__ import annotations

import importlib.util
import os
import sys
from pathlib import Path

import numpy as np
import torch

sys.dont_write_bytecode = True
if "GSPLAT_REF_ROOT" not in os.environ and __name__ == "__main__":
    sys.exit("set GSPLAT_REF_ROOT to the path of a reference checkout")
REF = Path(os.environ.get("GSPLAT_REF_ROOT", "."))
OUT = Path(__file__).resolve().parent


def _load(name: str, path: Path, extra_path: Path | None = None):
    if extra_path is not None and str(extra_path) not in sys.path:
        sys.path.insert(0, str(extra_path))
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def _np(t):
    return t.detach().cpu().numpy()


def raster_case(name, fn, means2d, conics, colors, opacities, depths, H, W, loss="square_mean", grad_image=None,
                **fn_kwargs):
    ins = [t.detach().clone().requires_grad_(True) for t in (means2d, conics, colors, opacities)]
    out = fn(*ins, depths, H, W, **fn_kwargs)
    if loss == "square_mean":
        out.square().mean().backward()
        gi = None
    else:
        out.backward(grad_image)
        gi = grad_image
    rec = dict(
        means2d=_np(means2d), conics=_np(conics), colors=_np(colors), opacities=_np(opacities), depths=_np(depths),
        H=np.int32(H), W=np.int32(W), image=_np(out), g_means2d=_np(ins[0].grad), g_conics=_np(ins[1].grad),
        g_colors=_np(ins[2].grad), g_opacities=_np(ins[3].grad), loss=np.array(loss),
    )
    if gi is not None:
        rec["grad_image"] = _np(gi)
    for k, v in fn_kwargs.items():
        rec["kw_" + k] = np.asarray(v)
    np.savez_compressed(OUT / f"{name}.npz", **rec)
    print("wrote", name, {k: v.shape for k, v in rec.items() if hasattr(v, "shape")})


def c0_like_inputs(B, G, H, W, seed, sigma_lo=0.5, sigma_hi=8.0):
    """BASELINE config-0 distribution (means uniform, sigma U[a,b], theta U[0,pi),
    opacity sigmoid(N(0,1)), rgb U[0,1], depth U[0.1,100])."""
    g = torch.Generator().manual_seed(seed)
    means = torch.rand(B, G, 2, generator=g) * torch.tensor([W, H], dtype=torch.float32)
    sig = torch.rand(B, G, 2, generator=g) * (sigma_hi - sigma_lo) + sigma_lo
    th = torch.rand(B, G, generator=g) * torch.pi
    op = torch.sigmoid(torch.randn(B, G, generator=g))
    rgb = torch.rand(B, G, 3, generator=g)
    depth = torch.rand(B, G, generator=g) * 99.9 + 0.1
    c, s = torch.cos(th), torch.sin(th)
    ia, ib = 1.0 / sig[..., 0] ** 2, 1.0 / sig[..., 1] ** 2
    conics = torch.stack([c * c * ia + s * s * ib, c * s * (ia - ib), s * s * ia + c * c * ib], -1)
    return means, conics, rgb, op, depth


def main():
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    rc = _load("ref_reference_check", REF / "variants/v8_project3d/tests/reference_check.py",
               REF / "variants/v8_project3d")
    bfm = _load("ref_benchmark_full_matrix", REF / "benchmarks/benchmark_full_matrix.py")
    v8p = sys.modules["torch_gsplat_bridge_v8_project3d.rasterize"]
    v72 = _load("ref_v72_reference", REF / "variants/v7_tiled_capture/torch_gsplat_bridge_v72/reference.py")

    # 1) reference_check.check_case fixtures (B=1, B=2), dense_reference, loss=mean(out^2).
    torch.manual_seed(0)
    G, H, W = 4, 16, 16
    for B in (1, 2):
        torch.manual_seed(0)
        means2d = torch.tensor([[[4.2, 5.1], [8.0, 7.5], [11.2, 8.1], [6.4, 12.0]],
                                [[3.7, 4.4], [7.1, 10.2], [12.2, 3.4], [10.4, 12.5]]])[:B]
        conics = torch.tensor([[[0.35, 0.02, 0.42], [0.28, -0.01, 0.33], [0.25, 0.04, 0.31], [0.40, 0.00, 0.27]],
                               [[0.31, 0.03, 0.38], [0.45, 0.01, 0.29], [0.22, -0.02, 0.35], [0.27, 0.05, 0.41]]])[:B]
        colors = torch.rand(B, G, 3)
        opacities = torch.tensor([[0.8, 0.6, 0.5, 0.7], [0.65, 0.55, 0.75, 0.45]])[:B]
        depths = torch.tensor([[0.1, 0.2, 0.3, 0.4], [0.3, 0.1, 0.4, 0.2]])[:B]
        raster_case(f"check_case_b{B}", rc.dense_reference, means2d, conics, colors, opacities, depths, H, W)

    # 2) check_saturated_many_splats fixture (seed 123), saturating_reference with white bg.
    torch.manual_seed(123)
    B, G, H, W = 1, 64, 32, 32
    means2d = torch.randn(B, G, 2)
    means2d = means2d * torch.tensor([W * 0.2, H * 0.2]) + torch.tensor([W * 0.5, H * 0.5])
    means2d[..., 0].clamp_(0, W - 1)
    means2d[..., 1].clamp_(0, H - 1)
    sigmas = torch.rand(B, G, 2) * 8.0 + 3.0
    conics = torch.stack([1.0 / sigmas[..., 0].square(), torch.zeros(B, G), 1.0 / sigmas[..., 1].square()], -1)
    colors = torch.rand(B, G, 3)
    opacities = torch.rand(B, G) * 0.45 + 0.45
    depths = (torch.arange(G, dtype=torch.float32) / float(G - 1)).view(1, G)
    raster_case("saturated_many_splats", rc.saturating_reference, means2d, conics, colors, opacities, depths, H, W,
                bg=(1.0, 1.0, 1.0))

    # 3) config-0 distribution at a fixture size, N(0,1) upstream grad, both oracles.
    B, G, H, W = 2, 96, 48, 40
    m, q, c, o, d = c0_like_inputs(B, G, H, W, seed=7)
    gimg = torch.randn(B, H, W, 3, generator=torch.Generator().manual_seed(8))
    raster_case("c0like_saturating", rc.saturating_reference, m, q, c, o, d, H, W, loss="grad_image",
                grad_image=gimg, bg=(0.0, 0.0, 0.0))
    raster_case("c0like_dense_torch_direct", lambda *a: bfm.dense_torch_reference(*a), m, q, c, o, d, H, W,
                loss="grad_image", grad_image=gimg)

    # 4) projection: the reference's torch restatement, with behind-camera splats.
    g = torch.Generator().manual_seed(11)
    B, G = 2, 64
    means3d = torch.randn(B, G, 3, generator=g) * 2.0
    means3d[:, :8, 2] = -torch.rand(8, generator=g) - 0.1  # behind the camera
    means3d[..., 2] += 4.0 * (torch.arange(G) >= 8).float()
    scales = torch.exp(torch.randn(B, G, 3, generator=g) * 0.5 - 1.0)
    quats = torch.randn(B, G, 4, generator=g)
    quats = quats / quats.norm(dim=-1, keepdim=True)
    opac = torch.sigmoid(torch.randn(B, G, generator=g))
    c2w = torch.eye(4).repeat(B, 1, 1)
    c2w[1, :3, 3] = torch.tensor([0.3, -0.2, 0.5])
    ang = 0.2
    c2w[1, :3, :3] = torch.tensor([[np.cos(ang), 0.0, np.sin(ang)], [0.0, 1.0, 0.0], [-np.sin(ang), 0.0, np.cos(ang)]],
                                  dtype=torch.float32)
    cam = torch.tensor([[300.0, 310.0, 64.0, 48.0], [280.0, 290.0, 60.0, 50.0]])
    ins = [t.clone().requires_grad_(True) for t in (means3d, scales, quats, opac, c2w, cam)]
    outs = v8p._torch_project_pinhole_gaussians_batched(*ins, 1e-4)
    ups = [torch.randn(t.shape, generator=g) for t in outs]
    torch.autograd.backward(outs, ups)
    np.savez_compressed(
        OUT / "project_pinhole.npz",
        means3d=_np(means3d), scales=_np(scales), quats=_np(quats), opacities=_np(opac), c2w=_np(c2w), cam=_np(cam),
        near_plane=np.float32(1e-4), means2d=_np(outs[0]), conics=_np(outs[1]), proj_opacities=_np(outs[2]),
        depths=_np(outs[3]), up_means2d=_np(ups[0]), up_conics=_np(ups[1]), up_opacities=_np(ups[2]),
        up_depths=_np(ups[3]), g_means3d=_np(ins[0].grad), g_scales=_np(ins[1].grad), g_quats=_np(ins[2].grad),
        g_opacities=_np(ins[3].grad), g_c2w=_np(ins[4].grad), g_cam=_np(ins[5].grad),
    )
    print("wrote project_pinhole")

    # 5) tiled_scan_work on a small offsets table.
    offs = torch.tensor([[0, 3, 3, 10, 12, 12, 20, 21, 30, 30, 31, 33, 40]], dtype=torch.int32)  # B=1, 12 tiles
    work = v72.tiled_scan_work(offs, height=40, width=60, tile_size=16)
    np.savez_compressed(OUT / "tiled_scan_work.npz", offsets=_np(offs), height=np.int32(40), width=np.int32(60),
                        work=np.int64(work))
    print("wrote tiled_scan_work", work)


if __name__ == "__main__":
    main()
