"""View-dependent colours from spherical harmonics (degree 0-3), differentiable.

Not part of the reference API, whose 3D entry point takes raw RGB colours
(variants/v8_project3d/torch_gsplat_bridge_v8_project3d/rasterize.py:958-1003). The
output plugs into `rasterize_pinhole_gaussians(..., colors=...)`:

    colors = spherical_harmonics_colors(sh, means3d, camera_to_world)   # [B,G,3]
    image = rasterize_pinhole_gaussians(means3d, scales, quats, opacities, colors, ...)

colour = max(0, 0.5 + sum_k sh[:, k] * Y_k(normalize(mean - camera centre))), the
camera centre being the translation column of the camera-to-world matrix.
"""
from __future__ import annotations

from typing import Optional

import torch
from torch import Tensor

from .rasterize import _ops

_K_OF_DEGREE = {0: 1, 1: 4, 2: 9, 3: 16}


class _ShColors(torch.autograd.Function):
    """gsplat_b200::sh_fwd / sh_bwd."""

    @staticmethod
    def forward(ctx, sh: Tensor, means3d: Tensor, c2w: Tensor, degree: int):
        colors = _ops().sh_fwd(sh, means3d, c2w, degree)
        ctx.save_for_backward(sh, means3d, c2w, colors)
        ctx.degree = degree
        return colors

    @staticmethod
    def backward(ctx, g_colors: Tensor):
        sh, means3d, c2w, colors = ctx.saved_tensors
        need = ctx.needs_input_grad
        g_sh, g_means, g_c2w = _ops().sh_bwd(sh, means3d, c2w, colors, g_colors, ctx.degree, bool(need[1]),
                                             bool(need[2]))
        return (g_sh if need[0] else None), g_means, g_c2w, None


def spherical_harmonics_colors(sh_coeffs: Tensor, means3d: Tensor, camera_to_world: Optional[Tensor] = None,
                               degree: Optional[int] = None) -> Tensor:
    """sh_coeffs [G, K, 3] (K = (degree+1)^2 >= the degree used), means3d [G, 3],
    camera_to_world [4,4] or [B,4,4] (default identity) -> colours [G,3] or [B,G,3].
    `degree` defaults to the largest one the coefficients hold."""
    if sh_coeffs.ndim != 3 or sh_coeffs.shape[-1] != 3:
        raise ValueError("sh_coeffs must have shape [G, K, 3]")
    if means3d.ndim != 2 or means3d.shape[-1] != 3 or means3d.shape[0] != sh_coeffs.shape[0]:
        raise ValueError("means3d must have shape [G, 3] matching sh_coeffs")
    if means3d.device.type != "cuda" or sh_coeffs.device != means3d.device:
        raise ValueError("sh_coeffs and means3d must be on the same CUDA device")
    if sh_coeffs.dtype != torch.float32 or means3d.dtype != torch.float32:
        raise ValueError("sh_coeffs and means3d must be float32")
    K = sh_coeffs.shape[1]
    if degree is None:
        degree = max(d for d, k in _K_OF_DEGREE.items() if k <= K) if K >= 1 else -1
    if degree not in _K_OF_DEGREE or _K_OF_DEGREE[degree] > K:
        raise ValueError(f"degree {degree} needs {_K_OF_DEGREE.get(degree, '?')} coefficients; got {K}")
    sh = sh_coeffs[:, :_K_OF_DEGREE[degree]].contiguous()
    batched = camera_to_world is not None and camera_to_world.ndim == 3
    if camera_to_world is None:
        c2w = torch.eye(4, dtype=torch.float32, device=means3d.device)[None]
    else:
        c2w = camera_to_world.to(device=means3d.device, dtype=torch.float32)
        if c2w.shape == (4, 4):
            c2w = c2w[None]
        if c2w.ndim != 3 or c2w.shape[1:] != (4, 4):
            raise ValueError("camera_to_world must be [4,4] or [B,4,4]")
    c2w = c2w.contiguous()
    colors = _ShColors.apply(sh, means3d.contiguous(), c2w, degree)
    return colors if batched else colors[0]
