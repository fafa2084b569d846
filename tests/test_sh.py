"""Spherical-harmonic colours: the torch restatement of the real SH basis
(oracle/torch_ref.py) is checked against known values and orthonormality on the
sphere (CPU); the CUDA kernels are checked against it, forward and backward (GPU)."""
from __future__ import annotations

import math

import pytest
import torch

from oracle import torch_ref as TR


def _fibonacci_sphere(n: int) -> torch.Tensor:
    i = torch.arange(n, dtype=torch.float64) + 0.5
    z = 1 - 2 * i / n
    r = torch.sqrt(1 - z * z)
    phi = math.pi * (3 - math.sqrt(5)) * i
    return torch.stack([r * torch.cos(phi), r * torch.sin(phi), z], -1)


def test_sh_basis_zonal_values():
    """Y_l0 at the pole is sqrt((2l+1)/(4 pi)); the other terms vanish there."""
    Y = TR.sh_basis(torch.tensor([[0.0, 0.0, 1.0]], dtype=torch.float64), 3)[0]
    expect = torch.zeros(16, dtype=torch.float64)
    for l, k in ((0, 0), (1, 2), (2, 6), (3, 12)):
        expect[k] = math.sqrt((2 * l + 1) / (4 * math.pi))
    assert torch.allclose(Y, expect, atol=1e-12)


def test_sh_basis_orthonormal_on_sphere():
    d = _fibonacci_sphere(200_000)
    Y = TR.sh_basis(d, 3)
    gram = (Y.T @ Y) * (4 * math.pi / d.shape[0])
    assert torch.allclose(gram, torch.eye(16, dtype=torch.float64), atol=2e-4)


def _case(G, B, seed, K=16):
    g = torch.Generator().manual_seed(seed)
    sh = torch.randn(G, K, 3, generator=g) * 0.5
    means = torch.randn(G, 3, generator=g) * 5.0
    c2w = torch.eye(4).repeat(B, 1, 1)
    c2w[:, :3, 3] = torch.randn(B, 3, generator=g) * 20.0
    return sh, means, c2w


@pytest.mark.gpu
@pytest.mark.parametrize("degree", [0, 1, 2, 3])
@pytest.mark.parametrize("B", [1, 3])
def test_sh_colors_match_torch_reference(degree, B):
    import torch_gsplat_bridge_fast as tgb

    dev = torch.device("cuda:0")
    sh, means, c2w = _case(3000, B, seed=degree * 10 + B)
    up = torch.randn(B, 3000, 3, generator=torch.Generator().manual_seed(7))
    ref_in = [t.clone().double().requires_grad_(True) for t in (sh, means, c2w)]
    ref = TR.sh_colors_reference(*ref_in, degree)
    ref.backward(up.double())
    gpu_in = [t.to(dev).requires_grad_(True) for t in (sh, means, c2w)]
    out = tgb.spherical_harmonics_colors(gpu_in[0], gpu_in[1], gpu_in[2], degree=degree)
    out.backward(up.to(dev))
    assert (out.detach().cpu().double() - ref.detach()).abs().max() <= 1e-5
    for a, r in zip(gpu_in, ref_in):
        ga = a.grad.cpu().double()
        gr = r.grad if r.grad is not None else torch.zeros_like(ga)  # degree 0: no direction dependence
        assert (ga - gr).abs().max() <= 1e-4 * max(gr.abs().max().item(), 1e-12), (degree, B)
