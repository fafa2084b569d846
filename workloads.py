"""Seeded synthetic workloads for the five configurations of BASELINE.json.

No public dataset is used by the reference or named by the benchmark config, so
these generators stand in with the stated shapes and value distributions:
  c0  B=1, 512x512, G=512 uniform 2D splats (the CPU-runnable dense case)
  c1  B=1, 1920x1080, G=65,536, 80% in 8 gaussian clusters (sigma 40 px), 20% uniform
  c2  B=4, 1024x512, G=2,048/view, 16 depth layers, sigma U[8,32], opacity U[0.3,0.7]
  c3  B=1, 4096x4096, G=65,536 uniform, sigma U[0.5,8]  (the headline config)
  c4  G=2^20 shared 3D Gaussians, 8 pinhole cameras 1920x1080, 60 deg fov, radius-25 sphere
Inputs are drawn on the CPU from a seeded torch.Generator (field order: means,
sigma, rotation, opacity, rgb, depth, grad_image) and then moved to the device.
Means are not clamped to the screen. 2D covariances are R diag(sx^2, sy^2) R^T
and are passed as their inverse (the conic a, b, c).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

CONFIGS = ("c0", "c1", "c2", "c3", "c4")


@dataclass
class Splats2D:
    means2d: torch.Tensor  # [B,G,2]
    conics: torch.Tensor  # [B,G,3]
    colors: torch.Tensor  # [B,G,3]
    opacities: torch.Tensor  # [B,G]
    depths: torch.Tensor  # [B,G]
    height: int
    width: int

    def to(self, device):
        return Splats2D(*(t.to(device) for t in self.tensors()), self.height, self.width)

    def tensors(self):
        return (self.means2d, self.conics, self.colors, self.opacities, self.depths)

    @property
    def B(self):
        return self.means2d.shape[0]

    @property
    def G(self):
        return self.means2d.shape[1]


@dataclass
class Splats3D:
    means3d: torch.Tensor  # [G,3]
    scales: torch.Tensor  # [G,3] linear
    quats: torch.Tensor  # [G,4] (r,i,j,k), normalised
    opacities: torch.Tensor  # [G] probabilities
    colors: torch.Tensor  # [G,3]
    camera_to_world: torch.Tensor  # [V,4,4]
    camera_params: torch.Tensor  # [V,4] fx, fy, cx, cy
    height: int
    width: int

    def to(self, device):
        return Splats3D(self.means3d.to(device), self.scales.to(device), self.quats.to(device),
                        self.opacities.to(device), self.colors.to(device), self.camera_to_world.to(device),
                        self.camera_params.to(device), self.height, self.width)


def conic_from_sigma(sig: torch.Tensor, theta: torch.Tensor) -> torch.Tensor:
    c, s = torch.cos(theta), torch.sin(theta)
    ia, ib = 1.0 / sig[..., 0].square(), 1.0 / sig[..., 1].square()
    return torch.stack([c * c * ia + s * s * ib, c * s * (ia - ib), s * s * ia + c * c * ib], -1).contiguous()


def make_2d(B: int, G: int, H: int, W: int, seed: int, *, sigma=(0.5, 8.0), kind: str = "uniform") -> Splats2D:
    g = torch.Generator().manual_seed(seed)
    scale = torch.tensor([W, H], dtype=torch.float32)
    if kind == "uniform":
        means = torch.rand(B, G, 2, generator=g) * scale
    elif kind == "clustered":
        n_cl = 8
        centres = torch.rand(B, n_cl, 2, generator=g) * scale
        which = torch.randint(0, n_cl, (B, G), generator=g)
        clustered = torch.gather(centres, 1, which[..., None].expand(B, G, 2)) + torch.randn(B, G, 2, generator=g) * 40.0
        uniform = torch.rand(B, G, 2, generator=g) * scale
        pick = torch.rand(B, G, 1, generator=g) < 0.8
        means = torch.where(pick, clustered, uniform)
    elif kind == "layered":
        means = torch.rand(B, G, 2, generator=g) * scale
    else:
        raise ValueError(kind)
    sig = torch.rand(B, G, 2, generator=g) * (sigma[1] - sigma[0]) + sigma[0]
    theta = torch.rand(B, G, generator=g) * math.pi
    if kind == "layered":
        opac = torch.rand(B, G, generator=g) * 0.4 + 0.3
    else:
        opac = torch.sigmoid(torch.randn(B, G, generator=g))
    rgb = torch.rand(B, G, 3, generator=g)
    if kind == "layered":
        layer = torch.randint(0, 16, (B, G), generator=g).float()
        depth = layer + torch.rand(B, G, generator=g) * 0.5
    else:
        depth = torch.rand(B, G, generator=g) * 99.9 + 0.1
    return Splats2D(means.contiguous(), conic_from_sigma(sig, theta), rgb.contiguous(), opac.contiguous(),
                    depth.contiguous(), H, W)


def grad_image(B: int, H: int, W: int, seed: int) -> torch.Tensor:
    return torch.randn(B, H, W, 3, generator=torch.Generator().manual_seed(seed))


def config_2d(name: str, seed: int = 0) -> Splats2D:
    if name == "c0":
        return make_2d(1, 512, 512, 512, seed)
    if name == "c1":
        return make_2d(1, 65536, 1080, 1920, seed, sigma=(1.0, 6.0), kind="clustered")
    if name == "c2":
        return make_2d(4, 2048, 512, 1024, seed, sigma=(8.0, 32.0), kind="layered")
    if name == "c3":
        return make_2d(1, 65536, 4096, 4096, seed)
    raise ValueError(f"not a 2D config: {name}")


def look_at_c2w(position: torch.Tensor) -> torch.Tensor:
    """Camera-to-world [4,4] with camera +z (column 2) towards the origin,
    x right and y down (columns 0, 1), translation in column 3."""
    fwd = -position / position.norm()
    up = torch.tensor([0.0, 0.0, 1.0]) if abs(float(fwd[2])) < 0.95 else torch.tensor([0.0, 1.0, 0.0])
    right = torch.linalg.cross(fwd, up)
    right = right / right.norm()
    down = torch.linalg.cross(fwd, right)
    M = torch.eye(4)
    M[:3, 0], M[:3, 1], M[:3, 2], M[:3, 3] = right, down, fwd, position
    return M


def config_3d(G: int = 1 << 20, views: int = 8, seed: int = 0, H: int = 1080, W: int = 1920,
              radius: float = 25.0) -> Splats3D:
    g = torch.Generator().manual_seed(seed)
    means = torch.randn(G, 3, generator=g) * 10.0
    scales = torch.exp(torch.randn(G, 3, generator=g) * 0.5 - 1.0)
    quats = torch.randn(G, 4, generator=g)
    quats = quats / quats.norm(dim=-1, keepdim=True)
    opac = torch.sigmoid(torch.randn(G, generator=g))
    rgb = torch.rand(G, 3, generator=g)
    dirs = torch.randn(views, 3, generator=g)
    dirs = dirs / dirs.norm(dim=-1, keepdim=True)
    c2w = torch.stack([look_at_c2w(d * radius) for d in dirs])
    f = (W / 2) / math.tan(math.radians(30.0))
    cam = torch.tensor([[f, f, W / 2, H / 2]] * views, dtype=torch.float32)
    return Splats3D(means.contiguous(), scales.contiguous(), quats.contiguous(), opac.contiguous(), rgb.contiguous(),
                    c2w.contiguous(), cam, H, W)


TRACE_KEYS = ("means2d", "conics", "colors", "opacities", "depths")


def load_trace(path: str, height: int, width: int, batch: int = 0, gaussians: int = 0) -> Splats2D:
    """A recorded frame batch instead of synthetic splats: a torch.save'd dict
    with the five projected-splat tensors ([G,...] or [B,G,...]), truncated to
    the requested batch/gaussian counts when they are positive. Same contract
    as the reference benchmark's real_trace case
    (variants/v8/benchmarks/benchmark_mps.py:26-46)."""
    data = torch.load(path, map_location="cpu")
    missing = [k for k in TRACE_KEYS if k not in data]
    if missing:
        raise ValueError(f"trace file is missing {missing[0]!r}")
    ts = [data[k].to(dtype=torch.float32) for k in TRACE_KEYS]
    if ts[0].ndim == 2:
        ts = [t.unsqueeze(0) for t in ts]
    B0, G0 = ts[0].shape[:2]
    B = min(B0, batch) if batch > 0 else B0
    G = min(G0, gaussians) if gaussians > 0 else G0
    ts = [t[:B, :G].contiguous() for t in ts]
    return Splats2D(*ts, height, width)
