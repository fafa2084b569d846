"""B200 (sm_100a) differentiable Gaussian-splat rasterizer, drop-in for the
torch API of nbardy/fast-mac-gsplat (torch_gsplat_bridge_fast/__init__.py:1-2 and
variants/v8_project3d/torch_gsplat_bridge_v8_project3d/__init__.py:1-21)."""
from .rasterize import (
    ProjectedGaussianRasterizer,
    check_device_errors,
    RasterConfig,
    RuntimeShaderConfig,
    get_runtime_shader_config,
    profile_projected_gaussians,
    project_pinhole_gaussians,
    rasterize_pinhole_gaussians,
    rasterize_projected_gaussians,
)
from .sh import spherical_harmonics_colors

__all__ = [
    "RasterConfig",
    "RuntimeShaderConfig",
    "get_runtime_shader_config",
    "ProjectedGaussianRasterizer",
    "project_pinhole_gaussians",
    "rasterize_pinhole_gaussians",
    "rasterize_projected_gaussians",
    "profile_projected_gaussians",
    "spherical_harmonics_colors",
]
