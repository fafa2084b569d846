"""Shared test helpers (golden fixtures, error metrics)."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"

# Parity gates: image max-abs <= 1e-4, gradients <= 1e-3 relative,
# relative error of a gradient tensor = max|g - g_ref| / max(max|g_ref|, 1e-12).
IMAGE_ATOL = 1e-4
GRAD_RTOL = 1e-3
# The reference's own fixture tolerance (variants/v8_project3d/tests/reference_check.py:165-169).
REF_FIXTURE_ATOL = 1e-5


def golden(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz") as z:
        return {k: z[k] for k in z.files}


def max_abs(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.max(np.abs(a - b))) if a.size else 0.0


def rel_err(g, ref) -> float:
    g = np.asarray(g, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    if g.size == 0:
        return 0.0
    return float(np.max(np.abs(g - ref)) / max(float(np.max(np.abs(ref))), 1e-12))


def np_(t) -> np.ndarray:
    if isinstance(t, torch.Tensor):
        return t.detach().cpu().numpy()
    return np.asarray(t)


def upstream_grad(case: dict) -> np.ndarray:
    """The upstream image gradient a golden case was made with."""
    if str(case["loss"]) == "square_mean":
        img = case["image"].astype(np.float32)
        return (2.0 * img / img.size).astype(np.float32)
    return case["grad_image"].astype(np.float32)


def rel_err_finite(g, ref) -> float:
    """rel_err over entries finite on both sides; the non-finite pattern must agree
    (near-plane splats overflow to inf/nan identically in kernel and reference)."""
    g = np.asarray(g, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    fin_g, fin_r = np.isfinite(g), np.isfinite(ref)
    mismatch = np.mean(fin_g != fin_r) if g.size else 0.0
    assert mismatch <= 1e-5, f"finite pattern differs on {mismatch:.2e} of entries"
    both = fin_g & fin_r
    return rel_err(g[both], ref[both])
