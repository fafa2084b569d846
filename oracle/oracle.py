"""ctypes wrapper over the C oracle (oracle/gsplat_oracle.c) — test infrastructure.

Builds oracle/_build/liboracle.so on first use when it is missing (gcc + make).
All arrays are numpy, C-contiguous, fp32/int32/uint64.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from dataclasses import dataclass
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "liboracle.so"
REC = 12


class OrcMeta(C.Structure):
    _fields_ = [
        ("height", C.c_int32),
        ("width", C.c_int32),
        ("tile_size", C.c_int32),
        ("batch_size", C.c_int32),
        ("gaussians_per_batch", C.c_int32),
        ("alpha_threshold", C.c_float),
        ("transmittance_threshold", C.c_float),
        ("background", C.c_float * 3),
        ("eps", C.c_float),
        ("max_alpha", C.c_float),
    ]


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = C.CDLL(str(LIB_PATH))
        p = C.c_void_p
        L.orc_bin_prepare.restype = C.c_int64
        L.orc_bin_prepare.argtypes = [C.POINTER(OrcMeta)] + [p] * 8
        L.orc_bin_emit.restype = None
        L.orc_bin_emit.argtypes = [C.POINTER(OrcMeta), p, p, C.c_int64, p, p, p]
        L.orc_render_forward.restype = None
        L.orc_render_forward.argtypes = [C.POINTER(OrcMeta)] + [p] * 6
        L.orc_render_backward.restype = None
        L.orc_render_backward.argtypes = [C.POINTER(OrcMeta)] + [p] * 5
        L.orc_project_forward.restype = None
        L.orc_project_forward.argtypes = [C.c_int, C.c_int] + [p] * 6 + [C.c_float] + [p] * 4
        L.orc_depth_key.restype = C.c_uint32
        L.orc_depth_key.argtypes = [C.c_float]
        L.orc_det_log.restype = C.c_double
        L.orc_det_log.argtypes = [C.c_double]
        _lib = L
    return _lib


@dataclass
class Meta:
    height: int
    width: int
    batch_size: int
    gaussians_per_batch: int
    alpha_threshold: float = 1.0 / 255.0
    transmittance_threshold: float = 1e-4
    background: tuple = (0.0, 0.0, 0.0)
    eps: float = 1e-8
    max_alpha: float = 0.99

    def c(self) -> OrcMeta:
        m = OrcMeta()
        m.height, m.width, m.tile_size = self.height, self.width, 16
        m.batch_size, m.gaussians_per_batch = self.batch_size, self.gaussians_per_batch
        m.alpha_threshold, m.transmittance_threshold = self.alpha_threshold, self.transmittance_threshold
        m.background = (C.c_float * 3)(*self.background)
        m.eps, m.max_alpha = self.eps, self.max_alpha
        return m

    @property
    def tiles_x(self):
        return (self.width + 15) // 16

    @property
    def tiles_y(self):
        return (self.height + 15) // 16

    @property
    def total_tiles(self):
        return self.tiles_x * self.tiles_y * self.batch_size


def _f32(x):
    return np.ascontiguousarray(np.asarray(x, dtype=np.float32))


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def bin_prepare(meta: Meta, means2d, conics, colors, opacities, depths):
    """-> perm [BG] int32, rec [BG,12] f32, pair_offsets [BG+1] int32, total P."""
    BG = meta.batch_size * meta.gaussians_per_batch
    arrs = [_f32(a).reshape(-1) for a in (means2d, conics, colors, opacities, depths)]
    perm = np.zeros(BG, np.int32)
    rec = np.zeros((BG, REC), np.float32)
    off = np.zeros(BG + 1, np.int32)
    mc = meta.c()
    P = lib().orc_bin_prepare(C.byref(mc), *map(_ptr, arrs), _ptr(perm), _ptr(rec), _ptr(off))
    return perm, rec, off, int(P)


def bin_emit(meta: Meta, rec, pair_offsets, P):
    """-> keys [P] uint64, binned_ids [P] int32, tile_offsets [tiles+1] int32."""
    rec = _f32(rec)
    off = np.ascontiguousarray(pair_offsets, dtype=np.int32)
    keys = np.zeros(max(P, 1), np.uint64)
    ids = np.zeros(max(P, 1), np.int32)
    toff = np.zeros(meta.total_tiles + 1, np.int32)
    mc = meta.c()
    lib().orc_bin_emit(C.byref(mc), _ptr(rec), _ptr(off), P, _ptr(keys), _ptr(ids), _ptr(toff))
    return keys[:P], ids[:P], toff


def render_forward(meta: Meta, rec, tile_offsets, ids):
    """-> image [B,H,W,3], final_T [B,H,W], last_idx [B,H,W]."""
    B, H, W = meta.batch_size, meta.height, meta.width
    out = np.zeros((B, H, W, 3), np.float32)
    T = np.zeros((B, H, W), np.float32)
    last = np.zeros((B, H, W), np.int32)
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    if ids.size == 0:
        ids = np.zeros(1, np.int32)
    mc = meta.c()
    lib().orc_render_forward(C.byref(mc), _ptr(_f32(rec)), _ptr(np.ascontiguousarray(tile_offsets, np.int32)),
                             _ptr(ids), _ptr(out), _ptr(T), _ptr(last))
    return out, T, last


def render_backward(meta: Meta, rec, tile_offsets, ids, grad_rgb):
    """-> grad_rec [BG,12] (depth-rank order, packed layout)."""
    BG = meta.batch_size * meta.gaussians_per_batch
    g = np.zeros((max(BG, 1), REC), np.float32)
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    if ids.size == 0:
        ids = np.zeros(1, np.int32)
    mc = meta.c()
    lib().orc_render_backward(C.byref(mc), _ptr(_f32(rec)), _ptr(np.ascontiguousarray(tile_offsets, np.int32)),
                              _ptr(ids), _ptr(_f32(grad_rgb)), _ptr(g))
    return g[:BG]


def unsort_grads(meta: Meta, perm, grad_rec):
    """Packed rank-order grads -> (g_means2d [B,G,2], g_conics [B,G,3], g_colors [B,G,3], g_opac [B,G])."""
    B, G = meta.batch_size, meta.gaussians_per_batch
    gr = np.asarray(grad_rec).reshape(B, G, REC)
    perm = np.asarray(perm).reshape(B, G)
    out = np.zeros((B, G, REC), np.float32)
    for b in range(B):
        out[b, perm[b]] = gr[b]
    return out[..., 0:2], out[..., 2:5], out[..., 6:9], out[..., 5]


def project_forward(means3d, scales, quats, opacities, c2w, cam, near_plane):
    m3 = _f32(means3d)
    B, G = m3.shape[:2]
    out_m = np.zeros((B, G, 2), np.float32)
    out_c = np.zeros((B, G, 3), np.float32)
    out_o = np.zeros((B, G), np.float32)
    out_d = np.zeros((B, G), np.float32)
    lib().orc_project_forward(B, G, _ptr(m3), _ptr(_f32(scales)), _ptr(_f32(quats)), _ptr(_f32(opacities)),
                              _ptr(_f32(c2w)), _ptr(_f32(cam)), float(near_plane), _ptr(out_m), _ptr(out_c),
                              _ptr(out_o), _ptr(out_d))
    return out_m, out_c, out_o, out_d


def full_forward_backward(meta: Meta, means2d, conics, colors, opacities, depths, grad_image):
    """Whole pipeline on the CPU: binning, forward, backward, un-sort."""
    perm, rec, off, P = bin_prepare(meta, means2d, conics, colors, opacities, depths)
    keys, ids, toff = bin_emit(meta, rec, off, P)
    img, T, last = render_forward(meta, rec, toff, ids)
    grad_rec = render_backward(meta, rec, toff, ids, grad_image)
    grads = unsort_grads(meta, perm, grad_rec)
    return dict(perm=perm, rec=rec, pair_offsets=off, P=P, keys=keys, ids=ids, tile_offsets=toff, image=img,
                final_T=T, last_idx=last, grad_rec=grad_rec, grads=grads)


def tile_stop_counts(meta: Meta, tile_offsets, last_idx, max_fast_pairs: int) -> np.ndarray:
    """Per-tile stop count as tile_fast_forward_state writes it
    (variants/v8_project3d/csrc/metal/gsplat_v8_project3d_kernels.metal:875-923): 0 for an
    empty tile and for a tile above max_fast_pairs (left to the overflow path,
    :876-884); otherwise the max over the tile's in-image pixels of local_stop,
    the number of list entries the pixel walked (chunk_start + j + 1 up to and
    including the entry that saturated it, :903-916). last_idx [B,H,W] is the C
    oracle's per-pixel count of consumed entries, which is that local_stop."""
    B, H, W = meta.batch_size, meta.height, meta.width
    tx, ty = (W + 15) // 16, (H + 15) // 16
    counts = np.diff(np.asarray(tile_offsets, dtype=np.int64)).reshape(B, ty, tx)
    pad = np.zeros((B, ty * 16, tx * 16), dtype=np.int64)
    pad[:, :H, :W] = np.asarray(last_idx, dtype=np.int64).reshape(B, H, W)
    stop = pad.reshape(B, ty, 16, tx, 16).max(axis=(2, 4))
    stop[(counts == 0) | (counts > int(max_fast_pairs))] = 0
    return stop.reshape(-1)


def profile_stop_stats(counts, stops) -> dict:
    """The stop statistics of profile_projected_gaussians
    (variants/v8_project3d/torch_gsplat_bridge_v8_project3d/rasterize.py:1070-1085) from
    per-tile pair counts and stop counts."""
    import torch

    c = torch.as_tensor(np.asarray(counts), dtype=torch.float32)
    s = torch.as_tensor(np.asarray(stops), dtype=torch.float32)
    ratio = torch.where(c > 0, s / torch.clamp(c, min=1.0), torch.zeros_like(s))
    return {"mean_stop_count": float(s.mean().item()), "p95_stop_count": float(torch.quantile(s, 0.95).item()),
            "max_stop_count": int(s.max().item()), "mean_stop_ratio": float(ratio.mean().item()),
            "p95_stop_ratio": float(torch.quantile(ratio, 0.95).item())}
