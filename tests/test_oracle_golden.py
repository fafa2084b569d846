"""Pins the oracles (torch restatements and the C oracle) to golden vectors made
by running the reference's own torch code (tests/golden/make_golden.py)."""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from helpers import GRAD_RTOL, REF_FIXTURE_ATOL, golden, max_abs, rel_err, upstream_grad
from oracle import oracle as O
from oracle import torch_ref as TR

RASTER_CASES = [
    ("check_case_b1", "dense", (0.0, 0.0, 0.0)),
    ("check_case_b2", "dense", (0.0, 0.0, 0.0)),
    ("saturated_many_splats", "saturating", (1.0, 1.0, 1.0)),
    ("c0like_saturating", "saturating", (0.0, 0.0, 0.0)),
    ("c0like_dense_torch_direct", "dense", (0.0, 0.0, 0.0)),
]


def _torch_inputs(c):
    return [torch.tensor(c[k], requires_grad=(k != "depths")) for k in
            ("means2d", "conics", "colors", "opacities", "depths")]


@pytest.mark.parametrize("name,kind,bg", RASTER_CASES)
def test_torch_restatement_matches_reference(name, kind, bg):
    c = golden(name)
    H, W = int(c["H"]), int(c["W"])
    m, q, col, o, d = _torch_inputs(c)
    fn = TR.dense_reference if kind == "dense" else TR.saturating_reference
    out = fn(m, q, col, o, d, H, W, bg=bg)
    out.backward(torch.tensor(upstream_grad(c)))
    assert max_abs(out.detach(), c["image"]) <= 1e-6
    for t, key in ((m, "g_means2d"), (q, "g_conics"), (col, "g_colors"), (o, "g_opacities")):
        assert rel_err(t.grad, c[key]) <= 1e-5, key


@pytest.mark.parametrize("name,kind,bg", RASTER_CASES)
def test_c_oracle_matches_reference(name, kind, bg):
    """The tiled C oracle (binning + compositing + reverse backward) reproduces
    the reference's dense torch renderer. For `dense` cases no pixel saturates,
    so the early stop does not change the result."""
    c = golden(name)
    H, W = int(c["H"]), int(c["W"])
    B, G = c["means2d"].shape[:2]
    meta = O.Meta(H, W, B, G, background=bg)
    r = O.full_forward_backward(meta, c["means2d"], c["conics"], c["colors"], c["opacities"], c["depths"],
                                upstream_grad(c))
    assert max_abs(r["image"], c["image"]) <= REF_FIXTURE_ATOL
    for g, key in zip(r["grads"], ("g_means2d", "g_conics", "g_colors", "g_opacities")):
        assert rel_err(g, c[key]) <= GRAD_RTOL, key
        assert max_abs(g, c[key]) <= 1e-4, key


def test_dense_and_saturating_agree_when_unsaturated():
    c = golden("c0like_dense_torch_direct")
    s = golden("c0like_saturating")
    assert max_abs(c["image"], s["image"]) <= 1e-4


def test_projection_restatement_matches_reference():
    c = golden("project_pinhole")
    ins = [torch.tensor(c[k], requires_grad=True) for k in ("means3d", "scales", "quats", "opacities", "c2w", "cam")]
    outs = TR.project_pinhole(*ins, float(c["near_plane"]))
    for o, key in zip(outs, ("means2d", "conics", "proj_opacities", "depths")):
        assert max_abs(o.detach(), c[key]) <= 1e-5 * max(1.0, float(np.abs(c[key]).max())), key
    torch.autograd.backward(outs, [torch.tensor(c[k]) for k in ("up_means2d", "up_conics", "up_opacities",
                                                               "up_depths")])
    for t, key in zip(ins, ("g_means3d", "g_scales", "g_quats", "g_opacities", "g_c2w", "g_cam")):
        assert rel_err(t.grad, c[key]) <= 1e-5, key


def test_c_oracle_projection_matches_reference():
    c = golden("project_pinhole")
    outs = O.project_forward(c["means3d"], c["scales"], c["quats"], c["opacities"], c["c2w"], c["cam"],
                             float(c["near_plane"]))
    for o, key in zip(outs, ("means2d", "conics", "proj_opacities", "depths")):
        assert rel_err(o, c[key]) <= 1e-5, key


def test_tiled_scan_work_matches_reference():
    c = golden("tiled_scan_work")
    got = TR.tiled_scan_work(torch.tensor(c["offsets"][0]), height=int(c["height"]), width=int(c["width"]))
    assert got == int(c["work"])


# --- binning restatement checks ------------------------------------------------


def test_det_log_is_accurate():
    L = O.lib()
    xs = np.concatenate([np.geomspace(1e-8, 1.0, 2000, endpoint=False), [0.5, 0.7071, 0.999999, 1e-8]])
    for x in xs:
        got = L.orc_det_log(float(x))
        ref = math.log(float(x))
        assert abs(got - ref) <= 4e-16 * max(1.0, abs(ref)), x


def test_depth_key_orders_like_torch_argsort():
    vals = np.array([3.0, -0.0, 0.0, -1.0, np.inf, -np.inf, np.nan, 1e-30, -1e-30, 2.0, 0.0, -0.0, np.nan, 5.0],
                    dtype=np.float32)
    L = O.lib()
    keys = np.array([L.orc_depth_key(float(v)) for v in vals], dtype=np.uint64)
    order = np.lexsort((np.arange(len(vals)), keys))
    ref = torch.argsort(torch.tensor(vals), stable=True).numpy()
    assert np.array_equal(order, ref)


def _py_tile_count(m, a, b, c, op, H, W, thr=1.0 / 255.0, eps=1e-8):
    """Independent pure-Python/numpy float32 restatement of count_tiles
    (…gsplat_v8_project3d_kernels.metal:530-572, 697-741)."""
    f = np.float32
    if not (f(op) > f(thr)):
        return []
    ratio = max(f(thr) / max(f(op), f(eps)), f(eps))
    tau = f(-2.0 * math.log(float(ratio)))
    if not (np.isfinite(tau) and tau > 0):
        return []
    a, b, c, mx, my = f(a), f(b), f(c), f(m[0]), f(m[1])
    det = max(a * c - b * b, f(eps))
    hx = np.sqrt(max(tau * c / det, f(0)))
    hy = np.sqrt(max(tau * a / det, f(0)))
    x0 = max(0, int(np.floor(mx - hx - f(0.5))))
    x1 = min(W - 1, int(np.ceil(mx + hx - f(0.5))))
    y0 = max(0, int(np.floor(my - hy - f(0.5))))
    y1 = min(H - 1, int(np.ceil(my + hy - f(0.5))))
    if x0 > x1 or y0 > y1:
        return []

    def q(dx, dy):
        return a * dx * dx + f(2) * b * dx * dy + c * dy * dy

    out = []
    tx_n = (W + 15) // 16
    for ty in range(y0 // 16, y1 // 16 + 1):
        ry0 = f(ty * 16) + f(0.5)
        ry1 = min(f(H - 1) + f(0.5), f((ty + 1) * 16 - 1) + f(0.5))
        for tx in range(x0 // 16, x1 // 16 + 1):
            rx0 = f(tx * 16) + f(0.5)
            rx1 = min(f(W - 1) + f(0.5), f((tx + 1) * 16 - 1) + f(0.5))
            if rx0 <= mx <= rx1 and ry0 <= my <= ry1:
                out.append(ty * tx_n + tx)
                continue
            dx0, dx1, dy0, dy1 = rx0 - mx, rx1 - mx, ry0 - my, ry1 - my
            qmin = min(q(dx0, dy0), q(dx0, dy1), q(dx1, dy0), q(dx1, dy1))
            if c > f(1e-8):
                for dxe in (dx0, dx1):
                    dy = min(max(-(b / c) * dxe, dy0), dy1)
                    qmin = min(qmin, q(dxe, dy))
            if a > f(1e-8):
                for dye in (dy0, dy1):
                    dx = min(max(-(b / a) * dye, dx0), dx1)
                    qmin = min(qmin, q(dx, dye))
            if qmin <= tau:
                out.append(ty * tx_n + tx)
    return out


def test_c_oracle_binning_matches_python_restatement():
    from workloads import make_2d

    s = make_2d(1, 300, 70, 90, seed=3, sigma=(0.5, 12.0))
    meta = O.Meta(70, 90, 1, 300)
    perm, rec, off, P = O.bin_prepare(meta, *(t.numpy() for t in s.tensors()))
    keys, ids, toff = O.bin_emit(meta, rec, off, P)
    for r in range(300):
        R = rec[r]
        want = _py_tile_count(R[0:2], R[2], R[3], R[4], R[5], 70, 90)
        got_tiles = sorted(int(k >> 32) for k, v in zip(keys, ids) if v == r)
        assert got_tiles == sorted(want), r


def test_binning_covers_every_visible_pixel():
    """A splat is listed for every tile holding a pixel where it is visible."""
    from workloads import make_2d

    H, W, G = 64, 80, 200
    s = make_2d(1, G, H, W, seed=5, sigma=(0.5, 10.0))
    meta = O.Meta(H, W, 1, G)
    perm, rec, off, P = O.bin_prepare(meta, *(t.numpy() for t in s.tensors()))
    keys, ids, toff = O.bin_emit(meta, rec, off, P)
    listed = set(zip((keys >> np.uint64(32)).astype(np.int64).tolist(), ids.tolist()))
    ys, xs = np.mgrid[0:H, 0:W].astype(np.float32) + np.float32(0.5)
    for r in range(G):
        R = rec[r]
        dx, dy = xs - R[0], ys - R[1]
        power = np.float32(-0.5) * (R[2] * dx * dx + np.float32(2) * R[3] * dx * dy + R[4] * dy * dy)
        alpha = np.minimum(np.float32(0.99), R[5] * np.exp(power))
        vis = (power <= 0) & (alpha >= np.float32(1.0 / 255.0) * np.float32(1.0001))
        for ty, tx in set(zip(*(np.nonzero(vis)[0] // 16, np.nonzero(vis)[1] // 16))):
            assert (int(ty) * ((W + 15) // 16) + int(tx), r) in listed, (r, ty, tx)


def test_c_oracle_ordering_is_depth_rank_within_tile():
    from workloads import make_2d

    s = make_2d(2, 150, 48, 64, seed=9, sigma=(2.0, 9.0))
    meta = O.Meta(48, 64, 2, 150)
    perm, rec, off, P = O.bin_prepare(meta, *(t.numpy() for t in s.tensors()))
    keys, ids, toff = O.bin_emit(meta, rec, off, P)
    depths = s.depths.numpy()
    for b in range(2):
        ref_perm = torch.argsort(torch.tensor(depths[b]), stable=True).numpy()
        assert np.array_equal(perm[b * 150:(b + 1) * 150], ref_perm)
    for t in range(meta.total_tiles):
        seg = ids[toff[t]:toff[t + 1]]
        assert np.all(np.diff(seg) > 0)
        assert np.all((keys[toff[t]:toff[t + 1]] >> np.uint64(32)) == t)


@pytest.mark.parametrize("name,bg", [("saturated_many_splats", (1.0, 1.0, 1.0)), ("c0like_saturating", (0, 0, 0))])
def test_pixel_sampled_saturating_matches_reference(name, bg):
    c = golden(name)
    H, W = int(c["H"]), int(c["W"])
    yy, xx = torch.meshgrid(torch.arange(H), torch.arange(W), indexing="ij")
    px, py = xx.reshape(-1), yy.reshape(-1)
    B = c["means2d"].shape[0]
    up = torch.tensor(upstream_grad(c))
    ins = _torch_inputs(c)
    outs = []
    for b in range(B):
        outs.append(TR.saturating_reference_pixels(ins[0][b], ins[1][b], ins[2][b], ins[3][b], ins[4][b], px, py,
                                                   bg=bg, chunk=17).reshape(H, W, 3))
    out = torch.stack(outs)
    out.backward(up)
    assert max_abs(out.detach(), c["image"]) <= 1e-5
    for t, key in zip(ins[:4], ("g_means2d", "g_conics", "g_colors", "g_opacities")):
        assert rel_err(t.grad, c[key]) <= 1e-4, key


def test_tile_stop_counts_follow_the_reference_definition():
    """oracle.tile_stop_counts / profile_stop_stats restate the per-tile stop count
    of tile_fast_forward_state (…kernels.metal:875-923: max over in-image pixels,
    0 for empty tiles and tiles above max_fast_pairs) and the statistics of
    profile_projected_gaussians (…/rasterize.py:1070-1085)."""
    meta = O.Meta(20, 40, 1, 1)  # 2 x 3 tiles; the bottom row of tiles is 4 pixels high
    counts = np.array([5, 0, 3000, 7, 2, 9], dtype=np.int64)
    toff = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
    last = np.zeros((1, 20, 40), dtype=np.int32)
    last[0, 3, 5], last[0, 9, 1] = 4, 5  # tile 0 -> 5
    last[0, 2, 20] = 1  # tile 1 is empty -> 0
    last[0, 0, 33] = 3000  # tile 2 is above the cap -> 0
    last[0, 17, 3] = 6  # tile 3 -> 6
    last[0, 19, 39] = 9  # tile 5 -> 9 (tile 4 stays 0)
    stops = O.tile_stop_counts(meta, toff, last, 2048)
    assert stops.tolist() == [5, 0, 0, 6, 0, 9]
    st = O.profile_stop_stats(counts, stops)
    assert st["max_stop_count"] == 9 and abs(st["mean_stop_count"] - 20 / 6) < 1e-6
    ratio = np.array([5 / 5, 0, 0, 6 / 7, 0, 9 / 9])
    assert abs(st["mean_stop_ratio"] - ratio.mean()) < 1e-6
    assert abs(st["p95_stop_ratio"] - float(np.quantile(ratio, 0.95))) < 1e-6
