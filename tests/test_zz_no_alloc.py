"""The allocation-free forward entry point (gsb_render_forward_noalloc) against the
regular one (gsb_render_forward, caller-provided workspace), through the C ABI.

Some callers cannot allocate device memory: a host that owns all of it and hands
this library only input and output buffers. The compositing forward needs no
scratch (the CTA kernel for long tiles finds them itself), so that entry point
takes no workspace. This test runs it twice in a row on a scene with long tiles
and checks both results against the workspace entry point at the tolerance the
compositing tests use.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

import torch_gsplat_bridge_fast as tgb
from helpers import IMAGE_ATOL, max_abs, np_
from torch_gsplat_bridge_fast import _native as N
from torch_gsplat_bridge_fast.rasterize import _bin, _render_forward
from workloads import config_2d

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _noalloc_forward(st, cfg, B):
    L = N.load()
    H, W = cfg.height, cfg.width
    out = torch.full((B, H, W, 3), float("nan"), device=DEV)
    final_T = torch.full((B, H, W), float("nan"), device=DEV)
    last_idx = torch.full((B, H, W), -7, dtype=torch.int32, device=DEV)
    pair_rec = torch.empty((max(st.P, 1), N.GSB_REC_FLOATS), device=DEV)
    status = torch.zeros(N.GSB_STATUS_WORDS, dtype=torch.int32, device=DEV)
    rc = L.gsb_render_forward_noalloc(st.meta, N.ptr(st.rec), N.ptr(st.tile_offsets), N.ptr(st.binned_ids),
                                      N.ptr(out), N.ptr(final_T), N.ptr(last_idx), N.ptr(pair_rec),
                                      N.ptr(status), N.stream_ptr(DEV))
    N.check(rc, "gsb_render_forward_noalloc")
    torch.cuda.synchronize()
    assert int(status[N.GSB_STATUS_ERROR]) == 0
    return out, final_T, last_idx


def test_noalloc_forward_matches_workspace_forward_twice():
    s = config_2d("c1", seed=0)  # clustered: has tiles above the warp-kernel cap (the CTA kernel's share)
    cfg = tgb.RasterConfig(s.height, s.width)
    st = _bin(cfg, *(t.to(DEV) for t in s.tensors()))
    counts = np.diff(st.tile_offsets.cpu().numpy())
    assert counts.max() > 64
    ref_out, ref_T, ref_last, _ = _render_forward(st, cfg, s.B, save_state=True)
    torch.cuda.synchronize()
    for _ in range(2):
        out, final_T, last_idx = _noalloc_forward(st, cfg, s.B)
        assert max_abs(np_(out), np_(ref_out)) <= IMAGE_ATOL
        assert max_abs(np_(final_T), np_(ref_T)) <= IMAGE_ATOL
        assert np.array_equal(np_(last_idx), np_(ref_last))


def test_noalloc_forward_has_no_tile_cap():
    """The compositing kernels need no scratch, so a frame of 4 x 4112^2 pixels
    (264,196 tiles) is not refused for capacity; with no buffers the call fails
    its argument check instead."""
    L = N.load()
    meta = N.make_meta(4112, 4112, 4, 1, 1 / 255, 1e-4, (0.0, 0.0, 0.0))
    rc = L.gsb_render_forward_noalloc(C.byref(meta), None, None, None, None, None, None, None, None, None)
    assert rc == 1  # GSB_ERR_INVALID_ARGUMENT, not GSB_ERR_CAPACITY (4)
