"""GPU binning parity through the C ABI: depth permutation, packed records, scan
offsets, 64-bit pair keys, sorted intersection lists and tile ranges must be
bit-identical to the C oracle (oracle/gsplat_oracle.c)."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

import torch_gsplat_bridge_fast as tgb
from torch_gsplat_bridge_fast import _native as N
from torch_gsplat_bridge_fast.rasterize import _bin
from oracle import oracle as O
from workloads import Splats2D, config_2d, make_2d

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def gpu_bin(s: Splats2D):
    cfg = tgb.RasterConfig(s.height, s.width)
    st = _bin(cfg, *(t.to(DEV).contiguous() for t in s.tensors()))
    torch.cuda.synchronize()
    return dict(perm=st.perm.cpu().numpy().reshape(-1), rec=st.rec.cpu().numpy(),
                pair_offsets=st.pair_offsets.cpu().numpy(), P=st.P,
                keys=st.keys.cpu().numpy().view(np.uint64), ids=st.binned_ids.cpu().numpy(),
                tile_offsets=st.tile_offsets.cpu().numpy())


def cpu_bin(s: Splats2D):
    meta = O.Meta(s.height, s.width, s.B, s.G)
    perm, rec, off, P = O.bin_prepare(meta, *(t.numpy() for t in s.tensors()))
    keys, ids, toff = O.bin_emit(meta, rec, off, P)
    return dict(perm=perm, rec=rec, pair_offsets=off, P=P, keys=keys, ids=ids, tile_offsets=toff)


def assert_bin_equal(g, c):
    assert g["P"] == c["P"]
    assert np.array_equal(g["perm"], c["perm"])
    assert np.array_equal(g["rec"].view(np.uint32), c["rec"].view(np.uint32))
    assert np.array_equal(g["pair_offsets"], c["pair_offsets"])
    assert np.array_equal(g["keys"], c["keys"])
    assert np.array_equal(g["ids"], c["ids"])
    assert np.array_equal(g["tile_offsets"], c["tile_offsets"])


@pytest.mark.parametrize("name", ["c0", "c1", "c2", "c3"])
def test_binning_bit_exact_configs(name):
    s = config_2d(name, seed=0)
    assert_bin_equal(gpu_bin(s), cpu_bin(s))


@pytest.mark.parametrize("B,G,H,W,sigma", [
    (1, 1, 16, 16, (2.0, 3.0)),
    (1, 7, 17, 33, (0.5, 30.0)),
    (3, 513, 70, 90, (0.5, 12.0)),
    (2, 4097, 129, 257, (1.0, 40.0)),
    (5, 3000, 31, 47, (0.5, 8.0)),
    (2, 20001, 200, 300, (0.5, 4.0)),
    (1, 65537, 256, 256, (0.5, 2.0)),
    (1, 300_001, 1024, 1024, (0.5, 2.0)),  # from 2^16 splats: pair offsets by reduce-then-scan
    (2, 140_001, 512, 768, (0.5, 3.0)),
])
def test_binning_bit_exact_ragged(B, G, H, W, sigma):
    s = make_2d(B, G, H, W, seed=B * 1000 + G, sigma=sigma)
    assert_bin_equal(gpu_bin(s), cpu_bin(s))


def test_binning_edge_values():
    """Ties, signed zeros, NaN/inf depths, degenerate conics, zero/over-unit
    opacities and off-screen or non-finite means bin identically."""
    s = make_2d(2, 600, 64, 96, seed=77, sigma=(0.5, 20.0))
    d = s.depths
    d[0, :50] = 1.0  # ties
    d[0, 50:60] = -0.0
    d[0, 60:70] = 0.0
    d[0, 70] = float("nan")
    d[0, 71] = float("inf")
    d[0, 72] = -float("inf")
    d[1, :100] = -torch.rand(100) * 10
    o = s.opacities
    o[0, 100:120] = 0.0
    o[0, 120:130] = 1.0 / 255.0
    o[0, 130:140] = 1.7
    o[1, 200:210] = float("nan")
    q = s.conics
    q[0, 150:160] = torch.tensor([1.0, 2.0, 1.0])  # det < 0
    q[0, 160:170] = torch.tensor([0.0, 0.0, 0.0])
    q[0, 170:175] = torch.tensor([1e-12, 0.0, 1e-12])  # huge support
    m = s.means2d
    m[0, 180:190] = torch.tensor([-500.0, 30.0])
    m[0, 190:200] = torch.tensor([5e9, -5e9])
    m[1, 300:305] = float("nan")
    m[1, 305:310] = float("inf")
    assert_bin_equal(gpu_bin(s), cpu_bin(s))


def test_binning_row_walk_edges():
    """k_prepare finds most hit tiles row by row from the support ellipse's
    extent in each tile row (with margins on both sides of the threshold) and
    sends only the tiles between the sure and the possible runs to the exact
    ellipse-rectangle test. Splats near the limits of that walk must bin
    exactly as the oracle does: axis ratios around the admitted 64:1 (k =
    4096), minor radii down to a few hundredths of a pixel, opacities just
    above the alpha threshold (tiny tau), means on tile edges, pixel centres
    and tile centres, and frames whose last tile row and column are one pixel
    wide."""
    B, G, H, W = 2, 6000, 16 * 20 + 1, 16 * 24 + 1
    g = torch.Generator().manual_seed(4242)
    s = make_2d(B, G, H, W, seed=4243)
    major = torch.exp(torch.rand(B, G, generator=g) * (np.log(80.0) - np.log(0.03)) + np.log(0.03))
    ratios = torch.tensor([1.0, 8.0, 32.0, 60.0, 63.9, 64.0, 64.1, 66.0, 80.0, 200.0, 1000.0])
    ratio = ratios[torch.randint(0, len(ratios), (B, G), generator=g)]
    theta = torch.rand(B, G, generator=g) * np.pi
    theta[:, ::7] = 0.0
    theta[:, 1::7] = np.pi / 4
    from workloads import conic_from_sigma
    s.conics.copy_(conic_from_sigma(torch.stack([major, major / ratio], -1), theta))
    m = s.means2d
    third = G // 3
    k = torch.randint(0, 24, (B, third), generator=g).float() * 16.0
    off = torch.tensor([0.0, 0.5, 8.0, 15.5, 16.0])[torch.randint(0, 5, (B, third), generator=g)]
    m[:, :third, 0] = k + off
    m[:, :third, 1] = torch.randint(0, 20, (B, third), generator=g).float() * 16.0 + 8.0
    m[:, third:2 * third] = torch.floor(m[:, third:2 * third]) + 0.5
    o = s.opacities
    o[:, ::5] = (1.0 / 255.0) * (1.0 + 1e-6)
    o[:, 1::5] = 1.0
    assert_bin_equal(gpu_bin(s), cpu_bin(s))


@pytest.mark.parametrize("B,G", [(1, 65536), (1, 40001), (1, 65537), (2, 30001), (3, 8192), (2, 8193)])
def test_depth_order_with_ties(B, G):
    """Depths drawn from 37 values: the depth order must keep input order within
    each tie, across sort partitions and across views (one view: 32-bit keys)."""
    s = make_2d(B, G, 96, 128, seed=G + B, sigma=(0.5, 3.0))
    s.depths.copy_(torch.floor(s.depths / 100.0 * 37.0) + 0.5)
    assert_bin_equal(gpu_bin(s), cpu_bin(s))


def test_binning_empty_and_zero_pairs():
    s = make_2d(1, 64, 32, 32, seed=1)
    s.opacities.zero_()  # nothing visible -> P = 0
    g = gpu_bin(s)
    assert g["P"] == 0 and np.all(g["tile_offsets"] == 0)
    assert_bin_equal(g, cpu_bin(s))


def test_binning_is_deterministic():
    s = config_2d("c1", seed=3)
    a, b = gpu_bin(s), gpu_bin(s)
    for k in ("perm", "pair_offsets", "keys", "ids", "tile_offsets"):
        assert np.array_equal(a[k], b[k]), k


def _sort(keys: np.ndarray, vals: np.ndarray, begin: int, end: int):
    L = N.load()
    n = keys.size
    k_in = torch.from_numpy(keys.view(np.int64)).to(DEV)
    v_in = torch.from_numpy(vals.view(np.int32)).to(DEV)
    k_out = torch.empty_like(k_in)
    v_out = torch.empty_like(v_in)
    status = torch.zeros(8, dtype=torch.int32, device=DEV)
    ws_n = L.gsb_radix_sort_pairs_workspace_size(n, begin, end)
    ws = torch.empty(max(ws_n, 1), dtype=torch.uint8, device=DEV)
    rc = L.gsb_radix_sort_pairs(N.ptr(k_in), N.ptr(v_in), N.ptr(k_out), N.ptr(v_out), n, begin, end, N.ptr(status),
                                N.ptr(ws), ws_n, N.stream_ptr(DEV))
    N.check(rc, "sort")
    torch.cuda.synchronize()
    assert int(status[1]) == 0
    return k_out.cpu().numpy().view(np.uint64), v_out.cpu().numpy().view(np.uint32)


@pytest.mark.parametrize("n,begin,end", [(1, 0, 8), (4095, 0, 32), (4096, 32, 48), (4097, 5, 19),
                                         (100_000, 0, 64), (1_000_003, 32, 45), (300_000, 0, 0),
                                         (2_000_001, 10, 11), (700_001, 40, 51),
                                         (28_673, 3, 40), (32_768, 0, 64), (32_769, 0, 33),
                                         (4_194_304, 0, 16), (4_200_001, 0, 40), (5_000_003, 29, 64)])
def test_radix_sort_is_stable_and_exact(n, begin, end):
    """Sizes on both sides of the partition sizes (1,024 / 2,048 / 4,096 keys)
    and of the item-count switches, full and partial last partitions; from
    2^22 keys the first pass takes its prefixes from the reduce-then-scan
    kernels instead of the look-back."""
    rng = np.random.default_rng(n + begin)
    keys = rng.integers(0, 2**63, n, dtype=np.uint64) | (rng.integers(0, 2, n, dtype=np.uint64) << np.uint64(63))
    keys[: n // 3] &= np.uint64(0xFFFF0000FFFF00FF)  # many ties
    vals = np.arange(n, dtype=np.uint32)
    k, v = _sort(keys, vals, begin, end)
    width = end - begin
    if width == 0:
        assert np.array_equal(k, keys) and np.array_equal(v, vals)
        return
    mask = np.uint64((1 << width) - 1) if width < 64 else np.uint64(0xFFFFFFFFFFFFFFFF)
    digit = (keys >> np.uint64(begin)) & mask
    order = np.argsort(digit, kind="stable")
    assert np.array_equal(v, vals[order])
    assert np.array_equal(k, keys[order])


@pytest.mark.parametrize("name", ["c1", "c2"])
def test_emit_without_masks_matches(name):
    """gsb_bin_emit re-tests every candidate tile when no hit masks are given
    (tile_masks = NULL, the C-ABI example's path); its pairs must equal those
    written from the masks, and the oracle's."""
    s = config_2d(name, seed=3)
    cfg = tgb.RasterConfig(s.height, s.width)
    st = _bin(cfg, *(t.to(DEV).contiguous() for t in s.tensors()))
    L = N.load()
    T = st.tile_offsets.numel() - 1
    keys = torch.empty(st.P, dtype=torch.int64, device=DEV)
    ids = torch.empty(st.P, dtype=torch.int32, device=DEV)
    toff = torch.empty(T + 1, dtype=torch.int32, device=DEV)
    status = torch.zeros(N.GSB_STATUS_WORDS, dtype=torch.int32, device=DEV)
    wsb = int(L.gsb_bin_emit_workspace_size(st.meta, st.P))
    ws = torch.empty(max(wsb, 1), dtype=torch.uint8, device=DEV)
    N.check(L.gsb_bin_emit(st.meta, N.ptr(st.rec), N.ptr(st.pair_offsets), None, st.P, N.ptr(keys), N.ptr(ids),
                           N.ptr(toff), N.ptr(status), N.ptr(ws), wsb, N.stream_ptr(DEV)), "gsb_bin_emit")
    torch.cuda.synchronize()
    assert int(status[N.GSB_STATUS_ERROR]) == 0
    assert torch.equal(keys, st.keys) and torch.equal(ids, st.binned_ids) and torch.equal(toff, st.tile_offsets)
    c = cpu_bin(s)
    assert np.array_equal(keys.cpu().numpy().view(np.uint64), c["keys"])


@pytest.mark.parametrize("B,G,H,W,sigma", [
    (1, 1, 16, 16, (2.0, 3.0)),          # one tile: no sort pass, k_ranges path
    (1, 7, 17, 33, (0.5, 30.0)),         # 6 tiles, most of them empty: one pass
    (1, 300, 256, 256, (0.5, 4.0)),      # 256 tiles: one 8-bit pass
    (1, 60, 1024, 1024, (0.5, 3.0)),     # sparse: long runs of empty tiles
    (2, 4097, 129, 257, (1.0, 40.0)),
    (5, 2000, 2048, 2048, (0.5, 6.0)),   # 81,920 tiles: three passes
    (5, 500, 4096, 4096, (0.5, 3.0)),    # 327,680 tiles, 1,280 blocks of 256
    (1, 20000, 4096, 4096, (20.0, 60.0)),  # 4.2M pairs: reduce-then-scan first pass, ranges in the last
])
def test_emit_tile_ranges_without_keys(B, G, H, W, sigma):
    """gsb_bin_emit_ranges (the host runtime's call for many pairs per tile):
    the last tile-sort pass records each tile's and each 256-tile block's
    first pair and k_ranges_fix fills the offsets (empty tiles and empty
    blocks included); ids and offsets must equal gsb_bin_emit's and the
    oracle's."""
    s = make_2d(B, G, H, W, seed=B * 7 + G, sigma=sigma)
    cfg = tgb.RasterConfig(s.height, s.width)
    st = _bin(cfg, *(t.to(DEV).contiguous() for t in s.tensors()))
    L = N.load()
    T = st.tile_offsets.numel() - 1
    ids = torch.full((max(st.P, 1),), -7, dtype=torch.int32, device=DEV)
    toff = torch.full((T + 1,), -7, dtype=torch.int32, device=DEV)
    status = torch.zeros(N.GSB_STATUS_WORDS, dtype=torch.int32, device=DEV)
    wsb = int(L.gsb_bin_emit_workspace_size(st.meta, st.P))
    ws = torch.empty(max(wsb, 1), dtype=torch.uint8, device=DEV)
    N.check(L.gsb_bin_emit_ranges(st.meta, N.ptr(st.rec), N.ptr(st.pair_offsets), None, st.P, N.ptr(ids),
                                  N.ptr(toff), N.ptr(status), N.ptr(ws), wsb, N.stream_ptr(DEV)),
            "gsb_bin_emit_ranges")
    torch.cuda.synchronize()
    assert int(status[N.GSB_STATUS_ERROR]) == 0
    assert torch.equal(ids[:st.P], st.binned_ids) and torch.equal(toff, st.tile_offsets)
    c = cpu_bin(s)
    assert np.array_equal(ids[:st.P].cpu().numpy(), c["ids"])
    assert np.array_equal(toff.cpu().numpy(), c["tile_offsets"])


def test_emit_tile_ranges_without_pairs():
    """No visible splat: gsb_bin_emit_ranges writes all-zero tile offsets."""
    s = make_2d(2, 64, 40, 70, seed=5, sigma=(1.0, 4.0))
    s.opacities.zero_()
    cfg = tgb.RasterConfig(s.height, s.width)
    st = _bin(cfg, *(t.to(DEV).contiguous() for t in s.tensors()))
    assert st.P == 0
    L = N.load()
    T = st.tile_offsets.numel() - 1
    ids = torch.empty(1, dtype=torch.int32, device=DEV)
    toff = torch.full((T + 1,), -7, dtype=torch.int32, device=DEV)
    status = torch.zeros(N.GSB_STATUS_WORDS, dtype=torch.int32, device=DEV)
    wsb = int(L.gsb_bin_emit_workspace_size(st.meta, 0))
    ws = torch.empty(max(wsb, 1), dtype=torch.uint8, device=DEV)
    N.check(L.gsb_bin_emit_ranges(st.meta, N.ptr(st.rec), N.ptr(st.pair_offsets), None, 0, N.ptr(ids),
                                  N.ptr(toff), N.ptr(status), N.ptr(ws), wsb, N.stream_ptr(DEV)),
            "gsb_bin_emit_ranges")
    torch.cuda.synchronize()
    assert int(toff.abs().sum()) == 0


@pytest.mark.parametrize("sigma,G,H,W", [
    ((20.0, 120.0), 600, 512, 640),   # hundreds to thousands of candidate tiles per splat: hit bits
    ((150.0, 300.0), 300, 1024, 1024),  # every splat covers the frame: the bit region (8 words a splat) fills up
])
def test_large_splat_hit_bits_match_oracle(sigma, G, H, W):
    """Splats with more than 64 candidate tiles keep their hit bits in the
    region after tile_masks' slots, and k_emit reads them instead of testing the
    tiles again; when the region is full the remaining splats are tested again.
    Both ways, the keys, lists and ranges equal the oracle's bit for bit, and
    the region's cursor (status word GSB_STATUS_MASK_WORDS) shows bits were
    handed out."""
    s = make_2d(2, G, H, W, seed=21, sigma=sigma)
    g = gpu_bin(s)
    c = cpu_bin(s)
    assert_bin_equal(g, c)
    cfg = tgb.RasterConfig(s.height, s.width)
    st = _bin(cfg, *(t.to(DEV).contiguous() for t in s.tensors()))
    torch.cuda.synchronize()
    used = int(st.status[N.GSB_STATUS_MASK_WORDS])
    capacity = 8 * s.B * s.G
    assert used > 0
    if sigma[0] >= 150.0:
        assert used > capacity  # asked for more than the region holds: some splats re-tested


def test_radix_sort_accepts_keys_that_are_not_16_byte_aligned():
    """The exported sort takes a caller's pointers: keys one element into a
    tensor are 8-byte but not 16-byte aligned, so the histogram pass must read
    them one by one instead of with 16-byte loads."""
    L = N.load()
    n = 100_001
    rng = np.random.default_rng(11)
    keys = rng.integers(0, 2**40, n + 1, dtype=np.uint64)
    vals = np.arange(n + 1, dtype=np.uint32)
    k_all = torch.from_numpy(keys.view(np.int64)).to(DEV)
    v_all = torch.from_numpy(vals.view(np.int32)).to(DEV)
    k_in, v_in = k_all[1:], v_all[1:]
    assert k_in.data_ptr() % 16 == 8
    k_out, v_out = torch.empty_like(k_in), torch.empty_like(v_in)
    status = torch.zeros(N.GSB_STATUS_WORDS, dtype=torch.int32, device=DEV)
    ws_n = L.gsb_radix_sort_pairs_workspace_size(n, 0, 40)
    ws = torch.empty(ws_n, dtype=torch.uint8, device=DEV)
    N.check(L.gsb_radix_sort_pairs(N.ptr(k_in), N.ptr(v_in), N.ptr(k_out), N.ptr(v_out), n, 0, 40, N.ptr(status),
                                   N.ptr(ws), ws_n, N.stream_ptr(DEV)), "sort")
    torch.cuda.synchronize()
    assert int(status[N.GSB_STATUS_ERROR]) == 0
    order = np.argsort(keys[1:], kind="stable")
    assert np.array_equal(k_out.cpu().numpy().view(np.uint64), keys[1:][order])
    assert np.array_equal(v_out.cpu().numpy().view(np.uint32), vals[1:][order])
