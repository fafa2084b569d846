"""CPU-side checks: the C-ABI library loads and exports every declared symbol,
argument validation needs no GPU, and the host API mirrors the reference's
configuration and error behaviour."""
from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

import pytest
import torch

import torch_gsplat_bridge_fast as tgb
from torch_gsplat_bridge_fast import _native as N
from torch_gsplat_bridge_fast.rasterize import _choose_batch_chunk_size

HEADER = Path(__file__).resolve().parents[1] / "include" / "gsplat_b200.h"


def _declared_symbols():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(gsb_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    L = N.load()
    declared = _declared_symbols()
    assert declared, "no declarations parsed"
    for name in declared:
        assert hasattr(L, name), name
    assert set(declared) == set(N.EXPORTED)


def _header_defines():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return {k: int(v) for k, v in re.findall(r"#define\s+(GSB_[A-Z0-9_]+)\s+(\d+)u?\b", text)}


def test_binding_constants_match_the_header():
    """The ctypes binding mirrors the header's constants (status-block layout,
    record size, peer buffer layout, device error flags) with the same values."""
    defines = _header_defines()
    must = [k for k in defines if k.startswith(("GSB_STATUS_", "GSB_REC_", "GSB_PEER_"))]
    assert "GSB_STATUS_WORDS" in must and "GSB_STATUS_TILE_CLAIM" in must
    for name in must:
        assert getattr(N, name) == defines[name], name
    for name, value in defines.items():
        if hasattr(N, name):
            assert getattr(N, name) == value, name
        if name.startswith("GSB_DEVERR_"):
            assert getattr(N, name[4:]) == value, name  # DEVERR_* in the binding
    words = [v for k, v in defines.items() if k.startswith("GSB_STATUS_") and k != "GSB_STATUS_WORDS"]
    assert max(words) + 1 <= defines["GSB_STATUS_WORDS"]


def test_device_error_decoding_names_every_flag():
    for flag, text in [(N.DEVERR_LOOKBACK_TIMEOUT, "look-back"), (N.DEVERR_PAIR_OVERFLOW, "pair count"),
                       (N.DEVERR_BOUNDS, "out of bounds"), (N.DEVERR_PEER_TIMEOUT, "peer rank")]:
        msg = N.decode_device_error(flag, 3)
        assert text in msg and "unknown" not in msg, msg
    assert "unknown" in N.decode_device_error(0, 0)


def test_version_and_status_strings():
    L = N.load()
    assert L.gsb_version() >= 100
    assert L.gsb_status_string(0) == b"ok"
    assert b"tile_size" in L.gsb_status_string(2)


def _meta(**kw):
    d = dict(height=64, width=80, batch_size=2, gaussians_per_batch=100, alpha_threshold=1 / 255,
             transmittance_threshold=1e-4, background=(0, 0, 0))
    d.update(kw)
    return N.make_meta(**d)


def test_workspace_queries_without_gpu():
    L = N.load()
    m = _meta()
    assert L.gsb_bin_prepare_workspace_size(C.byref(m)) > 100 * 2 * 8
    assert L.gsb_bin_emit_workspace_size(C.byref(m), 1000) > 1000 * 12
    assert L.gsb_bin_emit_workspace_size(C.byref(m), 0) >= 0
    assert L.gsb_radix_sort_pairs_workspace_size(1 << 20, 32, 48) > (1 << 20) * 12
    assert L.gsb_render_workspace_size(C.byref(m)) == 0  # compositing needs no scratch
    bad = _meta(tile_size=8)
    assert L.gsb_bin_prepare_workspace_size(C.byref(bad)) == 0


def test_sort_workspace_carves_prefix_scratch_from_2_22_keys():
    """From 2^22 keys with two or more passes, the first pass takes its
    prefixes from the reduce-then-scan kernels, whose per-partition counts
    (4,096-key partitions, 256 words per pass) and group sums (256-partition
    groups) are carved after the look-back words; one-pass sorts and shorter
    inputs carve none."""
    L = N.load()
    n = 1 << 22
    parts, groups = n // 4096, n // 4096 // 256
    for begin, end, passes in ((0, 16, 2), (3, 40, 5), (0, 64, 8)):
        grow = L.gsb_radix_sort_pairs_workspace_size(n, begin, end) - \
            L.gsb_radix_sort_pairs_workspace_size(n - 1, begin, end)
        scratch = 4 * 256 * passes * (parts + groups)
        assert scratch <= grow < scratch + 4096, (begin, end, grow, scratch)
    one = L.gsb_radix_sort_pairs_workspace_size(n, 0, 8) - L.gsb_radix_sort_pairs_workspace_size(n - 1, 0, 8)
    assert one < 4096


def test_argument_validation_without_gpu():
    L = N.load()
    bad = _meta(tile_size=8)
    rc = L.gsb_bin_prepare(C.byref(bad), *([None] * 9), None, 0, None)
    assert rc == 2  # GSB_ERR_UNSUPPORTED
    m = _meta()
    rc = L.gsb_bin_prepare(C.byref(m), *([None] * 9), None, 0, None)
    assert rc == 1  # null pointers
    rc = L.gsb_render_forward(C.byref(_meta(height=0)), None, None, None, None, None, None, None, None, None, 0, None)
    assert rc == 1
    rc = L.gsb_radix_sort_pairs(None, None, None, None, -1, 0, 8, None, None, 0, None)
    assert rc == 1
    rc = L.gsb_radix_sort_pairs(None, None, None, None, 1 << 31, 0, 8, None, None, 0, None)
    assert rc == 4  # capacity
    with pytest.raises(N.NativeError, match="status 2"):
        N.check(2, "x")


def test_raster_config_defaults_and_aliases():
    from torch_gsplat_bridge_fast.rasterize import _runtime_validate

    cfg = tgb.RasterConfig(height=32, width=48)
    assert cfg.tile_size == 16 and cfg.max_fast_pairs == 2048 and cfg.enable_overflow_fallback
    assert cfg.max_tile_pairs == 4096 and cfg.pair_cap == 2048
    # The root API's positional form (torch_gsplat_bridge_fast/rasterize.py:15-23):
    # the 4th field is max_tile_pairs = 4096, and the config validates.
    root = tgb.RasterConfig(32, 48, 16, 4096, 1.0 / 255.0, 1e-4, (0.0, 0.0, 0.0))
    assert root.max_tile_pairs == 4096 and root.background == (0.0, 0.0, 0.0)
    _runtime_validate(root)
    assert tgb.RasterConfig(32, 48, 16, 1000).pair_cap == 1000
    # v8's fields 5-17 keep their positions (variants/v8/…/rasterize.py:65-82).
    v8 = tgb.RasterConfig(32, 48, 16, 2048, 0.01, 1e-3, (1.0, 1.0, 1.0), False, "serial", 100, 200, True, "auto",
                          False, "never", 32, 1000)
    assert (v8.alpha_threshold, v8.transmittance_threshold, v8.background) == (0.01, 1e-3, (1.0, 1.0, 1.0))
    assert (v8.enable_overflow_fallback, v8.batch_strategy, v8.batch_launch_limit_tiles) == (False, "serial", 100)
    assert (v8.batch_launch_limit_gaussians, v8.use_active_tiles, v8.active_policy) == (200, True, "auto")
    assert (v8.sort_active_tiles_by_count, v8.stop_count_mode, v8.stop_count_dense_threshold) == (False, "never", 32)
    assert v8.max_pairs_per_launch == 1000 and v8.pair_cap == 2048
    _runtime_validate(v8)
    # v8's keyword cap, checked against the runtime fast cap as v8 does.
    assert tgb.RasterConfig(32, 48, max_fast_pairs=512).pair_cap == 512
    with pytest.raises(ValueError, match="exceeds compiled fast cap"):
        _runtime_validate(tgb.RasterConfig(32, 48, max_fast_pairs=4096))
    for bad, msg in ((dict(active_policy="sometimes"), "active_policy"), (dict(stop_count_mode="x"), "stop_count_mode"),
                     (dict(stop_count_dense_threshold=0), "stop_count_dense_threshold"),
                     (dict(max_pairs_per_launch=-1), "max_pairs_per_launch")):
        with pytest.raises(ValueError, match=msg):
            _runtime_validate(tgb.RasterConfig(32, 48, **bad))


def test_runtime_shader_config_env(monkeypatch):
    rt = tgb.get_runtime_shader_config()
    assert (rt.tile_size, rt.threads, rt.chunk_size, rt.fast_cap, rt.simdgroups) == (16, 256, 64, 2048, 8)
    monkeypatch.setenv("GSP_TILE_SIZE", "12")
    with pytest.raises(ValueError, match="GSP_TILE_SIZE"):
        tgb.get_runtime_shader_config()
    monkeypatch.setenv("GSP_TILE_SIZE", "16")
    monkeypatch.setenv("GSP_CHUNK", "0")
    with pytest.raises(ValueError, match="GSP_CHUNK"):
        tgb.get_runtime_shader_config()


def _inputs(B=None, G=8, device="cpu"):
    shp = (G,) if B is None else (B, G)
    return (torch.zeros(*shp, 2, device=device), torch.zeros(*shp, 3, device=device),
            torch.zeros(*shp, 3, device=device), torch.zeros(*shp, device=device), torch.zeros(*shp, device=device))


def test_input_validation_messages():
    cfg = tgb.RasterConfig(16, 16)
    with pytest.raises(ValueError, match="must be on CUDA"):
        tgb.rasterize_projected_gaussians(*_inputs(), cfg)
    m, q, c, o, d = _inputs()
    with pytest.raises(ValueError, match="same device"):
        tgb.rasterize_projected_gaussians(m.to("meta"), q, c, o, d, cfg)
    with pytest.raises(ValueError, match="must be on CUDA"):
        tgb.project_pinhole_gaussians(torch.zeros(4, 3), torch.zeros(4, 3), torch.zeros(4, 4), torch.zeros(4),
                                      1.0, 1.0, 0.0, 0.0)
    with pytest.raises(ValueError, match="config is required"):
        tgb.rasterize_pinhole_gaussians(torch.zeros(4, 3), torch.zeros(4, 3), torch.zeros(4, 4), torch.zeros(4),
                                        torch.zeros(4, 3), 1.0, 1.0, 0.0, 0.0)


def test_batch_chunk_policy_matches_reference():
    cfg = tgb.RasterConfig(4096, 4096)
    assert _choose_batch_chunk_size(cfg, 1, 65536, 65536) == 1
    assert _choose_batch_chunk_size(tgb.RasterConfig(512, 1024), 4, 2048, 2048) == 4
    assert _choose_batch_chunk_size(tgb.RasterConfig(512, 1024, batch_strategy="serial"), 4, 2048, 2048) == 1
    assert _choose_batch_chunk_size(cfg, 8, 65536, 65536) == 4


def test_trace_replay_loader(tmp_path):
    """The trace format of the reference benchmark's real_trace case: a dict of the
    five splat tensors, [G,...] or [B,G,...], truncated to the requested sizes."""
    from workloads import load_trace, make_2d

    s = make_2d(2, 300, 64, 80, seed=4)
    path = tmp_path / "trace.pt"
    torch.save({k: t for k, t in zip(("means2d", "conics", "colors", "opacities", "depths"), s.tensors())}, path)
    t = load_trace(str(path), 64, 80, batch=1, gaussians=200)
    assert (t.B, t.G, t.height, t.width) == (1, 200, 64, 80)
    assert torch.equal(t.means2d, s.means2d[:1, :200])
    torch.save({k: v[0] for k, v in zip(("means2d", "conics", "colors", "opacities", "depths"), s.tensors())}, path)
    assert load_trace(str(path), 64, 80).means2d.shape == (1, 300, 2)
    torch.save({"means2d": s.means2d}, path)
    with pytest.raises(ValueError, match="missing"):
        load_trace(str(path), 64, 80)


_OPS = ("rasterize_fwd", "bin", "render_fwd_eval", "render_fwd_train", "render_bwd", "project_fwd", "project_bwd",
        "sh_fwd", "sh_bwd")


def test_torch_op_namespace_registered_for_cuda_only():
    """torch.ops.gsplat_b200 mirrors the reference's op namespace
    (variants/v8_project3d/csrc/bindings.cpp:173-193) with scalar meta
    arguments; only the CUDA dispatch key has kernels, so CPU tensors raise
    instead of reaching a fallback."""
    from torch_gsplat_bridge_fast.rasterize import _host_args, _ops

    ops = _ops()
    for name in _OPS:
        schema = str(getattr(ops, name).default._schema)
        assert schema.startswith(f"gsplat_b200::{name}("), schema
    raster = "int height, int width, float alpha_threshold, float transmittance_threshold, float bg_r, float bg_g, " \
             "float bg_b, float eps, float max_alpha"
    for name in ("rasterize_fwd", "bin", "render_fwd_eval", "render_fwd_train", "render_bwd"):
        assert raster in str(getattr(ops, name).default._schema), name
    assert "Tensor(a!) status" in str(ops.render_bwd.default._schema)
    args = _host_args(tgb.RasterConfig(16, 16))
    assert len(args) == 9
    cpu = (torch.zeros(1, 4, 2), torch.zeros(1, 4, 3), torch.zeros(1, 4, 3), torch.zeros(1, 4), torch.zeros(1, 4))
    with pytest.raises(NotImplementedError, match="CPU"):
        ops.rasterize_fwd(*cpu, *args, False, -1)
    with pytest.raises(NotImplementedError, match="CPU"):
        ops.sh_fwd(torch.zeros(4, 1, 3), torch.zeros(4, 3), torch.eye(4)[None], 0)


def _fast_div_magic(d):
    """make_fast_div (csrc/gsb_host.cuh): shift = ceil(log2 d),
    mul = floor(2^32 (2^shift - d) / d) + 1."""
    shift = 0
    while (1 << shift) < d:
        shift += 1
    return ((1 << 32) * ((1 << shift) - d)) // d + 1, shift


def test_fast_division_by_invariant_matches_integer_division():
    """tile_coord divides tile ids by the tiles per image and per row with
    fast_div: q = (umulhi(n, mul) + n) >> shift (csrc/gsb_common.cuh). Checked
    against exact division for every divisor a raster can produce up to 2^16,
    a spread of larger ones, and numerators at the ends of the int32 range and
    at every multiple boundary."""
    import numpy as np

    rng = np.random.default_rng(0)
    divisors = list(range(1, 1 << 16, 37)) + [2 ** k for k in range(31)] + [2 ** k - 1 for k in range(2, 32)] + \
        [2 ** k + 1 for k in range(2, 31)] + [int(x) for x in rng.integers(1, 2 ** 31 - 1, 200)]
    for d in divisors:
        mul, shift = _fast_div_magic(d)
        assert 0 <= mul < 2 ** 32 and shift <= 31
        n = np.concatenate([rng.integers(0, 2 ** 31 - 1, 2000, dtype=np.int64), np.arange(0, 64),
                            np.array([2 ** 31 - 1, 2 ** 31 - 2]),
                            np.clip(np.arange(1, 40) * d + np.array([-1, 0, 1])[:, None], 0, 2 ** 31 - 1).ravel()])
        n = n.astype(np.uint64)
        hi = (n * np.uint64(mul)) >> np.uint64(32)
        s = hi + n
        assert int(s.max()) < 2 ** 32
        q = s >> np.uint64(shift)
        assert np.array_equal(q, n // np.uint64(d)), d
