"""Drop-in torch API of the B200 Gaussian-splat rasterizer.

Mirrors the public surface of nbardy/fast-mac-gsplat:
  torch_gsplat_bridge_fast/rasterize.py:15-184 (RasterConfig, rasterize_projected_gaussians,
      ProjectedGaussianRasterizer; [G,...] inputs)
  variants/v8_project3d/torch_gsplat_bridge_v8_project3d/rasterize.py:16-1105 ([B,G,...] inputs,
      RuntimeShaderConfig, project_pinhole_gaussians, rasterize_pinhole_gaussians,
      profile_projected_gaussians)
with the same argument meaning, defaults, exception types and messages (CUDA
replaces MPS). Every op runs the sm_100a kernels of libgsplat_b200.so through its
C ABI on the current CUDA stream; there is no CPU fallback.
"""
from __future__ import annotations

import functools
import os
import threading
from dataclasses import dataclass
from typing import Any, Dict, Optional, Tuple

import torch
from torch import Tensor

from . import _native as N


# ---------------------------------------------------------------------------
# Configuration
# ---------------------------------------------------------------------------
@dataclass(frozen=True)
class RuntimeShaderConfig:
    """Runtime kernel configuration (…/v8_project3d/…/rasterize.py:16-52). The B200
    kernels are compiled for 16x16 tiles; chunk_size/fast_cap are validated and
    reported for compatibility (the global sort has no per-tile capacity)."""

    tile_size: int
    threads: int
    chunk_size: int
    fast_cap: int
    simdgroups: int


def _env_int(name: str, default: int) -> int:
    raw = os.environ.get(name)
    if raw is None or raw == "":
        return int(default)
    return int(raw)


def get_runtime_shader_config() -> RuntimeShaderConfig:
    tile_size = _env_int("GSP_TILE_SIZE", 16)
    chunk_size = _env_int("GSP_CHUNK", 64)
    fast_cap = _env_int("GSP_FAST_CAP", 2048)
    if tile_size not in (8, 16, 32):
        raise ValueError(f"GSP_TILE_SIZE must be one of 8, 16, 32; got {tile_size}")
    threads = tile_size * tile_size
    if threads > 1024:
        raise ValueError(f"tile_size={tile_size} implies {threads} threads, which exceeds 1024")
    if chunk_size <= 0:
        raise ValueError("GSP_CHUNK must be positive")
    if fast_cap <= 0:
        raise ValueError("GSP_FAST_CAP must be positive")
    return RuntimeShaderConfig(tile_size=tile_size, threads=threads, chunk_size=chunk_size, fast_cap=fast_cap,
                               simdgroups=(threads + 31) // 32)


@dataclass(frozen=True)
class RasterConfig:
    """Superset of the reference configs (root rasterize.py:15-23; v8_project3d
    rasterize.py:55-67; v8 rasterize.py:65-82).

    Positional order follows the root API, whose package name this one keeps:
    the 4th field is the root's per-tile cap `max_tile_pairs` (default 4096), so
    `RasterConfig(h, w, 16, 4096)` works as it does there. The v8 name of the
    cap, `max_fast_pairs` (default 2048), is a keyword field at the end; as in
    v8 it is checked against the runtime fast cap (GSP_FAST_CAP). Fields 5 and
    on keep both versions' positions. The cap in force (`pair_cap`) is the
    smaller of the two. Tiles over the cap are rendered exactly (what the
    reference's overflow fallback produces, and what the root kernel would
    refuse); with `enable_overflow_fallback=False` the v8 error is raised
    instead. The v8 scheduling knobs (active tiles, stop-count mode, pair
    budgets) are accepted and have no effect: they tune Metal launch overhead
    and per-tile capacities that the B200 pipeline (one global sort, per-pixel
    stop state) does not have."""

    height: int
    width: int
    tile_size: int = 16
    max_tile_pairs: int = 4096
    alpha_threshold: float = 1.0 / 255.0
    transmittance_threshold: float = 1e-4
    background: Tuple[float, float, float] = (0.0, 0.0, 0.0)
    enable_overflow_fallback: bool = True
    batch_strategy: str = "auto"  # auto | flatten | serial
    batch_launch_limit_tiles: int = 262144
    batch_launch_limit_gaussians: int = 262144
    use_active_tiles: bool = False
    active_policy: str = "off"
    sort_active_tiles_by_count: bool = True
    stop_count_mode: str = "adaptive"
    stop_count_dense_threshold: int = 64
    max_pairs_per_launch: int = 0
    max_fast_pairs: int = 2048

    @property
    def pair_cap(self) -> int:
        return int(min(self.max_tile_pairs, self.max_fast_pairs))


_validated: Dict[Any, RuntimeShaderConfig] = {}


def _runtime_validate(config: RasterConfig) -> RuntimeShaderConfig:
    """Checks the config against the runtime shader config (read from the
    environment on every call, as the reference does); a (config, environment)
    pair that passed once is remembered."""
    env = (os.environ.get("GSP_TILE_SIZE"), os.environ.get("GSP_CHUNK"), os.environ.get("GSP_FAST_CAP"))
    try:
        hit = _validated.get((config, env))
    except TypeError:  # unhashable config field
        hit = None
    if hit is not None:
        return hit
    rt = _runtime_validate_uncached(config)
    try:
        if len(_validated) < 256:
            _validated[(config, env)] = rt
    except TypeError:
        pass
    return rt


def _runtime_validate_uncached(config: RasterConfig) -> RuntimeShaderConfig:
    rt = get_runtime_shader_config()
    if config.tile_size != rt.tile_size:
        raise ValueError(
            f"RasterConfig.tile_size={config.tile_size} does not match runtime shader tile size {rt.tile_size}. "
            "Set GSP_TILE_SIZE before importing/running the extension, or adjust RasterConfig."
        )
    if config.tile_size != 16:
        raise ValueError("The B200 kernels are specialized for 16x16 tiles.")
    if config.max_fast_pairs > rt.fast_cap:
        raise ValueError(
            f"RasterConfig.max_fast_pairs={config.max_fast_pairs} exceeds compiled fast cap {rt.fast_cap}. "
            "Lower the runtime cap or set GSP_FAST_CAP before import."
        )
    if config.batch_strategy not in ("auto", "flatten", "serial"):
        raise ValueError("batch_strategy must be one of: auto, flatten, serial")
    # The v8 policy knobs have no effect here, but invalid values are refused
    # with v8's messages (variants/v8/torch_gsplat_bridge_v8/rasterize.py:97-106).
    if config.active_policy not in ("off", "on", "auto"):
        raise ValueError("active_policy must be one of: off, on, auto")
    if config.stop_count_mode not in ("always", "never", "adaptive"):
        raise ValueError("stop_count_mode must be one of: always, never, adaptive")
    if config.stop_count_dense_threshold <= 0:
        raise ValueError("stop_count_dense_threshold must be positive")
    if config.max_pairs_per_launch < 0:
        raise ValueError("max_pairs_per_launch must be non-negative")
    if config.height <= 0 or config.width <= 0:
        raise ValueError("height and width must be positive")
    return rt


# ---------------------------------------------------------------------------
# Input checks (…/v8_project3d/…/rasterize.py:128-240)
# ---------------------------------------------------------------------------
def _normalize_inputs(means2d, conics, colors, opacities, depths):
    if means2d.ndim == 2:
        return (means2d.unsqueeze(0), conics.unsqueeze(0), colors.unsqueeze(0), opacities.unsqueeze(0),
                depths.unsqueeze(0), False)
    if means2d.ndim != 3:
        raise ValueError("means2d must have shape [G,2] or [B,G,2]")
    return means2d, conics, colors, opacities, depths, True


def _check_inputs(means2d: Tensor, conics: Tensor, colors: Tensor, opacities: Tensor, depths: Tensor) -> None:
    tensors = {"means2d": means2d, "conics": conics, "colors": colors, "opacities": opacities, "depths": depths}
    if len({t.device for t in tensors.values()}) != 1:
        raise ValueError("means2d/conics/colors/opacities/depths must be on the same device")
    if means2d.device.type != "cuda":
        raise ValueError("B200 rasterizer inputs must be on CUDA")
    for name, t in tensors.items():
        if t.dtype != torch.float32:
            raise ValueError(f"{name} must be float32")
    if means2d.ndim not in (2, 3):
        raise ValueError("means2d must have shape [G,2] or [B,G,2]")
    if conics.ndim != means2d.ndim or colors.ndim != means2d.ndim:
        raise ValueError("conics/colors rank must match means2d rank")
    if opacities.ndim != means2d.ndim - 1 or depths.ndim != means2d.ndim - 1:
        raise ValueError("opacities/depths rank must be one less than means2d rank")
    if means2d.shape[-1] != 2:
        raise ValueError("means2d must have last dim = 2")
    if conics.shape[-1] != 3:
        raise ValueError("conics must have last dim = 3")
    if colors.shape[-1] != 3:
        raise ValueError("colors must have last dim = 3")
    if means2d.shape[:-1] != conics.shape[:-1] or means2d.shape[:-1] != colors.shape[:-1]:
        raise ValueError("means2d/conics/colors batch/G dimensions must match")
    if means2d.shape[:-1] != opacities.shape or means2d.shape[:-1] != depths.shape:
        raise ValueError("means2d/opacities/depths batch/G dimensions must match")


def _normalize_3d_inputs(means3d, scales, quats, opacities):
    if opacities.ndim >= 1 and opacities.shape[-1:] == (1,):
        opacities = opacities.squeeze(-1)
    if means3d.ndim == 2:
        return means3d.unsqueeze(0), scales.unsqueeze(0), quats.unsqueeze(0), opacities.unsqueeze(0), False
    if means3d.ndim != 3:
        raise ValueError("means3d must have shape [G,3] or [B,G,3]")
    return means3d, scales, quats, opacities, True


def _normalize_colors(colors: Tensor, batch_size: int, gaussians: int, was_batched: bool) -> Tensor:
    if colors.ndim == 2:
        colors_b = colors.unsqueeze(0)
    elif colors.ndim == 3:
        colors_b = colors
    else:
        raise ValueError("colors must have shape [G,3] or [B,G,3]")
    if colors_b.shape != (batch_size, gaussians, 3):
        expected = "[B,G,3]" if was_batched else "[G,3]"
        raise ValueError(f"colors must match Gaussian shape {expected}; got {tuple(colors.shape)}")
    return colors_b


def _check_3d_inputs(means3d: Tensor, scales: Tensor, quats: Tensor, opacities: Tensor) -> None:
    tensors = {"means3d": means3d, "scales": scales, "quats": quats, "opacities": opacities}
    if len({t.device for t in tensors.values()}) != 1:
        raise ValueError("means3d/scales/quats/opacities must be on the same device")
    if means3d.device.type != "cuda":
        raise ValueError("B200 projection inputs must be on CUDA")
    for name, t in tensors.items():
        if t.dtype != torch.float32:
            raise ValueError(f"{name} must be float32")
    if means3d.ndim not in (2, 3) or means3d.shape[-1] != 3:
        raise ValueError("means3d must have shape [G,3] or [B,G,3]")
    if scales.shape != means3d.shape:
        raise ValueError("scales must match means3d shape")
    if quats.shape[:-1] != means3d.shape[:-1] or quats.shape[-1] != 4:
        raise ValueError("quats must have shape [G,4] or [B,G,4]")
    op_shape = opacities.shape[:-1] if opacities.ndim >= 1 and opacities.shape[-1:] == (1,) else opacities.shape
    if op_shape != means3d.shape[:-1]:
        raise ValueError("opacities must have shape [G], [G,1], [B,G], or [B,G,1]")


# ---------------------------------------------------------------------------
# Native pipeline helpers
# ---------------------------------------------------------------------------
_tls = threading.local()
_host_mod = None


def _host():
    """The native host runtime (_gsb_host, built in-tree next to libgsplat_b200.so).
    Loading it registers the torch.ops.gsplat_b200 op namespace."""
    global _host_mod
    if _host_mod is None:
        try:
            from . import _gsb_host as mod
        except ImportError as e:
            raise RuntimeError(
                "gsplat_b200 native host module _gsb_host is missing or does not load. Build it first "
                "(python fast-mac-gsplat_b200/build_native.py or __graft_entry__.build())."
            ) from e
        _host_mod = mod
    return _host_mod


_ops_ns = None


def _ops():
    """torch.ops.gsplat_b200: rasterize_fwd, bin, render_fwd_eval,
    render_fwd_train, render_bwd, project_fwd, project_bwd, sh_fwd, sh_bwd
    (CUDA dispatch key only)."""
    global _ops_ns
    if _ops_ns is None:
        _host()
        _ops_ns = torch.ops.gsplat_b200
    return _ops_ns


def set_kernel_timer(enabled: bool) -> None:
    """Turns per-phase CUDA-event timing of the autograd path on or off (phases:
    bin_prepare, bin_emit, render_fwd, render_bwd, unsort; events on the
    launching stream). Read the times with kernel_times()."""
    _host().set_phase_timing(bool(enabled))


def kernel_times() -> Dict[str, list]:
    """Milliseconds of each timed phase since set_kernel_timer(True), in call
    order per phase name (synchronizes); clears the record."""
    return dict(_host().take_phase_times())


def _debug_checks() -> bool:
    return os.environ.get("GSPLAT_B200_CHECK", "0") not in ("", "0")


def _pinned(name: str, n: int, dtype) -> Tensor:
    buf = getattr(_tls, name, None)
    if buf is None or buf.numel() < n:
        buf = torch.empty(n, dtype=dtype, pin_memory=True)
        setattr(_tls, name, buf)
    return buf


def _read_status(status: Tensor) -> list:
    """Synchronous read of a status block (used by the optional debug checks
    and the overflow check); raises on a device error flag."""
    host = _pinned("status_host", N.GSB_STATUS_WORDS, torch.int32)
    host.copy_(status, non_blocking=True)
    torch.cuda.current_stream(status.device).synchronize()
    vals = [int(v) & 0xFFFFFFFF for v in host.tolist()]
    if vals[N.GSB_STATUS_ERROR]:
        raise RuntimeError(N.decode_device_error(vals[N.GSB_STATUS_ERROR], vals[N.GSB_STATUS_ERROR_SITE]))
    return vals


class _ErrorSlots:
    """A small ring of pinned status copies and events for deferred device-error
    reads (one per forward or backward call). It is shared by all threads, so an
    error raised by a backward that autograd ran on its own device thread is
    reported to the thread that calls the next forward."""

    def __init__(self, n: int = 16):
        self.host = torch.empty((n, N.GSB_STATUS_WORDS), dtype=torch.int32, pin_memory=True)
        self.rows = [self.host[i] for i in range(n)]
        self.view = self.host.numpy()
        self.events = [torch.cuda.Event() for _ in range(n)]
        self.streams = [None] * n
        self.next = 0

    def check(self, i: int, synced_stream=None) -> None:
        stream = self.streams[i]
        if stream is None:
            return
        self.streams[i] = None
        if stream != synced_stream:
            self.events[i].synchronize()
        flags = int(self.view[i, N.GSB_STATUS_ERROR]) & 0xFFFFFFFF
        if flags:
            site = int(self.view[i, N.GSB_STATUS_ERROR_SITE]) & 0xFFFFFFFF
            raise RuntimeError(N.decode_device_error(flags, site))


_error_lock = threading.Lock()
_error_ring: Optional[_ErrorSlots] = None


def _defer_error_check(status: Tensor, stream) -> None:
    """Copies a call's status block to pinned memory without waiting; the next
    forward's host sync (or check_device_errors()) reads and raises its errors."""
    global _error_ring
    with _error_lock:
        if _error_ring is None:
            _error_ring = _ErrorSlots()
        slots = _error_ring
        i = slots.next
        slots.next = (i + 1) % len(slots.rows)
        slots.check(i)  # the slot's previous copy is long done by now
        slots.rows[i].copy_(status, non_blocking=True)
        slots.events[i].record(stream)
        slots.streams[i] = stream.cuda_stream


def check_device_errors(_synced_stream=None) -> None:
    """Raises RuntimeError if any earlier call's kernels reported a device-side
    error (bounded-wait timeout, pair overflow, index out of bounds)."""
    if _synced_stream is None and _host_mod is not None:
        _host_mod.check_device_errors()
    with _error_lock:
        slots = _error_ring
        if slots is None:
            return
        n = len(slots.rows)
        for k in range(n):
            slots.check((slots.next + k) % n, _synced_stream)


def _aligned(t: Tensor, align: int = 16) -> Tensor:
    t = t.contiguous()
    if t.data_ptr() % align:
        t = t.clone()
    return t


def _make_meta(config: RasterConfig, B: int, G: int) -> N.GsbRasterMeta:
    return N.make_meta(config.height, config.width, B, G, config.alpha_threshold, config.transmittance_threshold,
                       config.background)


_meta_cached = functools.lru_cache(maxsize=64)(_make_meta)


def _meta_for(config: RasterConfig, B: int, G: int) -> N.GsbRasterMeta:
    """Packed C meta; the library only reads it, so one instance per (config, B, G)
    is shared across calls."""
    try:
        return _meta_cached(config, B, G)
    except TypeError:  # a config holding an unhashable value (e.g. a list background)
        return _make_meta(config, B, G)


class _BinState:
    __slots__ = ("meta", "perm", "rec", "pair_offsets", "P", "keys", "binned_ids", "tile_offsets", "status")


def _bin(config: RasterConfig, means2d_b: Tensor, conics_b: Tensor, colors_b: Tensor, opacities_b: Tensor,
         depths_b: Tensor) -> _BinState:
    """Depth sort, exact tile counts, scan, emit, stable tile sort, tile ranges
    (replaces metal_bin, variants/v8_project3d/csrc/metal/gsplat_metal.mm:317-379)."""
    L = N.load()
    B, G = means2d_b.shape[:2]
    dev = means2d_b.device
    meta = _meta_for(config, B, G)
    BG = B * G
    st = _BinState()
    st.meta = meta
    ws_bytes = int(L.gsb_bin_prepare_workspace_size(meta))
    st.status = torch.empty(N.GSB_STATUS_WORDS, dtype=torch.int32, device=dev)  # cleared by gsb_bin_count
    st.perm = torch.empty((B, G), dtype=torch.int32, device=dev)
    st.rec = torch.empty((BG, N.GSB_REC_FLOATS), dtype=torch.float32, device=dev)
    st.pair_offsets = torch.empty(BG + 1, dtype=torch.int32, device=dev)
    tile_masks = torch.empty((int(L.gsb_bin_tile_masks_size(meta)) + 7) // 8, dtype=torch.int64, device=dev)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
    cur = torch.cuda.current_stream(dev)
    stream = cur.cuda_stream
    # Locals keep every (possibly copied) input alive until the launch returns.
    m2 = _aligned(means2d_b, 8)
    q2, c2, o2, d2 = (t.contiguous() for t in (conics_b, colors_b, opacities_b, depths_b))
    N.check(L.gsb_bin_count(meta, N.ptr(m2), N.ptr(q2), N.ptr(o2), N.ptr(d2), N.ptr(tile_masks), N.ptr(st.status),
                            N.ptr(ws), ws_bytes, stream), "gsb_bin_count")
    # The pair total is read as soon as the count kernel is done, while the depth
    # sort and scan run: the host wait overlaps GPU work.
    total_host = _pinned("total_host", 1, torch.int64)
    total_host.copy_(st.status[N.GSB_STATUS_PAIR_TOTAL64:N.GSB_STATUS_PAIR_TOTAL64 + 2].view(torch.int64),
                     non_blocking=True)
    counted = getattr(_tls, "counted_event", None)
    if counted is None:
        counted = _tls.counted_event = torch.cuda.Event()
    counted.record(cur)
    N.check(L.gsb_bin_sort_scan(meta, N.ptr(m2), N.ptr(q2), N.ptr(c2), N.ptr(o2), N.ptr(d2), N.ptr(st.perm),
                                N.ptr(st.rec), N.ptr(st.pair_offsets), N.ptr(tile_masks), N.ptr(st.status),
                                N.ptr(ws), ws_bytes, stream), "gsb_bin_sort_scan")
    counted.synchronize()
    check_device_errors(stream)  # earlier calls' copies on this stream are complete now
    P = int(total_host[0])
    if P >= 2**31 - 1:
        raise RuntimeError(f"gsplat_b200: {P} tile-splat pairs exceed the supported 2^31 - 1")
    st.P = P
    T = B * ((config.height + 15) // 16) * ((config.width + 15) // 16)
    ws2_bytes = int(L.gsb_bin_emit_workspace_size(meta, P))
    st.binned_ids = torch.empty(P, dtype=torch.int32, device=dev)
    st.tile_offsets = torch.empty(T + 1, dtype=torch.int32, device=dev)
    st.keys = torch.empty(P, dtype=torch.int64, device=dev)
    ws2 = torch.empty(max(ws2_bytes, 1), dtype=torch.uint8, device=dev)
    N.check(L.gsb_bin_emit(meta, N.ptr(st.rec), N.ptr(st.pair_offsets), N.ptr(tile_masks), P, N.ptr(st.keys),
                           N.ptr(st.binned_ids),
                           N.ptr(st.tile_offsets), N.ptr(st.status), N.ptr(ws2), ws2_bytes, stream), "gsb_bin_emit")
    if _debug_checks():
        _read_status(st.status)
    return st


def _render_forward(st: _BinState, config: RasterConfig, B: int, save_state: bool):
    L = N.load()
    dev = st.status.device
    H, W = config.height, config.width
    out = torch.empty((B, H, W, 3), dtype=torch.float32, device=dev)
    final_T = last_idx = pair_rec = None
    ws_bytes = int(L.gsb_render_workspace_size(st.meta))
    if save_state:
        final_T = torch.empty((B, H, W), dtype=torch.float32, device=dev)
        last_idx = torch.empty((B, H, W), dtype=torch.int32, device=dev)
        pair_rec = torch.empty((max(st.P, 1), N.GSB_REC_FLOATS), dtype=torch.float32, device=dev)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
    cur = torch.cuda.current_stream(dev)
    N.check(L.gsb_render_forward(st.meta, N.ptr(st.rec), N.ptr(st.tile_offsets), N.ptr(st.binned_ids), N.ptr(out),
                                 N.ptr(final_T), N.ptr(last_idx), N.ptr(pair_rec), N.ptr(st.status), N.ptr(ws),
                                 ws_bytes, cur.cuda_stream), "gsb_render_forward")
    if _debug_checks():
        _read_status(st.status)
    else:
        _defer_error_check(st.status, cur)
    return out, final_T, last_idx, pair_rec


# eps and max_alpha are fixed in the reference's meta (root rasterize.py:135-136).
_EPS = 1e-8
_MAX_ALPHA = 0.99


def _host_args(config: RasterConfig):
    """The scalar raster arguments of the torch.ops.gsplat_b200 schemas:
    height, width, alpha_threshold, transmittance_threshold, bg_r, bg_g, bg_b,
    eps, max_alpha."""
    bg = [float(c) for c in config.background]
    return (config.height, config.width, float(config.alpha_threshold), float(config.transmittance_threshold), *bg,
            _EPS, _MAX_ALPHA)


class _RasterizeProjectedGaussiansB200(torch.autograd.Function):
    """Training path (…/v8_project3d/…/rasterize.py:691-852; root rasterize.py:26-106).
    Saves the per-pixel final transmittance and last-contributor index instead of
    per-tile stop counts; backward un-sorts into input order; depth grad is zero.
    Each direction is one torch op (gsplat_b200::rasterize_fwd / render_bwd)."""

    @staticmethod
    def forward(ctx, means2d_b, conics_b, colors_b, opacities_b, depths_b, config: RasterConfig):
        cap = -1 if config.enable_overflow_fallback else config.pair_cap
        args = _host_args(config)
        res = _ops().rasterize_fwd(means2d_b, conics_b, colors_b, opacities_b, depths_b, *args, True, cap)
        out, perm, rec, tile_offsets, binned_ids, final_T, last_idx, pair_rec, status = res
        ctx.save_for_backward(perm, rec, tile_offsets, binned_ids, final_T, last_idx, pair_rec, status)
        ctx.host_args = args
        ctx.depths_shape = depths_b.shape
        return out

    @staticmethod
    def backward(ctx, grad_out: Tensor):
        need = ctx.needs_input_grad
        g_means, g_conics, g_colors, g_opac = _ops().render_bwd(*ctx.saved_tensors, grad_out, *ctx.host_args,
                                                                [bool(x) for x in need[:4]])
        dev = grad_out.device
        g_depths = torch.zeros(ctx.depths_shape, dtype=torch.float32, device=dev) if need[4] else None
        return g_means, g_conics, g_colors, g_opac, g_depths, None


def _rasterize_chunk_eval(means2d_b, conics_b, colors_b, opacities_b, depths_b, config: RasterConfig) -> Tensor:
    """No-grad path (…/v8_project3d/…/rasterize.py:855-907): no saved state."""
    cap = -1 if config.enable_overflow_fallback else config.pair_cap
    return _ops().rasterize_fwd(means2d_b, conics_b, colors_b, opacities_b, depths_b, *_host_args(config), False,
                                cap)[0]


def _should_use_training_path(means2d: Tensor, conics: Tensor, colors: Tensor, opacities: Tensor) -> bool:
    if not torch.is_grad_enabled():
        return False
    return bool(means2d.requires_grad or conics.requires_grad or colors.requires_grad or opacities.requires_grad)


def _choose_batch_chunk_size(config: RasterConfig, batch_size: int, gaussians_per_batch: int,
                             tiles_per_image: int) -> int:
    """Same chunking policy as …/v8_project3d/…/rasterize.py:681-688 (outputs do not
    depend on it; it bounds per-launch memory)."""
    if config.batch_strategy == "flatten":
        return batch_size
    if config.batch_strategy == "serial":
        return 1
    by_tiles = max(1, config.batch_launch_limit_tiles // max(tiles_per_image, 1))
    by_gaussians = max(1, config.batch_launch_limit_gaussians // max(gaussians_per_batch, 1))
    return max(1, min(batch_size, by_tiles, by_gaussians))


def _rasterize_batched(means2d_b, conics_b, colors_b, opacities_b, depths_b, config: RasterConfig) -> Tensor:
    B, G = means2d_b.shape[:2]
    tiles_y = (config.height + config.tile_size - 1) // config.tile_size
    tiles_x = (config.width + config.tile_size - 1) // config.tile_size
    chunk_b = _choose_batch_chunk_size(config, B, G, tiles_y * tiles_x)
    train_mode = _should_use_training_path(means2d_b, conics_b, colors_b, opacities_b)
    outs = []
    for b0 in range(0, B, chunk_b):
        b1 = min(B, b0 + chunk_b)
        full = (means2d_b, conics_b, colors_b, opacities_b, depths_b)
        # A single chunk passes the inputs themselves: a slice would make autograd
        # allocate and copy a full-size gradient per input.
        args = [t if chunk_b >= B else t[b0:b1] for t in full]
        if train_mode:
            outs.append(_RasterizeProjectedGaussiansB200.apply(*args, config))
        else:
            with torch.no_grad():
                outs.append(_rasterize_chunk_eval(*args, config))
    return torch.cat(outs, dim=0) if len(outs) > 1 else outs[0]


def rasterize_projected_gaussians(means2d: Tensor, conics: Tensor, colors: Tensor, opacities: Tensor,
                                  depths: Tensor, config: RasterConfig) -> Tensor:
    """[G,...] -> [H,W,3] or [B,G,...] -> [B,H,W,3] (root rasterize.py:144-175;
    …/v8_project3d/…/rasterize.py:941-955)."""
    _check_inputs(means2d, conics, colors, opacities, depths)
    means2d_b, conics_b, colors_b, opacities_b, depths_b, was_batched = _normalize_inputs(
        means2d, conics, colors, opacities, depths)
    _runtime_validate(config)
    out = _rasterize_batched(means2d_b, conics_b, colors_b, opacities_b, depths_b, config)
    return out if was_batched else out.squeeze(0)


# ---------------------------------------------------------------------------
# Pinhole projection (…/v8_project3d/…/rasterize.py:243-572, 958-1003)
# ---------------------------------------------------------------------------
def _camera_scalar_batch(value, batch_size: int, device: torch.device, dtype: torch.dtype, name: str) -> Tensor:
    if torch.is_tensor(value):
        value = value.to(device=device, dtype=dtype)
        if value.ndim == 0:
            return value.expand(batch_size)
        if value.numel() == batch_size:
            return value.reshape(batch_size)
        raise ValueError(f"{name} must be scalar or have {batch_size} values")
    return torch.full((batch_size,), float(value), device=device, dtype=dtype)


def _camera_to_world_batch(camera_to_world, batch_size: int, device: torch.device, dtype: torch.dtype) -> Tensor:
    if camera_to_world is None:
        return torch.eye(4, device=device, dtype=dtype).unsqueeze(0).expand(batch_size, -1, -1).contiguous()
    camera_to_world = camera_to_world.to(device=device, dtype=dtype)
    if camera_to_world.shape == (4, 4):
        return camera_to_world.unsqueeze(0).expand(batch_size, -1, -1).contiguous()
    if camera_to_world.shape == (batch_size, 4, 4):
        return camera_to_world.contiguous()
    raise ValueError(f"camera_to_world must be [4,4] or [{batch_size},4,4]")


def _projection_backward_requested(*values) -> bool:
    if not torch.is_grad_enabled():
        return False
    return any(torch.is_tensor(v) and v.requires_grad for v in values)


def _project_forward_native(means3d_b, scales_b, quats_b, opacities_b, c2w_b, camera_params, near_plane):
    return tuple(_ops().project_fwd(means3d_b, scales_b, quats_b, opacities_b, c2w_b, camera_params,
                                    float(near_plane)))


class _ProjectPinholeGaussiansB200(torch.autograd.Function):
    """…/v8_project3d/…/rasterize.py:371-481."""

    @staticmethod
    def forward(ctx, means3d_b, scales_b, quats_b, opacities_b, c2w_b, camera_params, near_plane: float):
        outs = _project_forward_native(means3d_b, scales_b, quats_b, opacities_b, c2w_b, camera_params, near_plane)
        ctx.save_for_backward(means3d_b, scales_b, quats_b, opacities_b, c2w_b, camera_params)
        ctx.near_plane = float(near_plane)
        return outs

    @staticmethod
    def backward(ctx, g_m2d, g_con, g_op, g_depth):
        means3d_b, scales_b, quats_b, opacities_b, c2w_b, camera_params = ctx.saved_tensors
        if not any(ctx.needs_input_grad[:6]):
            return (None,) * 7
        grads = list(_ops().project_bwd(g_m2d, g_con, g_op, g_depth, means3d_b, scales_b, quats_b, opacities_b,
                                        c2w_b, camera_params, ctx.near_plane))
        for i, need in enumerate(ctx.needs_input_grad[:6]):
            if not need:
                grads[i] = None
        return (*grads, None)


def _project_pinhole_gaussians_batched(means3d_b, scales_b, quats_b, opacities_b, fx, fy, cx, cy, camera_to_world,
                                       near_plane: float):
    B = means3d_b.shape[0]
    dev, dt = means3d_b.device, means3d_b.dtype
    camera_params = torch.stack(
        [_camera_scalar_batch(v, B, dev, dt, n) for v, n in ((fx, "fx"), (fy, "fy"), (cx, "cx"), (cy, "cy"))], dim=1
    ).contiguous()
    c2w_b = _camera_to_world_batch(camera_to_world, B, dev, dt)
    if _projection_backward_requested(means3d_b, scales_b, quats_b, opacities_b, c2w_b, camera_params):
        return _ProjectPinholeGaussiansB200.apply(means3d_b, scales_b, quats_b, opacities_b, c2w_b, camera_params,
                                                  float(near_plane))
    with torch.no_grad():
        return _project_forward_native(means3d_b, scales_b, quats_b, opacities_b, c2w_b, camera_params, near_plane)


def project_pinhole_gaussians(means3d: Tensor, scales: Tensor, quats: Tensor, opacities: Tensor, fx, fy, cx, cy,
                              camera_to_world=None, near_plane: float = 1e-4):
    """-> (means2d, conics, projected_opacities, depths) (…/rasterize.py:544-572)."""
    _check_3d_inputs(means3d, scales, quats, opacities)
    m, s, q, o, was_batched = _normalize_3d_inputs(means3d, scales, quats, opacities)
    out = _project_pinhole_gaussians_batched(m.contiguous(), s.contiguous(), q.contiguous(), o.contiguous(), fx, fy,
                                             cx, cy, camera_to_world, near_plane)
    if was_batched:
        return out
    return tuple(t[0] for t in out)


def rasterize_pinhole_gaussians(means3d: Tensor, scales: Tensor, quats: Tensor, opacities: Tensor, colors: Tensor,
                                fx, fy, cx, cy, camera_to_world=None, near_plane: float = 1e-4,
                                config: RasterConfig | None = None) -> Tensor:
    """Project then rasterize (…/rasterize.py:958-1003)."""
    if config is None:
        raise ValueError("config is required")
    _check_3d_inputs(means3d, scales, quats, opacities)
    m, s, q, o, was_batched = _normalize_3d_inputs(means3d, scales, quats, opacities)
    B, G = m.shape[:2]
    colors_b = _normalize_colors(colors, B, G, was_batched)
    if colors_b.device != m.device:
        raise ValueError("colors must be on the same device as means3d")
    if colors_b.dtype != torch.float32:
        raise ValueError("colors must be float32")
    means2d, conics, proj_op, depths = _project_pinhole_gaussians_batched(
        m.contiguous(), s.contiguous(), q.contiguous(), o.contiguous(), fx, fy, cx, cy, camera_to_world, near_plane)
    _runtime_validate(config)
    out = _rasterize_batched(means2d.contiguous(), conics.contiguous(), colors_b.contiguous(), proj_op.contiguous(),
                             depths.contiguous(), config)
    return out if was_batched else out.squeeze(0)


# ---------------------------------------------------------------------------
# Profiling (…/v8_project3d/…/rasterize.py:1006-1096)
# ---------------------------------------------------------------------------
def _tile_stop_counts(last_idx: Tensor, counts: Tensor, config: RasterConfig) -> Tensor:
    """The reference's per-tile stop count (…kernels.metal:875-923) from the
    per-pixel state: the max over the tile's in-image pixels of last_idx (the
    entries a pixel walked: the saturating index + 1, or the tile's count), and
    0 for an empty tile or one above the pair cap, which the reference's fast
    kernel leaves to its overflow path (:876-884)."""
    B, H, W = last_idx.shape
    ty, tx = (H + 15) // 16, (W + 15) // 16
    cnt = counts.view(B, ty, tx).to(torch.int64)
    pad = torch.zeros((B, ty * 16, tx * 16), dtype=torch.int64, device=last_idx.device)
    pad[:, :H, :W] = last_idx.to(torch.int64)
    stop = pad.view(B, ty, 16, tx, 16).amax(dim=(2, 4))
    stop = torch.where((cnt > 0) & (cnt <= int(config.pair_cap)), stop, torch.zeros_like(stop))
    return stop.reshape(-1)


@torch.no_grad()
def profile_projected_gaussians(means2d: Tensor, conics: Tensor, colors: Tensor, opacities: Tensor, depths: Tensor,
                                config: RasterConfig, *, run_forward: bool = False,
                                return_image: bool = False) -> Dict[str, Any]:
    _check_inputs(means2d, conics, colors, opacities, depths)
    means2d_b, conics_b, colors_b, opacities_b, depths_b, was_batched = _normalize_inputs(
        means2d, conics, colors, opacities, depths)
    B, G = means2d_b.shape[:2]
    _runtime_validate(config)
    tiles_y = (config.height + config.tile_size - 1) // config.tile_size
    tiles_x = (config.width + config.tile_size - 1) // config.tile_size
    chunk_b = _choose_batch_chunk_size(config, B, G, tiles_y * tiles_x)
    all_counts, all_stops, images = [], [], []
    for b0 in range(0, B, chunk_b):
        b1 = min(B, b0 + chunk_b)
        args = [t[b0:b1].contiguous() for t in (means2d_b, conics_b, colors_b, opacities_b, depths_b)]
        st = _bin(config, *args)
        counts = (st.tile_offsets[1:] - st.tile_offsets[:-1])
        all_counts.append(counts.cpu().to(torch.float32))
        if run_forward or return_image:
            out, final_T, last_idx, _ = _render_forward(st, config, b1 - b0, save_state=True)
            if return_image:
                images.append(out)
            all_stops.append(_tile_stop_counts(last_idx, counts, config).cpu().to(torch.float32))
    counts_cpu = torch.cat(all_counts) if all_counts else torch.zeros(0)
    stats: Dict[str, Any] = {
        "batch_size": int(B),
        "gaussians_per_batch": int(G),
        "height": int(config.height),
        "width": int(config.width),
        "tile_size": int(config.tile_size),
        "tiles": int(counts_cpu.numel()),
        "total_pairs": int(counts_cpu.sum().item()) if counts_cpu.numel() else 0,
        "mean_pairs_per_tile": float(counts_cpu.mean().item()) if counts_cpu.numel() else 0.0,
        "p95_pairs_per_tile": float(torch.quantile(counts_cpu, 0.95).item()) if counts_cpu.numel() else 0.0,
        "max_pairs_per_tile": int(counts_cpu.max().item()) if counts_cpu.numel() else 0,
        "overflow_tile_count": int((counts_cpu > int(config.pair_cap)).sum().item()) if counts_cpu.numel() else 0,
        "chosen_batch_chunk": int(chunk_b),
    }
    if all_stops:
        stop_cpu = torch.cat(all_stops)
        denom = torch.clamp(counts_cpu, min=1.0)
        ratio = torch.where(counts_cpu > 0, stop_cpu / denom, torch.zeros_like(stop_cpu))
        stats.update({
            "mean_stop_count": float(stop_cpu.mean().item()),
            "p95_stop_count": float(torch.quantile(stop_cpu, 0.95).item()),
            "max_stop_count": int(stop_cpu.max().item()),
            "mean_stop_ratio": float(ratio.mean().item()),
            "p95_stop_ratio": float(torch.quantile(ratio, 0.95).item()),
        })
    if return_image:
        out = torch.cat(images, dim=0) if len(images) > 1 else images[0]
        return {"image": out if was_batched else out[0], "stats": stats}
    return stats


class ProjectedGaussianRasterizer(torch.nn.Module):
    def __init__(self, config: RasterConfig):
        super().__init__()
        self.config = config

    def forward(self, means2d: Tensor, conics: Tensor, colors: Tensor, opacities: Tensor, depths: Tensor) -> Tensor:
        return rasterize_projected_gaussians(means2d, conics, colors, opacities, depths, self.config)
