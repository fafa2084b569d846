"""ctypes binding of the sm_100a C ABI (include/gsplat_b200.h) in libgsplat_b200.so.

This replaces the reference's TORCH_LIBRARY/MPS dispatch layer
(csrc/bindings.cpp:7-52, variants/v8_project3d/csrc/bindings.cpp:173-193). Calls pass
raw device pointers and the current torch CUDA stream; the library never
allocates. There is no CPU or MPS fallback: a missing library or a non-CUDA
tensor is an error.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libgsplat_b200.so"

GSB_STATUS_TOTAL_PAIRS = 0
GSB_STATUS_ERROR = 1
GSB_STATUS_MAX_TILE_COUNT = 2
GSB_STATUS_ERROR_SITE = 3
GSB_STATUS_PAIR_TOTAL64 = 4
GSB_STATUS_MASK_WORDS = 6
GSB_STATUS_TILE_CLAIM = 8
GSB_STATUS_WORDS = 16
GSB_REC_FLOATS = 12
GSB_PEER_MAX_RANKS = 8
GSB_PEER_FLAG_BYTES = 256
GSB_PEER_HANDLE_BYTES = 64
GSB_SORT_NOALLOC_MAX_PAIRS = 262144
GSB_SORT_NOALLOC_SCRATCH_BYTES = 6 << 20
GSB_DEVERR_PEER_TIMEOUT = 8

DEVERR_LOOKBACK_TIMEOUT = 1
DEVERR_PAIR_OVERFLOW = 2
DEVERR_BOUNDS = 4
DEVERR_PEER_TIMEOUT = GSB_DEVERR_PEER_TIMEOUT

# Every symbol include/gsplat_b200.h declares (checked by the ABI test).
EXPORTED = (
    "gsb_version",
    "gsb_status_string",
    "gsb_kernel_launches",
    "gsb_fma_probe_out_floats",
    "gsb_fma_probe",
    "gsb_bin_prepare_workspace_size",
    "gsb_bin_prepare",
    "gsb_bin_count",
    "gsb_bin_tile_masks_size",
    "gsb_bin_sort_scan",
    "gsb_bin_emit_workspace_size",
    "gsb_bin_emit",
    "gsb_bin_emit_ranges",
    "gsb_tile_stats",
    "gsb_render_workspace_size",
    "gsb_render_forward",
    "gsb_render_backward",
    "gsb_render_backward_inputs",
    "gsb_unsort_grads",
    "gsb_project_forward",
    "gsb_project_backward",
    "gsb_radix_sort_pairs_workspace_size",
    "gsb_radix_sort_pairs",
    "gsb_radix_sort_pairs_noalloc",
    "gsb_sh_forward",
    "gsb_sh_backward",
    "gsb_peer_buffer_alloc",
    "gsb_peer_buffer_free",
    "gsb_peer_handle",
    "gsb_peer_open",
    "gsb_peer_close",
    "gsb_peer_allreduce_sum",
)


class GsbRasterMeta(C.Structure):
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


class NativeError(RuntimeError):
    """A nonzero status from the C ABI."""


_lib = None


def load() -> C.CDLL:
    """Loads libgsplat_b200.so (built in-tree by build_native.py)."""
    global _lib
    if _lib is not None:
        return _lib
    path = Path(os.environ.get("GSPLAT_B200_LIB", str(LIB_PATH)))
    if not path.exists():
        raise RuntimeError(
            f"gsplat_b200 native library not found at {path}. Build it first "
            "(python fast-mac-gsplat_b200/build_native.py or __graft_entry__.build())."
        )
    L = C.CDLL(str(path))
    p, sz, i32, i64, f32 = C.c_void_p, C.c_size_t, C.c_int32, C.c_int64, C.c_float
    M = C.POINTER(GsbRasterMeta)
    sig = {
        "gsb_version": (C.c_int, []),
        "gsb_status_string": (C.c_char_p, [C.c_int]),
        "gsb_kernel_launches": (C.c_uint64, []),
        "gsb_fma_probe_out_floats": (i64, [i32]),
        "gsb_fma_probe": (C.c_int, [i32, i32, i32, p, p]),
        "gsb_bin_prepare_workspace_size": (sz, [M]),
        "gsb_bin_prepare": (C.c_int, [M, p, p, p, p, p, p, p, p, p, p, sz, p]),
        "gsb_bin_count": (C.c_int, [M, p, p, p, p, p, p, p, sz, p]),
        "gsb_bin_tile_masks_size": (sz, [M]),
        "gsb_bin_sort_scan": (C.c_int, [M, p, p, p, p, p, p, p, p, p, p, p, sz, p]),
        "gsb_bin_emit_workspace_size": (sz, [M, i64]),
        "gsb_bin_emit": (C.c_int, [M, p, p, p, i64, p, p, p, p, p, sz, p]),
        "gsb_bin_emit_ranges": (C.c_int, [M, p, p, p, i64, p, p, p, p, sz, p]),
        "gsb_tile_stats": (C.c_int, [M, p, p, p]),
        "gsb_render_workspace_size": (sz, [M]),
        "gsb_render_forward": (C.c_int, [M, p, p, p, p, p, p, p, p, p, sz, p]),
        "gsb_render_backward": (C.c_int, [M, p, p, p, p, p, p, p, p, p, p, sz, p]),
        "gsb_render_backward_inputs": (C.c_int, [M, p, p, p, p, p, p, p, p, p, p, p, p, p, p]),
        "gsb_unsort_grads": (C.c_int, [M, p, p, p, p, p, p, p]),
        "gsb_project_forward": (C.c_int, [i32, i32, p, p, p, p, p, p, f32, p, p, p, p, p]),
        "gsb_project_backward": (C.c_int, [i32, i32] + [p] * 10 + [f32] + [p] * 7),
        "gsb_radix_sort_pairs_workspace_size": (sz, [i64, C.c_int, C.c_int]),
        "gsb_radix_sort_pairs": (C.c_int, [p, p, p, p, i64, C.c_int, C.c_int, p, p, sz, p]),
        "gsb_radix_sort_pairs_noalloc": (C.c_int, [p, p, p, p, i64, C.c_int, C.c_int, p, p]),
        "gsb_sh_forward": (C.c_int, [i32, i32, i32, p, p, p, p, p]),
        "gsb_sh_backward": (C.c_int, [i32, i32, i32, p, p, p, p, p, p, p, p, p]),
        "gsb_peer_buffer_alloc": (C.c_int, [sz, C.POINTER(p)]),
        "gsb_peer_buffer_free": (C.c_int, [p]),
        "gsb_peer_handle": (C.c_int, [p, p]),
        "gsb_peer_open": (C.c_int, [p, C.POINTER(p)]),
        "gsb_peer_close": (C.c_int, [p]),
        "gsb_peer_allreduce_sum": (C.c_int, [i32, i32, C.POINTER(p), i64, C.c_uint32, C.c_uint64, p, p]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = load().gsb_status_string(rc).decode()
        raise NativeError(f"{what} failed with status {rc}: {msg}")


def ptr(t: torch.Tensor | None):
    """Device pointer of a tensor as an int (None -> NULL)."""
    return None if t is None else t.data_ptr()


def stream_ptr(device: torch.device):
    return torch.cuda.current_stream(device).cuda_stream


def make_meta(height: int, width: int, batch_size: int, gaussians_per_batch: int, alpha_threshold: float,
              transmittance_threshold: float, background, eps: float = 1e-8, max_alpha: float = 0.99,
              tile_size: int = 16) -> GsbRasterMeta:
    m = GsbRasterMeta()
    m.height, m.width, m.tile_size = int(height), int(width), int(tile_size)
    m.batch_size, m.gaussians_per_batch = int(batch_size), int(gaussians_per_batch)
    m.alpha_threshold = float(alpha_threshold)
    m.transmittance_threshold = float(transmittance_threshold)
    m.background = (C.c_float * 3)(*[float(x) for x in background])
    m.eps, m.max_alpha = float(eps), float(max_alpha)
    return m


def decode_device_error(flags: int, site: int) -> str:
    parts = []
    if flags & DEVERR_LOOKBACK_TIMEOUT:
        parts.append("decoupled look-back wait exceeded its spin limit")
    if flags & DEVERR_PAIR_OVERFLOW:
        parts.append("pair count overflow (emit/scan mismatch or > 2^31 pairs)")
    if flags & DEVERR_BOUNDS:
        parts.append("index out of bounds")
    if flags & DEVERR_PEER_TIMEOUT:
        parts.append("a peer rank did not reach the gradient-sum barrier in time")
    return f"gsplat_b200 device error (flags={flags}, site={site}): " + "; ".join(parts or ["unknown"])
