"""Benchmark of the B200 rasterizer hot path (one JSON line on rank 0).

Metric: fwd+bwd ms at 4096^2 x 64K splats and Gsplat-px evals/s.
A step is one training pass over one view of the headline config c3
(B=1, 4096x4096, G=65,536 uniform 2D splats): depth sort + binning + forward
compositing + backward with a N(0,1) grad_image, through the public API.
Work unit E = sum over tiles of valid_pixels x pairs(tile) (the reference's
tiled_scan_work). Multi-GPU: one process per GPU (torchrun), each rank renders its
own view (seed = rank), no data-path collective: weak scaling.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

--config c4 runs the shared-3D-scene step instead (G=2^20 Gaussians, one 1080p
camera per rank): projection, binning, compositing fwd+bwd, projection VJP, then
the per-Gaussian gradients summed across ranks with NCCL all-reduce.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (ROOT, ROOT / "fast-mac-gsplat_b200"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

import torch  # noqa: E402

METRIC = "Gsplat-px evals/s, fwd+bwd at 4096x4096 x 65,536 splats (ms_per_step = fwd+bwd ms)"
UNIT = "Gsplat-px evals/s"
CONFIG_NAME = "c3"
L2_FLUSH_BYTES = 256 << 20


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("b200", "reference"), default="b200")
    ap.add_argument("--config", default=CONFIG_NAME, choices=("c0", "c1", "c2", "c3", "c4"))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-splits", action="store_true",
                    help="skip the c2 (views split over ranks) and c4 (shared scene + gradient sum) lines")
    ap.add_argument("--trace", default="",
                    help="replay a recorded batch (torch.save'd dict of means2d/conics/colors/opacities/depths) "
                         "instead of the synthetic config; with --height/--width")
    ap.add_argument("--matrix", action="store_true",
                    help="one JSON line per BASELINE config c0-c4: forward-only and forward+backward ms")
    ap.add_argument("--height", type=int, default=4096)
    ap.add_argument("--width", type=int, default=4096)
    ap.add_argument("--allreduce", choices=("peer", "nccl"), default="peer",
                    help="c4 with several GPUs: gradient sum by the library's NVLink peer-memory kernel "
                         "(default) or by NCCL all-reduce (the baseline)")
    ap.add_argument("--sh-degree", type=int, default=-1,
                    help="c4 only: colours from spherical harmonics of this degree (0-3) instead of RGB")
    return ap.parse_args()


def dist_env():
    return int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("LOCAL_RANK", "0"))


def tiled_work(tile_offsets: torch.Tensor, B: int, H: int, W: int) -> int:
    """E = sum_t valid_px(t) * count(t) for a flat [B*tiles+1] offsets array."""
    off = tile_offsets.to("cpu", torch.int64)
    tx, ty = (W + 15) // 16, (H + 15) // 16
    counts = (off[1:] - off[:-1]).view(B, ty, tx)
    h = torch.full((ty,), 16, dtype=torch.int64)
    h[-1] = H - (ty - 1) * 16
    w = torch.full((tx,), 16, dtype=torch.int64)
    w[-1] = W - (tx - 1) * 16
    return int((counts * (h[:, None] * w[None, :])[None]).sum())


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def load_traffic(kernel: str, config: str):
    """Per-launch DRAM bytes from the committed ncu summary (profiles/traffic.txt,
    lines `kernel config bytes_per_launch`), or None."""
    p = ROOT / "profiles" / "traffic.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        parts = line.split()
        if len(parts) >= 3 and parts[0] == kernel and parts[1] == config and not line.startswith("#"):
            try:
                return float(parts[2])
            except ValueError:
                return None
    return None


class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"gsb_clocks_{os.getpid()}.csv"

    def __enter__(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.fh, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.fh.close()

    def summary(self):
        if self.proc is None or not self.path.exists():
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for line in self.path.read_text().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) >= 9:
                rows.append(f)
        self.path.unlink(missing_ok=True)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        smax = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": reasons, "samples": len(rows)}


# Algorithmic FP32 operations per Gsplat-px evaluation (an FMA counts 2): the
# forward's exponent, alpha, transmittance and colour update; the backward's
# recompute, transmittance inverse, colour/opacity/conic/mean VJPs and its share
# of the per-splat reduction (reference kernels …metal:574-592, 834-840, 1013-1039).
FLOPS_PER_EVAL = {"render_fwd": 23, "render_bwd": 60}


def algorithmic_bytes(kernel: str, B: int, H: int, W: int, G: int, P: int) -> int:
    """Bytes one launch must move at minimum (reads + writes)."""
    px = B * H * W
    tiles = B * ((H + 15) // 16) * ((W + 15) // 16)
    rec = 36 * B * G  # 9 floats of splat params
    if kernel == "render_fwd":  # rgb + final_T + last_idx out, ids + ranges + params in
        return px * (12 + 4 + 4) + P * 4 + tiles * 8 + rec
    if kernel == "render_bwd":  # grad rgb + state in, ids + ranges + params in, 9 grads out
        return px * (12 + 4 + 4) + P * 4 + tiles * 8 + rec + 36 * B * G
    if kernel == "bin_emit":  # params in, pairs out, sort read+write per pass (2 passes), ranges
        return rec + P * 12 * (1 + 2 * 2) + tiles * 4
    if kernel == "bin_prepare":  # params+depth in, keys, sort passes, records out, offsets
        return B * G * (40 + 12 * (1 + 2 * 4) + 48 + 4)
    if kernel == "unsort":
        return B * G * (48 + 36 + 4)
    return 0


def fp32_probe(dev, reps: int = 5):
    """Measured FP32 peak (TFLOP/s): the library's FFMA and FFMA2 probe kernels
    (gsb_fma_probe) on a full-occupancy grid, best of `reps` launches each after
    a warm-up, CUDA events on the launching stream (a burst figure, like the
    compositing kernels' launches of a fraction of a millisecond)."""
    from torch_gsplat_bridge_fast import _native

    L = _native.load()
    blocks, iters = 8, 65536
    n = int(L.gsb_fma_probe_out_floats(blocks))
    out = torch.empty(n, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    res = {}
    for packed, name in ((0, "ffma"), (1, "ffma2")):
        flops = n * iters * 8 * 2 * (2 if packed else 1)
        _native.check(L.gsb_fma_probe(packed, blocks, iters, _native.ptr(out), stream), "gsb_fma_probe")
        best = None
        for _ in range(reps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            _native.check(L.gsb_fma_probe(packed, blocks, iters, _native.ptr(out), stream), "gsb_fma_probe")
            e1.record()
            e1.synchronize()
            ms = e0.elapsed_time(e1)
            best = ms if best is None else min(best, ms)
        res[name] = round(flops / (best * 1e-3) / 1e12, 2)
    return res


def cpu_model() -> str:
    try:
        out = subprocess.run(["lscpu"], capture_output=True, text=True, timeout=10).stdout
        for line in out.splitlines():
            if line.startswith("Model name:"):
                return line.split(":", 1)[1].strip()
    except (OSError, subprocess.SubprocessError):
        pass
    return "unknown"


def time_steps_back_to_back(step, steps: int, flush):
    """K steps enqueued back to back, an L2 flush before each (outside the step
    events); every step's events are read after the final synchronize."""
    evs = []
    for _ in range(steps):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        step()
        e1.record()
        evs.append((e0, e1))
    torch.cuda.synchronize()
    return [a.elapsed_time(b) for a, b in evs]


def _max_over_ranks(x: float, dev, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _sum_over_ranks(x: float, dev, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def bench_c2_sharded(dev, rank: int, world: int, steps: int, flush):
    """Config 2 (B=4 independent 1024x512 views) with its views split over the
    ranks (torch_gsplat_bridge_fast.distributed.shard_views, round robin): each
    rank renders and differentiates its views as one batch, no collective.
    Strong scaling: the 4 views are fixed, so ranks beyond 4 have none. Time =
    max over ranks of the mean step."""
    import torch_gsplat_bridge_fast as tgb
    from torch_gsplat_bridge_fast.distributed import shard_views
    from torch_gsplat_bridge_fast.rasterize import _bin
    from workloads import config_2d, grad_image

    s = config_2d("c2", seed=0)
    views = shard_views(s.B, world, rank)
    E_mine, ms = 0.0, 0.0
    if views:
        idx = torch.tensor(views)
        base = [t[idx].contiguous().to(dev) for t in s.tensors()]
        g = grad_image(s.B, s.height, s.width, seed=1000)[idx].contiguous().to(dev)
        cfg = tgb.RasterConfig(s.height, s.width)
        st = _bin(cfg, *base)
        E_mine = float(tiled_work(st.tile_offsets, len(views), s.height, s.width))
        del st

        def step():
            ins = [t.detach().requires_grad_(i < 4) for i, t in enumerate(base)]
            tgb.rasterize_projected_gaussians(*ins, cfg).backward(g)

        for _ in range(3):
            step()
        torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    if views:
        ms = statistics.mean(time_steps_back_to_back(step, steps, flush))
    ms_max = _max_over_ranks(ms, dev, world)
    E_all = _sum_over_ranks(E_mine, dev, world)
    return {"workload": "c2: B=4 views, 1024x512, G=2,048 per view, fwd+bwd; views split over ranks",
            "ranks_with_views": min(world, s.B), "views_rank0": len(shard_views(s.B, world, 0)),
            "ms_per_step": round(ms_max, 4), "value": round(E_all / (ms_max * 1e-3) / 1e9, 3),
            "unit": UNIT, "scaling": "strong (4 views in total)"}


def bench_c4_shared(dev, rank: int, world: int, steps: int, flush, allreduce: str = "peer", sh_degree: int = 3):
    """Config 4's shared-scene training step: 2^20 Gaussians on every rank,
    rank r renders camera r mod 8 (projection, SH colours, binning, compositing
    fwd+bwd, projection VJP), then the per-Gaussian gradients (59 floats with
    SH degree 3) are summed across ranks by PeerGradAllReduce (the library's
    NVLink peer-memory kernel) or NCCL. Weak scaling: one view per rank."""
    import torch_gsplat_bridge_fast as tgb
    from torch_gsplat_bridge_fast.distributed import PeerGradAllReduce, SharedGradAllReduce
    from torch_gsplat_bridge_fast.rasterize import _bin
    from workloads import config_3d, grad_image

    sc = config_3d(seed=0)
    view = rank % sc.camera_to_world.shape[0]
    H, W, G = sc.height, sc.width, sc.means3d.shape[0]
    cfg = tgb.RasterConfig(H, W)
    fx, fy, cx, cy = (float(v) for v in sc.camera_params[view])
    c2w = sc.camera_to_world[view].to(dev)
    params = [t.to(dev).requires_grad_(True) for t in (sc.means3d, sc.scales, sc.quats, sc.opacities, sc.colors)]
    deg = sh_degree
    if deg >= 0:  # colour from SH: (deg+1)^2 x 3 coefficients per Gaussian replace the RGB
        K = (deg + 1) ** 2
        gsh = torch.Generator().manual_seed(11)
        sh = torch.randn(G, K, 3, generator=gsh) * 0.2
        sh[:, 0] = (sc.colors - 0.5) / 0.28209479177387814  # degree-0 term reproduces the RGB
        params[4] = sh.to(dev).requires_grad_(True)

    def colors_of(p):
        return tgb.spherical_harmonics_colors(p[4], p[0], c2w, degree=deg) if deg >= 0 else p[4]

    gimg = grad_image(1, H, W, seed=2000 + rank)[0].to(dev)
    with torch.no_grad():
        m2, q2, o2, d2 = tgb.project_pinhole_gaussians(*params[:4], fx, fy, cx, cy, camera_to_world=c2w)
        st = _bin(cfg, m2[None].contiguous(), q2[None].contiguous(), colors_of(params)[None].contiguous(),
                  o2[None].contiguous(), d2[None].contiguous())
        E = float(tiled_work(st.tile_offsets, 1, H, W))
        del st
    reducer = None
    if world > 1:
        reducer = PeerGradAllReduce(params) if allreduce == "peer" else SharedGradAllReduce(params)
    floats_per_gaussian = sum(p[0].numel() for p in params)
    nbytes = sum(p.numel() for p in params) * 4
    ex_evs = []

    def step(record=False):
        for p in params:
            p.grad = None
        img = tgb.rasterize_pinhole_gaussians(*params[:4], colors_of(params), fx, fy, cx, cy, camera_to_world=c2w,
                                              config=cfg)
        img.backward(gimg)
        if reducer is not None:
            a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a0.record()
            reducer()
            a1.record()
            if record:
                ex_evs.append((a0, a1))

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    step_ms = time_steps_back_to_back(lambda: step(True), steps, flush)
    ms = statistics.mean(step_ms)
    ex_ms = statistics.mean(a.elapsed_time(b) for a, b in ex_evs) if ex_evs else 0.0
    if isinstance(reducer, PeerGradAllReduce):
        reducer.check_errors()
    ms_max = _max_over_ranks(ms, dev, world)
    ex_max = _max_over_ranks(ex_ms, dev, world)
    E_all = _sum_over_ranks(E, dev, world)
    out = {"workload": f"c4: G={G} shared 3D Gaussians, SH degree {deg} colours, one {W}x{H} camera per rank "
                       f"(view = rank mod 8), fwd+bwd + gradient sum over ranks",
           "ms_per_step": round(ms_max, 4), "value": round(E_all / (ms_max * 1e-3) / 1e9, 3), "unit": UNIT,
           "scaling": "weak (one view per rank)", "grad_floats_per_gaussian": floats_per_gaussian,
           "exchange": None}
    if reducer is not None:
        out["exchange"] = {"impl": "NVLink peer-memory kernel (gsb_peer_allreduce_sum)" if allreduce == "peer"
                           else "NCCL all-reduce", "bytes": nbytes, "ms": round(ex_max, 4),
                           "share_of_step": round(ex_max / ms_max, 4),
                           "busbw_GBs": round(2 * (world - 1) / world * nbytes / (ex_max * 1e-3) / 1e9, 1),
                           "includes": "pack of the .grad tensors into the flat buffer and the sum"}
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        if isinstance(reducer, PeerGradAllReduce):
            reducer.close()
    return out


def run_b200(args):
    import torch.distributed as dist

    import torch_gsplat_bridge_fast as tgb
    from torch_gsplat_bridge_fast import _native
    from torch_gsplat_bridge_fast.rasterize import _bin, kernel_times, set_kernel_timer
    from workloads import config_2d, grad_image

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)

    if args.trace:
        from workloads import load_trace

        s = load_trace(args.trace, args.height, args.width)
    else:
        s = config_2d(args.config, seed=rank)
    B, G, H, W = s.B, s.G, s.height, s.width
    cfg = tgb.RasterConfig(H, W)
    base = [t.to(dev) for t in s.tensors()]
    gimg = grad_image(B, H, W, seed=1000 + rank).to(dev)
    st = _bin(cfg, *base)
    E = tiled_work(st.tile_offsets, B, H, W)
    P = st.P
    del st
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)

    def step():
        ins = [t.detach().requires_grad_(i < 4) for i, t in enumerate(base)]
        out = tgb.rasterize_projected_gaussians(*ins, cfg)
        out.backward(gimg)
        return ins

    for _ in range(max(args.warmup, 3)):
        flush.zero_()  # the flush's first launch is warm too before the bracket
        step()
    torch.cuda.synchronize()

    L = _native.load()
    step_ms = []
    with ClockSampler(local) as clocks:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        launches0 = L.gsb_kernel_launches()
        t_bracket = time.perf_counter()
        # Steps are enqueued back to back: the host prepares step k+1 while the
        # GPU runs step k (as in a training loop), and each step's events are
        # read after the bracket's final synchronize. Host latency before a
        # step's first launch is then not counted as device time.
        evs = []
        for _ in range(args.steps):
            flush.zero_()  # L2 flush between timed steps (outside the step events)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            step()
            e1.record()
            evs.append((e0, e1))
        torch.cuda.synchronize()
        step_ms = [a.elapsed_time(b) for a, b in evs]
        if world > 1:
            dist.barrier()
        bracket_ms = (time.perf_counter() - t_bracket) * 1e3
        launches = L.gsb_kernel_launches() - launches0
        # Forward only (the no-grad path, BASELINE config 3's first figure).

        def fwd_only():
            with torch.no_grad():
                tgb.rasterize_projected_gaussians(*base, cfg)

        for _ in range(3):
            flush.zero_()
            fwd_only()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        fwd_ms = statistics.mean(time_steps_back_to_back(fwd_only, args.steps, flush))
        # Per-kernel durations (the rooflines' denominators): the same K steps
        # again with the host runtime's per-phase events on. An event recorded
        # between two kernels ends their programmatic launch overlap (about
        # 26 us per c3 step for the 10 events), so the step time above is taken
        # without them.
        set_kernel_timer(True)
        for _ in range(args.steps):
            flush.zero_()
            step()
        torch.cuda.synchronize()
        kt = kernel_times()
        set_kernel_timer(False)
    clock = clocks.summary()
    ms = statistics.mean(step_ms)
    ms_med = statistics.median(step_ms)

    ms_max = _max_over_ranks(ms, dev, world)
    fwd_ms_max = _max_over_ranks(fwd_ms, dev, world)
    wall_ms = _max_over_ranks(bracket_ms / args.steps, dev, world)
    value = world * E / (ms_max * 1e-3) / 1e9
    probe = fp32_probe(dev)

    # Dominant kernel roofline (HBM-bound compositing / binning kernels).
    totals = {k: sum(v) for k, v in kt.items()}
    dom = max(totals, key=totals.get)
    dom_ms = statistics.mean(kt[dom])
    alg = algorithmic_bytes(dom, B, H, W, G, P)
    peak, peak_kind = load_peaks()
    achieved = alg / (dom_ms * 1e-3) / 1e9
    traffic = load_traffic("k_" + dom, args.config)
    kernels = {k: {"launches_per_step": len(v) / args.steps, "avg_ms": statistics.mean(v),
                   "share": totals[k] / max(sum(totals.values()), 1e-9)} for k, v in kt.items()}
    # The compositing kernels are FP32-issue bound, not HBM bound: their second
    # roofline is the FP32 pipe (algorithmic FLOPs per Gsplat-px eval x E).
    # Peak: the measured FFMA / FFMA2 probe (the better of the two), with the
    # nominal 148 SMs x 128 lanes x 2 x max clock for context.
    fp32_peak = max(probe.values())
    fp32_nominal = 148 * 128 * 2 * float(clock.get("sm_max_mhz") or 1965.0) * 1e6 / 1e12
    roof_fp32 = {}
    for k, fpe in FLOPS_PER_EVAL.items():
        if k in kt:
            tf = fpe * E / (statistics.mean(kt[k]) * 1e-3) / 1e12
            roof_fp32[k] = {"bound": "fp32", "achieved": round(tf, 2), "peak": round(fp32_peak, 1),
                            "peak_kind": "measured: FFMA/FFMA2 probe kernel (gsb_fma_probe), burst, this run",
                            "nominal_peak": round(fp32_nominal, 1), "unit": "TFLOP/s",
                            "frac": round(tf / fp32_peak, 4), "flops_per_eval": fpe,
                            "avg_launch_ms": round(statistics.mean(kt[k]), 4)}

    splits = None
    if not args.no_splits and not args.trace:
        splits = {"c2_views_sharded": bench_c2_sharded(dev, rank, world, min(args.steps, 50), flush),
                  "c4_shared_scene": bench_c4_shared(dev, rank, world, min(args.steps, 10), flush,
                                                     allreduce=args.allreduce)}

    e2e = None
    if not args.no_e2e:
        e2e = measure_e2e(tgb, s, gimg.cpu(), cfg, dev, E, steps=min(args.steps, 10))

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and not args.trace:
        cpu = cpu_baseline(args.config, seed=0)

    if rank == 0:
        default_workload = args.config == CONFIG_NAME and not args.trace
        line = {
            "metric": METRIC if default_workload else f"Gsplat-px evals/s, fwd+bwd at {W}x{H} x {G:,} splats x {B} views",
            "value": round(value, 3),
            "unit": UNIT,
            "n_gpus": world,
            "steps": args.steps,
            "warmup": max(args.warmup, 3),
            "ms_per_step": round(ms_max, 4),
            "ms_per_step_median": round(ms_med, 4),
            "wall_ms_per_step": round(wall_ms, 4),
            "bracket_ms": round(bracket_ms, 2),
            "forward_only": {"ms_per_step": round(fwd_ms_max, 4),
                             "value": round(world * E / (fwd_ms_max * 1e-3) / 1e9, 3), "unit": UNIT,
                             "path": "no-grad forward (binning + compositing), same inputs and flush"},
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "fp32",
            "data": f"recorded trace {os.path.basename(args.trace)}" if args.trace
            else "synthetic (seeded; BASELINE config distributions)",
            "config": {"workload": (f"trace {os.path.basename(args.trace)}" if args.trace else args.config)
                       + f": B={B}, {W}x{H}, G={G} 2D splats per GPU, fwd+bwd",
                       "pairs_per_view": P, "evals_per_view_E": E, "l2": "flushed (256 MB write) between steps",
                       "parallelism": f"views sharded, {world} rank(s), no collective"},
            "gpu_launches": int(launches),
            "kernels": kernels,
            "kernel_timing": "per-phase CUDA events on the launching stream, over a second run of the same K "
                             "steps right after the timed one (the events end the programmatic launch overlap "
                             "between kernels, so the timed steps run without them)",
            "roofline": {"kernel": dom, "bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "peak_kind": f"{peak_kind} copy bandwidth", "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "algorithmic_bytes_per_launch": alg,
                         "traffic": traffic, "avg_launch_ms": round(dom_ms, 4),
                         "binding": "FP32 issue, not HBM: the binding fraction is roofline_fp32[kernel].frac "
                                    "(bound names hbm because the contract offers only hbm or tensor)"},
            "roofline_fp32": roof_fp32,
            "fp32_probe_tflops": probe,
            "multi_gpu_splits": splits,
            "clocks": clock,
            "e2e": e2e,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def _time_steps(step, steps):
    for _ in range(3):
        step()
    torch.cuda.synchronize()
    times = []
    for _ in range(steps):
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        step()
        e1.record()
        e1.synchronize()
        times.append(e0.elapsed_time(e1))
    return statistics.mean(times)


def measure_e2e(tgb, s, gimg_cpu, cfg, dev, E, steps):
    """Same metric through the public API from pinned host buffers, every step:
    H2D of the splat tensors, fwd, the reference harness's loss
    out.square().mean() (benchmark_full_matrix.py) and its backward on the
    device, then D2H of the loss and the four gradients. A second figure ships
    the N(0,1) grad_image of the device-resident bench from the host instead
    (201 MB per step at c3, PCIe-bound)."""
    host = [t.contiguous().pin_memory() for t in s.tensors()]
    ghost = gimg_cpu.contiguous().pin_memory()
    outs = [torch.empty(t.shape, dtype=t.dtype).pin_memory() for t in host[:4]]
    loss_host = torch.empty((), dtype=torch.float32).pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in host)
    d2h = sum(t.numel() * t.element_size() for t in outs)

    def step_loss():
        ins = [t.to(dev, non_blocking=True).requires_grad_(i < 4) for i, t in enumerate(host)]
        out = tgb.rasterize_projected_gaussians(*ins, cfg)
        loss = out.square().mean()
        loss.backward()
        loss_host.copy_(loss.detach(), non_blocking=True)
        for o, t in zip(outs, ins[:4]):
            o.copy_(t.grad, non_blocking=True)

    def step_gimg():
        ins = [t.to(dev, non_blocking=True).requires_grad_(i < 4) for i, t in enumerate(host)]
        g = ghost.to(dev, non_blocking=True)
        out = tgb.rasterize_projected_gaussians(*ins, cfg)
        out.backward(g)
        for o, t in zip(outs, ins[:4]):
            o.copy_(t.grad, non_blocking=True)

    ms = _time_steps(step_loss, steps)
    ms_g = _time_steps(step_gimg, steps)
    g_bytes = ghost.numel() * ghost.element_size()
    return {"value": round(E / (ms * 1e-3) / 1e9, 3), "unit": UNIT, "ms_per_step": round(ms, 4),
            "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h + 4),
            "loss": "out.square().mean() on the device (the reference benchmark harness's loss)",
            "with_grad_image_from_host": {"value": round(E / (ms_g * 1e-3) / 1e9, 3), "ms_per_step": round(ms_g, 4),
                                          "h2d_bytes_per_step": int(h2d + g_bytes),
                                          "d2h_bytes_per_step": int(d2h)}}


def cpu_baseline(config: str, seed: int, steps: int = 1):
    """The C oracle (a restatement of the reference's algorithm; the reference
    itself is Metal-only) timed on this host's cores on one full step of the
    same workload: binning + forward + backward."""
    import numpy as np

    from oracle import oracle as O
    from workloads import config_2d, grad_image

    s = config_2d(config, seed=seed)
    g = grad_image(s.B, s.height, s.width, seed=1000).numpy()
    arrs = [t.numpy() for t in s.tensors()]
    meta = O.Meta(s.height, s.width, s.B, s.G)
    times = []
    E = 0
    for _ in range(steps):
        t0 = time.perf_counter()
        r = O.full_forward_backward(meta, *arrs, g)
        times.append(time.perf_counter() - t0)
        cnt = np.diff(r["tile_offsets"]).astype(np.int64)
        E = tiled_work(torch.from_numpy(r["tile_offsets"]), s.B, s.height, s.width)
    t = statistics.mean(times)
    cores = int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1))
    return {"value": round(E / t / 1e9, 4), "unit": UNIT, "cores": cores, "kind": "port",
            "seconds_per_step": round(t, 3), "cpu_model": cpu_model(),
            "sample": f"one full {config} fwd+bwd step (C oracle: binning + composite + reverse backward)",
            "torch_reference_c0": torch_reference_c0()}


def torch_reference_c0():
    """The reference's own torch CPU path on config 0 (the only config under
    its 64M-evaluation torch work limit): dense_torch_reference
    (benchmarks/benchmark_full_matrix.py:128-152, restated in
    oracle/torch_ref.dense_reference and pinned to the original's output by
    tests/golden/c0like_dense_torch_direct.npz), forward + autograd backward of
    a N(0,1) grad_image, all host threads. Dense work: every pixel x splat."""
    from oracle import torch_ref as TR
    from workloads import config_2d, grad_image

    s = config_2d("c0", seed=0)
    g = grad_image(1, s.height, s.width, seed=1000)
    threads = os.cpu_count() or 1
    prev = torch.get_num_threads()
    torch.set_num_threads(threads)
    try:
        ins = [t.clone().requires_grad_(i < 4) for i, t in enumerate(s.tensors())]
        t0 = time.perf_counter()
        out = TR.dense_reference(*ins, s.height, s.width)
        t1 = time.perf_counter()
        out.backward(g)
        t2 = time.perf_counter()
    finally:
        torch.set_num_threads(prev)
    dense = s.B * s.height * s.width * s.G
    return {"seconds_fwd": round(t1 - t0, 2), "seconds_fwd_bwd": round(t2 - t0, 2), "threads": threads,
            "dense_evals": dense, "dense_evals_per_s": round(dense / (t2 - t0) / 1e9, 4),
            "sample": "c0 (512x512, G=512) fwd+bwd, one run"}


def run_reference(args):
    """Reference arm: the reference is Metal-only (no CPU or CUDA build), so its
    algorithm runs as the C oracle port on this host's cores, same config/metric."""
    rank, world, _ = dist_env()
    if rank != 0:
        return
    import numpy as np

    from oracle import oracle as O
    from workloads import config_2d, grad_image

    s = config_2d(args.config, seed=0)
    g = grad_image(s.B, s.height, s.width, seed=1000).numpy()
    arrs = [t.numpy() for t in s.tensors()]
    meta = O.Meta(s.height, s.width, s.B, s.G)
    for _ in range(max(args.warmup, 3)):
        r = O.full_forward_backward(meta, *arrs, g)
    E = tiled_work(torch.from_numpy(r["tile_offsets"]), s.B, s.height, s.width)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        O.full_forward_backward(meta, *arrs, g)
        times.append(time.perf_counter() - t0)
    t = statistics.mean(times)
    cores = int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1))
    value = E / t / 1e9
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(value, 4),
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": max(args.warmup, 3),
        "ms_per_step": round(t * 1e3, 2),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "fp32",
        "data": "synthetic (seeded; BASELINE config distributions)",
        "config": {"workload": f"{args.config}: B={s.B}, {s.width}x{s.height}, G={s.G} 2D splats, fwd+bwd",
                   "evals_per_view_E": E},
        "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": cores, "kind": "port",
                         "cpu_model": cpu_model(),
                         "sample": f"one full {args.config} fwd+bwd step per timed step"},
        "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_shared3d(args):
    import torch.distributed as dist

    import torch_gsplat_bridge_fast as tgb
    from torch_gsplat_bridge_fast import _native
    from torch_gsplat_bridge_fast.distributed import PeerGradAllReduce, SharedGradAllReduce
    from torch_gsplat_bridge_fast.rasterize import _bin
    from workloads import config_3d, grad_image

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    sc = config_3d(seed=0)  # the same scene on every rank
    view = rank % sc.camera_to_world.shape[0]
    H, W, G = sc.height, sc.width, sc.means3d.shape[0]
    cfg = tgb.RasterConfig(H, W)
    fx, fy, cx, cy = (float(v) for v in sc.camera_params[view])
    c2w = sc.camera_to_world[view].to(dev)
    params = [t.to(dev).requires_grad_(True) for t in (sc.means3d, sc.scales, sc.quats, sc.opacities, sc.colors)]
    deg = args.sh_degree
    if deg >= 0:  # colour from SH: 48 (degree 3) coefficients per Gaussian replace the RGB
        K = (deg + 1) ** 2
        gsh = torch.Generator().manual_seed(11)
        sh = torch.randn(G, K, 3, generator=gsh) * 0.2
        sh[:, 0] = (sc.colors - 0.5) / 0.28209479177387814  # degree-0 term reproduces the RGB
        params[4] = sh.to(dev).requires_grad_(True)

    def colors_of(p):
        return tgb.spherical_harmonics_colors(p[4], p[0], c2w, degree=deg) if deg >= 0 else p[4]
    gimg = grad_image(1, H, W, seed=2000 + rank)[0].to(dev)
    with torch.no_grad():
        m2, q2, o2, d2 = tgb.project_pinhole_gaussians(*params[:4], fx, fy, cx, cy, camera_to_world=c2w)
        st = _bin(cfg, m2[None].contiguous(), q2[None].contiguous(), colors_of(params)[None].contiguous(),
                  o2[None].contiguous(), d2[None].contiguous())
        E = tiled_work(st.tile_offsets, 1, H, W)
        P = st.P
        del st
    reducer = None
    if world > 1:
        reducer = PeerGradAllReduce(params) if args.allreduce == "peer" else SharedGradAllReduce(params)
    reducer_floats = sum(p[0].numel() for p in params)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)

    def step(timing=None):
        for p in params:
            p.grad = None
        img = tgb.rasterize_pinhole_gaussians(*params[:4], colors_of(params), fx, fy, cx, cy, camera_to_world=c2w,
                                              config=cfg)
        img.backward(gimg)
        if reducer is not None:
            if timing is not None:
                timing[0].record()
            reducer()
            if timing is not None:
                timing[1].record()

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    L = _native.load()
    step_ms, ar_ms = [], []
    with ClockSampler(local) as clocks:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        launches0 = L.gsb_kernel_launches()
        evs = []
        for _ in range(args.steps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            step((a0, a1))
            e1.record()
            evs.append((e0, e1, a0, a1))
        torch.cuda.synchronize()  # every step's events are read after the bracket
        for e0, e1, a0, a1 in evs:
            step_ms.append(e0.elapsed_time(e1))
            if reducer is not None:
                ar_ms.append(a0.elapsed_time(a1))
        if world > 1:
            dist.barrier()
        launches = L.gsb_kernel_launches() - launches0
    clock = clocks.summary()
    ms = statistics.mean(step_ms)
    stats = torch.tensor([ms, float(E)], device=dev, dtype=torch.float64)
    if world > 1:
        mx = stats[:1].clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        tot = stats[1:].clone()
        dist.all_reduce(tot, op=dist.ReduceOp.SUM)
        ms_max, E_total = float(mx.item()), float(tot.item())
    else:
        ms_max, E_total = ms, float(E)
    allreduce = None
    if reducer is not None:
        t = statistics.mean(ar_ms) * 1e-3
        nbytes = reducer.bytes
        allreduce = {"impl": "peer-memory kernel (gsb_peer_allreduce_sum)" if args.allreduce == "peer"
                     else "NCCL all-reduce", "bytes": nbytes, "avg_ms": round(t * 1e3, 4),
                     "algbw_GBs": round(nbytes / t / 1e9, 1),
                     "busbw_GBs": round(2 * (world - 1) / world * nbytes / t / 1e9, 1),
                     "includes": "pack into the flat buffer and the sum; the summed grads are views into the buffer"
                     if args.allreduce == "peer" else "pack into the flat buffer, the sum, copy back"}
        if args.allreduce == "peer":
            reducer.check_errors()
    if rank == 0:
        line = {
            "metric": "Gsplat-px evals/s, c4 shared-3D fwd+bwd + gradient all-reduce",
            "value": round(E_total / (ms_max * 1e-3) / 1e9, 3),
            "unit": UNIT,
            "n_gpus": world,
            "steps": args.steps,
            "warmup": max(args.warmup, 3),
            "ms_per_step": round(ms_max, 4),
            "ms_per_step_median": round(statistics.median(step_ms), 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "fp32",
            "data": "synthetic (seeded; BASELINE c4 distributions)",
            "config": {"workload": f"c4: G={G} shared 3D Gaussians, one {W}x{H} camera per rank (view = rank mod 8)",
                       "pairs_rank0_view": P, "evals_rank0_view": E, "evals_all_ranks": E_total,
                       "l2": "flushed (256 MB write) between steps",
                       "parallelism": f"{world} rank(s); per-Gaussian grads ({reducer_floats} floats) summed with "
                                      + ("the NVLink peer-memory kernel" if args.allreduce == "peer" else "NCCL all-reduce"),
            "colors": f"spherical harmonics degree {deg}" if deg >= 0 else "RGB"},
            "gpu_launches": int(launches),
            "allreduce": allreduce,
            "clocks": clock,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        if isinstance(reducer, PeerGradAllReduce):
            reducer.close()
        dist.barrier()
        dist.destroy_process_group()


def _median_ms(fn, reps: int, warmup: int = 3) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    evs = []
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        evs.append((e0, e1))
    torch.cuda.synchronize()  # back-to-back repetitions, read after the last
    return statistics.median(a.elapsed_time(b) for a, b in evs)


def run_matrix(args):
    """Forward-only (no-grad path) and forward+backward medians on c0-c3 (2D
    splats) and c4 (3D scene, one camera), one JSON line each: the table of the
    reference's benchmark_full_matrix.py for this renderer."""
    import torch_gsplat_bridge_fast as tgb
    from torch_gsplat_bridge_fast.rasterize import _bin
    from workloads import config_2d, config_3d, grad_image

    dev = torch.device("cuda", 0)
    reps = max(args.steps, 5)
    for name in ("c0", "c1", "c2", "c3"):
        s = config_2d(name, seed=0)
        cfg = tgb.RasterConfig(s.height, s.width)
        base = [t.to(dev) for t in s.tensors()]
        g = grad_image(s.B, s.height, s.width, seed=1000).to(dev)
        st = _bin(cfg, *base)
        E, P = tiled_work(st.tile_offsets, s.B, s.height, s.width), st.P
        del st

        def fwd():
            with torch.no_grad():
                tgb.rasterize_projected_gaussians(*base, cfg)

        def fwd_bwd():
            ins = [t.detach().requires_grad_(i < 4) for i, t in enumerate(base)]
            tgb.rasterize_projected_gaussians(*ins, cfg).backward(g)

        f_ms, fb_ms = _median_ms(fwd, reps), _median_ms(fwd_bwd, reps)
        print(json.dumps({"matrix": name, "B": s.B, "G": s.G, "H": s.height, "W": s.width, "pairs": P, "evals": E,
                          "fwd_ms": round(f_ms, 4), "fwd_bwd_ms": round(fb_ms, 4),
                          "fwd_bwd_gsplat_px_per_s": round(E / (fb_ms * 1e-3) / 1e9, 3)}), flush=True)
    sc = config_3d(seed=0)
    cfg = tgb.RasterConfig(sc.height, sc.width)
    fx, fy, cx, cy = (float(v) for v in sc.camera_params[0])
    c2w = sc.camera_to_world[0].to(dev)
    params = [t.to(dev) for t in (sc.means3d, sc.scales, sc.quats, sc.opacities, sc.colors)]
    gimg = grad_image(1, sc.height, sc.width, seed=2000)[0].to(dev)

    def fwd3():
        with torch.no_grad():
            tgb.rasterize_pinhole_gaussians(*params, fx, fy, cx, cy, camera_to_world=c2w, config=cfg)

    def fwd_bwd3():
        ps = [p.detach().requires_grad_(True) for p in params]
        tgb.rasterize_pinhole_gaussians(*ps, fx, fy, cx, cy, camera_to_world=c2w, config=cfg).backward(gimg)

    f_ms, fb_ms = _median_ms(fwd3, reps), _median_ms(fwd_bwd3, reps)
    print(json.dumps({"matrix": "c4", "G": sc.means3d.shape[0], "H": sc.height, "W": sc.width, "views": 1,
                      "fwd_ms": round(f_ms, 4), "fwd_bwd_ms": round(fb_ms, 4)}), flush=True)


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
        return
    if not torch.cuda.is_available():
        print(json.dumps({"metric": METRIC, "error": "no CUDA device"}))
        sys.exit(1)
    if args.matrix:
        run_matrix(args)
        return
    if args.config == "c4":
        run_shared3d(args)
        return
    run_b200(args)


if __name__ == "__main__":
    main()
