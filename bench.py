"""Benchmark of the Gaussian-splatting hot path on B200 (BASELINE.json metric).

Default workload (config 3): full data-parallel training step, 3M Gaussians,
SH degree 3, 64 views at 1920x1080 on seeded radius-4 sphere poses, L1 loss
against seeded uniform targets, view-sharded forward+backward, NCCL
all-reduce of the gradient arena, fused Adam. Metric: views/s (whole job).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config c3|c2|c4|c1]

For N > 1 launch with torch.distributed.run (one rank per GPU). Rank 0 prints
one JSON line. Timing: CUDA events on the working stream, barrier +
synchronize on both sides, max over ranks. Inputs (708 MB of parameters,
1.6 GB of targets) are larger than the 126 MB L2, so no flush is needed.
"""
import argparse
import ctypes as C
import importlib
import json
import math
import os
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
# Nominal FP32 (non-tensor) rate of a B200: 148 SMs x 128 lanes x 2 flop x 1.965 GHz.
FP32_NOMINAL_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12

CONFIGS = {
    "c3": dict(n=3_000_000, seed=0x6A5D0003, extent=1.0, views=64, W=1920, H=1080, radius=4.0,
               poses="sphere", train=True),
    "c2": dict(n=1_000_000, seed=0x6A5D0002, extent=1.0, views=1, W=1920, H=1080, radius=4.0,
               poses="sphere", train=True),
    "c4": dict(n=6_000_000, seed=0x6A5D0004, extent=3.0, views=256, W=3840, H=2160, radius=8.0,
               poses="orbit", train=False),
    "c1": dict(pairs=30_000_000, seed=0x6A5D0001, tiles=8160),
}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="c3", choices=sorted(CONFIGS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--exchange", default="fused", choices=["fused", "nccl"],
                    help="N>1 gradient exchange: fused NVLink reduce+Adam+broadcast kernel, or NCCL all-reduce")
    ap.add_argument("--no-tile-hints", action="store_true",
                    help="occluded binning without each view's per-tile depth cut from its previous forward")
    ap.add_argument("--multicast", default="auto", choices=["auto", "on", "off"],
                    help="fused exchange through the NVSwitch multicast object (auto: from 4 ranks on) or "
                         "over plain peer loads/stores")
    ap.add_argument("--views", type=int, default=None,
                    help="profiling knob: override the number of views of --config (small ncu cases)")
    ap.add_argument("--binning", default="occluded", choices=["occluded", "contributing", "reference"],
                    help="tile lists: contributing pairs binned in depth slices without Gaussians whose "
                         "tiles are already opaque (default), contributing pairs only, or the reference's "
                         "full lists")
    ap.add_argument("--t-stop", type=float, default=None,
                    help="transmittance stop (default: the reference's 1e-3; the north star names 1e-4)")
    return ap.parse_args()


def binning_of(gs, args):
    return {"occluded": gs._abi.GSC_BIN_OCCLUDED, "contributing": gs._abi.GSC_BIN_CONTRIBUTING,
            "reference": gs._abi.GSC_BIN_REFERENCE}[args.binning]


def t_stop_of(args):
    return 1e-3 if args.t_stop is None else args.t_stop


def workload_config(args, cfg, world):
    """The `config` object of both arms' lines: the workload only (what the
    run measured lives in `workload_stats`), so the two arms' configs are equal."""
    if args.config in ("c3", "c2"):
        return {"workload": f"{args.config}: train step, {cfg['n']} Gaussians SH3, {cfg['views']} views "
                            f"{cfg['W']}x{cfg['H']}, L1, gradient exchange + fused Adam",
                "global_batch_views": cfg["views"], "parallelism": f"dp{world} (views)",
                "binning": args.binning, "t_stop": t_stop_of(args),
                "l2": "inputs larger than L2 (708 MB params + 1.6 GB targets), no flush"}
    if args.config == "c4":
        return {"workload": f"c4: render-only, {cfg['n']} Gaussians, {cfg['views']} views "
                            f"{cfg['W']}x{cfg['H']}", "parallelism": f"views/{world}",
                "binning": args.binning, "t_stop": t_stop_of(args),
                "l2": "inputs larger than L2, no flush"}
    end_bit = 32 + int(math.ceil(math.log2(cfg["tiles"])))
    return {"workload": f"c1: stable sort of {cfg['pairs']} pairs by bits [0,{end_bit})",
            "parallelism": f"independent sorts/{world}", "l2": "inputs (360 MB) larger than L2, no flush"}


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    except Exception:
        return dict(PEAKS_FALLBACK), "fallback"


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        try:
            fd, self.path = tempfile.mkstemp(prefix=f"bench_clocks_gpu{self.gpu}_", suffix=".csv")
            self.f = os.fdopen(fd, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.f,
                stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.f.close()

    def summary(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    smax = float(parts[2])
                except ValueError:
                    continue
                for name, val in zip(names, parts[5:9]):
                    if val.lower().startswith("active"):
                        reasons.add(name)
        med = float(np.median(sm)) if sm else None
        try:
            os.unlink(self.path)
        except OSError:
            pass
        return {"sm_mhz": med, "sm_max_mhz": smax, "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# setup
# ---------------------------------------------------------------------------
def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def make_cameras(gs, cfg):
    if cfg["poses"] == "sphere":
        eyes = gs.sphere_poses(cfg["views"], cfg["radius"], cfg["seed"] + 101)
    else:
        eyes = gs.orbit_poses(cfg["views"], cfg["radius"])
    return [gs.make_camera(cfg["W"], cfg["H"], tuple(e)) for e in eyes]


def make_targets(cfg, lo, hi):
    """Seeded U[0,1] RGB targets of views [lo, hi) in pinned host memory."""
    import torch
    H, W = cfg["H"], cfg["W"]
    out = torch.empty(hi - lo, H, W, 3, dtype=torch.float32).pin_memory()
    for v in range(lo, hi):
        rng = np.random.default_rng(cfg["seed"] * 1000 + v)
        out[v - lo].copy_(torch.from_numpy(rng.random((H, W, 3), dtype=np.float32)))
    return out


class Timer:
    """CUDA events on the working stream, barrier + synchronize on both sides."""

    def __init__(self, torch, world):
        self.torch, self.world = torch, world

    def _fence(self):
        if self.world > 1:
            self.torch.distributed.barrier()
        self.torch.cuda.synchronize()

    def __enter__(self):
        self._fence()
        self.a = self.torch.cuda.Event(enable_timing=True)
        self.b = self.torch.cuda.Event(enable_timing=True)
        self.a.record()
        return self

    def __exit__(self, *exc):
        self.b.record()
        self._fence()
        self.ms = self.a.elapsed_time(self.b)

    def max_over_ranks(self):
        if self.world == 1:
            return self.ms
        t = self.torch.tensor([self.ms], device="cuda", dtype=self.torch.float64)
        self.torch.distributed.all_reduce(t, op=self.torch.distributed.ReduceOp.MAX)
        return float(t.item())


def profile_pge(gs, ctx, reset=True):
    v = C.c_uint64()
    gs._abi.check(gs._abi.lib().gsc_profile_pge(ctx, C.byref(v), 1 if reset else 0))
    return int(v.value)


def profile_read(gs, ctx, reset=True):
    _abi = gs._abi
    ms = (C.c_double * len(_abi.STAGES))()
    calls = (C.c_int64 * len(_abi.STAGES))()
    kern = (C.c_int64 * len(_abi.STAGES))()
    _abi.check(_abi.lib().gsc_profile_read(ctx, ms, calls, kern, 1 if reset else 0))
    return {name: {"ms": ms[i], "calls": calls[i], "kernels": kern[i]}
            for i, name in enumerate(_abi.STAGES)}


def pge_count(gs, rctx):
    """Pixel-Gaussian evaluations of the frame's last forward: per pixel, the
    tile-list entries visited before the T > t_stop test failed."""
    _abi = gs._abi
    W, H = rctx.width, rctx.height
    last = rctx.get(_abi.GSC_FRAME_LAST, np.uint32).reshape(H, W).astype(np.int64)
    fT = rctx.get(_abi.GSC_FRAME_FINAL_T, np.float32).reshape(H, W)
    rng = rctx.get(_abi.GSC_FRAME_RANGES, np.uint32).reshape(-1, 2).astype(np.int64)
    tx = (W + 15) // 16
    ty_idx = np.arange(H)[:, None] // 16
    tx_idx = np.arange(W)[None, :] // 16
    tile = ty_idx * tx + tx_idx
    length = (rng[:, 1] - rng[:, 0])[tile]
    stopped = fT <= rctx.config.t_stop
    visited = np.where(stopped, last, length)
    return int(visited.sum())


# ---------------------------------------------------------------------------
# algorithmic work per stage (bytes, or FP32 ops for compositing)
# ---------------------------------------------------------------------------
# DRAM bytes per launch of the dominant kernel on a config-3 view: ncu's
# dram__bytes_read + write of composite_bwd on the config-2 scene (96.5 MB at
# 148.5 M pixel-Gaussian evaluations), scaled by the evaluations of a
# config-3 view (199.3 M); the backward's traffic is its list entries' splat
# records and per-pixel state, which grow with them.
TRAFFIC_C3 = {"composite_bwd": 130e6}

PREPROCESS_B = 284      # read 236 (pos 12, log_scale 12, rot 16, logit 4, SH 192) + write 48 (splat record)
PARAM_ROW_B = 236  # the 59 floats of one Gaussian
GRAD2D_B = 36      # screen-space gradient row of one view
ADAM_B = 28 * 59        # read p, g, m, v + write p, m, v per float
FWD_FLOP_PER_PGE = 15
BWD_FLOP_PER_PGE = 30


def sort_bytes_per_pair(end_bit, key_bytes=8):
    """Histogram read + one read and one write of the pair per 8-bit pass."""
    passes = (end_bit + 7) // 8
    return key_bytes + 2 * (key_bytes + 4) * passes


def packed_sort_bytes(bits, hist=True, hi=False):
    """Packed (key << 32 | value) u64 words: histogram read (unless the producer
    counted the digits), read and write per pass; the last pass writes the 4-byte
    values (and the 4-byte keys with `hi`)."""
    passes = (bits + 7) // 8
    return (8 if hist else 0) + 16 * (passes - 1) + 8 + 4 + (4 if hi else 0)


# First depth slice of occluded binning (GS_OCC_FRAC1 of the library): the
# later slice's pair counting gathers the remaining positions again.
OCC_FIRST_SLICE = 0.2


def stage_work(n, binned, kept, pge, tiles, end_bit, batch=1, occluded=False, views_per_step=1, tile_cut=False):
    """Algorithmic work of each stage for ONE view: (bound, bytes or flops).

    Binning of a view = a stable depth sort of the N Gaussians (per view: 32 bits,
    4 passes; batched: one sort of view << 56 | (bits(depth) - bits(near)) << 28 |
    index words by 28 + ceil(log2(batch)) bits, 4 passes), a gather-scan and
    emission of packed (tile << 32 | id) words in depth order, which also counts
    the tile digits, and a stable sort of those words by the tile bits
    (end_bit - 32 bits) whose last pass writes the ids and the tile ranges.
    `binned`: pairs emitted and sorted per view (with occluded binning, those
    of both depth slices); `kept`: pairs in the final lists. The preprocess
    and its backward run once per `batch` views: parameters read once,
    gradient rows read and written once, one grad2d row per view. Adam runs
    once per step over every parameter: its share of one view is the step's
    bytes over the `views_per_step` this rank renders. tile_cut: occluded
    binning with each view's per-tile depth cut, whose two slices both walk
    every depth position (order + 32 B record read, count and sub-mask
    written) and whose emissions read the counts back."""
    tb = end_bit - 32
    depth_bits = 28 + max(1, (batch - 1).bit_length()) if batch > 1 else 32
    later = (1.0 - OCC_FIRST_SLICE) * n if occluded else 0.0
    slices = 2 if occluded else 1
    scan_b = 20 * n + 36 * later
    emit_b = (4 + 32) * n + 8 * binned
    if occluded and tile_cut:
        scan_b = 2 * (4 + 32 + 4 + 8) * n
        emit_b = 2 * 4 * n + 8 * binned
    return {
        # one launch per `batch` views: parameters read once, per view a 48 B splat
        # record + 32 B binning record + 8 B packed depth word
        "preprocess": ("hbm", (PARAM_ROW_B / batch + 88) * n),
        # order + binning-record word gather and the block-sum scan; the later
        # slice gathers order + the 32 B record again (skip test)
        "scan": ("hbm", scan_b),
        "emit": ("hbm", emit_b),  # order + 32 B binning record (or the cut's counts); packed pairs
        # depth sort (per view, or one per batch) + tile sorts of the binned pairs
        "sort": ("hbm", packed_sort_bytes(depth_bits, hi=batch == 1) * n + packed_sort_bytes(tb, hist=False) * binned),
        # empty ranges {~0, 0} -> {0, 0} per slice; occluded: the kept ids copied
        "ranges": ("hbm", 8 * tiles * slices + (8 * kept + 8 * tiles if occluded else 0)),
        "composite_fwd": ("fp32", FWD_FLOP_PER_PGE * pge),
        "composite_bwd": ("fp32", BWD_FLOP_PER_PGE * pge),
        "preprocess_bwd": ("hbm", (3 * PARAM_ROW_B / batch + GRAD2D_B) * n),
        "adam": ("hbm", ADAM_B * n / views_per_step),
    }


def rooflines(stats, work, peaks, views):
    """Per stage: algorithmic work of one view / the stage's device time per
    view (its CUDA-event milliseconds over the traced steps / views)."""
    out = {}
    for name, (bound, amount) in work.items():
        s = stats.get(name)
        if not s or s["calls"] == 0 or s["ms"] <= 0:
            continue
        per_view_s = s["ms"] / 1e3 / views
        if bound == "hbm":
            ach = amount / per_view_s / 1e9
            peak = peaks["hbm_gbs"]
            unit = "GB/s"
        else:
            ach = amount / per_view_s / 1e12
            peak = FP32_NOMINAL_TFLOPS
            unit = "TFLOP/s"
        out[name] = {"bound": bound, "achieved": round(ach, 2), "peak": round(peak, 1), "unit": unit,
                     "frac": round(ach / peak, 4), "ms_per_view": round(per_view_s * 1e3, 4),
                     "stage_calls": s["calls"], "kernels": s["kernels"], "share": None}
    tot = sum(stats[k]["ms"] for k in stats)
    for k in out:
        out[k]["share"] = round(stats[k]["ms"] / tot, 4) if tot else None
    return out


def profile_pairs(gs, ctx, reset=True):
    v = (C.c_uint64 * 2)()
    gs._abi.check(gs._abi.lib().gsc_profile_pairs(ctx, v, 1 if reset else 0))
    return int(v[0]), int(v[1])


# ---------------------------------------------------------------------------
# CPU baseline: the oracle port on the host cores (bounded sample)
# ---------------------------------------------------------------------------
def cpu_view_seconds(gs, arrays, cam, rcfg, target, threads, with_backward=True):
    from oracle import oracle as O
    O.set_threads(threads)
    sc = O.Scene(arrays)
    t = time.perf_counter()
    if with_backward:
        O.render_view(sc, cam.to_struct(), rcfg, target, 1.0 / target.size)
    else:
        O.render_view(sc, cam.to_struct(), rcfg)
    return time.perf_counter() - t


def cpu_adam_seconds(n, threads):
    from oracle import oracle as O
    O.set_threads(threads)
    rng = np.random.default_rng(0)
    groups = []
    for w, lr in ((3, 1.6e-4), (3, 5e-3), (4, 1e-3), (1, 5e-2), (48, 2.5e-3)):
        p = rng.standard_normal(n * w, dtype=np.float32)
        groups.append({"param": p, "grad": p.copy(), "m": np.zeros_like(p), "v": np.zeros_like(p),
                       "lr": lr})
    t = time.perf_counter()
    O.adam_step(groups, 0.9, 0.999, 1e-8, 1, 1.0 / 64)
    return time.perf_counter() - t


def cpu_baseline_train(gs, cfg, arrays, cams, rcfg, targets_host, threads):
    """One full view forward+backward (+ Adam over all parameters / views)."""
    tgt = targets_host[0].numpy()
    tv = cpu_view_seconds(gs, arrays, cams[0], rcfg, tgt, threads)
    ta = cpu_adam_seconds(cfg["n"], threads)
    per_view = tv + ta / cfg["views"]
    return {"value": round(1.0 / per_view, 4), "unit": "views/s", "cores": threads, "kind": "port",
            "sample": (f"1 view (view 0, {cfg['W']}x{cfg['H']}, {cfg['n']} Gaussians) fwd+bwd+L1 "
                       f"in {tv:.2f} s + Adam over all {cfg['n']}x59 floats in {ta:.2f} s / "
                       f"{cfg['views']} views; CPU oracle (C++ restatement, OpenMP)")}


# ---------------------------------------------------------------------------
# ours: training configs (c3, c2)
# ---------------------------------------------------------------------------
def run_train(args, cfg, rank, world, local, peaks, peak_kind):
    import torch
    gs = importlib.import_module("crystal-gausplat_b200")
    trainer_mod = importlib.import_module("crystal-gausplat_b200.trainer")
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    pg = torch.distributed.group.WORLD if world > 1 else None
    arrays = gs.synthetic_arrays(cfg["n"], cfg["seed"], cfg["extent"])
    g = gs.Gaussian3D(arrays, device=dev)
    cams = make_cameras(gs, cfg)
    rcfg = gs.default_config(binning=binning_of(gs, args), t_stop=args.t_stop)
    tr = trainer_mod.DataParallelTrainer(g, cams, rcfg, process_group=pg, exchange=args.exchange,
                                         multicast={"auto": "auto", "on": True, "off": False}[args.multicast],
                                         tile_hints=not args.no_tile_hints)
    host_t = make_targets(cfg, tr.lo, tr.hi)
    dev_t = host_t.to(dev)
    ctx = gs.context(dev)
    lib = gs._abi.lib()

    def targets(v):
        return dev_t[v - tr.lo]

    for _ in range(args.warmup):
        tr.step(targets)
    torch.cuda.synchronize()

    def one_step(counts):
        tr.zero()
        for v in tr.my_views:
            tr.view_fwd_bwd(v, targets(v))
            counts[0] += tr.last_ctx.num_rendered
        tr.reduce_and_step()

    # timed region: tracing off
    k0 = lib.gsc_kernel_count(ctx)
    keys_total = [0]
    with ClockSampler(local) as clk:
        with Timer(torch, world) as tm:
            for _ in range(args.steps):
                one_step(keys_total)
    ms = tm.max_over_ranks()
    launches = int(lib.gsc_kernel_count(ctx) - k0)
    keys_total = keys_total[0]
    views_done = args.steps * cfg["views"]
    value = views_done / (ms / 1e3)

    # a second pass of the same steps with the library's per-stage CUDA events
    # (stage times, pixel-Gaussian evaluations): the roofline's kernel times
    profile_read(gs, ctx, reset=True)
    profile_pge(gs, ctx, reset=True)
    profile_pairs(gs, ctx, reset=True)
    lib.gsc_profile_enable(ctx, 1)
    with Timer(torch, world) as tm_traced:
        for _ in range(args.steps):
            one_step([0])
    lib.gsc_profile_enable(ctx, 0)
    ms_traced = tm_traced.max_over_ranks()
    stats = profile_read(gs, ctx, reset=True)

    my_views = max(1, tr.hi - tr.lo)
    pge = profile_pge(gs, ctx) / (args.steps * my_views)  # exact mean over this rank's views
    keys_per_view = keys_total / (args.steps * my_views)
    tiles = ((cfg["W"] + 15) // 16) * ((cfg["H"] + 15) // 16)
    end_bit = 32 + int(math.ceil(math.log2(tiles)))
    binned, kept = (c / (args.steps * my_views) for c in profile_pairs(gs, ctx))
    occluded = rcfg.binning == gs._abi.GSC_BIN_OCCLUDED
    work = stage_work(cfg["n"], binned, kept, pge, tiles, end_bit, batch=tr.batch, occluded=occluded,
                      views_per_step=my_views, tile_cut=bool(tr.tile_hints))
    roof = rooflines(stats, work, peaks, args.steps * my_views)

    e2e = None
    if not args.no_e2e:
        feeder = trainer_mod.HostTargetFeeder(host_t, dev)
        tr.step_from_host(feeder)
        tr.loss.item()
        with Timer(torch, world) as tm2:
            for _ in range(args.steps):
                tr.step_from_host(feeder)
                float(tr.loss.item())  # device -> host read of the step's loss
        ms2 = tm2.max_over_ranks()
        e2e = {"value": round(views_done / (ms2 / 1e3), 3), "unit": "views/s",
               "h2d_bytes_per_step": int(cfg["views"] * cfg["H"] * cfg["W"] * 3 * 4),
               "d2h_bytes_per_step": 4 * world,
               "path": "DataParallelTrainer.step_from_host: Rasterizer.forward/backward + Adam through "
                       "the C ABI, each view's target copied from pinned host on a side stream"}

    result = None
    if rank == 0:
        dominant = max(roof, key=lambda k: roof[k]["share"] or 0) if roof else None
        hbm_stages = [k for k in roof if roof[k]["bound"] == "hbm"]
        top_hbm = max(hbm_stages, key=lambda k: roof[k]["share"] or 0) if hbm_stages else None
        result = {
            "metric": f"views/s fwd+bwd ({cfg['n'] // 1_000_000}M Gauss, {cfg['H']}p)",
            "value": round(value, 3), "unit": "views/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded Gaussians, poses and U[0,1] targets per BASELINE.json)",
            "config": workload_config(args, cfg, world),
            "workload_stats": {"exchange": tr.exchange, "exchange_path": tr.exchange_path,
                               "tile_hints": bool(tr.tile_hints),
                               "backward_batch_views": tr.batch,
                               "contributing_pairs_per_view": round(keys_per_view),
                               "binned_pairs_per_view": round(binned), "kept_pairs_per_view": round(kept),
                               "pge_per_view": round(pge),
                               "traced_pass_ms_per_step": round(ms_traced / args.steps, 3),
                               "stage_times": "per-stage CUDA events of a second, traced pass of "
                                              "the same steps (the timed region runs untraced)"},
            "gpu_launches": launches,
            "clocks": clk.summary(),
            "e2e": e2e,
            "roofline": dict(roof[dominant], kernel=dominant,
                             peak_kind="nominal FP32" if roof[dominant]["bound"] == "fp32" else peak_kind,
                             traffic=TRAFFIC_C3.get(dominant) if args.config == "c3" else None)
            if dominant else None,
            "roofline_hbm": dict(roof[top_hbm], kernel=top_hbm, peak_kind=peak_kind,
                                 traffic=TRAFFIC_C3.get(top_hbm) if args.config == "c3" else None)
            if top_hbm else None,
            "stages": roof,
        }
        if world == 1 and not args.no_cpu_baseline:
            from oracle import oracle as O
            result["cpu_baseline"] = cpu_baseline_train(
                gs, cfg, arrays, cams, O.default_config(binning=gs._abi.GSC_BIN_REFERENCE, t_stop=args.t_stop),
                host_t, os.cpu_count())
    return result


def reference_train(args, cfg, world):
    """--impl reference: the oracle port on all host threads, one view per step.
    Nothing here loads the CUDA library: the configuration comes from the
    oracle, the scene and cameras from the package's host-only helpers."""
    from oracle import oracle as O
    gs = importlib.import_module("crystal-gausplat_b200")
    arrays = gs.synthetic_arrays(cfg["n"], cfg["seed"], cfg["extent"])
    cams = make_cameras(gs, cfg)
    rcfg = O.default_config(binning=gs._abi.GSC_BIN_REFERENCE, t_stop=args.t_stop)  # the reference's lists
    threads = os.cpu_count()
    H, W = cfg["H"], cfg["W"]
    ta = cpu_adam_seconds(cfg["n"], threads)
    times = []
    for i in range(args.warmup + args.steps):
        v = i % cfg["views"]
        tgt = np.random.default_rng(cfg["seed"] * 1000 + v).random((H, W, 3), dtype=np.float32)
        t = cpu_view_seconds(gs, arrays, cams[v], rcfg, tgt, threads)
        if i >= args.warmup:
            times.append(t + ta / cfg["views"])
    per_view = float(np.mean(times))
    value = 1.0 / per_view
    return {"impl": "reference", "metric": f"views/s fwd+bwd ({cfg['n'] // 1_000_000}M Gauss, {H}p)",
            "value": round(value, 4), "unit": "views/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(per_view * 1e3, 1), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": workload_config(args, cfg, world),
            "cpu_baseline": {"value": round(value, 4), "unit": "views/s", "cores": threads, "kind": "port",
                             "sample": "one view of the workload per step (fwd+bwd+L1, the reference's "
                                       "full tile lists) + Adam over all parameters / views; the reference "
                                       "(Crystal + Metal) cannot build here, so the C++ oracle restating "
                                       "it runs"},
            "e2e": {"value": round(value, 4), "unit": "views/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


# ---------------------------------------------------------------------------
# ours: render sweep (c4) and sort alone (c1)
# ---------------------------------------------------------------------------
def run_render(args, cfg, rank, world, local, peaks, peak_kind):
    import torch
    gs = importlib.import_module("crystal-gausplat_b200")
    trainer_mod = importlib.import_module("crystal-gausplat_b200.trainer")
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    arrays = gs.synthetic_arrays(cfg["n"], cfg["seed"], cfg["extent"])
    g = gs.Gaussian3D(arrays, device=dev)
    cams = make_cameras(gs, cfg)
    rcfg = gs.default_config(binning=binning_of(gs, args), t_stop=args.t_stop)
    lo, hi = trainer_mod.shard(len(cams), rank, world)
    kb = gs._abi.GSC_MAX_BATCH_VIEWS  # views per Rasterizer.forward_batch (one preprocess pass)
    rctxs = [gs.RasterizerContext(dev) for _ in range(kb)]
    imgs = [torch.empty(cfg["H"], cfg["W"], 3, device=dev) for _ in range(kb)]
    ctx = gs.context(dev)
    lib = gs._abi.lib()

    def render_all(host_imgs=None):
        keys = 0
        for v0 in range(lo, hi, kb):
            views = list(range(v0, min(v0 + kb, hi)))
            gs.Rasterizer.forward_batch(g, [cams[v] for v in views], rctxs, config=rcfg,
                                        images=imgs[:len(views)])
            keys += sum(c.num_rendered for c in rctxs[:len(views)])
            if host_imgs is not None:
                for k in range(len(views)):
                    host_imgs[k].copy_(imgs[k], non_blocking=True)
        return keys

    for _ in range(args.warmup):
        render_all()
    torch.cuda.synchronize()
    k0 = lib.gsc_kernel_count(ctx)
    keys_total = 0
    with ClockSampler(local) as clk:  # timed region: tracing off
        with Timer(torch, world) as tm:
            for _ in range(args.steps):
                keys_total += render_all()
    ms = tm.max_over_ranks()
    launches = int(lib.gsc_kernel_count(ctx) - k0)
    # the same steps again with the library's per-stage events (stage times, PGE)
    profile_read(gs, ctx, reset=True)
    profile_pge(gs, ctx, reset=True)
    profile_pairs(gs, ctx, reset=True)
    lib.gsc_profile_enable(ctx, 1)
    for _ in range(args.steps):
        render_all()
    lib.gsc_profile_enable(ctx, 0)
    stats = profile_read(gs, ctx, reset=True)
    pix = args.steps * cfg["views"] * cfg["W"] * cfg["H"]
    value = pix / 1e6 / (ms / 1e3)
    pge = profile_pge(gs, ctx) / max(1, args.steps * (hi - lo))
    tiles = ((cfg["W"] + 15) // 16) * ((cfg["H"] + 15) // 16)
    end_bit = 32 + int(math.ceil(math.log2(tiles)))
    kpv = keys_total / max(1, args.steps * (hi - lo))
    binned, kept = (c / max(1, args.steps * (hi - lo)) for c in profile_pairs(gs, ctx))
    roof = rooflines(stats, stage_work(cfg["n"], binned, kept, pge, tiles, end_bit, batch=kb,
                                       occluded=rcfg.binning == gs._abi.GSC_BIN_OCCLUDED),
                     peaks, args.steps * (hi - lo))
    e2e = None
    if not args.no_e2e:
        host_imgs = [torch.empty(cfg["H"], cfg["W"], 3).pin_memory() for _ in range(kb)]
        with Timer(torch, world) as tm2:
            for _ in range(args.steps):
                render_all(host_imgs)
        ms2 = tm2.max_over_ranks()
        e2e = {"value": round(pix / 1e6 / (ms2 / 1e3), 2), "unit": "MPix/s", "h2d_bytes_per_step": 0,
               "d2h_bytes_per_step": int(cfg["views"] * cfg["H"] * cfg["W"] * 12),
               "path": "Rasterizer.forward_batch (8 views per preprocess pass) through the C ABI; "
                       "every image read back to pinned host"}
    if rank != 0:
        return None
    dominant = max(roof, key=lambda k: roof[k]["share"] or 0)
    res = {"metric": "render MPix/s (6M Gauss, 4K)", "value": round(value, 2), "unit": "MPix/s",
           "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
           "ms_per_step": round(ms / args.steps, 3), "higher_is_better": True, "scaling": "strong",
           "vs_baseline": None, "dtype": "f32", "data": "synthetic",
           "config": workload_config(args, cfg, world),
           "workload_stats": {"contributing_pairs_per_view": round(kpv), "binned_pairs_per_view": round(binned),
                              "kept_pairs_per_view": round(kept), "pge_per_view": round(pge)},
           "gpu_launches": launches, "clocks": clk.summary(), "e2e": e2e,
           "roofline": dict(roof[dominant], kernel=dominant, traffic=None,
                            peak_kind="nominal FP32" if roof[dominant]["bound"] == "fp32" else peak_kind),
           "stages": roof}
    if world == 1 and not args.no_cpu_baseline:
        from oracle import oracle as O
        t = cpu_view_seconds(gs, arrays, cams[0], O.default_config(binning=gs._abi.GSC_BIN_REFERENCE, t_stop=args.t_stop),
                             None, os.cpu_count(), with_backward=False)
        res["cpu_baseline"] = {"value": round(cfg["W"] * cfg["H"] / 1e6 / t, 3), "unit": "MPix/s",
                               "cores": os.cpu_count(), "kind": "port",
                               "sample": f"1 view (view 0) forward, {t:.2f} s, CPU oracle (OpenMP)"}
    return res


def sort_input(cfg, n):
    rng = np.random.default_rng(cfg["seed"])
    tiles = rng.integers(0, cfg["tiles"], n, dtype=np.uint64)
    depth = rng.uniform(0.5, 10.0, n).astype(np.float32).view(np.uint32).astype(np.uint64)
    return (tiles << np.uint64(32)) | depth, np.arange(n, dtype=np.uint32)


def run_sort(args, cfg, rank, world, local, peaks, peak_kind):
    import torch
    gs = importlib.import_module("crystal-gausplat_b200")
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    n = cfg["pairs"]
    keys, vals = sort_input(cfg, n)
    k0d = torch.from_numpy(keys.view(np.int64)).to(dev)
    v0d = torch.from_numpy(vals.view(np.int32)).to(dev)
    kd, vd = k0d.clone(), v0d.clone()
    end_bit = 32 + int(math.ceil(math.log2(cfg["tiles"])))
    ctx = gs.context(dev)
    lib = gs._abi.lib()
    for _ in range(args.warmup):
        kd.copy_(k0d); vd.copy_(v0d)
        gs.GPURadixSort.sort(kd, vd, n, 0, end_bit)
    torch.cuda.synchronize()
    profile_read(gs, ctx, reset=True)
    k0 = lib.gsc_kernel_count(ctx)
    lib.gsc_profile_enable(ctx, 1)
    with ClockSampler(local) as clk:
        with Timer(torch, world) as tm:
            for _ in range(args.steps):
                kd.copy_(k0d); vd.copy_(v0d)  # restore the unsorted input (outside the sort stage)
                gs.GPURadixSort.sort(kd, vd, n, 0, end_bit)
    lib.gsc_profile_enable(ctx, 0)
    stats = profile_read(gs, ctx, reset=True)
    sort_ms = stats["sort"]["ms"]
    if world > 1:
        t = torch.tensor([sort_ms], device=dev, dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        sort_ms = float(t.item())
    value = world * args.steps * n / 1e6 / (sort_ms / 1e3)
    per = sort_ms / 1e3 / args.steps
    ach = sort_bytes_per_pair(end_bit) * n / per / 1e9  # 8-byte keys, 8-bit digits
    e2e = None
    if not args.no_e2e:
        hk = torch.from_numpy(keys.view(np.int64)).pin_memory()
        hv = torch.from_numpy(vals.view(np.int32)).pin_memory()
        with Timer(torch, world) as tm2:
            for _ in range(args.steps):
                kd.copy_(hk, non_blocking=True); vd.copy_(hv, non_blocking=True)
                gs.GPURadixSort.sort(kd, vd, n, 0, end_bit)
                hk2 = kd.to("cpu", non_blocking=False)
                hv2 = vd.to("cpu", non_blocking=False)
        ms2 = tm2.max_over_ranks()
        e2e = {"value": round(world * args.steps * n / 1e6 / (ms2 / 1e3), 1), "unit": "Mkey/s",
               "h2d_bytes_per_step": n * 12, "d2h_bytes_per_step": n * 12,
               "path": "GPURadixSort.sort (gsc_sort_pairs_u64) with host keys/values in and out"}
    if rank != 0:
        return None
    res = {"metric": "sort Mkey/s (30M u64/u32 pairs)", "value": round(value, 1), "unit": "Mkey/s",
           "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per * 1e3, 4),
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u64",
           "data": "synthetic (tile in [0,8160) << 32 | fp32 depth bits, depth U[0.5,10])",
           "config": workload_config(args, cfg, world),
           "gpu_launches": int(lib.gsc_kernel_count(ctx) - k0), "clocks": clk.summary(), "e2e": e2e,
           "roofline": {"kernel": "sort", "bound": "hbm", "achieved": round(ach, 1),
                        "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": round(ach / peaks["hbm_gbs"], 4),
                        "traffic": None, "peak_kind": peak_kind,
                        "bytes_per_pair": sort_bytes_per_pair(end_bit)}}
    if world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = reference_sort(args, cfg, bounded=True)["cpu_baseline"]
    return res


def reference_sort(args, cfg, bounded=False, world=1):
    from oracle import oracle as O
    n = 3_000_000
    keys, vals = sort_input(cfg, n)
    times = []
    reps = 2 if bounded else args.warmup + args.steps
    for i in range(reps):
        t = time.perf_counter()
        O.sort_pairs(keys, vals, 0, 45)
        times.append(time.perf_counter() - t)
    per = float(np.mean(times[-max(1, len(times) - (0 if bounded else args.warmup)):]))
    v = n / 1e6 / per
    return {"impl": "reference", "metric": "sort Mkey/s (30M u64/u32 pairs)", "value": round(v, 2),
            "unit": "Mkey/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(per * 1e3, 1), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u64", "data": "synthetic",
            "config": workload_config(args, cfg, world),
            "cpu_baseline": {"value": round(v, 2), "unit": "Mkey/s", "cores": 1, "kind": "port",
                             "sample": "3M of the 30M pairs per step, std::stable_sort (the reference's CPU key "
                                       "sort, rasterizer.cr:250-255, is a comparison sort)"},
            "e2e": {"value": round(v, 2), "unit": "Mkey/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


def reference_render(args, cfg, world):
    from oracle import oracle as O
    gs = importlib.import_module("crystal-gausplat_b200")
    arrays = gs.synthetic_arrays(cfg["n"], cfg["seed"], cfg["extent"])
    cams = make_cameras(gs, cfg)
    rcfg = O.default_config(binning=gs._abi.GSC_BIN_REFERENCE, t_stop=args.t_stop)  # the reference's lists
    times = []
    for i in range(args.warmup + args.steps):
        t = cpu_view_seconds(gs, arrays, cams[i % len(cams)], rcfg, None, os.cpu_count(), False)
        if i >= args.warmup:
            times.append(t)
    v = cfg["W"] * cfg["H"] / 1e6 / float(np.mean(times))
    return {"impl": "reference", "metric": "render MPix/s (6M Gauss, 4K)", "value": round(v, 3),
            "unit": "MPix/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(float(np.mean(times)) * 1e3, 1), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": workload_config(args, cfg, world),
            "cpu_baseline": {"value": round(v, 3), "unit": "MPix/s", "cores": os.cpu_count(),
                             "kind": "port", "sample": "one view per step, CPU oracle (OpenMP)"},
            "e2e": {"value": round(v, 3), "unit": "MPix/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


def emit_line(res, out_fd):
    """The one JSON result line, on the process's original standard output."""
    os.write(out_fd, (json.dumps(res) + "\n").encode())


def main():
    args = parse()
    rank, world, local = dist_env()
    # Everything but the result line (NCCL's version banner, library chatter)
    # goes to standard error, so standard output carries exactly one line.
    sys.stdout.flush()
    out_fd = os.dup(1)
    os.dup2(2, 1)
    cfg = dict(CONFIGS[args.config])
    if args.views:
        cfg["views"] = args.views
    if args.impl == "reference":
        if rank == 0:
            if args.config == "c1":
                res = reference_sort(args, cfg, world=world)
            elif args.config == "c4":
                res = reference_render(args, cfg, world)
            else:
                res = reference_train(args, cfg, world)
            emit_line(res, out_fd)
        return
    import torch
    if world > 1:
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", device_id=torch.device("cuda", local))
    peaks, peak_kind = load_peaks()
    if args.config in ("c3", "c2"):
        res = run_train(args, cfg, rank, world, local, peaks, peak_kind)
    elif args.config == "c4":
        res = run_render(args, cfg, rank, world, local, peaks, peak_kind)
    else:
        res = run_sort(args, cfg, rank, world, local, peaks, peak_kind)
    if rank == 0:
        emit_line(res, out_fd)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
