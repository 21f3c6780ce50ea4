"""Benchmark of the localcorr hot path (RAFT pyramid correlation, fwd+bwd).

Contract: ``python bench.py --gpus N --steps K --warmup W [--impl ours|reference]``
prints ONE JSON line on rank 0. Under torchrun (N>1) each rank runs its
shard of the workload with no collective in the data path (row-band
workloads: one all-gather per frame); the timed region is bracketed by a
barrier and a device synchronisation on both sides and the elapsed time is
the max over ranks.

Workload (default, benchmark configuration 2): RAFT 1/8-resolution training
correlation, float16, a global batch of B=8 split over the N GPUs (8/N images
per rank: strong scaling, as the configuration is defined), C=256, 135x240,
4 levels, radius 4. ``raft_train_1080p_weak`` runs B=8 on every GPU instead
(weak scaling).
fmap1/fmap2 ~ N(0,1) (the 1/sqrt(C) is the block's output scale), coords =
grid + N(0, 6^2) flow with 5% of the pixels pushed out of bounds, 12 lookups
per step with coords perturbed by N(0,1) each. One step = block build (NHWC
transpose + pyramid) + 12 x (forward + backward) + the pyramid/transpose
backward, through the public API (get_localcorr_block + autograd).
Metric: lookups = B*H*W*L*(2r+1)^2 per lookup call; value = Glookups/s of
the whole job. Inputs (265 MB of maps + 2 GB of upstream gradients per GPU)
are larger than L2, so no explicit flush is needed between steps.

Workload raft_4k_rowband (benchmark configuration 4, forward only): one
B=1, C=256, 270x480 frame with smooth flow (sinusoids up to 40 px), 24
lookups per step, split into one row band per GPU (strong scaling): each rank
builds its band's pyramid levels, one all-gather assembles the frame's
pyramid on every rank (localcorr_b200.bands), and the lookups of the band run
locally; value = the frame's lookups per second.

Every workload except the row bands replays its timed steps from a CUDA
graph captured through the public API after the warm-up (the step's work is
unchanged; the graph removes the host launch gaps that dominate at one image
per GPU); the per-kernel times of the roofline come from an eager pass.

The reference arm (--impl reference) times the reference's CPU path as
restated in oracle/oracle.py (the all-pairs matmul + grid_sample formulation
of onnx_generic.py:58-156) on the host cores, on a bounded sample.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

CONFIGS = {
    # name: (B per GPU, C, H, W, levels, radius, lookups per step, dtype)
    # global batch 8 split over the ranks (strong scaling)
    "raft_train_1080p": dict(B=8, C=256, H=135, W=240, L=4, r=4, iters=12, dtype="f16",
                             coords="gauss_oob", fdist="normal", backward=True, split=True),
    # B=8 on every rank (weak scaling)
    "raft_train_1080p_weak": dict(B=8, C=256, H=135, W=240, L=4, r=4, iters=12, dtype="f16",
                                  coords="gauss_oob", fdist="normal", backward=True),
    "raft_cpu_case": dict(B=1, C=256, H=46, W=62, L=4, r=4, iters=1, dtype="f32",
                          coords="uniform8", fdist="normal", backward=True),
    "raft_4k_inference": dict(B=1, C=256, H=270, W=480, L=4, r=4, iters=24, dtype="f16",
                              coords="smooth", fdist="normal", backward=False),
    # the same 4K frame split into one row band per GPU (strong scaling): one
    # all-gather of the band pyramids per frame, then 24 local lookups per band
    "raft_4k_rowband": dict(B=1, C=256, H=270, W=480, L=4, r=4, iters=24, dtype="f16",
                            coords="smooth", fdist="normal", backward=False, bands=True),
    "highbatch_r3": dict(B=8, C=128, H=64, W=128, L=4, r=3, iters=1, dtype="f16",
                         coords="uniform64", fdist="uniform", backward=True),
    "highbatch_r4": dict(B=8, C=128, H=64, W=128, L=4, r=4, iters=1, dtype="f16",
                         coords="uniform64", fdist="uniform", backward=True),
    "highbatch_r8": dict(B=8, C=128, H=64, W=128, L=4, r=8, iters=1, dtype="f16",
                         coords="uniform64", fdist="uniform", backward=True),
    # PWC-Net spatial correlation over a 5-level feature pyramid (benchmark
    # configuration 3): B=8, patch 9, [C, H, W] per level
    # (its 15 kernels are short, so the step is replayed from a CUDA graph)
    "pwc_spatial_f32": dict(kind="spatial", B=8, r=4, iters=1, dtype="f32", backward=True,
                            levels=[(196, 7, 16), (128, 14, 32), (96, 28, 64), (64, 56, 128),
                                    (32, 112, 256)], split=True, graph=True),
    "pwc_spatial_f16": dict(kind="spatial", B=8, r=4, iters=1, dtype="f16", backward=True,
                            levels=[(196, 7, 16), (128, 14, 32), (96, 28, 64), (64, 56, 128),
                                    (32, 112, 256)], split=True, graph=True),
}
DEFAULT = "raft_train_1080p"
METRIC = "corr Glookups/s fwd+bwd (B*H*W*L*(2r+1)^2)"


def metric_name(cfg):
    """The headline metric; forward-only workloads count forward lookups."""
    return METRIC if cfg["backward"] else METRIC.replace("fwd+bwd", "fwd")


def _env_rank():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)),
            int(os.environ.get("WORLD_SIZE", 1)))


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d.get("hbm_gbs", 6650.0)), "measured"
    return 6650.0, "fallback"


def max_over_ranks(value, dist, device):
    """The job's elapsed time: the slowest rank's (no-op on one process)."""
    if dist is None:
        return float(value)
    t = torch.tensor([float(value)], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(value, dist, device):
    """Whole-job total of a per-rank count (no-op on one process)."""
    if dist is None:
        return value
    t = torch.tensor([float(value)], device=device, dtype=torch.float64)
    dist.all_reduce(t)
    return t.item()


def lookups_per_call(cfg):
    if cfg.get("kind") == "spatial":
        # one call = every level of the pyramid: B*H*W*(2r+1)^2 per level
        return sum(cfg["B"] * h * w for _, h, w in cfg["levels"]) * (2 * cfg["r"] + 1) ** 2
    return cfg["B"] * cfg["H"] * cfg["W"] * cfg["L"] * (2 * cfg["r"] + 1) ** 2


def algorithmic_bytes(cfg, kernel):
    """Bytes each tensor of one engine call occupies, touched once (storage dtype).

    A row band's call covers its rows of fmap1/coords/output and, of the
    frame's pyramid, the band's share of the rows."""
    es = 2 if cfg["dtype"] == "f16" else 4
    b, c, h, w, L, r = cfg["B"], cfg["C"], cfg["H"], cfg["W"], cfg["L"], cfg["r"]
    rows = cfg.get("band_rows", h)
    p = b * rows * w
    pyr = sum(b * (h >> l) * (w >> l) * c for l in range(L)) * es * rows // max(1, h)
    f1 = p * c * es
    coords = 2 * p * es
    out = p * L * (2 * r + 1) ** 2 * es
    fwd = f1 + pyr + coords + out
    if kernel == "pyramid_fwd":
        return fwd
    if kernel == "pyramid_bwd_fmap1":
        # grad_fmap1 with the grad_fmap2 records kept: reads f1, pyramid,
        # coords, corr_grad; writes grad_f1
        return fwd + f1
    if kernel == "pyramid_bwd_pull":
        # grad_fmap2 of a block's lookups (up to 12 per call): their f1,
        # coords and corr_grad in, the float32 grad pyramid out once
        n = min(cfg["iters"], 12)
        return f1 + n * (coords + out) + pyr * (4 // es)
    # backward: reads f1, pyramid, coords, corr_grad; writes grad_f1 and the
    # float32 grad pyramid (the C ABI's accumulator).
    return fwd + f1 + pyr * (4 // es)


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 200 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.mark = 0
        self._thr = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, FileNotFoundError):
            self.proc = None
            return
        self._thr = threading.Thread(target=self._read, daemon=True)
        self._thr.start()
        # nvidia-smi needs about a second to print its first sample; the timed
        # region starts only once sampling runs, and earlier samples are dropped.
        t0 = time.time()
        while not self.lines and time.time() - t0 < 10.0 and self.proc.poll() is None:
            time.sleep(0.05)
        self.mark = len(self.lines)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self._thr:
            self._thr.join(timeout=2)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        lines = self.lines[self.mark:] or self.lines
        for ln in lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() in ("active", "1", "yes"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax),
                "reasons": sorted(reasons), "samples": len(sm)}


def make_spatial_inputs(cfg, rank, device):
    """Configuration 3 inputs: per level input1 ~ N(0,1), input2 = input1
    rolled by an integer translation in [-4, 4]^2 per image plus N(0, 0.1^2)
    noise, upstream gradients ~ N(0,1); the rank's slice of the global batch."""
    g = torch.Generator().manual_seed(4321)
    dt = torch.float16 if cfg["dtype"] == "f16" else torch.float32
    gb = cfg.get("global_B", cfg["B"])
    lo, hi = rank * cfg["B"], (rank + 1) * cfg["B"]
    rd = 2 * cfg["r"] + 1
    host = {"in1": [], "in2": []}
    grads = []
    for c, h, w in cfg["levels"]:
        x1 = torch.randn(gb, c, h, w, generator=g)
        x2 = torch.empty_like(x1)
        for i in range(gb):
            ty, tx = (int(v) for v in torch.randint(-4, 5, (2,), generator=g))
            x2[i] = torch.roll(x1[i], shifts=(ty, tx), dims=(1, 2))
        x2 += 0.1 * torch.randn(x2.shape, generator=g)
        go = torch.randn(gb, rd, rd, h, w, generator=g)
        pin = (lambda t: t.pin_memory()) if torch.cuda.is_available() else (lambda t: t)
        host["in1"].append(pin(x1[lo:hi].to(dt).contiguous()))
        host["in2"].append(pin(x2[lo:hi].to(dt).contiguous()))
        grads.append(go[lo:hi].to(dt).contiguous())
    dev = {"in1": [t.to(device) for t in host["in1"]],
           "in2": [t.to(device) for t in host["in2"]],
           "grads": [t.to(device) for t in grads]}
    return host, dev


def run_spatial_step(cfg, in1, in2, grads):
    """One PWC step: the sampler (patch 9) forward on every level, then the
    backward of all of them; returns the input gradients of every level."""
    import localcorr_b200 as lc

    sampler = lc.get_localcorr_sampler(patch_size=2 * cfg["r"] + 1, corr_mode="localcorr_cuda")
    xs1 = [x.detach().requires_grad_(True) for x in in1]
    xs2 = [x.detach().requires_grad_(True) for x in in2]
    outs = [sampler(a, b) for a, b in zip(xs1, xs2)]
    torch.autograd.backward(outs, grads)
    return [x.grad for x in xs1], [x.grad for x in xs2]


def make_inputs(cfg, rank, device):
    """Seeded synthetic inputs of one rank: its own batch shard (weak
    scaling), its slice [rank*B, (rank+1)*B) of the one global batch all ranks
    share (cfg["split"], strong scaling), or (row-band workloads,
    cfg["band"] = (y0, y1)) its rows of the one frame all ranks share."""
    from oracle import oracle

    shared = cfg.get("bands") or cfg.get("split")
    seed = 0 if shared else rank
    g = torch.Generator().manual_seed(1234 + seed)
    dt = torch.float16 if cfg["dtype"] == "f16" else torch.float32
    b, c, h, w = cfg.get("global_B", cfg["B"]), cfg["C"], cfg["H"], cfg["W"]
    f1, f2 = oracle.make_fmaps(b, c, h, w, seed=1234 + seed, dist=cfg["fdist"])
    kind = cfg["coords"]
    if kind == "gauss_oob":
        c0 = oracle.make_coords_gauss_oob(b, h, w, 6.0, 0.05, seed=99 + seed)
    elif kind == "smooth":
        c0 = oracle.make_coords_smooth(b, h, w, 40.0, seed=99 + seed)
    elif kind == "uniform64":
        c0 = oracle.make_coords_uniform(b, h, w, 64.0, seed=99 + seed)
    else:
        c0 = oracle.make_coords_uniform(b, h, w, 8.0, seed=99 + seed)
    coords = []
    for i in range(cfg["iters"]):
        if i == 0:
            coords.append(c0)
        else:
            coords.append(coords[-1] + torch.randn(c0.shape, generator=g))
    if cfg.get("bands"):
        y0, y1 = cfg["band"]
        f1 = f1[:, :, y0:y1].contiguous()
        f2 = f2[:, :, y0:y1].contiguous()
        coords = [co[:, :, y0:y1].contiguous() for co in coords]
        h = y1 - y0
    rd = 2 * cfg["r"] + 1
    grads = None
    if cfg["backward"]:
        grads = [torch.randn(b, cfg["L"] * rd * rd, h, w, generator=g).to(dt)
                 for _ in range(cfg["iters"])]
    if cfg.get("split"):
        lo, hi = rank * cfg["B"], (rank + 1) * cfg["B"]
        f1 = f1[lo:hi].contiguous()
        f2 = f2[lo:hi].contiguous()
        coords = [co[lo:hi].contiguous() for co in coords]
        if grads is not None:
            grads = [gg[lo:hi].contiguous() for gg in grads]
    pin = (lambda t: t.pin_memory()) if torch.cuda.is_available() else (lambda t: t)
    host = dict(
        f1=pin(f1.to(dt)), f2=pin(f2.to(dt)),
        coords=[pin(co.to(dt)) for co in coords],
    )
    dev = dict(
        f1=host["f1"].to(device), f2=host["f2"].to(device),
        coords=[co.to(device) for co in host["coords"]],
        grads=[gg.to(device) for gg in grads] if grads is not None else None,
    )
    return host, dev


def run_step(cfg, f1, f2, coords, grads):
    import localcorr_b200 as lc

    if cfg.get("bands"):
        from localcorr_b200 import bands

        with torch.no_grad():
            block = bands.LocalCorrRowBandBlock(f1, f2, cfg["H"], num_levels=cfg["L"],
                                                radius=cfg["r"])
            outs = [block(co) for co in coords]
        return outs[-1], None
    if cfg["backward"]:
        f1 = f1.detach().requires_grad_(True)
        f2 = f2.detach().requires_grad_(True)
        block = lc.get_localcorr_block(f1, f2, num_levels=cfg["L"], radius=cfg["r"],
                                       corr_mode="localcorr_cuda")
        outs = [block(co) for co in coords]
        torch.autograd.backward(outs, grads)
        return f1.grad, f2.grad
    with torch.no_grad():
        block = lc.get_localcorr_block(f1, f2, num_levels=cfg["L"], radius=cfg["r"],
                                       corr_mode="localcorr_cuda")
        outs = [block(co) for co in coords]
    return outs[-1], None


def time_band_exchange(cfg, f2_band, steps, device, dist, world, rank):
    """The row-band step's collective alone: the all-gather of the band
    pyramids into the frame's pyramid (bands.gather_pyramid), timed with CUDA
    events over `steps` exchanges after warm-up, max over ranks. Every rank
    runs the same collectives in the same order."""
    from localcorr_b200 import bands

    b, c = f2_band.shape[0], f2_band.shape[1]
    layout = bands.RowBandLayout(b, c, cfg["H"], cfg["W"], cfg["L"], world)
    local = torch.ops.localcorr.pyramid_build(f2_band, cfg["L"])
    for _ in range(3):
        bands.gather_pyramid(layout, local, rank)
    torch.cuda.synchronize(device)
    dist.barrier()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        bands.gather_pyramid(layout, local, rank)
    end.record()
    torch.cuda.synchronize(device)
    ms = start.elapsed_time(end) / steps
    ms = max_over_ranks(ms / 1e3, dist, device) * 1e3
    bytes_per_rank = layout.B * layout.max_band_elems * local.element_size()
    return {"collective": "all_gather of the band pyramids (NCCL)", "ms_per_frame": ms,
            "bytes_in_per_rank": bytes_per_rank * (world - 1),
            "note": "timed alone after the step, same buffers; the step's time includes it"}


def timed_loop(fn, steps, device):
    torch.cuda.synchronize(device)
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        fn()
    end.record()
    torch.cuda.synchronize(device)
    return start.elapsed_time(end) / 1e3


def cpu_spatial_sample(cfg):
    """Time the reference's standard-ops spatial correlation (shifted slices
    of a zero-padded map, onnx_generic.py:159-198, restated as
    oracle.spatial_corr) on the host cores: one image of every level,
    float32, forward and backward."""
    from oracle import oracle

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    r = cfg["r"]
    g = torch.Generator().manual_seed(8)
    t0 = time.perf_counter()
    n = 0
    for c, h, w in cfg["levels"]:
        x1 = torch.randn(1, c, h, w, generator=g).requires_grad_(True)
        x2 = torch.randn(1, c, h, w, generator=g).requires_grad_(True)
        out = oracle.spatial_corr(x1, x2, r, dtype=torch.float32)
        out.backward(torch.ones_like(out))
        n += h * w * (2 * r + 1) ** 2
    dt = time.perf_counter() - t0
    return {"value": n / dt / 1e9, "unit": "Glookups/s", "cores": threads, "kind": "port",
            "sample": "1 image of each of the 5 levels, fp32, fwd+bwd, "
                      "oracle/oracle.py:spatial_corr (onnx_generic.py:159-198 form)",
            "seconds": dt}


def cpu_baseline_sample(cfg, seconds_hint=20.0):
    """Time the reference CPU formulation (restated in oracle/oracle.py) on a
    bounded sample: one image, a band of fmap1 rows, float32; forward and
    backward, or forward only for the forward-only workloads."""
    from oracle import oracle

    if cfg.get("kind") == "spatial":
        return cpu_spatial_sample(cfg)
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    c, h, w, L, r = cfg["C"], cfg["H"], cfg["W"], cfg["L"], cfg["r"]
    bwd = bool(cfg["backward"])
    rows = max(1, min(h, 32))
    f1, f2 = oracle.make_fmaps(1, c, h, w, seed=5)
    co = oracle.make_coords_gauss_oob(1, h, w, 6.0, 0.05, seed=6)
    f1 = f1[:, :, :rows].contiguous().requires_grad_(bwd)
    f2 = f2.clone().requires_grad_(bwd)
    co = co[:, :, :rows].contiguous()
    t0 = time.perf_counter()
    with torch.set_grad_enabled(bwd):
        out = oracle.pyramid_corr_matmul(f1, f2, co, L, r) / math.sqrt(c)
        if bwd:
            out.backward(torch.ones_like(out))
    dt = time.perf_counter() - t0
    n = rows * w * L * (2 * r + 1) ** 2
    return {"value": n / dt / 1e9, "unit": "Glookups/s", "cores": threads, "kind": "port",
            "sample": f"1 image, {rows} of {h} fmap1 rows x {w} cols, C={c}, L={L}, r={r}, "
                      f"fp32, {'fwd+bwd' if bwd else 'fwd'}, oracle/oracle.py:pyramid_corr_matmul",
            "seconds": dt}


def reference_arm(args, cfg, cfg_name):
    rank, _, world = _env_rank()
    if rank != 0:
        return 0
    torch.set_num_threads(os.cpu_count() or 1)
    for _ in range(args.warmup):
        cpu_baseline_sample(cfg)
    vals = []
    t_total = 0.0
    for _ in range(args.steps):
        s = cpu_baseline_sample(cfg)
        vals.append(s["value"])
        t_total += s["seconds"]
    v = statistics.median(vals)
    line = {
        "impl": "reference", "metric": metric_name(cfg), "value": v, "unit": "Glookups/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * t_total / max(1, args.steps), "higher_is_better": True,
        "scaling": "strong" if (cfg.get("split") or cfg.get("bands")) else "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": cfg_name, "per_step": s["sample"]},
        "cpu_baseline": {k: s[k] for k in ("unit", "cores", "kind", "sample")} | {"value": v},
        "e2e": {"value": v, "unit": "Glookups/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=60)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", default=DEFAULT, choices=sorted(CONFIGS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=None,
                    help="override the per-GPU batch (smaller cases of a workload, for profiling)")
    ap.add_argument("--cuda-graph", choices=["auto", "on", "off"], default="auto",
                    help="replay the timed steps from a CUDA graph (auto: the workload's default)")
    args = ap.parse_args(argv)
    cfg = dict(CONFIGS[args.config])
    if args.batch is not None:
        cfg["B"] = args.batch
    # Timed steps replay from a CUDA graph captured through the public API,
    # except for row bands (their step holds an NCCL all-gather).
    cfg.setdefault("graph", not cfg.get("bands"))
    if args.cuda_graph != "auto":
        cfg["graph"] = args.cuda_graph == "on"
    if args.impl == "reference":
        return reference_arm(args, cfg, args.config)

    rank, local_rank, world = _env_rank()
    if cfg.get("split"):
        if cfg["B"] % world:
            raise SystemExit(f"{args.config}: the global batch {cfg['B']} does not split over "
                             f"{world} ranks")
        cfg["global_B"] = cfg["B"]
        cfg["B"] = cfg["B"] // world
    if cfg.get("bands"):
        from localcorr_b200 import bands

        cfg["band"] = bands.band_rows(cfg["H"], world, 1 << (cfg["L"] - 1))[rank]
        cfg["band_rows"] = cfg["band"][1] - cfg["band"][0]
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        os.environ.setdefault("NCCL_DEBUG", "WARN")  # keep stdout to the one JSON line
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=device)
    from localcorr_b200 import _lib, ops

    lib = _lib.require_library()
    spatial = cfg.get("kind") == "spatial"
    if spatial:
        host, dev = make_spatial_inputs(cfg, rank, device)
        names = ["in1", "in2"]

        def step_on(x):
            return run_spatial_step(cfg, x["in1"], x["in2"], dev["grads"])
    else:
        host, dev = make_inputs(cfg, rank, device)
        names = ["f1", "f2", "coords"]

        def step_on(x):
            return run_step(cfg, x["f1"], x["f2"], x["coords"], dev["grads"])

    def step():
        return step_on(dev)

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize(device)

    def barrier():
        if dist is not None:
            dist.barrier()

    use_graph = bool(cfg.get("graph"))

    def capture(fn):
        """Record one step of fn in a CUDA graph (after two warm-up runs on a
        side stream, as torch.cuda.graph requires); returns the graph, the
        step's (static) outputs and the library launches it holds."""
        side = torch.cuda.Stream(device)
        side.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(side):
            for _ in range(2):
                fn()
        torch.cuda.current_stream(device).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        lib.localCorrB200LaunchCount(1)
        with torch.cuda.graph(graph):
            res = fn()
        n = int(lib.localCorrB200LaunchCount(1))
        torch.cuda.synchronize(device)
        return graph, res, n

    records = []
    if use_graph:
        # Per-kernel times come from an eager pass (events recorded inside a
        # graph are not per replay); the timed steps replay the graph.
        ops.set_launch_timer(records)
        for _ in range(min(args.steps, 10)):
            step()
        torch.cuda.synchronize(device)
        ops.set_launch_timer(None)
        g_main, _, graph_launches = capture(step)
        timed_step = g_main.replay
    else:
        timed_step = step

    # ---- timed region: device-resident inputs ----
    sampler = ClockSampler(local_rank) if rank == 0 else None
    if sampler:
        sampler.start()
    if not use_graph:
        ops.set_launch_timer(records)
    lib.localCorrB200LaunchCount(1)
    barrier()
    elapsed = timed_loop(timed_step, args.steps, device)
    barrier()
    launches = int(lib.localCorrB200LaunchCount(1))
    if use_graph:
        launches = graph_launches * args.steps  # replayed, not issued from the host
    ops.set_launch_timer(None)
    clocks = sampler.stop() if sampler else None
    elapsed = max_over_ranks(elapsed, dist, device)
    launches = int(sum_over_ranks(launches, dist, device))

    # per-kernel durations (and algorithmic bytes, where the op knows them)
    # from the live events
    per, per_bytes = {}, {}
    for name, s_ev, e_ev, nb in records:
        per.setdefault(name, []).append(s_ev.elapsed_time(e_ev) / 1e3)
        per_bytes.setdefault(name, []).append(nb)
    kern = max(per, key=lambda k: sum(per[k])) if per else None

    # ---- end-to-end through the public API with host buffers ----
    # Every step copies its inputs (maps and coords) from pinned host memory
    # and reads its result (a gradient checksum) back to the host. The copy of
    # step i+1 runs on a copy stream while step i computes (two device input
    # sets), as a training loop with a prefetching loader does; each step's
    # copy and read-back are inside the timed region.
    def as_list(v):
        return v if isinstance(v, list) else [v]

    def shaped(flat):
        """The step's input dict from a flat tensor list (order of names)."""
        out, k = {}, 0
        for n in names:
            cnt = len(as_list(dev[n]))
            out[n] = flat[k:k + cnt] if isinstance(dev[n], list) else flat[k]
            k += cnt
        return out

    host_flat = [t for n in names for t in as_list(host[n])]
    dsets = [[torch.empty_like(t) for n in names for t in as_list(dev[n])] for _ in range(2)]
    if use_graph:
        # one graph per device input set, so the copies of step i+1 still
        # overlap step i
        graphed = [capture(lambda d=d: step_on(shaped(d)))[:2] for d in dsets]
    copy_stream = torch.cuda.Stream(device)
    main_stream = torch.cuda.current_stream(device)

    def checksum(g):
        if g is None:
            return 0.0
        if isinstance(g, list):
            return torch.stack([x.double().sum() for x in g]).sum()
        return g.double().sum()

    def e2e_timed(steps):
        ready = [torch.cuda.Event() for _ in range(2)]
        freed = [torch.cuda.Event() for _ in range(2)]
        fetched = [torch.cuda.Event() for _ in range(steps)]
        res_host = torch.empty(steps, dtype=torch.float64).pin_memory()
        vals = []

        def issue_copy(i):
            d = dsets[i % 2]
            with torch.cuda.stream(copy_stream):
                if i >= 2:
                    copy_stream.wait_event(freed[i % 2])
                for dt_, ht_ in zip(d, host_flat):
                    dt_.copy_(ht_, non_blocking=True)
                ready[i % 2].record(copy_stream)

        torch.cuda.synchronize(device)
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record(main_stream)
        copy_stream.wait_event(start)
        issue_copy(0)
        for i in range(steps):
            if i + 1 < steps:
                issue_copy(i + 1)
            d = dsets[i % 2]
            main_stream.wait_event(ready[i % 2])
            if use_graph:
                graphed[i % 2][0].replay()
                g1, g2 = graphed[i % 2][1]
            else:
                g1, g2 = step_on(shaped(d))
            chk = checksum(g1) + checksum(g2)
            res_host[i:i + 1].copy_(chk.reshape(1), non_blocking=True)
            fetched[i].record(main_stream)
            freed[i % 2].record(main_stream)
            if i >= 1:
                fetched[i - 1].synchronize()
                vals.append(float(res_host[i - 1]))
        end.record(main_stream)
        torch.cuda.synchronize(device)
        vals.append(float(res_host[steps - 1]))
        return start.elapsed_time(end) / 1e3, vals

    e2e_timed(2)
    barrier()
    e2e_elapsed, _ = e2e_timed(args.steps)
    barrier()
    e2e_elapsed = max_over_ranks(e2e_elapsed, dist, device)

    exchange = None
    if cfg.get("bands") and world > 1:
        exchange = time_band_exchange(cfg, dev["f2"], max(args.steps, 10), device, dist, world,
                                      rank)

    lookups_step = lookups_per_call(cfg) * cfg["iters"]
    shards = 1 if cfg.get("bands") else world  # row bands split one frame
    value = lookups_step * args.steps * shards / elapsed / 1e9
    e2e_value = lookups_step * args.steps * shards / e2e_elapsed / 1e9
    h2d = sum(t.numel() * t.element_size() for t in host_flat)

    line = None
    if rank == 0:
        peak, peak_kind = _peaks()
        roof = None
        if kern:
            dur = statistics.mean(per[kern])
            nbs = per_bytes[kern]
            if all(nb is not None for nb in nbs):
                # calls of different sizes (the levels of a pyramid)
                abytes = sum(nbs) / len(nbs)
                achieved = sum(nbs) / sum(per[kern]) / 1e9
            else:
                # with the deferred grad_fmap2 pull, a lookup's backward call
                # computes grad_fmap1 only
                deferred = kern == "pyramid_bwd" and "pyramid_bwd_pull" in per
                abytes = algorithmic_bytes(cfg, "pyramid_bwd_fmap1" if deferred else kern)
                achieved = abytes / dur / 1e9
            traffic = None
            tf = ROOT / "profiles" / "traffic.json"
            if tf.exists():
                # bytes of one call at the capture's batch, scaled to this
                # rank's images (independent work units)
                tj = json.loads(tf.read_text())
                tkey = ("pyramid_bwd_fmap1" if kern == "pyramid_bwd" and "pyramid_bwd_pull" in per
                        else kern)
                traffic = tj.get(f"{args.config}:{tkey}")
                if traffic is not None and tj.get("batch"):
                    traffic = traffic * cfg["B"] / tj["batch"]
            roof = {"bound": "hbm", "kernel": kern, "achieved": achieved, "peak": peak,
                    "peak_source": peak_kind, "unit": "GB/s", "frac": achieved / peak,
                    "traffic": traffic, "algorithmic_bytes": abytes,
                    "launch_ms": 1e3 * dur, "launches_timed": len(per[kern]),
                    "share_of_step": sum(per[kern]) / elapsed,
                    "per_kernel_ms": {k: 1e3 * statistics.mean(v) for k, v in per.items()}}
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            cpu = cpu_baseline_sample(cfg)
            cpu.pop("seconds", None)
        line = {
            "metric": metric_name(cfg), "value": value, "unit": "Glookups/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(3, args.warmup),
            "ms_per_step": 1e3 * elapsed / args.steps, "higher_is_better": True,
            "scaling": "strong" if (cfg.get("bands") or cfg.get("split")) else "weak",
            "vs_baseline": None,
            "dtype": cfg["dtype"], "data": "synthetic",
            "config": {"workload": args.config, "B_per_gpu": cfg["B"], "global_batch":
                       cfg["B"] * shards, "C": cfg.get("C"), "H": cfg.get("H"),
                       "W": cfg.get("W"),
                       "levels": cfg["levels"] if spatial else cfg["L"], "radius": cfg["r"],
                       "lookups_per_step": cfg["iters"], "backward": cfg["backward"],
                       "parallelism": (f"row-band x{world}: one all-gather of the band "
                                       "pyramids per frame" if cfg.get("bands") else
                                       f"batch-split x{world}: {cfg['B']} of the global "
                                       f"{cfg['B'] * shards} images per rank, no collective"
                                       if cfg.get("split") else
                                       f"batch-shard x{world}, no collective"),
                       "l2": ("inputs larger than L2 (no flush)" if not spatial else
                              "the step touches ~400/200 MB (fp32/fp16: inputs, "
                              "correlations, their gradients), more than L2; no flush"),
                       "cuda_graph": use_graph},
            "e2e": {"value": e2e_value, "unit": "Glookups/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": 8,
                    "note": "inputs of step i+1 copied on a second stream during step i; "
                            "the read-back is a float64 checksum of the step's gradients "
                            "(they stay on the device, as in a training loop)"},
            "gpu_launches": launches,
            "roofline": roof,
            "cpu_baseline": cpu,
            "clocks": clocks,
        }
        if exchange is not None:
            line["exchange"] = exchange
        print(json.dumps(line), flush=True)
    # graphs go before the process group (none holds a collective, but a
    # graph that did would keep the exit waiting)
    if use_graph:
        del g_main, graphed
        torch.cuda.synchronize(device)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
