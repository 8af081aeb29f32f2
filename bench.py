"""Benchmark: propagated edges/sec of the Scheme-A large-reservoir churn step.

Workload (the configuration the metric's 1/2/4/8-GPU
figures are quoted on): 1,048,576 tanh units + 16 inputs, fan-in 256
(268,435,456 recurrent + 16,777,216 input edges, one PIPELINE bucket), one
step = forward propagation of every live edge with the 0.1% magnitude prune
fused in, the tanh apply, per-unit Philox proposals, the total-order
selection of 0.1% of the recurrent edges and the pipeline slot claim.
Scheme-A: the capacity axis is split into N contiguous bands, one per rank;
the per-unit partials are combined over NVLink peer memory in one kernel with
the apply, the claim's per-level free counts riding on the same barrier
(strong scaling: the arena is fixed).

value  = live edges x steps x N-independent / max-over-ranks device time of K
         steps (inputs resident in HBM, arena 3.7 GB >> 126 MB L2).
e2e    = the same metric through the public make_step API with each step's
         inputs copied from pinned host memory and the step's overflow flag
         and grown count read back (as the reference's Driver does each step).
--impl reference runs the reference's algorithm on the host cores (the C
oracle restatement; JAX, which the reference needs, is not installed on this
image) on rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import pathlib
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "propagated edges/sec per step (Scheme-A large reservoir churn step)"
UNIT = "edges/s"
# DRAM bytes (read + write) per swept mirror entry of the fused forward+prune
# sweep, from one ncu capture of the 2^18-unit reservoir with the full-size
# chunk of 2048 units (579.7 MB over 71,303,168 entries per launch); the
# traffic reported for a full launch is this figure times its swept entries
# (traffic grows in proportion to them)
NCU_TRAFFIC_BYTES_PER_ENTRY = 8.13


def _env_int(name: str, default: int) -> int:
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


def parse() -> argparse.Namespace:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="engine", choices=["engine", "reference"])
    ap.add_argument("--units-log2", type=int, default=20, help="reservoir size (2**x units)")
    ap.add_argument("--fan-in", type=int, default=256)
    ap.add_argument("--chunk-bits", type=int, default=None,
                    help="mirror destination chunk (2**x units); default: the largest the unit count allows, "
                         "capped at 13 (11 for the full-size reservoir)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-steps", type=int, default=3)
    ap.add_argument("--kernel-breakdown", action="store_true",
                    help="after the timing, print (stderr, rank 0) every kernel's device time per step over five "
                         "graph replays, from the profiler's activity records")
    return ap.parse_args()


def config(args):
    from plastax_b200.configs import ReservoirConfig

    return ReservoirConfig(num_units=1 << args.units_log2, fan_in=args.fan_in)


def workload_desc(cfg, n_gpus: int) -> dict:
    return {
        "workload": "scheme_a_reservoir_churn (BASELINE configs[4])",
        "units": cfg.num_units + cfg.num_inputs,
        "fan_in": cfg.fan_in,
        "live_edges": cfg.live_edges,
        "churn_per_step": cfg.k,
        "propagation": "pipeline",
        "parallelism": f"scheme_a_conn_shard{n_gpus}",
        "l2": f"inputs larger than L2: each rank sweeps {8 * cfg.live_edges / n_gpus / 1e9:.2f} GB of mirror entries "
              f"per step (L2 126 MB)",
    }


# ---------------------------------------------------------------------------
# host (CPU) arena + oracle step: the reference arm and the cpu_baseline
# ---------------------------------------------------------------------------
def host_reservoir(cfg):
    """The reservoir arena built on the host (seeded numpy), source-major."""
    import ctypes

    from oracle import oracle as orc
    from plastax_b200 import topo

    rng = np.random.default_rng(cfg.seed)
    n_in, n_res = cfg.num_inputs, cfg.num_units
    n = n_in + n_res
    rec_src = (rng.integers(0, n_res, cfg.recurrent_edges, dtype=np.int32) + n_in).astype(np.int32)
    rec_dst = np.repeat(np.arange(n_res, dtype=np.int32) + n_in, cfg.fan_in)
    src = np.concatenate([rec_src, np.tile(np.arange(n_in, dtype=np.int32), n_res)])
    del rec_src
    dst = np.concatenate([rec_dst, np.repeat(np.arange(n_res, dtype=np.int32) + n_in, n_in)])
    del rec_dst
    w = np.concatenate([(rng.standard_normal(cfg.recurrent_edges, dtype=np.float32) * np.float32(cfg.sigma)),
                        rng.uniform(-1, 1, cfg.input_edges).astype(np.float32)])
    # generated in ascending-destination order per source, so a stable sort by
    # source alone is the builder's packed (src, dst) order
    perm = np.empty(src.size, np.int64)
    orc.lib().pxo_stable_order_by_key(ctypes.c_int64(src.size), orc._p(src), ctypes.c_int32(n), orc._p(perm))
    live = src.size
    cap = topo.capacity_policy(live, headroom=cfg.capacity_headroom, align=cfg.capacity_align)
    b = {"from_id": np.zeros(cap, np.int32), "to_id": np.zeros(cap, np.int32), "dead": np.ones(cap, np.uint8),
         "weight": np.zeros(cap, np.float32)}
    b["from_id"][:live] = src[perm]
    b["to_id"][:live] = dst[perm]
    b["weight"][:live] = w[perm]
    b["dead"][:live] = 0
    level = np.ones(n, np.int32)
    level[:n_in] = 0
    return b, level, live


def cpu_run(cfg, steps: int, warmup: int, threads: int):
    """Time the oracle's reservoir churn step on the host; returns
    (seconds per step list, live edges)."""
    from oracle.steps import ReservoirOracle

    b, level, live = host_reservoir(cfg)
    n = cfg.num_inputs + cfg.num_units
    act = np.zeros(n, np.float32)
    ro = ReservoirOracle(b, act, level, live, num_inputs=cfg.num_inputs, num_res=cfg.num_units, tau=cfg.tau,
                         k=cfg.k, init_a=cfg.sigma * math.sqrt(3.0), seed=cfg.seed, threads=threads)
    rng = np.random.default_rng(1)
    times = []
    for i in range(warmup + steps):
        x = rng.standard_normal(cfg.num_inputs).astype(np.float32)
        t0 = time.perf_counter()
        ro.step(x)
        dt = time.perf_counter() - t0
        if i >= warmup:
            times.append(dt)
    return times, live


def reference_arm(args) -> None:
    rank = _env_int("RANK", 0)
    if rank != 0:
        return
    from oracle import oracle as orc

    cfg = config(args)
    threads = orc.max_threads()
    steps = max(1, min(args.steps, 5))
    warmup = min(args.warmup, 1)
    times, live = cpu_run(cfg, steps, warmup, threads)
    per_step = float(np.median(times))
    value = live / per_step
    sample = (f"{steps} timed full-size churn steps (median) after {warmup} warm-up, of the "
              f"{args.steps} requested: the oracle restatement of the reference's step on {threads} host "
              f"threads (forward+prune, proposals, total order, the claim's free-slot lists; the in-order "
              f"candidate assignment sequential)")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": steps, "warmup": warmup, "ms_per_step": per_step * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)",
        "config": workload_desc(cfg, 1),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# clocks sampling during the timed region
# ---------------------------------------------------------------------------
class Clocks:
    """SM clocks and throttle reasons of one GPU, sampled every 5 ms by NVML
    in a background thread while the timed region runs (reads only)."""

    HW_SLOWDOWN, HW_THERMAL, SW_THERMAL, SW_POWER_CAP = 0x8, 0x40, 0x20, 0x4

    def __init__(self, index: int) -> None:
        import threading

        self.index = index
        self.samples: list[tuple[float, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None

    def _run(self) -> None:
        import pynvml

        pynvml.nvmlInit()
        h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
        self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
        while not self._stop.is_set():
            mhz = float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
            reasons = int(pynvml.nvmlDeviceGetCurrentClocksEventReasons(h))
            self.samples.append((mhz, reasons))
            self._stop.wait(0.005)
        pynvml.nvmlShutdown()

    def start(self) -> None:
        import threading

        try:
            import pynvml  # noqa: F401
        except ImportError:
            return
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._thread.start()

    def stop(self) -> dict:
        if self._thread is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"], "samples": 0}
        self._stop.set()
        self._thread.join(timeout=5)
        names = {self.HW_SLOWDOWN: "hw_slowdown", self.HW_THERMAL: "hw_thermal_slowdown",
                 self.SW_THERMAL: "sw_thermal_slowdown", self.SW_POWER_CAP: "sw_power_cap"}
        seen = sorted({nm for _, r in self.samples for bit, nm in names.items() if r & bit})
        mhz = [m for m, _ in self.samples]
        return {"sm_mhz": float(np.median(mhz)) if mhz else None, "sm_max_mhz": self.max_mhz, "reasons": seen,
                "samples": len(mhz)}


def measured_peak_hbm() -> tuple[float, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(path.read_text())["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


# ---------------------------------------------------------------------------
# engine arm
# ---------------------------------------------------------------------------
def engine_arm(args) -> None:
    import torch
    import torch.distributed as dist

    world = _env_int("WORLD_SIZE", 1)
    rank = _env_int("RANK", 0)
    local = _env_int("LOCAL_RANK", 0)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    from plastax_b200 import StepInputs, make_step
    from plastax_b200.configs import build_reservoir
    from plastax_b200.types import ShardSpec

    cfg = config(args)
    sharding = ShardSpec("conns", world) if world > 1 else None
    net, static, state = build_reservoir(cfg, dev, sharding=sharding, shard_rank=rank)
    torch.cuda.synchronize()
    step = make_step(net, static, device=dev)
    step.mirror_chunk_bits = args.chunk_bits
    W, Kst = max(args.warmup, 3), args.steps
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234)
    inputs_dev = torch.randn((W + 2 * Kst, cfg.num_inputs), generator=gen, device=dev)

    # per-launch time of the dominant kernel (the fused forward + prune sweep),
    # CUDA events on the launching stream around each launch of the timed steps
    fwd_events: list[tuple] = []
    import plastax_b200.kernels as K

    fwd_name = "mirror_forward" if step.use_mirror else "forward_prune"
    orig_fp = getattr(K, fwd_name)

    def timed_forward_prune(*a, **kw):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        orig_fp(*a, **kw)
        e.record()
        fwd_events.append((s, e))

    for i in range(W):
        step(state, StepInputs(inputs_dev[i]))
    torch.cuda.synchronize()
    swept_entries = int(step.mirrors[0].gfill.sum().item()) if step.use_mirror else static.local_capacity(0)
    # eager steps with CUDA events on the launching stream around every launch
    # of the dominant kernel (a graph replay hides per-kernel boundaries)
    setattr(K, fwd_name, timed_forward_prune)
    n_eager = min(Kst, 10)
    for i in range(n_eager):
        step(state, StepInputs(inputs_dev[W + i]))
    torch.cuda.synchronize()
    setattr(K, fwd_name, orig_fp)
    use_graph = step.capturable()
    if use_graph:
        step.capture(state, StepInputs(inputs_dev[0]))
    if world > 1:
        dist.barrier()
    clocks = Clocks(local)
    clocks.start()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0.record()
    for i in range(Kst):
        step(state, StepInputs(inputs_dev[(W + i) % inputs_dev.shape[0]]))
    t1.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    elapsed_ms = t0.elapsed_time(t1)
    fwd_ms = [s.elapsed_time(e) for s, e in fwd_events]

    # e2e: host inputs in pinned memory, H2D inside the region, D2H of the
    # step's overflow flag + grown count
    host_in = torch.randn((Kst, cfg.num_inputs), generator=torch.Generator().manual_seed(7)).pin_memory()
    readback = torch.zeros(2, dtype=torch.int32).pin_memory()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(Kst):
        res = step(state, StepInputs(host_in[i]))
        out = torch.stack([res.grown.to(torch.int32), res.overflow.to(torch.int32)])
        readback.copy_(out, non_blocking=True)
        torch.cuda.current_stream().synchronize()  # the Driver reads the flag every step
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    clk = clocks.stop()

    if world > 1:
        t = torch.tensor([elapsed_ms, e2e_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed_ms, e2e_ms = float(t[0]), float(t[1])
    ms_per_step = elapsed_ms / Kst
    live = cfg.live_edges
    value = live * Kst / (elapsed_ms / 1e3)
    e2e = live * Kst / (e2e_ms / 1e3)

    # roofline of the fused forward + prune sweep: algorithmic bytes per
    # launch = 8 B per swept mirror entry (packed ids + weight; the canonical
    # sweep streams 13 B per slot instead) + 8 B per unit (activation read,
    # accumulator written)
    n = static.num_units
    per_entry = 8 if step.use_mirror else 13
    alg_bytes = per_entry * swept_entries + 8 * n
    fwd_avg_s = float(np.mean(fwd_ms)) / 1e3 if fwd_ms else float("nan")
    achieved = alg_bytes / fwd_avg_s / 1e9
    peak, peak_kind = measured_peak_hbm()
    traffic = NCU_TRAFFIC_BYTES_PER_ENTRY * swept_entries if step.use_mirror else None

    # launches of this library's kernels per step, counted once by the profiler
    launches_per_step = count_launches(step, state, inputs_dev[0], dev)
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": Kst, "warmup": W,
        "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic (seeded reservoir, N(0,1) inputs)", "config": workload_desc(cfg, world),
        "e2e": {"value": e2e, "unit": UNIT, "h2d_bytes_per_step": 4 * cfg.num_inputs, "d2h_bytes_per_step": 8,
                "ms_per_step": e2e_ms / Kst},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": traffic,
                     "kernel": ("mirror_sweep_kernel<sum, abs-below prune> (destination-grouped sweep + fused "
                                "prune)" if step.use_mirror else
                                "forward_vec4_kernel<sum, prune> (canonical sweep + prune)"),
                     "bytes_per_entry": per_entry, "entries_per_launch": swept_entries,
                     "kernel_ms": fwd_avg_s * 1e3, "alg_bytes_per_launch": alg_bytes, "peak_kind": peak_kind,
                     "share_of_step": (fwd_avg_s * 1e3) / ms_per_step},
        "clocks": clk,
        "cuda_graph": use_graph,
        "gpu_launches": launches_per_step * Kst,
    }
    if args.kernel_breakdown:
        kernel_breakdown(step, state, inputs_dev[0], rank)
    # a CUDA graph holding NCCL calls must be released before the process
    # group is destroyed, or the exit waits forever; the peer-memory group is
    # unmapped collectively
    step.close()
    del step
    import gc

    gc.collect()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        del state
        torch.cuda.empty_cache()
        from oracle import oracle as orc

        threads = orc.max_threads()
        times, _ = cpu_run(cfg, args.cpu_steps, 0, threads)
        per = float(np.median(times))
        line["cpu_baseline"] = {
            "value": live / per, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{len(times)} full-size churn steps of the oracle restatement (median) on {threads} host "
                      f"threads (forward+prune, proposals, total order, the claim's free-slot lists; the in-order "
                      f"candidate assignment sequential)",
            "ms_per_step": per * 1e3}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def kernel_breakdown(step, state, x, rank: int, replays: int = 5) -> None:
    """Every kernel's device time per step over `replays` graph replays (or
    eager steps), from the profiler's activity records; rank 0 prints it to
    stderr. Every rank runs the same steps (collectives stay matched)."""
    import collections
    import sys

    import torch
    from torch.profiler import ProfilerActivity, profile

    from plastax_b200 import StepInputs

    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(replays):
            step(state, StepInputs(x))
        torch.cuda.synchronize()
    if rank != 0:
        return
    tot: dict = collections.defaultdict(lambda: [0, 0.0])
    for evt in prof.events():
        if evt.device_type == torch.autograd.DeviceType.CUDA:
            name = evt.name.split("(")[0][:80]
            tot[name][0] += 1
            tot[name][1] += evt.device_time_total
    print(f"kernel breakdown: {replays} steps, device time per step", file=sys.stderr)
    for name, (cnt, us) in sorted(tot.items(), key=lambda kv: -kv[1][1]):
        print(f"  {cnt / replays:5.1f}/step {us / replays:10.1f} us  {name}", file=sys.stderr)


def count_launches(step, state, x, dev) -> int:
    """Kernels of libpxb launched by one step, counted with the profiler: the
    library's own kernels (namespace pxb) and the CUB kernels it instantiates
    (the step calls no torch sort or scan)."""
    import torch
    from torch.profiler import ProfilerActivity, profile

    from plastax_b200 import StepInputs

    names = ("pxb::", "cub::")
    graph, step.graph = step.graph, None  # count an eager step's launches
    try:
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            step(state, StepInputs(x))
            torch.cuda.synchronize()
        n = 0
        for evt in prof.events():
            if evt.device_type == torch.autograd.DeviceType.CUDA and any(k in evt.name for k in names):
                n += 1
        return n
    except Exception:  # profiler unavailable: fall back to the step's own count
        return -1
    finally:
        step.graph = graph


def main() -> None:
    args = parse()
    if args.impl == "reference":
        reference_arm(args)
        return
    engine_arm(args)


if __name__ == "__main__":
    main()
