"""Benchmark: propagated edges/sec of the Scheme-A large-reservoir churn step.

Workload (the large-reservoir churn configuration the metric's 1/2/4/8-GPU
figures are quoted on): 1,048,576 tanh units + 16 inputs, fan-in 256
(268,435,456 recurrent + 16,777,216 input edges, one PIPELINE bucket), one
step = forward propagation of every live edge with the exact 0.1% lowest-|w|
prune fused in (k = 268,435 edges, ties by slot), the tanh apply, per-unit
Philox proposals, the total-order selection of k winners and the pipeline
slot claim: k edges leave and k enter every step, so the live-edge count
is constant. The line's `churn` object holds the device-counted pruned,
grown and overflowed totals of the timed steps, and the run fails unless
every timed step pruned and grew exactly k.
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
    ap.add_argument("--steps", type=int, default=200)
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
        "workload": f"scheme_a_reservoir_churn: 2^{cfg.num_units.bit_length() - 1} tanh units + {cfg.num_inputs} "
                    f"inputs, fan-in {cfg.fan_in}, exact {cfg.churn:.1%} lowest-|w| prune + per-unit proposal "
                    f"regrowth every step",
        "units": cfg.num_units + cfg.num_inputs,
        "fan_in": cfg.fan_in,
        "live_edges": cfg.live_edges,
        "churn_per_step": cfg.k,
        "prune": "lowest_k (exact, ties by slot)" if cfg.prune == "lowest_k" else f"|w| < {cfg.tau:.4g}",
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
                         k=cfg.k, init_a=cfg.sigma * math.sqrt(3.0), seed=cfg.seed, threads=threads,
                         prune=cfg.prune)
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


def host_threads() -> int:
    """Every host core this process may run on (whatever OMP_NUM_THREADS a
    launcher exported: torchrun sets it to 1)."""
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except AttributeError:
        return max(1, os.cpu_count() or 1)


def reference_arm(args) -> None:
    rank = _env_int("RANK", 0)
    if rank != 0:
        return
    cfg = config(args)
    threads = host_threads()
    steps = max(1, min(args.steps, 5))
    warmup = min(args.warmup, 1)
    times, live = cpu_run(cfg, steps, warmup, threads)
    per_step = float(np.median(times))
    value = live / per_step
    sample = (f"{steps} timed full-size churn steps (median) after {warmup} warm-up, of the "
              f"{args.steps} requested, each pruning and regrowing k = {cfg.k} edges: the oracle restatement of "
              f"the reference's step on {threads} host threads (forward, the exact lowest-|w| prune, proposals, "
              f"total order, the claim's free-slot lists; the in-order candidate assignment sequential)")
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
    in a background thread while the timed regions run (reads only).
    `start()` returns once the first sample is taken, so a short timed
    region is covered; `pause()` / `resume()` bracket the untimed work
    between two timed regions."""

    HW_SLOWDOWN, HW_THERMAL, SW_THERMAL, SW_POWER_CAP = 0x8, 0x40, 0x20, 0x4

    def __init__(self, index: int) -> None:
        import threading

        self.index = index
        self.samples: list[tuple[float, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._ready = threading.Event()
        self._on = threading.Event()
        self._thread = None
        self.error = None

    def _run(self) -> None:
        try:
            import pynvml

            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
        except Exception as e:  # noqa: BLE001 -- reported in the line
            self.error = f"nvml: {e}"
            self._ready.set()
            return
        first = True
        while not self._stop.is_set():
            if self._on.is_set():
                mhz = float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
                reasons = int(pynvml.nvmlDeviceGetCurrentClocksEventReasons(h))
                self.samples.append((mhz, reasons))
                if first:
                    self._ready.set()
                    first = False
            self._stop.wait(0.005)
        pynvml.nvmlShutdown()

    def start(self) -> None:
        import threading

        self._on.set()
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._thread.start()
        self._ready.wait(timeout=30)

    def pause(self) -> None:
        self._on.clear()

    def resume(self) -> None:
        self._on.set()

    def stop(self) -> dict:
        if self._thread is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["sampler not started"], "samples": 0}
        self._stop.set()
        self._thread.join(timeout=5)
        names = {self.HW_SLOWDOWN: "hw_slowdown", self.HW_THERMAL: "hw_thermal_slowdown",
                 self.SW_THERMAL: "sw_thermal_slowdown", self.SW_POWER_CAP: "sw_power_cap"}
        seen = sorted({nm for _, r in self.samples for bit, nm in names.items() if r & bit})
        if self.error:
            seen.append(self.error)
        mhz = [m for m, _ in self.samples]
        return {"sm_mhz": float(np.median(mhz)) if mhz else None, "sm_max_mhz": self.max_mhz, "reasons": seen,
                "samples": len(mhz)}


def measured_peak_hbm() -> tuple[float, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(path.read_text())["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


class _EventTimer:
    """CUDA events around every call of a wrapped function, on the stream
    it launches on (torch's current stream)."""

    def __init__(self, fn) -> None:
        self.fn = fn
        self.events: list[tuple] = []
        self.on = True

    def __call__(self, *a, **kw):
        import torch

        if not self.on:
            return self.fn(*a, **kw)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        out = self.fn(*a, **kw)
        e.record()
        self.events.append((s, e))
        return out

    def ms(self) -> list[float]:
        return [s.elapsed_time(e) for s, e in self.events]


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

    for i in range(W):
        step(state, StepInputs(inputs_dev[i]))
    torch.cuda.synchronize()
    if not step.check_status():
        raise RuntimeError("bench: a mirror lost an edge during the warm-up")
    swept_entries = int(step.mirrors[0].gfill.sum().item()) if step.use_mirror else static.local_capacity(0)
    # eager steps with CUDA events on the launching stream around every launch
    # of the dominant kernel (the fused forward + prune sweep) and of the
    # mirror's upkeep (the claim's inserts); a graph replay hides per-kernel
    # boundaries
    import plastax_b200.kernels as K

    if step.lowk is not None:
        sweep_t = _EventTimer(step.lowk.sweep)
        step.lowk.sweep = sweep_t
        sel_t = _EventTimer(step.lowk.select)
        step.lowk.select = sel_t
    else:
        fwd_name = "mirror_forward" if step.use_mirror else "forward_prune"
        sweep_t = _EventTimer(getattr(K, fwd_name))
        setattr(K, fwd_name, sweep_t)
        sel_t = None
    ins_t = _EventTimer(K.mirror_insert)
    K.mirror_insert = ins_t
    n_eager = min(Kst, 10)
    for i in range(n_eager):
        step(state, StepInputs(inputs_dev[W + i]))
    torch.cuda.synchronize()
    sweep_t.on = ins_t.on = False
    if sel_t is not None:
        sel_t.on = False
    use_graph = step.capturable()
    if use_graph:
        step.capture(state, StepInputs(inputs_dev[0]))
    if world > 1:
        dist.barrier()
    clocks = Clocks(local)
    clocks.start()
    totals0 = step.lowk.totals.clone() if step.lowk is not None else None
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
    clocks.pause()
    if world > 1:
        dist.barrier()
    elapsed_ms = t0.elapsed_time(t1)
    churn_dev = (step.lowk.totals - totals0) if step.lowk is not None else None

    # e2e: host inputs in pinned memory, H2D inside the region, D2H of the
    # step's overflow flag + grown count
    host_in = torch.randn((Kst, cfg.num_inputs), generator=torch.Generator().manual_seed(7)).pin_memory()
    readback = torch.zeros(2, dtype=torch.int32).pin_memory()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks.resume()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    short = 0
    for i in range(Kst):
        res = step(state, StepInputs(host_in[i]))
        out = torch.stack([res.grown.to(torch.int32), res.overflow.to(torch.int32)])
        readback.copy_(out, non_blocking=True)
        torch.cuda.current_stream().synchronize()  # the Driver reads the flag every step
        short += int(readback[0]) != cfg.k or int(readback[1]) != 0
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    clk = clocks.stop()
    step.check_status()  # raises on any device fault bit

    # churn over the timed steps, device-counted (pruned summed over ranks)
    churn = None
    if churn_dev is not None:
        if world > 1:
            dist.all_reduce(churn_dev[:1], op=dist.ReduceOp.SUM)
        pruned, grown, overflowed, firings = (int(v) for v in churn_dev.cpu().tolist())
        churn = {"steps": firings, "pruned": pruned, "grown": grown, "overflowed": overflowed,
                 "k_per_step": cfg.k, "e2e_steps_short_of_k": short}
        if firings != Kst or pruned != Kst * cfg.k or grown != Kst * cfg.k or overflowed != 0 or short:
            raise RuntimeError(f"bench: the timed steps did not churn k = {cfg.k} edges each: {churn}")

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
    fwd_ms = sweep_t.ms()
    fwd_avg_s = float(np.mean(fwd_ms)) / 1e3 if fwd_ms else float("nan")
    achieved = alg_bytes / fwd_avg_s / 1e9
    peak, peak_kind = measured_peak_hbm()
    traffic = NCU_TRAFFIC_BYTES_PER_ENTRY * swept_entries if step.use_mirror else None
    # the same launch against the canonical arena's 13 B per live slot (the
    # bytes a sweep of the canonical columns would stream for these edges)
    canon_bytes = 13 * (live // world) + 8 * n
    ins_ms = float(np.mean(ins_t.ms())) if ins_t.events else None
    sel_ms = float(np.mean(sel_t.ms())) if sel_t is not None and sel_t.events else None

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
                     "kernel": ("mirror_sweep_kernel<sum, lowest-k prune> (destination-grouped sweep + fused exact "
                                "prune)" if step.lowk is not None else
                                "mirror_sweep_kernel<sum, abs-below prune>" if step.use_mirror else
                                "forward_vec4_kernel<sum, prune> (canonical sweep + prune)"),
                     "bytes_per_entry": per_entry, "entries_per_launch": swept_entries,
                     "kernel_ms": fwd_avg_s * 1e3, "alg_bytes_per_launch": alg_bytes, "peak_kind": peak_kind,
                     "share_of_step": (fwd_avg_s * 1e3) / ms_per_step,
                     "canonical_13B_per_slot": {"bytes": canon_bytes,
                                                "achieved": canon_bytes / fwd_avg_s / 1e9,
                                                "frac": canon_bytes / fwd_avg_s / 1e9 / peak},
                     "upkeep_ms": {"mirror_insert": ins_ms, "lowk_select": sel_ms}},
        "churn": churn,
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
        threads = host_threads()
        times, _ = cpu_run(cfg, args.cpu_steps, 0, threads)
        per = float(np.median(times))
        line["cpu_baseline"] = {
            "value": live / per, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{len(times)} full-size churn steps of the oracle restatement (median), each pruning and "
                      f"regrowing k = {cfg.k} edges, on {threads} host threads (forward, the exact lowest-|w| "
                      f"prune, proposals, total order, the claim's free-slot lists; the in-order candidate "
                      f"assignment sequential)",
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
