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
TRAINING = ("esn", "dst", "mlp", "mlp50", "units")
# nominal FP32 (non-tensor) FMA peak of a B200: 148 SMs x 128 lanes x 2 FLOP
# x 1.965 GHz (no measured figure exists for it; stated as nominal)
FP32_NOMINAL_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12
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
    ap.add_argument("--config", default="reservoir", choices=["reservoir", *TRAINING],
                    help="reservoir: the Scheme-A large-reservoir churn step (the headline); esn: the streaming "
                         "echo-state reservoir; dst: dynamic sparse training; mlp / mlp50: the sparse MLP at 10%% "
                         "/ 50%% density, batch 256; units: the unit lifecycle (training configurations run as "
                         "independent replicas when N > 1)")
    ap.add_argument("--units-log2", type=int, default=20, help="reservoir size (2**x units)")
    ap.add_argument("--fan-in", type=int, default=256)
    ap.add_argument("--prune", default="lowest_k", choices=["lowest_k", "threshold"],
                    help="lowest_k: the exact 0.1%% lowest-|w| prune every step (the workload); threshold: the fixed "
                         "|w| < 0.0012533 sigma rule (prunes 0.1%% on the first step only; for profiling the sweep's "
                         "other prune path, the churn check is then skipped)")
    ap.add_argument("--chunk-bits", type=int, default=None,
                    help="mirror destination chunk (2**x units); default: the largest the unit count allows, "
                         "capped at 13 (11 for the full-size reservoir)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-steps", type=int, default=3)
    ap.add_argument("--phase-times", action="store_true",
                    help="add the step's main-stream phases (CUDA events over the eager steps; the phase ends at "
                         "the named boundary) to the line: rank 0's and the max over ranks")
    ap.add_argument("--select-fork", default="auto", choices=["auto", "start", "sweep", "launch", "post"],
                    help="where the next step's growth selection forks onto the side stream: at the step's start, "
                         "after the propagation, from just before the sweep with the sweep launched first "
                         "(launch), or from the sweep's end before its tombstones and the combine (post) "
                         "(auto: at the sweep's end under Scheme-A, at the sweep's launch on one GPU)")
    ap.add_argument("--graph-priority", action="store_true",
                    help="replay the step's graph with the side stream's selection at low priority")
    ap.add_argument("--trace", default=None,
                    help="with --kernel-breakdown: write the replays' kernel timeline as a Chrome trace to this path "
                         "('{rank}' is replaced by the rank)")
    ap.add_argument("--kernel-breakdown", action="store_true",
                    help="after the timing, print (stderr, rank 0) every kernel's device time per step over five "
                         "graph replays, from the profiler's activity records")
    return ap.parse_args()


def config(args):
    from plastax_b200.configs import ReservoirConfig

    return ReservoirConfig(num_units=1 << args.units_log2, fan_in=args.fan_in, prune=args.prune)


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

    def __init__(self, fn, lead_cycles: int = 0) -> None:
        self.fn = fn
        self.events: list[tuple] = []
        self.on = True
        # a spin of this many GPU cycles queued before the start event keeps
        # the GPU busy while the host enqueues the call, so the events time
        # the kernels and not the host's launch gaps
        self.lead_cycles = lead_cycles
        self.slots: list[int] = []

    def __call__(self, *a, **kw):
        import torch

        if not self.on:
            return self.fn(*a, **kw)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if self.lead_cycles:
            torch.cuda._sleep(self.lead_cycles)
        s.record()
        out = self.fn(*a, **kw)
        e.record()
        self.events.append((s, e))
        # the slots the call sweeps: its bucket's capacity (or the fused
        # step's descriptor's)
        a0 = a[0] if a else None
        self.slots.append(int(a0["dead"].numel()) if isinstance(a0, dict) else int(getattr(a0, "cap", 0)))
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
    if args.select_fork != "auto":
        step.select_after_sweep = args.select_fork == "sweep"
        step.select_at_launch = args.select_fork == "launch"
        step.select_post_sweep = args.select_fork == "post"
    step.graph_priority = args.graph_priority
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
    if args.phase_times:
        step.phase_marks = []
    for i in range(n_eager):
        step(state, StepInputs(inputs_dev[W + i]))
    torch.cuda.synchronize()
    phases = step.phase_times() if args.phase_times else None
    step.phase_marks = None
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

    # e2e: host inputs, H2D inside the region, D2H of the step's grown count
    # and overflow flag read by the host every step (as the Driver reads the
    # flag); with a graph both copies are nodes of the step's graph
    # (StepFn.capture(host_io=True)), from and into pinned buffers
    host_in = torch.randn((Kst, cfg.num_inputs), generator=torch.Generator().manual_seed(7)).pin_memory()
    readback = torch.zeros(2, dtype=torch.int32).pin_memory()
    if use_graph:
        step.capture(state, StepInputs(inputs_dev[0]), host_io=True)
        readback = step.host_flags
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
        if not use_graph:
            out = torch.stack([res.grown.to(torch.int32), res.overflow.to(torch.int32)])
            readback.copy_(out, non_blocking=True)
        torch.cuda.current_stream().synchronize()  # the Driver reads the flag every step
        grown_i, over_i = readback.tolist()
        short += grown_i != cfg.k or over_i != 0
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
        if cfg.prune == "lowest_k" and (firings != Kst or pruned != Kst * cfg.k or grown != Kst * cfg.k
                                        or overflowed != 0 or short):
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
    if phases is not None:
        names = sorted(phases)
        vec = torch.tensor([phases[n] for n in names], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(vec, op=dist.ReduceOp.MAX)
        line["phases_ms"] = {"rank0": phases, "max_over_ranks": dict(zip(names, vec.tolist(), strict=True)),
                             "note": "eager steps (launch gaps included), main stream; each phase ends at its "
                                     "named boundary"}
    if args.kernel_breakdown:
        kernel_breakdown(lambda: step(state, StepInputs(inputs_dev[0])), rank, trace=args.trace)
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


def kernel_breakdown(run_step, rank: int, replays: int = 5, trace: str | None = None) -> dict:
    """Every kernel's device time per step over `replays` calls of
    `run_step` (graph replays, or eager steps), from the profiler's activity
    records; rank 0 prints it to stderr and returns {kernel: us per step}.
    Every rank runs the same steps (collectives stay matched)."""
    import collections
    import sys

    import torch
    from torch.profiler import ProfilerActivity, profile

    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(replays):
            run_step()
        torch.cuda.synchronize()
    if trace:
        # every rank's kernel timeline (start, duration, stream) as a Chrome trace
        prof.export_chrome_trace(trace.replace("{rank}", str(rank)))
    if rank != 0:
        return {}
    tot: dict = collections.defaultdict(lambda: [0, 0.0])
    for evt in prof.events():
        if evt.device_type == torch.autograd.DeviceType.CUDA:
            name = evt.name.split("(")[0][:80]
            tot[name][0] += 1
            tot[name][1] += evt.device_time_total
    print(f"kernel breakdown: {replays} steps, device time per step", file=sys.stderr)
    for name, (cnt, us) in sorted(tot.items(), key=lambda kv: -kv[1][1]):
        print(f"  {cnt / replays:5.1f}/step {us / replays:10.1f} us  {name}", file=sys.stderr)
    return {name: us / replays for name, (_, us) in tot.items()}


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


# ---------------------------------------------------------------------------
# the training configurations (one GPU; independent replicas when N > 1)
# ---------------------------------------------------------------------------
def training_case(kind: str, dev, steps: int):
    """The network, state, step and per-step inputs of a training
    configuration, with what its bench line reports; with dev None only the
    inputs and the description (the reference arm builds its own host
    state)."""
    import torch

    from plastax_b200 import configs as C
    from plastax_b200 import make_step

    g = np.random.default_rng(11)
    case: dict = {"kind": kind}
    if kind == "esn":
        cfg = C.C1
        xs = g.standard_normal(steps + cfg.delay).astype(np.float32)
        case.update(x=xs[cfg.delay:, None], t=xs[:-cfg.delay, None], passes=1,
                    desc={"workload": f"streaming echo-state reservoir: {cfg.units} tanh units, fan-in {cfg.fan_in}, "
                                      f"spectral radius {cfg.rho}, 1 input, a linear readout trained by LMS "
                                      f"(lr {cfg.lr}) on the input delayed {cfg.delay} steps",
                          "propagation": "pipeline", "parallelism": "replicas"},
                    bytes_per_slot={"forward": 13, "update": 17})
        if dev is not None:
            from plastax_b200 import Driver

            # streamed through Driver.scan: K steps as one device loop
            net, static, state = C.build_esn(cfg, dev)
            step = Driver(net, static, state, device=dev)
            case["scan"] = True
    elif kind == "dst":
        cfg = C.C3
        w1, w2 = C.dst_teacher(cfg)
        x = g.standard_normal((steps, cfg.num_inputs)).astype(np.float32)
        t = (np.tanh(x @ w1.T) @ w2.T).astype(np.float32)
        case.update(x=x, t=t, passes=2, cfg=cfg,
                    desc={"workload": f"dynamic sparse training: {cfg.num_inputs} inputs + {cfg.hidden} tanh + "
                                      f"{cfg.num_outputs} linear outputs, 2^20 live edges of 2^21, MSE vs a "
                                      f"64-256-8 teacher, SGD lr {cfg.lr}; every {cfg.every} steps the {cfg.k} "
                                      f"lowest-|w| edges pruned and {cfg.k} regrown from {cfg.proposals} "
                                      f"|grad*act|-scored proposals per unit",
                          "propagation": "pipeline", "parallelism": "replicas"},
                    bytes_per_slot={"forward": 13, "backward": 13, "update": 17})
        if dev is not None:
            net, static, state = C.build_dst(cfg, dev)
            step = make_step(net, static, device=dev)
    elif kind in ("mlp", "mlp50"):
        cfg = C.C2 if kind == "mlp" else dataclasses_replace(C.C2, density=0.5)
        xs, ts = zip(*(C.mlp_batch(cfg, g) for _ in range(min(steps, 16))))
        reps = -(-steps // len(xs))
        case.update(x=np.stack(xs * reps)[:steps], t=np.stack(ts * reps)[:steps], passes=2, batch=cfg.batch,
                    desc={"workload": f"sparse MLP 784-1000-1000-10 at density {cfg.density} (batch {cfg.batch}, "
                                      f"N(0,1) images, uniform one-hot labels), ReLU, softmax cross-entropy, SGD "
                                      f"lr {cfg.lr}, exact batch-mean update",
                          "propagation": "topological", "parallelism": "replicas", "global_batch": cfg.batch},
                    bytes_per_slot={"forward": 13, "backward": 13, "update": 17})
        case["cfg"] = cfg
        if dev is not None:
            net, static, state = C.build_mlp(cfg, dev)
            step = make_step(net, static, batch_size=cfg.batch, device=dev)
    elif kind == "units":
        cfg = C.C4
        x = g.standard_normal((steps, cfg.num_inputs)).astype(np.float32)
        t = np.stack([x[i] @ C.units_target_map(cfg, i // cfg.resample) for i in range(steps)])[:, None]
        case.update(x=x, t=t.astype(np.float32), passes=2,
                    desc={"workload": f"unit lifecycle: {cfg.live_units} live of {cfg.unit_capacity} unit slots, "
                                      f"edge capacity 2^{cfg.edge_capacity_log2}, ReLU, UPGD, a utility trace, "
                                      f"every {cfg.interval} steps one spawn and the 1st-percentile units pruned, "
                                      f"{cfg.proposals} deeper proposals per unit",
                          "propagation": "topological", "parallelism": "replicas"},
                    bytes_per_slot={"forward": 13, "backward": 13, "update": 17 + 16})
        if dev is not None:
            from plastax_b200 import Driver

            net, static, state = C.build_units(cfg, dev)
            # the Driver's exactness checks every 10 steps (its check_every),
            # the plain steps replayed from one graph per signature
            step = Driver(net, static, state, device=dev, check_every=cfg.interval, graphs=True)
    else:
        raise ValueError(kind)
    if dev is not None:
        case.update(net=net, static=static, state=state, step=step)
    return case


def dataclasses_replace(obj, **kw):
    import dataclasses

    return dataclasses.replace(obj, **kw)


def _edge_pass_timers():
    """CUDA-event timers around every edge-pass kernel the training steps
    launch (the canonical and batched sweeps and updates)."""
    import plastax_b200.kernels as K

    names = ("forward_accumulate", "forward_prune", "backward_accumulate", "backward_update", "batched_forward",
             "batched_backward", "batched_update", "pipeline_train")
    timers = {}
    for nm in names:
        t = _EventTimer(getattr(K, nm), lead_cycles=200_000)
        t.on = False
        setattr(K, nm, t)
        timers[nm] = t
    return timers


def training_arm(args) -> None:
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
    from plastax_b200 import Driver, StepInputs

    W, Kst = max(args.warmup, 3), args.steps
    timers = _edge_pass_timers()
    case = training_case(args.config, dev, W + 2 * Kst + 16)
    step, state = case["step"], case["state"]
    X = torch.from_numpy(case["x"]).to(dev)
    T = torch.from_numpy(case["t"]).to(dev)
    driver = isinstance(step, Driver)

    def run(i, x, t):
        if driver:
            step.step(StepInputs(x, t))
            return step.last_loss
        return step(state, StepInputs(x, t)).loss

    for i in range(W):
        run(i, X[i], T[i])
    torch.cuda.synchronize()
    # the edge passes' device time, CUDA events on the launching stream, over
    # eager steps (a graph replay hides per-kernel boundaries)
    for t in timers.values():
        t.on = True
    n_eager = min(Kst, 20)
    inner = getattr(step, "_step", None) if driver else None
    if inner is not None and hasattr(inner, "auto_graphs"):
        inner.auto_graphs = False  # the timed steps run eagerly
    timed_steps = 0  # eager steps whose edge passes were timed (a replayed graph's are not)
    for i in range(n_eager):
        before = sum(len(t.events) for t in timers.values())
        run(W + i, X[W + i], T[W + i])
        timed_steps += sum(len(t.events) for t in timers.values()) > before
    torch.cuda.synchronize()
    for t in timers.values():
        t.on = False
    if inner is not None and hasattr(inner, "auto_graphs"):
        inner.auto_graphs = bool(getattr(step, "_graphs", False))
    scan = bool(case.get("scan"))
    use_graph = (not driver) and hasattr(step, "capturable") and step.capturable()
    if scan:
        # the chunk's loop graph is built by a first scan of the same shape
        step.scan(StepInputs(X[W:W + Kst], T[W:W + Kst]))
        torch.cuda.synchronize()
        use_graph = "Driver.scan: the chunk's steps as one device loop"
    elif use_graph:
        step.capture(state, StepInputs(X[0], T[0]))
    elif not driver and hasattr(step, "auto_graphs"):
        # one graph per signature of the periodic phases, each captured at
        # its second occurrence: step through a whole period (twice the
        # longest) before timing so every signature is captured
        step.auto_graphs = True
        for _ in range(step.period() + 2):
            run(0, X[0], T[0])
        torch.cuda.synchronize()
        use_graph = f"one graph per periodic-phase signature ({len(step._graphs)})"
    if world > 1:
        dist.barrier()
    clocks = Clocks(local)
    clocks.start()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    t0.record()
    if scan:
        step.scan(StepInputs(X[W:W + Kst], T[W:W + Kst]))
    else:
        for i in range(Kst):
            run(W + i, X[W + i], T[W + i])
    t1.record()
    torch.cuda.synchronize()
    clocks.pause()
    elapsed_ms = t0.elapsed_time(t1)
    breakdown = None
    if args.kernel_breakdown:
        # the same replays' kernels, warm, from the profiler's activity records
        breakdown = kernel_breakdown(lambda: run(0, X[0], T[0]), rank, replays=20, trace=args.trace)
    # e2e: each step's inputs and targets from pinned host memory, the loss
    # read back every step
    hx = torch.from_numpy(case["x"][W + Kst:W + 2 * Kst]).pin_memory()
    ht = torch.from_numpy(case["t"][W + Kst:W + 2 * Kst]).pin_memory()
    back = torch.zeros(1, dtype=torch.float32).pin_memory()
    if world > 1:
        dist.barrier()
    clocks.resume()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(Kst):
        loss = run(i, hx[i].to(dev, non_blocking=True), ht[i].to(dev, non_blocking=True))
        back.copy_(loss.reshape(1), non_blocking=True)
        torch.cuda.current_stream().synchronize()
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    clk = clocks.stop()
    if world > 1:
        tt = torch.tensor([elapsed_ms, e2e_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        elapsed_ms, e2e_ms = float(tt[0]), float(tt[1])
    st = case["state"] if not driver else step.state
    live = sum(int((b["dead"] == 0).sum()) for b in st.conns)
    caps = sum(int(b["dead"].numel()) for b in st.conns)
    batch = case.get("batch", 1)
    per_step = live * case["passes"] * batch
    value = world * per_step * Kst / (elapsed_ms / 1e3)
    e2e = world * per_step * Kst / (e2e_ms / 1e3)
    # the edge passes' roofline: algorithmic bytes over every slot of the
    # swept buckets (the reference's passes read capacity), per pass kind
    bps = case["bytes_per_slot"]
    pass_bytes = {"forward_accumulate": bps.get("forward", 13), "forward_prune": bps.get("forward", 13),
                  "backward_accumulate": bps.get("backward", 13), "backward_update": bps.get("update", 17),
                  "batched_forward": bps.get("forward", 13), "batched_backward": bps.get("backward", 13),
                  "batched_update": bps.get("update", 17),
                  # the fused pipeline step: one read of every slot feeds both
                  # sums, a second read and the weight write the update
                  "pipeline_train": 13 + bps.get("update", 17)}
    ms_total, bytes_total, launches = 0.0, 0, 0
    for nm, t in timers.items():
        ms = t.ms()
        if not ms:
            continue
        ms_total += float(np.sum(ms))
        launches += len(ms)
    # bytes per eager step: every bucket swept once per pass kind present
    kinds = [nm for nm, t in timers.items() if t.events]
    # the fused pipeline step reads only the slots below a PIPELINE arena's
    # tail (the rest were never claimed); the separate passes read capacity
    swept = caps
    if st.tail_start is not None and "pipeline_train" in kinds:
        swept = min(caps, int(st.tail_start.item()))
    # every timed call's algorithmic bytes over the slots it swept (calls
    # replayed inside a graph are not timed and not counted)
    for nm in kinds:
        for sl in timers[nm].slots:
            bytes_total += pass_bytes[nm] * (min(sl, swept) if nm == "pipeline_train" else sl)
    achieved = bytes_total / (ms_total / 1e3) / 1e9 if ms_total else float("nan")
    timed_steps = max(1, timed_steps)
    peak, peak_kind = measured_peak_hbm()
    roof = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
            "traffic": None, "kernel": "edge passes (" + ", ".join(kinds) + ")",
            "alg_bytes_per_step": bytes_total / timed_steps, "kernel_ms_per_step": ms_total / timed_steps,
            "share_of_step": (ms_total / timed_steps) / (elapsed_ms / Kst), "peak_kind": peak_kind,
            "timed_eager_steps": timed_steps,
            "arena_slots": caps, "swept_slots": swept, "l2_resident": caps * 13 < 126e6,
            # the same step as the reference's separate passes over capacity
            "reference_pass_bytes_per_step": caps * sum(bps.values())}
    if batch > 1:
        flops = 3 * 2 * batch * live  # forward, backward and update products per edge per sample
        tf = flops / ((ms_total / timed_steps) / 1e3) / 1e12
        roof["fp32"] = {"achieved_tflops": tf, "peak_tflops": FP32_NOMINAL_TFLOPS, "peak_kind": "nominal",
                        "frac": tf / FP32_NOMINAL_TFLOPS, "flops_per_step": flops}
    line = {
        "metric": f"propagated edges/sec per step ({case['desc']['workload'].split(':')[0]})",
        "value": value, "unit": "edges/s", "n_gpus": world, "steps": Kst, "warmup": W,
        "ms_per_step": elapsed_ms / Kst, "us_per_step": 1e3 * elapsed_ms / Kst, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded network and inputs)",
        "config": {**case["desc"], "live_edges": live, "edge_passes_per_step": case["passes"] * batch,
                   "l2": "arena smaller than L2 (126 MB): every pass after the first reads L2"
                   if roof["l2_resident"] else "arena larger than L2"},
        "e2e": {"value": e2e, "unit": "edges/s", "h2d_bytes_per_step": int(hx[0].numel() * 4 + ht[0].numel() * 4),
                "d2h_bytes_per_step": 4, "ms_per_step": e2e_ms / Kst},
        "roofline": roof, "clocks": clk, "cuda_graph": use_graph,
    }
    if breakdown:
        line["kernels_us_per_step"] = {k: round(v, 2) for k, v in sorted(breakdown.items(), key=lambda kv: -kv[1])}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = training_cpu_baseline(args.config, case, max(1, args.cpu_steps))
    if rank == 0:
        print(json.dumps(line), flush=True)
    if driver:
        step.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def training_cpu_baseline(kind: str, case: dict, steps: int) -> dict:
    """The oracle's step of the same configuration on the host, a bounded
    sample of steps (median), from the state the engine started from."""
    import math

    from plastax_b200 import configs as C

    batch = case.get("batch", 1)
    times = []
    threads = host_threads()
    if kind == "esn":
        from oracle.steps import EsnOracle

        cfg = C.C1
        src, dst, w = C.esn_edges(cfg)
        net, static, state = C.build_esn(cfg, "cpu")
        b = {k: v.numpy().copy() for k, v in state.conns[0].items()}
        ro = EsnOracle(b, state.units["activation"].numpy().copy(), input_id=0, output_id=cfg.units + 1, lr=cfg.lr)
        n_steps = max(steps, 200)
        for i in range(n_steps):
            t0 = time.perf_counter()
            ro.step(float(case["x"][i, 0]), float(case["t"][i, 0]))
            times.append(time.perf_counter() - t0)
        live, sample, cores = int((b["dead"] == 0).sum()), f"{n_steps} ESN steps of the oracle restatement", 1
    elif kind == "dst":
        from oracle.steps import DstOracle

        cfg = case["cfg"]
        net, static, state = C.build_dst(cfg, "cpu")
        b = {k: v.numpy().copy() for k, v in state.conns[0].items()}
        u = {k: v.numpy().copy() for k, v in state.units.items()}
        ro = DstOracle(b, u["activation"], u["grad_pre_act"], u["level"], int(state.tail_start.item()),
                       num_inputs=cfg.num_inputs, num_outputs=cfg.num_outputs, lr=cfg.lr, k=cfg.k, every=cfg.every,
                       proposals=cfg.proposals, seed=cfg.seed, threads=threads)
        n_steps = max(steps, 25)
        for i in range(n_steps):
            t0 = time.perf_counter()
            ro.step(case["x"][i], case["t"][i])
            times.append(time.perf_counter() - t0)
        # the structural step every `every` steps, weighed in at its rate
        struct = times[0]
        plain = float(np.median(times[1:]))
        per = plain + (struct - plain) / cfg.every
        live = int((b["dead"] == 0).sum())
        sample = (f"{n_steps} DST steps of the oracle restatement (the forward, backward and update single-threaded, "
                  f"the structural phase on {threads} threads): median plain step plus the first (structural) "
                  f"step's excess spread over {cfg.every} steps")
        line = {"value": live * 2 / per, "unit": "edges/s", "cores": threads, "kind": "port", "sample": sample,
                "ms_per_step": per * 1e3}
        return line
    elif kind in ("mlp", "mlp50"):
        from oracle.batched import batched_step

        net, static, state_h = C.build_mlp(case["cfg"], "cpu")
        buckets = [{k: v.numpy().copy() for k, v in bk.items()} for bk in state_h.conns]
        level = state_h.units["level"].numpy()
        is_input = np.zeros(level.size, np.uint8)
        is_input[list(static.input_ids)] = 1
        n_steps = max(1, min(steps, 3))
        for i in range(n_steps):
            t0 = time.perf_counter()
            batched_step(buckets, level, is_input, static.input_ids, static.output_ids, case["x"][i], case["t"][i],
                         fwd_act="relu", bwd_act="relu", loss="softmax", opt=dict(kind="sgd", lr=0.01),
                         out_act="identity")
            times.append(time.perf_counter() - t0)
        live = sum(int((bk["dead"] == 0).sum()) for bk in buckets)
        sample, cores = f"{n_steps} batched steps of the numpy restatement (batch {batch})", 1
    elif kind == "units":
        from oracle.steps import UnitsOracle

        cfg = C.C4
        net, static, state = C.build_units(cfg, "cpu")
        buckets = [{k: v.numpy().copy() for k, v in bk.items()} for bk in state.conns]
        units = {k: v.numpy().copy() for k, v in state.units.items()}
        ro = UnitsOracle(buckets, units, input_ids=static.input_ids, output_ids=static.output_ids,
                         num_levels=static.num_levels, net=net)
        n_steps = max(steps, 11)
        for i in range(n_steps):
            t0 = time.perf_counter()
            ro.step(case["x"][i], case["t"][i])
            times.append(time.perf_counter() - t0)
        # the structural step (a unit spawned) every `interval` steps, weighed in at its rate
        plain = float(np.median([tt for i, tt in enumerate(times) if i % cfg.interval]))
        struct = float(np.mean([tt for i, tt in enumerate(times) if i % cfg.interval == 0]))
        per_step = plain + (struct - plain) / cfg.interval
        live = sum(int((bk["dead"] == 0).sum()) for bk in buckets)
        sample = (f"{n_steps} unit-lifecycle steps of the oracle restatement, single-threaded (UPGD's scale, the "
                  f"forward and backward level by level, the trace, UPGD, the quantile prune, the spawn every "
                  f"{cfg.interval} steps; the regrowth not included): median plain step plus the spawn steps' "
                  f"excess spread over {cfg.interval} steps")
        return {"value": live * case["passes"] / per_step, "unit": "edges/s", "cores": 1, "kind": "port",
                "sample": sample, "ms_per_step": per_step * 1e3}
    else:
        raise ValueError(kind)
    per = float(np.median(times))
    return {"value": live * case["passes"] * batch / per, "unit": "edges/s", "cores": cores, "kind": "port",
            "sample": sample, "ms_per_step": per * 1e3}


def training_reference_arm(args) -> None:
    rank = _env_int("RANK", 0)
    if rank != 0:
        return
    case = training_case(args.config, None, max(args.steps, 200) + 32)
    base = training_cpu_baseline(args.config, case, max(1, args.cpu_steps))
    line = {"impl": "reference", "metric": f"propagated edges/sec per step "
                                           f"({case['desc']['workload'].split(':')[0]})",
            "value": base["value"], "unit": "edges/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": 0,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded network and inputs)", "config": case["desc"], "cpu_baseline": base,
            "e2e": {"value": base["value"], "unit": "edges/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main() -> None:
    args = parse()
    if args.config != "reservoir":
        (training_reference_arm if args.impl == "reference" else training_arm)(args)
        return
    if args.impl == "reference":
        reference_arm(args)
        return
    engine_arm(args)


if __name__ == "__main__":
    main()
