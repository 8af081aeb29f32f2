"""Step assembly (mirrors src/plastax/step.py:45-356 and the phase order of
src/plastax/phases.py:87-176).

`make_step(net, static)` returns a StepFn: `step(state, inputs) ->
StepResult(state, overflow, loss, growth_remainder, grown)`. As in the
reference (jit with donate_argnums=0) the state's buffers pass to the step:
it updates them in place on the device and returns the same state object.
All buffers a step needs (accumulators, candidate lists, sort and claim
scratch) are allocated once when the StepFn is built; a step allocates
nothing on the device and never synchronises with the host unless the
growth rule declares `on_overflow = "error"`.

Phase order: forward, loss, backward, update_unit, update_conn, prune_unit,
prune_conn, add_unit (every structural_interval steps), add_conn. Fusions,
each legal only where it cannot change a result:
- prune into forward (src/plastax/phases.py:1629-1700, plan_prune_fusion):
  a MagnitudePrune reads only the weight, so it rides on the forward's read
  of every slot when no update_conn writes weights in between;
- update_conn into backward (TOPOLOGICAL): bucket l's destinations are all
  finalized before bucket l is swept in the reverse walk, so each slot's
  optimizer step uses the same grad[dst] the separate update pass would.
Scheme-A: each rank sweeps its capacity band; the per-unit partials are
all-reduced with NCCL (the monoid's collective, src/plastax/monoid.py:175)
before every apply, and the claim all-gathers the per-domain free counts.
"""

from __future__ import annotations

import ctypes
import dataclasses
import os
from typing import Any

import numpy as np
import torch

from plastax_b200 import _lib
from plastax_b200 import kernels as K
from plastax_b200.state import NetworkState, NetworkStatic
from plastax_b200.traits import (
    DestinationThresholdPrune,
    MagnitudePrune,
    MSELoss,
    Network,
    AffineUnitUpdate,
    LowestMagnitudePrune,
    ProposeAddConn,
    ScoreAddConn,
    SoftmaxCrossEntropyLoss,
)
from plastax_b200.types import ACTIVATION, LEVEL, PRUNED, Propagation


# the largest in-degree for which the mirror's fixed-point sum stays within
# 1e-6 of the exact sum of its float32 products in every case (each product
# below 2^-7 is rounded to 2^-31, an error of at most 2^-32)
FIXED_EXACT_FAN_IN = int(1e-6 * 2 ** 32)


@dataclasses.dataclass(frozen=True)
class StepInputs:
    """Clamped inputs + targets for one step (src/plastax/phases.py:68-83).
    Host (numpy) or device tensors; host values are copied to the device."""

    inputs: Any
    targets: Any = None


@dataclasses.dataclass
class GrowthRemainder:
    """The claim's inputs and which candidates it dropped
    (src/plastax/phases.py:2799-2820), for a growth-only retry."""

    src: torch.Tensor
    dst: torch.Tensor
    weight: torch.Tensor
    dropped: torch.Tensor


@dataclasses.dataclass
class StepResult:
    """src/plastax/step.py:45-67. `overflow`, `grown` and `loss` are device
    scalars; reading them on the host synchronises."""

    state: NetworkState
    overflow: torch.Tensor
    loss: torch.Tensor
    growth_remainder: GrowthRemainder | None
    grown: torch.Tensor


def _dist():
    import torch.distributed as dist

    return dist


class StepFn:
    """A built step: preallocated buffers plus the phase sequence."""

    def __init__(self, net: type[Network], static: NetworkStatic, device: torch.device,
                 fuse_prune: bool = True, fuse_train: bool = True) -> None:
        self.net, self.static, self.dev = net, static, device
        n = static.num_units
        fp = net.forward_pass
        self.pipeline = static.propagation is Propagation.PIPELINE
        self.num_buckets = len(static.level_capacities)
        self.fwd_monoid = fp.combine.lowered()
        self.fwd_identity = fp.combine.identity
        self.acc = torch.empty(n, dtype=torch.float32, device=device)
        self.input_ids = torch.tensor(static.input_ids, dtype=torch.int64, device=device)
        self.output_ids = torch.tensor(static.output_ids, dtype=torch.int32, device=device)
        # unit roles for the applies: 1 input (skipped), 2 output (its own
        # activation when the passes declare one), 0 hidden
        fp, bp = net.forward_pass, net.backward_pass
        out_fwd = fp.output_activation
        out_bwd = None if bp is None else (bp.output_activation or out_fwd)
        self.fwd_act = fp.activation if out_fwd is None else (fp.activation, out_fwd)
        self.bwd_act = None if bp is None else (bp.activation if out_bwd is None else (bp.activation, out_bwd))
        is_input = np.zeros(n, np.uint8)
        if out_fwd is not None or out_bwd is not None:
            is_input[list(static.output_ids)] = 2
        is_input[list(static.input_ids)] = 1
        self.is_input = torch.from_numpy(is_input).to(device)
        # the pipeline backward applies to every unit, inputs included
        # (src/plastax/sweep.py:402-450), so its roles mark only the outputs
        self.bwd_roles = None
        if out_bwd is not None:
            self.bwd_roles = torch.from_numpy(np.where(is_input == 1, 0, is_input).astype(np.uint8)).to(device)
        self.loss_buf = torch.zeros(1, dtype=torch.float32, device=device)
        self.loss_b1 = torch.zeros(1, dtype=torch.float32, device=device)
        self.sharded = static.sharding is not None and static.num_shards > 1
        self.reduce_op = fp.combine.torch_reduce_op() if self.sharded else None
        # fusion legality: a prune that reads only weights rides on the
        # forward's read of every edge when no update_conn rewrites them; the
        # exact lowest-|w| prune does so on a one-bucket mirror
        pc = net.prune_conn
        self.lowk_prune = (fuse_prune and isinstance(pc, LowestMagnitudePrune) and net.update_conn is None
                           and net.prune_unit is None and self.num_buckets == 1)
        self.fuse_prune = fuse_prune and (isinstance(pc, MagnitudePrune) or self.lowk_prune) \
            and net.update_conn is None
        self.lowk = None
        self._lowk_fired = False
        # CUDA events at the phase boundaries of eager steps, when a caller
        # sets a list here (a profiling aid: `phase_times()` reads them)
        self.phase_marks: list | None = None
        self.fuse_update = (not self.pipeline and net.update_conn is not None and net.backward_pass is not None
                            and net.update_unit is None)
        self.opt = net.update_conn.struct() if net.update_conn is not None else None
        self.opt_cols = net.update_conn.cols if net.update_conn is not None else K.OPT_COLS
        # UPGD: the utility scale per destination unit, in the state's column
        self.upgd_local = net.update_conn is not None and net.update_conn.kind == "upgd" \
            and net.update_conn.eta == "local"
        self.ac: ProposeAddConn | ScoreAddConn | None = net.add_conn
        self.is_score = isinstance(self.ac, ScoreAddConn)
        # The forward reads a destination-grouped mirror of each bucket when
        # no phase rewrites weights in place (the mirror holds its own copy)
        # and any prune rides on the forward sweep.
        self.use_mirror = (net.update_conn is None and (net.prune_conn is None or self.fuse_prune)
                           and net.prune_unit is None)  # unit pruning tombstones edges outside the sweep
        self.mirrors: list | None = None
        self.mirror_chunk_bits: int | None = None  # destination chunk of the mirror (None: the largest allowed)
        # spare entries per mirror group for growth inserts (fraction, minimum)
        self.mirror_slack, self.mirror_min_slack = 0.05, 64
        self.bitmaps: list[torch.Tensor] | None = None
        # the mirror's sum is exact fixed point (int64 accumulators beside
        # the float side for non-finite or huge products)
        self.acc_fixed = (torch.zeros(n, dtype=torch.int64, device=device)
                          if self.use_mirror and self.fwd_monoid == "sum" else None)
        # Scheme-A over several buckets: each bucket's forward partial is
        # reduced alone, then combined into the carried accumulator
        # (src/plastax/sweep.py:157-175, monoid.py:175-204)
        self.per_bucket_reduce = self.sharded and self.num_buckets > 1
        # the pipeline sweep's Scheme-A combine + apply as one kernel over
        # NVLink peer memory (the group is built at the first bind)
        self.peers = None
        self._counts_on_barrier = False
        self.level_before = self.level_totals = None
        self.peer_reduce = (self.sharded and self.pipeline and self.acc_fixed is not None
                            and torch.device(device).type == "cuda"
                            and os.environ.get("PLASTAX_B200_PEER_REDUCE", "1") != "0")
        if self.per_bucket_reduce:
            self.part = torch.empty(n, dtype=torch.float32, device=device)
            self.part_fixed = None if self.acc_fixed is None else torch.zeros_like(self.acc_fixed)
        self._bound: int | None = None
        self.step_dev = torch.zeros(1, dtype=torch.int32, device=device)
        self.graph = None  # a captured CUDA graph of the step body (see capture)
        self._host_io = False  # the graph copies the step's host inputs and flags (see capture)
        self._io_src = None  # while capturing a host-I/O graph: the staging buffer's device address
        self.graph_priority = False  # capture main / side streams at high / low priority (see capture)
        self._graph_exec = None
        # with auto_graphs, steps whose work depends on periodic phases replay
        # one captured graph per signature (see _replay_or_capture)
        self.auto_graphs = False
        self._graphs: dict = {}
        self._sig_seen: dict = {}
        self._clear_flags = False  # the step claimed nothing: its end clears grown / overflow
        self.side = None
        self.unit_lifecycle = net.prune_unit is not None or net.add_unit is not None
        if isinstance(net.prune_conn, LowestMagnitudePrune) and self.sharded and not (
                self.lowk_prune and self.peer_reduce):
            raise NotImplementedError("the lowest-|w| prune under Scheme-A is lowered for a one-bucket PIPELINE "
                                      "arena swept through its mirror (sum combine over peer memory) only")
        if self.unit_lifecycle and self.sharded:
            raise NotImplementedError("the unit lifecycle under Scheme-A has no lowering (single device only, as in "
                                      "the reference)")
        if net.add_unit is not None and self.pipeline:
            raise NotImplementedError("add_unit on a PIPELINE net has no engine lowering (its claim domains are the "
                                      "static levels)")
        if self.ac is not None:
            self._build_growth()
            # proposals scored by the site RNG alone depend on the levels and
            # the step counter only, never on this step's propagation, prune
            # or update: their selection may overlap the forward sweep (not
            # per-connection proposals, which come from the post-prune arena)
            if (not self.is_score and not self.unit_lifecycle and self.ac.score in ("uniform", "uniform_q256")
                    and not self.ac.dedupe_live
                    and self.ac.proposer != "per_connection" and torch.device(device).type == "cuda"):
                self.side = torch.cuda.Stream(device=device)
        # ... and, when growth fires every step, the next step's selection
        # runs a whole step ahead, beside this step's passes and claim
        self.ahead = self.side is not None and self.capturable() and self.ac is not None and self.k > 0
        self._ahead_ready = False
        # where the next step's selection forks from the step (see _body_ahead):
        # after the propagation under Scheme-A, where the sweep is short and
        # the latency-bound claim leaves SMs idle; on one GPU from just
        # before the sweep, captured after its launch, so the sweep takes the
        # SMs first and the selection fills them as its CTAs retire (forked
        # at the step's start, the proposals held the SMs the sweep waited for)
        self.select_after_sweep = self.sharded
        self.select_at_launch = not self.sharded
        self._sweep_fork = None
        # under Scheme-A from the lowest-|w| sweep's end, before its tombstones
        # and the combine: the selection then overlaps the latency-bound
        # combine and ends before the claim (forked after the propagation it
        # outlasted the step by ~10 us at N=2)
        self.select_post_sweep = self.sharded
        self._post_fork = None
        # work that needs every rank's combine but not the threshold bin's
        # selection (the list take) runs beside that one-CTA selection
        self._after_combine = None
        self._take_pending = False
        # with the prune and growth firing every step, the next step's plan
        # of the lowest-|w| prune is made right after this step's claim, on
        # its own stream beside the mirror insert (it reads the histograms
        # the claim's committed edges update, nothing the insert writes)
        pc = net.prune_conn
        self.plan_ahead = bool(self.lowk_prune and pc.every <= 1 and self.ac is not None and self.k > 0
                               and self.capturable() and torch.device(device).type == "cuda")
        self.plan_stream = torch.cuda.Stream(device=device) if self.plan_ahead else None
        self._plan_ready = False
        self._plan_pending = False
        # on one GPU with propagation only, the sweep's deferred tombstones
        # are written on their own stream beside the apply and the threshold
        # bin's selection: they touch other slots and mirror entries, and
        # the prune phase waits for them before anything reads the arena
        self.flush_split = bool(self.lowk_prune and not self.sharded and net.backward_pass is None
                                and net.update_conn is None and not self.unit_lifecycle
                                and torch.device(device).type == "cuda")
        self.flush_stream = torch.cuda.Stream(device=device) if self.flush_split else None
        self._flush_pending = False
        self._init_train_fused(fuse_train)
        # under Scheme-A the selection a step ahead is shared out: each rank
        # ranks its share of the full bins into every rank's winner columns
        # (peer memory, bound with the group), which the next step reads
        # after its combine's barrier; three lists, so a rank selecting step
        # t + 1's never overwrites one a slower peer has yet to take
        self.shard_select = bool(self.ahead and self.sharded and self.fast_select and self.peer_reduce
                                 and not self.train_fused and static.num_shards <= _lib.SELECT_MAX_WORLD)
        # on one GPU with the tombstones on their own stream, the list's take
        # and the accumulators' clear move from before the sweep into the
        # flush's shadow (after the threshold bin's selection); the lists
        # alternate by step parity so the side stream's next list never
        # overwrites the one still to be taken
        self.late_io = bool(self.flush_split and self.plan_ahead and self.ahead and not self.shard_select)
        self.win_blocks = 3 if self.shard_select else (2 if self.late_io else 1)
        self.sel_shard = None
        if self.ahead:
            self.claim_next = None if self.shard_select else tuple(
                torch.empty(self.win_blocks * t.numel(), dtype=t.dtype, device=device) for t in self.claim_in)
            self.sel_step_dev = torch.zeros(1, dtype=torch.int32, device=device)
            if self.late_io:
                self.sel_shard = K.select_shard(0, 1, self.win_blocks, [tuple(c.data_ptr() for c in self.claim_next)])
        self.launches = 0

    def _init_train_fused(self, fuse_train: bool) -> None:
        """Whether a step's propagation and update run as the fused pipeline
        training step (pxb_pipeline_train_step): a single-device PIPELINE net
        with one bucket, sum forward and backward, an MSE loss or none, an
        update_conn other than UPGD and no unit-side phase in between."""
        net, n = self.net, self.static.num_units
        uc, bp, loss = net.update_conn, net.backward_pass, net.loss
        self.train_fused = bool(
            fuse_train and self.pipeline and not self.sharded and self.num_buckets == 1 and uc is not None
            and uc.kind != "upgd" and uc.scale_field is None and net.update_unit is None
            and not self.unit_lifecycle and self.fwd_monoid == "sum"
            and (bp is None or bp.combine.lowered() == "sum")
            and (loss is None or isinstance(loss, MSELoss))
            and (loss is None or bp is None or bp.seed_field.name == loss.seed_field.name)
            and torch.device(self.dev).type == "cuda"
            and n <= int(_lib.lib().pxb_pipeline_train_max_units(int(bp is not None))))
        self.train_desc = None
        if not self.train_fused:
            return
        size = _lib.query_size("pxb_pipeline_train_scratch_bytes", ctypes.c_int32(n))
        self.train_scratch = torch.zeros(size, dtype=torch.uint8, device=self.dev)
        target_of = np.full(n, -1, np.int32)
        target_of[list(self.static.output_ids)] = np.arange(len(self.static.output_ids), dtype=np.int32)
        self.train_target_of = torch.from_numpy(target_of).to(self.dev)

    def _bind_train(self, state: NetworkState) -> None:
        """The fused training step's descriptor for `state` (its columns)."""
        net, units, b = self.net, state.units, state.conns[0]
        bp, loss, uc = net.backward_pass, net.loss, net.update_conn
        m, v, t = (b.get(c) for c in self.opt_cols)
        pruned = units.get(PRUNED.name)
        d = _lib.PipelineTrain()
        d.cap = int(b["dead"].numel())
        d.from_id, d.to_id, d.dead, d.weight = (K.ptr(b[c]) for c in ("from_id", "to_id", "dead", "weight"))
        d.opt_m, d.opt_v, d.opt_t = K.ptr(m), K.ptr(v), K.ptr(t)
        d.num_units = self.static.num_units
        d.act = K.ptr(units[ACTIVATION.name])
        d.grad = K.ptr(units[bp.grad_field.name]) if bp is not None else None
        d.seed = K.ptr(units[loss.seed_field.name]) if loss is not None else None
        d.roles = K.ptr(self.is_input)
        d.pruned = K.ptr(pruned)
        d.fwd_act = _lib.act_code(self.fwd_act)
        d.bwd_act = _lib.act_code(self.bwd_act) if bp is not None else 0
        d.num_outputs = len(self.static.output_ids)
        d.target_of = K.ptr(self.train_target_of)
        d.output_ids = K.ptr(self.output_ids)
        d.loss = K.ptr(self.loss_buf) if loss is not None else None
        d.update_grad = K.ptr(units[uc.grad_field.name])
        d.opt = self.opt
        d.scratch = K.ptr(self.train_scratch)
        # a PIPELINE arena's slots past tail_start were never claimed
        d.tail_start = K.ptr(state.tail_start) if state.tail_start is not None else None
        self.train_desc = d

    def _train(self, state: NetworkState, inputs: StepInputs) -> None:
        """Forward, loss, backward and update_conn as the fused pipeline
        training step (three kernels; the same values as the separate
        passes, with both sums exact in fixed point)."""
        d = self.train_desc
        t = None
        if self.net.loss is not None:
            t = inputs.targets
            if t is None:
                raise ValueError("a network with a loss needs StepInputs.targets")
            if not isinstance(t, torch.Tensor):
                t = torch.from_numpy(np.ascontiguousarray(t, np.float32))
            t = t.to(self.dev, non_blocking=True).reshape(-1)
        d.target = K.ptr(t)
        K.pipeline_train(d)
        self._mark("train")
        self.launches += 3

    # -- per-state device indices ---------------------------------------------
    def _bind(self, state: NetworkState) -> None:
        """Build the mirror and free-slot bitmaps of `state` (once per state
        object; the step owns the state between calls, as with donation)."""
        if self._bound == id(state):
            return
        from plastax_b200.mirror import Mirror

        st = self.static
        level = state.units[LEVEL.name]
        self._level = level
        if self.use_mirror:
            self.mirrors = [Mirror(b, st.num_units, chunk_bits=self.mirror_chunk_bits, slack=self.mirror_slack,
                                   min_slack=self.mirror_min_slack) for b in state.conns]
            fan = max(m.max_in_degree for m in self.mirrors)
            if self.acc_fixed is not None and fan > FIXED_EXACT_FAN_IN:
                import warnings

                warnings.warn(f"a unit has {fan} in-edges: the mirror's fixed-point sum rounds each product below "
                              f"2^-7 to 2^-31, so its error bound ({fan} * 2^-32) exceeds 1e-6; the sum is still "
                              f"independent of order but may differ from the correctly rounded sum by more",
                              stacklevel=2)
        if self.peer_reduce:
            from plastax_b200.peers import PeerGroup

            if self.peers is None:
                self.peers = PeerGroup(st.num_units, self.dev,
                                       lowk_cap=self._lowk_list_cap() if self.lowk_prune else 0,
                                       win_k=self.k if self.shard_select else 0, win_blocks=self.win_blocks)
                self.acc_fixed = self.peers.acc_fixed
                self.acc = self.peers.acc_side
                if self.shard_select:
                    self.claim_next = self.peers.win_cols
                    self.sel_shard = K.select_shard(self.peers.rank, self.peers.world, self.win_blocks,
                                                    self.peers.win_ptrs)
            # the activation column lives in the group's region: peers write it
            self.peers.act.copy_(state.units[ACTIVATION.name])
            state.units[ACTIVATION.name] = self.peers.act
        if self.ac is not None:
            mode = _lib.CLAIM_PIPELINE if self.pipeline else _lib.CLAIM_TOPOLOGICAL
            self.bitmaps = [K.free_bitmap_build(mode, b, level, state.tail_start, self.num_levels,
                                                shard_base=st.shard_base(i)) for i, b in enumerate(state.conns)]
        if self.lowk_prune:
            from plastax_b200.lowk import LowestK

            if self.lowk is None:
                self.lowk = LowestK(self.net.prune_conn.k, self.dev, list_cap=self._lowk_list_cap(),
                                    slot_base=st.shard_base(0), peers=self.peers)
            combine = combine_min = None
            if self.sharded:
                combine = lambda h: _dist().all_reduce(h, op=_dist().ReduceOp.SUM)  # noqa: E731
                combine_min = lambda h: _dist().all_reduce(h, op=_dist().ReduceOp.MIN)  # noqa: E731
            self.lowk.build_hist(state.conns, combine=combine, combine_min=combine_min)
        uc = self.net.update_conn
        if uc is not None and uc.scale_field is not None:
            self.opt = uc.struct(state.units[uc.scale_field.name])
        if self.unit_lifecycle:
            self._bind_units(state)
        if self.train_fused:
            self._bind_train(state)
        self.step_dev.fill_(state.step)
        if self.late_io:
            K.clear_accumulators(self.acc, self.fwd_identity, self.acc_fixed)
        self._ahead_ready = False
        self._plan_ready = False
        self._bound = id(state)

    def _mark(self, name: str) -> None:
        if self.phase_marks is not None and self.graph is None and not torch.cuda.is_current_stream_capturing():
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self.phase_marks.append((name, ev))

    def phase_times(self) -> dict[str, float]:
        """Mean milliseconds of each phase over the marked eager steps (the
        span from the previous mark to the named one; synchronises), and
        clears the marks."""
        marks, self.phase_marks = self.phase_marks or [], []
        torch.cuda.synchronize(self.dev)
        tot: dict[str, float] = {}
        cnt: dict[str, int] = {}
        for (_, a), (name, b) in zip(marks, marks[1:]):
            if name == "start":
                continue
            tot[name] = tot.get(name, 0.0) + a.elapsed_time(b)
            cnt[name] = cnt.get(name, 0) + 1
        return {k: tot[k] / cnt[k] for k in tot}

    def _lowk_list_cap(self) -> int:
        pc = self.net.prune_conn
        if pc.list_capacity is not None:
            return int(pc.list_capacity)
        return max(1 << 16, int(pc.k))

    def status_words(self) -> dict[str, int]:
        """Every device status word of the step, read in one host sync
        (only the words this step keeps): `mirror` (bit 0 an insert found no
        room, bit 1 a sweep's bulk copy never completed), `peers` (bit 0 a
        wait for a peer gave up), `select` (bit 0 a selection bin held more
        keys than it ranks), `lowk` (bit 0 a prune list overflowed, bit 1
        the prune's counts disagreed with its histogram)."""
        words, names = [], []
        if self.mirrors:
            words.append(torch.stack([m.status[0] for m in self.mirrors]).amax().reshape(1))
            names.append("mirror")
        if self.peers is not None:
            words.append(self.peers.status.reshape(1))
            names.append("peers")
        if getattr(self, "fs_status", None) is not None:
            words.append(self.fs_status.reshape(1))
            names.append("select")
        if self.lowk is not None:
            words.append(self.lowk.status.reshape(1))
            names.append("lowk")
        if not words:
            return {}
        vals = torch.cat([w.to(torch.int32) for w in words]).cpu().tolist()
        return dict(zip(names, vals, strict=True))

    def check_status(self) -> bool:
        """Read every status word (one host sync) and raise PxbError for a
        fault: a sweep whose bulk copy never completed, a peer wait that gave
        up (the step is incomplete), a selection bin that overflowed (fewer
        winners than k were listed), a lowest-|w| prune that overflowed its
        list or disagreed with its histogram. Returns whether every mirror
        still holds every live edge (False: `invalidate()` rebuilds them)."""
        w = self.status_words()
        faults = []
        if w.get("mirror", 0) & 2:
            faults.append("mirror sweep: a bulk copy never completed (status bit 1)")
        if w.get("peers", 0) & 1:
            faults.append("Scheme-A combine: a wait for a peer gave up; the step's activations are incomplete")
        if w.get("select", 0) & 1:
            faults.append("growth selection: a bin held more keys than it ranks; the winner list is incomplete")
        if w.get("lowk", 0) & 1:
            faults.append("lowest-|w| prune: the threshold bin held more edges than the list capacity "
                          f"({self._lowk_list_cap()}); raise LowestMagnitudePrune(list_capacity=...)")
        if w.get("lowk", 0) & 2:
            faults.append("lowest-|w| prune: the swept counts disagree with the histogram (the arena changed "
                          "outside the step without invalidate())")
        if faults:
            raise _lib.PxbError("; ".join(faults))
        return not (w.get("mirror", 0) & 1)

    def mirrors_healthy(self) -> bool:
        """Whether every mirror still holds every live edge, after checking
        every status word (`check_status`; one host read)."""
        return self.check_status()

    def invalidate(self) -> None:
        """Drop the per-state indices (call after editing a state's columns
        outside the step); they are rebuilt on the next call."""
        self._bound = None
        self.mirrors = None
        self.bitmaps = None
        self.release_graph()

    def _bm(self, bucket: int) -> tuple[torch.Tensor | None, torch.Tensor | None]:
        """(free bitmap, the level column naming its rows) of a bucket."""
        if self.bitmaps is None:
            return None, None
        return self.bitmaps[bucket], None if not self.pipeline else self._level

    # -- ScoreAddConn candidates ----------------------------------------------
    def _build_score_candidates(self) -> None:
        """The grid a ScoreAddConn draws (src/plastax/phases.py:4655-4690):
        a shortlist of M units when 0 < M < num_units (per source level for
        shortlist_per_level), else every ordered pair."""
        ac, st, dev = self.ac, self.static, self.dev
        n = st.num_units
        M = ac.shortlist_size
        self.use_shortlist = ac.candidates in ("shortlist", "shortlist_per_level") and M is not None and 0 < M < n
        self.use_per_level = self.use_shortlist and ac.candidates == "shortlist_per_level"
        side = int(M) if self.use_shortlist else n
        self.grids = self.num_buckets if self.use_per_level else 1
        self.pool_side = side
        self.n_cand = self.grids * side * side
        if self.n_cand >= 1 << 31:
            raise NotImplementedError(f"ScoreAddConn: {self.grids} x {side}^2 candidates exceed the int32 candidate "
                                      f"index (declare a shortlist)")
        if self.use_shortlist:
            self.unit_ids = torch.arange(n, dtype=torch.int32, device=dev)
            self.imp = torch.empty(n, dtype=torch.float32, device=dev)
            self.rows = torch.empty(self.grids * side, dtype=torch.int32, device=dev)
            self.cols = torch.empty(self.grids * side, dtype=torch.int32, device=dev) if self.use_per_level else None
            need = K.topk_unique_scratch(n, side, n)
            self.imp_scratch = torch.empty(max(need, 1), dtype=torch.uint8, device=dev)

    @staticmethod
    def _field(units: dict, f) -> torch.Tensor:
        name = f if isinstance(f, str) else f.name
        if name not in units:
            raise ValueError(f"ScoreAddConn: the state has no unit field {name!r}")
        return units[name]

    def _score_form(self, units: dict):
        form = self.ac.score
        kind = form[0]
        if kind == "grad_act":
            return K.pair_score(_lib.PAIR_ABS_PRODUCT, x_src=units[ACTIVATION.name],
                                x_dst=self._field(units, self.ac.grad_field))
        if kind in ("abs_product", "product"):
            return K.pair_score(_lib.PAIR_ABS_PRODUCT if kind == "abs_product" else _lib.PAIR_PRODUCT,
                                x_src=self._field(units, form[1]), x_dst=self._field(units, form[2]))
        if kind == "modular":
            return K.pair_score(_lib.PAIR_MODULAR, a=int(form[1]), b=int(form[2]), m=int(form[3]), c=int(form[4]),
                                scale=float(form[5]))
        return K.pair_score(_lib.PAIR_MODULAR_PREDICATE, a=int(form[1]), b=int(form[2]), m=int(form[3]),
                            c=int(form[4]))

    def _importance_form(self, units: dict):
        form = self.ac.importance
        if form[0] == "abs_field":
            return K.pair_score(_lib.PAIR_ABS_PRODUCT, x_src=self._field(units, form[1]))
        if form[0] == "field":
            return K.pair_score(_lib.PAIR_PRODUCT, x_src=self._field(units, form[1]))
        return K.pair_score(_lib.PAIR_MODULAR, a=int(form[1]), m=int(form[2]), c=int(form[3]), scale=float(form[4]))

    def _score_candidates(self, state: NetworkState, window: dict) -> None:
        """The step's scored grid into the candidate columns: importance
        ranked on the device (ties by ascending id, the first M of the
        (-importance, id) order), then one pass that scores and windows every
        (row, column) pair (src/plastax/phases.py:3668-3746, :4760-4860)."""
        ac, units = self.ac, state.units
        n = self.static.num_units
        score = self._score_form(units)
        grid = dict(level=window["level"], pruned=window["pruned"], max_level_gap=ac.max_level_gap,
                    direction=self.direction, allow_self_loops=ac.allow_self_loops,
                    src_level_bound=window["src_level_bound"], out=self.cand)
        if not self.use_shortlist:
            K.propose_grid(n, 1, n, n, score, **grid)
            self.launches += 1
            return
        imp = self._importance_form(units)
        M, pruned, level = self.pool_side, window["pruned"], window["level"]
        if not self.use_per_level:
            K.unit_importance(n, imp, pruned=pruned, level=level, out=self.imp)
            K.topk_unique(self.imp, self.unit_ids, n, M, out=self.rows, scratch=self.imp_scratch)
            K.propose_grid(n, 1, M, M, score, row_ids=self.rows, col_ids=self.rows, **grid)
            self.launches += 4
            return
        for b in range(self.grids):
            K.unit_importance(n, imp, pruned=pruned, level=level, mask_kind=1, bucket=b, out=self.imp)
            K.topk_unique(self.imp, self.unit_ids, n, M, out=self.rows[b * M:(b + 1) * M], scratch=self.imp_scratch)
            K.unit_importance(n, imp, pruned=pruned, level=level, mask_kind=2, bucket=b,
                              max_level_gap=ac.max_level_gap, direction=self.direction, out=self.imp)
            K.topk_unique(self.imp, self.unit_ids, n, M, out=self.cols[b * M:(b + 1) * M], scratch=self.imp_scratch)
        K.propose_grid(n, self.grids, M, M, score, row_ids=self.rows, col_ids=self.cols, per_grid_bucket=True,
                       **grid)
        self.launches += 1 + 6 * self.grids

    # -- growth buffers ------------------------------------------------------
    def _build_growth(self) -> None:
        ac, st, dev = self.ac, self.static, self.dev
        n = st.num_units
        P = getattr(ac, "proposals_per_proposer", 0)
        if self.is_score:
            self._build_score_candidates()
        elif ac.proposer == "per_unit":
            self.n_cand = n * P
        elif ac.proposer == "global":
            self.n_cand = P
        else:
            # every rank's connections take part (under Scheme-A the bands are
            # gathered into the whole arena first: gather_arena)
            self.conn_slots = sum(int(c) for c in st.level_capacities)
            self.n_cand = self.conn_slots * P
            self.conn_scratch = torch.empty(max(K.conn_rank_scratch(self.conn_slots, n), 1), dtype=torch.uint8,
                                            device=dev)
            self.arena_all = None
            if self.sharded:
                self.arena_all = {"from_id": torch.empty(self.conn_slots, dtype=torch.int32, device=dev),
                                  "to_id": torch.empty(self.conn_slots, dtype=torch.int32, device=dev),
                                  "dead": torch.empty(self.conn_slots, dtype=torch.uint8, device=dev)}
        src_lo, dst_lo = getattr(ac, "src_lo", 0), getattr(ac, "dst_lo", 0)
        src_n = getattr(ac, "src_n", None)
        src_n = src_n if src_n is not None else n - src_lo
        if getattr(ac, "proposer", "") == "global" and (src_lo < 0 or src_n < 1 or src_lo + src_n > n):
            raise ValueError(f"ProposeAddConn: sources [{src_lo}, {src_lo + src_n}) exceed the {n} units")
        self.src_n = src_n
        # the cap: per source level (the default) or once per step; "all"
        # keeps every finite candidate
        self.k_sel = self.n_cand if ac.selection == "all" else max(0, min(int(ac.max_new_per_level), self.n_cand))
        self.per_level = ac.level_cap_scope == "source_level" and ac.selection != "all"
        self.sel_levels = st.num_levels
        self.k = min(self.n_cand, self.sel_levels * self.k_sel) if self.per_level else self.k_sel
        self.cand = (torch.empty(self.n_cand, dtype=torch.int32, device=dev),
                     torch.empty(self.n_cand, dtype=torch.int32, device=dev),
                     torch.empty(self.n_cand, dtype=torch.float32, device=dev))
        dst_n = getattr(ac, "dst_n", None)
        dst_n = dst_n if dst_n is not None else n - dst_lo
        if dst_lo < 0 or dst_n < 1 or dst_lo + dst_n > n:
            raise ValueError(f"ProposeAddConn: destinations [{dst_lo}, {dst_lo + dst_n}) exceed the {n} units")
        # One proposal per unit: every candidate's source is its own unit, so
        # (score, src) is a unique key in the total order and a radix select
        # of the first k replaces the full sort.
        self.unique_src = P == 1 and getattr(ac, "proposer", "") == "per_unit" and not self.per_level
        self.perm = torch.empty(self.n_cand if not self.unique_src else max(self.k, 1), dtype=torch.int32, device=dev)
        need = K.topk_unique_scratch(self.n_cand, self.k, n) if self.unique_src else K.total_order_scratch(self.n_cand, n)
        self.order_scratch = torch.empty(max(need, 1), dtype=torch.uint8, device=dev)
        self.win = torch.empty(max(self.k, 1), dtype=torch.int32, device=dev)
        k_listed = self.n_cand if self.per_level else self.k
        self.sel_scratch = torch.empty(max(K.select_step_scratch(self.n_cand, k_listed), 1), dtype=torch.uint8,
                                       device=dev)
        if self.per_level:
            self.win_all = torch.empty(max(self.n_cand, 1), dtype=torch.int32, device=dev)
            self.win_count = torch.zeros(1, dtype=torch.int32, device=dev)
            self.cap_scratch = torch.zeros(3 * self.sel_levels + 1, dtype=torch.int32, device=dev)
        kk = max(self.k, 1)
        self.claim_in = (torch.empty(kk, dtype=torch.int32, device=dev), torch.empty(kk, dtype=torch.int32, device=dev),
                         torch.empty(kk, dtype=torch.float32, device=dev), torch.empty(kk, dtype=torch.uint8, device=dev))
        self.extra_defaults: dict[str, torch.Tensor] = {}
        builtin = {"from_id", "to_id", "dead", "weight"}
        for spec in st.conn_fields:
            if spec.name in builtin:
                continue
            from plastax_b200.state import torch_dtype

            self.extra_defaults[spec.name] = torch.full((kk,), spec.default, dtype=torch_dtype(spec), device=dev)
        self.num_levels = st.num_levels if self.pipeline else 1
        self.claim_ws = [K.ClaimWorkspace(st.local_capacity(b), self.k, self.num_levels, dev)
                         for b in range(self.num_buckets)]
        self.init_kind = {"const": _lib.INIT_CONST, "dyadic": _lib.INIT_DYADIC,
                          "hash_uniform": _lib.INIT_HASH_UNIFORM}[ac.init[0]]
        self.init_a = float(ac.init[1]) if len(ac.init) > 1 else 0.0
        self.score_kind = -1 if self.is_score else {"uniform": _lib.SCORE_UNIFORM,
                                                    "uniform_q256": _lib.SCORE_UNIFORM_Q256,
                                                    "grad_act": _lib.SCORE_GRAD_ACT}[ac.score]
        self.direction = {"any": 0, "deeper": 1, "same_or_deeper": 2}[ac.direction]
        # one proposal per unit scored by the site RNG: the fused selection
        # (keys binned and ranked, no sort pass) replaces propose + top-k +
        # level listing + gather
        self.fast_select = (self.unique_src and not self.is_score and ac.score in ("uniform", "uniform_q256")
                            and ac.level_cap_scope == "step" and ac.selection == "top_k"
                            and self.static.num_levels <= 8 and self.k > 0
                            and not ac.dedupe_live and not ac.dedupe_step)
        self.dedupe = ac.dedupe_live or ac.dedupe_step
        if self.dedupe:
            self.dedupe_scratch = torch.empty(max(K.dedupe_scratch(self.n_cand), 1), dtype=torch.uint8, device=dev)
            self.live_hit = torch.empty(max(self.n_cand, 1), dtype=torch.uint8, device=dev)
        if self.fast_select:
            need = K.select_unique_scratch(n, self.k, self.static.num_levels, self.score_kind)
            self.fs_scratch = torch.empty(max(need, 1), dtype=torch.uint8, device=dev)
            self.fs_status = torch.zeros(1, dtype=torch.int32, device=dev)
        self.grown = torch.zeros((), dtype=torch.int32, device=dev)
        self.overflow = torch.zeros((), dtype=torch.bool, device=dev)
        self.placed = torch.empty(kk, dtype=torch.int32, device=dev)
        self.committed = torch.zeros(kk, dtype=torch.uint8, device=dev)
        if self.sharded:
            G = st.num_shards
            self.gather_buf = torch.zeros((G, self.num_levels), dtype=torch.int32, device=dev)
            self.level_before = torch.zeros(self.num_levels, dtype=torch.int32, device=dev)
            self.level_totals = torch.zeros(self.num_levels, dtype=torch.int32, device=dev)

    # -- collectives -----------------------------------------------------------
    def _combine_partials(self, acc: torch.Tensor, acc_fixed: torch.Tensor | None = None) -> None:
        if self.sharded:
            _dist().all_reduce(acc, op=self.reduce_op)
            if acc_fixed is not None:
                _dist().all_reduce(acc_fixed, op=_dist().ReduceOp.SUM)

    # -- phases -----------------------------------------------------------------
    def _scatter_inputs(self, state: NetworkState, inputs: StepInputs) -> None:
        x = inputs.inputs
        if not isinstance(x, torch.Tensor):
            x = torch.from_numpy(np.ascontiguousarray(x, np.float32))
        if self._io_src is not None:
            # a host-I/O graph: the kernel reads the pinned staging buffer
            K.scatter_inputs(self.input_ids, self._io_src, state.units[ACTIVATION.name])
            return
        x = x.to(self.dev, non_blocking=True).reshape(-1)
        state.units[ACTIVATION.name].index_copy_(0, self.input_ids, x)

    def _accumulate_bucket(self, state: NetworkState, i: int, act: torch.Tensor, acc: torch.Tensor,
                           acc_fixed: torch.Tensor | None) -> None:
        """Forward accumulate of bucket i, with the prune fused when legal."""
        net, b = self.net, state.conns[i]
        bm, bm_level = self._bm(i)
        if self.use_mirror:
            m = self.mirrors[i]
            lowk = self.lowk_prune and self._lowk_fires(state)
            if lowk and not self._plan_ready:
                self.lowk.make_plan()
            # a side branch forked from just before the sweep and captured
            # after it: it depends on nothing the sweep does, and the sweep's
            # launch comes first
            fork, self._sweep_fork = self._sweep_fork, None
            ev = None
            if fork is not None:
                ev = torch.cuda.Event()
                ev.record()
            if lowk:
                self._plan_ready = False
                post, self._post_fork = self._post_fork, None
                split = self.flush_split or post is not None
                self.lowk.sweep(m, act, acc, acc_fixed, self.fwd_monoid, b["dead"], bm, bm_level,
                                flush=not split)
                self._lowk_fired = True
                self.launches += 1
                if post is not None:
                    post()  # the next step's selection, from the sweep's end
                if not self.flush_split and split:
                    self.lowk.flush(m, self.fwd_monoid, b["dead"], bm, bm_level)
                    self.launches += 1
                if self.flush_split:
                    self.flush_stream.wait_stream(torch.cuda.current_stream(self.dev))
                    with torch.cuda.stream(self.flush_stream):
                        self.lowk.flush(m, self.fwd_monoid, b["dead"], bm, bm_level)
                    self._flush_pending = True
                    self.launches += 1
            elif self.lowk_prune:
                K.mirror_forward(m, act, acc, acc_fixed=acc_fixed, monoid=self.fwd_monoid)
            elif self.fuse_prune:
                K.mirror_forward(m, act, acc, acc_fixed=acc_fixed, monoid=self.fwd_monoid,
                                 prune_kind=_lib.PRUNE_ABS_BELOW, threshold=net.prune_conn.threshold,
                                 dead=b["dead"], free_bitmap=bm, bitmap_words=(b["dead"].numel() + 31) // 32,
                                 bitmap_level=bm_level)
            else:
                K.mirror_forward(m, act, acc, acc_fixed=acc_fixed, monoid=self.fwd_monoid)
        elif self.fuse_prune:
            K.forward_prune(b, act, acc, monoid=self.fwd_monoid, prune_kind=_lib.PRUNE_ABS_BELOW,
                            threshold=net.prune_conn.threshold, free_bitmap=bm, bitmap_level=bm_level)
        else:
            K.forward_accumulate(b, act, acc, self.fwd_monoid)
        if self.use_mirror and fork is not None:
            fork(ev)

    def _forward_bucket(self, state: NetworkState, i: int, act: torch.Tensor) -> None:
        """Bucket i's forward partial, reduced across shards, in the carried
        accumulator."""
        if not self.per_bucket_reduce:
            self._accumulate_bucket(state, i, act, self.acc, self.acc_fixed)
            self._combine_partials(self.acc, self.acc_fixed)
            return
        K.fill(self.part, self.fwd_identity)
        if self.part_fixed is not None:
            self.part_fixed.zero_()
        self._accumulate_bucket(state, i, act, self.part, self.part_fixed)
        self._combine_partials(self.part, self.part_fixed)
        if self.fwd_monoid == "sum":
            self.acc.add_(self.part)
            if self.part_fixed is not None:
                self.acc_fixed.add_(self.part_fixed)
        elif self.fwd_monoid == "max":
            torch.maximum(self.acc, self.part, out=self.acc)
        else:
            torch.minimum(self.acc, self.part, out=self.acc)

    def _upgd_eta(self, state: NetworkState) -> None:
        """UPGD's local utility scale (examples/upgd.py:83-128, v1): every
        destination's max over its incoming live edges' stored utilities
        (the previous step's), -inf without one, written for the live
        non-input units; a max sweep with the utilities as weights and unit
        activations of one (each product is the utility itself)."""
        uc = self.net.update_conn
        n = self.static.num_units
        if getattr(self, "_eta_acc", None) is None:
            self._eta_acc = torch.empty(n, dtype=torch.float32, device=self.dev)
            self._ones = torch.ones(n, dtype=torch.float32, device=self.dev)
        K.fill(self._eta_acc, float("-inf"))
        util = uc.cols[0]
        for b in state.conns:
            K.forward_accumulate({"from_id": b["from_id"], "to_id": b["to_id"], "dead": b["dead"], "weight": b[util]},
                                 self._ones, self._eta_acc, "max")
            self.launches += 1
        if self.sharded:
            _dist().all_reduce(self._eta_acc, op=_dist().ReduceOp.MAX)
        K.unit_apply(self._eta_acc, state.units[uc.scale_field.name], mode=0, act_kind="identity", monoid="max",
                     is_input=self.is_input, pruned=state.units.get(PRUNED.name))
        self.launches += 2

    def _forward(self, state: NetworkState) -> None:
        if self.upgd_local:
            self._upgd_eta(state)
        net, st, units = self.net, self.static, state.units
        act = units[ACTIVATION.name]
        pruned = units.get(PRUNED.name)
        fp = net.forward_pass
        if not (self.late_io and self.ahead):  # else cleared by the previous step (and at bind)
            K.clear_accumulators(self.acc, self.fwd_identity, self.acc_fixed)
        if self.pipeline:
            if self.peers is not None:
                from plastax_b200.peers import scheme_a_apply

                self._accumulate_bucket(state, 0, act, self.acc, self.acc_fixed)
                self._mark("sweep")
                # with the prune in the sweep nothing touches the arena before
                # the claim: its per-domain free counts are final here and ride
                # on the combine's barrier instead of an all-gather
                counts = None
                self._counts_on_barrier = (self.ac is not None and self.k > 0 and self._fires(state)
                                           and self.num_levels <= _lib.PEER_MAX_LEVELS)
                if self._counts_on_barrier:
                    ws = self.claim_ws[0]
                    bm, _ = self._bm(0)
                    K.claim_prepare(_lib.CLAIM_PIPELINE, state.conns[0], units[LEVEL.name], state.tail_start, ws,
                                    shard_base=self.static.shard_base(0), free_bitmap=bm)
                    counts = ws.level_counts
                scheme_a_apply(self.peers, self.fwd_act, is_input=self.is_input, pruned=pruned,
                               level_counts=counts, level_before=self.level_before, level_totals=self.level_totals)
                self._mark("combine")
                self.launches += 3
                if self._after_combine is not None:
                    hook, self._after_combine = self._after_combine, None
                    hook()
                if self._lowk_fired:
                    # every rank's sweep is complete: select the threshold
                    # bin's edges, adding every rank's to the barrier's counts
                    self._lowk_select(state, adjust=self._counts_on_barrier)
                    self._mark("select")
                return
            self._forward_bucket(state, 0, act)
            self._mark("sweep")
            K.unit_apply(self.acc, act, mode=0, act_kind=self.fwd_act, monoid=self.fwd_monoid,
                         is_input=self.is_input, pruned=pruned, acc_fixed=self.acc_fixed)
            self._mark("apply")
            self.launches += 3
            return
        level = units[LEVEL.name]
        for l in range(self.num_buckets):
            self._forward_bucket(state, l, act)
            K.unit_apply(self.acc, act, mode=0, act_kind=self.fwd_act, monoid=self.fwd_monoid, level=level,
                         target_level=l + 1, is_input=self.is_input, pruned=pruned, acc_fixed=self.acc_fixed)
            self.launches += 2

    def _loss(self, state: NetworkState, inputs: StepInputs) -> None:
        loss = self.net.loss
        if loss is None:
            return
        t = inputs.targets
        if t is None:
            raise ValueError("a network with a loss needs StepInputs.targets")
        if not isinstance(t, torch.Tensor):
            t = torch.from_numpy(np.ascontiguousarray(t, np.float32))
        t = t.to(self.dev, non_blocking=True).reshape(-1)
        if isinstance(loss, MSELoss):
            K.mse_loss(self.output_ids, state.units[ACTIVATION.name], t, state.units[loss.seed_field.name],
                       self.loss_buf)
        elif isinstance(loss, SoftmaxCrossEntropyLoss):
            # the one-sample case of the batched loss ([N] == [N, 1] rows)
            K.batched_loss(_lib.LOSS_SOFTMAX_CE, self.output_ids, 1, state.units[ACTIVATION.name], t,
                           state.units[loss.seed_field.name], self.loss_b1, self.loss_buf)
        else:
            raise NotImplementedError(f"loss {type(loss).__name__} has no engine lowering")
        self.launches += 1

    def _backward(self, state: NetworkState) -> None:
        net = self.net
        bp = net.backward_pass
        if bp is None:
            return
        units = state.units
        act, grad = units[ACTIVATION.name], units[bp.grad_field.name]
        seed = units.get(bp.seed_field.name)
        pruned = units.get(PRUNED.name)
        K.fill(self.acc, 0.0)
        if self.pipeline:
            K.backward_accumulate(state.conns[0], grad, self.acc, "sum")
            self._combine_partials(self.acc)
            K.unit_apply(self.acc, grad, mode=1, act_kind=self.bwd_act, act=act, seed=seed, is_input=self.bwd_roles,
                         pruned=pruned)
            self.launches += 3
            return
        level = units[LEVEL.name]
        L = self.num_buckets
        K.unit_apply(self.acc, grad, mode=1, act_kind=self.bwd_act, act=act, seed=seed, level=level,
                     target_level=L, is_input=self.is_input, pruned=pruned)
        for l in range(L - 1, 0, -1):
            b = state.conns[l]
            if self.fuse_update:
                K.backward_update(b, grad, act, self.acc, self.opt, self.opt_cols)
            else:
                K.backward_accumulate(b, grad, self.acc, "sum")
            self._combine_partials(self.acc)
            K.unit_apply(self.acc, grad, mode=1, act_kind=self.bwd_act, act=act, seed=seed, level=level,
                         target_level=l, is_input=self.is_input, pruned=pruned)
            self.launches += 2
        if self.fuse_update and L > 0:
            K.backward_update(state.conns[0], grad, act, None, self.opt, self.opt_cols)  # bucket 0: update only
            self.launches += 1

    def _update_conn(self, state: NetworkState) -> None:
        net = self.net
        if net.update_conn is None or self.fuse_update:
            return
        units = state.units
        grad, act = units[net.update_conn.grad_field.name], units[ACTIVATION.name]
        for b in state.conns:
            K.backward_update(b, grad, act, None, self.opt, self.opt_cols)
            self.launches += 1

    # -- unit lifecycle (src/plastax/phases.py:1148-1193, :1245-1425) ---------
    def _bind_units(self, state: NetworkState) -> None:
        st, net, dev = self.static, self.net, self.dev
        n = st.num_units
        specs = {spec.name: spec for spec in st.unit_fields}
        cols = [(state.units[name], spec.default) for name, spec in specs.items()
                if name not in (LEVEL.name, PRUNED.name)]
        self.unit_reset = K.unit_columns(cols)
        exempt = torch.zeros(n, dtype=torch.uint8, device=dev)
        io = list(st.input_ids) + list(st.output_ids)
        if io:
            exempt[torch.tensor(io, dtype=torch.long, device=dev)] = 1
        self.unit_exempt = exempt
        self.unit_doomed = torch.zeros(n, dtype=torch.uint8, device=dev)
        pu = net.prune_unit
        if pu is not None:
            self.unit_thr = torch.full((1,), float(pu.threshold) if pu.threshold is not None else 0.0,
                                       dtype=torch.float32, device=dev)
            if pu.quantile is not None:
                self.unit_q_scratch = torch.empty(max(K.unit_quantile_scratch(n), 1), dtype=torch.uint8, device=dev)
        au = net.add_unit
        if au is not None:
            self.unit_add_scratch = torch.empty(2 * n, dtype=torch.int32, device=dev)
            self.units_added = torch.zeros((), dtype=torch.int32, device=dev)
            self.unit_overflow = torch.zeros((), dtype=torch.uint8, device=dev)
            init_dst = init_src = None
            scale = 1.0
            if au.init is not None:
                from plastax_b200.traits import _field_name

                init_dst = state.units[_field_name(au.init[1])]
                init_src = state.units[_field_name(au.init[2])]
                scale = float(au.init[3])
            kind = _lib.SPAWN_ARGMAX if type(au).__name__ == "ArgmaxSpawn" else _lib.SPAWN_FIELD_AT_LEAST
            self.unit_spawn = _lib.UnitSpawn(kind, self._unit_col(state, au.field).data_ptr(),
                                             float(getattr(au, "threshold", 0.0)), int(au.offset),
                                             int(net.max_levels) - 1, K.ptr(init_dst), K.ptr(init_src), scale)

    @staticmethod
    def _unit_col(state: NetworkState, f) -> torch.Tensor:
        from plastax_b200.traits import _field_name

        name = _field_name(f)
        if name not in state.units:
            raise ValueError(f"unit rule: the state has no unit field {name!r}")
        return state.units[name]

    def _update_unit(self, state: NetworkState) -> None:
        uu = self.net.update_unit
        if uu is None:
            return
        pruned = state.units.get(PRUNED.name)
        field = self._unit_col(state, uu.field)
        if isinstance(uu, AffineUnitUpdate):
            K.unit_update(_lib.UNIT_UPDATE_AFFINE, field, a=uu.scale, b=uu.shift, pruned=pruned)
        else:
            kind = _lib.UNIT_UPDATE_TRACE_ABS if uu.absolute else _lib.UNIT_UPDATE_TRACE
            K.unit_update(kind, field, src=self._unit_col(state, uu.source), a=uu.rate, pruned=pruned)
        self.launches += 1

    def _prune_unit(self, state: NetworkState) -> None:
        pu = self.net.prune_unit
        if pu is None:
            return
        pruned = state.units[PRUNED.name]
        field = self._unit_col(state, pu.field)
        if pu.quantile is not None:
            K.unit_quantile(field, float(pu.quantile), self.unit_thr, pruned=pruned, exempt=self.unit_exempt,
                            scratch=self.unit_q_scratch)
            self.launches += 3
        K.unit_prune(field, self.unit_thr, pruned, self.unit_doomed, self.unit_reset, exempt=self.unit_exempt)
        for i, b in enumerate(state.conns):
            bm, bm_level = self._bm(i)
            K.kill_unit_edges(b, self.unit_doomed, free_bitmap=bm, bitmap_level=bm_level)
        self.launches += 1 + len(state.conns)

    def _add_unit(self, state: NetworkState) -> None:
        au = self.net.add_unit
        if au is None:
            return
        interval = int(getattr(self.net, "structural_interval", 1))
        if interval > 1 and state.step % interval != 0:
            self.units_added.zero_()
            self.unit_overflow.zero_()
        else:
            K.unit_add(self.unit_spawn, state.units[PRUNED.name], state.units[LEVEL.name], self.unit_reset,
                       self.unit_add_scratch, self.units_added, self.unit_overflow)
            self.launches += 1
        state.units_added, state.unit_overflow = self.units_added, self.unit_overflow

    def _lowk_fires(self, state: NetworkState) -> bool:
        every = self.net.prune_conn.every
        return every <= 1 or state.step % every == 0

    def _lowk_select(self, state: NetworkState, adjust: bool = False) -> None:
        """The threshold bin's selection of the exact lowest-|w| prune (after
        every rank's sweep); with `adjust` every rank's selected edges are
        added to the per-domain counts that rode on the peer barrier."""
        bm, bm_level = self._bm(0)
        self.lowk.select(self.mirrors[0], state.conns[0]["dead"], bm, bm_level,
                         num_levels=self.num_levels if adjust else 0,
                         level_before=self.level_before if adjust else None,
                         level_totals=self.level_totals if adjust else None)
        self.launches += 1

    def _prune(self, state: NetworkState) -> None:
        pc = self.net.prune_conn
        if self._lowk_fired and self.peers is None:
            self._lowk_select(state)
        if self.late_io and self.ahead:
            # beside the tombstones: this step's list into the claim's inputs,
            # the accumulators cleared for the next sweep (the apply has read them)
            K.select_take(self.k, self.win_blocks, self.step_dev, self.claim_next, self.claim_in)
            K.clear_accumulators(self.acc, self.fwd_identity, self.acc_fixed)
            self.launches += 2
        if self._flush_pending:
            # the sweep's tombstones are written: the arena is whole again
            torch.cuda.current_stream(self.dev).wait_stream(self.flush_stream)
            self._flush_pending = False
        if pc is None or self.fuse_prune:
            return
        n = self.static.num_units
        if isinstance(pc, LowestMagnitudePrune):
            self._prune_lowest(state, pc)
            return
        for i, b in enumerate(state.conns):
            bm, bm_level = self._bm(i)
            if isinstance(pc, MagnitudePrune):
                K.prune_conn(b, n, prune_kind=_lib.PRUNE_ABS_BELOW, threshold=pc.threshold, free_bitmap=bm,
                             bitmap_level=bm_level)
            elif isinstance(pc, DestinationThresholdPrune):
                K.prune_conn(b, n, prune_kind=_lib.PRUNE_ABS_BELOW_DST, unit_threshold=state.units[pc.field.name],
                             free_bitmap=bm, bitmap_level=bm_level)
            self.launches += 1

    def _prune_lowest(self, state: NetworkState, pc: LowestMagnitudePrune) -> None:
        """The k live edges of lowest |w| (ties by ascending slot, buckets in
        order) are tombstoned, on the steps `pc.every` divides."""
        if pc.every > 1 and state.step % pc.every != 0:
            return
        st = self.static
        caps = [int(b["dead"].numel()) for b in state.conns]
        total = sum(caps)
        k = min(int(pc.k), total)
        if k == 0:
            return
        if getattr(self, "_low_score", None) is None or self._low_score.numel() != total:
            self._low_score = torch.empty(max(total, 1), dtype=torch.float32, device=self.dev)
            self._low_slot = torch.empty(max(total, 1), dtype=torch.int32, device=self.dev)
            self._low_idx = torch.empty(max(k, 1), dtype=torch.int32, device=self.dev)
            self._low_scratch = torch.empty(max(K.topk_unique_scratch(total, k, total), 1), dtype=torch.uint8,
                                            device=self.dev)
        base = 0
        for b, cap in zip(state.conns, caps, strict=True):
            K.lowest_keys(b, base, self._low_score, self._low_slot)
            base += cap
        K.topk_unique(self._low_score[:total], self._low_slot[:total], total, k, out=self._low_idx,
                      scratch=self._low_scratch)
        base = 0
        for i, (b, cap) in enumerate(zip(state.conns, caps, strict=True)):
            bm, bm_level = self._bm(i)
            K.prune_selected(b, k, self._low_idx, self._low_score, base, st.num_units, free_bitmap=bm,
                             bitmap_level=bm_level)
            base += cap
        self.launches += 2 * len(caps) + 4

    def _fires(self, state: NetworkState) -> bool:
        ac = self.ac
        interval = int(getattr(self.net, "structural_interval", 1))
        fire = interval <= 1 or state.step % interval == 0
        trig = ac.trigger
        if isinstance(trig, tuple) and trig and trig[0] == "every":
            fire = fire and state.step % int(trig[1]) == 0
        elif trig not in ("every_step",):
            raise NotImplementedError(f"growth trigger {trig!r} has no engine lowering")
        return fire

    def _select(self, state: NetworkState, out: tuple | None = None, step_dev: torch.Tensor | None = None) -> None:
        """Growth selection: proposals, the first k in the total order and
        the level-major winner list (src/plastax/phases.py:3813-3860,
        :4208-4487, :5043-5058), gathered into the claim's input columns
        (`out`, default the claim's own), for the step `step_dev` holds."""
        out = self.claim_in if out is None else out
        step_dev = self.step_dev if step_dev is None else step_dev
        ac, st, units = self.ac, self.static, state.units
        n = st.num_units
        level = units[LEVEL.name]
        pruned = units.get(PRUNED.name)
        if self.is_score:
            self._score_candidates(state, dict(level=level, pruned=pruned,
                                               src_level_bound=0 if self.pipeline else self.num_buckets))
            self._select_candidates(state, out)
            return
        dst_n = ac.dst_n if ac.dst_n is not None else n - ac.dst_lo
        grad = units.get(ac.grad_field.name) if ac.score == "grad_act" else None
        if self.fast_select:
            # the step-ahead list under Scheme-A: this rank's share, into every rank's columns
            shard = self.sel_shard if self.sel_shard is not None and out is self.claim_next else None
            K.propose_select_unique(n, st.seed, state.step, dst_lo=ac.dst_lo, dst_n=dst_n, score_kind=self.score_kind,
                                    level=level, k=self.k, num_levels=st.num_levels, init_kind=self.init_kind,
                                    init_a=self.init_a, pruned=pruned, max_level_gap=ac.max_level_gap,
                                    direction=self.direction, allow_self_loops=ac.allow_self_loops,
                                    src_level_bound=0 if self.pipeline else self.num_buckets,
                                    step_dev=step_dev, status=self.fs_status, scratch=self.fs_scratch,
                                    out=out, shard=shard)
            self.launches += 6
            return
        window = dict(level=level, grad=grad, act=units[ACTIVATION.name], pruned=pruned,
                      max_level_gap=ac.max_level_gap, direction=self.direction,
                      allow_self_loops=ac.allow_self_loops,
                      src_level_bound=0 if self.pipeline else self.num_buckets, step_dev=step_dev)
        if ac.proposer == "per_unit":
            K.propose_per_unit(n, ac.proposals_per_proposer, st.seed, state.step, dst_lo=ac.dst_lo, dst_n=dst_n,
                               score_kind=self.score_kind, out=self.cand, **window)
        elif ac.proposer == "global":
            K.propose_global(ac.proposals_per_proposer, st.seed, state.step, n, src_lo=ac.src_lo, src_n=self.src_n,
                             dst_lo=ac.dst_lo, dst_n=dst_n, score_kind=self.score_kind, out=self.cand, **window)
        else:
            conns = state.conns
            if self.sharded:
                arena = gather_arena(conns, st, out=self.arena_all)
                self.launches += 3 * len(conns)
            else:
                arena = conns[0] if len(conns) == 1 else {
                    c: torch.cat([b[c] for b in conns]) for c in ("from_id", "to_id", "dead")}
            K.propose_per_conn(arena, ac.proposals_per_proposer, st.seed, state.step, n, dst_lo=ac.dst_lo,
                               dst_n=dst_n, score_kind=self.score_kind, scratch=self.conn_scratch, out=self.cand,
                               **window)
        self._select_candidates(state, out)

    def _select_candidates(self, state: NetworkState, out: tuple) -> None:
        """The candidate list's threshold veto, dedupes, total order, caps and
        level-major winner list, gathered into `out`."""
        ac = self.ac
        n = self.static.num_units
        level = state.units[LEVEL.name]
        if ac.selection == "threshold":
            # below the threshold is a veto (src/plastax/phases.py:4324-4487)
            sc = self.cand[2]
            sc.masked_fill_(sc < float(ac.threshold), float("-inf"))
        src, dst, score = self.cand
        if self.dedupe:
            combine = None
            if self.sharded and ac.dedupe_live:
                # a pair live on any rank is a duplicate everywhere (the
                # reference's pmax of the local marks)
                combine = lambda hit: _dist().all_reduce(hit, op=_dist().ReduceOp.MAX)  # noqa: E731
            K.dedupe(src, dst, score, buckets=list(state.conns) if ac.dedupe_live else [],
                     step_repeats=ac.dedupe_step, live_hit=self.live_hit, scratch=self.dedupe_scratch,
                     combine_hits=combine)
            self.launches += 4
        if self.unique_src:
            top = K.topk_unique(score, src, n, self.k, out=self.perm, scratch=self.order_scratch)
        else:
            top = K.total_order(score, src, dst, n, perm=self.perm, scratch=self.order_scratch)
        if self.per_level:
            # every candidate listed levels ascending, then each level's first k
            K.select_step(top, score, src, level, self.n_cand, win=self.win_all, scratch=self.sel_scratch,
                          num_levels=self.sel_levels)
            K.cap_per_level(self.win_all, src, level, self.sel_levels, self.k_sel, self.win, self.win_count,
                            self.cap_scratch)
        else:
            K.select_step(top, score, src, level, self.k, win=self.win, scratch=self.sel_scratch,
                          num_levels=self.static.num_levels)
        kk = min(self.k, self.n_cand)
        K.gather_winners(self.win, kk, self.k, src, dst, score, init_kind=self.init_kind, init_a=self.init_a,
                         out=out)
        self.launches += 4 + 5

    def _take(self) -> None:
        """This step's shared list into the claim's inputs, on the plan
        stream (idle between the step's start and its claim) when there is
        one; the claim joins it."""
        main = torch.cuda.current_stream(self.dev)
        if self.plan_stream is not None:
            self.plan_stream.wait_stream(main)
            with torch.cuda.stream(self.plan_stream):
                K.select_take(self.k, self.win_blocks, self.step_dev, self.claim_next, self.claim_in)
        else:
            K.select_take(self.k, self.win_blocks, self.step_dev, self.claim_next, self.claim_in)
        self._take_pending = True
        self.launches += 1

    def _add_conn(self, state: NetworkState, selected: bool = False) -> GrowthRemainder | None:
        """Growth: the selection (unless it already ran on the side stream)
        and the claim into the post-prune arena."""
        if self._take_pending:
            if self.plan_stream is not None:
                torch.cuda.current_stream(self.dev).wait_stream(self.plan_stream)
            self._take_pending = False
        ac = self.ac
        if ac is None:
            return None
        st = self.static
        level = state.units[LEVEL.name]
        if not self._fires(state) or self.k == 0:
            # cleared by the step's end (pxb_step_end), one launch with the
            # step counter
            self._clear_flags = True
            state.grown, state.overflow = self.grown, self.overflow
            return None
        if not selected:
            self._select(state)
        cs, cd, cw, grow = self.claim_in
        max_new = -1 if ac.max_new_per_step is None else int(ac.max_new_per_step)
        remainder = self._claim(state, cs, cd, cw, grow, max_new, fresh=True)
        if ac.on_overflow == "error" and bool(self.overflow.item()):
            raise RuntimeError('add_conn overflow: selected candidates exceeded the free connection capacity '
                               '(the rule declares on_overflow = "error").')
        return remainder

    def _claim(self, state: NetworkState, cs: torch.Tensor, cd: torch.Tensor, cw: torch.Tensor, grow: torch.Tensor,
               max_new: int, *, fresh: bool) -> GrowthRemainder:
        """The claim of a level-major candidate list into every bucket
        (src/plastax/phases.py:2853-3106): grown (+)= the committed count
        (from 0 when `fresh`), overflow = whether any growable candidate was
        dropped, needs_resort |= a committed edge into a level <= its
        source's. Returns the list with its dropped flags."""
        st = self.static
        level = state.units[LEVEL.name]
        if self.pipeline:
            # the winners are listed levels ascending: the claim partitions
            mode = _lib.CLAIM_PIPELINE | _lib.CLAIM_LEVEL_MAJOR
            buckets = [(0, grow)]
        else:
            mode = _lib.CLAIM_TOPOLOGICAL
            # step scope: the winners list is level-major; the per-step cap
            # ranks growable winners in that order across buckets
            g = grow.bool()
            if max_new >= 0:
                g = g & (torch.cumsum(g.to(torch.int32), 0) <= max_new)
            lv = level[cs.long()]
            buckets = [(bk, (g & (lv == bk)).to(torch.uint8)) for bk in range(self.num_buckets)]
            max_new = -1
        if not fresh:
            self.overflow.zero_()
        for bi, (bk, gb) in enumerate(buckets):
            b, ws = state.conns[bk], self.claim_ws[bk]
            base = st.shard_base(bk)
            bm, _ = self._bm(bk)
            before = totals = None
            counts_ready = self._counts_on_barrier and fresh
            if counts_ready:
                # the counts pass ran after the sweep and rode on the peer barrier
                before, totals = self.level_before, self.level_totals
                if self._lowk_fired:
                    # the lowest-|w| selection freed more slots since (its
                    # edges are in before/totals): refresh this rank's tiles
                    K.claim_prepare(mode, b, level, state.tail_start, ws, shard_base=base, free_bitmap=bm)
            else:
                K.claim_prepare(mode, b, level, state.tail_start, ws, shard_base=base, free_bitmap=bm)
            if self.sharded and not counts_ready:
                dist = _dist()
                dist.all_gather_into_tensor(self.gather_buf, ws.level_counts)
                rank = st.shard_rank
                before = self.gather_buf[:rank].sum(0, dtype=torch.int32) if rank else torch.zeros_like(
                    ws.level_counts)
                totals = self.gather_buf.sum(0, dtype=torch.int32)
            K.claim_commit(mode, b, level, state.tail_start, ws, cs, cd, cw, gb, max_new=max_new, shard_base=base,
                           global_cap=st.level_capacities[bk], level_before=before, level_totals=totals,
                           extra=self.extra_defaults, free_bitmap=bm, placed=self.placed,
                           committed=self.committed if self.lowk is not None else None)
            self._mark("claim")
            if self.lowk is not None:
                # the committed edges enter the prune's histogram (every rank
                # adds every rank's: the histogram is the whole arena's)
                if self.plan_ahead and fresh:
                    main = torch.cuda.current_stream(self.dev)
                    self.plan_stream.wait_stream(main)
                    with torch.cuda.stream(self.plan_stream):
                        self.lowk.hist_add(cw, self.committed, ws.counts, tally=fresh)
                        self.lowk.make_plan()
                    self._plan_pending = True
                    self.launches += 2
                else:
                    self.lowk.hist_add(cw, self.committed, ws.counts, tally=fresh)
                self.launches += 1
                self._mark("hist_add")
            if self.use_mirror:
                K.mirror_insert(self.mirrors[bk], cs, cd, cw, self.placed)
                self._mark("insert")
            K.growth_flags(ws.counts, reset=fresh and bi == 0, grown=self.grown, overflow=self.overflow,
                           needs_resort=state.needs_resort)
            self.launches += 12
        state.grown, state.overflow = self.grown, self.overflow
        if len(buckets) == 1:
            dropped = self.claim_ws[buckets[0][0]].overflowed
        else:
            # each candidate belongs to one bucket: the buckets' flags OR
            dropped = self.claim_ws[0].overflowed.clone()
            for bk in range(1, len(buckets)):
                dropped |= self.claim_ws[bk].overflowed
        return GrowthRemainder(cs, cd, cw, dropped)

    def retry(self, state: NetworkState, remainder: GrowthRemainder) -> tuple[NetworkState, GrowthRemainder]:
        """Claim a remainder's dropped candidates into `state` (after a
        regrow), in the list order, with the step's claim rule
        (src/plastax/phases.py:5206-5290): grown adds the new edges to the
        state's, overflow says whether candidates are still left; no other
        phase runs and the step counter is untouched."""
        if self.ac is None:
            raise ValueError("growth retry: the network has no add_conn rule")
        self._bind(state)
        self._level = state.units[LEVEL.name]
        self._counts_on_barrier = False
        k = remainder.src.numel()
        if k != self.k:
            raise ValueError(f"growth retry: the remainder holds {k} candidates, the step's list {self.k}")
        if state.grown is not None:
            self.grown.copy_(state.grown)
        grow = remainder.dropped.to(torch.uint8)
        out = self._claim(state, remainder.src, remainder.dst, remainder.weight, grow, -1, fresh=False)
        return state, out

    def _body(self, state: NetworkState, inputs: StepInputs) -> GrowthRemainder | None:
        """The device work of one step (no host synchronisation)."""
        self._level = state.units[LEVEL.name]
        self._lowk_fired = False
        self._clear_flags = False
        if self.ahead:
            return self._body_ahead(state, inputs)
        # selection that reads nothing the step writes runs on the side
        # stream, concurrently with the propagation passes
        early = self.side is not None and self._fires(state) and self.k > 0
        if early:
            self.side.wait_stream(torch.cuda.current_stream(self.dev))
            with torch.cuda.stream(self.side):
                self._select(state)
        self._scatter_inputs(state, inputs)
        if self.train_fused:
            self._train(state, inputs)
        else:
            self._forward(state)
            self._loss(state, inputs)
            self._backward(state)
            self._update_unit(state)
            self._update_conn(state)
        self._prune_unit(state)
        self._prune(state)
        self._add_unit(state)
        if early:
            torch.cuda.current_stream(self.dev).wait_stream(self.side)
        remainder = self._add_conn(state, selected=early)
        self._step_end()
        return remainder

    def _step_end(self) -> None:
        if self._plan_pending:
            # the next step's plan is made: join its stream
            torch.cuda.current_stream(self.dev).wait_stream(self.plan_stream)
            self._plan_pending = False
            self._plan_ready = True
        clear = self._clear_flags
        self._clear_flags = False
        K.step_end(self.step_dev, self.grown if clear else None, self.overflow if clear else None)
        self.launches += 1

    def _body_ahead(self, state: NetworkState, inputs: StepInputs) -> GrowthRemainder | None:
        """The step with its selection computed one step earlier: this step's
        winners come from the buffer the previous step's side branch filled,
        and the side stream selects the next step's while the passes, the
        claim and the insert run (it joins at the end of the step)."""
        main = torch.cuda.current_stream(self.dev)
        self._mark("start")
        if not self._ahead_ready:  # the first step of a bound state selects its own
            self._select(state, out=self.claim_next, step_dev=self.step_dev)
            self._ahead_ready = True
        if not self.shard_select and not self.late_io:
            # the list the previous step selected, its four columns in one launch
            K.select_take(self.k, 1, None, self.claim_next, self.claim_in)
            self.launches += 1
        torch.add(self.step_dev, 1, out=self.sel_step_dev)

        def select_next(ev=None):
            if ev is None:
                self.side.wait_stream(main)
            else:
                self.side.wait_event(ev)
            with torch.cuda.stream(self.side):
                self._select(state, out=self.claim_next, step_dev=self.sel_step_dev)

        if self.shard_select:
            # every rank's share of this step's list was stored before its
            # combine signalled: the barrier orders them before the take
            self._after_combine = self._take
        # the next step's selection reads only levels and the step counter;
        # it overlaps either the whole step, the step from the sweep's launch
        # on, or only what follows the propagation (the persistent sweep
        # holds every SM while it runs)
        at_launch = self.select_at_launch and self.use_mirror and not self.train_fused
        post = self.select_post_sweep and not at_launch and self.use_mirror and not self.train_fused
        if at_launch:
            self._sweep_fork = select_next
        elif post:
            self._post_fork = select_next
        elif not self.select_after_sweep:
            select_next()
        self._scatter_inputs(state, inputs)
        self._mark("inputs")
        if self.train_fused:
            self._train(state, inputs)
        else:
            self._forward(state)
            if (at_launch and self._sweep_fork is not None) or (post and self._post_fork is not None):
                # no sweep ran through the mirror (or without the lowest-|w| prune): fork here
                self._sweep_fork = self._post_fork = None
                select_next()
            if self.shard_select and not self._take_pending:
                # no combine ran: take the list here
                self._after_combine = None
                self._take()
            if self.select_after_sweep and not (at_launch or post):
                select_next()
            self._loss(state, inputs)
            self._backward(state)
            self._update_unit(state)
            self._update_conn(state)
        if self.select_after_sweep and self.train_fused:
            select_next()
        self._prune(state)
        remainder = self._add_conn(state, selected=True)
        self._step_end()
        self._mark("flags")
        main.wait_stream(self.side)
        self._mark("side_join")
        return remainder

    def capturable(self) -> bool:
        """Whether every step runs the same device work (a CUDA graph can
        replay it): growth fires every step and never raises on overflow."""
        ac = self.ac
        interval = int(getattr(self.net, "structural_interval", 1))
        if self.net.add_unit is not None and interval > 1:
            return False
        if isinstance(self.net.prune_conn, LowestMagnitudePrune) and self.net.prune_conn.every > 1:
            return False
        return ac is None or (ac.trigger == "every_step" and interval <= 1 and ac.on_overflow != "error")

    def _signature(self, state: NetworkState) -> tuple[bool, bool, bool]:
        """Which periodic phases this step runs: (growth on its trigger or
        interval, add_unit on its interval, a lowest-|w| prune on its
        period). Steps of one signature run the same device work."""
        net = self.net
        interval = int(getattr(net, "structural_interval", 1))
        unit = net.add_unit is not None and (interval <= 1 or state.step % interval == 0)
        grow = self.ac is not None and self._fires(state)
        pc = net.prune_conn
        low = isinstance(pc, LowestMagnitudePrune) and (pc.every <= 1 or state.step % pc.every == 0)
        return (grow, unit, low)

    def period(self) -> int:
        """The least common multiple of the periodic phases' periods: every
        signature occurs within this many steps."""
        import math

        net, ps = self.net, [1]
        interval = int(getattr(net, "structural_interval", 1))
        if interval > 1:
            ps.append(interval)
        trig = getattr(self.ac, "trigger", None)
        if isinstance(trig, tuple) and trig and trig[0] == "every":
            ps.append(int(trig[1]))
        pc = net.prune_conn
        if isinstance(pc, LowestMagnitudePrune) and pc.every > 1:
            ps.append(int(pc.every))
        return math.lcm(*ps)

    def _graph_safe(self, sig: tuple[bool, bool, bool]) -> bool:
        """Whether a step of this signature may be captured: no host read
        inside it (an overflow that must raise), no unit spawn."""
        grow, unit, _ = sig
        if unit:
            return False
        return not (grow and self.ac is not None and self.ac.on_overflow == "error")

    def _replay_or_capture(self, state: NetworkState, inputs: StepInputs):
        """With `auto_graphs`, a step of a signature seen before replays
        that signature's graph (captured here at its second occurrence);
        returns (ran, remainder). Without it, counts the signature."""
        sig = self._signature(state)
        entry = self._graphs.get(sig) if self.auto_graphs else None
        if entry is None or entry[0] != id(state):
            if (not self.auto_graphs or self._sig_seen.get((sig, id(state)), 0) < 1
                    or not self._graph_safe(sig)):
                self._sig_seen[(sig, id(state))] = self._sig_seen.get((sig, id(state)), 0) + 1
                return False, None
            x = torch.as_tensor(inputs.inputs, dtype=torch.float32).to(self.dev).reshape(-1).clone()
            t = None if inputs.targets is None else torch.as_tensor(inputs.targets, dtype=torch.float32).to(
                self.dev).reshape(-1).clone()
            gin = StepInputs(x, t)
            torch.cuda.synchronize(self.dev)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                rem = self._body(state, gin)
            entry = (id(state), g, gin, rem)
            self._graphs[sig] = entry
        _, g, gin, rem = entry
        self._copy_in(gin, inputs)
        g.replay()
        return True, rem

    @staticmethod
    def _copy_in(buf: StepInputs, inputs: StepInputs) -> None:
        x = inputs.inputs
        if not isinstance(x, torch.Tensor):
            x = torch.from_numpy(np.ascontiguousarray(x, np.float32))
        buf.inputs.copy_(x.reshape(-1), non_blocking=True)
        if inputs.targets is not None and buf.targets is not None:
            t = inputs.targets
            if not isinstance(t, torch.Tensor):
                t = torch.from_numpy(np.ascontiguousarray(t, np.float32))
            buf.targets.copy_(t.reshape(-1), non_blocking=True)

    def capture(self, state: NetworkState, inputs: StepInputs, *, keep_graph: bool = False,
                host_io: bool = False) -> None:
        """Capture one step of `state` as a CUDA graph; later calls with the
        same state replay it (inputs and targets are copied into the graph's
        input buffers first). Call after at least one eager step, so every
        kernel and index is initialised; the shapes of `inputs` (and
        targets) are fixed from then on. `keep_graph` keeps the cudaGraph_t
        (`self.graph.raw_cuda_graph()`), for a device-side loop over it.

        With `host_io` the step's host traffic is part of the graph: a call
        copies host inputs into pinned staging buffers (a host copy), the
        graph copies them to the device first and ends by copying the step's
        growth flags (grown, overflow as int32) into the pinned
        `self.host_flags`, valid once the stream has synchronised. A call
        waits until the previous replay is complete before it refills the
        staging buffers."""
        if not self.capturable():
            raise ValueError("this step's work depends on the step count (trigger or interval); it cannot be "
                             "replayed from one graph")
        self._bind(state)
        if self.plan_ahead and not self._plan_ready:
            raise ValueError("capture a step after at least one eager step of the bound state (the graph "
                             "expects the prune's plan made by the step before it)")
        x = torch.as_tensor(inputs.inputs, dtype=torch.float32).to(self.dev).reshape(-1).clone()
        t = None if inputs.targets is None else torch.as_tensor(inputs.targets, dtype=torch.float32).to(
            self.dev).reshape(-1).clone()
        self._graph_in = StepInputs(x, t)
        self._host_io = bool(host_io)
        if self._host_io:
            self._host_in = StepInputs(torch.empty(x.numel(), dtype=torch.float32).pin_memory(),
                                       None if t is None else torch.empty(t.numel(), dtype=torch.float32).pin_memory())
            self.host_flags = torch.zeros(2, dtype=torch.int32).pin_memory()
            self._io_done = torch.cuda.Event()
            in_dev = K.host_device_pointer(self._host_in.inputs)
            self._host_in_np = self._host_in.inputs.numpy()  # host copies without torch's dispatch
            flags_dev = K.host_device_pointer(self.host_flags)
        torch.cuda.synchronize(self.dev)
        self._drop_exec()
        prio = self.graph_priority and self.side is not None
        g = torch.cuda.CUDAGraph(keep_graph=keep_graph or prio)
        # with graph_priority the main stream's kernels are captured at high
        # priority, the side stream's (the next step's selection) at the
        # lowest, and the graph is instantiated to honour them
        cap = torch.cuda.Stream(device=self.dev, priority=-1) if prio else None
        with torch.cuda.graph(g, stream=cap):
            if self._host_io:
                # the first kernel reads the inputs from the pinned staging
                # buffer and the last writes the flags into the pinned ones:
                # no copy nodes (targets, when any, are copied)
                self._io_src = in_dev
                if t is not None:
                    self._graph_in.targets.copy_(self._host_in.targets, non_blocking=True)
            try:
                self._graph_rem = self._body(state, self._graph_in)
            finally:
                self._io_src = None
            if self._host_io:
                K.flags_out(state.grown, state.overflow, flags_dev)
        if prio:
            exec_ = ctypes.c_void_p()
            _lib.call("pxb_graph_instantiate", ctypes.c_void_p(g.raw_cuda_graph()), ctypes.c_int32(1),
                      ctypes.byref(exec_))
            self._graph_exec = exec_
        self.graph = g
        self._graph_state = id(state)
        self._graph_kept = keep_graph

    def _drop_exec(self) -> None:
        if getattr(self, "_graph_exec", None) is not None:
            _lib.call("pxb_graph_exec_destroy", self._graph_exec)
        self._graph_exec = None

    def release_graph(self) -> None:
        """Drop the captured graph and its buffers. A graph that holds NCCL
        calls must be released before the process group is destroyed."""
        self._drop_exec()
        self.graph = None
        self._graph_rem = None
        self._graph_in = None
        self._host_io = False
        self._graphs = {}
        self._sig_seen = {}

    def close(self) -> None:
        """Release the graph and the peer-memory group (collective under
        Scheme-A: every rank calls it, before the process group goes)."""
        self.release_graph()
        if self.peers is not None:
            self.peers.close()
            self.peers = None

    def __call__(self, state: NetworkState, inputs: StepInputs) -> StepResult:
        self._bind(state)
        if self.graph is not None and self._graph_state == id(state):
            x = inputs.inputs
            if not isinstance(x, torch.Tensor):
                x = torch.from_numpy(np.ascontiguousarray(x, np.float32))
            dst = self._graph_in
            if self._host_io:
                # the graph reads the staging buffers: the previous replay
                # must have read them
                self._io_done.synchronize()
                dst = self._host_in
                if x.device.type == "cpu":
                    self._host_in_np[:] = x.reshape(-1).numpy()
                else:
                    dst.inputs.copy_(x.reshape(-1))
            else:
                dst.inputs.copy_(x.reshape(-1), non_blocking=True)
            if inputs.targets is not None and dst.targets is not None:
                t = inputs.targets
                if not isinstance(t, torch.Tensor):
                    t = torch.from_numpy(np.ascontiguousarray(t, np.float32))
                dst.targets.copy_(t.reshape(-1), non_blocking=not self._host_io)
            if self._graph_exec is not None:
                _lib.call("pxb_graph_launch", self._graph_exec, K._stream())
            else:
                self.graph.replay()
            if self._host_io:
                self._io_done.record()
            remainder = self._graph_rem
        else:
            # eager steps are counted per signature even before auto_graphs
            # is set, so a later capture needs no further eager occurrence
            ran, remainder = (self._replay_or_capture(state, inputs) if not self.capturable() else (False, None))
            if not ran:
                remainder = self._body(state, inputs)
        state.step += 1
        grown = state.grown if state.grown is not None else torch.zeros((), dtype=torch.int32, device=self.dev)
        overflow = state.overflow if state.overflow is not None else torch.zeros((), dtype=torch.bool,
                                                                                 device=self.dev)
        return StepResult(state=state, overflow=overflow, loss=self.loss_buf[0], growth_remainder=remainder,
                          grown=grown)


def gather_arena(conns, static: NetworkStatic, out: dict | None = None, group=None) -> dict[str, torch.Tensor]:
    """The whole arena's (from_id, to_id, dead), bucket-major in global slot
    order, on every rank (src/plastax/phases.py:3863-3917, the per-connection
    proposer's `_gather_replicated` of the edge keys): rank r holds positions
    [r * cap / G, (r + 1) * cap / G) of each bucket, so one all-gather per
    column and bucket lays the bands end to end."""
    caps = [int(c) for c in static.level_capacities]
    total = sum(caps)
    dev = conns[0]["dead"].device
    if out is None:
        out = {"from_id": torch.empty(total, dtype=torch.int32, device=dev),
               "to_id": torch.empty(total, dtype=torch.int32, device=dev),
               "dead": torch.empty(total, dtype=torch.uint8, device=dev)}
    dist = _dist()
    off = 0
    for b, bucket in enumerate(conns):
        for col in ("from_id", "to_id", "dead"):
            dist.all_gather_into_tensor(out[col][off:off + caps[b]], bucket[col].contiguous(), group=group)
        off += caps[b]
    return out


def make_step(net: type[Network], static: NetworkStatic, *, batch_size: int | None = None, layout: str = "auto",
              fuse_prune: str | bool = "auto", growth: str = "auto", device: torch.device | str = "cuda",
              fuse_train: bool = True) -> StepFn:
    """Build the step for `net` on `static` (src/plastax/step.py:76-237).

    Raises ValueError for an unknown knob, as the reference does.
    `fuse_train=False` keeps a PIPELINE net's forward, loss, backward and
    update as separate passes where the fused training step would apply.
    """
    if layout not in ("auto", "edges", "csr", "triton", "xla"):
        raise ValueError(f"make_step: unknown layout {layout!r}")
    if growth not in ("auto", "xla", "triton"):
        raise ValueError(f"make_step: unknown growth engine {growth!r}")
    if fuse_prune not in ("auto", True, False):
        raise ValueError(f"make_step: unknown fuse_prune {fuse_prune!r}")
    if batch_size is not None:
        if batch_size < 1:
            raise ValueError("make_step: batch_size must be >= 1")
        if net.propagation is Propagation.PIPELINE:
            raise ValueError("make_step: batch_size is for TOPOLOGICAL (feed-forward) nets; a PIPELINE net carries "
                             "per-sample recurrent state between steps")
        if net.batch_reduction is None:
            raise ValueError(f"make_step: a batched step needs {net.__name__}.batch_reduction (e.g. "
                             "MeanFloatFirstRest())")
        from plastax_b200.batched import BatchedStepFn

        return BatchedStepFn(net, static, batch_size, torch.device(device))
    return StepFn(net, static, torch.device(device), fuse_prune=fuse_prune is not False, fuse_train=fuse_train)


def make_growth_retry(net: type[Network], static: NetworkStatic, *, device: torch.device | str = "cuda"):
    """The growth-only retry for a regrown static (src/plastax/step.py:320-356):
    `(state, remainder) -> (state, still dropped)`."""
    fn = StepFn(net, static, torch.device(device))
    return fn.retry
