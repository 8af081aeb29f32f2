"""The host driver (src/plastax/driver.py): the step loop with exact regrow
on overflow and resort, and `scan`, a chunk of steps run as one device-side
loop.

`Driver.step` runs one step; if its growth overflowed, every full bucket
grows (`grow_bucket`) and the candidates the claim dropped claim the new
room (`StepFn.retry`) until none is left, so the step commits exactly what
it would have with the larger buckets (src/plastax/driver.py:134-168).
Then a TOPOLOGICAL net whose `needs_resort` is raised resorts; a PIPELINE
net never does. `check_every=N > 1` reads the flags every N steps only, with
the reference's relaxed semantics (src/plastax/driver.py:340-360).

`Driver.scan` runs a chunk of K steps without a host round trip per step:
the step's CUDA graph is the body of a conditional WHILE node
(csrc/loop.cu) that copies row i of the chunk into the step's inputs, runs
the step, records the loss (or the outputs' activations) into row i, and
stops itself right after a step that overflowed or needs a resort. The host
then completes that step as `step` does, rebuilds the step for the new
static configuration and re-enters the loop at the next row, so the result
is step for step what K calls of `step` produce
(src/plastax/driver.py:170-317).
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from plastax_b200 import _lib
from plastax_b200 import kernels as K
from plastax_b200.state import NetworkState, NetworkStatic, grow_bucket, live_conn_count
from plastax_b200.step import GrowthRemainder, StepFn, StepInputs, make_step
from plastax_b200.topo import resort
from plastax_b200.traits import Network
from plastax_b200.types import ACTIVATION, Propagation


class _Loop:
    """One built device-side loop over a captured step graph."""

    def __init__(self, fn: StepFn, rows: int, x: torch.Tensor, t: torch.Tensor | None, counter: torch.Tensor,
                 status: torch.Tensor, loss_rec: torch.Tensor | None, out_rec: torch.Tensor | None,
                 out_ids: torch.Tensor | None, state: NetworkState, resorts: bool) -> None:
        gi = fn._graph_in
        p = K.ptr
        self.desc = _lib.LoopDesc(
            p(counter), rows, p(x), x.shape[1], p(gi.inputs), p(t), 0 if t is None else t.shape[1],
            p(gi.targets) if t is not None else None, p(fn.loss_buf), p(loss_rec), p(state.units[ACTIVATION.name]),
            p(out_ids), 0 if out_ids is None else out_ids.numel(), p(out_rec),
            p(state.overflow) if state.overflow is not None else None,
            p(state.needs_resort) if state.needs_resort is not None else None, 1 if resorts else 0, p(status))
        handle = ctypes.c_void_p()
        _lib.call("pxb_loop_build", ctypes.c_void_p(fn.graph.raw_cuda_graph()), ctypes.byref(self.desc),
                  ctypes.byref(handle))
        self.handle = handle
        self.fn = fn

    def launch(self) -> None:
        _lib.call("pxb_loop_launch", self.handle, K._stream())

    def close(self) -> None:
        if self.handle:
            _lib.call("pxb_loop_destroy", self.handle)
            self.handle = None

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:  # noqa: BLE001 -- interpreter shutdown
            pass


class Driver:
    """Runs a network's step loop, owning regrow on overflow and resort
    (src/plastax/driver.py:65-132)."""

    def __init__(self, net: type[Network], static: NetworkStatic, state: NetworkState, *, check_every: int = 1,
                 batch_size: int | None = None, layout: str = "auto", fuse_prune: str | bool = "auto",
                 growth: str = "auto", device: torch.device | str = "cuda", graphs: bool = False) -> None:
        if check_every < 1:
            raise ValueError(f"Driver: check_every must be >= 1, got {check_every}")
        self._net, self._static, self._state = net, static, state
        self._batch_size, self._layout, self._fuse_prune, self._growth = batch_size, layout, fuse_prune, growth
        self.dev = torch.device(device)
        self._resorts = net.propagation is Propagation.TOPOLOGICAL
        # with graphs, a step whose periodic phases (growth, unit spawn,
        # prune) follow a schedule replays one CUDA graph per signature
        # (StepFn.auto_graphs); the steps that read the host stay eager
        self._graphs = graphs
        self._check_every = check_every
        self._since_check = 0
        self._overflowed = torch.zeros((), dtype=torch.bool, device=self.dev)
        self._step = self._make_step()
        self._loop: _Loop | None = None
        self._loop_key = None
        self._counter = torch.zeros(1, dtype=torch.int32, device=self.dev)
        self._bufs: dict = {}
        self._out_ids = torch.tensor(static.output_ids, dtype=torch.int32, device=self.dev)
        self._status = torch.zeros(1, dtype=torch.int32, device=self.dev)
        self.retraces = 0  # step rebuilds after a regrow or a resort
        self.last_loss: torch.Tensor | None = None  # the last `step`'s loss (device scalar)

    # -- the reference's API ------------------------------------------------
    @property
    def state(self) -> NetworkState:
        return self._state

    @property
    def static(self) -> NetworkStatic:
        return self._static

    def step(self, inputs: StepInputs) -> None:
        """One exact step: complete an overflowing growth, then resort
        (src/plastax/driver.py:134-168)."""
        if self._check_every > 1:
            self._deferred_step(inputs)
            return
        result = self._step(self._state, inputs)
        self.last_loss = result.loss
        state = self._complete_growth(result.state, result.growth_remainder)
        self._check_mirrors()
        self._state = self._resort_if_due(state)

    def scan(self, inputs: StepInputs, *, record: str | None = None, steps: int | None = None) -> torch.Tensor:
        """Run a chunk of steps as one device-side loop; exact, like `step`
        (src/plastax/driver.py:170-260).

        `inputs.inputs` is (K, num_inputs) (targets (K, num_outputs)).
        `record` None keeps each step's loss ((K,) on the device), "outputs"
        the output units' activations ((K, num_outputs)); rows at or beyond
        `steps` are zero."""
        x = self._chunk(inputs.inputs, "inputs", "x")
        length = x.shape[0]
        t = None if inputs.targets is None else self._chunk(inputs.targets, "targets", "t")
        if t is not None and t.shape[0] != length:
            raise ValueError(f"Driver.scan: targets chunk axis ({t.shape[0]},) does not match the inputs' "
                             f"({length},)")
        count = length if steps is None else int(steps)
        if not 0 <= count <= length:
            raise ValueError(f"Driver.scan: steps must be in [0, {length}], got {steps}")
        if record not in (None, "outputs"):
            raise ValueError(f"Driver.scan: record must be None (the loss) or 'outputs', got {record!r}")
        out_ids = None
        shape: tuple = (length,)
        if record == "outputs":
            out_ids = self._out_ids
            shape = (length, out_ids.numel())
        recs = self._buffer(("rec", record), shape)
        recs.zero_()
        start = 0
        while start < count:
            fn = self._step
            if not isinstance(fn, StepFn) or not fn.capturable():
                # no single graph replays this step: the host loop, recording on the device
                self._record_eager(x, t, start, recs, out_ids)
                start += 1
                continue
            if fn.graph is None or fn._graph_state != id(self._state) or not fn._graph_kept:
                # a fresh step: one eager step initialises it, then the capture
                self._record_eager(x, t, start, recs, out_ids)
                start += 1
                if start >= count or self._step is not fn:
                    continue
                fn.capture(self._state, StepInputs(x[start], None if t is None else t[start]), keep_graph=True)
                self._drop_loop()
            key = (id(fn), fn._graph_state, x.data_ptr(), length, count, None if t is None else t.data_ptr(),
                   recs.data_ptr(), record)
            if self._loop is None or self._loop_key != key:
                self._drop_loop()
                self._loop = _Loop(fn, count, x, t, self._counter, self._status,
                                   recs if record is None else None, recs if record == "outputs" else None, out_ids,
                                   self._state, self._resorts)
                self._loop_key = key
            self._counter.fill_(start)
            self._loop.launch()
            done, halted = divmod(int(self._status.item()), 2)
            ran = done - start
            self._state.step += ran
            self._check_mirrors()
            if halted:
                # finish step done - 1 on the host (its remainder is the graph's)
                state = self._complete_growth(self._state, fn._graph_rem)
                self._state = self._resort_if_due(state)
            start = done
        return recs.clone()

    # -- internals ------------------------------------------------------------
    def _buffer(self, key, shape: tuple) -> torch.Tensor:
        """A persistent device buffer (the loop graph bakes in its address)."""
        buf = self._bufs.get(key)
        if buf is None or tuple(buf.shape) != tuple(shape):
            buf = torch.zeros(shape, dtype=torch.float32, device=self.dev)
            self._bufs[key] = buf
        return buf

    def _chunk(self, a, what: str, key: str) -> torch.Tensor:
        if not isinstance(a, torch.Tensor):
            a = torch.from_numpy(np.ascontiguousarray(a, np.float32))
        if a.ndim < 2:
            raise ValueError(f"Driver.scan: {what} need a leading chunk axis, got shape {tuple(a.shape)}")
        a = a.reshape(a.shape[0], -1)
        buf = self._buffer(("chunk", key), tuple(a.shape))
        buf.copy_(a, non_blocking=True)
        return buf

    def _record_eager(self, x, t, row: int, recs: torch.Tensor, out_ids) -> None:
        self.step(StepInputs(x[row], None if t is None else t[row]))
        if out_ids is not None:
            recs[row] = self._state.units[ACTIVATION.name][out_ids.long()]
        elif self.last_loss is not None:
            recs[row] = self.last_loss

    def _drop_loop(self) -> None:
        if self._loop is not None:
            self._loop.close()
        self._loop = None
        self._loop_key = None

    def _check_mirrors(self) -> None:
        """Read every device status word of the step (raising PxbError for a
        fault: a bulk copy or peer wait that gave up, a selection bin or
        prune list that overflowed) and rebuild the step's mirrors when one
        lost an edge (its inserts found no room): the canonical arena stays
        complete, so a rebuild restores the sweep's input exactly."""
        fn = self._step
        if isinstance(fn, StepFn) and not fn.mirrors_healthy():
            self._drop_loop()
            fn.invalidate()

    def _make_step(self):
        fn = make_step(self._net, self._static, batch_size=self._batch_size, layout=self._layout,
                       fuse_prune=self._fuse_prune, growth=self._growth, device=self.dev)
        if self._graphs and isinstance(fn, StepFn):
            fn.auto_graphs = True
        return fn

    def _rebuild(self) -> None:
        self._drop_loop()
        close = getattr(self._step, "close", None)
        if close is not None:
            close()
        self._step = self._make_step()
        self.retraces += 1

    def _free_slots(self, state: NetworkState, level: int) -> int:
        """Slots any level can still claim in bucket `level`
        (src/plastax/driver.py:373-383)."""
        capacity = self._static.level_capacities[level]
        if self._static.propagation is Propagation.PIPELINE:
            return capacity - int(state.tail_start.item())
        return capacity - live_conn_count(state, level)

    def _complete_growth(self, state: NetworkState, remainder) -> NetworkState:
        """Regrow every full bucket and claim the dropped candidates until
        none is left (src/plastax/driver.py:319-331)."""
        while state.overflow is not None and bool(state.overflow.item()):
            if remainder is None:
                raise RuntimeError("Driver: a step overflowed without a growth remainder")
            # the remainder's columns live in the old step's buffers: keep them
            remainder = GrowthRemainder(remainder.src.clone(), remainder.dst.clone(), remainder.weight.clone(),
                                        remainder.dropped.clone())
            grew = False
            for level in range(len(self._static.level_capacities)):
                if self._free_slots(state, level) == 0:
                    self._static, state = grow_bucket(self._static, state, level)
                    grew = True
            if not grew:
                raise RuntimeError("Driver: the growth overflowed but no bucket is full; the dropped candidates "
                                   "have nowhere to go")
            self._rebuild()
            state, remainder = self._step.retry(state, remainder)
        return state

    def _resort_if_due(self, state: NetworkState) -> NetworkState:
        """Resort a TOPOLOGICAL net whose flag is raised; PIPELINE never
        (src/plastax/driver.py:333-338)."""
        if self._resorts and state.needs_resort is not None and bool(state.needs_resort.item()):
            self._static, state = resort(self._static, state)
            self._rebuild()
        return state

    def _deferred_step(self, inputs: StepInputs) -> None:
        """One check_every > 1 step (src/plastax/driver.py:340-360)."""
        result = self._step(self._state, inputs)
        self.last_loss = result.loss
        self._state = result.state
        if result.overflow is not None:
            self._overflowed |= result.overflow
        self._since_check += 1
        if self._since_check < self._check_every:
            return
        self._since_check = 0
        self._check_mirrors()
        if bool(self._overflowed.item()):
            self._overflowed.zero_()
            ac = self._net.add_conn
            want = (getattr(ac, "max_new_per_level", None) or 1) if ac is not None else 1
            state = self._state
            grew = False
            for level in range(len(self._static.level_capacities)):
                if self._free_slots(state, level) < want:
                    self._static, state = grow_bucket(self._static, state, level)
                    grew = True
            self._state = state
            if grew:
                self._rebuild()
        self._state = self._resort_if_due(self._state)

    def close(self) -> None:
        self._drop_loop()
        close = getattr(self._step, "close", None)
        if close is not None:
            close()


__all__ = ["Driver"]
