"""The batched step, make_step(batch_size=B) (src/plastax/step.py:76-237).

For TOPOLOGICAL (feed-forward) nets: `StepInputs` carries (B, num_inputs)
inputs and (B, num_outputs) targets. Forward, loss and backward run per
sample against the shared connections, on unit columns laid out [N, B] (one
row of B samples per unit, csrc/batched.cu): each bucket's edges are read
once for the whole batch. The connection update is the exact batch-mean
gradient (src/plastax/phases.py:434-483). The per-sample unit columns then
reduce to the state's columns by the net's `batch_reduction`
(MeanFloatFirstRest: the batch mean of every float column), and prune and
growth run once on the reduced state, as the streaming step runs them.
`StepResult.loss` is the batch mean.
"""

from __future__ import annotations

import numpy as np
import torch

from plastax_b200 import _lib
from plastax_b200 import kernels as K
from plastax_b200.state import NetworkState, NetworkStatic
from plastax_b200.step import StepFn, StepInputs, StepResult
from plastax_b200.traits import (
    DestinationThresholdPrune,
    LowestMagnitudePrune,
    MagnitudePrune,
    MSELoss,
    Network,
    SoftmaxCrossEntropyLoss,
)
from plastax_b200.types import ACTIVATION, LEVEL


class BatchedStepFn:
    """A built batched step: [N, B] unit rows plus a streaming StepFn whose
    structural phases run on the reduced state."""

    def __init__(self, net: type[Network], static: NetworkStatic, batch_size: int, device: torch.device) -> None:
        if batch_size % 4 != 0 or batch_size > 1024:
            raise ValueError(f"make_step: the batched engine moves unit rows as float4: batch_size must be a "
                             f"multiple of 4 and at most 1024, got {batch_size}")
        if net.update_unit is not None or net.prune_unit is not None or net.add_unit is not None:
            raise NotImplementedError("a batched step has no unit-lifecycle lowering yet (update_unit runs per "
                                      "sample, prune_unit and add_unit on the reduced state)")
        if net.update_conn is not None and net.update_conn.kind == "upgd":
            raise NotImplementedError("a batched step has no UPGD lowering (the rule declares no exact "
                                      "per-sample / batch pair)")
        if net.forward_pass.combine.lowered() != "sum":
            raise NotImplementedError("a batched step lowers the linear (sum) forward only")
        if static.sharding is not None and static.num_shards > 1:
            raise NotImplementedError("a batched step under Scheme-A sharding has no engine lowering (its [N, B] "
                                      "partials would need a reduction per level)")
        self.net, self.static, self.dev, self.batch = net, static, device, int(batch_size)
        self.inner = StepFn(net, static, device)
        self.inner.use_mirror = False  # rows move per edge; the mirror serves the streaming sweep
        self.inner.acc_fixed = None
        self.inner.peer_reduce = False
        self.inner.ahead = False  # the structural phases run on the reduced state, in the step
        n, B = static.num_units, self.batch
        z = lambda: torch.zeros((n, B), dtype=torch.float32, device=device)  # noqa: E731
        self.act_b, self.acc_b = z(), z()
        bp, loss = net.backward_pass, net.loss
        self.grad_b = z() if bp is not None else None
        self.seed_b = z() if loss is not None else None
        self.loss_b = torch.zeros(B, dtype=torch.float32, device=device)
        self.launches = 0
        # the [N, B] rows an update_conn reads its gradient from
        self.upd_grad_b = None
        uc = net.update_conn
        if uc is not None:
            name = uc.grad_field.name
            if bp is not None and name == bp.grad_field.name:
                self.upd_grad_b = self.grad_b
            elif loss is not None and name == loss.seed_field.name:
                self.upd_grad_b = self.seed_b
            else:
                raise NotImplementedError(f"update_conn reads {name!r}, which no batched phase writes")

    @property
    def num_levels(self) -> int:
        return len(self.static.level_capacities)

    def _rows(self, x, cols: int) -> torch.Tensor:
        if not isinstance(x, torch.Tensor):
            x = torch.from_numpy(np.ascontiguousarray(x, np.float32))
        x = x.to(self.dev, dtype=torch.float32).reshape(self.batch, cols)
        return x.contiguous()

    def _prune(self, state: NetworkState) -> None:
        pc = self.net.prune_conn
        if pc is None:
            return
        if isinstance(pc, LowestMagnitudePrune):
            self.inner._prune_lowest(state, pc)
            return
        n = self.static.num_units
        for i, b in enumerate(state.conns):
            bm, bm_level = self.inner._bm(i)
            if isinstance(pc, MagnitudePrune):
                K.prune_conn(b, n, prune_kind=_lib.PRUNE_ABS_BELOW, threshold=pc.threshold, free_bitmap=bm,
                             bitmap_level=bm_level)
            elif isinstance(pc, DestinationThresholdPrune):
                K.prune_conn(b, n, prune_kind=_lib.PRUNE_ABS_BELOW_DST, unit_threshold=state.units[pc.field.name],
                             free_bitmap=bm, bitmap_level=bm_level)
            self.launches += 1

    def __call__(self, state: NetworkState, inputs: StepInputs) -> StepResult:
        net, inner, units = self.net, self.inner, state.units
        inner._bind(state)
        inner._level = units[LEVEL.name]
        level, is_input = units[LEVEL.name], inner.is_input
        L = self.num_levels
        x = self._rows(inputs.inputs, len(self.static.input_ids))
        self.act_b.index_copy_(0, inner.input_ids, x.t().contiguous())
        # forward, level by level (src/plastax/phases.py:972-1015)
        fp = net.forward_pass
        self.acc_b.zero_()
        for lv in range(L):
            K.batched_forward(state.conns[lv], self.act_b, self.acc_b)
            K.batched_unit_apply(self.acc_b, self.act_b, mode=0, act_kind=inner.fwd_act, level=level,
                                 target_level=lv + 1, is_input=is_input)
            self.launches += 2
        # loss, per sample; the batch mean to StepResult.loss
        loss = net.loss
        if loss is not None:
            if inputs.targets is None:
                raise ValueError("a network with a loss needs StepInputs.targets")
            t = self._rows(inputs.targets, len(self.static.output_ids))
            kind = _lib.LOSS_SOFTMAX_CE if isinstance(loss, SoftmaxCrossEntropyLoss) else _lib.LOSS_MSE
            if not isinstance(loss, (MSELoss, SoftmaxCrossEntropyLoss)):
                raise NotImplementedError(f"loss {type(loss).__name__} has no engine lowering")
            K.batched_loss(kind, inner.output_ids, self.batch, self.act_b, t, self.seed_b, self.loss_b,
                           inner.loss_buf)
            self.launches += 2
        # backward, deepest level first (src/plastax/phases.py:1049-1104)
        bp = net.backward_pass
        if bp is not None:
            self.acc_b.zero_()
            K.batched_unit_apply(self.acc_b, self.grad_b, mode=1, act_kind=inner.bwd_act, act=self.act_b,
                                 seed=self.seed_b, level=level, target_level=L, is_input=is_input)
            for lv in range(L - 1, 0, -1):
                K.batched_backward(state.conns[lv], self.grad_b, self.acc_b)
                K.batched_unit_apply(self.acc_b, self.grad_b, mode=1, act_kind=inner.bwd_act, act=self.act_b,
                                     seed=self.seed_b, level=level, target_level=lv, is_input=is_input)
                self.launches += 2
        # the exact batch-mean connection update (src/plastax/phases.py:434-483)
        if net.update_conn is not None:
            for b in state.conns:
                K.batched_update(b, self.upd_grad_b, self.act_b, inner.opt)
                self.launches += 1
        # per-sample unit columns -> the state's (batch_reduction)
        K.batch_mean(self.act_b, units[ACTIVATION.name])
        if bp is not None:
            K.batch_mean(self.grad_b, units[bp.grad_field.name])
        if loss is not None:
            K.batch_mean(self.seed_b, units[loss.seed_field.name])
        # structural phases once, on the reduced state
        self._prune(state)
        inner._clear_flags = False
        remainder = inner._add_conn(state)
        inner._step_end()
        state.step += 1
        grown = state.grown if state.grown is not None else torch.zeros((), dtype=torch.int32, device=self.dev)
        overflow = state.overflow if state.overflow is not None else torch.zeros((), dtype=torch.bool,
                                                                                 device=self.dev)
        return StepResult(state=state, overflow=overflow, loss=inner.loss_buf[0], growth_remainder=remainder,
                          grown=grown)


__all__ = ["BatchedStepFn"]
