"""Reference-order step restatements built from the oracle primitives.

TEST INFRASTRUCTURE ONLY (the checker and the CPU baseline; the engine never
imports it). Each step runs the reference's phase order
(src/plastax/phases.py:87-176) with the oracle's sequential primitives.
"""

from __future__ import annotations

import numpy as np

from oracle import oracle as orc


def lowbias32(x: np.ndarray) -> np.ndarray:
    """The lowbias32 integer hash (the one the claim-digest tests hash with,
    tests/test_growth_claim.py:34-41 of the reference)."""
    x = x.astype(np.uint32)
    x = x ^ (x >> np.uint32(16))
    x = (x * np.uint32(0x7FEB352D)).astype(np.uint32)
    x = x ^ (x >> np.uint32(15))
    x = (x * np.uint32(0x846CA68B)).astype(np.uint32)
    return x ^ (x >> np.uint32(16))


def init_weight(kind: str, a: float, src: np.ndarray, dst: np.ndarray, salt: int = 0) -> np.ndarray:
    """Growth init weights of the recognised rules (see plastax_b200.traits)."""
    if kind == "const":
        return np.full(src.shape, a, np.float32)
    if kind == "dyadic":
        return (((3 * src.astype(np.int64) + 5 * dst) % 16 - 8) / 8.0).astype(np.float32)
    h = lowbias32(np.uint32(0x9E3779B9) ^ src.astype(np.uint32))
    h = lowbias32(h ^ dst.astype(np.uint32))
    h = lowbias32(h ^ np.uint32(salt))
    u = (h >> np.uint32(8)).astype(np.float32) * np.float32(1.0 / 16777216.0)
    return (np.float32(a) * (np.float32(2.0) * u - np.float32(1.0))).astype(np.float32)


def lowest_prune(buckets: list[dict], k: int) -> int:
    """Tombstone the k live edges of lowest |w| over the buckets in order
    (ties by ascending global slot; NaN weights never selected), in place;
    returns the number pruned. The engine's LowestMagnitudePrune."""
    w = np.concatenate([np.abs(b["weight"].astype(np.float32)) for b in buckets])
    live = np.concatenate([b["dead"] == 0 for b in buckets]) & ~np.isnan(w)
    slots = np.flatnonzero(live)
    order = slots[np.lexsort((slots, w[slots]))][:k]
    base = 0
    for b in buckets:
        cap = b["dead"].size
        sel = order[(order >= base) & (order < base + cap)] - base
        b["dead"][sel] = 1
        base += cap
    return int(order.size)


class ReservoirOracle:
    """The reservoir churn step (PIPELINE: forward, prune, per-unit
    proposal growth with a step-scoped cap, pipeline claim) on host arrays.
    `prune` "lowest_k": the k live edges of lowest |w| go every step (ties
    by slot); "threshold": every edge with |w| < tau."""

    def __init__(self, bucket: dict, act: np.ndarray, level: np.ndarray, tail_start: int, *, num_inputs: int,
                 num_res: int, tau: float, k: int, init_a: float, seed: int = 0, threads: int = 1,
                 prune: str = "lowest_k") -> None:
        if prune not in ("lowest_k", "threshold"):
            raise ValueError(f"unknown prune {prune!r}")
        self.b, self.act, self.level = bucket, act, level
        self.tail = int(tail_start)
        self.n = act.size
        self.num_inputs, self.num_res = num_inputs, num_res
        self.tau, self.k, self.init_a, self.seed = tau, k, init_a, seed
        self.prune = prune
        self.last_pruned = 0
        self.threads = threads
        self.is_input = np.zeros(self.n, np.uint8)
        self.is_input[:num_inputs] = 1
        self.step_count = 0
        self.last_counts = np.zeros(4, np.int32)

    def step(self, inputs: np.ndarray) -> None:
        n, b = self.n, self.b
        self.act[: self.num_inputs] = inputs
        acc = np.zeros(n, np.float32)
        lowest = self.prune == "lowest_k"
        if self.threads > 1:
            # the forward with the threshold prune fused (a threshold of 0
            # prunes nothing: the lowest-k prune runs after it)
            orc.forward_prune_mt(b, self.act, n, 0.0 if lowest else self.tau, acc, self.threads)
        else:
            orc.forward_accumulate(b, self.act, n, "sum", acc)
        orc.unit_apply(n, 0, "tanh", "sum", acc, None, None, None, 0, self.is_input, None, self.act)
        if lowest:
            self.last_pruned = orc.lowest_prune(b, self.k, self.threads)
        elif self.threads <= 1:
            dead0 = int(b["dead"].sum())
            orc.prune(b, n, 1, self.tau)
            self.last_pruned = int(b["dead"].sum()) - dead0
        th = self.threads
        src, dst, score = orc.propose_per_unit(n, 1, self.seed, self.step_count, self.num_inputs, self.num_res, 0,
                                               self.level, max_level_gap=1, threads=th)
        perm = orc.total_order(score, src, dst, threads=th)
        win = orc.select_step(perm, src, self.level, self.k)
        cs, cd = src[win].copy(), dst[win].copy()
        cw = init_weight("hash_uniform", self.init_a, cs, cd)
        grow = np.isfinite(score[win]).astype(np.uint8)
        if win.size < self.k:  # padding entries are not growable
            pad = self.k - win.size
            cs = np.concatenate([cs, np.zeros(pad, np.int32)])
            cd = np.concatenate([cd, np.zeros(pad, np.int32)])
            cw = np.concatenate([cw, np.zeros(pad, np.float32)])
            grow = np.concatenate([grow, np.zeros(pad, np.uint8)])
        self.last_counts, _, self.tail = orc.claim_pipeline(b, self.level, self.tail, cs, cd, cw, grow, threads=th)
        self.step_count += 1


class EsnOracle:
    """The ESN step (PIPELINE): inputs scattered, one forward sweep from the
    previous activations (sum accumulated in double, rounded once), tanh on
    the reservoir and identity on the readout, the MSE seed on the readout,
    then LMS on every live edge (w -= lr * seed[dst] * act[src]; zero seed
    on every other unit, an exact no-op there)."""

    def __init__(self, bucket: dict, act: np.ndarray, *, input_id: int, output_id: int, lr: float) -> None:
        self.b, self.act = bucket, act
        self.n = act.size
        self.input_id, self.output_id, self.lr = input_id, output_id, lr
        self.seed = np.zeros(self.n, np.float32)
        self.skip = np.zeros(self.n, np.uint8)
        self.skip[[input_id, output_id]] = 1

    def step(self, x: float, target: float) -> float:
        n = self.n
        self.act[self.input_id] = np.float32(x)
        acc = np.zeros(n, np.float32)
        orc.forward_accumulate(self.b, self.act, n, "sum", acc)
        new = self.act.copy()
        orc.unit_apply(n, 0, "tanh", "sum", acc, None, None, None, 0, self.skip, None, new)
        new[self.output_id] = acc[self.output_id]
        self.act = new
        err = np.float32(new[self.output_id] - np.float32(target))
        self.seed[:] = 0
        self.seed[self.output_id] = err
        orc.update_conn(self.b, self.seed, self.act, n, dict(kind="sgd", lr=self.lr))
        return float(np.float32(np.float32(0.5) * err * err))


class DstOracle:
    """The dynamic-sparse-training step (PIPELINE, the engine's phase order,
    src/plastax/phases.py:87-176): inputs scattered; the forward from the
    previous activations (tanh, the outputs linear); the MSE seed on the
    outputs; the pipelined backward from the previous step's gradients
    (grad = (acc + seed) * act'); SGD on every live edge
    (w -= lr * grad[dst] * act[src]); every `every` steps the k live edges of
    lowest |w| pruned, then per-unit proposals (P per unit, dst uniform over
    the non-input units, score |grad[dst] * act[src]|) ranked in the total
    order, the first k claimed with weight 0 (the pipeline claim).

    `teacher_force(...)` overwrites the float state (weights, activations,
    gradients) with another implementation's before a structural phase, so
    the structure can be compared bit for bit while the float sums drift
    apart within tolerance."""

    def __init__(self, bucket: dict, act: np.ndarray, grad: np.ndarray, level: np.ndarray, tail_start: int, *,
                 num_inputs: int, num_outputs: int, lr: float, k: int, every: int, proposals: int, seed: int = 0,
                 threads: int = 1) -> None:
        self.b, self.act, self.grad, self.level = bucket, act, grad, level
        self.n = act.size
        self.tail = int(tail_start)
        self.num_inputs, self.num_outputs = num_inputs, num_outputs
        self.out = np.arange(self.n - num_outputs, self.n)
        self.lr, self.k, self.every, self.P, self.seed_ = lr, k, every, proposals, seed
        self.threads = threads
        self.is_input = np.zeros(self.n, np.uint8)
        self.is_input[:num_inputs] = 1
        self.seed = np.zeros(self.n, np.float32)
        self.step_count = 0
        self.last_counts = np.zeros(4, np.int32)
        self.last_pruned = 0

    def forward_phase(self, x: np.ndarray, t: np.ndarray) -> float:
        n, b = self.n, self.b
        self.act[: self.num_inputs] = x
        acc = np.zeros(n, np.float32)
        orc.forward_accumulate(b, self.act, n, "sum", acc)
        new = self.act.copy()
        orc.unit_apply(n, 0, "tanh", "sum", acc.copy(), None, None, None, 0, self.is_input, None, new)
        new[self.out] = acc[self.out]
        self.act[:] = new
        diff = (self.act[self.out] - np.asarray(t, np.float32)).astype(np.float32)
        self.seed[:] = 0
        self.seed[self.out] = diff
        loss = np.float32(0)
        for d in diff:
            loss = np.float32(loss + np.float32(np.float32(0.5) * d) * d)
        acc = np.zeros(n, np.float32)
        orc.backward_accumulate(b, self.grad, n, "sum", acc)
        newg = self.grad.copy()
        # every unit, inputs included (src/plastax/sweep.py:402-450); the
        # linear outputs' derivative is 1
        orc.unit_apply(n, 1, "tanh", "sum", acc.copy(), self.act, self.seed, None, 0, None, None, newg)
        newg[self.out] = (acc[self.out] + self.seed[self.out]).astype(np.float32)
        self.grad[:] = newg
        orc.update_conn(b, self.grad, self.act, n, dict(kind="sgd", lr=self.lr))
        return float(loss)

    def fires(self) -> bool:
        return self.step_count % self.every == 0

    def teacher_force(self, weight: np.ndarray, act: np.ndarray, grad: np.ndarray) -> None:
        self.b["weight"][:] = weight
        self.act[:] = act
        self.grad[:] = grad

    def structural_phase(self) -> None:
        n, b = self.n, self.b
        self.last_pruned = orc.lowest_prune(b, self.k, self.threads)
        src, dst, score = orc.propose_per_unit(n, self.P, self.seed_, self.step_count, self.num_inputs,
                                               n - self.num_inputs, 2, self.level, grad=self.grad, act=self.act,
                                               max_level_gap=1, threads=self.threads)
        perm = orc.total_order(score, src, dst, threads=self.threads)
        win = orc.select_step(perm, src, self.level, self.k)
        cs, cd = src[win].copy(), dst[win].copy()
        cw = np.zeros(cs.size, np.float32)
        grow = np.isfinite(score[win]).astype(np.uint8)
        if win.size < self.k:
            pad = self.k - win.size
            cs = np.concatenate([cs, np.zeros(pad, np.int32)])
            cd = np.concatenate([cd, np.zeros(pad, np.int32)])
            cw = np.concatenate([cw, np.zeros(pad, np.float32)])
            grow = np.concatenate([grow, np.zeros(pad, np.uint8)])
        self.last_counts, _, self.tail = orc.claim_pipeline(b, self.level, self.tail, cs, cd, cw, grow,
                                                            threads=self.threads)

    def step(self, x: np.ndarray, t: np.ndarray) -> float:
        loss = self.forward_phase(x, t)
        if self.fires():
            self.structural_phase()
        self.step_count += 1
        return loss


class UnitsOracle:
    """The unit-lifecycle step (TOPOLOGICAL, single device; the engine's phase
    order, src/plastax/phases.py:87-176): UPGD's local scale (the max of each
    destination's incoming utilities, examples/upgd.py:83-128); the forward
    level by level (ReLU, the output linear); the MSE seed; the backward level
    by level; the utility trace update; UPGD on every live edge; the units
    below the utility quantile pruned; every `interval` steps one unit
    spawned from the highest-utility parent. Growth is not part of it: the
    per-unit proposals run every `interval` steps on a few thousand units and
    the step's cost is the propagation. Composed from the oracle's parts,
    each checked on its own against the GPU."""

    def __init__(self, buckets: list[dict], units: dict, *, input_ids, output_ids, num_levels: int, net,
                 trace: str = "utility") -> None:
        from oracle import units as ou
        from oracle import upgd as og

        self.ou, self.og = ou, og
        self.b, self.u = buckets, units
        self.n = units["activation"].size
        self.inputs, self.outputs = np.asarray(input_ids), np.asarray(output_ids)
        self.L = num_levels
        self.net = net
        self.trace = trace
        self.is_input = np.zeros(self.n, np.uint8)
        self.is_input[self.inputs] = 1
        self.exempt = np.zeros(self.n, bool)
        self.exempt[np.concatenate([self.inputs, self.outputs])] = True
        self.defaults = {k: np.zeros((), v.dtype) for k, v in units.items() if k not in ("level", "pruned")}
        uc = net.update_conn
        self.kw = dict(lr=uc.lr, beta=uc.b1, sigma=uc.b2, eps=uc.eps)
        self.interval = int(net.structural_interval)
        self.count = 0

    def step(self, x: np.ndarray, t: np.ndarray) -> float:
        ou, og, u, n = self.ou, self.og, self.u, self.n
        level, pruned, act = u["level"], u["pruned"], u["activation"]
        nb, out = len(self.b), self.outputs
        eta = og.eta_local(self.b, n, "upgd/util", u["upgd/eta"], self.is_input.astype(bool))
        u["upgd/eta"][:] = eta
        act[self.inputs] = x
        # bucket l holds the edges into level l + 1
        acc = np.zeros(n, np.float32)
        for lv in range(nb):
            orc.forward_accumulate(self.b[lv], act, n, "sum", acc)
            pre = acc[out].copy()
            orc.unit_apply(n, 0, "relu", "sum", acc, None, None, level, lv + 1, self.is_input, pruned, act)
            top = level[out] == lv + 1
            act[out[top]] = pre[top]  # the linear output
        seed = u["loss_grad"]
        seed[:] = 0
        diff = (act[out] - np.asarray(t, np.float32)).astype(np.float32)
        seed[out] = diff
        loss = np.float32(0)
        for d in diff:
            loss = np.float32(loss + np.float32(np.float32(0.5) * d) * d)
        grad = u["grad_pre_act"]
        acc = np.zeros(n, np.float32)
        for lv in range(nb, 0, -1):
            if lv < nb:
                orc.backward_accumulate(self.b[lv], grad, n, "sum", acc)
            pre = acc[out].copy()
            orc.unit_apply(n, 1, "relu", "sum", acc, act, seed, level, lv, self.is_input, pruned, grad)
            top = level[out] == lv
            grad[out[top]] = (pre[top] + seed[out[top]]).astype(np.float32)
        ou.update_unit(u, pruned, self.net.update_unit)
        for b in self.b:
            og.update(b, grad, act, eta, **self.kw)
        ou.prune_unit(u, pruned, self.exempt, self.defaults, self.b, self.net.prune_unit)
        if self.interval <= 1 or self.count % self.interval == 0:
            ou.add_unit(u, pruned, level, self.defaults, self.net.add_unit, int(self.net.max_levels))
        self.count += 1
        return float(loss)
