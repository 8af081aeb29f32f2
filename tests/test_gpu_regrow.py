"""Regrow, growth retry and resort on the device (src/plastax/state.py:238-313,
src/plastax/step.py:320-356, src/plastax/phases.py:5206-5290,
src/plastax/topo.py:303-452).

- An overflowing step, then grow_bucket and the growth retry, leaves exactly
  the arena a step on the bigger bucket would have (the reference's claim:
  the remainder lands where growth would have put it had the bucket been that
  large from the start).
- resort keeps the live edges, recomputes the levels, compacts every bucket
  stably by source (old relative order within a source) and resets the
  pipeline tail; it equals a numpy restatement of the same rule.
"""

from __future__ import annotations

import dataclasses

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _net(k, thr):
    import plastax_b200 as px

    class Net(px.Network):
        forward_pass = px.ForwardPass("tanh")
        propagation = px.Propagation.PIPELINE
        prune_conn = px.MagnitudePrune(thr)
        add_conn = px.ProposeAddConn(proposals_per_proposer=1, max_new_per_level=k, dst_lo=2,
                                     level_cap_scope="step", init=("hash_uniform", 0.2))

    return Net


def _arena(cuda, Net, n=800, e=6000, seed=71):
    import plastax_b200 as px

    rng = np.random.default_rng(seed)
    src, dst = rng.integers(0, n, e), rng.integers(2, n, e)
    w = (rng.standard_normal(e) * 0.1).astype(np.float32)
    return px.NetworkBuilder.from_edges(Net, n, src, dst, weights=w, input_ids=(0, 1), output_ids=(),
                                        capacity_headroom=0.0, capacity_align=64, device=cuda)


def test_overflow_grow_and_retry_equals_the_bigger_bucket(cuda):
    import torch

    import plastax_b200 as px

    Net = _net(700, 0.001)
    static, state = _arena(cuda, Net)
    # the same arena, grown before the step
    big_static, big_state = px.grow_bucket(static, dataclasses.replace(
        state, conns=tuple({k: v.clone() for k, v in b.items()} for b in state.conns),
        units={k: v.clone() for k, v in state.units.items()}, tail_start=state.tail_start.clone()), 0)
    x = px.StepInputs(np.ones(2, np.float32))
    res = px.make_step(Net, static, device=cuda)(state, x)
    assert bool(res.overflow.item()), "the tight bucket must overflow"
    grown_first = int(res.grown.item())
    new_static, state = px.grow_bucket(static, state, 0)
    assert new_static.level_capacities == big_static.level_capacities
    retry = px.make_growth_retry(Net, new_static, device=cuda)
    state, rem = retry(state, res.growth_remainder)
    assert not bool(state.overflow.item())
    big = px.make_step(Net, big_static, device=cuda)(big_state, x)
    assert int(state.grown.item()) == int(big.grown.item()) > grown_first
    for col in ("from_id", "to_id", "dead", "weight"):
        np.testing.assert_array_equal(state.conns[0][col].cpu().numpy(), big_state.conns[0][col].cpu().numpy(),
                                      err_msg=col)
    assert int(state.tail_start.item()) == int(big_state.tail_start.item())
    assert int(rem.dropped.sum().item()) == 0
    torch.cuda.synchronize()


def _resort_reference(b, n):
    """Live edges in old order, stably ordered by source, padded with dead."""
    live = b["dead"] == 0
    idx = np.flatnonzero(live)
    order = idx[np.argsort(b["from_id"][idx], kind="stable")]
    return {k: v[order] for k, v in b.items()}


def test_resort_compacts_and_relevels(cuda):
    import torch

    import plastax_b200 as px

    Net = _net(300, 0.05)
    static, state = _arena(cuda, Net, seed=72)
    step = px.make_step(Net, static, device=cuda)
    for i in range(4):
        step(state, px.StepInputs(np.full(2, 0.5 * i, np.float32)))
    before = {k: v.cpu().numpy() for k, v in state.conns[0].items()}
    new_static, new_state = px.resort(static, state)
    after = {k: v.cpu().numpy() for k, v in new_state.conns[0].items()}
    want = _resort_reference(before, static.num_units)
    live = int((before["dead"] == 0).sum())
    assert int(new_state.tail_start.item()) == live
    for col in ("from_id", "to_id", "dead", "weight"):
        np.testing.assert_array_equal(after[col][:live], want[col], err_msg=col)
    assert (after["dead"][live:] == 1).all()
    assert new_static.level_capacities[0] >= static.level_capacities[0]
    want_lv = px.topo.initial_levels(static.num_units, want["from_id"], want["to_id"], allow_cycles=True,
                                     input_ids=(0, 1))
    np.testing.assert_array_equal(new_state.units["level"].cpu().numpy(), want_lv.cpu().numpy())
    assert not bool(new_state.needs_resort.item())
    # the resorted state steps
    res = px.make_step(Net, new_static, device=cuda)(new_state, px.StepInputs(np.ones(2, np.float32)))
    assert int(res.grown.item()) > 0
    torch.cuda.synchronize()
