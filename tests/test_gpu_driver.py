"""The Driver (src/plastax/driver.py) on the GPU.

- `scan` runs a chunk as one device-side loop (the step's graph inside a
  conditional WHILE node) and stops itself after a step that overflowed or
  needs a resort; the host completes that step and re-enters. Step for step
  it equals K calls of `Driver.step`: the same arena, capacities, step count
  and per-step losses, through tail exhaustion and regrow (PIPELINE) and
  through resorts (TOPOLOGICAL).
- `Driver.step` completes an overflowing step exactly: the regrown arena
  equals the one a step on the bigger bucket commits.
"""

from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _pipeline(cuda):
    import plastax_b200 as px

    class Net(px.Network):
        forward_pass = px.ForwardPass("tanh")
        loss = px.MSELoss()
        propagation = px.Propagation.PIPELINE
        prune_conn = px.MagnitudePrune(0.01)
        add_conn = px.ProposeAddConn(proposals_per_proposer=1, max_new_per_level=300, dst_lo=2,
                                     level_cap_scope="step", init=("hash_uniform", 0.2))

    rng = np.random.default_rng(17)
    n, e = 900, 8000
    src, dst = rng.integers(0, n, e), rng.integers(2, n, e)
    w = (rng.standard_normal(e) * 0.2).astype(np.float32)
    static, state = px.NetworkBuilder.from_edges(Net, n, src, dst, weights=w, input_ids=(0, 1), output_ids=(5, 6),
                                                 capacity_headroom=0.0, capacity_align=256, device=cuda)
    return Net, static, state


def _topological(cuda):
    """Three layers; growth from the second half of layer 1 into its first
    half: the first step's same-level edges raise needs_resort, the resort
    lifts the first half a level (no cycle can form)."""
    import plastax_b200 as px

    class Net(px.Network):
        forward_pass = px.ForwardPass("tanh")
        add_conn = px.ProposeAddConn(proposals_per_proposer=200, max_new_per_level=5, proposer="global", src_lo=40,
                                     src_n=20, dst_lo=20, dst_n=20, score="uniform", direction="same_or_deeper",
                                     init=("dyadic",))

    rng = np.random.default_rng(5)
    src = np.concatenate([rng.integers(0, 20, 200), rng.integers(20, 60, 300)])
    dst = np.concatenate([rng.integers(20, 60, 200), rng.integers(60, 100, 300)])
    static, state = px.NetworkBuilder.from_edges(Net, 100, src, dst, input_ids=tuple(range(4)), output_ids=(99,),
                                                 capacity_headroom=0.5, capacity_align=64, device=cuda)
    return Net, static, state


def _chunk(static, k, seed=3):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((k, len(static.input_ids))).astype(np.float32)
    t = rng.standard_normal((k, len(static.output_ids))).astype(np.float32) if static.output_ids else None
    return x, t


def _arena(state):
    return [{k: v.cpu().numpy() for k, v in b.items()} for b in state.conns]


@pytest.mark.parametrize("build", ["pipeline", "topological"])
def test_scan_equals_the_step_loop(cuda, build):
    import torch

    import plastax_b200 as px

    make = _pipeline if build == "pipeline" else _topological
    k = 12
    Net, static, state = make(cuda)
    x, t = _chunk(static, k)
    ref = px.Driver(Net, static, state, device=cuda)
    losses = []
    for i in range(k):
        ref.step(px.StepInputs(x[i], None if t is None else t[i]))
        losses.append(float(ref.last_loss.item()))
    Net2, static2, state2 = make(cuda)
    drv = px.Driver(Net2, static2, state2, device=cuda)
    rec = drv.scan(px.StepInputs(x, t))
    torch.cuda.synchronize()
    assert drv.state.step == ref.state.step == k
    assert drv.static.level_capacities == ref.static.level_capacities
    assert ref.retraces > 0, "the case must regrow or resort inside the chunk"
    assert drv.retraces == ref.retraces
    for a, b in zip(_arena(drv.state), _arena(ref.state), strict=True):
        for col in a:
            np.testing.assert_array_equal(a[col], b[col], err_msg=col)
    np.testing.assert_array_equal(drv.state.units["activation"].cpu().numpy(),
                                  ref.state.units["activation"].cpu().numpy())
    np.testing.assert_array_equal(rec.cpu().numpy(), np.array(losses, np.float32))
    # a second chunk reuses the loop and stays in step
    x2, t2 = _chunk(static, k, seed=4)
    for i in range(k):
        ref.step(px.StepInputs(x2[i], None if t2 is None else t2[i]))
    drv.scan(px.StepInputs(x2, t2), record="outputs")
    for a, b in zip(_arena(drv.state), _arena(ref.state), strict=True):
        for col in a:
            np.testing.assert_array_equal(a[col], b[col], err_msg=col)
    drv.close()
    ref.close()


def test_scan_steps_and_validation(cuda):
    import plastax_b200 as px

    Net, static, state = _pipeline(cuda)
    drv = px.Driver(Net, static, state, device=cuda)
    x, t = _chunk(static, 6)
    rec = drv.scan(px.StepInputs(x, t), steps=4)
    assert drv.state.step == 4
    assert float(rec[4].item()) == 0.0 and float(rec[5].item()) == 0.0
    with pytest.raises(ValueError, match="chunk axis"):
        drv.scan(px.StepInputs(x[0], t[0]))
    with pytest.raises(ValueError, match="steps must be"):
        drv.scan(px.StepInputs(x, t), steps=7)
    with pytest.raises(ValueError, match="record"):
        drv.scan(px.StepInputs(x, t), record="grown")
    drv.close()


def test_driver_graphs_follow_the_eager_steps(cuda):
    """Driver(graphs=True) on a unit-lifecycle net (a unit spawned every 10
    steps, the units below the utility quantile pruned, UPGD, growth on the
    interval): the steps between spawns replay one captured graph per
    signature, the spawn steps run eagerly, and the run follows the all-eager
    Driver: the same pruned units and spawns, weights within 1e-4."""
    import torch

    import plastax_b200 as px

    TRACE = px.FieldSpec.float32("utility")
    n_in, hidden, cap = 32, 2048, 4096

    class Net(px.Network):
        forward_pass = px.ForwardPass("relu")
        backward_pass = px.BackwardPass("relu")
        loss = px.MSELoss()
        update_conn = px.optim.upgd(lr=0.01, beta=0.99, sigma=0.001)
        update_unit = px.TraceUnitUpdate(TRACE, "activation", 0.05)
        prune_unit = px.FieldBelowPrune(TRACE, quantile=0.01)
        add_unit = px.ArgmaxSpawn(TRACE, offset=1)
        add_conn = px.ProposeAddConn(proposals_per_proposer=8, max_new_per_level=64, dst_lo=n_in,
                                     score="uniform", max_level_gap=2, direction="deeper")
        extra_unit_fields = (TRACE,)
        unit_capacity = cap
        structural_interval = 10

    rng = np.random.default_rng(4)
    n = n_in + hidden + 1
    src = np.concatenate([rng.integers(0, n_in, 8000), rng.integers(n_in, n_in + hidden, 4000)])
    dst = np.concatenate([rng.integers(n_in, n_in + hidden, 8000), np.full(4000, n - 1)])
    w = (rng.standard_normal(src.size) * 0.1).astype(np.float32)
    xs = rng.standard_normal((25, n_in)).astype(np.float32)
    runs = []
    for graphs in (False, True):
        static, state = px.NetworkBuilder.from_edges(Net, n, src, dst, weights=w, input_ids=tuple(range(n_in)),
                                                     output_ids=(n - 1,), capacity_headroom=0.5, device=cuda)
        drv = px.Driver(Net, static, state, device=cuda, graphs=graphs)
        spawned = 0
        for i in range(25):
            drv.step(px.StepInputs(xs[i], np.array([xs[i, :4].sum()], np.float32)))
            spawned += int(drv.state.units_added.item())
        torch.cuda.synchronize()
        if graphs:
            assert len(drv._step._graphs) >= 1, "no step signature was captured"
        runs.append((drv, spawned))
    (a, sa), (b, sb) = runs
    assert sa == sb == 3
    np.testing.assert_array_equal(a.state.units["pruned"].cpu().numpy(), b.state.units["pruned"].cpu().numpy())
    for ba, bb in zip(a.state.conns, b.state.conns, strict=True):
        np.testing.assert_array_equal(ba["dead"].cpu().numpy(), bb["dead"].cpu().numpy())
        np.testing.assert_allclose(ba["weight"].cpu().numpy(), bb["weight"].cpu().numpy(), rtol=1e-4, atol=1e-5)
    a.close()
    b.close()
