"""End-to-end parity of the reservoir churn step (make_step on the GPU) with
the oracle's reference-order step, several steps in a row.

Structure must be bit-exact every step: tombstones, the claimed slots and
every written column, tail_start, grown. Activations within 1e-5 rel / 1e-6
abs. At the benchmark's full size the same step is checked through
size-independent properties (live-edge conservation, claim accounting,
ids in range) since the oracle needs minutes per step there.
"""

from __future__ import annotations

import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _run(cuda, cfg, steps, sharded_bands=1, graph=False, ahead=True):
    import torch

    from oracle.steps import ReservoirOracle
    from plastax_b200 import StepInputs, make_step
    from plastax_b200.configs import build_reservoir

    net, static, state = build_reservoir(cfg, cuda)
    b = {k: v.cpu().numpy().copy() for k, v in state.conns[0].items()}
    ref = ReservoirOracle(b, state.units["activation"].cpu().numpy().copy(), state.units["level"].cpu().numpy().copy(),
                          int(state.tail_start.item()), num_inputs=cfg.num_inputs, num_res=cfg.num_units,
                          tau=cfg.tau, k=cfg.k, init_a=cfg.sigma * math.sqrt(3.0), seed=cfg.seed, prune=cfg.prune)
    step = make_step(net, static, device=cuda)
    # the site-RNG selection runs one step ahead on the side stream by default
    assert step.ahead
    step.ahead = ahead
    rng = np.random.default_rng(5)
    for i in range(steps):
        x = rng.standard_normal(cfg.num_inputs).astype(np.float32)
        if graph and i == 1:  # capture after one eager step, replay from then on
            step.capture(state, StepInputs(x))
        res = step(state, StepInputs(x))
        ref.step(x)
        got = {k: v.cpu().numpy() for k, v in res.state.conns[0].items()}
        for col in ("from_id", "to_id", "dead", "weight"):
            np.testing.assert_array_equal(got[col], ref.b[col], err_msg=f"step {i} column {col}")
        np.testing.assert_allclose(res.state.units["activation"].cpu().numpy(), ref.act, rtol=1e-5, atol=1e-6)
        assert int(res.state.tail_start.item()) == ref.tail
        assert int(res.grown.item()) == int(ref.last_counts[0])
        assert bool(res.overflow.item()) == bool(ref.last_counts[1] > 0)
    torch.cuda.synchronize()


@pytest.mark.parametrize("log2,fan_in,churn,prune", [(12, 16, 0.01, "lowest_k"), (14, 32, 0.001, "lowest_k"),
                                                     (10, 8, 0.2, "lowest_k"), (12, 16, 0.01, "threshold"),
                                                     (10, 8, 0.2, "threshold")])
def test_reservoir_churn_matches_oracle(cuda, log2, fan_in, churn, prune):
    from plastax_b200.configs import ReservoirConfig

    _run(cuda, ReservoirConfig(num_units=1 << log2, fan_in=fan_in, churn=churn, capacity_align=256, prune=prune),
         steps=6)


def test_reservoir_churn_replayed_from_a_cuda_graph_matches_oracle(cuda):
    """The captured step (device-side step counter keying the proposals)
    replays the same structure as the eager one, step after step."""
    from plastax_b200.configs import ReservoirConfig

    _run(cuda, ReservoirConfig(num_units=1 << 12, fan_in=16, churn=0.01, capacity_align=256), steps=6, graph=True)


@pytest.mark.parametrize("graph", [False, True])
def test_reservoir_churn_with_selection_in_step_matches_oracle(cuda, graph):
    """The selection run inside its own step (beside the sweep, not one
    step ahead) gives the same structure."""
    from plastax_b200.configs import ReservoirConfig

    _run(cuda, ReservoirConfig(num_units=1 << 12, fan_in=16, churn=0.01, capacity_align=256), steps=5, graph=graph,
         ahead=False)


def test_reservoir_overflow_into_tail_exhaustion(cuda):
    """A churn larger than the dead slots + tail: the claim overflows and
    the flag and counts still match the oracle."""
    from plastax_b200.configs import ReservoirConfig

    cfg = ReservoirConfig(num_units=1 << 10, fan_in=8, churn=0.3, capacity_align=64, capacity_headroom=0.0)
    _run(cuda, cfg, steps=4)


def _order_keys(w, slots):
    """The prune's total order as int64 keys: bits(|w|) << 32 | slot."""
    import torch

    bits = (w.view(torch.int32) & 0x7FFFFFFF).to(torch.int64)
    return (bits << 32) | slots.to(torch.int64)


@pytest.mark.slow
def test_full_size_churn_properties(cuda):
    """The benchmark's full-size churn step, 30 steps in a row (the first
    eager, the rest replayed from the step's CUDA graph, as the benchmark
    runs it): each prunes exactly k edges and grows exactly k (no overflow),
    so the live-edge count stays constant; the pruned edges are the k
    lowest of the (|w|, slot) order (checked on three steps: every survivor
    orders after every pruned edge); every live id stays in range."""
    import torch

    from plastax_b200 import StepInputs, make_step
    from plastax_b200.configs import C5, build_reservoir

    net, static, state = build_reservoir(C5, cuda)
    step = make_step(net, static, device=cuda)
    n = static.num_units
    b = state.conns[0]
    live0 = int((b["dead"] == 0).sum())
    tail0 = int(state.tail_start.item())
    slots = torch.arange(b["dead"].numel(), dtype=torch.int32, device=cuda)
    x0 = torch.randn(C5.num_inputs, device=cuda)
    for i in range(30):
        check = i in (0, 11, 29)
        if check:
            live_b = b["dead"] == 0
            before = {c: b[c].clone() for c in ("from_id", "to_id", "weight")}
        if i == 1:
            step.capture(state, StepInputs(x0))
        res = step(state, StepInputs(torch.randn(C5.num_inputs, device=cuda)))
        assert int(res.grown.item()) == C5.k and not bool(res.overflow.item()), i
        assert int((b["dead"] == 0).sum()) == live0, i
        if check:
            # a live-before slot that is dead now, or holds another edge, was pruned
            same = (b["from_id"] == before["from_id"]) & (b["to_id"] == before["to_id"]) & (
                b["weight"].view(torch.int32) == before["weight"].view(torch.int32)) & (b["dead"] == 0)
            gone = live_b & ~same
            assert int(gone.sum()) == C5.k, i
            keep = live_b & same & ~torch.isnan(before["weight"])
            kg = _order_keys(before["weight"][gone], slots[gone])
            kk = _order_keys(before["weight"][keep], slots[keep])
            assert int(kg.max()) < int(kk.min()), i
            del live_b, before, same, gone, keep, kg, kk
        liv = b["dead"] == 0
        assert int(b["from_id"][liv].min()) >= 0 and int(b["from_id"][liv].max()) < n
        assert int(b["to_id"][liv].min()) >= C5.num_inputs and int(b["to_id"][liv].max()) < n
        assert int(state.tail_start.item()) >= tail0
    assert step.check_status()
    tot = step.lowk.totals.cpu().tolist()
    assert tot == [30 * C5.k, 30 * C5.k, 0, 30]
