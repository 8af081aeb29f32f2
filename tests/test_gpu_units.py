"""The unit lifecycle on the GPU (src/plastax/phases.py:1148-1193,
:1245-1425).

- The seven unit_lifecycle_v1 goldens of the reference, through the step's
  own phase methods on the device: update_unit on every live unit,
  prune_unit (I/O exempt, permanent, incident edges tombstoned, columns reset,
  LEVEL kept), add_unit (lowest free ids in ascending parent order, a slot
  pruned in the same step reused, overflow, level clamp).
- A random state of 4,096 slots: the same phases against oracle/units.py,
  bit for bit (quantile threshold, argmax spawner, trace update).
- A C4-shaped step loop (update_unit trace, UPGD, unit pruning below a
  quantile, one spawn every 10 steps, per-unit proposal growth): the
  invariants every step must keep.
"""

from __future__ import annotations

import numpy as np
import pytest

from tests.test_oracle_goldens import UNIT_GOLDENS, check_unit_outcome, unit_case_arrays, unit_rules

pytestmark = pytest.mark.gpu


def _net(rules, capacity, max_levels, extra=None):
    import plastax_b200 as px

    attrs = dict(forward_pass=px.ForwardPass("tanh"), unit_capacity=capacity, max_levels=max_levels, **rules)
    attrs.update(extra or {})
    return type("Net", (px.Network,), attrs)


def _live_edges(state):
    out = []
    for b in state.conns:
        h = {k: v.cpu().numpy() for k, v in b.items()}
        out += [(int(s), int(d), float(w)) for s, d, w, x in zip(h["from_id"], h["to_id"], h["weight"], h["dead"],
                                                                strict=True) if x == 0]
    return out


@pytest.mark.parametrize("case", UNIT_GOLDENS, ids=[c["name"] for c in UNIT_GOLDENS])
def test_unit_goldens_on_the_device(cuda, case):
    import torch

    import plastax_b200 as px

    rules = {k: v for k, v in unit_rules(case["rules"]).items() if v is not None}
    n = case["capacity"]
    Net = _net(rules, n, case["max_levels"])
    act, level, pruned, exempt, b = unit_case_arrays(case)
    io_in = tuple(u["id"] for u in case["initial_units"] if u["is_input"])
    io_out = tuple(u["id"] for u in case["initial_units"] if u["is_output"])
    static, state = px.NetworkBuilder.from_edges(Net, n, b["from_id"], b["to_id"], weights=b["weight"],
                                                 input_ids=io_in, output_ids=io_out, device=cuda)
    state.units["activation"].copy_(torch.from_numpy(act))
    state.units["level"].copy_(torch.from_numpy(level))
    state.units["pruned"].copy_(torch.from_numpy(pruned))
    step = px.make_step(Net, static, device=cuda)
    step._bind(state)
    step._update_unit(state)
    step._prune_unit(state)
    children = overflow = None
    if "add_unit" in rules:
        before = state.units["pruned"].cpu().numpy().copy()
        step._add_unit(state)
        after = state.units["pruned"].cpu().numpy()
        children = [int(i) for i in np.flatnonzero((before == 1) & (after == 0))]
        overflow = bool(state.unit_overflow.item())
        assert int(state.units_added.item()) == len(children)
    torch.cuda.synchronize()
    u = {k: v.cpu().numpy() for k, v in state.units.items()}
    check_unit_outcome(case, u["activation"], u["level"], u["pruned"], _live_edges(state), children, overflow)


def test_unit_phases_match_the_oracle(cuda):
    import torch

    import plastax_b200 as px
    from oracle import units as ou

    rng = np.random.default_rng(77)
    n_built, cap = 3500, 4096
    TRACE = px.FieldSpec.float32("trace")
    rules = dict(update_unit=px.TraceUnitUpdate(TRACE, "activation", 0.25),
                 prune_unit=px.FieldBelowPrune(TRACE, quantile=0.01),
                 add_unit=px.ArgmaxSpawn(TRACE, offset=2, init=("scale_parent", TRACE, TRACE, 0.5)))
    Net = _net(rules, cap, 64, dict(extra_unit_fields=(TRACE,)))
    # a DAG: every edge goes to a higher id
    src = rng.integers(0, 3000, 40_000)
    dst = src + rng.integers(1, 500, 40_000)
    keep = dst < n_built
    static, state = px.NetworkBuilder.from_edges(Net, n_built, src[keep], dst[keep], input_ids=tuple(range(8)),
                                                 output_ids=(3499,), capacity_headroom=0.1, device=cuda)
    act = np.tanh(rng.standard_normal(cap)).astype(np.float32)
    trace = np.abs(rng.standard_normal(cap)).astype(np.float32)
    trace[100] = trace.max() + 1.0  # a clear argmax parent
    pr = state.units["pruned"].cpu().numpy().copy()
    earlier = rng.choice(np.arange(200, n_built - 1), 30, replace=False)
    pr[earlier] = 1  # some slots pruned earlier (not the argmax parent, 100)
    state.units["activation"].copy_(torch.from_numpy(act))
    state.units["trace"].copy_(torch.from_numpy(trace))
    state.units["pruned"].copy_(torch.from_numpy(pr))
    host = [{k: v.cpu().numpy().copy() for k, v in b.items()} for b in state.conns]
    units = {k: v.cpu().numpy().copy() for k, v in state.units.items()}
    step = px.make_step(Net, static, device=cuda)
    step._bind(state)
    step._update_unit(state)
    step._prune_unit(state)
    step._add_unit(state)
    torch.cuda.synchronize()
    # the oracle on the host copies
    exempt = np.zeros(cap, bool)
    exempt[list(static.input_ids) + list(static.output_ids)] = True
    defaults = {name: np.zeros((), units[name].dtype) for name in units if name not in ("level", "pruned")}
    pruned = units["pruned"]
    ou.update_unit(units, pruned, rules["update_unit"])
    doomed = ou.prune_unit(units, pruned, exempt, defaults, host, rules["prune_unit"])
    children, overflow = ou.add_unit(units, pruned, units["level"], defaults, rules["add_unit"], 64)
    assert doomed.sum() > 10 and len(children) == 1 and not overflow
    got = {k: v.cpu().numpy() for k, v in state.units.items()}
    for name in units:
        np.testing.assert_array_equal(got[name], units[name], err_msg=name)
    for bk, ref in zip(state.conns, host, strict=True):
        np.testing.assert_array_equal(bk["dead"].cpu().numpy(), ref["dead"])
    assert int(state.units_added.item()) == 1 and not bool(state.unit_overflow.item())


def test_c4_shaped_loop_keeps_the_invariants(cuda):
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
    static, state = px.NetworkBuilder.from_edges(Net, n, src, dst, weights=w, input_ids=tuple(range(n_in)),
                                                 output_ids=(n - 1,), capacity_headroom=0.5, device=cuda)
    drv = px.Driver(Net, static, state, device=cuda)
    io = set(range(n_in)) | {n - 1}
    live_units = int((state.units["pruned"] == 0).sum())
    for i in range(25):
        x = rng.standard_normal(n_in).astype(np.float32)
        drv.step(px.StepInputs(x, np.array([x[:4].sum()], np.float32)))
        st = drv.state
        pruned = st.units["pruned"].cpu().numpy()
        assert not any(pruned[j] for j in io), "inputs and outputs are never pruned"
        for b in st.conns:
            h = {k: v.cpu().numpy() for k, v in b.items()}
            live = h["dead"] == 0
            assert not pruned[h["from_id"][live]].any() and not pruned[h["to_id"][live]].any(), \
                "no live edge touches a pruned unit"
        added = int(st.units_added.item())
        assert added == (1 if i % 10 == 0 else 0)
        lv = st.units["level"].cpu().numpy()
        assert lv.min() >= 0 and lv.max() <= Net.max_levels - 1
        now = int((st.units["pruned"] == 0).sum())
        assert now <= live_units + added
        live_units = now
    torch.cuda.synchronize()
    drv.close()
