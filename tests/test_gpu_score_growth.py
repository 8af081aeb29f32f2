"""ScoreAddConn on the GPU: the exhaustive grid, the importance shortlist and
the per-level shortlists (src/plastax/phases.py:3640-3746, :4690-4860).

- The step's candidate columns (endpoints, windowed scores, in the engine's
  grid order) equal the oracle's (oracle/growth.score_grid_engine, pinned
  to the registry's captured lists by the CPU golden tests) bit for bit, for
  every candidate kind and lowered score / importance form.
- One step of a layered TOPOLOGICAL net per rule: the arena after the step
  equals the oracle's selection (oracle/growth.select) claimed bucket by
  bucket by the oracle's C topological claim on host copies.
"""

from __future__ import annotations

import math

import numpy as np
import pytest

from oracle import growth as og
from oracle import oracle as orc
from oracle.steps import init_weight

pytestmark = pytest.mark.gpu

N_BUILT, N_SLOTS, N_IN = 200, 216, 8
LAYERS = (0, 8, 80, 150, 200)  # unit ranges of the four levels


def _layered(seed=3):
    """Edges from each layer to the next; every unit past layer 0 has one."""
    rng = np.random.default_rng(seed)
    src, dst = [], []
    for lo, mid, hi in zip(LAYERS[:-2], LAYERS[1:-1], LAYERS[2:], strict=True):
        for d in range(mid, hi):
            for s_ in rng.choice(np.arange(lo, mid), size=min(3, mid - lo), replace=False):
                src.append(int(s_))
                dst.append(d)
    return np.array(src), np.array(dst)


def _build(cuda, rule):
    import plastax_b200 as px

    class Net(px.Network):
        forward_pass = px.ForwardPass("tanh")
        add_conn = rule
        unit_capacity = N_SLOTS

    src, dst = _layered()
    rng = np.random.default_rng(9)
    w = (rng.standard_normal(src.size) * 0.5).astype(np.float32)
    static, state = px.NetworkBuilder.from_edges(Net, N_BUILT, src, dst, weights=w, input_ids=tuple(range(N_IN)),
                                                 output_ids=(), capacity_headroom=0.3, capacity_align=64,
                                                 device=cuda)
    return Net, static, state


def _oracle_cands(rule, state, static):
    units = {k: v.cpu().numpy() for k, v in state.units.items()}
    return og.score_grid_engine(units["level"], units["pruned"], candidates=rule.candidates,
                                shortlist_size=rule.shortlist_size, score=rule.score,
                                importance_form=rule.importance, cols=units, num_buckets=len(static.level_capacities),
                                topological=True, max_level_gap=rule.max_level_gap, direction=rule.direction,
                                allow_self_loops=rule.allow_self_loops)


MOD = ("modular", 3, 5, 17, 8, 0.125)
MOD_IMP = ("modular", 7, 13, 0, 0.25)


def _rules():
    import plastax_b200 as px

    return {
        "exhaustive_modular_topk": px.ScoreAddConn(score=MOD, max_new_per_level=40, init=("dyadic",),
                                                   max_level_gap=2),
        "exhaustive_predicate_all": px.predicate_add_conn(("modular_predicate", 1, 1, 2, 0), init=("const", 0.25),
                                                          max_level_gap=1, direction="deeper"),
        "shortlist_abs_product_step": px.ScoreAddConn(
            score=("abs_product", "activation", "activation"), candidates="shortlist", shortlist_size=40,
            importance=("abs_field", "activation"), max_new_per_level=30, level_cap_scope="step",
            dedupe_live=True, init=("hash_uniform", 0.1), max_level_gap=3),
        "per_level_modular_threshold": px.ScoreAddConn(
            score=MOD, candidates="shortlist_per_level", shortlist_size=24, importance=MOD_IMP,
            selection="threshold", threshold=0.0, max_new_per_level=20, direction="deeper", init=("dyadic",)),
        "per_level_product_step_cap": px.ScoreAddConn(
            score=("product", "activation", "activation"), candidates="shortlist_per_level", shortlist_size=24,
            importance=("field", "activation"), max_new_per_level=40, level_cap_scope="step", max_new_per_step=25,
            dedupe_step=True, init=("const", -0.5), max_level_gap=2, direction="same_or_deeper"),
    }


RULES = ["exhaustive_modular_topk", "exhaustive_predicate_all", "shortlist_abs_product_step",
         "per_level_modular_threshold", "per_level_product_step_cap"]


@pytest.mark.parametrize("name", RULES)
def test_score_candidates_match_the_oracle(cuda, name):
    import torch

    import plastax_b200 as px

    rule = _rules()[name]
    Net, static, state = _build(cuda, rule)
    # distinct, signed activations so the importance ranking and the
    # product scores see real values (and a tie or two: every 17th repeats)
    rng = np.random.default_rng(4)
    act = rng.standard_normal(N_SLOTS).astype(np.float32)
    act[::17] = act[1]
    state.units["activation"].copy_(torch.from_numpy(act))
    step = px.make_step(Net, static, device=cuda)
    step._bind(state)
    units = state.units
    step._score_candidates(state, dict(level=units["level"], pruned=units["pruned"],
                                       src_level_bound=len(static.level_capacities)))
    s_ref, d_ref, sc_ref = _oracle_cands(rule, state, static)
    src, dst, sc = (t.cpu().numpy() for t in step.cand)
    np.testing.assert_array_equal(src, s_ref)
    np.testing.assert_array_equal(dst, d_ref)
    np.testing.assert_array_equal(sc, sc_ref)
    assert np.isfinite(sc).sum() > 0


@pytest.mark.parametrize("name", RULES)
def test_score_growth_step_matches_the_oracle(cuda, name):
    import plastax_b200 as px

    rule = _rules()[name]
    Net, static, state = _build(cuda, rule)
    nb = len(static.level_capacities)
    before = [{k: v.cpu().numpy().copy() for k, v in b.items()} for b in state.conns]
    step = px.make_step(Net, static, device=cuda)
    x = np.random.default_rng(2).standard_normal(N_IN).astype(np.float32)
    res = step(state, px.StepInputs(x))
    # the selection, from the step's own post-forward unit columns
    src, dst, sc = _oracle_cands(rule, state, static)
    units_np = {k: v.cpu().numpy() for k, v in state.units.items()}
    level, pruned = units_np["level"], units_np["pruned"]
    cands = [[int(a), int(b), ("-inf" if math.isinf(c) else float(c)), i]
             for i, (a, b, c) in enumerate(zip(src, dst, sc, strict=True))]
    units = [[i, int(level[i]), bool(pruned[i])] for i in range(N_SLOTS)]
    edges = [[int(a), int(b)] for bk in before for a, b, d in zip(bk["from_id"], bk["to_id"], bk["dead"],
                                                                  strict=True) if d == 0]
    winners = og.select(units, edges, cands, capacity=N_SLOTS, max_level_gap=rule.max_level_gap,
                        direction=rule.direction, allow_self_loops=rule.allow_self_loops,
                        dedupe_live=rule.dedupe_live, dedupe_step=rule.dedupe_step, selection=rule.selection,
                        max_new_per_level=rule.max_new_per_level, max_new_per_step=rule.max_new_per_step,
                        threshold=rule.threshold, level_cap_scope=rule.level_cap_scope)
    w_src = np.array([cands[i][0] for i in winners], np.int32)
    w_dst = np.array([cands[i][1] for i in winners], np.int32)
    init = rule.init
    w_w = init_weight(init[0], float(init[1]) if len(init) > 1 else 0.0, w_src, w_dst)
    grown = 0
    for bk in range(nb):
        sel = np.flatnonzero(level[w_src] == bk)
        counts, _ = orc.claim_topological(before[bk], level, w_src[sel], w_dst[sel], w_w[sel],
                                          np.ones(sel.size, np.uint8))
        grown += int(counts[0])
    for bk in range(nb):
        for col in ("from_id", "to_id", "dead", "weight"):
            np.testing.assert_array_equal(state.conns[bk][col].cpu().numpy(), before[bk][col],
                                          err_msg=f"{name}: bucket {bk} column {col}")
    assert int(res.grown.item()) == grown
    assert grown > 0
    assert bool(res.overflow.item()) == (grown < len(winners))
