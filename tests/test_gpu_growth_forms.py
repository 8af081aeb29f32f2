"""The growth forms beyond one RNG proposal per unit, on the GPU.

- The global and per-connection proposers reproduce the candidate lists the
  reference generated for the golden registry (tests/golden/
  growth_registry.json: global_propose_v1, conn_propose_v1).
- One churn step of a small PIPELINE net for each proposer x selection (top_k,
  threshold, all) x cap scope (source level, step) x dedupe: the step's
  committed arena equals the oracle's selection (oracle/growth.select, pinned
  by the registry) claimed by the oracle's C claim on a host copy.
"""

from __future__ import annotations

import json
import math
import pathlib

import numpy as np
import pytest

from oracle import oracle as orc
from oracle.growth import select as og_select
from oracle.steps import init_weight

pytestmark = pytest.mark.gpu

REGISTRY = json.loads((pathlib.Path(__file__).resolve().parent / "golden" / "growth_registry.json").read_text())


def _k():
    from plastax_b200 import kernels

    return kernels


@pytest.mark.parametrize("proposer", ["global", "per_connection"])
def test_proposers_reproduce_the_registry_candidates(cuda, proposer):
    import torch

    kern = _k()
    seen = 0
    for case in REGISTRY:
        p = case["params"]
        if p.get("proposer") != proposer or not case["calls"]:
            continue
        sel = case["calls"][0][1]
        units, edges = sel["units"], sel["edges"]
        if any(u[2] for u in units):
            continue  # the registry's lists skip pruned proposers; the engine vetoes them
        n = len(units)
        level = torch.tensor([u[1] for u in units], dtype=torch.int32, device=cuda)
        P = p["proposals_per_proposer"]
        win = dict(level=level, max_level_gap=1 << 20, allow_self_loops=True)
        if proposer == "global":
            src, dst, score = kern.propose_global(P, p["network_seed"], p["step"], n, src_lo=0, src_n=n, dst_lo=0,
                                                  dst_n=n, score_kind=1, **win)
        else:
            b = {"from_id": torch.tensor([e[0] for e in edges], dtype=torch.int32, device=cuda),
                 "to_id": torch.tensor([e[1] for e in edges], dtype=torch.int32, device=cuda),
                 "dead": torch.zeros(len(edges), dtype=torch.uint8, device=cuda),
                 "weight": torch.zeros(len(edges), dtype=torch.float32, device=cuda)}
            src, dst, score = kern.propose_per_conn(b, P, p["network_seed"], p["step"], n, dst_lo=0, dst_n=n,
                                                    score_kind=1, **win)
        got = [[int(s), int(d), float(sc), i] for i, (s, d, sc) in
               enumerate(zip(src.cpu().tolist(), dst.cpu().tolist(), score.cpu().tolist(), strict=True))]
        assert got == [[c[0], c[1], float(c[2]), c[3]] for c in sel["cands"]], case["name"]
        seen += 1
    assert seen >= 3


FORMS = [
    ("per_unit", 3, "top_k", "source_level", False, False),
    ("per_unit", 3, "top_k", "step", True, True),
    ("per_unit", 1, "threshold", "source_level", False, False),
    ("global", 4000, "top_k", "source_level", True, False),
    ("global", 4000, "all", "step", False, True),
    ("global", 3000, "threshold", "step", False, False),
    ("per_connection", 1, "top_k", "source_level", False, True),
    ("per_connection", 2, "top_k", "step", True, False),
]


@pytest.mark.parametrize("proposer,P,selection,scope,ded_live,ded_step", FORMS)
def test_growth_step_matches_the_oracle(cuda, proposer, P, selection, scope, ded_live, ded_step):
    import torch

    import plastax_b200 as px

    kern = _k()
    rng = np.random.default_rng(61)
    n, e = 600, 5000
    src = rng.integers(0, n, e)
    dst = rng.integers(2, n, e)
    k = 300

    class Net(px.Network):
        forward_pass = px.ForwardPass("tanh")
        propagation = px.Propagation.PIPELINE
        add_conn = px.ProposeAddConn(proposals_per_proposer=P, max_new_per_level=k, dst_lo=2, proposer=proposer,
                                     selection=selection, threshold=0.6 if selection == "threshold" else None,
                                     level_cap_scope=scope, score="uniform_q256", init=("hash_uniform", 0.1),
                                     dedupe_live=ded_live, dedupe_step=ded_step, max_level_gap=2)

    static, state = px.NetworkBuilder.from_edges(Net, n, src, dst, weights=np.full(e, 0.5, np.float32),
                                                 input_ids=(0, 1), output_ids=(), capacity_headroom=0.05,
                                                 device=cuda)
    step = px.make_step(Net, static, device=cuda)
    b0 = {kk: v.cpu().numpy().copy() for kk, v in state.conns[0].items()}
    level = state.units["level"].cpu().numpy().copy()
    tail = int(state.tail_start.item())
    # the step's own candidates (their generation is pinned above)
    ac = Net.add_conn
    d_level = state.units["level"]
    win = dict(level=d_level, max_level_gap=ac.max_level_gap)
    if proposer == "per_unit":
        cs, cd, sc = kern.propose_per_unit(n, P, static.seed, 0, dst_lo=2, dst_n=n - 2, score_kind=1, **win)
    elif proposer == "global":
        cs, cd, sc = kern.propose_global(P, static.seed, 0, n, src_lo=0, src_n=n, dst_lo=2, dst_n=n - 2,
                                         score_kind=1, **win)
    else:
        cs, cd, sc = kern.propose_per_conn(state.conns[0], P, static.seed, 0, n, dst_lo=2, dst_n=n - 2,
                                           score_kind=1, **win)
    cands = [[int(a), int(b), float(c), i] for i, (a, b, c) in
             enumerate(zip(cs.cpu().tolist(), cd.cpu().tolist(), sc.cpu().tolist(), strict=True))]
    cands = [[a, b, ("-inf" if math.isinf(c) else c), i] for a, b, c, i in cands]
    units = [[i, int(level[i]), False] for i in range(n)]
    live = b0["dead"] == 0
    edges = [[int(a), int(b)] for a, b in zip(b0["from_id"][live], b0["to_id"][live], strict=True)]
    winners = og_select(units, edges, cands, capacity=n, max_level_gap=ac.max_level_gap, dedupe_live=ded_live,
                        dedupe_step=ded_step, selection=selection, max_new_per_level=k,
                        threshold=ac.threshold, level_cap_scope=scope)
    w_src = np.array([cands[i][0] for i in winners], np.int32)
    w_dst = np.array([cands[i][1] for i in winners], np.int32)
    w_w = init_weight("hash_uniform", 0.1, w_src, w_dst)
    counts, _, new_tail = orc.claim_pipeline(b0, level, tail, w_src, w_dst, w_w, np.ones(w_src.size, np.uint8))
    res = step(state, px.StepInputs(np.zeros(2, np.float32)))
    for col in ("from_id", "to_id", "dead", "weight"):
        np.testing.assert_array_equal(state.conns[0][col].cpu().numpy(), b0[col], err_msg=col)
    assert int(res.grown.item()) == int(counts[0]) and int(state.tail_start.item()) == new_tail
    assert int(counts[0]) > 0
