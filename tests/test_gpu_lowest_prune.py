"""The k-lowest-|w| prune (LowestMagnitudePrune) on the GPU against
oracle/steps.lowest_prune: exactly min(k, live) live edges tombstoned, the
lowest |w| first, ties (quantised weights) by ascending slot across the
buckets in order; a C3-shaped step (SGD, the prune every 3 steps, regrowth
by |grad[dst] * act[src]|-scored per-unit proposals) keeps the edge count."""

from __future__ import annotations

import numpy as np
import pytest

from oracle.steps import lowest_prune

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("k", [1, 777, 5000, 10**6])
def test_lowest_prune_matches_the_oracle(cuda, k):
    import torch

    import plastax_b200 as px

    class Net(px.Network):
        forward_pass = px.ForwardPass("tanh")
        prune_conn = px.LowestMagnitudePrune(k)

    rng = np.random.default_rng(k)
    n = 400
    src = np.concatenate([rng.integers(0, 100, 3000), rng.integers(100, 250, 3000)])
    dst = np.concatenate([rng.integers(100, 250, 3000), rng.integers(250, 400, 3000)])
    # quantised weights: many exact ties, both signs, some zeros
    w = (np.round(rng.standard_normal(src.size) * 16) / 64).astype(np.float32)
    static, state = px.NetworkBuilder.from_edges(Net, n, src, dst, weights=w, input_ids=(0, 1), output_ids=(),
                                                 capacity_headroom=0.2, device=cuda)
    assert len(state.conns) >= 2
    for b in state.conns:  # a few tombstones already
        b["dead"][::11] = 1
    host = [{kk: v.cpu().numpy().copy() for kk, v in b.items()} for b in state.conns]
    step = px.make_step(Net, static, device=cuda)
    step(state, px.StepInputs(np.zeros(2, np.float32)))
    torch.cuda.synchronize()
    pruned = lowest_prune(host, k)
    live_before = sum(int((h["dead"] == 0).sum()) for h in host) + pruned
    assert pruned == min(k, live_before)
    for b, h in zip(state.conns, host, strict=True):
        np.testing.assert_array_equal(b["dead"].cpu().numpy(), h["dead"])


def test_c3_shaped_churn_keeps_the_edge_count(cuda):
    import torch

    import plastax_b200 as px

    k = 200

    class Net(px.Network):
        forward_pass = px.ForwardPass("tanh")
        backward_pass = px.BackwardPass("tanh")
        loss = px.MSELoss()
        propagation = px.Propagation.PIPELINE
        update_conn = px.optim.sgd(1e-3)
        prune_conn = px.LowestMagnitudePrune(k, every=3)
        add_conn = px.ProposeAddConn(proposals_per_proposer=64, max_new_per_level=k, score="grad_act",
                                     level_cap_scope="step", trigger=("every", 3), dst_lo=16)

    rng = np.random.default_rng(3)
    n, e = 600, 20_000
    src, dst = rng.integers(0, n, e), rng.integers(16, n, e)
    keep = src != dst
    src, dst = src[keep], dst[keep]
    w = (rng.standard_normal(src.size) / 8).astype(np.float32)
    static, state = px.NetworkBuilder.from_edges(Net, n, src, dst, weights=w, input_ids=tuple(range(16)),
                                                 output_ids=(598, 599), capacity_headroom=0.05, device=cuda)
    step = px.make_step(Net, static, device=cuda)
    live0 = int((state.conns[0]["dead"] == 0).sum())
    for i in range(7):
        x = rng.standard_normal(16).astype(np.float32)
        res = step(state, px.StepInputs(x, np.zeros(2, np.float32)))
        live = int((state.conns[0]["dead"] == 0).sum())
        if i % 3 == 0:
            assert int(res.grown.item()) == k and not bool(res.overflow.item())
        assert live == live0
    torch.cuda.synchronize()
