"""The exact lowest-|w| prune fused into the mirror sweep (csrc/lowk.cu) on
the GPU, against the oracle's lowest_prune (oracle/steps.py, itself checked
against the C restatement and the lexsort definition on the CPU).

Bit-exact on the dead column: the k live edges of lowest |w| go, ties by
ascending slot, a NaN weight never; k beyond the live count prunes every
non-NaN live edge. The histogram the plan reads stays equal to the arena's
over consecutive firings (status 0). Two Scheme-A ranks are emulated on one
GPU through their lists (no rank waits on another: the sweeps and
selections run one after the other on one stream), so the multi-rank
selection and its claim-count adjustment are checked where only one GPU is.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle.steps import lowest_prune

pytestmark = pytest.mark.gpu


def _net(k, list_capacity=None, every=1):
    import plastax_b200 as px

    class Net(px.Network):
        forward_pass = px.ForwardPass("tanh")
        propagation = px.Propagation.PIPELINE
        prune_conn = px.LowestMagnitudePrune(k, every=every, list_capacity=list_capacity)

    return Net


def _arena(rng, n, e, quantised, specials):
    src = rng.integers(0, n, e)
    dst = rng.integers(4, n, e)
    if quantised:  # many exact ties, both signs, zeros
        w = np.round(rng.standard_normal(e) * 16) / 64
    else:
        w = rng.standard_normal(e) * 0.05
    w = w.astype(np.float32)
    if specials:
        w[rng.integers(0, e, 25)] = np.nan
        w[rng.integers(0, e, 25)] = np.inf
        w[rng.integers(0, e, 25)] = -np.inf
        w[rng.integers(0, e, 25)] = -0.0
    return src, dst, w


@pytest.mark.parametrize("k,quantised,specials", [(1, False, False), (777, True, False), (5000, False, True),
                                                  (40_000, True, True), (10**7, False, True)])
def test_fused_lowest_prune_matches_the_oracle(cuda, k, quantised, specials):
    """Three consecutive firings through make_step (the mirror sweep with the
    plan, the lists and the selection) tombstone exactly the oracle's set."""
    import torch

    import plastax_b200 as px

    rng = np.random.default_rng(k)
    n, e = 3000, 60_000
    src, dst, w = _arena(rng, n, e, quantised, specials)
    Net = _net(k)
    static, state = px.NetworkBuilder.from_edges(Net, n, src, dst, weights=w, input_ids=(0, 1, 2, 3),
                                                 output_ids=(), capacity_headroom=0.2, device=cuda)
    b = state.conns[0]
    b["dead"][::13] = 1  # a few tombstones already
    host = {kk: v.cpu().numpy().copy() for kk, v in b.items()}
    step = px.make_step(Net, static, device=cuda)
    assert step.use_mirror and step.lowk_prune
    for i in range(3):
        live = int((host["dead"] == 0).sum())
        want = lowest_prune([host], k)
        step(state, px.StepInputs(np.zeros(4, np.float32)))
        torch.cuda.synchronize()
        np.testing.assert_array_equal(b["dead"].cpu().numpy(), host["dead"], err_msg=f"firing {i}")
        assert step.lowk.plan_host()["pruned"] == want <= min(k, live)
        assert step.check_status()  # histogram in step with the arena, no list overflow


def test_fused_lowest_prune_with_growth_matches_the_oracle(cuda):
    """The reservoir churn step with the exact prune (k pruned, k regrown,
    the histogram raised by the committed edges): several steps equal to
    the oracle's, the live-edge count constant."""
    import math

    import torch

    from oracle.steps import ReservoirOracle
    from plastax_b200 import StepInputs, make_step
    from plastax_b200.configs import ReservoirConfig, build_reservoir

    cfg = ReservoirConfig(num_units=1 << 13, fan_in=32, churn=0.004, capacity_align=256)
    net, static, state = build_reservoir(cfg, cuda)
    b = state.conns[0]
    host = {kk: v.cpu().numpy().copy() for kk, v in b.items()}
    ref = ReservoirOracle(host, state.units["activation"].cpu().numpy().copy(),
                          state.units["level"].cpu().numpy().copy(), int(state.tail_start.item()),
                          num_inputs=cfg.num_inputs, num_res=cfg.num_units, tau=cfg.tau, k=cfg.k,
                          init_a=cfg.sigma * math.sqrt(3.0), seed=cfg.seed, threads=4)
    step = make_step(net, static, device=cuda)
    live0 = int((host["dead"] == 0).sum())
    rng = np.random.default_rng(2)
    for i in range(40):
        x = rng.standard_normal(cfg.num_inputs).astype(np.float32)
        if i == 3:
            step.capture(state, StepInputs(x))
        res = step(state, StepInputs(x))
        ref.step(x)
        got = {kk: v.cpu().numpy() for kk, v in b.items()}
        for col in ("from_id", "to_id", "dead", "weight"):
            np.testing.assert_array_equal(got[col], ref.b[col], err_msg=f"step {i} column {col}")
        np.testing.assert_allclose(state.units["activation"].cpu().numpy(), ref.act, rtol=1e-5, atol=1e-6)
        assert ref.last_pruned == cfg.k
        assert int(res.grown.item()) == cfg.k and not bool(res.overflow.item())
        assert int((b["dead"] == 0).sum().item()) == live0
    assert step.check_status()
    tot = step.lowk.totals.cpu().tolist()
    assert tot == [40 * cfg.k, 40 * cfg.k, 0, 40]
    torch.cuda.synchronize()


def test_mirror_overflow_entries_take_part(cuda):
    """With no spare entries in the mirror's groups, inserts spill into the
    mirror's overflow list; its edges are pruned and listed like the rest."""
    import math

    from oracle.steps import ReservoirOracle
    from plastax_b200 import StepInputs, make_step
    from plastax_b200.configs import ReservoirConfig, build_reservoir

    cfg = ReservoirConfig(num_units=1 << 12, fan_in=16, churn=0.05, capacity_align=256)
    net, static, state = build_reservoir(cfg, cuda)
    b = state.conns[0]
    host = {kk: v.cpu().numpy().copy() for kk, v in b.items()}
    ref = ReservoirOracle(host, state.units["activation"].cpu().numpy().copy(),
                          state.units["level"].cpu().numpy().copy(), int(state.tail_start.item()),
                          num_inputs=cfg.num_inputs, num_res=cfg.num_units, tau=cfg.tau, k=cfg.k,
                          init_a=cfg.sigma * math.sqrt(3.0), seed=cfg.seed)
    step = make_step(net, static, device=cuda)
    # groups of 128 units x 32 in-edges fill whole 2048-entry tiles: with
    # no spare entries, a group gaining more edges than it lost spills
    step.mirror_slack, step.mirror_min_slack, step.mirror_chunk_bits = 0.0, 0, 7
    rng = np.random.default_rng(4)
    spilled = 0
    for i in range(12):
        x = rng.standard_normal(cfg.num_inputs).astype(np.float32)
        step(state, StepInputs(x))
        ref.step(x)
        spilled = max(spilled, int(step.mirrors[0].ovf_count.item()))
        np.testing.assert_array_equal(b["dead"].cpu().numpy(), ref.b["dead"], err_msg=f"step {i}")
        np.testing.assert_array_equal(b["weight"].cpu().numpy(), ref.b["weight"], err_msg=f"step {i}")
        np.testing.assert_allclose(state.units["activation"].cpu().numpy(), ref.act, rtol=1e-5, atol=1e-6)
    assert spilled > 0, "the case must reach the mirror's overflow list"
    assert step.check_status()


def test_list_overflow_raises(cuda):
    """A threshold bin holding more edges than the list: the status word
    reports it and check_status raises (no silent short prune)."""
    import plastax_b200 as px

    rng = np.random.default_rng(1)
    n, e = 1000, 20_000
    src, dst = rng.integers(0, n, e), rng.integers(4, n, e)
    w = np.full(e, 0.25, np.float32)  # one bin holds every edge
    Net = _net(100, list_capacity=64)
    static, state = px.NetworkBuilder.from_edges(Net, n, src, dst, weights=w, input_ids=(0, 1, 2, 3),
                                                 output_ids=(), device=cuda)
    step = px.make_step(Net, static, device=cuda)
    step(state, px.StepInputs(np.zeros(4, np.float32)))
    with pytest.raises(px.PxbError, match="list capacity"):
        step.check_status()


@pytest.mark.parametrize("check_every", [1, 3])
def test_driver_raises_on_a_status_word(cuda, check_every):
    """The Driver reads the step's status words on its checks (every step,
    or every check_every-th) and raises instead of stepping on."""
    import plastax_b200 as px

    rng = np.random.default_rng(2)
    n, e = 1000, 20_000
    src, dst = rng.integers(0, n, e), rng.integers(4, n, e)
    w = np.full(e, 0.25, np.float32)
    Net = _net(100, list_capacity=64)
    static, state = px.NetworkBuilder.from_edges(Net, n, src, dst, weights=w, input_ids=(0, 1, 2, 3),
                                                 output_ids=(), device=cuda)
    drv = px.Driver(Net, static, state, check_every=check_every, device=cuda)
    x = px.StepInputs(np.zeros(4, np.float32))
    with pytest.raises(px.PxbError, match="list capacity"):
        for _ in range(check_every):
            drv.step(x)
    drv.close()


def test_firing_every_third_step(cuda):
    import torch

    import plastax_b200 as px

    rng = np.random.default_rng(9)
    n, e = 2000, 30_000
    src, dst, w = _arena(rng, n, e, True, False)
    Net = _net(300, every=3)
    static, state = px.NetworkBuilder.from_edges(Net, n, src, dst, weights=w, input_ids=(0, 1, 2, 3),
                                                 output_ids=(), device=cuda)
    host = {kk: v.cpu().numpy().copy() for kk, v in state.conns[0].items()}
    step = px.make_step(Net, static, device=cuda)
    for i in range(7):
        if i % 3 == 0:
            lowest_prune([host], 300)
        step(state, px.StepInputs(np.zeros(4, np.float32)))
        torch.cuda.synchronize()
        np.testing.assert_array_equal(state.conns[0]["dead"].cpu().numpy(), host["dead"], err_msg=f"step {i}")
    assert step.check_status()


class _FakePeers:
    """Two ranks' list areas in one process (the layout PeerGroup gives)."""

    def __init__(self, cap, world, dev):
        import torch

        self.world, self.lowk_cap = world, cap
        self.keys = [torch.zeros(2 * cap, dtype=torch.int64, device=dev) for _ in range(world)]
        self.levels = [torch.zeros(2 * cap, dtype=torch.int32, device=dev) for _ in range(world)]
        self.counts = [torch.zeros(4, dtype=torch.int64, device=dev) for _ in range(world)]
        arr = lambda ts: torch.tensor([t.data_ptr() for t in ts], dtype=torch.int64, device=dev)  # noqa: E731
        self.p_lkey, self.p_llevel, self.p_lcount = arr(self.keys), arr(self.levels), arr(self.counts)

    def view(self, rank):
        v = _FakePeers.__new__(_FakePeers)
        v.__dict__.update(self.__dict__)
        v.rank = rank
        v.lowk_key, v.lowk_level, v.lowk_count = self.keys[rank], self.levels[rank], self.counts[rank]
        return v


@pytest.mark.parametrize("k,quantised", [(3000, False), (2500, True)])
def test_two_rank_selection_emulated_on_one_gpu(cuda, k, quantised):
    """Two Scheme-A bands, each with its mirror, plan and list; the lists of
    both ranks feed each rank's selection: the union of the bands' prunes is
    the one-arena prune, and each rank's per-domain counts gain every rank's
    selected edges (ranks before it into `before`)."""
    import torch

    from plastax_b200.lowk import LowestK
    from plastax_b200.mirror import Mirror

    rng = np.random.default_rng(k)
    n, cap, world = 2048, 1 << 16, 2
    src, dst, w = _arena(rng, n, cap, quantised, True)
    level = np.ones(n, np.int32)
    level[:4] = 0
    dead = (rng.random(cap) < 0.05).astype(np.uint8)
    whole = {"from_id": torch.tensor(src, dtype=torch.int32, device=cuda),
             "to_id": torch.tensor(dst, dtype=torch.int32, device=cuda),
             "dead": torch.tensor(dead, device=cuda), "weight": torch.tensor(w, device=cuda)}
    lv = torch.tensor(level, device=cuda)
    band = cap // world
    bands = [{c: t[r * band:(r + 1) * band] for c, t in whole.items()} for r in range(world)]
    mirrors = [Mirror(bd, n) for bd in bands]
    fp = _FakePeers(8192, world, cuda)
    lks = [LowestK(k, cuda, list_cap=8192, slot_base=r * band, peers=fp.view(r)) for r in range(world)]
    for lk in lks:
        lk.build_hist([whole])
    act = torch.zeros(n, dtype=torch.float32, device=cuda)
    acc = torch.zeros(n, dtype=torch.float32, device=cuda)
    accf = torch.zeros(n, dtype=torch.int64, device=cuda)
    host = {"dead": dead.copy(), "weight": w}
    for firing in range(3):
        before_dead = host["dead"].copy()
        lowest_prune([host], k)
        for lk in lks:
            lk.make_plan()
        for r in range(world):
            lks[r].sweep(mirrors[r], act, acc, accf, "sum", bands[r]["dead"], None, lv)
        plan = lks[0].plan_host()
        base_b = [torch.full((2,), 100 * r, dtype=torch.int32, device=cuda) for r in range(world)]
        base_t = [torch.full((2,), 1000, dtype=torch.int32, device=cuda) for _ in range(world)]
        for r in range(world):
            lks[r].select(mirrors[r], bands[r]["dead"], None, lv, num_levels=2, level_before=base_b[r],
                          level_totals=base_t[r])
        torch.cuda.synchronize()
        np.testing.assert_array_equal(whole["dead"].cpu().numpy(), host["dead"], err_msg=f"firing {firing}")
        assert sum(int(lk.status.item()) for lk in lks) == 0
        # the selected edges of the threshold bin, per rank and domain
        newly = np.flatnonzero((before_dead == 0) & (host["dead"] == 1))
        bits = np.abs(w[newly]).view(np.uint32)
        tie = newly[(bits >= plan["lo_bits"]) & (bits < plan["hi_bits"])]
        per = np.zeros((world, 2), np.int64)
        for s in tie:
            per[s // band, level[src[s]]] += 1
        for r in range(world):
            assert base_t[r].cpu().tolist() == [1000 + int(per[:, lvl].sum()) for lvl in range(2)]
            assert base_b[r].cpu().tolist() == [100 * r + int(per[:r, lvl].sum()) for lvl in range(2)]
