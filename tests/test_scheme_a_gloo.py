"""Scheme-A connection sharding over two gloo ranks on the CPU (no GPU).

Each rank builds only its capacity band of the arena (NetworkBuilder with a
ShardSpec), computes its forward partial with the oracle, and the partials
are all-reduced (src/plastax/monoid.py:175-204): the result equals the
single-arena forward. The pipeline claim's cross-rank arithmetic is checked
the same way: every rank all-gathers the per-domain free counts, derives the
counts of the ranks before it and the global totals, and places exactly the
candidates whose global free-slot rank (or tail position) falls in its band
(src/plastax/phases.py:3023-3106); the bands together equal the oracle's
claim on the whole arena.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case():
    rng = np.random.default_rng(3)
    n, e = 300, 6000
    src = rng.integers(0, n, e)
    dst = rng.integers(0, n, e)
    w = (rng.standard_normal(e) * 0.1).astype(np.float32)
    act = rng.standard_normal(n).astype(np.float32)
    return n, src, dst, w, act


def _net():
    import plastax_b200 as px

    class Net(px.Network):
        forward_pass = px.ForwardPass("tanh")
        propagation = px.Propagation.PIPELINE

    return Net


def _band_claim(b, level, tail, base, cap_global, src, dst, before, totals):
    """One rank's pipeline claim from the gathered counts (restated on host)."""
    nl = totals.size
    local_lists = [[] for _ in range(nl)]
    for s in range(b["dead"].size):
        if b["dead"][s] and base + s < tail:
            local_lists[level[b["from_id"][s]]].append(s)
    own_rank = {}
    seen = [0] * nl
    spill = 0
    placed = []
    for i in range(src.size):
        lv = level[src[i]]
        r = seen[lv]
        seen[lv] += 1
        if r < totals[lv]:
            lr = r - before[lv]
            if 0 <= lr < len(local_lists[lv]):
                placed.append((local_lists[lv][lr], i))
        else:
            pos = tail + spill
            spill += 1
            if pos < cap_global and base <= pos < base + b["dead"].size:
                placed.append((pos - base, i))
    del own_rank
    for slot, i in placed:
        b["from_id"][slot], b["to_id"][slot], b["dead"][slot], b["weight"][slot] = src[i], dst[i], 0, 1.0


def _worker(rank: int, port: int, out: dict) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        import plastax_b200 as px
        from oracle import oracle as orc

        n, src, dst, w, act = _case()
        static, state = px.NetworkBuilder.from_edges(
            _net(), n, src, dst, weights=w, input_ids=(0,), output_ids=(), capacity_align=64, capacity_headroom=0.1,
            sharding=px.ShardSpec("conns", WORLD), shard_rank=rank, device="cpu")
        b = {k: v.numpy().copy() for k, v in state.conns[0].items()}
        # forward partial over this band, all-reduced
        part = np.zeros(n, np.float32)
        orc.forward_accumulate(b, act, n, "sum", part)
        t = torch.from_numpy(part)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        out_fwd = t.numpy().copy()
        # prune a slice, then claim candidates across the bands
        orc.prune(b, n, 1, 0.02)
        level = (np.arange(n) % 3).astype(np.int32)
        base = static.shard_base(0)
        tail = int(state.tail_start.item())
        local = np.zeros(3, np.int64)
        for s in range(b["dead"].size):
            if b["dead"][s] and base + s < tail:
                local[level[b["from_id"][s]]] += 1
        gathered = [torch.zeros(3, dtype=torch.int64) for _ in range(WORLD)]
        dist.all_gather(gathered, torch.from_numpy(local))
        allc = torch.stack(gathered).numpy()
        before, totals = allc[:rank].sum(0), allc.sum(0)
        rng = np.random.default_rng(9)
        k = 400
        cs = rng.integers(0, n, k).astype(np.int32)
        cs = cs[np.argsort(level[cs], kind="stable")]
        cd = rng.integers(0, n, k).astype(np.int32)
        _band_claim(b, level, tail, base, static.level_capacities[0], cs, cd, before, totals)
        bands = [None] * WORLD
        dist.all_gather_object(bands, {kk: v.tolist() for kk, v in b.items()})
        if rank == 0:
            out["fwd"] = out_fwd
            out["bands"] = bands
            out["claim_in"] = (level, tail, cs, cd)
    finally:
        dist.destroy_process_group()


def _run(rank, port, q):
    out = {}
    _worker(rank, port, out)
    if rank == 0:
        q.put(out)


@pytest.mark.timeout(300)
def test_scheme_a_two_gloo_ranks_equal_one_arena():
    import plastax_b200 as px
    from oracle import oracle as orc

    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_run, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    out = q.get(timeout=240)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    n, src, dst, w, act = _case()
    _, full = px.NetworkBuilder.from_edges(_net(), n, src, dst, weights=w, input_ids=(0,), output_ids=(),
                                           capacity_align=64, capacity_headroom=0.1, device="cpu")
    b = {k: v.numpy().copy() for k, v in full.conns[0].items()}
    ref = np.zeros(n, np.float32)
    orc.forward_accumulate(b, act, n, "sum", ref)
    np.testing.assert_allclose(out["fwd"], ref, rtol=1e-5, atol=1e-6)
    orc.prune(b, n, 1, 0.02)
    level, tail, cs, cd = out["claim_in"]
    orc.claim_pipeline(b, level, tail, cs, cd, np.ones(cs.size, np.float32), np.ones(cs.size, np.uint8))
    for col in ("from_id", "to_id", "dead", "weight"):
        got = np.concatenate([np.asarray(band[col]) for band in out["bands"]]).astype(b[col].dtype)
        np.testing.assert_array_equal(got, b[col], err_msg=col)


def _gather_worker(rank: int, port: int, q) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        import plastax_b200 as px
        from plastax_b200.step import gather_arena

        Net, n, src, dst = _layered_net()
        static, state = px.NetworkBuilder.from_edges(
            Net, n, src, dst, input_ids=(0, 1), output_ids=(), capacity_align=64, capacity_headroom=0.2,
            sharding=px.ShardSpec("conns", WORLD), shard_rank=rank, device="cpu")
        for b in state.conns:  # a few tombstones, so dead slots sit among the live ones
            b["dead"][::7] = 1
        got = gather_arena(state.conns, static)
        if rank == 0:
            q.put({k: v.numpy().copy() for k, v in got.items()})
    finally:
        dist.destroy_process_group()


def _layered_net():
    import plastax_b200 as px

    class Net(px.Network):
        forward_pass = px.ForwardPass("tanh")
        add_conn = px.ProposeAddConn(proposals_per_proposer=2, max_new_per_level=8, proposer="per_connection")

    rng = np.random.default_rng(12)
    n = 120
    src = np.concatenate([rng.integers(0, 40, 300), rng.integers(40, 80, 300)])
    dst = np.concatenate([rng.integers(40, 80, 300), rng.integers(80, 120, 300)])
    return Net, n, src, dst


@pytest.mark.timeout(300)
def test_per_connection_arena_gather_equals_the_whole_arena():
    """Under Scheme-A the per-connection proposer ranks every rank's
    connections: the gathered bands, bucket-major, are the unsharded arena's
    (from_id, to_id, dead) slot for slot (src/plastax/phases.py:3863-3917)."""
    import plastax_b200 as px

    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_gather_worker, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    got = q.get(timeout=240)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    Net, n, src, dst = _layered_net()
    static, full = px.NetworkBuilder.from_edges(Net, n, src, dst, input_ids=(0, 1), output_ids=(), capacity_align=64,
                                                capacity_headroom=0.2, device="cpu")
    assert len(full.conns) >= 2
    G = WORLD
    for col in ("from_id", "to_id", "dead"):
        parts = []
        for b in full.conns:
            c = b[col].numpy().copy()
            if col == "dead":
                band = c.size // G
                for r in range(G):  # each rank tombstoned every 7th slot of its own band
                    c[r * band:(r + 1) * band][::7] = 1
            parts.append(c)
        np.testing.assert_array_equal(got[col], np.concatenate(parts), err_msg=col)
