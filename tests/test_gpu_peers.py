"""Scheme-A combine + apply over NVLink peer memory (csrc/peer.cu).

The two-rank test needs two GPUs (run on a multi-GPU box; skipped on one):
the sharded step with the peer-memory combine must equal the one-GPU step bit
for bit -- the forward's sums are exact fixed point, so sharding cannot
change them, and the claim's bands concatenate to the one-arena claim. The
bounded wait is checked on one GPU: a peer that never signals makes the wait
give up, report status bit 0, and return.
"""

from __future__ import annotations

import ctypes
import os
import socket
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_peer_wait_gives_up_and_reports(cuda):
    import torch

    from plastax_b200 import _lib
    from plastax_b200.peers import scheme_a_apply

    n, world = 4096, 2
    # two "ranks" in this process; rank 1 never runs, so its flags stay 0
    fixed = [torch.zeros(n, dtype=torch.int64, device=cuda) for _ in range(world)]
    side = [torch.zeros(n, dtype=torch.float32, device=cuda) for _ in range(world)]
    act = [torch.full((n,), 7.0, dtype=torch.float32, device=cuda) for _ in range(world)]
    flags = [torch.zeros(2 * world, dtype=torch.int32, device=cuda) for _ in range(world)]
    fixed[0][5] = 3 << 31
    arr = lambda ts: torch.tensor([t.data_ptr() for t in ts], dtype=torch.int64, device=cuda)  # noqa: E731
    p_fixed, p_side, p_act, p_flags = arr(fixed), arr(side), arr(act), arr(flags)
    words = torch.zeros(4, dtype=torch.int32, device=cuda)
    w = words.data_ptr()

    class G:
        struct = _lib.PeerGroup(0, world, p_fixed.data_ptr(), p_side.data_ptr(), p_act.data_ptr(),
                                p_flags.data_ptr(), None, w, w + 4, w + 8)

    G.n = n
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    scheme_a_apply(G, "identity", wait_polls=2000)
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 5.0
    assert int(words[2].item()) & 1, "the timed-out wait must be reported"
    assert int(words[0].item()) == 1, "the epoch still advances"
    # nothing was reduced: the activations are untouched
    assert float(act[0][5].item()) == 7.0
    # rank 0 did signal both rows of its own flags and of the silent peer
    assert flags[1].cpu().tolist()[0] == 1 and flags[1].cpu().tolist()[2] == 1


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cfg():
    from plastax_b200.configs import ReservoirConfig

    return ReservoirConfig(num_units=1 << 12, fan_in=16, churn=0.01, capacity_align=256)


def _collect(q, procs, n, timeout=500.0):
    """n results from the rank processes; fails as soon as a rank exits
    with an error instead of waiting out the whole timeout."""
    import queue

    got, t0 = {}, time.monotonic()
    while len(got) < n:
        try:
            r, out = q.get(timeout=2.0)
            got[r] = out
        except queue.Empty:
            dead = [p.exitcode for p in procs if p.exitcode not in (None, 0)]
            if dead:
                raise AssertionError(f"a rank exited with {dead[0]}")
            if time.monotonic() - t0 > timeout:
                raise AssertionError("the ranks did not report in time")
    return got


def _inputs(steps, m):
    return np.random.default_rng(8).standard_normal((steps, m)).astype(np.float32)


def _run(rank, world, port, steps, q):
    import datetime

    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        from plastax_b200 import StepInputs, make_step
        from plastax_b200.configs import build_reservoir
        from plastax_b200.types import ShardSpec

        cfg = _cfg()
        net, static, state = build_reservoir(cfg, dev, sharding=ShardSpec("conns", world), shard_rank=rank)
        step = make_step(net, static, device=dev)
        assert step.peer_reduce
        xs = _inputs(steps, cfg.num_inputs)
        for i in range(steps):
            if i == 2:
                step.capture(state, StepInputs(torch.from_numpy(xs[i]).to(dev)))
            step(state, StepInputs(torch.from_numpy(xs[i]).to(dev)))
        torch.cuda.synchronize()
        out = {k: v.cpu().numpy() for k, v in state.conns[0].items()}
        out["activation"] = state.units["activation"].cpu().numpy()
        out["status"] = int(step.peers.status.item())
        out["tail"] = int(state.tail_start.item())
        step.close()
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(600)
def test_two_rank_peer_step_equals_one_gpu_step(cuda):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from plastax_b200 import StepInputs, make_step
    from plastax_b200.configs import build_reservoir

    steps = 6
    cfg = _cfg()
    net, static, state = build_reservoir(cfg, cuda)
    step = make_step(net, static, device=cuda)
    xs = _inputs(steps, cfg.num_inputs)
    for i in range(steps):
        step(state, StepInputs(torch.from_numpy(xs[i]).to(cuda)))
    torch.cuda.synchronize()
    want = {k: v.cpu().numpy() for k, v in state.conns[0].items()}
    want_act = state.units["activation"].cpu().numpy()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_run, args=(r, 2, port, steps, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = _collect(q, procs, 2)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(2):
        assert got[r]["status"] == 0
        np.testing.assert_array_equal(got[r]["activation"], want_act, err_msg=f"rank {r} activations")
        assert got[r]["tail"] == int(state.tail_start.item())
    for col in want:
        np.testing.assert_array_equal(np.concatenate([got[0][col], got[1][col]]), want[col], err_msg=col)


def _per_conn_case(dev, world=1, rank=0):
    import plastax_b200 as px

    class Net(px.Network):
        forward_pass = px.ForwardPass("tanh")
        propagation = px.Propagation.PIPELINE
        prune_conn = px.MagnitudePrune(0.02)
        add_conn = px.ProposeAddConn(proposals_per_proposer=2, max_new_per_level=120, dst_lo=2,
                                     proposer="per_connection", score="uniform_q256", init=("hash_uniform", 0.1),
                                     level_cap_scope="step")

    rng = np.random.default_rng(31)
    n, e = 700, 9000
    src, dst = rng.integers(0, n, e), rng.integers(2, n, e)
    w = (rng.standard_normal(e) * 0.1).astype(np.float32)
    kw = dict(sharding=px.ShardSpec("conns", world), shard_rank=rank) if world > 1 else {}
    static, state = px.NetworkBuilder.from_edges(Net, n, src, dst, weights=w, input_ids=(0, 1), output_ids=(),
                                                 capacity_headroom=0.1, capacity_align=256, device=dev, **kw)
    return Net, static, state


def _run_per_conn(rank, world, port, steps, q):
    import datetime

    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        from plastax_b200 import StepInputs, make_step

        Net, static, state = _per_conn_case(dev, world, rank)
        step = make_step(Net, static, device=dev)
        xs = _inputs(steps, 2)
        for i in range(steps):
            step(state, StepInputs(torch.from_numpy(xs[i]).to(dev)))
        torch.cuda.synchronize()
        out = {k: v.cpu().numpy() for k, v in state.conns[0].items()}
        out["grown"] = int(state.grown.item())
        step.close()
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(600)
def test_two_rank_per_connection_proposer_equals_one_gpu(cuda):
    """The per-connection proposer under Scheme-A ranks every rank's
    connections (the bands gathered into the whole arena): two ranks grow
    exactly the edges one GPU grows."""
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from plastax_b200 import StepInputs, make_step

    steps = 3
    Net, static, state = _per_conn_case(cuda)
    step = make_step(Net, static, device=cuda)
    xs = _inputs(steps, 2)
    for i in range(steps):
        step(state, StepInputs(torch.from_numpy(xs[i]).to(cuda)))
    torch.cuda.synchronize()
    want = {k: v.cpu().numpy() for k, v in state.conns[0].items()}
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_run_per_conn, args=(r, 2, port, steps, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = _collect(q, procs, 2)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert got[0]["grown"] == got[1]["grown"] == int(state.grown.item()) > 0
    for col in want:
        np.testing.assert_array_equal(np.concatenate([got[0][col], got[1][col]]), want[col], err_msg=col)


@pytest.mark.parametrize("world", [2, 5])
def test_combine_of_emulated_ranks_on_one_gpu(cuda, world):
    """Every rank's combine (scheme_a_apply_kernel) run one after another on
    one GPU over `world` emulated regions, every flag set beforehand so no
    wait depends on another kernel: each rank reduces its slice of the
    units from every region (exact int64 sum, the float side added in rank
    order), skips inputs and pruned units, and stores the activation into
    every region."""
    import torch

    from plastax_b200 import _lib
    from plastax_b200.peers import scheme_a_apply

    n = 10_001
    rng = np.random.default_rng(17)
    fixed = [torch.from_numpy(rng.integers(-(1 << 33), 1 << 33, n)).to(cuda) for _ in range(world)]
    side = [torch.from_numpy((rng.standard_normal(n) * 1e-3).astype(np.float32)).to(cuda) for _ in range(world)]
    for q in range(world):  # units whose fixed-point sum is zero take the side sum alone
        fixed[q][:50] = 0
    act = [torch.full((n,), 7.0, dtype=torch.float32, device=cuda) for _ in range(world)]
    flags = [torch.ones(2 * world, dtype=torch.int32, device=cuda) for _ in range(world)]
    role = np.zeros(n, np.uint8)
    role[rng.choice(n, 300, replace=False)] = 1
    pruned = (rng.random(n) < 0.05).astype(np.uint8)
    arr = lambda ts: torch.tensor([t.data_ptr() for t in ts], dtype=torch.int64, device=cuda)  # noqa: E731
    p_fixed, p_side, p_act, p_flags = arr(fixed), arr(side), arr(act), arr(flags)
    words = [torch.zeros(4, dtype=torch.int32, device=cuda) for _ in range(world)]
    for r in range(world):
        w = words[r].data_ptr()

        class G:
            struct = _lib.PeerGroup(r, world, p_fixed.data_ptr(), p_side.data_ptr(), p_act.data_ptr(),
                                    p_flags.data_ptr(), None, w, w + 4, w + 8)

        G.n = n
        scheme_a_apply(G, "identity", is_input=torch.from_numpy(role).to(cuda),
                       pruned=torch.from_numpy(pruned).to(cuda), wait_polls=1000)
    torch.cuda.synchronize()
    assert [int(wd[2].item()) for wd in words] == [0] * world
    f = sum(x.cpu().numpy() for x in fixed)
    s = np.zeros(n, np.float32)
    for q in range(world):
        s = (s + side[q].cpu().numpy()).astype(np.float32)
    want = np.where(f != 0, (f.astype(np.float32) * np.float32(2.0 ** -_lib.FIXED_FRAC_BITS)) + s, s)
    want = want.astype(np.float32)
    skip = (role == 1) | (pruned == 1)
    want[skip] = 7.0
    for q in range(world):
        np.testing.assert_array_equal(act[q].cpu().numpy(), want, err_msg=f"region {q}")
