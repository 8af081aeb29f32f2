"""The growth selection shared out over the ranks of a Scheme-A group
(pxb_propose_select_unique_sharded), with the ranks emulated on one GPU.

Each emulated rank's call ranks its share of the full bins and stores the
winners into every rank's columns; the calls run one after another on one
stream, so no kernel waits on another. Once every rank has run, every rank's
list must equal the one-rank selection's row for row, only the list of
(step mod blocks) may be written, and pxb_select_take must copy that list
out.
"""

from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SENTINEL = 0x5A


def _k():
    from plastax_b200 import kernels

    return kernels


@pytest.mark.parametrize("n,k,levels,world,blocks,opts", [
    (5000, 1300, 2, 2, 3, {}), (1 << 16, 20_000, 3, 3, 3, {"direction": 1}), (40_000, 9000, 5, 8, 2,
                                                                              {"pruned": True}),
    (70_000, 70_000, 2, 4, 3, {}), (20_000, 19_990, 8, 5, 1, {"gap": 0}), (777, 1, 2, 2, 3, {}),
    (1_048_592, 268_435, 1, 8, 3, {})])
def test_shared_selection_equals_the_one_rank_selection(cuda, n, k, levels, world, blocks, opts):
    import torch

    kern = _k()
    rng = np.random.default_rng(41)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)  # noqa: E731
    level = np.sort(rng.integers(0, levels, n)).astype(np.int32)
    d_level = t(level)
    d_pruned = t((rng.random(n) < 0.2).astype(np.uint8)) if opts.get("pruned") else None
    seed, step, dst_lo = 11, 37, 3
    kw = dict(dst_lo=dst_lo, dst_n=n - dst_lo, score_kind=0, level=d_level, k=k, num_levels=levels, init_kind=2,
              init_a=0.05, pruned=d_pruned, max_level_gap=opts.get("gap", 1), direction=opts.get("direction", 0))
    step_dev = torch.tensor([step], dtype=torch.int32, device=cuda)
    want = kern.propose_select_unique(n, seed, step, step_dev=step_dev, **kw)
    want = [c.cpu().numpy() for c in want]
    # every emulated rank's columns: `blocks` lists of k, a sentinel first
    cols = []
    for _ in range(world):
        cols.append((torch.full((blocks * k,), SENTINEL, dtype=torch.int32, device=cuda),
                     torch.full((blocks * k,), SENTINEL, dtype=torch.int32, device=cuda),
                     torch.full((blocks * k,), float(SENTINEL), dtype=torch.float32, device=cuda),
                     torch.full((blocks * k,), SENTINEL, dtype=torch.uint8, device=cuda)))
    ptrs = [tuple(c.data_ptr() for c in cs) for cs in cols]
    status = torch.zeros(world, dtype=torch.int32, device=cuda)
    for r in range(world):
        shard = kern.select_shard(r, world, blocks, ptrs)
        kern.propose_select_unique(n, seed, step, step_dev=step_dev, status=status[r:r + 1], shard=shard, **kw)
    torch.cuda.synchronize()
    assert status.cpu().tolist() == [0] * world
    b = step % blocks
    for r in range(world):
        for name, col, ref in zip(("src", "dst", "weight", "growable"), cols[r], want, strict=True):
            got = col.cpu().numpy().reshape(blocks, k)
            np.testing.assert_array_equal(got[b], ref, err_msg=f"rank {r} {name}")
            others = np.delete(got, b, axis=0)
            assert (others == SENTINEL).all(), f"rank {r} {name}: a list other than step mod blocks was written"
    # the take copies list (step mod blocks) out in one launch
    out = (torch.empty(k, dtype=torch.int32, device=cuda), torch.empty(k, dtype=torch.int32, device=cuda),
           torch.empty(k, dtype=torch.float32, device=cuda), torch.empty(k, dtype=torch.uint8, device=cuda))
    kern.select_take(k, blocks, step_dev, cols[world - 1], out)
    for name, col, ref in zip(("src", "dst", "weight", "growable"), out, want, strict=True):
        np.testing.assert_array_equal(col.cpu().numpy(), ref, err_msg=f"take {name}")


def test_shared_selection_rotates_with_the_device_step(cuda):
    """Under graph replay the device step picks the list: three calls at
    steps s, s + 1, s + 2 fill the three lists, each equal to its step's
    one-rank selection."""
    import torch

    kern = _k()
    n, k, levels, world, blocks = 9000, 2000, 2, 2, 3
    rng = np.random.default_rng(42)
    level = torch.from_numpy(np.sort(rng.integers(0, levels, n)).astype(np.int32)).to(cuda)
    kw = dict(dst_lo=0, dst_n=n, score_kind=1, level=level, k=k, num_levels=levels, init_kind=0, init_a=0.25)
    cols = [(torch.zeros(blocks * k, dtype=torch.int32, device=cuda),
             torch.zeros(blocks * k, dtype=torch.int32, device=cuda),
             torch.zeros(blocks * k, dtype=torch.float32, device=cuda),
             torch.zeros(blocks * k, dtype=torch.uint8, device=cuda)) for _ in range(world)]
    ptrs = [tuple(c.data_ptr() for c in cs) for cs in cols]
    step_dev = torch.zeros(1, dtype=torch.int32, device=cuda)
    base = 100
    for i in range(blocks):
        step_dev.fill_(base + i)
        for r in range(world):
            kern.propose_select_unique(n, 5, 0, step_dev=step_dev, shard=kern.select_shard(r, world, blocks, ptrs),
                                       **kw)
    for i in range(blocks):
        want = kern.propose_select_unique(n, 5, base + i, **kw)
        b = (base + i) % blocks
        for r in range(world):
            for col, ref in zip(cols[r], want, strict=True):
                np.testing.assert_array_equal(col.cpu().numpy().reshape(blocks, k)[b], ref.cpu().numpy())


def test_selection_forked_at_the_sweep_launch_changes_nothing(cuda):
    """Where the next step's selection forks (the step's start, just before
    the sweep with the sweep launched first, the sweep's end, or after the
    propagation) is only a scheduling choice: eager steps and graph replays
    are equal."""
    import torch

    from plastax_b200 import StepInputs, make_step
    from plastax_b200.configs import ReservoirConfig, build_reservoir

    cfg = ReservoirConfig(num_units=1 << 12, fan_in=16, churn=0.01, capacity_align=256)
    xs = np.random.default_rng(8).standard_normal((7, cfg.num_inputs)).astype(np.float32)
    got = []
    for mode in ("start", "launch", "post", "sweep"):
        net, static, state = build_reservoir(cfg, cuda)
        step = make_step(net, static, device=cuda)
        assert step.ahead
        step.select_after_sweep = mode == "sweep"
        step.select_at_launch = mode == "launch"
        step.select_post_sweep = mode == "post"
        for i in range(len(xs)):
            x = StepInputs(torch.from_numpy(xs[i]).to(cuda))
            if i == 3:
                step.capture(state, x)
            step(state, x)
        torch.cuda.synchronize()
        assert int(state.grown.item()) > 0
        got.append({**{c: v.cpu().numpy() for c, v in state.conns[0].items()},
                    "activation": state.units["activation"].cpu().numpy()})
        step.close()
    for j in range(1, len(got)):
        for c in got[0]:
            np.testing.assert_array_equal(got[j][c], got[0][c], err_msg=f"{c} (fork mode {j})")
