"""The training configurations at their stated shapes (plastax_b200/configs.py)
against the oracle, on the GPU.

- C2, the sparse MLP 784-1000-1000-10 at density 0.1 (179 K edges), B=256:
  two batched steps (forward, softmax cross-entropy, backward, the exact
  batch-mean SGD update, the mean reduction) against oracle/batched.py,
  within 1e-5 relative / 1e-6 absolute per value.
- C3, dynamic sparse training (4,168 units, 2^20 live edges, k = 10,486 every
  100 steps): the structural steps 0 and 100 and the plain step 1. Each
  checked step starts the oracle from the GPU's state before it. Its forward
  phase (forward, backward, SGD) matches within tolerance; then, teacher
  forced (the oracle's activations and gradients replaced by the GPU's,
  its SGD rerun from the GPU's weights), its structural phase (exact
  lowest-|w| prune, 64 per-unit proposals scored |grad * act|, the total
  order, the step-scope selection, the pipeline claim) gives the GPU's
  columns bit for bit.
- C4, the unit lifecycle (8,192 of 65,536 unit slots, 2^22 edge slots,
  UPGD): 20 steps of the configuration's own step (a unit spawned every 10
  steps, units below the 1st utility percentile pruned), then its unit
  phases from the reached state against oracle/units.py bit for bit.
"""

from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-5, 1e-6


def _host(state):
    return ([{k: v.cpu().numpy().copy() for k, v in b.items()} for b in state.conns],
            {k: v.cpu().numpy().copy() for k, v in state.units.items()})


def test_c2_sparse_mlp_steps_match_the_restatement(cuda):
    import plastax_b200 as px
    from oracle.batched import batched_step
    from plastax_b200 import configs as C

    cfg = C.C2
    net, static, state = C.build_mlp(cfg, cuda)
    assert state.conns and sum(int((b["dead"] == 0).sum()) for b in state.conns) > 170_000
    step = px.make_step(net, static, batch_size=cfg.batch, device=cuda)
    host, units = _host(state)
    level = units["level"]
    is_input = np.zeros(level.size, np.uint8)
    is_input[list(static.input_ids)] = 1
    rng = np.random.default_rng(5)
    for it in range(2):
        x, t = C.mlp_batch(cfg, rng)
        res = step(state, px.StepInputs(x, t))
        want = batched_step(host, level, is_input, static.input_ids, static.output_ids, x, t, fwd_act="relu",
                            bwd_act="relu", loss="softmax", opt=net.update_conn.oracle_args(), out_act="identity")
        np.testing.assert_allclose(float(res.loss.item()), float(want["loss"]), rtol=RTOL, atol=ATOL)
        got = {k: v.cpu().numpy() for k, v in state.units.items()}
        np.testing.assert_allclose(got["activation"], want["activation"], rtol=RTOL, atol=ATOL,
                                   err_msg=f"step {it} activation")
        np.testing.assert_allclose(got["grad_pre_act"], want["grad"], rtol=RTOL, atol=ATOL, err_msg=f"step {it} grad")
        for bi, b in enumerate(state.conns):
            np.testing.assert_allclose(b["weight"].cpu().numpy(), host[bi]["weight"], rtol=RTOL, atol=ATOL,
                                       err_msg=f"step {it} bucket {bi} weights")
            np.testing.assert_array_equal(b["dead"].cpu().numpy(), host[bi]["dead"])


def _dst_inputs(cfg, rng):
    from plastax_b200 import configs as C

    w1, w2 = C.dst_teacher(cfg)
    x = rng.standard_normal(cfg.num_inputs).astype(np.float32)
    t = (w2 @ np.tanh(w1 @ x)).astype(np.float32)
    return x, t


def test_c3_dst_structural_steps_match_the_oracle_teacher_forced(cuda):
    import torch

    import plastax_b200 as px
    from oracle import oracle as orc
    from oracle.steps import DstOracle
    from plastax_b200 import configs as C

    cfg = C.C3
    net, static, state = C.build_dst(cfg, cuda)
    step = px.make_step(net, static, device=cuda)
    rng = np.random.default_rng(3)
    threads = max(1, min(16, orc.max_threads()))
    checked = {0: True, 1: False, 100: True}
    for i in range(101):
        x, t = _dst_inputs(cfg, rng)
        if i not in checked:
            step(state, px.StepInputs(x, t))
            continue
        (b,), u = _host(state)
        tail = int(state.tail_start.item())
        res = step(state, px.StepInputs(x, t))
        torch.cuda.synchronize()
        (gb,), gu = _host(state)
        # the forward phase from the same starting state: floats within tolerance
        ro = DstOracle({k: v.copy() for k, v in b.items()}, u["activation"].copy(), u["grad_pre_act"].copy(),
                       u["level"], tail, num_inputs=cfg.num_inputs, num_outputs=cfg.num_outputs, lr=cfg.lr,
                       k=cfg.k, every=cfg.every, proposals=cfg.proposals, seed=cfg.seed, threads=threads)
        ro.step_count = i
        loss = ro.forward_phase(x, t)
        np.testing.assert_allclose(float(res.loss.item()), loss, rtol=RTOL, atol=ATOL, err_msg=f"step {i} loss")
        np.testing.assert_allclose(gu["activation"], ro.act, rtol=RTOL, atol=ATOL, err_msg=f"step {i} activation")
        np.testing.assert_allclose(gu["grad_pre_act"], ro.grad, rtol=RTOL, atol=ATOL, err_msg=f"step {i} grad")
        fwd_w = ro.b["weight"].copy()  # the oracle's own SGD, before any structural change
        assert ro.fires() == checked[i]
        if not checked[i]:
            for name in ("dead", "from_id", "to_id"):
                np.testing.assert_array_equal(gb[name], b[name], err_msg=f"plain step {i} changed {name}")
            live = gb["dead"] == 0
            np.testing.assert_allclose(gb["weight"][live], fwd_w[live], rtol=RTOL, atol=ATOL,
                                       err_msg=f"step {i} weights")
            continue
        # teacher forced: the GPU's activations and gradients, SGD from the GPU's starting weights
        tf = {k: v.copy() for k, v in b.items()}
        ro.b = tf
        ro.act[:] = gu["activation"]
        ro.grad[:] = gu["grad_pre_act"]
        orc.update_conn(tf, ro.grad, ro.act, ro.n, dict(kind="sgd", lr=cfg.lr))
        before = {k: v.copy() for k, v in tf.items()}
        ro.structural_phase()
        assert ro.last_pruned == cfg.k
        touched = np.zeros(tf["dead"].size, bool)
        for name in ("dead", "from_id", "to_id", "weight"):
            touched |= before[name] != tf[name]
        assert int(((tf["dead"] == 0) & touched).sum()) > 0, f"step {i}: nothing regrown"
        for name in ("dead", "from_id", "to_id", "weight"):
            np.testing.assert_array_equal(gb[name], tf[name], err_msg=f"step {i} structural {name}")
        # the untouched live edges also carry the oracle's own (not forced) SGD within tolerance
        keep = (gb["dead"] == 0) & ~touched
        np.testing.assert_allclose(gb["weight"][keep], fwd_w[keep], rtol=RTOL, atol=ATOL, err_msg=f"step {i} weights")
        assert int(state.tail_start.item()) == ro.tail


def test_c4_unit_phases_at_the_stated_shape_match_the_oracle(cuda):
    import torch

    import plastax_b200 as px
    from oracle import units as ou
    from plastax_b200 import configs as C

    cfg = C.C4
    net, static, state = C.build_units(cfg, cuda)
    step = px.make_step(net, static, device=cuda)
    rng = np.random.default_rng(4)
    tmap = C.units_target_map(cfg, 0)
    added = 0
    for _ in range(20):
        x = rng.standard_normal(cfg.num_inputs).astype(np.float32)
        step(state, px.StepInputs(x, np.array([float(tmap @ x)], np.float32)))
        added += int(state.units_added.item())
    assert added == 2, f"a unit spawns every {cfg.interval} steps, {added} in 20"
    units0 = {k: v.cpu().numpy() for k, v in state.units.items()}
    assert int(units0["pruned"].sum()) > 0, "no unit was pruned"
    # the unit phases from the reached state, on the device and in the oracle
    host, units = _host(state)
    assert state.step % cfg.interval == 0
    step._update_unit(state)
    step._prune_unit(state)
    step._add_unit(state)
    torch.cuda.synchronize()
    exempt = np.zeros(cfg.unit_capacity, bool)
    exempt[list(static.input_ids) + list(static.output_ids)] = True
    defaults = {name: np.zeros((), units[name].dtype) for name in units if name not in ("level", "pruned")}
    pruned = units["pruned"]
    ou.update_unit(units, pruned, net.update_unit)
    doomed = ou.prune_unit(units, pruned, exempt, defaults, host, net.prune_unit)
    children, overflow = ou.add_unit(units, pruned, units["level"], defaults, net.add_unit, int(net.max_levels))
    assert doomed.sum() > 0 and len(children) == 1 and not overflow
    got = {k: v.cpu().numpy() for k, v in state.units.items()}
    for name in units:
        np.testing.assert_array_equal(got[name], units[name], err_msg=name)
    for bk, ref in zip(state.conns, host, strict=True):
        np.testing.assert_array_equal(bk["dead"].cpu().numpy(), ref["dead"])
    assert int(state.units_added.item()) == 1 and not bool(state.unit_overflow.item())
