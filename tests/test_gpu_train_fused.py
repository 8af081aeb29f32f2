"""The fused pipeline training step (csrc/train.cu) against the separate
passes it replaces and against the oracle, on the GPU.

The same PIPELINE net and state are stepped twice: through the fused step
(forward and backward accumulated in one pass, exact fixed-point sums, the
applies and MSE seed, then the update) and through the separate canonical
passes (make_step(fuse_train=False)). Activations, gradients, seeds, the loss
and every weight and optimizer column agree within 1e-5 relative / 1e-6
absolute over several steps, for every fused optimizer; the delta-rule
readout without a backward pass (an ESN) and products beyond the fixed-point
range (the float side) too. One step is also checked against the oracle's
passes (oracle/pxo.c) directly.
"""

from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-5, 1e-6


def _net(opt, backward=True, grad_field=None):
    import plastax_b200 as px

    attrs = dict(forward_pass=px.ForwardPass("tanh", output_activation="identity"), loss=px.MSELoss(),
                 update_conn=opt, propagation=px.Propagation.PIPELINE)
    if backward:
        attrs["backward_pass"] = px.BackwardPass("tanh")
    return type("Net", (px.Network,), attrs)


def _edges(rng, n, e, n_in):
    src = rng.integers(0, n, e)
    dst = rng.integers(n_in, n, e)
    w = (rng.standard_normal(e) / np.sqrt(max(1, e // n))).astype(np.float32)
    return src, dst, w


def _pair(cuda, Net, n, src, dst, w, n_in, n_out):
    import plastax_b200 as px

    out = []
    for fuse in (True, False):
        static, state = px.NetworkBuilder.from_edges(Net, n, src, dst, weights=w, input_ids=tuple(range(n_in)),
                                                     output_ids=tuple(range(n - n_out, n)), capacity_headroom=0.3,
                                                     device=cuda)
        step = px.make_step(Net, static, device=cuda, fuse_train=fuse)
        assert step.train_fused == fuse
        out.append((static, state, step))
    return out


def _compare(a, b, what):
    for name in a.units:
        np.testing.assert_allclose(a.units[name].cpu().numpy(), b.units[name].cpu().numpy(), rtol=RTOL, atol=ATOL,
                                   err_msg=f"{what}: unit column {name}")
    for ba, bb in zip(a.conns, b.conns, strict=True):
        for col in ba:
            if col in ("dead", "from_id", "to_id"):
                np.testing.assert_array_equal(ba[col].cpu().numpy(), bb[col].cpu().numpy(), err_msg=f"{what} {col}")
            else:
                np.testing.assert_allclose(ba[col].cpu().numpy(), bb[col].cpu().numpy(), rtol=RTOL, atol=ATOL,
                                           err_msg=f"{what}: conn column {col}")


@pytest.mark.parametrize("opt_kind,n", [("sgd", 3000), ("momentum", 3000), ("adam", 3000), ("rmsprop", 3000),
                                        ("sgd", 9000), ("adam", 14000)])
def test_fused_step_equals_the_separate_passes(cuda, opt_kind, n):
    """From 3,000 units up to 14,000, near the largest count whose four
    accumulator words per unit fit one CTA's shared memory."""
    import plastax_b200 as px

    opt = {"sgd": px.optim.sgd(0.01), "momentum": px.optim.momentum(0.01, 0.9), "adam": px.optim.adam(0.003),
           "rmsprop": px.optim.rmsprop(0.003)}[opt_kind]
    Net = _net(opt)
    rng = np.random.default_rng(7)
    n_in, n_out = 16, 8
    src, dst, w = _edges(rng, n, 30 * n, n_in)
    (_, sa, fa), (_, sb, fb) = _pair(cuda, Net, n, src, dst, w, n_in, n_out)
    for i in range(6):
        x = rng.standard_normal(n_in).astype(np.float32)
        t = rng.standard_normal(n_out).astype(np.float32)
        la = fa(sa, px.StepInputs(x, t)).loss
        lb = fb(sb, px.StepInputs(x, t)).loss
        np.testing.assert_allclose(float(la.item()), float(lb.item()), rtol=RTOL, atol=ATOL, err_msg=f"loss {i}")
        _compare(sa, sb, f"{opt_kind} step {i}")


def test_fused_readout_without_a_backward(cuda):
    """The ESN's delta rule: no backward pass, the update reads the loss
    seed column (grad_field = loss_grad)."""
    import plastax_b200 as px
    from plastax_b200.traits import LOSS_GRAD

    Net = _net(px.optim.sgd(0.01, grad_field=LOSS_GRAD), backward=False)
    rng = np.random.default_rng(8)
    n, n_in, n_out = 1026, 1, 1
    src, dst, w = _edges(rng, n, 18_000, n_in)
    (_, sa, fa), (_, sb, fb) = _pair(cuda, Net, n, src, dst, w, n_in, n_out)
    for i in range(8):
        x = rng.standard_normal(n_in).astype(np.float32)
        t = rng.standard_normal(n_out).astype(np.float32)
        fa(sa, px.StepInputs(x, t))
        fb(sb, px.StepInputs(x, t))
        _compare(sa, sb, f"readout step {i}")


def test_fused_products_beyond_the_fixed_range(cuda):
    """Products of magnitude >= 2^20 and non-finite ones take the float side
    of both sums; the rest stay exact."""
    import torch

    import plastax_b200 as px

    Net = _net(px.optim.sgd(1e-9))
    rng = np.random.default_rng(9)
    n, n_in, n_out = 500, 4, 2
    src, dst, w = _edges(rng, n, 8000, n_in)
    w[:5] = 3.0e6  # w * act up to 3e6 (tanh act <= 1, inputs ~N(0,1))
    (_, sa, fa), (_, sb, fb) = _pair(cuda, Net, n, src, dst, w, n_in, n_out)
    for s in (sa, sb):
        s.units["activation"][n_in:].copy_(torch.linspace(-1, 1, n - n_in, device=cuda))
    for i in range(3):
        x = (rng.standard_normal(n_in) * 4).astype(np.float32)
        t = rng.standard_normal(n_out).astype(np.float32)
        fa(sa, px.StepInputs(x, t))
        fb(sb, px.StepInputs(x, t))
        _compare(sa, sb, f"side step {i}")


def test_fused_step_matches_the_oracle_passes(cuda):
    """One fused step against oracle/pxo.c's forward, apply, MSE seed,
    backward, apply and SGD update on the same host copy."""
    import torch

    import plastax_b200 as px
    from oracle import oracle as orc

    Net = _net(px.optim.sgd(0.02))
    rng = np.random.default_rng(10)
    n, n_in, n_out = 2000, 8, 4
    src, dst, w = _edges(rng, n, 60_000, n_in)
    static, state = px.NetworkBuilder.from_edges(Net, n, src, dst, weights=w, input_ids=tuple(range(n_in)),
                                                 output_ids=tuple(range(n - n_out, n)), device=cuda)
    step = px.make_step(Net, static, device=cuda)
    assert step.train_fused
    act0 = np.tanh(rng.standard_normal(n)).astype(np.float32)
    grad0 = (rng.standard_normal(n) * 0.1).astype(np.float32)
    state.units["activation"].copy_(torch.from_numpy(act0))
    state.units["grad_pre_act"].copy_(torch.from_numpy(grad0))
    b = {k: v.cpu().numpy().copy() for k, v in state.conns[0].items()}
    x = rng.standard_normal(n_in).astype(np.float32)
    t = rng.standard_normal(n_out).astype(np.float32)
    res = step(state, px.StepInputs(x, t))
    # the oracle
    is_in = np.zeros(n, np.uint8)
    is_in[:n_in] = 1
    out = np.arange(n - n_out, n)
    act = act0.copy()
    act[:n_in] = x
    acc = np.zeros(n, np.float32)
    orc.forward_accumulate(b, act, n, "sum", acc)
    new = act.copy()
    orc.unit_apply(n, 0, "tanh", "sum", acc.copy(), None, None, None, 0, is_in, None, new)
    new[out] = acc[out]
    seed = np.zeros(n, np.float32)
    seed[out] = new[out] - t
    loss = np.float32(0)
    for d in seed[out]:
        loss = np.float32(loss + np.float32(np.float32(0.5) * d) * d)
    acc = np.zeros(n, np.float32)
    orc.backward_accumulate(b, grad0, n, "sum", acc)
    g = grad0.copy()
    orc.unit_apply(n, 1, "tanh", "sum", acc.copy(), new, seed, None, 0, None, None, g)
    g[out] = acc[out] + seed[out]
    orc.update_conn(b, g, new, n, dict(kind="sgd", lr=0.02))
    got = {k: v.cpu().numpy() for k, v in state.units.items()}
    np.testing.assert_allclose(float(res.loss.item()), float(loss), rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(got["activation"], new, rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(got["grad_pre_act"], g, rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(got["loss_grad"][out], seed[out], rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(state.conns[0]["weight"].cpu().numpy(), b["weight"], rtol=RTOL, atol=ATOL)


def test_plain_graph_replay_equals_eager_steps(cuda):
    """A DST-shaped net (prune and growth every 5 steps) with auto_graphs:
    the plain and the structural steps each replay their own CUDA graph
    (captured at their second occurrence) and give the same state bit for
    bit as every step eager (the fused sums are exact, so the two runs are
    deterministic)."""
    import torch

    import plastax_b200 as px

    class Net(px.Network):
        forward_pass = px.ForwardPass("tanh", output_activation="identity")
        backward_pass = px.BackwardPass("tanh")
        loss = px.MSELoss()
        update_conn = px.optim.sgd(0.01)
        prune_conn = px.LowestMagnitudePrune(300, every=5)
        add_conn = px.ProposeAddConn(proposals_per_proposer=8, max_new_per_level=300, dst_lo=8, score="grad_act",
                                     level_cap_scope="step", trigger=("every", 5))
        propagation = px.Propagation.PIPELINE

    rng = np.random.default_rng(12)
    n, n_in, n_out = 1200, 8, 4
    src, dst, w = _edges(rng, n, 30_000, n_in)
    runs = []
    for graph in (False, True):
        static, state = px.NetworkBuilder.from_edges(Net, n, src, dst, weights=w, input_ids=tuple(range(n_in)),
                                                     output_ids=tuple(range(n - n_out, n)), capacity_headroom=0.2,
                                                     device=cuda)
        step = px.make_step(Net, static, device=cuda)
        assert step.train_fused and not step.capturable() and step.period() == 5
        step.auto_graphs = graph
        g = np.random.default_rng(3)
        for i in range(17):
            x = g.standard_normal(n_in).astype(np.float32)
            t = g.standard_normal(n_out).astype(np.float32)
            step(state, px.StepInputs(x, t))
        torch.cuda.synchronize()
        assert len(step._graphs) == (2 if graph else 0)
        runs.append(state)
    a, b = runs
    for name in a.units:
        np.testing.assert_array_equal(a.units[name].cpu().numpy(), b.units[name].cpu().numpy(), err_msg=name)
    for col in a.conns[0]:
        np.testing.assert_array_equal(a.conns[0][col].cpu().numpy(), b.conns[0][col].cpu().numpy(), err_msg=col)
    assert int(a.tail_start.item()) == int(b.tail_start.item())
