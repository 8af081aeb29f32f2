"""UPGD on the GPU (examples/upgd.py:135-208) against oracle/upgd.py.

Parity unpinned against the reference (the rule lives in an example, with no
golden vectors): the oracle restates it operation by operation in float32.
The utility trace and the step column are elementwise float32 arithmetic in
the same order on both sides and must match exactly; the weight goes through
pow / exp / log / cos, whose last bits differ between libraries, and must
match within 1e-5 relative / 1e-6 absolute.

- The fused backward + update kernel with the UPGD bundle, on a random bucket
  with tombstones, several steps in a row (the step column advances).
- One step of a TOPOLOGICAL MLP with the UPGD bundle: the local utility
  scale written by the step (each destination's max over its incoming
  utilities, before the update) and the updated columns, from the step's own
  gradients and activations; then the v0 (global) scale set by the caller.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import upgd as ou
from tests._arena import random_bucket, to_device

pytestmark = pytest.mark.gpu

KW = dict(lr=0.05, beta=0.9, sigma=0.01, eps=1e-8)


def test_upgd_kernel_matches_the_oracle(cuda):
    import torch

    from plastax_b200 import kernels as K
    from plastax_b200 import optim

    rng = np.random.default_rng(21)
    n, cap, live = 3000, 40_000, 36_000
    b = random_bucket(rng, n, cap, live, dead_frac=0.05)
    b["upgd/util"] = np.zeros(cap, np.float32)
    b["upgd/t"] = np.zeros(cap, np.float32)
    grad = (rng.standard_normal(n) * 0.3).astype(np.float32)
    act = np.tanh(rng.standard_normal(n)).astype(np.float32)
    eta = np.abs(rng.standard_normal(n) * 0.01).astype(np.float32)
    eta[::7] = -np.inf  # destinations with no incoming utility: the floor applies
    db = to_device(b, cuda)
    g_d, a_d, e_d = (torch.from_numpy(x).to(cuda) for x in (grad, act, eta))
    opt = optim.upgd(**KW)
    st = opt.struct(e_d)
    for _ in range(3):
        K.backward_update(db, g_d, a_d, None, st, opt.cols)
        ou.update(b, grad, act, eta, **KW)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(db["upgd/t"].cpu().numpy(), b["upgd/t"])
    np.testing.assert_allclose(db["upgd/util"].cpu().numpy(), b["upgd/util"], rtol=1e-5, atol=1e-7)
    np.testing.assert_allclose(db["weight"].cpu().numpy(), b["weight"], rtol=1e-5, atol=1e-6)
    assert float(np.abs(b["upgd/util"]).max()) > 0


def _mlp(cuda, eta_mode):
    import plastax_b200 as px

    class Net(px.Network):
        forward_pass = px.ForwardPass("relu")
        backward_pass = px.BackwardPass("relu")
        loss = px.MSELoss()
        update_conn = px.optim.upgd(**KW, eta=eta_mode)

    rng = np.random.default_rng(8)
    layers = (0, 16, 80, 140, 144)
    src, dst = [], []
    for lo, mid, hi in zip(layers[:-2], layers[1:-1], layers[2:], strict=True):
        for d in range(mid, hi):
            for s_ in rng.choice(np.arange(lo, mid), size=6, replace=False):
                src.append(int(s_))
                dst.append(d)
    src, dst = np.array(src), np.array(dst)
    w = (rng.standard_normal(src.size) * 0.4).astype(np.float32)
    static, state = px.NetworkBuilder.from_edges(Net, 144, src, dst, weights=w, input_ids=tuple(range(16)),
                                                 output_ids=tuple(range(140, 144)), capacity_headroom=0.1,
                                                 device=cuda)
    # a non-zero utility history, so the scale is not all zeros
    import torch

    for b in state.conns:
        hist = (np.random.default_rng(3).standard_normal(b["dead"].numel()) * 0.01).astype(np.float32)
        b["upgd/util"].copy_(torch.from_numpy(hist))
        b["upgd/t"].fill_(4.0)
    return Net, static, state


@pytest.mark.parametrize("eta_mode", ["local", "global"])
def test_upgd_step_matches_the_oracle(cuda, eta_mode):
    import torch

    import plastax_b200 as px

    Net, static, state = _mlp(cuda, eta_mode)
    step = px.make_step(Net, static, device=cuda)
    rng = np.random.default_rng(1)
    x = rng.standard_normal(16).astype(np.float32)
    t = rng.standard_normal(4).astype(np.float32)
    if eta_mode == "global":
        px.optim.upgd_global_eta(state)
    before = [{k: v.cpu().numpy().copy() for k, v in b.items()} for b in state.conns]
    eta_before = state.units["upgd/eta"].cpu().numpy().copy()
    step(state, px.StepInputs(x, t))
    torch.cuda.synchronize()
    units = {k: v.cpu().numpy() for k, v in state.units.items()}
    n = static.num_units
    if eta_mode == "local":
        skip = np.zeros(n, bool)
        skip[list(static.input_ids)] = True
        eta = ou.eta_local(before, n, "upgd/util", eta_before, skip)
    else:
        live_util = np.concatenate([b["upgd/util"][b["dead"] == 0] for b in before])
        eta = np.full(n, max(max(0.0, float(live_util.max())), 1e-8), np.float32)
    np.testing.assert_array_equal(units["upgd/eta"], eta)
    for bk, ref in zip(state.conns, before, strict=True):
        ou.update(ref, units["grad_pre_act"], units["activation"], eta, **KW)
        np.testing.assert_array_equal(bk["upgd/t"].cpu().numpy(), ref["upgd/t"])
        np.testing.assert_allclose(bk["upgd/util"].cpu().numpy(), ref["upgd/util"], rtol=1e-5, atol=1e-7)
        np.testing.assert_allclose(bk["weight"].cpu().numpy(), ref["weight"], rtol=1e-5, atol=1e-6)
