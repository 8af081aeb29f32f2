"""The streaming echo-state reservoir (1,024 tanh units, fan-in 16, a linear
readout trained online by LMS) on the GPU against the oracle's ESN step
(oracle/steps.EsnOracle).

- Per step, at checkpoints: one oracle step from the GPU's own pre-step
  state matches the GPU step within 1e-5 relative / 1e-6 absolute
  (activations, every weight, the loss).
- Drift over 10,000 steps of the reservoir and readout: a free-running
  oracle from the same start stays within 1e-4 of the GPU (the reservoir
  contracts at spectral radius 0.9).
- The online LMS (lr 1e-3) over 300 steps, checked every 30 steps (no drift
  bound there: two free-running copies part at the rate the update grows).
  Run longer it diverges, on the oracle as on the GPU: in a PIPELINE sweep the
  readout's output reads the previous step's reservoir state while the
  delta rule reads the current one, and that lag makes the update grow
  without bound for any learning rate.
"""

from __future__ import annotations

import dataclasses

import numpy as np
import pytest

from oracle.steps import EsnOracle

pytestmark = pytest.mark.gpu


def _snapshot(state):
    return ({k: v.cpu().numpy().copy() for k, v in state.conns[0].items()},
            state.units["activation"].cpu().numpy().copy())


def _run(cuda, lr, steps, every, drift_bound):
    import torch

    import plastax_b200 as px
    from plastax_b200.configs import C1, build_esn

    cfg = dataclasses.replace(C1, lr=lr)
    net, static, state = build_esn(cfg, cuda)
    out = cfg.units + 1
    b0, act0 = _snapshot(state)
    free = EsnOracle(b0, act0, input_id=0, output_id=out, lr=cfg.lr)
    step = px.make_step(net, static, device=cuda)
    xs = np.random.default_rng(0).standard_normal(steps).astype(np.float32)
    for t in range(steps):
        x = xs[t]
        target = xs[t - cfg.delay] if t >= cfg.delay else np.float32(0.0)
        inputs = px.StepInputs(np.array([x], np.float32), np.array([target], np.float32))
        one = None
        if t % every == 0 or t == steps - 1:
            bs, acts = _snapshot(state)
            one = EsnOracle(bs, acts, input_id=0, output_id=out, lr=cfg.lr)
            one_loss = one.step(float(x), float(target))
        if t == 1:
            step.capture(state, inputs)
        res = step(state, inputs)
        free.step(float(x), float(target))
        if one is not None:
            b, act = _snapshot(state)
            np.testing.assert_allclose(act, one.act, rtol=1e-5, atol=1e-6, err_msg=f"step {t} activations")
            np.testing.assert_allclose(b["weight"], one.b["weight"], rtol=1e-5, atol=1e-6,
                                       err_msg=f"step {t} weights")
            np.testing.assert_allclose(float(res.loss.item()), one_loss, rtol=1e-5, atol=1e-6,
                                       err_msg=f"step {t} loss")
    torch.cuda.synchronize()
    if drift_bound is not None:
        b, act = _snapshot(state)
        drift_act = float(np.max(np.abs(act - free.act)))
        drift_w = float(np.max(np.abs(b["weight"] - free.b["weight"])))
        assert drift_act < drift_bound and drift_w < drift_bound, (drift_act, drift_w)


def test_esn_ten_thousand_steps_drift(cuda):
    _run(cuda, 0.0, 10_000, 500, 1e-4)


def test_esn_online_lms(cuda):
    # per step only: the lagged update amplifies any difference between two
    # free-running copies (last-bit sum orders included), so no drift bound
    _run(cuda, 1e-3, 300, 30, None)
