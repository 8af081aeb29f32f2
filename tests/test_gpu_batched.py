"""The batched step (make_step(batch_size=B)) against its numpy restatement
(oracle/batched.py): per-sample forward, loss and backward, the exact
batch-mean update and the mean reduction, two steps in a row, for MSE + sgd
and softmax cross-entropy + adam on a small layered net.
"""

from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _mlp(widths, density, rng):
    offsets = np.concatenate([[0], np.cumsum(widths)])
    frm, to = [], []
    for layer in range(len(widths) - 1):
        a = np.arange(offsets[layer], offsets[layer + 1])
        b = np.arange(offsets[layer + 1], offsets[layer + 2])
        s, d = np.meshgrid(a, b, indexing="ij")
        keep = rng.random(s.shape) < density
        frm.append(s[keep])
        to.append(d[keep])
    frm, to = np.concatenate(frm).astype(np.int32), np.concatenate(to).astype(np.int32)
    w = (rng.standard_normal(frm.size) * 0.3).astype(np.float32)
    return int(offsets[-1]), list(range(widths[0])), list(range(int(offsets[-2]), int(offsets[-1]))), frm, to, w


@pytest.mark.parametrize("loss_kind,opt_kind,hidden,out_act", [
    ("mse", "sgd", "tanh", None), ("softmax", "adam", "tanh", None),
    ("softmax", "sgd", "relu", "identity"),  # the sparse-MLP shape: ReLU hidden units, linear logits
])
def test_batched_step_matches_the_restatement(cuda, loss_kind, opt_kind, hidden, out_act):
    import torch

    import plastax_b200 as px
    from oracle.batched import batched_step

    rng = np.random.default_rng(51)
    n, inputs, outputs, frm, to, w = _mlp([24, 40, 32, 10], 0.4, rng)
    opt = px.optim.sgd(0.05) if opt_kind == "sgd" else px.optim.adam(0.01)

    class Net(px.Network):
        forward_pass = px.ForwardPass(hidden, output_activation=out_act)
        backward_pass = px.BackwardPass(hidden)
        loss = px.MSELoss() if loss_kind == "mse" else px.SoftmaxCrossEntropyLoss()
        update_conn = opt
        batch_reduction = px.MeanFloatFirstRest()
        propagation = px.Propagation.TOPOLOGICAL

    static, state = px.NetworkBuilder.from_edges(Net, n, frm, to, weights=w, input_ids=inputs, output_ids=outputs,
                                                 capacity_headroom=0.1, device=cuda)
    step = px.make_step(Net, static, batch_size=8, device=cuda)
    host = [{k: v.cpu().numpy().copy() for k, v in b.items()} for b in state.conns]
    level = state.units["level"].cpu().numpy()
    is_input = np.zeros(n, np.uint8)
    is_input[inputs] = 1
    for it in range(2):
        x = rng.standard_normal((8, len(inputs))).astype(np.float32)
        if loss_kind == "mse":
            t = rng.standard_normal((8, len(outputs))).astype(np.float32)
        else:
            t = np.eye(len(outputs), dtype=np.float32)[rng.integers(0, len(outputs), 8)]
        res = step(state, px.StepInputs(x, t))
        want = batched_step(host, level, is_input, inputs, outputs, x, t, fwd_act=hidden, bwd_act=hidden,
                            loss="mse" if loss_kind == "mse" else "softmax", opt=opt.oracle_args(),
                            out_act=out_act)
        np.testing.assert_allclose(float(res.loss.item()), float(want["loss"]), rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(state.units["activation"].cpu().numpy(), want["activation"], rtol=1e-5,
                                   atol=1e-6, err_msg=f"step {it} activation")
        np.testing.assert_allclose(state.units["grad_pre_act"].cpu().numpy(), want["grad"], rtol=1e-5, atol=1e-6,
                                   err_msg=f"step {it} grad")
        np.testing.assert_allclose(state.units["loss_grad"].cpu().numpy(), want["seed"], rtol=1e-5, atol=1e-6)
        for bi, b in enumerate(state.conns):
            np.testing.assert_allclose(b["weight"].cpu().numpy(), host[bi]["weight"], rtol=1e-5, atol=1e-6,
                                       err_msg=f"step {it} bucket {bi} weights")
            np.testing.assert_array_equal(b["dead"].cpu().numpy(), host[bi]["dead"])
    torch.cuda.synchronize()
