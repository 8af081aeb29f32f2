"""The batched step restated in numpy (make_step(batch_size=B),
src/plastax/step.py:76-237).

TEST INFRASTRUCTURE ONLY (the checker; the engine never imports it).

Per sample: the topological forward (src/plastax/phases.py:972-1015), the
loss (MSE, scripts/parity/reference.py:338-352; softmax cross-entropy,
src/plastax/traits.py:205-250) and the backward (:1049-1104); then the exact
batch-mean connection update (:434-483, sgd / adam of src/plastax/optim) and
the MeanFloatFirstRest reduction of the unit columns (traits.py:811-838).
Products are float32; segment sums accumulate in double and round once, as
the oracle's streaming sums do.
"""

from __future__ import annotations

import numpy as np

F32 = np.float32


def act_fn(kind: str, x: np.ndarray) -> np.ndarray:
    x = x.astype(F32)
    if kind == "tanh":
        return np.tanh(x).astype(F32)
    if kind == "relu":
        return np.maximum(x, F32(0)).astype(F32)
    if kind == "sigmoid":
        return (F32(1) / (F32(1) + np.exp(-x))).astype(F32)
    return x


def act_prime(kind: str, a: np.ndarray) -> np.ndarray:
    if kind == "tanh":
        return (F32(1) - a * a).astype(F32)
    if kind == "relu":
        return (a > 0).astype(F32)
    if kind == "sigmoid":
        return (a * (F32(1) - a)).astype(F32)
    return np.ones_like(a, F32)


def _segment(idx: np.ndarray, vals: np.ndarray, n: int) -> np.ndarray:
    """Per-unit sums of [E, B] products, double accumulation, one rounding."""
    out = np.zeros((n, vals.shape[1]), np.float64)
    np.add.at(out, idx, vals.astype(np.float64))
    return out.astype(F32)


def batched_step(buckets: list[dict], level: np.ndarray, is_input: np.ndarray, input_ids, output_ids,
                 x: np.ndarray, t: np.ndarray, *, fwd_act: str, bwd_act: str, loss: str, opt: dict,
                 out_act: str | None = None) -> dict:
    """One batched step; `buckets` are updated in place. Returns the batch
    loss and the reduced activation / grad / seed columns. `out_act` is the
    output units' activation (and derivative) when it differs."""
    n = level.size
    is_out = np.zeros(n, bool)
    if out_act is not None:
        is_out[np.asarray(output_ids)] = True

    def fwd(sel, v):
        return np.where(is_out[sel][:, None], act_fn(out_act or fwd_act, v), act_fn(fwd_act, v)).astype(F32)

    def prime(sel, a):
        return np.where(is_out[sel][:, None], act_prime(out_act or bwd_act, a), act_prime(bwd_act, a)).astype(F32)
    B = x.shape[0]
    L = len(buckets)
    act = np.zeros((n, B), F32)
    act[np.asarray(input_ids)] = x.T
    applyable = ~is_input.astype(bool)
    acc = np.zeros((n, B), F32)
    for lv, b in enumerate(buckets):
        live = b["dead"] == 0
        f, d, w = b["from_id"][live], b["to_id"][live], b["weight"][live]
        acc = (acc.astype(np.float64) + _segment(d, w[:, None] * act[f], n)).astype(F32)
        sel = (level == lv + 1) & applyable
        act[sel] = fwd(sel, acc[sel])
        acc[sel] = 0
    out = np.asarray(output_ids)
    seed = np.zeros((n, B), F32)
    losses = np.zeros(B, F32)
    a_out = act[out].T  # [B, k]
    if loss == "mse":
        d = (a_out - t).astype(F32)
        seed[out] = d.T
        for bb in range(B):
            tot = F32(0)
            for j in range(out.size):
                tot = F32(tot + F32(F32(0.5) * d[bb, j]) * d[bb, j])
            losses[bb] = tot
    else:
        m = a_out.max(axis=1, keepdims=True)
        z = (a_out - m).astype(F32)
        e = np.exp(z).astype(F32)
        s = np.zeros(B, F32)
        for j in range(out.size):
            s = (s + e[:, j]).astype(F32)
        seed[out] = (e / s[:, None] - t).astype(F32).T
        lse = np.log(s).astype(F32)
        for bb in range(B):
            tot = F32(0)
            for j in range(out.size):
                tot = F32(tot + F32(t[bb, j] * F32(lse[bb] - z[bb, j])))
            losses[bb] = tot
    tot = F32(0)
    for bb in range(B):
        tot = F32(tot + losses[bb])
    batch_loss = F32(tot / F32(B))
    grad = np.zeros((n, B), F32)
    sel = (level == L) & applyable
    grad[sel] = ((seed[sel]) * prime(sel, act[sel])).astype(F32)
    for lv in range(L - 1, 0, -1):
        b = buckets[lv]
        live = b["dead"] == 0
        f, d, w = b["from_id"][live], b["to_id"][live], b["weight"][live]
        acc = _segment(f, w[:, None] * grad[d], n)
        sel = (level == lv) & applyable
        grad[sel] = ((acc[sel] + seed[sel]) * prime(sel, act[sel])).astype(F32)
    for b in buckets:
        live = b["dead"] == 0
        f, d = b["from_id"][live], b["to_id"][live]
        g = ((grad[d] * act[f]).astype(np.float64).sum(axis=1) / B).astype(F32)
        w = b["weight"][live]
        if opt["kind"] == "sgd":
            w = (w - F32(opt["lr"]) * g).astype(F32)
        elif opt["kind"] == "adam":
            b1, b2, eps, lr = F32(opt["b1"]), F32(opt["b2"]), F32(opt["eps"]), F32(opt["lr"])
            tt = (b["opt/t"][live] + F32(1)).astype(F32)
            mm = (b1 * b["opt/m"][live] + (F32(1) - b1) * g).astype(F32)
            vv = (b2 * b["opt/v"][live] + (F32(1) - b2) * (g * g)).astype(F32)
            mh = (mm / (F32(1) - b1 ** tt)).astype(F32)
            vh = (vv / (F32(1) - b2 ** tt)).astype(F32)
            w = (w - lr * (mh / (np.sqrt(vh) + eps))).astype(F32)
            b["opt/m"][live], b["opt/v"][live], b["opt/t"][live] = mm, vv, tt
        b["weight"][live] = w
    mean = lambda a: (a.astype(np.float64).sum(axis=1) / B).astype(F32)  # noqa: E731
    return {"loss": batch_loss, "activation": mean(act), "grad": mean(grad), "seed": mean(seed)}


__all__ = ["act_fn", "act_prime", "batched_step"]
