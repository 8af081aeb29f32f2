"""UPGD's per-edge update and its local utility scale, in numpy float32.

TEST INFRASTRUCTURE ONLY (the checker; the engine never imports it).

Restates examples/upgd.py:135-208 (UpgdUpdate.incoming) and the v1 scale of
:83-128 (UpgdForward: each destination's max over its incoming edges' stored
utilities), operation by operation in float32, and the edge hash of
examples/dst_sparse.py:77-85 in uint32 arithmetic.
"""

from __future__ import annotations

import numpy as np

F = np.float32


def hash01(a, b, c) -> np.ndarray:
    """Three int words -> float32 in [0, 1) (examples/dst_sparse.py:77-85)."""
    with np.errstate(over="ignore"):
        h = (np.asarray(a).astype(np.uint32) + np.uint32(0x9E3779B1)) * np.uint32(0x85EBCA77)
        h = (h ^ np.asarray(b).astype(np.uint32)) * np.uint32(0xC2B2AE3D)
        h = (h ^ np.asarray(c).astype(np.uint32)) * np.uint32(0x27D4EB2F)
        h = h ^ (h >> np.uint32(15))
        h = h * np.uint32(0x2C1B3C6D)
        h = h ^ (h >> np.uint32(13))
    return ((h >> np.uint32(8)).astype(F) / F(1 << 24)).astype(F)


def eta_local(buckets: list[dict], n: int, util_col: str, old_eta: np.ndarray, skip: np.ndarray) -> np.ndarray:
    """v1 scale: per destination the max of its incoming live edges' utility
    (-inf without one); units where `skip` is set keep their old value."""
    acc = np.full(n, -np.inf, F)
    for b in buckets:
        live = b["dead"] == 0
        np.maximum.at(acc, b["to_id"][live].astype(np.int64), b[util_col][live].astype(F))
    return np.where(skip, old_eta, acc).astype(F)


def update(b: dict, grad: np.ndarray, act: np.ndarray, eta: np.ndarray, *, lr: float, beta: float, sigma: float,
           eps: float, util_col: str = "upgd/util", t_col: str = "upgd/t") -> None:
    """UpgdUpdate.incoming on every live slot of the bucket, in place."""
    live = np.flatnonzero(b["dead"] == 0)
    src = b["from_id"][live].astype(np.int64)
    dst = b["to_id"][live].astype(np.int64)
    w = b["weight"][live].astype(F)
    beta_, lr_, sig_, eps_ = F(beta), F(lr), F(sigma), F(eps)
    with np.errstate(all="ignore"):
        gradient = (grad[dst].astype(F) * act[src].astype(F)).astype(F)
        inst = ((-gradient) * w).astype(F)
        step = (b[t_col][live].astype(F) + F(1.0)).astype(F)
        util = ((beta_ * b[util_col][live].astype(F)).astype(F) + ((F(1.0) - beta_) * inst).astype(F)).astype(F)
        corrected = (util / np.maximum((F(1.0) - np.power(beta_, step)).astype(F), eps_)).astype(F)
        scale = np.maximum(eta[dst].astype(F), eps_)
        x = (corrected / scale).astype(F)
        gated = (F(1.0) / (F(1.0) + np.exp(-x).astype(F))).astype(F)
        salt = step.astype(np.int32)
        u1 = np.maximum(hash01(src, dst, salt), F(1e-7))
        u2 = hash01(dst, src, salt)
        gauss = (np.sqrt((F(-2.0) * np.log(u1).astype(F)).astype(F)).astype(F)
                 * np.cos((F(2.0 * np.pi) * u2).astype(F)).astype(F)).astype(F)
        noise = (sig_ * gauss).astype(F)
        new_w = (w - ((lr_ * (gradient + noise).astype(F)).astype(F) * (F(1.0) - gated).astype(F)).astype(F)).astype(F)
    b["weight"][live] = new_w
    b[util_col][live] = util
    b[t_col][live] = step


__all__ = ["eta_local", "hash01", "update"]
