"""Seeded synthetic arenas for the parity tests (numpy on the host)."""

from __future__ import annotations

import numpy as np


def random_bucket(rng: np.random.Generator, n: int, cap: int, live: int, *, source_major: bool = True,
                  dead_frac: float = 0.0, opt_cols: tuple[str, ...] = (), weight_scale: float = 0.25) -> dict:
    """A bucket with `live` edges among `cap` slots, built like
    NetworkBuilder.from_edges (source-major, padding tombstoned), then a
    `dead_frac` share of the live slots tombstoned in place (their ids kept,
    as a prune leaves them)."""
    src = rng.integers(0, n, live).astype(np.int32)
    dst = rng.integers(0, n, live).astype(np.int32)
    if source_major:
        order = np.argsort(src.astype(np.int64) * n + dst, kind="stable")
        src, dst = src[order], dst[order]
    b = {
        "from_id": np.zeros(cap, np.int32),
        "to_id": np.zeros(cap, np.int32),
        "dead": np.ones(cap, np.uint8),
        "weight": np.zeros(cap, np.float32),
    }
    b["from_id"][:live] = src
    b["to_id"][:live] = dst
    b["dead"][:live] = 0
    b["weight"][:live] = (rng.standard_normal(live) * weight_scale).astype(np.float32)
    if dead_frac > 0:
        kill = rng.random(live) < dead_frac
        b["dead"][:live][kill] = 1
    for name in opt_cols:
        b[name] = np.zeros(cap, np.float32)
        if name != "opt/t":
            b[name][:live] = (rng.standard_normal(live) * 0.01).astype(np.float32)
        if name == "opt/v":
            b[name] = np.abs(b[name])
    return b


def to_device(b: dict, device) -> dict:
    import torch

    return {k: torch.from_numpy(np.ascontiguousarray(v)).to(device) for k, v in b.items()}


def to_host(b: dict) -> dict:
    return {k: v.cpu().numpy() for k, v in b.items()}
