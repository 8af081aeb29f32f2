"""Initial levels and capacity sizing (mirrors src/plastax/topo.py:35-131, :455-506).

Levels decide bucket membership in TOPOLOGICAL mode and claim domains in
PIPELINE mode, so they must equal the reference's: longest-path levels from
the in-degree-0 units, computed here as a frontier relaxation (round r
settles the units whose last predecessor settled in round r - 1, and every
out-edge of the round's frontier lifts its destination to r + 1). Edges into
input units are ignored (inputs sit at level 0); with cycles allowed
(PIPELINE) the units on a cycle keep the level the frontier last assigned.
"""

from __future__ import annotations

import math

import torch


def initial_levels(num_units: int, src, dst, *, allow_cycles: bool = False,
                   input_ids: tuple[int, ...] = ()) -> torch.Tensor:
    """Per-unit int32 levels; `src`/`dst` are numpy arrays or torch tensors
    (the relaxation runs on their device)."""
    src_t = torch.as_tensor(src).to(torch.int64)
    dst_t = torch.as_tensor(dst).to(device=src_t.device, dtype=torch.int64)
    dev = src_t.device
    if input_ids and src_t.numel():
        inputs = torch.as_tensor(list(input_ids), dtype=torch.int64, device=dev)
        into_input = torch.isin(dst_t, inputs)
        if bool(into_input.any()):
            if not allow_cycles:
                initial_levels(num_units, src_t, dst_t)  # the cycle check sees every edge
            keep = ~into_input
            return initial_levels(num_units, src_t[keep], dst_t[keep], allow_cycles=allow_cycles)
    levels = torch.zeros(num_units, dtype=torch.int32, device=dev)
    if src_t.numel() == 0:
        return levels
    remaining = torch.bincount(dst_t, minlength=num_units)
    settled = remaining == 0
    frontier = settled.clone()
    done = int(settled.sum())
    r = 0
    while bool(frontier.any()):
        hit = dst_t[frontier[src_t]]
        levels[hit] = r + 1
        remaining -= torch.bincount(hit, minlength=num_units)
        reached = (remaining == 0) & ~settled
        settled |= reached
        frontier = reached
        done += int(reached.sum())
        r += 1
    if done != num_units and not allow_cycles:
        raise ValueError("initial_levels: edges do not form a DAG (cycle detected)")
    return levels


def capacity_policy(live: int, *, min_bucket: int = 64, headroom: float = 0.0, align: int | None = None) -> int:
    """Bucket capacity for `live` connections (src/plastax/topo.py:455-506):
    next power of two of live*(1+headroom) (at least min_bucket), or with
    `align` the next multiple of it."""
    if headroom < 0.0:
        raise ValueError(f"capacity_policy: headroom must be >= 0, got {headroom}")
    if align is not None and align < 1:
        raise ValueError(f"capacity_policy: align must be >= 1, got {align}")
    target = math.ceil(max(live, 0) * (1.0 + headroom))
    if align is not None:
        target = max(target, min_bucket)
        return -(-target // align) * align
    if live <= 0:
        return min_bucket
    return max(1 << (target - 1).bit_length(), min_bucket)
