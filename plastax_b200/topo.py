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


def resort(static, state):
    """Recompute levels, redistribute the live edges into buckets and compact
    each bucket (src/plastax/topo.py:303-452).

    Levels come from the live edges (longest path; a TOPOLOGICAL cycle
    raises). Each new bucket takes, in their old relative order, the live
    edges whose source now sits at its level (PIPELINE: one bucket of every
    live edge), stably ordered by source on the device (pxb_resort_order),
    at capacity max(policy(live), old capacity); PIPELINE's tail_start
    becomes the live count. Returns a new (static, state).
    """
    import dataclasses

    import torch

    from plastax_b200 import kernels as K
    from plastax_b200.state import torch_dtype
    from plastax_b200.types import LEVEL, Propagation

    if static.num_shards > 1:
        raise NotImplementedError("resort under Scheme-A has no engine lowering (it moves edges across bands)")
    n = static.num_units
    pipeline = static.propagation is Propagation.PIPELINE
    flat = {s.name: torch.cat([b[s.name] for b in state.conns]) for s in static.conn_fields}
    dev = flat["dead"].device
    live = flat["dead"] == 0
    lv_dev = initial_levels(n, flat["from_id"][live], flat["to_id"][live], allow_cycles=pipeline,
                            input_ids=tuple(static.input_ids)).to(device=dev, dtype=torch.int32)
    max_level = int(lv_dev.max().item()) if n else 0
    if pipeline:
        num_buckets = 1
        in_bucket = [live]
    else:
        num_buckets = max(max_level + (1 if static.deepest_grows else 0), 1)
        owner = lv_dev[flat["from_id"].clamp(0, n - 1).long()]
        in_bucket = [live & (owner == b) for b in range(num_buckets)]
    counts = [int(m.sum().item()) for m in in_bucket]
    old_caps = static.level_capacities
    caps = tuple(max(capacity_policy(c, headroom=static.capacity_headroom, align=static.capacity_align),
                     old_caps[i] if i < len(old_caps) else 0) for i, c in enumerate(counts))
    conns = []
    for b, mask in enumerate(in_bucket):
        idx = torch.nonzero(mask).flatten()
        cols = {s.name: torch.full((caps[b],), s.default, dtype=torch_dtype(s), device=dev)
                for s in static.conn_fields}
        for s in static.conn_fields:
            cols[s.name][: idx.numel()] = flat[s.name][idx]
        perm = K.resort_order(cols, n).long()
        conns.append({name: col[perm] for name, col in cols.items()})
    units = dict(state.units)
    units[LEVEL.name] = lv_dev
    new_static = dataclasses.replace(static, level_capacities=caps, num_levels=max_level + 1)
    tail = torch.tensor([counts[0] if pipeline else 0], dtype=torch.int64, device=dev)
    new_state = dataclasses.replace(state, units=units, conns=tuple(conns),
                                    needs_resort=torch.zeros((), dtype=torch.bool, device=dev), tail_start=tail)
    return new_static, new_state
