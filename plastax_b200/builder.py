"""Vectorised construction (mirrors src/plastax/builder.py:177-661, from_edges).

The arena layout is part of the parity contract (the claim's slot indices and
every column digest depend on it), so it follows the reference's assembler:
longest-path levels; PIPELINE puts every edge in one bucket, TOPOLOGICAL
buckets edges by source level (plus a deepest-level bucket when the network
grows connections); each bucket is ordered source-major by one stable sort
of the packed key src * num_units + dst (parallel edges keep insertion
order); capacities come from `capacity_policy`; the padding is tombstoned at
the column defaults; PIPELINE's `tail_start` is the live count.

Edge columns may be numpy arrays (host sort) or CUDA tensors (device sort,
for arenas of hundreds of millions of edges). Under Scheme-A this process
keeps only its rank's contiguous band of every bucket.
"""

from __future__ import annotations

from collections.abc import Mapping, Sequence
from typing import Any

import numpy as np
import torch

from plastax_b200 import topo
from plastax_b200.state import NetworkState, NetworkStatic, filled_columns, torch_dtype
from plastax_b200.traits import Network
from plastax_b200.types import DEAD, FROM_ID, LEVEL, PRUNED, TO_ID, WEIGHT, Propagation, ShardSpec


class NetworkBuilder:
    """Construction entry points (src/plastax/builder.py:80-176)."""

    @classmethod
    def from_edges(cls, net: type[Network], num_units: int, from_ids, to_ids, *, weights=None,
                   input_ids: Sequence[int], output_ids: Sequence[int], globals_: Any = None,
                   extra_conn_columns: Mapping[str, Any] | None = None, capacity_headroom: float = 0.0,
                   capacity_align: int | None = None, sharding: ShardSpec | None = None, shard_rank: int = 0,
                   device: torch.device | str = "cuda") -> tuple[NetworkStatic, NetworkState]:
        dev = torch.device(device)
        src = torch.as_tensor(from_ids).to(device=dev, dtype=torch.int32)
        dst = torch.as_tensor(to_ids).to(device=dev, dtype=torch.int32)
        if src.ndim != 1 or dst.shape != src.shape:
            raise ValueError("from_edges: from_ids and to_ids must be 1-D arrays of equal length, got "
                             f"{tuple(src.shape)} and {tuple(dst.shape)}")
        capacity = net.unit_capacity
        num_slots = num_units if capacity is None else capacity
        if num_slots < num_units:
            raise ValueError(f"from_edges: unit_capacity {capacity} is below the {num_units} built units")
        for uid in (*input_ids, *output_ids):
            if not 0 <= uid < num_units:
                raise ValueError(f"from_edges: unit id {uid} out of range [0, {num_units})")
        if src.numel():
            lo = min(int(src.min()), int(dst.min()))
            hi = max(int(src.max()), int(dst.max()))
            if lo < 0 or hi >= num_units:
                raise ValueError(f"from_edges: an edge endpoint is out of range [0, {num_units})")
        effective = sharding if sharding is not None else net.sharding
        shards = 1 if effective is None else effective.num_shards
        if effective is not None and capacity_align is not None and capacity_align % shards:
            raise ValueError(f"from_edges: capacity_align {capacity_align} is not a multiple of num_shards {shards}")
        if capacity_headroom < 0:
            raise ValueError("from_edges: capacity_headroom must be >= 0")
        pipeline = net.propagation is Propagation.PIPELINE
        levels = topo.initial_levels(num_units, src, dst, allow_cycles=pipeline, input_ids=tuple(input_ids))

        conn_specs = net.conn_fields()
        extra = {k: torch.as_tensor(v).to(dev) for k, v in (extra_conn_columns or {}).items()}
        settable = {s.name for s in conn_specs} - {FROM_ID.name, TO_ID.name, DEAD.name}
        for name in extra:
            if name not in settable:
                raise ValueError(f"from_edges: unknown or non-settable conn column {name!r}")
        w = None if weights is None else torch.as_tensor(weights).to(device=dev, dtype=torch.float32)

        if pipeline:
            bucket_of = torch.zeros_like(src)
            num_buckets = 1
            deepest_grows = False
        else:
            bucket_of = levels[src.long()] if src.numel() else src
            max_level = int(levels.max()) if levels.numel() else 0
            deepest_grows = net.add_conn is not None
            num_buckets = max(max_level + (1 if deepest_grows else 0), 1)

        conns = []
        caps = []
        live_total = 0
        for b in range(num_buckets):
            idx = torch.nonzero(bucket_of == b).flatten() if num_buckets > 1 else torch.arange(
                src.numel(), device=dev)
            key = src[idx].to(torch.int64) * num_units + dst[idx].to(torch.int64)
            order = idx[torch.sort(key, stable=True).indices]
            del key
            live = int(order.numel())
            live_total += live
            cap = topo.capacity_policy(live, headroom=capacity_headroom, align=capacity_align)
            if cap % shards:
                raise ValueError(f"from_edges: bucket {b} capacity {cap} is not divisible by num_shards {shards}")
            band = cap // shards
            lo_pos, hi_pos = shard_rank * band, (shard_rank + 1) * band
            cols = filled_columns(conn_specs, band, dev)
            n_live = max(0, min(hi_pos, live) - lo_pos)
            if n_live > 0:
                sub = order[lo_pos:lo_pos + n_live]
                cols[FROM_ID.name][:n_live] = src[sub]
                cols[TO_ID.name][:n_live] = dst[sub]
                cols[DEAD.name][:n_live] = 0
                if w is not None:
                    cols[WEIGHT.name][:n_live] = w[sub]
                for name, vals in extra.items():
                    cols[name][:n_live] = vals[sub].to(cols[name].dtype)
            conns.append(cols)
            caps.append(cap)
            del order

        unit_specs = net.unit_fields()
        units = filled_columns(unit_specs, num_slots, dev)
        units[LEVEL.name][:num_units] = levels.to(torch.int32)
        units[LEVEL.name][num_units:] = 0
        if PRUNED.name in units:
            units[PRUNED.name][:] = 0
            units[PRUNED.name][num_units:] = 1
        num_levels = int(units[LEVEL.name].max()) + 1 if num_slots else 1
        static = NetworkStatic(
            num_units=num_slots, propagation=net.propagation, unit_fields=unit_specs, conn_fields=conn_specs,
            level_capacities=tuple(caps), input_ids=tuple(int(i) for i in input_ids),
            output_ids=tuple(int(i) for i in output_ids), sharding=effective, shard_rank=shard_rank,
            capacity_headroom=capacity_headroom, capacity_align=capacity_align, seed=net.seed,
            deepest_grows=deepest_grows, num_levels=num_levels)
        state = NetworkState(
            units=units, conns=tuple(conns), globals_=globals_,
            needs_resort=torch.zeros((), dtype=torch.bool, device=dev),
            grown=torch.zeros((), dtype=torch.int32, device=dev),
            overflow=torch.zeros((), dtype=torch.bool, device=dev),
            tail_start=torch.tensor([live_total if pipeline else 0], dtype=torch.int64, device=dev))
        return static, state


def host_columns(state: NetworkState) -> list[dict[str, np.ndarray]]:
    """Every bucket's columns copied to host numpy arrays."""
    return [{k: v.detach().cpu().numpy() for k, v in b.items()} for b in state.conns]


__all__ = ["NetworkBuilder", "host_columns", "torch_dtype"]
