"""Arena state: static configuration + device-resident SOA columns
(mirrors src/plastax/state.py:22-313).

`NetworkStatic` is the hashable configuration a step is built against;
`NetworkState` holds the unit columns, one column dict per bucket (under
Scheme-A only this rank's capacity band), the user globals, and the
framework scalars. The scalars a step computes on the device (`needs_resort`,
`grown`, `overflow`, `tail_start`) stay device tensors so a step never waits
on the host; `step` is a host int, advanced once per step exactly as the
reference's counter is.
"""

from __future__ import annotations

import dataclasses
from typing import Any

import numpy as np
import torch

from plastax_b200.types import PRUNED, FieldSpec, Propagation, ShardSpec

Columns = dict[str, torch.Tensor]


def torch_dtype(spec: FieldSpec) -> torch.dtype:
    return {np.dtype(np.float32): torch.float32, np.dtype(np.int32): torch.int32,
            np.dtype(np.uint8): torch.uint8}[spec.dtype]


@dataclasses.dataclass(frozen=True)
class NetworkStatic:
    """Static network configuration (src/plastax/state.py:22-80).

    `level_capacities` are GLOBAL bucket capacities; under Scheme-A each rank
    holds `capacity // num_shards` slots per bucket, starting at
    `shard_rank * capacity // num_shards`.
    """

    num_units: int
    propagation: Propagation
    unit_fields: tuple[FieldSpec, ...]
    conn_fields: tuple[FieldSpec, ...]
    level_capacities: tuple[int, ...]
    input_ids: tuple[int, ...]
    output_ids: tuple[int, ...]
    sharding: ShardSpec | None = None
    shard_rank: int = 0
    capacity_headroom: float = 0.0
    capacity_align: int | None = None
    seed: int = 0
    deepest_grows: bool = False
    num_levels: int = 1  # max unit level + 1 (claim domains)

    @property
    def num_shards(self) -> int:
        return 1 if self.sharding is None else self.sharding.num_shards

    def local_capacity(self, bucket: int) -> int:
        return self.level_capacities[bucket] // self.num_shards

    def shard_base(self, bucket: int) -> int:
        return self.shard_rank * self.local_capacity(bucket)


@dataclasses.dataclass
class NetworkState:
    """Mutable arena state (src/plastax/state.py:83-145)."""

    units: Columns
    conns: tuple[Columns, ...]
    globals_: Any
    needs_resort: torch.Tensor
    step: int = 0
    grown: torch.Tensor | None = None
    overflow: torch.Tensor | None = None
    tail_start: torch.Tensor | None = None
    units_added: int = 0
    unit_overflow: bool = False


def filled_columns(specs: tuple[FieldSpec, ...], capacity: int, device: torch.device | str) -> Columns:
    return {s.name: torch.full((capacity,), s.default, dtype=torch_dtype(s), device=device) for s in specs}


def make_empty_state(static: NetworkStatic, globals_: Any, device: torch.device | str) -> NetworkState:
    """Arenas at capacity with every slot tombstoned (src/plastax/state.py:148-177)."""
    units = filled_columns(static.unit_fields, static.num_units, device)
    conns = tuple(filled_columns(static.conn_fields, static.local_capacity(b), device)
                  for b in range(len(static.level_capacities)))
    return NetworkState(units=units, conns=conns, globals_=globals_,
                        needs_resort=torch.zeros((), dtype=torch.bool, device=device),
                        grown=torch.zeros((), dtype=torch.int32, device=device),
                        overflow=torch.zeros((), dtype=torch.bool, device=device),
                        tail_start=torch.zeros(1, dtype=torch.int64, device=device))


def live_conn_count(state: NetworkState, level: int | None = None) -> int:
    """Live connections of this rank's band (src/plastax/state.py:180-198)."""
    buckets = state.conns if level is None else (state.conns[level],)
    return int(sum(int((b["dead"] == 0).sum().item()) for b in buckets))


def live_unit_mask(units: Columns) -> torch.Tensor | None:
    pruned = units.get(PRUNED.name)
    return None if pruned is None else pruned == 0


def grow_bucket(static: NetworkStatic, state: NetworkState, level: int) -> tuple[NetworkStatic, NetworkState]:
    """Pad one bucket with never-used slots (src/plastax/state.py:238-313).

    The new capacity is the sizing policy for live + 1 edges, at least twice
    the old (1.5x with an alignment). The padding takes every column's
    default (tombstoned), so in PIPELINE mode it extends the never-used tail
    and `tail_start` stays put. Returns a new (static, state); the step is
    rebuilt for the new static (make_step), as the reference retraces.
    """
    from plastax_b200.topo import capacity_policy

    if static.num_shards > 1:
        raise NotImplementedError("grow_bucket under Scheme-A has no engine lowering (the bands would move)")
    old = static.level_capacities[level]
    live = live_conn_count(state, level)
    policy = capacity_policy(live + 1, headroom=static.capacity_headroom, align=static.capacity_align)
    if static.capacity_align is None:
        floor = old * 2
    else:
        floor = capacity_policy(old + old // 2, align=static.capacity_align)
    new_cap = max(policy, floor)
    pad = new_cap - old
    cols = state.conns[level]
    dev = cols["dead"].device
    grown = {s.name: torch.cat([cols[s.name], torch.full((pad,), s.default, dtype=torch_dtype(s), device=dev)])
             for s in static.conn_fields}
    conns = tuple(grown if i == level else c for i, c in enumerate(state.conns))
    caps = tuple(new_cap if i == level else c for i, c in enumerate(static.level_capacities))
    new_static = dataclasses.replace(static, level_capacities=caps)
    new_state = dataclasses.replace(state, conns=conns)
    return new_static, new_state
