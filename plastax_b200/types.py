"""SOA column specs and shared enums (mirrors src/plastax/_types.py:1-134).

A network is a struct of arrays: unit columns of length `num_units` and, per
bucket, connection columns of length `capacity`. The built-in columns keep
the reference's names, dtypes and defaults; the engine stores the reference's
bool columns as uint8 (0/1) so they are addressable bytes on the device.
"""

from __future__ import annotations

import dataclasses
import enum

import numpy as np


class Propagation(enum.Enum):
    """Sweep scheduling mode (src/plastax/_types.py:39-43)."""

    TOPOLOGICAL = "topological"
    PIPELINE = "pipeline"


@dataclasses.dataclass(frozen=True)
class ShardSpec:
    """Scheme-A connection sharding (src/plastax/_types.py:46-62): the
    capacity axis of every bucket is split into `num_shards` contiguous bands,
    one per rank; units and globals are replicated."""

    axis_name: str
    num_shards: int


@dataclasses.dataclass(frozen=True)
class FieldSpec:
    """One SOA column (src/plastax/_types.py:65-116)."""

    name: str
    dtype: np.dtype
    default: float | int | bool

    @staticmethod
    def float32(name: str, default: float = 0.0) -> FieldSpec:
        return FieldSpec(name, np.dtype(np.float32), float(default))

    @staticmethod
    def int32(name: str, default: int = 0) -> FieldSpec:
        return FieldSpec(name, np.dtype(np.int32), int(default))

    @staticmethod
    def boolean(name: str, default: bool = False) -> FieldSpec:
        # bool columns live as uint8 bytes on the device
        return FieldSpec(name, np.dtype(np.uint8), bool(default))


# built-in connection columns (src/plastax/_types.py:119-122)
FROM_ID = FieldSpec.int32("from_id")
TO_ID = FieldSpec.int32("to_id")
DEAD = FieldSpec.boolean("dead", default=True)
WEIGHT = FieldSpec.float32("weight")

# built-in unit columns (src/plastax/_types.py:126-132)
ACTIVATION = FieldSpec.float32("activation")
LEVEL = FieldSpec.int32("level")
PRUNED = FieldSpec.boolean("pruned", default=True)

BUILTIN_CONN_FIELDS = (FROM_ID, TO_ID, DEAD, WEIGHT)
