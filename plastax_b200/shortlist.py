"""Shortlist coverage of a ScoreAddConn rule (src/plastax/phases.py:3540-3637).

A shortlisted rule draws a bucket's candidates from the top-M sources at its
level crossed with the top-M eligible destinations, so M bounds how many
distinct units a bucket can grow into. These host-side reports read the
built state's LEVEL column (runtime data, not static configuration).
"""

from __future__ import annotations

import dataclasses

import numpy as np

from plastax_b200.types import LEVEL


@dataclasses.dataclass(frozen=True)
class ShortlistCoverage:
    """How much of one bucket's destination population a shortlist can reach:
    the bucket index, the declared shortlist size M, the units at the bucket's
    source level, the units it may grow into (strictly deeper, within the
    rule's level gap) and whether M reaches all of them."""

    bucket: int
    candidate_units: int
    source_units: int
    destination_units: int
    covered: bool


def shortlist_coverage(net, static, state) -> tuple[ShortlistCoverage, ...]:
    """One report per bucket; empty when the net declares no shortlist (the
    exhaustive grid covers everything)."""
    ac = net.add_conn
    kind = str(getattr(ac, "candidates", "exhaustive"))
    size = getattr(ac, "shortlist_size", None) if kind != "exhaustive" else None
    if ac is None or size is None:
        return ()
    levels = np.asarray(state.units[LEVEL.name].cpu().numpy() if hasattr(state.units[LEVEL.name], "cpu")
                        else state.units[LEVEL.name])
    gap = int(getattr(ac, "max_level_gap", 1))
    out = []
    for bucket in range(len(static.level_capacities)):
        sources = int(np.sum(levels == bucket))
        destinations = int(np.sum((levels > bucket) & (levels <= bucket + gap)))
        out.append(ShortlistCoverage(bucket, int(size), sources, destinations, int(size) >= destinations))
    return tuple(out)


def recommended_shortlist(net, static, state) -> int:
    """The smallest shortlist that reaches every eligible destination in every
    bucket (a floor: the churn volume may ask for more), 0 without one."""
    return max((c.destination_units for c in shortlist_coverage(net, static, state)), default=0)


__all__ = ["ShortlistCoverage", "recommended_shortlist", "shortlist_coverage"]
