"""The unit lifecycle phases in numpy (update_unit, prune_unit, add_unit).

TEST INFRASTRUCTURE ONLY (the checker; the engine never imports it).

Restates src/plastax/phases.py:1148-1193 (update_unit: every live unit,
against the pre-phase columns), :1245-1307 (prune_unit: live, non-I/O units
the predicate selects are marked PRUNED, their columns reset to the declared
defaults except LEVEL, every incident connection tombstoned) and :1310-1425
(add_unit: parents from the pre-phase state, ascending id, take the free
slots -- PRUNED at the start of the phase -- ascending; a child resets to
its defaults, goes live at level clamp(level(parent) + offset, 1,
max_levels - 1), and gets the init write; a parent past the last free slot is
dropped and raises unit_overflow), for the engine's lowered rule forms.
"""

from __future__ import annotations

import numpy as np

F = np.float32


def _name(f) -> str:
    return f if isinstance(f, str) else f.name


def update_unit(cols: dict, pruned: np.ndarray, rule) -> None:
    """AffineUnitUpdate / TraceUnitUpdate on every live unit, in place."""
    live = pruned == 0
    f = cols[_name(rule.field)]
    if type(rule).__name__ == "AffineUnitUpdate":
        new = ((f.astype(F) * F(rule.scale)).astype(F) + F(rule.shift)).astype(F)
    else:
        src = cols[_name(rule.source)].astype(F)
        if rule.absolute:
            src = np.abs(src)
        a = F(rule.rate)
        new = (((F(1.0) - a) * f.astype(F)).astype(F) + (a * src).astype(F)).astype(F)
    f[live] = new[live]


def quantile_threshold(values: np.ndarray, candidates: np.ndarray, q: float) -> np.float32:
    """The value at rank floor(q * m) of the m candidate values ascending
    (NaN excluded), -inf when m == 0."""
    v = np.sort(values[candidates & ~np.isnan(values)].astype(F))
    if v.size == 0:
        return F(-np.inf)
    r = min(int(np.floor(np.float64(F(q)) * v.size)), v.size - 1)
    return F(v[r])


def prune_unit(cols: dict, pruned: np.ndarray, exempt: np.ndarray, defaults: dict, buckets: list[dict],
               rule) -> np.ndarray:
    """FieldBelowPrune; returns the doomed mask. `defaults` maps every unit
    column but LEVEL and PRUNED to its default."""
    f = cols[_name(rule.field)].astype(F)
    if rule.quantile is not None:
        thr = quantile_threshold(f, (pruned == 0) & ~exempt, rule.quantile)
    else:
        thr = F(rule.threshold)
    doomed = (f < thr) & (pruned == 0) & ~exempt
    for name, default in defaults.items():
        cols[name][doomed] = default
    pruned[doomed] = 1
    for b in buckets:
        n = doomed.size
        fr, to = b["from_id"].astype(np.int64), b["to_id"].astype(np.int64)
        hit = ((fr >= 0) & (fr < n) & doomed[np.clip(fr, 0, n - 1)]) | ((to >= 0) & (to < n) & doomed[np.clip(to, 0, n - 1)])
        b["dead"][hit & (b["dead"] == 0)] = 1
    return doomed


def add_unit(cols: dict, pruned: np.ndarray, level: np.ndarray, defaults: dict, rule, max_levels: int
             ) -> tuple[list[int], bool]:
    """FieldSpawn / ArgmaxSpawn; returns (the children's ids, unit_overflow)."""
    n = pruned.size
    f = cols[_name(rule.field)].astype(F)
    live = pruned == 0
    if type(rule).__name__ == "ArgmaxSpawn":
        parents = np.zeros(n, bool)
        cand = np.flatnonzero(live & ~np.isnan(f))
        if cand.size:
            best = cand[np.argmax(f[cand])]  # argmax returns the first (lowest id) of equal maxima
            parents[best] = True
    else:
        parents = live & (f >= F(rule.threshold))
    free = np.flatnonzero(pruned != 0)
    par = np.flatnonzero(parents)
    placed = min(par.size, free.size)
    children = []
    init = rule.init
    src_vals = cols[_name(init[2])].astype(F).copy() if init is not None else None
    for k in range(placed):
        c, p = int(free[k]), int(par[k])
        for name, default in defaults.items():
            cols[name][c] = default
        level[c] = int(np.clip(int(level[p]) + int(rule.offset), 1, max_levels - 1))
        if init is not None:
            cols[_name(init[1])][c] = F(src_vals[p] * F(init[3]))
        pruned[c] = 0
        children.append(c)
    return children, bool(par.size > free.size)


__all__ = ["add_unit", "prune_unit", "quantile_threshold", "update_unit"]
