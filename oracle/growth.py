"""Growth selection and claim models on the oracle's primitives.

TEST INFRASTRUCTURE ONLY (the checker; the engine never imports it).

`select` restates the selection stages of the growth phase
(src/plastax/phases.py:4490-5132) over an explicit candidate list: the
validity window (:4061-4108), the live-edge and within-step dedupes (:4111-4205),
the total order (:4208-4321, via pxo_total_order), per-source-level or
step-scoped top_k / threshold / all (:4324-4487, :4838-4936), the level-major
listing and `max_new_per_step` (:5043-5058). The claim helpers realise each
claim model on an actual arena and run the oracle's C claims on it.
"""

from __future__ import annotations

import numpy as np

from oracle import oracle as orc

NEG_INF = np.float32(-np.inf)


def _score(x) -> np.float32:
    if isinstance(x, str):
        return np.float32({"inf": np.inf, "-inf": -np.inf, "nan": np.nan}[x])
    return np.float32(x)


def select(units: list, edges: list, cands: list, *, capacity: int, max_level_gap: int = 1,
           direction: str = "any", allow_self_loops: bool = False, dedupe_live: bool = False,
           dedupe_step: bool = False, selection: str = "top_k", max_new_per_level: int | None = None,
           max_new_per_step: int | None = None, threshold: float | None = None,
           level_cap_scope: str = "source_level", topological: bool = True) -> list[int]:
    """Indices (into `cands`) of the selected candidates, in commit order.

    units: [id, level, pruned] rows; edges: live [src, dst] pairs;
    cands: [src, dst, score, index] rows (listed in increasing index).
    """
    n = len(units)
    level = np.array([u[1] for u in units], np.int32)
    pruned = np.array([u[2] for u in units], bool)
    src = np.array([c[0] for c in cands], np.int64)
    dst = np.array([c[1] for c in cands], np.int64)
    score = np.array([_score(c[2]) for c in cands], np.float32)
    m = len(cands)
    ok = (src >= 0) & (src < capacity) & (dst >= 0) & (dst < capacity) & (src < n) & (dst < n)
    s_safe = np.where(ok, src, 0)
    d_safe = np.where(ok, dst, 0)
    ok &= ~pruned[s_safe] & ~pruned[d_safe]
    if not allow_self_loops:
        ok &= src != dst
    ls, ld = level[s_safe], level[d_safe]
    ok &= np.abs(ld - ls) <= max_level_gap
    if direction == "deeper":
        ok &= ld > ls
    elif direction == "same_or_deeper":
        ok &= ld >= ls
    score = np.where(ok & np.isfinite(score), score, NEG_INF).astype(np.float32)
    if dedupe_live:
        live = {(int(a), int(b)) for a, b in edges}
        dup = np.array([(int(a), int(b)) in live for a, b in zip(src, dst, strict=True)], bool)
        score = np.where(dup, NEG_INF, score).astype(np.float32)
    # total order on (-score, src, dst, list position); positions increase
    # with the candidate index, so they break ties the same way
    order = orc.total_order(score, src.astype(np.int32), dst.astype(np.int32))
    if dedupe_step:
        seen: set = set()
        for i in order:
            if score[i] == NEG_INF:
                continue
            key = (int(src[i]), int(dst[i]))
            if key in seen:
                score[i] = NEG_INF
            else:
                seen.add(key)
        order = orc.total_order(score, src.astype(np.int32), dst.astype(np.int32))
    finite = [int(i) for i in order if score[i] != NEG_INF]

    def take(pool: list[int]) -> list[int]:
        if selection == "top_k":
            return pool[:max_new_per_level]
        if selection == "threshold":
            return [i for i in pool if score[i] >= np.float32(threshold)][:max_new_per_level]
        return pool

    if level_cap_scope == "step" and selection != "all":
        winners = take(finite)
    else:
        by_level: dict[int, list[int]] = {}
        for i in finite:
            by_level.setdefault(int(ls[i]), []).append(i)
        winners = [i for lv in sorted(by_level) for i in take(by_level[lv])]
    winners = sorted(winners, key=lambda i: int(ls[i]))  # stable: levels ascending
    if max_new_per_step is not None:
        winners = winners[:max_new_per_step]
    del topological, m
    return winners


def claim(units: list, selected: list, *, free_slots: int | None = None, dead_per_level: dict | None = None,
          tail: int | None = None, free_per_level: dict | None = None) -> dict:
    """Run the oracle's C claim on an arena realising the claim model, and
    report the outcome as the spec's commit stage does
    (scripts/parity/reference.py:860-932): `selected` rows are [src, dst, score]."""
    level = np.array([u[1] for u in units], np.int32)
    n = len(units)
    src = np.array([s[0] for s in selected], np.int32)
    dst = np.array([s[1] for s in selected], np.int32)
    w = np.ones(len(selected), np.float32)
    grow = np.ones(len(selected), np.uint8)
    extra: dict = {}
    committed_mask = np.zeros(len(selected), bool)
    if free_per_level is None:
        if free_slots is not None:
            dead_per_level, tail = {}, free_slots
        # dead slots of each level (their former source sits at that level),
        # then the never-used tail
        owners = {lv: int(np.flatnonzero(level == lv)[0]) for lv in np.unique(level)}
        froms = []
        for lv, c in sorted((int(k), int(v)) for k, v in dead_per_level.items()):
            froms += [owners[lv]] * c
        used = len(froms)
        cap = used + int(tail)
        b = {"from_id": np.zeros(max(cap, 1), np.int32), "to_id": np.zeros(max(cap, 1), np.int32),
             "dead": np.ones(max(cap, 1), np.uint8), "weight": np.zeros(max(cap, 1), np.float32)}
        b["from_id"][:used] = froms
        if cap == 0:  # no slot at all: every growable candidate overflows
            b = {k: v[:0] for k, v in b.items()}
        counts, over, new_tail = orc.claim_pipeline(b, level, used, src, dst, w, grow)
        committed_mask = (grow == 1) & (over == 0)
        extra["tail_used"] = int(counts[2])
        if free_slots is not None:
            extra = {}
    else:
        left = {int(k): int(v) for k, v in free_per_level.items()}
        for lv in sorted(left):
            sel = np.flatnonzero(level[src] == lv) if len(selected) else np.zeros(0, np.int64)
            cap = left[lv]
            b = {"from_id": np.zeros(cap, np.int32), "to_id": np.zeros(cap, np.int32),
                 "dead": np.ones(cap, np.uint8), "weight": np.zeros(cap, np.float32)}
            counts, over = orc.claim_topological(b, level, src[sel], dst[sel], w[sel], grow[sel])
            committed_mask[sel] = over == 0
            left[lv] = cap - int(counts[0])
        extra["regrow_levels"] = sorted(lv for lv, f in left.items() if f == 0)
    committed = [i for i in range(len(selected)) if committed_mask[i]]
    needs_resort = any(level[dst[i]] <= level[src[i]] for i in committed)
    return {"committed": [[int(selected[i][0]), int(selected[i][1])] for i in committed],
            "grown": len(committed), "conn_overflow": len(committed) < len(selected),
            "needs_resort": bool(needs_resort), **extra}


__all__ = ["claim", "select"]
