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


# ---------------------------------------------------------------------------
# ScoreAddConn candidate grids (src/plastax/phases.py:3640-3746, :4690-4860;
# scripts/parity/reference.py:616-713)
# ---------------------------------------------------------------------------
def _floor_mod(x: np.ndarray, m: int) -> np.ndarray:
    return np.mod(x, m)  # numpy's mod is the floor mod, as Python's


def pair_score(form: tuple, src: np.ndarray, dst: np.ndarray, cols: dict) -> np.ndarray:
    """The lowered score forms, float32: |x[src]*y[dst]|, x[src]*y[dst],
    (((a*src + b*dst) mod m) - c) * scale, and the modular predicate (0 or
    -inf). `cols` maps unit field names to float32 columns."""
    kind = form[0]
    src = np.asarray(src, np.int64)
    dst = np.asarray(dst, np.int64)
    if kind == "grad_act":
        form = ("abs_product", "activation", cols["__grad_field__"])
        kind = "abs_product"
    if kind in ("abs_product", "product"):
        x = np.asarray(cols[form[1]], np.float32)[src]
        y = np.asarray(cols[form[2]], np.float32)[dst]
        p = (x * y).astype(np.float32)
        return np.abs(p) if kind == "abs_product" else p
    a, b, m = int(form[1]), int(form[2]), int(form[3])
    r = _floor_mod(a * src + b * dst, m)
    if kind == "modular":
        return ((r - int(form[4])).astype(np.float32) * np.float32(form[5])).astype(np.float32)
    return np.where(r == int(form[4]), np.float32(0.0), NEG_INF).astype(np.float32)


def importance(form: tuple, n: int, cols: dict) -> np.ndarray:
    """Per-unit importance, float32: |x[i]|, x[i] or (((a*i) mod m) - c) * scale."""
    if form[0] == "abs_field":
        return np.abs(np.asarray(cols[form[1]], np.float32)[:n])
    if form[0] == "field":
        return np.asarray(cols[form[1]], np.float32)[:n].copy()
    r = _floor_mod(int(form[1]) * np.arange(n, dtype=np.int64), int(form[2]))
    return ((r - int(form[3])).astype(np.float32) * np.float32(form[4])).astype(np.float32)


def ranked(imp: np.ndarray, eligible: np.ndarray) -> np.ndarray:
    """Unit ids ordered by (-importance, id) (lax.top_k's ranking: ties by
    ascending id), the ineligible ones ranking as -inf; a NaN importance
    ranks as -inf too."""
    key = np.where(eligible & ~np.isnan(imp), imp, NEG_INF).astype(np.float64)
    return np.lexsort((np.arange(imp.size), -key)).astype(np.int64)


def _in_window(level_src: np.ndarray, level_dst: np.ndarray, gap: int, direction: str) -> np.ndarray:
    ok = np.abs(level_dst - level_src) <= gap
    if direction == "deeper":
        ok &= level_dst > level_src
    elif direction == "same_or_deeper":
        ok &= level_dst >= level_src
    return ok


def score_grid_spec(units: list, *, capacity: int, candidates: str, shortlist_size: int | None, score: tuple,
                    importance_form: tuple | None, max_level_gap: int = 1, direction: str = "any",
                    cols: dict | None = None) -> list:
    """The reference spec's candidate list (live units only; index as the
    spec numbers it) from this module's ranking and score forms: the check
    that pins them to the registry's captured lists."""
    cols = cols or {}
    ids = np.array([u[0] for u in units if not u[2]], np.int64)
    lv = {u[0]: u[1] for u in units}
    n = capacity
    imp = importance(importance_form, n, cols) if importance_form is not None else None

    def rank(pool: np.ndarray) -> np.ndarray:
        elig = np.zeros(n, bool)
        elig[pool] = True
        return ranked(imp, elig)[: min(int(shortlist_size), pool.size)]

    out = []
    if candidates == "exhaustive":
        for s_ in ids:
            for d in ids:
                out.append([int(s_), int(d), float(pair_score(score, [s_], [d], cols)[0]), int(s_ * capacity + d)])
        return out
    if candidates == "shortlist":
        top = rank(ids)
        for i, s_ in enumerate(top):
            for k, d in enumerate(top):
                out.append([int(s_), int(d), float(pair_score(score, [s_], [d], cols)[0]), i * top.size + k])
        return out
    m = int(shortlist_size)
    for r, level in enumerate(sorted({lv[int(i)] for i in ids})):
        srcs = rank(np.array([i for i in ids if lv[int(i)] == level], np.int64))
        dsts = rank(np.array([i for i in ids if _in_window(np.int64(level), np.int64(lv[int(i)]), max_level_gap,
                                                             direction)], np.int64))
        for i, s_ in enumerate(srcs):
            for k, d in enumerate(dsts):
                out.append([int(s_), int(d), float(pair_score(score, [s_], [d], cols)[0]),
                            r * m * m + i * dsts.size + k])
    return out


def score_grid_engine(level: np.ndarray, pruned: np.ndarray | None, *, candidates: str, shortlist_size: int | None,
                      score: tuple, importance_form: tuple | None, cols: dict, num_buckets: int,
                      topological: bool, max_level_gap: int = 1, direction: str = "any",
                      allow_self_loops: bool = False) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """The engine's candidate columns for a ScoreAddConn step
    (src/plastax/phases.py:4690-4860): every unit slot takes part (a pruned
    one vetoed), a shortlist of M < N is the first M of the ranking (the
    ineligible units fill it at -inf), grids listed in order, row-major; the
    validity window applied (score -inf), grid g of the per-level shortlist
    admitting only sources at level g."""
    n = level.size
    live = np.ones(n, bool) if pruned is None else ~pruned.astype(bool)
    M = shortlist_size
    use_short = candidates in ("shortlist", "shortlist_per_level") and M is not None and 0 < M < n
    per_level = use_short and candidates == "shortlist_per_level"
    grid_of = None
    if not use_short:
        src = np.repeat(np.arange(n, dtype=np.int64), n)
        dst = np.tile(np.arange(n, dtype=np.int64), n)
    else:
        imp = importance(importance_form, n, cols)
        if not per_level:
            top = ranked(imp, live)[:M]
            src, dst = np.repeat(top, M), np.tile(top, M)
        else:
            ss, dd, gg = [], [], []
            for b in range(num_buckets):
                srow = ranked(imp, live & (level == b))[:M]
                dcol = ranked(imp, live & _in_window(np.int64(b), level.astype(np.int64), max_level_gap,
                                                     direction))[:M]
                ss.append(np.repeat(srow, M))
                dd.append(np.tile(dcol, M))
                gg.append(np.full(M * M, b, np.int64))
            src, dst, grid_of = np.concatenate(ss), np.concatenate(dd), np.concatenate(gg)
    sc = pair_score(score, src, dst, cols)
    ls, ld = level[src].astype(np.int64), level[dst].astype(np.int64)
    ok = live[src] & live[dst] & _in_window(ls, ld, max_level_gap, direction)
    if not allow_self_loops:
        ok &= src != dst
    if grid_of is not None:
        ok &= ls == grid_of
    if topological:
        ok &= ls < num_buckets
    sc = np.where(ok & np.isfinite(sc), sc, NEG_INF).astype(np.float32)
    return src.astype(np.int32), dst.astype(np.int32), sc


__all__ = ["claim", "importance", "pair_score", "ranked", "score_grid_engine", "score_grid_spec", "select"]
