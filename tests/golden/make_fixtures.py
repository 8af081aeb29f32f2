"""Generate the golden fixtures the CPU tests check the oracle against.

Run in a container that has the reference checkout (it imports the reference's
pure-NumPy parity spec and reads its test file); the outputs are committed so the
tests never need the reference at run time:

    python tests/golden/make_fixtures.py /path/to/plastax

Writes, next to this script:
- rng_vectors.json: Philox-4x32-10 words, site seeds and the uniform /
  uniform_int draws of the spec (scripts/parity/reference.py:147-225) for
  seeded random inputs;
- growth_registry.json: every growth_v2 registry golden of the reference
  (scripts/parity/emit.py), with the exact inputs the spec's selection and
  claim stages received while emitting it (captured by wrapping
  `select_growth` / `commit_growth` / `retry_growth`) and their outputs;
- growth_random.json: seeded random selection + claim cases run through the
  spec (ties, vetoes, windows, every claim model);
- passes.json: the passes_v1 goldens (exact dyadic forward/backward values);
- claim_digests.json: the churn configurations and final-state sha256 digests
  the reference pins its claim to (tests/test_growth_claim.py);
- unit_lifecycle.json: the unit_lifecycle_v1 goldens (update, prune, add).
"""

from __future__ import annotations

import ast
import copy
import json
import math
import pathlib
import sys

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent


def _load_spec(ref_root: pathlib.Path):
    sys.path.insert(0, str(ref_root / "scripts" / "parity"))
    sys.path.insert(0, str(ref_root / "tests"))
    import emit  # noqa: E402
    import reference as ref  # noqa: E402

    return ref, emit


def _cands_json(cands):
    return [[int(c["src"]), int(c["dst"]), _f(c["score"]), int(c["index"])] for c in cands]


def _f(x):
    x = float(x)
    if math.isinf(x):
        return "inf" if x > 0 else "-inf"
    if math.isnan(x):
        return "nan"
    return x


def _units_json(units):
    return [[int(u["id"]), int(u["level"]), bool(u["pruned"])] for u in units]


def capture_registry(ref, emit):
    log: list[tuple[str, dict]] = []
    sel0, com0, ret0 = ref.select_growth, ref.commit_growth, ref.retry_growth

    def select_growth(units, edges, cands, **kw):
        before = copy.deepcopy(cands)
        out = sel0(units, edges, cands, **kw)
        ids = {id(c): i for i, c in enumerate(cands)}
        log.append(("select", {
            "units": _units_json(units), "edges": [[e["src"], e["dst"]] for e in edges],
            "cands": _cands_json(before), "kwargs": kw, "selected": [ids[id(c)] for c in out]}))
        return out

    def commit_growth(units, edges, selected, **kw):
        live_before = [[e["src"], e["dst"]] for e in edges]
        sel = [[int(c["src"]), int(c["dst"]), _f(c["score"])] for c in selected]
        out = com0(units, edges, selected, init=kw.pop("init"), field_defaults=kw.pop("field_defaults"), **kw)
        log.append(("commit", {"units": _units_json(units), "edges": live_before, "selected": sel,
                               "kwargs": {k: ({str(a): b for a, b in v.items()} if isinstance(v, dict) else v)
                                          for k, v in kw.items()},
                               "outcome": json.loads(json.dumps(out, default=_f))}))
        return out

    def retry_growth(units, edges, selected, attempt, **kw):
        sel = [[int(c["src"]), int(c["dst"]), _f(c["score"])] for c in selected]
        out = ret0(units, edges, selected, attempt, **kw)
        log.append(("retry", {"selected": sel, "attempt_committed": len(attempt["committed"]),
                              "free_per_level": {str(a): b for a, b in kw["free_per_level"].items()},
                              "outcome": json.loads(json.dumps(out, default=_f))}))
        return out

    ref.select_growth, ref.commit_growth, ref.retry_growth = select_growth, commit_growth, retry_growth
    docs_calls = []
    doc0 = emit._doc

    def doc(name, requires, comment, **payload):
        d = doc0(name, requires, comment, **payload)
        docs_calls.append((d, list(log)))
        log.clear()
        return d

    emit._doc = doc
    emit.build_all()
    ref.select_growth, ref.commit_growth, ref.retry_growth = sel0, com0, ret0
    emit._doc = doc0
    out = []
    for d, calls in docs_calls:
        if d.get("requires") != "growth_v2":
            continue
        out.append({"name": d["name"], "params": d["params"], "rules": d["rules"], "expect": d["expect"],
                    "retry": d.get("retry"), "calls": calls})
    passes = [d for d, _ in docs_calls if d.get("requires") == "passes_v1"]
    return out, passes


def random_growth(ref, rng, n_cases=60):
    cases = []
    for case in range(n_cases):
        n = int(rng.integers(4, 24))
        levels = np.sort(rng.integers(0, 4, n))
        units = [ref.make_unit(i, int(levels[i]), pruned=bool(rng.random() < 0.1)) for i in range(n)]
        edges = [ref.make_edge(int(rng.integers(0, n)), int(rng.integers(0, n))) for _ in range(int(rng.integers(0, 20)))]
        m = int(rng.integers(1, 80))
        cands = []
        for j in range(m):
            s = int(rng.integers(-1, n + 1))
            d = int(rng.integers(0, n))
            sc = float(np.float32(np.floor(rng.random() * 6) / 4))
            if rng.random() < 0.1:
                sc = float("-inf")
            cands.append({"src": s, "dst": d, "score": sc, "index": j})
        kw = dict(
            capacity=n, max_level_gap=int(rng.integers(0, 3)),
            direction=["any", "deeper", "same_or_deeper"][int(rng.integers(0, 3))],
            allow_self_loops=bool(rng.random() < 0.3), dedupe_live=bool(rng.random() < 0.4),
            dedupe_step=bool(rng.random() < 0.4),
            selection=["top_k", "threshold", "all"][int(rng.integers(0, 3))],
            max_new_per_level=int(rng.integers(1, 12)),
            max_new_per_step=None if rng.random() < 0.6 else int(rng.integers(1, 15)),
            threshold=0.5, level_cap_scope=["source_level", "step"][int(rng.integers(0, 2))])
        before = copy.deepcopy(cands)
        selected = ref.select_growth(units, edges, cands, **kw)
        ids = {id(c): i for i, c in enumerate(cands)}
        sel_idx = [ids[id(c)] for c in selected]
        model = ["free_slots", "pipeline", "topological"][int(rng.integers(0, 3))]
        lv = sorted({u["level"] for u in units})
        if model == "free_slots":
            ck = {"free_slots": int(rng.integers(0, 10))}
        elif model == "pipeline":
            ck = {"dead_per_level": {int(l): int(rng.integers(0, 4)) for l in lv}, "tail": int(rng.integers(0, 6))}
        else:
            ck = {"free_per_level": {int(l): int(rng.integers(0, 5)) for l in range(max(lv) + 1)}}
        edges2 = copy.deepcopy(edges)
        outcome = ref.commit_growth(units, edges2, selected, init=lambda s, d: {"weight": 1.0},
                                    field_defaults={"weight": 0.0}, **ck)
        cases.append({"units": _units_json(units), "edges": [[e["src"], e["dst"]] for e in edges],
                      "cands": _cands_json(before), "kwargs": {k: v for k, v in kw.items()}, "selected": sel_idx,
                      "claim": {k: ({str(a): b for a, b in v.items()} if isinstance(v, dict) else v)
                                for k, v in ck.items()},
                      "outcome": json.loads(json.dumps(outcome, default=_f))})
    return cases


def rng_vectors(ref, rng):
    seeds = [int(x) for x in rng.integers(0, 2**63, 200, dtype=np.uint64)]
    ctrs = [int(x) for x in rng.integers(0, 2**63, 200, dtype=np.uint64)]
    words = [ref.philox32(s, c) for s, c in zip(seeds, ctrs, strict=True)]
    sites = []
    for _ in range(40):
        ns, st, key = int(rng.integers(0, 2**40)), int(rng.integers(0, 2**31)), int(rng.integers(0, 2**32))
        sites.append([ns, st, key, ref.site_seed(ns, st, 1, key)])
    draws = []
    for n in (1, 2, 7, 1000, 65536, 1 << 20, (1 << 24) - 1):
        for j in range(8):
            seed = ref.site_seed(7, 3, 1, j)
            r = ref.SiteRng(seed, j)
            draws.append([seed, j, n, r.uniform_int(n), float(r.uniform())])
    return {"philox": [[s, c, w] for s, c, w in zip(seeds, ctrs, words, strict=True)], "sites": sites,
            "draws": draws}


def claim_digests(ref_root: pathlib.Path):
    src = (ref_root / "tests" / "test_growth_claim.py").read_text()
    tree = ast.parse(src)
    out = {}
    for node in tree.body:
        if isinstance(node, (ast.Assign, ast.AnnAssign)):
            target = node.targets[0] if isinstance(node, ast.Assign) else node.target
            name = getattr(target, "id", None)
            if name in ("_CONFIGS", "_GOLDEN", "_STEPS"):
                value = node.value
                if isinstance(value, ast.Dict) and name == "_CONFIGS":
                    cfgs = {}
                    for k, v in zip(value.keys, value.values, strict=True):
                        cfg = {}
                        for kw in v.keywords:
                            cfg[kw.arg] = ast.literal_eval(kw.value)
                        cfgs[ast.literal_eval(k)] = cfg
                    out["configs"] = cfgs
                else:
                    out[name.strip("_").lower()] = ast.literal_eval(value)
    return out


def unit_goldens(ref_root: pathlib.Path):
    """The unit_lifecycle_v1 goldens (tests/golden/unit_*.json of the
    reference): initial units and edges, the rules, the expected outcome."""
    out = []
    for path in sorted((ref_root / "tests" / "golden").glob("unit_*.json")):
        doc = json.loads(path.read_text())
        out.append({k: doc[k] for k in ("name", "capacity", "field_defaults", "max_levels", "rules", "initial_units",
                                        "initial_edges", "expect")})
    return out


def main() -> int:
    if len(sys.argv) < 2:
        raise SystemExit("usage: python tests/golden/make_fixtures.py <plastax checkout>")
    ref_root = pathlib.Path(sys.argv[1]).resolve()
    ref, emit = _load_spec(ref_root)
    rng = np.random.default_rng(2024)
    registry, passes = capture_registry(ref, emit)
    (HERE / "growth_registry.json").write_text(json.dumps(registry, indent=0, default=_f))
    (HERE / "growth_random.json").write_text(json.dumps(random_growth(ref, rng), indent=0, default=_f))
    (HERE / "rng_vectors.json").write_text(json.dumps(rng_vectors(ref, rng), indent=0))
    (HERE / "passes.json").write_text(json.dumps(passes, indent=0, default=_f))
    (HERE / "claim_digests.json").write_text(json.dumps(claim_digests(ref_root), indent=1))
    (HERE / "unit_lifecycle.json").write_text(json.dumps(unit_goldens(ref_root), indent=0))
    print(f"wrote {len(registry)} registry growth cases, {len(passes)} passes goldens")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
