"""The CPU oracle against the reference's golden vectors (no GPU).

Fixtures come from tests/golden/make_fixtures.py, which imports the
reference's pure-NumPy parity spec and captures, for every growth_v2
registry golden, the exact candidate lists and claim inputs the spec
processed. The oracle must reproduce them bit for bit: Philox words and
site draws, the selection (validity, dedupes, total order, per-level or
step-scoped caps, max_new_per_step), every claim model's commits and flags,
and the passes_v1 forward/backward values (exact dyadic floats).
"""

from __future__ import annotations

import json
import pathlib

import numpy as np
import pytest

from oracle import growth as og
from oracle import oracle as orc

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"


def _load(name):
    return json.loads((GOLDEN / name).read_text())


def test_philox_words_match_the_spec():
    v = _load("rng_vectors.json")
    for seed, ctr, word in v["philox"]:
        assert orc.philox32(seed, ctr) == word
    words = orc.philox32_many(np.array([r[0] for r in v["philox"]], np.uint64),
                              np.array([r[1] for r in v["philox"]], np.uint64))
    assert [int(w) for w in words] == [r[2] for r in v["philox"]]


def test_site_seeds_and_draws_match_the_spec():
    v = _load("rng_vectors.json")
    for ns, st, key, want in v["sites"]:
        assert orc.site_seed(ns, st, 1, key) == want
    for seed, j, n, want_int, want_u in v["draws"]:
        r = orc.SiteRng(seed, j)
        assert r.uniform_int(n) == want_int
        assert float(r.uniform()) == want_u


REGISTRY = _load("growth_registry.json")


@pytest.mark.parametrize("case", REGISTRY, ids=[c["name"] for c in REGISTRY])
def test_registry_selection_and_claim(case):
    calls = case["calls"]
    if not calls:  # the trigger skipped the phase
        assert case["expect"]["grown"] == 0
        return
    last_commit = None
    for kind, call in calls:
        if kind == "select":
            got = og.select(call["units"], call["edges"], call["cands"], **call["kwargs"])
            assert got == call["selected"], f"{case['name']}: selection"
        elif kind == "commit":
            out = og.claim(call["units"], call["selected"], **call["kwargs"])
            want = call["outcome"]
            assert out["committed"] == [[c["src"], c["dst"]] for c in want["committed"]], case["name"]
            for key in ("grown", "conn_overflow", "needs_resort", "tail_used", "regrow_levels"):
                if key in want:
                    assert out[key] == want[key], f"{case['name']}: {key}"
            last_commit = want
    # the captured stages end in the golden's own expectation
    if case.get("retry") is None and last_commit is not None:
        assert last_commit == case["expect"]


# the reference's versioned conformance rules as the engine's lowered forms
# (scripts/parity/golden_rules.py: grid_score_v1, predicate_score_v1,
# importance_v1)
SCORE_RULES = {"grid_score_v1": ("modular", 3, 5, 17, 8, 0.125),
               "predicate_score_v1": ("modular_predicate", 1, 1, 2, 0)}
IMPORTANCE_RULES = {"importance_v1": ("modular", 7, 13, 0, 0.25)}
SCORE_CASES = [c for c in REGISTRY if c["name"].startswith("grow_score")]


@pytest.mark.parametrize("case", SCORE_CASES, ids=[c["name"] for c in SCORE_CASES])
def test_score_grids_reproduce_the_registry_candidates(case):
    """ScoreAddConn's exhaustive grid, shortlist and per-level shortlists:
    the oracle's ranking and lowered score forms give the spec's candidate
    lists (endpoints, scores, indices) exactly."""
    p, rules = case["params"], case["rules"]
    sel = case["calls"][0][1]
    got = og.score_grid_spec(sel["units"], capacity=p["capacity"], candidates=p["candidates"],
                             shortlist_size=p.get("shortlist_size"), score=SCORE_RULES[rules["score"]],
                             importance_form=IMPORTANCE_RULES.get(rules.get("importance")),
                             max_level_gap=p.get("max_level_gap", 1), direction=p.get("direction", "any"))
    want = [[c[0], c[1], (float("-inf") if c[2] == "-inf" else float(c[2])), c[3]] for c in sel["cands"]]
    assert got == want


def test_score_grid_engine_layout_holds_the_spec_candidates():
    """The engine's layout (every unit slot, shortlists padded with
    ineligible units, the window applied) lists the spec's valid candidates
    in the same relative order."""
    for case in SCORE_CASES:
        p, rules = case["params"], case["rules"]
        sel = case["calls"][0][1]
        n = p["capacity"]
        level = np.zeros(n, np.int32)
        pruned = np.ones(n, np.uint8)
        for uid, lv, pr in sel["units"]:
            level[uid], pruned[uid] = lv, pr
        nb = int(level[pruned == 0].max()) + 1
        src, dst, sc = og.score_grid_engine(level, pruned, candidates=p["candidates"],
                                            shortlist_size=p.get("shortlist_size"),
                                            score=SCORE_RULES[rules["score"]],
                                            importance_form=IMPORTANCE_RULES.get(rules.get("importance")), cols={},
                                            num_buckets=nb, topological=True, max_level_gap=p.get("max_level_gap", 1),
                                            direction=p.get("direction", "any"))
        got = [(int(a), int(b), float(c)) for a, b, c in zip(src, dst, sc, strict=True) if np.isfinite(c)]
        spec = [[c[0], c[1], c[2], c[3]] for c in sel["cands"]]
        spec_units = [[u[0], u[1], u[2]] for u in sel["units"]]
        level_of = {u[0]: u[1] for u in spec_units}
        want = []
        for s_, d, score, _ in spec:
            score = float("-inf") if score == "-inf" else float(score)
            ok = s_ != d and abs(level_of[d] - level_of[s_]) <= p.get("max_level_gap", 1)
            direction = p.get("direction", "any")
            if direction == "deeper":
                ok = ok and level_of[d] > level_of[s_]
            elif direction == "same_or_deeper":
                ok = ok and level_of[d] >= level_of[s_]
            if ok and np.isfinite(score):
                want.append((s_, d, score))
        assert got == want, case["name"]


RANDOM = _load("growth_random.json")


@pytest.mark.parametrize("i", range(len(RANDOM)))
def test_random_selection_and_claim(i):
    case = RANDOM[i]
    kw = dict(case["kwargs"])
    got = og.select(case["units"], case["edges"], case["cands"], **kw)
    assert got == case["selected"]
    sel = [[case["cands"][j][0], case["cands"][j][1], case["cands"][j][2]] for j in got]
    out = og.claim(case["units"], sel, **case["claim"])
    want = case["outcome"]
    assert out["committed"] == [[c["src"], c["dst"]] for c in want["committed"]]
    for key in ("grown", "conn_overflow", "needs_resort", "tail_used", "regrow_levels"):
        if key in want:
            assert out[key] == want[key], key


def test_per_unit_proposals_match_the_spec():
    """The registry's per-unit proposal lists (hash_propose_v1: dst =
    uniform_int(6) at sub 0, score = floor(u * 256) / 256 at sub 1)."""
    for case in REGISTRY:
        if case["params"].get("proposer") != "per_unit" or not case["calls"]:
            continue
        sel = case["calls"][0][1]
        units = sel["units"]
        n = len(units)
        P = case["params"]["proposals_per_proposer"]
        level = np.array([u[1] for u in units], np.int32)
        src, dst, score = orc.propose_per_unit(n, P, case["params"]["network_seed"], case["params"]["step"], 0, n, 1,
                                               level, max_level_gap=1 << 20, allow_self_loops=True)
        got = [[int(s), int(d), float(sc), int(i)] for i, (s, d, sc) in enumerate(zip(src, dst, score, strict=True))]
        assert got == [[c[0], c[1], float(c[2]), c[3]] for c in sel["cands"]], case["name"]


def _mlp(doc):
    """Units and the relu_mlp_v1 edges of a passes golden."""
    n_in, layers = doc["network"]["input_dim"], doc["network"]["layers"]
    n = n_in + sum(layers)
    edges = doc["initial_edges"]
    level = np.zeros(n, np.int32)
    off, lv = n_in, 1
    for width in layers:
        level[off:off + width] = lv
        off += width
        lv += 1
    b = {"from_id": np.array([e["src"] for e in edges], np.int32), "to_id": np.array([e["dst"] for e in edges], np.int32),
         "dead": np.zeros(len(edges), np.uint8),
         "weight": np.array([e["fields"]["weight"] for e in edges], np.float32)}
    return n, n_in, layers, level, b


@pytest.mark.parametrize("doc", _load("passes.json"), ids=lambda d: d["name"])
def test_passes_are_exact(doc):
    n, n_in, layers, level, b = _mlp(doc)
    is_input = np.zeros(n, np.uint8)
    is_input[:n_in] = 1
    act = np.zeros(n, np.float32)
    outputs = np.arange(n - layers[-1], n)
    for st in doc["steps"]:
        act[:n_in] = np.array(st["inputs"], np.float32)
        acc = np.zeros(n, np.float32)
        if doc["mode"] == "pipeline":
            orc.forward_accumulate(b, act, n, "sum", acc)
            orc.unit_apply(n, 0, "relu", "sum", acc, None, None, None, 0, is_input, None, act)
        else:
            for lv in range(1, len(layers) + 1):
                bl = {k: v[level[b["from_id"]] == lv - 1].copy() for k, v in b.items()}
                orc.forward_accumulate(bl, act, n, "sum", acc)
                orc.unit_apply(n, 0, "relu", "sum", acc, None, None, level, lv, is_input, None, act)
        assert act.tolist() == st["expect"]["activations"]
        if "grad_pre_act" in st["expect"]:
            seed = np.zeros(n, np.float32)
            t = np.array(st["targets"], np.float32)
            seed[outputs] = act[outputs] - t
            loss = np.float32(0)
            for d in seed[outputs]:
                loss = np.float32(loss + np.float32(0.5) * d * d)
            assert float(loss) == st["expect"]["loss"]
            grad = np.zeros(n, np.float32)
            acc = np.zeros(n, np.float32)
            top = len(layers)
            orc.unit_apply(n, 1, "relu", "sum", acc, act, seed, level, top, is_input, None, grad)
            for lv in range(top - 1, 0, -1):
                bl = {k: v[level[b["from_id"]] == lv].copy() for k, v in b.items()}
                orc.backward_accumulate(bl, grad, n, "sum", acc)
                orc.unit_apply(n, 1, "relu", "sum", acc, act, seed, level, lv, is_input, None, grad)
            assert [abs(g) for g in grad.tolist()] == [abs(g) for g in st["expect"]["grad_pre_act"]]


UNIT_GOLDENS = _load("unit_lifecycle.json")


def unit_rules(rules: dict):
    """The unit_lifecycle_v1 rules (scripts/parity/golden_rules.py:160-199) as
    the engine's lowered forms."""
    import plastax_b200 as px

    init = ("scale_parent", "activation", "activation", 0.5) if rules.get("init_unit") == "unit_child_init_v1" else None
    spawn = {"unit_spawn_v1": 1, "unit_spawn_deep_v1": 30000}
    return {
        "update_unit": px.AffineUnitUpdate("activation", 1.0, 0.125) if "update_unit" in rules else None,
        "prune_unit": px.FieldBelowPrune("activation", threshold=-0.5) if "prune_unit" in rules else None,
        "add_unit": (px.FieldSpawn("activation", 0.5, spawn[rules["add_unit"]], init) if "add_unit" in rules
                     else None),
    }


def unit_case_arrays(case):
    n = case["capacity"]
    act = np.zeros(n, np.float32)
    level = np.zeros(n, np.int32)
    pruned = np.ones(n, np.uint8)
    exempt = np.zeros(n, bool)
    for u in case["initial_units"]:
        i = u["id"]
        act[i], level[i], pruned[i] = u["fields"]["activation"], u["level"], u["pruned"]
        exempt[i] = u["is_input"] or u["is_output"]
    edges = case["initial_edges"]
    b = {"from_id": np.array([e["src"] for e in edges], np.int32), "to_id": np.array([e["dst"] for e in edges], np.int32),
         "dead": np.zeros(len(edges), np.uint8),
         "weight": np.array([e["fields"]["weight"] for e in edges], np.float32)}
    return act, level, pruned, exempt, b


def check_unit_outcome(case, act, level, pruned, live_edges, children=None, overflow=None):
    want = case["expect"]
    listed = set()
    for u in want["units"]:
        i = u["id"]
        listed.add(i)
        assert bool(pruned[i]) == u["pruned"], (case["name"], i)
        assert int(level[i]) == u["level"], (case["name"], i)
        assert float(act[i]) == u["fields"]["activation"], (case["name"], i)
    for i in range(case["capacity"]):
        if i not in listed:
            assert pruned[i], (case["name"], i)
    assert sorted(live_edges) == sorted((e["src"], e["dst"], e["fields"]["weight"]) for e in want["edges"])
    if children is not None and "children" in want:
        assert children == want["children"], case["name"]
    if overflow is not None and "unit_overflow" in want:
        assert overflow == want["unit_overflow"], case["name"]


@pytest.mark.parametrize("case", UNIT_GOLDENS, ids=[c["name"] for c in UNIT_GOLDENS])
def test_unit_lifecycle_goldens(case):
    """update_unit, prune_unit (exempt I/O, permanent, incident edges die) and
    add_unit (lowest free ids, same-step reuse, overflow, level clamp)."""
    from oracle import units as ou

    act, level, pruned, exempt, b = unit_case_arrays(case)
    cols = {"activation": act}
    defaults = {"activation": np.float32(case["field_defaults"]["activation"])}
    rules = unit_rules(case["rules"])
    children, overflow = None, None
    if rules["update_unit"] is not None:
        ou.update_unit(cols, pruned, rules["update_unit"])
    if rules["prune_unit"] is not None:
        ou.prune_unit(cols, pruned, exempt, defaults, [b], rules["prune_unit"])
    if rules["add_unit"] is not None:
        children, overflow = ou.add_unit(cols, pruned, level, defaults, rules["add_unit"], case["max_levels"])
    live = [(int(s), int(d), float(w)) for s, d, w, x in zip(b["from_id"], b["to_id"], b["weight"], b["dead"],
                                                                strict=True) if x == 0]
    check_unit_outcome(case, act, level, pruned, live, children, overflow)


def test_upgd_hash_matches_its_formula():
    """oracle/upgd.hash01 in uint32 numpy equals the three-word hash of
    examples/dst_sparse.py:77-85 evaluated with Python integers mod 2^32."""
    from oracle.upgd import hash01

    M = 0xFFFFFFFF

    def ref(a, b, c):
        h = ((a + 0x9E3779B1) & M) * 0x85EBCA77 & M
        h = ((h ^ b) * 0xC2B2AE3D) & M
        h = ((h ^ c) * 0x27D4EB2F) & M
        h ^= h >> 15
        h = (h * 0x2C1B3C6D) & M
        h ^= h >> 13
        return np.float32(h >> 8) / np.float32(1 << 24)

    rng = np.random.default_rng(5)
    a, b, c = (rng.integers(0, 1 << 31, 200) for _ in range(3))
    got = hash01(a, b, c)
    want = np.array([ref(int(x), int(y), int(z)) for x, y, z in zip(a, b, c, strict=True)], np.float32)
    np.testing.assert_array_equal(got, want)
    assert ((got >= 0) & (got < 1)).all()


def test_unit_quantile_threshold_edges():
    """The quantile rule: rank floor(q * m) of the m candidate values
    ascending, NaN excluded, -inf when nothing is a candidate."""
    from oracle.units import quantile_threshold

    v = np.array([5, 1, 4, np.nan, 2, 3], np.float32)
    cand = np.array([1, 1, 1, 1, 1, 0], bool)  # the last unit is exempt
    assert quantile_threshold(v, cand, 0.0) == 1.0
    assert quantile_threshold(v, cand, 0.5) == 4.0  # m = 4 (NaN out): sorted 1 2 4 5, rank 2
    assert quantile_threshold(v, cand, 1.0) == 5.0  # clamped to m - 1
    assert quantile_threshold(v, np.zeros(6, bool), 0.3) == np.float32(-np.inf)
