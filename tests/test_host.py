"""Host-side logic and the C ABI's surface, without a GPU."""

from __future__ import annotations

import ctypes
import pathlib
import re

import numpy as np
import pytest
import torch

ROOT = pathlib.Path(__file__).resolve().parent.parent


def _header_functions() -> list[str]:
    text = (ROOT / "include" / "pxb.h").read_text()
    return re.findall(r"PXB_API\s+[\w\s\*]+?\b(pxb_\w+)\s*\(", text)


def test_library_exports_every_declared_entry_point():
    from plastax_b200 import _lib

    names = _header_functions()
    assert len(names) >= 30
    handle = ctypes.CDLL(str(_lib.LIB_PATH))
    for name in names:
        assert hasattr(handle, name), f"{name} declared in pxb.h but not exported"
    assert set(names) == set(_lib.exported_names()), "the binding declares exactly the header's functions"


def test_abi_version_and_errors_without_a_gpu():
    from plastax_b200 import _lib

    lib = _lib.lib()
    assert lib.pxb_abi_version() == 1
    # argument errors are caught on the host before any device work
    rc = lib.pxb_forward_accumulate(ctypes.c_int64(-1), None, None, None, None, None, 0, 0, None, None)
    assert rc == 1 and "negative capacity" in _lib.last_error()
    rc = lib.pxb_total_order_noalloc(ctypes.c_int64((1 << 18) + 1), None, None, None, 10, None, None)
    assert rc == 1 and "exceeds the maximum" in _lib.last_error()
    with pytest.raises(_lib.PxbError, match="unknown monoid"):
        _lib.call("pxb_forward_accumulate", ctypes.c_int64(4), ctypes.c_void_p(16), ctypes.c_void_p(16),
                  ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.c_void_p(16), 4, 7, ctypes.c_void_p(16), None)


def test_newer_entry_points_reject_bad_arguments_on_the_host():
    """The grid, unit-lifecycle, lowest-prune, loop and UPGD entry points
    check their arguments before any device work (no GPU needed)."""
    from plastax_b200 import _lib

    lib = _lib.lib()
    p = ctypes.c_void_p(16)

    def err(rc, text):
        assert rc != 0 and text in _lib.last_error(), (rc, _lib.last_error())

    score = _lib.PairScore(_lib.PAIR_MODULAR, None, None, 3, 5, 17, 8, 0.125)
    err(lib.pxb_propose_grid(1 << 20, 2, 1 << 15, 1 << 15, None, None, 0, ctypes.byref(score), p, None, 1, 0, 0, 0,
                             p, p, p, None), "exceed the int32 candidate index")
    bad = _lib.PairScore(9, None, None, 0, 0, 1, 0, 1.0)
    err(lib.pxb_propose_grid(8, 1, 8, 8, None, None, 0, ctypes.byref(bad), p, None, 1, 0, 0, 0, p, p, p, None),
        "unknown or incomplete score form")
    pred = _lib.PairScore(_lib.PAIR_MODULAR_PREDICATE, None, None, 1, 1, 2, 0, 1.0)
    err(lib.pxb_unit_importance(8, ctypes.byref(pred), None, None, 0, 0, 1, 0, p, None), "importance form")
    err(lib.pxb_unit_update(8, 7, p, None, ctypes.c_float(1.0), ctypes.c_float(0.0), None, None), "unknown kind")
    err(lib.pxb_unit_quantile(8, p, None, None, ctypes.c_float(1.5), p, p, ctypes.c_size_t(1 << 20), None),
        "bad arguments")
    cols = _lib.UnitColumns()
    cols.count = 17
    err(lib.pxb_unit_prune(8, p, p, None, p, p, ctypes.byref(cols), None), "bad column list")
    spawn = _lib.UnitSpawn(5, 16, 0.5, 1, 10, None, None, 1.0)
    err(lib.pxb_unit_add(8, ctypes.byref(spawn), p, p, ctypes.byref(_lib.UnitColumns()), p, p, p, None),
        "unknown spawn kind")
    spawn = _lib.UnitSpawn(_lib.SPAWN_ARGMAX, 16, 0.5, 1, 0, None, None, 1.0)
    err(lib.pxb_unit_add(8, ctypes.byref(spawn), p, p, ctypes.byref(_lib.UnitColumns()), p, p, p, None),
        "max_level")
    err(lib.pxb_lowest_keys(ctypes.c_int64(1 << 30), p, p, ctypes.c_int64(1 << 30), p, p, None), "out of range")
    err(lib.pxb_loop_build(None, None, None), "NULL")
    err(lib.pxb_unit_apply(8, 0, 6 << 8, 0, p, None, None, None, None, 0, None, None, p, None),
        "unknown activation code")
    upgd = _lib.Optimizer(_lib.OPT["upgd"], 0.01, 0.9, 0.01, 1e-8, 0.0, None)
    err(lib.pxb_backward_update(ctypes.c_int64(0), None, None, None, None, None, None, 8, None, ctypes.byref(upgd),
                                p, None, p, None), "upgd needs")


@pytest.mark.parametrize("live,headroom,align,want", [
    (0, 0.0, None, 64), (1, 0.0, None, 64), (100, 0.0, None, 128), (128, 0.0, None, 128), (129, 0.0, None, 256),
    (1000, 0.1, None, 2048), (1000, 0.0, 256, 1024), (285_212_672, 0.01, 8192, 288_071_680), (10, 0.0, 7, 70)])
def test_capacity_policy(live, headroom, align, want):
    """src/plastax/topo.py:455-506: next power of two (>= 64), or the next
    multiple of `align` (>= 64) of live * (1 + headroom)."""
    from plastax_b200.topo import capacity_policy

    assert capacity_policy(live, headroom=headroom, align=align) == want


def test_capacity_policy_rejects_bad_knobs():
    from plastax_b200.topo import capacity_policy

    with pytest.raises(ValueError):
        capacity_policy(10, headroom=-0.1)
    with pytest.raises(ValueError):
        capacity_policy(10, align=0)


def test_initial_levels_longest_path_and_inputs():
    from plastax_b200.topo import initial_levels

    # 0 -> 2 -> 3, 1 -> 3, 0 -> 3 (skip): longest path puts 3 at level 2
    lv = initial_levels(4, np.array([0, 2, 1, 0]), np.array([2, 3, 3, 3]))
    assert lv.tolist() == [0, 0, 1, 2]
    # an edge into an input does not lift it
    lv = initial_levels(3, np.array([2, 0]), np.array([0, 1]), allow_cycles=True, input_ids=(0,))
    assert lv.tolist() == [0, 1, 0]
    with pytest.raises(ValueError, match="cycle"):
        initial_levels(2, np.array([0, 1]), np.array([1, 0]))
    # a reservoir cycle under PIPELINE: inputs 0, fed units 1, the rest keep the frontier's level
    lv = initial_levels(4, np.array([0, 1, 2, 3]), np.array([1, 2, 3, 1]), allow_cycles=True, input_ids=(0,))
    assert lv[0] == 0 and lv[1] == 1


def _small_net(prop, grow=False):
    import plastax_b200 as px

    class Net(px.Network):
        forward_pass = px.ForwardPass("tanh")
        propagation = prop
        add_conn = px.ProposeAddConn(proposals_per_proposer=1, max_new_per_level=4) if grow else None

    return Net


def test_builder_layout_source_major_padding_and_tail():
    import plastax_b200 as px

    rng = np.random.default_rng(0)
    n, e = 50, 400
    src = rng.integers(0, n, e)
    dst = rng.integers(0, n, e)
    w = rng.standard_normal(e).astype(np.float32)
    net = _small_net(px.Propagation.PIPELINE)
    static, state = px.NetworkBuilder.from_edges(net, n, src, dst, weights=w, input_ids=(0,), output_ids=(1,),
                                                 capacity_headroom=0.1, device="cpu")
    b = {k: v.numpy() for k, v in state.conns[0].items()}
    assert static.level_capacities == (512,)
    live = b["dead"] == 0
    assert live[:e].all() and not live[e:].any()
    key = b["from_id"][:e].astype(np.int64) * n + b["to_id"][:e]
    assert np.all(np.diff(key) >= 0)
    order = np.argsort(src.astype(np.int64) * n + dst, kind="stable")
    np.testing.assert_array_equal(b["weight"][:e], w[order])  # parallel edges keep insertion order
    assert int(state.tail_start.item()) == e
    assert (b["from_id"][e:] == 0).all() and (b["weight"][e:] == 0).all()


def test_builder_topological_buckets_and_deepest_bucket():
    import plastax_b200 as px

    src = np.array([0, 1, 2, 2, 3])
    dst = np.array([2, 2, 3, 4, 4])
    static, state = px.NetworkBuilder.from_edges(_small_net(px.Propagation.TOPOLOGICAL, grow=True), 5, src, dst,
                                                 input_ids=(0, 1), output_ids=(4,), device="cpu")
    # levels 0,0,1,2,3 -> buckets for source levels 0..2 plus the deepest (3)
    assert len(static.level_capacities) == 4 and static.deepest_grows
    froms = [b["from_id"][b["dead"] == 0].tolist() for b in state.conns]
    assert froms == [[0, 1], [2, 2], [3], []]


def test_builder_scheme_a_bands_concatenate_to_the_full_arena():
    import plastax_b200 as px

    rng = np.random.default_rng(1)
    n, e = 40, 1000
    src, dst = rng.integers(0, n, e), rng.integers(0, n, e)
    net = _small_net(px.Propagation.PIPELINE)
    _, full = px.NetworkBuilder.from_edges(net, n, src, dst, input_ids=(0,), output_ids=(), capacity_align=8,
                                           device="cpu")
    parts = []
    for r in range(4):
        st, s = px.NetworkBuilder.from_edges(net, n, src, dst, input_ids=(0,), output_ids=(), capacity_align=8,
                                             sharding=px.ShardSpec("conns", 4), shard_rank=r, device="cpu")
        assert st.shard_base(0) == r * st.local_capacity(0)
        parts.append(s.conns[0])
    for col in ("from_id", "to_id", "dead", "weight"):
        assert torch.equal(torch.cat([p[col] for p in parts]), full.conns[0][col])
    with pytest.raises(ValueError, match="multiple of num_shards"):
        px.NetworkBuilder.from_edges(net, n, src, dst, input_ids=(0,), output_ids=(), capacity_align=6,
                                     sharding=px.ShardSpec("conns", 4), device="cpu")


def test_traits_reject_forms_without_a_lowering():
    import plastax_b200 as px

    with pytest.raises(ValueError, match="unknown activation"):
        class Bad(px.Network):  # noqa: F841
            forward_pass = px.ForwardPass("softplus")
    with pytest.raises(NotImplementedError, match="prod"):
        class Bad2(px.Network):  # noqa: F841
            forward_pass = px.ForwardPass("tanh", px.monoid.prod)
    with pytest.raises(ValueError, match="unknown proposer"):
        class Bad3(px.Network):  # noqa: F841
            forward_pass = px.ForwardPass("tanh")
            add_conn = px.ProposeAddConn(proposals_per_proposer=1, max_new_per_level=1, proposer="shortlist")
    with pytest.raises(ValueError, match="threshold"):
        class Bad5(px.Network):  # noqa: F841
            forward_pass = px.ForwardPass("tanh")
            add_conn = px.ProposeAddConn(proposals_per_proposer=1, max_new_per_level=1, selection="threshold")
    with pytest.raises(NotImplementedError, match="prune_unit form"):
        class Bad4(px.Network):  # noqa: F841
            forward_pass = px.ForwardPass("tanh")
            prune_unit = object()


@pytest.mark.parametrize("kwargs,exc,match", [
    (dict(candidates="grid"), TypeError, "candidates"),
    (dict(candidates="shortlist", importance=("field", "activation")), TypeError, "shortlist_size"),
    (dict(candidates="shortlist", shortlist_size=4), TypeError, "importance"),
    (dict(candidates="shortlist", shortlist_size=True, importance=("field", "activation")), TypeError,
     "shortlist_size"),
    (dict(max_new_per_level=None), TypeError, "max_new_per_level"),
    (dict(selection="threshold"), TypeError, "threshold"),
    (dict(level_cap_scope="bucket"), TypeError, "level_cap_scope"),
    (dict(max_new_per_step=0), TypeError, "max_new_per_step"),
    (dict(direction="shallower"), TypeError, "direction"),
    (dict(dedupe_step=1), TypeError, "dedupe_step"),
    (dict(score=("cosine", "a", "b")), NotImplementedError, "score form"),
    (dict(score=("modular", 3, 5)), NotImplementedError, "score form"),
    (dict(candidates="shortlist", shortlist_size=4, importance=("random",)), NotImplementedError, "importance"),
])
def test_score_add_conn_validation(kwargs, exc, match):
    """ScoreAddConn's knob checks raise as the reference's
    (src/plastax/traits.py:1390-1520): TypeError for a bad knob, and
    NotImplementedError for a score form with no lowering."""
    import plastax_b200 as px

    base = dict(score=("modular", 3, 5, 17, 8, 0.125), max_new_per_level=4)
    base.update(kwargs)
    with pytest.raises(exc, match=match):
        class Bad(px.Network):  # noqa: F841
            forward_pass = px.ForwardPass("tanh")
            add_conn = px.ScoreAddConn(**base)


def test_score_add_conn_forms_and_predicate_adapter():
    import plastax_b200 as px

    with pytest.raises(ValueError, match="topological-only"):
        class Bad(px.Network):  # noqa: F841
            forward_pass = px.ForwardPass("tanh")
            propagation = px.Propagation.PIPELINE
            add_conn = px.ScoreAddConn(score=("modular", 3, 5, 17, 8, 0.125), max_new_per_level=2,
                                       candidates="shortlist_per_level", shortlist_size=2,
                                       importance=("modular", 7, 13, 0, 0.25))
    rule = px.predicate_add_conn(("modular_predicate", 1, 1, 2, 0))
    assert rule.selection == "all" and rule.dedupe_step and rule.max_new_per_level is None

    class Ok(px.Network):  # noqa: F841
        forward_pass = px.ForwardPass("tanh")
        add_conn = rule
    over = px.predicate_add_conn(("modular_predicate", 1, 1, 2, 0), selection="top_k", max_new_per_level=3,
                                 dedupe_step=False)
    assert over.selection == "top_k" and not over.dedupe_step


def test_make_step_rejects_unknown_knobs():
    import plastax_b200 as px

    net = _small_net(px.Propagation.PIPELINE)
    static, _ = px.NetworkBuilder.from_edges(net, 4, [0], [1], input_ids=(0,), output_ids=(), device="cpu")
    for kw in ({"layout": "dense"}, {"growth": "magic"}, {"fuse_prune": "maybe"}, {"batch_size": 0}):
        with pytest.raises(ValueError):
            px.make_step(net, static, device="cpu", **kw)


def test_optimizer_bundles_declare_their_columns():
    from plastax_b200 import optim

    assert [f.name for f in optim.adam(1e-3).state_fields] == ["opt/m", "opt/v", "opt/t"]
    assert [f.name for f in optim.momentum(0.1).state_fields] == ["opt/v"]
    assert optim.sgd(0.1).state_fields == ()
    assert optim.adamw(1e-3).weight_decay == 1e-4


def test_batched_step_rejects_what_it_cannot_run():
    """src/plastax/step.py:188-202: a batched step is for TOPOLOGICAL nets
    with a batch_reduction; the engine moves [N, B] rows as float4."""
    import plastax_b200 as px

    class Pipe(px.Network):
        forward_pass = px.ForwardPass("tanh")
        propagation = px.Propagation.PIPELINE
        batch_reduction = px.MeanFloatFirstRest()

    class NoReduce(px.Network):
        forward_pass = px.ForwardPass("tanh")
        propagation = px.Propagation.TOPOLOGICAL

    class Topo(px.Network):
        forward_pass = px.ForwardPass("tanh")
        propagation = px.Propagation.TOPOLOGICAL
        batch_reduction = px.MeanFloatFirstRest()

    for net in (Pipe, NoReduce):
        static, _ = px.NetworkBuilder.from_edges(net, 4, [0], [1], input_ids=(0,), output_ids=(1,), device="cpu")
        with pytest.raises(ValueError):
            px.make_step(net, static, batch_size=8, device="cpu")
    static, _ = px.NetworkBuilder.from_edges(Topo, 4, [0], [1], input_ids=(0,), output_ids=(1,), device="cpu")
    with pytest.raises(ValueError, match="multiple of 4"):
        px.make_step(Topo, static, batch_size=6, device="cpu")

    class Units(px.Network):
        forward_pass = px.ForwardPass("tanh")
        propagation = px.Propagation.TOPOLOGICAL
        batch_reduction = px.MeanFloatFirstRest()
        update_unit = px.AffineUnitUpdate("activation", 1.0, 0.125)

    static, _ = px.NetworkBuilder.from_edges(Units, 4, [0], [1], input_ids=(0,), output_ids=(1,), device="cpu")
    with pytest.raises(NotImplementedError, match="unit-lifecycle"):
        px.make_step(Units, static, batch_size=8, device="cpu")


def test_mean_float_first_rest_declares_every_column():
    import plastax_b200 as px

    r = px.MeanFloatFirstRest()
    assert r.reduction(px.ACTIVATION) == "mean"
    assert r.reduction(px.LEVEL) == "not_batched"
    assert r.reduction(px.PRUNED) == "not_batched"
    assert r.reduction(px.FieldSpec.int32("test/count")) == "first"


def test_driver_rejects_check_every_below_one():
    import plastax_b200 as px

    with pytest.raises(ValueError, match="check_every"):
        px.Driver(None, None, None, check_every=0, device="cpu")


def test_shortlist_coverage_reports():
    """src/plastax/phases.py:3540-3637: per bucket, the sources at its level,
    the destinations strictly deeper within the gap, and whether M reaches
    them; the recommendation is the widest bucket's destination count."""
    import plastax_b200 as px

    class Net(px.Network):
        forward_pass = px.ForwardPass("tanh")
        add_conn = px.ScoreAddConn(score=("modular", 3, 5, 17, 8, 0.125), max_new_per_level=2,
                                   candidates="shortlist_per_level", shortlist_size=3,
                                   importance=("modular", 7, 13, 0, 0.25))

    src = np.array([0, 0, 1, 2, 2, 3, 4])
    dst = np.array([2, 3, 3, 4, 5, 5, 6])
    static, state = px.NetworkBuilder.from_edges(Net, 7, src, dst, input_ids=(0, 1), output_ids=(6,), device="cpu")
    cov = px.shortlist_coverage(Net, static, state)
    lv = state.units["level"].numpy()
    assert len(cov) == len(static.level_capacities)
    for c in cov:
        assert c.source_units == int((lv == c.bucket).sum())
        assert c.destination_units == int(((lv > c.bucket) & (lv <= c.bucket + 1)).sum())
        assert c.covered == (3 >= c.destination_units)
    assert px.recommended_shortlist(Net, static, state) == max(c.destination_units for c in cov)

    class NoShort(px.Network):
        forward_pass = px.ForwardPass("tanh")
        add_conn = px.ScoreAddConn(score=("modular", 3, 5, 17, 8, 0.125), max_new_per_level=2)

    static2, state2 = px.NetworkBuilder.from_edges(NoShort, 7, src, dst, input_ids=(0, 1), output_ids=(6,),
                                                   device="cpu")
    assert px.shortlist_coverage(NoShort, static2, state2) == ()
    assert px.recommended_shortlist(NoShort, static2, state2) == 0
