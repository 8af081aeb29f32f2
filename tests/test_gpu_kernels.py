"""Parity of every libpxb kernel with the CPU oracle, through the C ABI.

Integer and structural outputs (tombstones, free counts, Philox words,
proposals, the total order, selections, claimed slots and every written
column) must match bit for bit. Float accumulations run in a different
order on the GPU (atomics / warp trees) than the oracle's slot-order sums,
so they are held to the north-star tolerance, |gpu - ref| <= 1e-6 + 1e-5 |ref|.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as orc
from tests._arena import random_bucket, to_device, to_host

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-5, 1e-6


def _k():
    from plastax_b200 import kernels

    return kernels


def _close(gpu, ref):
    np.testing.assert_allclose(gpu, ref, rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("cap,monoid", [(200_000, "sum"), (200_003, "sum"), (65_536, "max"), (65_537, "min")])
def test_forward_accumulate(cuda, cap, monoid):
    import torch

    k = _k()
    rng = np.random.default_rng(1)
    n = 3000
    b = random_bucket(rng, n, cap, int(cap * 0.8), dead_frac=0.05, weight_scale=0.1)
    act = rng.standard_normal(n).astype(np.float32)
    acc0 = (rng.standard_normal(n) * 0.1).astype(np.float32) if monoid == "sum" else np.full(
        n, -np.inf if monoid == "max" else np.inf, np.float32)
    ref = acc0.copy()
    orc.forward_accumulate(b, act, n, monoid, ref)
    db = to_device(b, cuda)
    acc = torch.from_numpy(acc0.copy()).to(cuda)
    k.forward_accumulate(db, torch.from_numpy(act).to(cuda), acc, monoid)
    got = acc.cpu().numpy()
    if monoid == "sum":
        _close(got, ref)
    else:
        np.testing.assert_array_equal(got, ref)


@pytest.mark.parametrize("cap,block_len", [(1 << 18, 1024), (1 << 18, 256), (100_004, 128), (99_999, 128)])
def test_forward_prune_fused(cuda, cap, block_len):
    import torch

    k = _k()
    rng = np.random.default_rng(2)
    n = 4096
    b = random_bucket(rng, n, cap, int(cap * 0.9), dead_frac=0.02, weight_scale=0.1)
    act = rng.standard_normal(n).astype(np.float32)
    thr = 0.01
    ref_acc = np.zeros(n, np.float32)
    orc.forward_accumulate(b, act, n, "sum", ref_acc)
    ref_b = {kk: v.copy() for kk, v in b.items()}
    ref_counts = orc.prune(ref_b, n, 1, thr, block_len=block_len)
    db = to_device(b, cuda)
    acc = torch.zeros(n, dtype=torch.float32, device=cuda)
    counts = torch.zeros((cap + block_len - 1) // block_len, dtype=torch.int32, device=cuda)
    k.forward_prune(db, torch.from_numpy(act).to(cuda), acc, threshold=thr, block_len=block_len, block_free=counts)
    _close(acc.cpu().numpy(), ref_acc)
    np.testing.assert_array_equal(db["dead"].cpu().numpy(), ref_b["dead"])
    np.testing.assert_array_equal(counts.cpu().numpy(), ref_counts)


def test_prune_per_destination_threshold(cuda):
    import torch

    k = _k()
    rng = np.random.default_rng(3)
    n, cap = 2000, 50_000
    b = random_bucket(rng, n, cap, 45_000, dead_frac=0.01)
    thr = np.abs(rng.standard_normal(n) * 0.05).astype(np.float32)
    ref_b = {kk: v.copy() for kk, v in b.items()}
    ref_counts = orc.prune(ref_b, n, 2, 0.0, thr, block_len=256)
    db = to_device(b, cuda)
    counts = torch.zeros((cap + 255) // 256, dtype=torch.int32, device=cuda)
    k.prune_conn(db, n, prune_kind=2, unit_threshold=torch.from_numpy(thr).to(cuda), block_len=256,
                 block_free=counts)
    np.testing.assert_array_equal(db["dead"].cpu().numpy(), ref_b["dead"])
    np.testing.assert_array_equal(counts.cpu().numpy(), ref_counts)


@pytest.mark.parametrize("monoid", ["sum", "max"])
def test_backward_accumulate(cuda, monoid):
    import torch

    k = _k()
    rng = np.random.default_rng(4)
    n, cap = 2500, 150_001
    b = random_bucket(rng, n, cap, 140_000, dead_frac=0.05, weight_scale=0.1)
    grad = (rng.standard_normal(n) * 0.5).astype(np.float32)
    init = 0.0 if monoid == "sum" else -np.inf
    ref = np.full(n, init, np.float32)
    orc.backward_accumulate(b, grad, n, monoid, ref)
    acc = torch.full((n,), init, dtype=torch.float32, device=cuda)
    k.backward_accumulate(to_device(b, cuda), torch.from_numpy(grad).to(cuda), acc, monoid)
    if monoid == "sum":
        _close(acc.cpu().numpy(), ref)
    else:
        np.testing.assert_array_equal(acc.cpu().numpy(), ref)


OPTS = {
    "sgd": dict(kind="sgd", lr=0.01),
    "momentum": dict(kind="momentum", lr=0.01, b1=0.9),
    "adam": dict(kind="adam", lr=1e-3, b1=0.9, b2=0.999, eps=1e-8),
    "adamw": dict(kind="adam", lr=1e-3, b1=0.9, b2=0.999, eps=1e-8, wd=1e-4),
    "rmsprop": dict(kind="rmsprop", lr=1e-3, b1=0.9, eps=1e-8),
}
OPT_COLS = {"sgd": (), "momentum": ("opt/v",), "adam": ("opt/m", "opt/v", "opt/t"),
            "adamw": ("opt/m", "opt/v", "opt/t"), "rmsprop": ("opt/v",)}


@pytest.mark.parametrize("name", sorted(OPTS))
@pytest.mark.parametrize("with_acc", [True, False])
def test_backward_update_fused(cuda, name, with_acc):
    import torch

    k = _k()
    rng = np.random.default_rng(5)
    n, cap = 3000, 120_000
    b = random_bucket(rng, n, cap, 110_000, dead_frac=0.03, opt_cols=OPT_COLS[name], weight_scale=0.1)
    grad = (rng.standard_normal(n) * 0.5).astype(np.float32)
    act = rng.standard_normal(n).astype(np.float32)
    ref_b = {kk: v.copy() for kk, v in b.items()}
    ref_acc = np.zeros(n, np.float32)
    if with_acc:
        orc.backward_accumulate(ref_b, grad, n, "sum", ref_acc)  # reads the old weights
    orc.update_conn(ref_b, grad, act, n, OPTS[name])
    db = to_device(b, cuda)
    acc = torch.zeros(n, dtype=torch.float32, device=cuda) if with_acc else None
    o = OPTS[name]
    opt = k.optimizer_struct(o["kind"], o["lr"], o.get("b1", 0.0), o.get("b2", 0.0), o.get("eps", 0.0),
                             o.get("wd", 0.0))
    k.backward_update(db, torch.from_numpy(grad).to(cuda), torch.from_numpy(act).to(cuda), acc, opt)
    hb = to_host(db)
    for col in ("weight", *OPT_COLS[name]):
        _close(hb[col], ref_b[col])
    if with_acc:
        _close(acc.cpu().numpy(), ref_acc)


@pytest.mark.parametrize("act_kind", ["tanh", "relu", "identity", "sigmoid"])
def test_unit_apply(cuda, act_kind):
    import torch

    k = _k()
    rng = np.random.default_rng(6)
    n = 10_000
    accv = rng.standard_normal(n).astype(np.float32)
    act = np.tanh(rng.standard_normal(n)).astype(np.float32)
    seed = rng.standard_normal(n).astype(np.float32)
    level = rng.integers(0, 4, n).astype(np.int32)
    is_input = (rng.random(n) < 0.1).astype(np.uint8)
    pruned = (rng.random(n) < 0.1).astype(np.uint8)
    for mode in (0, 1):
        ref_acc, ref_out = accv.copy(), act.copy()
        orc.unit_apply(n, mode, act_kind, "sum", ref_acc, act, seed if mode else None, level, 2, is_input, pruned,
                       ref_out)
        d_acc = torch.from_numpy(accv.copy()).to(cuda)
        d_out = torch.from_numpy(act.copy()).to(cuda)
        t = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
        k.unit_apply(d_acc, d_out, mode=mode, act_kind=act_kind, act=t(act), seed=t(seed) if mode else None,
                     level=t(level), target_level=2, is_input=t(is_input), pruned=t(pruned))
        _close(d_out.cpu().numpy(), ref_out)
        np.testing.assert_array_equal(d_acc.cpu().numpy(), ref_acc)


@pytest.mark.parametrize("batch", [256, 64, 12])
def test_batched_products_and_update(cuda, batch):
    import torch

    k = _k()
    rng = np.random.default_rng(7)
    n, cap = 1200, 40_000
    b = random_bucket(rng, n, cap, 36_000, dead_frac=0.02, weight_scale=0.1)
    x = rng.standard_normal((n, batch)).astype(np.float32)
    g = (rng.standard_normal((n, batch)) * 0.1).astype(np.float32)
    ref_f = np.zeros((n, batch), np.float32)
    orc.batched_product(b, x, n, False, ref_f)
    ref_bk = np.zeros((n, batch), np.float32)
    orc.batched_product(b, g, n, True, ref_bk)
    db = to_device(b, cuda)
    out = torch.zeros((n, batch), dtype=torch.float32, device=cuda)
    k.batched_forward(db, torch.from_numpy(x).to(cuda), out)
    _close(out.cpu().numpy(), ref_f)
    out.zero_()
    k.batched_backward(db, torch.from_numpy(g).to(cuda), out)
    _close(out.cpu().numpy(), ref_bk)
    ref_b = {kk: v.copy() for kk, v in b.items()}
    orc.batched_update(ref_b, g, x, n, OPTS["sgd"])
    k.batched_update(db, torch.from_numpy(g).to(cuda), torch.from_numpy(x).to(cuda),
                     k.optimizer_struct("sgd", 0.01))
    _close(db["weight"].cpu().numpy(), ref_b["weight"])


def test_philox_words(cuda):
    import torch

    k = _k()
    rng = np.random.default_rng(8)
    seed = rng.integers(0, 2**63, 100_000, dtype=np.uint64) * np.uint64(2) + rng.integers(0, 2, 100_000,
                                                                                           dtype=np.uint64)
    ctr = rng.integers(0, 2**63, 100_000, dtype=np.uint64)
    ref = orc.philox32_many(seed, ctr)
    got = k.philox32(torch.from_numpy(seed.view(np.int64)).to(cuda), torch.from_numpy(ctr.view(np.int64)).to(cuda))
    np.testing.assert_array_equal(got.cpu().numpy().view(np.uint32), ref)
    assert k.site_seed(7, 3, 1, 5) == orc.site_seed(7, 3, 1, 5)


@pytest.mark.parametrize("score_kind,proposals", [(0, 1), (1, 2), (0, 8), (2, 4)])
def test_propose_per_unit(cuda, score_kind, proposals):
    import torch

    k = _k()
    rng = np.random.default_rng(9)
    n = 20_000
    level = rng.integers(0, 3, n).astype(np.int32)
    pruned = (rng.random(n) < 0.05).astype(np.uint8)
    grad = rng.standard_normal(n).astype(np.float32)
    act = rng.standard_normal(n).astype(np.float32)
    for step in (0, 5, 123456):
        ref = orc.propose_per_unit(n, proposals, 0xC0FFEE, step, 3, n - 3, score_kind, level, grad=grad, act=act,
                                   pruned=pruned, max_level_gap=1, direction=0)
        t = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
        got = k.propose_per_unit(n, proposals, 0xC0FFEE, step, dst_lo=3, dst_n=n - 3, score_kind=score_kind,
                                 level=t(level), grad=t(grad), act=t(act), pruned=t(pruned), max_level_gap=1)
        for g_, r_ in zip(got, ref, strict=True):
            np.testing.assert_array_equal(g_.cpu().numpy(), r_)


def _adversarial_scores(rng, m):
    base = np.floor(rng.random(m) * 16).astype(np.float32) / 4  # many ties
    special = np.array([np.nan, np.inf, -np.inf, -0.0, 0.0, 1e-45, -1e-45, 3.4e38, -3.4e38], np.float32)
    idx = rng.integers(0, m, m // 10)
    base[idx] = special[rng.integers(0, special.size, idx.size)]
    return base


@pytest.mark.parametrize("m,id_bound", [(5000, 1000), (300_000, 65_536), (262_144, 1_048_592)])
def test_total_order(cuda, m, id_bound):
    import torch

    k = _k()
    rng = np.random.default_rng(10)
    score = _adversarial_scores(rng, m)
    src = rng.integers(0, min(id_bound, 50), m).astype(np.int32)  # dense ties on (src, dst)
    dst = rng.integers(0, id_bound, m).astype(np.int32)
    dst[: m // 3] = rng.integers(0, 20, m // 3)
    ref = orc.total_order(score, src, dst)
    t = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    got = k.total_order(t(score), t(src), t(dst), id_bound)
    np.testing.assert_array_equal(got.cpu().numpy(), ref)


@pytest.mark.parametrize("m,k", [(1_048_592, 268_435), (5000, 4999), (5000, 5000), (70_000, 1), (300_000, 150_000)])
def test_topk_unique_is_the_total_order_prefix(cuda, m, k):
    """Distinct sources (one proposal per unit): the radix-selected top k is
    exactly the first k of the oracle's total order."""
    import torch

    kern = _k()
    rng = np.random.default_rng(17)
    score = _adversarial_scores(rng, m)
    src = rng.permutation(m).astype(np.int32)
    dst = rng.integers(0, m, m).astype(np.int32)
    ref = orc.total_order(score, src, dst)[:k]
    t = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    got = kern.topk_unique(t(score), t(src), m, k)
    np.testing.assert_array_equal(got.cpu().numpy(), ref)


def test_select_step(cuda):
    import torch

    k = _k()
    rng = np.random.default_rng(11)
    m, n = 100_000, 5000
    src = rng.integers(0, n, m).astype(np.int32)
    score = _adversarial_scores(rng, m)
    level = rng.integers(0, 5, n).astype(np.int32)
    perm = orc.total_order(score, src, src)
    for kk in (1, 777, 50_000, 200_000):
        ref = orc.select_step(perm, src, level, kk)
        t = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
        got = k.select_step(t(perm), t(score), t(src), t(level), kk)
        np.testing.assert_array_equal(got.cpu().numpy(), ref)


def _claim_case(rng, cap, n, k, *, pipeline, dead_frac, tail_frac, levels=3):
    b = random_bucket(rng, n, cap, int(cap * (1 - tail_frac)), dead_frac=dead_frac)
    b["test/age"] = rng.integers(0, 100, cap).astype(np.int32)
    level = rng.integers(0, levels, n).astype(np.int32)
    src = rng.integers(-2, n + 2, k).astype(np.int32)  # a few out of range: clamped by the claim
    src = np.clip(src, 0, n - 1).astype(np.int32)
    dst = rng.integers(0, n, k).astype(np.int32)
    w = rng.standard_normal(k).astype(np.float32)
    grow = (rng.random(k) < 0.8).astype(np.uint8)
    age = rng.integers(0, 1000, k).astype(np.int32)
    if pipeline:  # claim order: levels ascending
        order = np.argsort(level[src], kind="stable")
        src, dst, w, grow, age = src[order], dst[order], w[order], grow[order], age[order]
    tail = int(cap * (1 - tail_frac))
    return b, level, tail, src, dst, w, grow, age


@pytest.mark.parametrize("level_major", [False, True])
@pytest.mark.parametrize("use_bitmap", [False, True])
@pytest.mark.parametrize("cap,k,dead_frac,tail_frac,max_new",
                         [(100_000, 5000, 0.02, 0.01, -1), (100_000, 20_000, 0.05, 0.02, -1),
                          (4096, 300, 0.1, 0.0, -1), (1 << 20, 30_000, 0.01, 0.005, 20_000), (777, 1000, 0.3, 0.1, -1)])
def test_claim_pipeline(cuda, cap, k, dead_frac, tail_frac, max_new, use_bitmap, level_major):
    """The list is level-major (non-growable entries interleaved); the
    level-major mode partitions where the other sorts, same result."""
    import torch

    kern = _k()
    rng = np.random.default_rng(12)
    n = 5000
    b, level, tail, src, dst, w, grow, age = _claim_case(rng, cap, n, k, pipeline=True, dead_frac=dead_frac,
                                                         tail_frac=tail_frac)
    ref_b = {kk: v.copy() for kk, v in b.items()}
    ref_counts, ref_over, ref_tail = orc.claim_pipeline(ref_b, level, tail, src, dst, w, grow, max_new=max_new,
                                                        extra={"test/age": age})
    db = to_device(b, cuda)
    t = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    d_level = t(level)
    d_tail = torch.tensor([tail], dtype=torch.int64, device=cuda)
    nl = int(level.max()) + 1
    ws = kern.ClaimWorkspace(cap, k, nl, cuda)
    bm = kern.free_bitmap_build(0, db, d_level, d_tail, nl) if use_bitmap else None
    mode = 0x100 if level_major else 0
    kern.claim_prepare(mode, db, d_level, d_tail, ws, free_bitmap=bm)
    kern.claim_commit(mode, db, d_level, d_tail, ws, t(src), t(dst), t(w), t(grow), max_new=max_new,
                      extra={"test/age": t(age)}, free_bitmap=bm)
    hb = to_host(db)
    if use_bitmap:  # the bitmaps stay equal to a rebuild from the new columns
        np.testing.assert_array_equal(bm.cpu().numpy(), kern.free_bitmap_build(0, db, d_level, d_tail, nl).cpu().numpy())
    for col in ref_b:
        np.testing.assert_array_equal(hb[col], ref_b[col], err_msg=col)
    np.testing.assert_array_equal(ws.counts.cpu().numpy(), ref_counts)
    np.testing.assert_array_equal(ws.overflowed.cpu().numpy()[:k], ref_over)
    assert int(d_tail.item()) == ref_tail


@pytest.mark.parametrize("use_bitmap", [False, True])
@pytest.mark.parametrize("cap,k,dead_frac", [(100_000, 5000, 0.03), (3000, 500, 0.1), (50_001, 10_000, 0.5)])
def test_claim_topological(cuda, cap, k, dead_frac, use_bitmap):
    import torch

    kern = _k()
    rng = np.random.default_rng(13)
    n = 3000
    b, level, _, src, dst, w, grow, age = _claim_case(rng, cap, n, k, pipeline=False, dead_frac=dead_frac,
                                                      tail_frac=0.05)
    ref_b = {kk: v.copy() for kk, v in b.items()}
    ref_counts, ref_over = orc.claim_topological(ref_b, level, src, dst, w, grow, extra={"test/age": age})
    db = to_device(b, cuda)
    t = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    ws = kern.ClaimWorkspace(cap, k, 1, cuda)
    bm = kern.free_bitmap_build(1, db, t(level), None, 1) if use_bitmap else None
    kern.claim_prepare(1, db, t(level), None, ws, free_bitmap=bm)
    kern.claim_commit(1, db, t(level), None, ws, t(src), t(dst), t(w), t(grow), extra={"test/age": t(age)},
                      free_bitmap=bm)
    hb = to_host(db)
    if use_bitmap:
        np.testing.assert_array_equal(bm.cpu().numpy(), kern.free_bitmap_build(1, db, t(level), None, 1).cpu().numpy())
    for col in ref_b:
        np.testing.assert_array_equal(hb[col], ref_b[col], err_msg=col)
    np.testing.assert_array_equal(ws.counts.cpu().numpy()[:2], ref_counts[:2])
    np.testing.assert_array_equal(ws.counts.cpu().numpy()[3], ref_counts[3])
    np.testing.assert_array_equal(ws.overflowed.cpu().numpy()[:k], ref_over)


@pytest.mark.parametrize("shards", [2, 4])
@pytest.mark.parametrize("pipeline,level_major", [(True, False), (True, True), (False, False)])
def test_claim_scheme_a_bands_match_one_device(cuda, shards, pipeline, level_major):
    """The Scheme-A claim over G capacity bands (each band claimed with the
    all-gathered per-domain counts of the bands before it) writes exactly the
    single-device claim (src/plastax/phases.py:2868-2874)."""
    import torch

    kern = _k()
    rng = np.random.default_rng(14)
    n, cap, k = 4000, 64_000, 6000
    b, level, tail, src, dst, w, grow, age = _claim_case(rng, cap, n, k, pipeline=pipeline, dead_frac=0.05,
                                                         tail_frac=0.03)
    mode = (0 if pipeline else 1) | (0x100 if level_major else 0)
    nl = int(level.max()) + 1 if pipeline else 1
    ref_b = {kk: v.copy() for kk, v in b.items()}
    if pipeline:
        orc.claim_pipeline(ref_b, level, tail, src, dst, w, grow)
    else:
        orc.claim_topological(ref_b, level, src, dst, w, grow)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)  # noqa: E731
    band = cap // shards
    parts = [{kk: t(v[g * band:(g + 1) * band]) for kk, v in b.items() if kk != "test/age"} for g in range(shards)]
    tails = [torch.tensor([tail], dtype=torch.int64, device=cuda) for _ in range(shards)]
    wss = [kern.ClaimWorkspace(band, k, nl, cuda) for _ in range(shards)]
    counts = []
    for g in range(shards):
        counts.append(kern.claim_prepare(mode, parts[g], t(level), tails[g], wss[g], shard_base=g * band).clone())
    allc = torch.stack(counts)  # the all-gather
    totals = allc.sum(0).to(torch.int32)
    for g in range(shards):
        before = allc[:g].sum(0).to(torch.int32) if g else torch.zeros(nl, dtype=torch.int32, device=cuda)
        kern.claim_commit(mode, parts[g], t(level), tails[g], wss[g], t(src), t(dst), t(w), t(grow),
                          shard_base=g * band, global_cap=cap, level_before=before.contiguous(),
                          level_totals=totals.contiguous())
    for col in ("from_id", "to_id", "dead", "weight"):
        got = np.concatenate([p[col].cpu().numpy() for p in parts])
        np.testing.assert_array_equal(got, ref_b[col], err_msg=col)
    for g in range(1, shards):
        assert int(tails[g].item()) == int(tails[0].item())


# ---------------------------------------------------------------------------
# destination-grouped mirror
# ---------------------------------------------------------------------------
def _mirror_multiset(m, b):
    """(slot, src, dst, weight) of every mirrored edge, sorted by slot."""
    word = m.word.cpu().numpy().view(np.uint32)
    live = word != 0xFFFFFFFF
    cb = m.chunk_bits
    ent = np.flatnonzero(live)
    grp = np.searchsorted(m.gbase.cpu().numpy(), ent, side="right") - 1
    src = (word[ent] >> cb).astype(np.int64)
    dst = (grp.astype(np.int64) << cb) | (word[ent] & ((1 << cb) - 1))
    out = [np.stack([m.slot.cpu().numpy()[ent].astype(np.int64), src, dst]).T]
    wts = [m.weight.cpu().numpy()[ent]]
    nov = int(min(m.ovf_count.item(), m.ovf_cap))
    if nov:
        os_ = m.ovf_src.cpu().numpy()[:nov]
        keep = os_ >= 0
        out.append(np.stack([m.ovf_slot.cpu().numpy()[:nov][keep], os_[keep],
                             m.ovf_dst.cpu().numpy()[:nov][keep]]).T.astype(np.int64))
        wts.append(m.ovf_weight.cpu().numpy()[:nov][keep])
    rows, w = np.concatenate(out), np.concatenate(wts)
    order = np.argsort(rows[:, 0], kind="stable")
    return rows[order], w[order]


def _canonical_multiset(hb):
    live = np.flatnonzero(hb["dead"] == 0)
    rows = np.stack([live, hb["from_id"][live], hb["to_id"][live]]).T.astype(np.int64)
    return rows, hb["weight"][live]


def _fixed_total(kern, acc, acc_fixed):
    """acc_fixed * 2^-31 + acc rounded once, through the unit apply."""
    import torch

    out = torch.empty_like(acc)
    kern.unit_apply(acc, out, mode=0, act_kind="identity", acc_fixed=acc_fixed)
    return out.cpu().numpy()


@pytest.mark.parametrize("n,cap,monoid", [(3000, 200_000, "sum"), (70_000, 400_000, "sum"), (5000, 100_000, "max"),
                                          (1 << 20, 1 << 20, "sum")])
def test_mirror_forward_prune(cuda, n, cap, monoid):
    import torch

    from plastax_b200.mirror import Mirror

    kern = _k()
    rng = np.random.default_rng(15)
    b = random_bucket(rng, n, cap, int(cap * 0.9), dead_frac=0.02, weight_scale=0.1)
    act = rng.standard_normal(n).astype(np.float32)
    level = rng.integers(0, 3, n).astype(np.int32)
    thr = 0.004
    init = 0.0 if monoid == "sum" else -np.inf
    ref_acc = np.full(n, init, np.float32)
    orc.forward_accumulate(b, act, n, monoid, ref_acc)
    ref_b = {kk: v.copy() for kk, v in b.items()}
    orc.prune(ref_b, n, 1, thr)
    db = to_device(b, cuda)
    t = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    d_level = t(level)
    tail = torch.tensor([cap], dtype=torch.int64, device=cuda)
    bm = kern.free_bitmap_build(0, db, d_level, tail, 3)
    m = Mirror(db, n)
    acc = torch.full((n,), init, dtype=torch.float32, device=cuda)
    acc_fixed = torch.zeros(n, dtype=torch.int64, device=cuda) if monoid == "sum" else None
    pruned = torch.zeros(1, dtype=torch.int32, device=cuda)
    kern.mirror_forward(m, t(act), acc, acc_fixed=acc_fixed, monoid=monoid, prune_kind=1, threshold=thr,
                        dead=db["dead"], free_bitmap=bm, bitmap_words=(cap + 31) // 32, bitmap_level=d_level,
                        pruned_count=pruned)
    if monoid == "sum":
        _close(_fixed_total(kern, acc, acc_fixed), ref_acc)
    else:
        np.testing.assert_array_equal(acc.cpu().numpy(), ref_acc)
    np.testing.assert_array_equal(db["dead"].cpu().numpy(), ref_b["dead"])
    assert int(pruned.item()) == int((ref_b["dead"] != b["dead"]).sum())
    np.testing.assert_array_equal(bm.cpu().numpy(), kern.free_bitmap_build(0, db, d_level, tail, 3).cpu().numpy())
    rows, w = _mirror_multiset(m, None)
    crows, cw = _canonical_multiset(to_host(db))
    np.testing.assert_array_equal(rows, crows)
    np.testing.assert_array_equal(w, cw)
    assert m.healthy()


@pytest.mark.parametrize("slack,ovf", [(0.05, 1 << 16), (0.0, 1 << 16)])
def test_mirror_tracks_claims(cuda, slack, ovf):
    """Prune + claim + insert for several steps: the mirror always holds
    exactly the canonical live edges (full groups spill to the overflow
    list, which the forward still sweeps)."""
    import torch

    from plastax_b200.mirror import Mirror

    kern = _k()
    rng = np.random.default_rng(16)
    n, cap, k = 4096, 300_000, 4000
    b = random_bucket(rng, n, cap, int(cap * 0.97), dead_frac=0.0, weight_scale=0.1)
    level = np.ones(n, np.int32)
    level[:16] = 0
    db = to_device(b, cuda)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)  # noqa: E731
    d_level = t(level)
    tail = torch.tensor([int(cap * 0.97)], dtype=torch.int64, device=cuda)
    bm = kern.free_bitmap_build(0, db, d_level, tail, 2)
    m = Mirror(db, n, slack=slack, min_slack=4 if slack == 0 else 64, ovf_cap=ovf)
    ws = kern.ClaimWorkspace(cap, k, 2, cuda)
    placed = torch.empty(k, dtype=torch.int32, device=cuda)
    hb = to_host(db)
    for step in range(5):
        act = rng.standard_normal(n).astype(np.float32)
        acc = torch.zeros(n, dtype=torch.float32, device=cuda)
        acc_fixed = torch.zeros(n, dtype=torch.int64, device=cuda)
        ref_acc = np.zeros(n, np.float32)
        orc.forward_accumulate(hb, act, n, "sum", ref_acc)
        kern.mirror_forward(m, t(act), acc, acc_fixed=acc_fixed, prune_kind=1, threshold=0.01, dead=db["dead"],
                            free_bitmap=bm, bitmap_words=(cap + 31) // 32, bitmap_level=d_level)
        _close(_fixed_total(kern, acc, acc_fixed), ref_acc)
        src = rng.integers(16, n, k).astype(np.int32)
        src = src[np.argsort(level[src], kind="stable")]
        dst = rng.integers(16, n, k).astype(np.int32)
        w = (rng.standard_normal(k) * 0.1).astype(np.float32)
        grow = np.ones(k, np.uint8)
        kern.claim_prepare(0, db, d_level, tail, ws, free_bitmap=bm)
        kern.claim_commit(0, db, d_level, tail, ws, t(src), t(dst), t(w), t(grow), free_bitmap=bm, placed=placed)
        kern.mirror_insert(m, t(src), t(dst), t(w), placed)
        hb = to_host(db)
        rows, mw = _mirror_multiset(m, None)
        crows, cw = _canonical_multiset(hb)
        np.testing.assert_array_equal(rows, crows, err_msg=f"step {step}")
        np.testing.assert_array_equal(mw, cw)
    assert m.healthy()


@pytest.mark.parametrize("frac", [28, 31])
def test_mirror_sum_is_exact_fixed_point(cuda, frac):
    """The mirror's sum equals the int64 sum of every float32 product rounded
    (half to even) to 2^-frac (in the accumulator's 2^-31 units), bit for bit,
    whatever the atomic order, with either of the sweep's fractions: large
    products (|p| >= 1), partials far beyond the 32-bit word's +-8 range (the
    carry into the high word), tiny products (rounded), one non-finite
    product (the float side), and two sweeps that must agree exactly."""
    import torch

    from plastax_b200.mirror import Mirror

    kern = _k()
    rng = np.random.default_rng(21)
    n, cap = 5000, 400_000
    b = random_bucket(rng, n, cap, cap - 1000, dead_frac=0.0, weight_scale=1.0)
    # skew the destinations so some units take thousands of edges
    hot = rng.random(cap) < 0.3
    b["to_id"][hot] = rng.integers(0, 8, int(hot.sum())).astype(np.int32)
    b["weight"][:] = (rng.standard_normal(cap) * rng.choice([1e-4, 0.05, 0.7, 40.0], cap)).astype(np.float32)
    act = (rng.standard_normal(n) * 2).astype(np.float32)
    b["weight"][7] = np.float32(3e7)  # a product beyond the fixed range goes to the float side
    act[b["from_id"][7]] = np.float32(2.0)
    db = to_device(b, cuda)
    t = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    m = Mirror(db, n, sum_frac_bits=frac)
    live = b["dead"] == 0
    p = (b["weight"][live] * act[b["from_id"][live]]).astype(np.float32)
    big = np.abs(p) >= np.float32(2.0 ** 20)
    units = np.rint(p[~big].astype(np.float64) * 2.0 ** frac).astype(np.int64) << (31 - frac)
    want_fixed = np.zeros(n, np.int64)
    np.add.at(want_fixed, b["to_id"][live][~big], units)
    got = []
    for _ in range(2):
        acc = torch.zeros(n, dtype=torch.float32, device=cuda)
        acc_fixed = torch.zeros(n, dtype=torch.int64, device=cuda)
        kern.mirror_forward(m, t(act), acc, acc_fixed=acc_fixed)
        np.testing.assert_array_equal(acc_fixed.cpu().numpy(), want_fixed)
        side = np.zeros(n, np.float32)
        np.add.at(side, b["to_id"][live][big], p[big])
        np.testing.assert_array_equal(acc.cpu().numpy(), side)
        got.append(_fixed_total(kern, acc, acc_fixed))
    assert int((np.abs(want_fixed) > (1 << (62 - frac))).sum()) > 0, "no unit exceeded the 32-bit word's range"
    np.testing.assert_array_equal(got[0], got[1])
    # one rounding of the exact sum, then the float side added as a float
    want = want_fixed.astype(np.float32) * np.float32(2.0 ** -31) + side
    np.testing.assert_array_equal(got[0], want)


def test_mirror_sum_of_thousands_of_small_products(cuda):
    """One destination takes 4,608 in-edges whose products all lie below 2^-7
    (so the fixed-point sum rounds every one of them), each 3/4 of a 2^-31 unit,
    so every rounding goes the same way (a quarter unit up); another takes
    4,096 random small products of both signs. The mirror of such a fan-in
    sums with 31 fractional bits, and both sums stay within 1e-5 relative /
    1e-6 absolute of the oracle's correctly rounded sum (the rounding error is
    at most in-degree * 2^-32: 9.5e-7 for 4,096 in-edges)."""
    import torch

    from plastax_b200.mirror import Mirror

    kern = _k()
    rng = np.random.default_rng(29)
    n, per = 4000, 4096
    cap = 2 * per + 512 + 20_000
    src = rng.integers(0, n, cap).astype(np.int32)
    dst = np.concatenate([np.full(per + 512, 5), np.full(per, 9), rng.integers(0, n, 20_000)]).astype(np.int32)
    act = np.ones(n, np.float32)
    w = np.empty(cap, np.float32)
    w[:per + 512] = np.float32(3 * 2.0 ** -34)  # 0.75 units of 2^-31: rounds up by 2^-33 every time
    w[per + 512:2 * per + 512] = (rng.standard_normal(per) * 2.0 ** -9).astype(np.float32)
    w[2 * per + 512:] = (rng.standard_normal(20_000) * 0.05).astype(np.float32)
    b = {"from_id": src, "to_id": dst, "dead": np.zeros(cap, np.uint8), "weight": w}
    db = to_device(b, cuda)
    t = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    m = Mirror(db, n)
    assert m.max_in_degree >= per and m.sum_frac_bits == 31  # the high fan-in takes the 31-bit sum
    acc = torch.zeros(n, dtype=torch.float32, device=cuda)
    acc_fixed = torch.zeros(n, dtype=torch.int64, device=cuda)
    kern.mirror_forward(m, t(act), acc, acc_fixed=acc_fixed)
    got = _fixed_total(kern, acc, acc_fixed)
    want = np.zeros(n, np.float32)
    orc.forward_accumulate(b, act, n, "sum", want)
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-6)
    assert abs(float(got[5]) - float(want[5])) > 0, "the first destination's products must be rounded"


@pytest.mark.parametrize("n,k,levels,kind,opts", [
    (5000, 1300, 2, 0, {}), (1 << 16, 20_000, 3, 0, {"direction": 1}), (70_000, 70_000, 2, 0, {}),
    (3000, 5000, 1, 1, {}), (40_000, 9000, 5, 1, {"pruned": True}), (1_048_592, 268_435, 2, 0, {"step_dev": True}),
    (20_000, 19_990, 8, 0, {"gap": 0}), (777, 1, 2, 0, {})])
def test_propose_select_unique_matches_the_staged_path(cuda, n, k, levels, kind, opts):
    """The fused selection gives exactly the rows of propose + top-k +
    level listing + gather: every candidate wins (k >= n), many invalid
    candidates (pruned units, a zero level gap), one winner, the full-size
    reservoir case with the device step counter."""
    import torch

    kern = _k()
    rng = np.random.default_rng(31)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)  # noqa: E731
    level = np.sort(rng.integers(0, levels, n)).astype(np.int32)
    pruned = (rng.random(n) < 0.2).astype(np.uint8) if opts.get("pruned") else None
    seed, step, dst_lo = 11, 37, 3
    dst_n = n - dst_lo
    gap = opts.get("gap", 1)
    direction = opts.get("direction", 0)
    step_dev = torch.tensor([step], dtype=torch.int32, device=cuda) if opts.get("step_dev") else None
    d_level = t(level)
    d_pruned = None if pruned is None else t(pruned)
    src, dst, score = kern.propose_per_unit(n, 1, seed, step, dst_lo=dst_lo, dst_n=dst_n, score_kind=kind,
                                            level=d_level, pruned=d_pruned, max_level_gap=gap, direction=direction,
                                            step_dev=step_dev)
    perm = kern.topk_unique(score, src, n, k)
    win = kern.select_step(perm, score, src, d_level, k, num_levels=levels)
    want = kern.gather_winners(win, min(k, n), k, src, dst, score, init_kind=2, init_a=0.05)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    got = kern.propose_select_unique(n, seed, step, dst_lo=dst_lo, dst_n=dst_n, score_kind=kind, level=d_level, k=k,
                                     num_levels=levels, init_kind=2, init_a=0.05, pruned=d_pruned, max_level_gap=gap,
                                     direction=direction, step_dev=step_dev, status=status)
    for name, a, b in zip(("src", "dst", "weight", "growable"), got, want, strict=True):
        np.testing.assert_array_equal(a.cpu().numpy(), b.cpu().numpy(), err_msg=name)
    assert int(status.item()) == 0


def test_propose_select_unique_matches_the_oracle(cuda):
    """The same rows from the oracle's proposals, total order and level-major
    step selection (q256 scores: many score ties, broken by source)."""
    import torch

    kern = _k()
    rng = np.random.default_rng(32)
    n, k, levels = 6000, 2500, 3
    level = rng.integers(0, levels, n).astype(np.int32)
    seed, step, dst_lo = 5, 9, 0
    src, dst, score = orc.propose_per_unit(n, 1, seed, step, dst_lo, n, 1, level)
    perm = orc.total_order(score, src, dst)
    win = orc.select_step(perm, src, level, k)
    got = kern.propose_select_unique(n, seed, step, dst_lo=dst_lo, dst_n=n, score_kind=1,
                                     level=torch.from_numpy(level).to(cuda), k=k, num_levels=levels, init_kind=0,
                                     init_a=0.5)
    np.testing.assert_array_equal(got[0].cpu().numpy(), src[win])
    np.testing.assert_array_equal(got[1].cpu().numpy(), dst[win])
    np.testing.assert_array_equal(got[3].cpu().numpy(), np.isfinite(score[win]).astype(np.uint8))


def _ref_dedupe(src, dst, score, live_pairs, dedupe_live, dedupe_step):
    """src/plastax/phases.py:4111-4205 restated: live pairs vetoed, then every
    copy of a pair after its first in the stable order of -score (NaN last)."""
    s = score.copy()
    if dedupe_live:
        hit = np.array([(int(a), int(b)) in live_pairs for a, b in zip(src, dst, strict=True)], bool)
        s[hit] = -np.inf
    if dedupe_step:
        seen, rep = set(), np.zeros(s.size, bool)
        for i in np.argsort(-s, kind="stable"):
            key = (int(src[i]), int(dst[i]))
            rep[i] = key in seen
            seen.add(key)
        s[rep] = -np.inf
    return s


@pytest.mark.parametrize("live,step", [(True, False), (False, True), (True, True)])
def test_dedupe_matches_the_reference_rule(cuda, live, step):
    import torch

    kern = _k()
    rng = np.random.default_rng(41)
    n_units, m, cap = 300, 60_000, 50_000
    src = rng.integers(0, n_units, m).astype(np.int32)
    dst = rng.integers(0, 40, m).astype(np.int32)  # narrow destinations: many repeated pairs
    score = (rng.integers(0, 50, m) / 8.0).astype(np.float32)  # ties
    score[rng.random(m) < 0.05] = -np.inf
    score[rng.random(m) < 0.01] = np.nan
    score[rng.random(m) < 0.02] = -0.0
    b = random_bucket(rng, n_units, cap, cap - 2000, dead_frac=0.1)
    b["to_id"][:] = np.clip(b["to_id"], 0, 39)
    live_pairs = {(int(a), int(c)) for a, c, d in zip(b["from_id"], b["to_id"], b["dead"], strict=True) if d == 0}
    want = _ref_dedupe(src, dst, score, live_pairs, live, step)
    db = to_device(b, cuda)
    t = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    d_score = t(score.copy())
    kern.dedupe(t(src), t(dst), d_score, buckets=[db] if live else [], step_repeats=step)
    got = d_score.cpu().numpy()
    np.testing.assert_array_equal(np.isnan(got), np.isnan(want))
    ok = ~np.isnan(want)
    np.testing.assert_array_equal(got[ok], want[ok])
    assert (got == -np.inf).sum() > (score == -np.inf).sum()  # something was vetoed
