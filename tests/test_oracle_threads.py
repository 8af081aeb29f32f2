"""The oracle's multi-threaded proposal, total order and pipeline claim (the
CPU reference arm's) give exactly the sequential results."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as orc


@pytest.mark.parametrize("threads", [2, 3, 8])
def test_threaded_proposals_equal_the_sequential(threads):
    rng = np.random.default_rng(threads)
    n = 20_000
    level = rng.integers(0, 3, n).astype(np.int32)
    pruned = (rng.random(n) < 0.05).astype(np.uint8)
    kw = dict(pruned=pruned, max_level_gap=1)
    seq = orc.propose_per_unit(n, 2, 7, 11, 16, n - 16, 1, level, **kw)
    mt = orc.propose_per_unit(n, 2, 7, 11, 16, n - 16, 1, level, threads=threads, **kw)
    for a, b in zip(seq, mt, strict=True):
        np.testing.assert_array_equal(a, b)


@pytest.mark.parametrize("threads,n", [(2, 10_001), (3, 50_000), (8, 65_537), (8, 5)])
def test_threaded_total_order_equals_the_sequential(threads, n):
    rng = np.random.default_rng(n)
    score = (rng.integers(-4, 5, n) / 4).astype(np.float32)  # many exact ties
    score[rng.random(n) < 0.02] = np.nan
    score[rng.random(n) < 0.02] = -0.0
    score[rng.random(n) < 0.02] = -np.inf
    src = rng.integers(0, 50, n).astype(np.int32)
    dst = rng.integers(0, 50, n).astype(np.int32)
    np.testing.assert_array_equal(orc.total_order(score, src, dst, threads=threads), orc.total_order(score, src, dst))


@pytest.mark.parametrize("threads,cap,k", [(2, 40_000, 3_000), (5, 100_003, 30_000), (8, 20_000, 50_000)])
def test_threaded_pipeline_claim_equals_the_sequential(threads, cap, k):
    rng = np.random.default_rng(cap)
    n = 3000
    level = rng.integers(0, 3, n).astype(np.int32)
    used = int(cap * 0.9)

    def arena():
        r = np.random.default_rng(1)
        b = {"from_id": r.integers(0, n, cap).astype(np.int32), "to_id": r.integers(0, n, cap).astype(np.int32),
             "dead": (r.random(cap) < 0.2).astype(np.uint8), "weight": r.standard_normal(cap).astype(np.float32)}
        b["dead"][used:] = 1
        return b

    cs = rng.integers(0, n, k).astype(np.int32)
    cs = cs[np.argsort(level[cs], kind="stable")]  # level-major, as the step lists them
    cd = rng.integers(0, n, k).astype(np.int32)
    cw = rng.standard_normal(k).astype(np.float32)
    grow = (rng.random(k) < 0.9).astype(np.uint8)
    b1, b2 = arena(), arena()
    c1, o1, t1 = orc.claim_pipeline(b1, level, used, cs, cd, cw, grow)
    c2, o2, t2 = orc.claim_pipeline(b2, level, used, cs, cd, cw, grow, threads=threads)
    np.testing.assert_array_equal(c1, c2)
    np.testing.assert_array_equal(o1, o2)
    assert t1 == t2
    for col in b1:
        np.testing.assert_array_equal(b1[col], b2[col], err_msg=col)
