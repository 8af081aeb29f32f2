"""The reference's claim digests, reproduced on the CPU (no GPU).

The reference pins its growth claim with the sha256 of every connection
column of every bucket (plus needs_resort and the per-step overflow flags)
after 24 churn steps of five small layered TOPOLOGICAL networks
(tests/test_growth_claim.py of the reference): hashed prune, hashed global
proposals or a hashed score grid, live-edge / within-step dedupe, per-bucket
top-k in the total order, the topological claim, tight and unaligned
capacities, an extra written and an extra defaulted column. The digests and
configurations are committed in tests/golden/claim_digests.json.

Here the arena comes from plastax_b200's NetworkBuilder (its layout is part
of what the digest pins), the test's hash policies are restated in numpy, and
the selection and claim run on the oracle. Matching all five digests pins the
builder's slot layout, the total order, per-bucket selection and the claim's
slot choice to the reference's own outputs.
"""

from __future__ import annotations

import hashlib
import json
import pathlib

import numpy as np
import pytest

from oracle import oracle as orc

GOLD = json.loads((pathlib.Path(__file__).resolve().parent / "golden" / "claim_digests.json").read_text())
U32 = np.uint32


def _mix(x):
    x = np.asarray(x).astype(U32)
    x = x ^ (x >> U32(16))
    x = (x * U32(0x7FEB352D)).astype(U32)
    x = x ^ (x >> U32(15))
    x = (x * U32(0x846CA68B)).astype(U32)
    return x ^ (x >> U32(16))


def _h(*parts):
    acc = U32(0x9E3779B9)
    for p in parts:
        acc = _mix(acc ^ np.asarray(p).astype(U32))
    return acc


def _build(cfg):
    """The reference test's layered net, built by plastax_b200's builder."""
    import plastax_b200 as px

    rng = np.random.default_rng(0)
    widths = cfg["widths"]
    offsets = np.concatenate([[0], np.cumsum(widths)])
    num_units = int(offsets[-1])
    frm, to = [], []
    for layer in range(len(widths) - 1):
        a = np.arange(offsets[layer], offsets[layer + 1])
        b = np.arange(offsets[layer + 1], offsets[layer + 2])
        src, dst = np.meshgrid(a, b, indexing="ij")
        keep = rng.random(src.shape) < cfg["density"]
        frm.append(src[keep])
        to.append(dst[keep])
    from_ids = np.concatenate(frm).astype(np.int32)
    to_ids = np.concatenate(to).astype(np.int32)

    class Net(px.Network):
        forward_pass = px.ForwardPass("identity")
        # growth is declared (its rule runs in numpy below); the builder gives
        # the deepest level its bucket, as it does for any growing network
        add_conn = px.ProposeAddConn(proposals_per_proposer=1, max_new_per_level=1)
        extra_conn_fields = (px.FieldSpec.int32("test/age"), px.FieldSpec.float32("test/trace", default=1.5))
        propagation = px.Propagation.TOPOLOGICAL

    static, state = px.NetworkBuilder.from_edges(
        Net, num_units, from_ids, to_ids, weights=np.ones(from_ids.size, np.float32),
        input_ids=list(range(widths[0])), output_ids=list(range(int(offsets[-2]), num_units)),
        capacity_headroom=cfg["headroom"], capacity_align=cfg["align"], device="cpu")
    buckets = [{k: v.numpy().copy() for k, v in b.items()} for b in state.conns]
    level = state.units["level"].numpy().copy()
    return num_units, buckets, level


def _digest(buckets, needs_resort, overflows):
    h = hashlib.sha256()
    for b in buckets:
        for name in sorted(b):
            h.update(name.encode())
            h.update(np.ascontiguousarray(b[name]).tobytes())
    h.update(bytes([bool(needs_resort)]))
    h.update(bytes(overflows))
    return h.hexdigest()[:16]


def _repeats_earlier(src, dst):
    seen, out = set(), np.zeros(src.size, bool)
    for i, key in enumerate(zip(src.tolist(), dst.tolist(), strict=True)):
        out[i] = key in seen
        seen.add(key)
    return out


def _step(cfg, t, n, buckets, level):
    """One churn step: prune, growth (select per bucket + claim), tick."""
    for b in buckets:  # _HashPrune
        h = _h(b["from_id"], b["to_id"], t, 7)
        b["dead"] |= ((h & U32(255)) < U32(cfg["rate"])).astype(np.uint8)
    num_buckets = len(buckets)
    gap = cfg.get("max_level_gap", 1)
    if cfg["grow"] == "propose":  # _HashProposals, proposer "global"
        j = np.arange(cfg["proposals"], dtype=np.int64)
        h = _h(j, t, 11)
        src = (h % U32(n)).astype(np.int32)
        h2 = _h(h, 13)
        dst = (h2 % U32(n)).astype(np.int32)
        score = ((h2 >> U32(8)) & U32(7)).astype(np.float32)
        score = np.where((h >> U32(24)) < U32(40), np.float32(-np.inf), score).astype(np.float32)
        ded_live = ded_step = cfg["dedupe"]
        k = min(cfg["k"], cfg["proposals"])
    else:  # _HashGrid over every (src, dst) pair, live-edge dedupe on
        src = np.repeat(np.arange(n, dtype=np.int32), n)
        dst = np.tile(np.arange(n, dtype=np.int32), n)
        h = _h(src, dst, t, 17)
        score = (h & U32(15)).astype(np.float32)
        score = np.where((h >> U32(28)) < U32(3), np.float32(-np.inf), score).astype(np.float32)
        ded_live, ded_step = True, False
        k = min(cfg["k"], n * n)
    ls, ld = level[src], level[dst]
    valid = (np.abs(ld - ls) <= gap) & (src != dst) & (ls < num_buckets)
    if ded_live:
        for i in np.flatnonzero(valid):
            b = buckets[ls[i]]
            live = b["dead"] == 0
            if np.any(live & (b["from_id"] == src[i]) & (b["to_id"] == dst[i])):
                valid[i] = False
    score = np.where(valid, score, np.float32(-np.inf)).astype(np.float32)
    if ded_step:
        by_score = np.argsort(-score, kind="stable")
        rep = np.zeros(score.size, bool)
        rep[by_score] = _repeats_earlier(src[by_score], dst[by_score])
        score = np.where(rep, np.float32(-np.inf), score).astype(np.float32)
    perm = orc.total_order(score, src, dst)
    win, filled = orc.select_per_segment(perm, ls, num_buckets, k)
    overflow = False
    resort = False
    for bk in range(num_buckets):
        top = win[bk]
        grow = (np.arange(k) < filled[bk]) & valid[top] & np.isfinite(score[top])
        cs, cd = src[top].astype(np.int32), dst[top].astype(np.int32)
        w = (((cs.astype(np.int64) * 3 + cd) % 17) - 8).astype(np.float32)
        age = (t + cs).astype(np.int32)
        trace = np.full(k, 1.5, np.float32)
        counts, over = orc.claim_topological(buckets[bk], level, cs, cd, w, grow.astype(np.uint8),
                                             extra={"test/age": age, "test/trace": trace})
        overflow |= bool(counts[1] > 0)
        resort |= bool(counts[3] > 0)
    return overflow, resort


@pytest.mark.parametrize("name", sorted(GOLD["configs"]))
def test_claim_digest_matches_the_reference(name):
    cfg = GOLD["configs"][name]
    n, buckets, level = _build(cfg)
    needs_resort = False
    overflows = []
    for t in range(GOLD["steps"]):
        over, resort = _step(cfg, t, n, buckets, level)
        needs_resort |= resort
        overflows.append(over)
    assert _digest(buckets, needs_resort, overflows) == GOLD["golden"][name]


def test_the_configs_exercise_overflow():
    cfg = GOLD["configs"]["propose_overflow"]
    n, buckets, level = _build(cfg)
    overs = [_step(cfg, t, n, buckets, level)[0] for t in range(GOLD["steps"])]
    assert any(overs) and not all(overs)
