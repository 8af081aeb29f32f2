"""The destination-grouped mirror of a bucket (see csrc/mirror.cu).

Built once from the canonical columns with one device-side sort (setup, not
the step), then kept current by the fused prune and the claim's inserts.
Live edges are grouped by destination chunk and kept in slot order (source-
major, as the builder lays the bucket out) inside a group: consecutive
entries then read neighbouring activations, so the sweep's gathers coalesce
(a destination-sorted group makes every gather its own L2 sector and was
measured 3.5x slower). Each group gets `slack` spare entries (at least
`min_slack`) for the edges growth inserts, and its capacity is rounded up
to the sweep's tile (PXB_MIRROR_TILE entries), so a tile lies in one group.
"""

from __future__ import annotations

import math

import numpy as np
import torch

from plastax_b200 import _lib


# the largest in-degree at which a mirror sums with 28 fractional bits: the
# rounding error of a destination is then at most 400 * 2^-29 = 7.5e-7
# (under 1e-6 with room for the in-degrees churn adds after the build)
FAST_SUM_FAN_IN = 400


class Mirror:
    def __init__(self, bucket: dict[str, torch.Tensor], num_units: int, *, slack: float = 0.05,
                 min_slack: int = 64, item_entries: int = 1 << 16, ovf_cap: int = 1 << 20,
                 chunk_bits: int | None = None, sum_frac_bits: int | None = None) -> None:
        dev = bucket["dead"].device
        n = int(num_units)
        src_bits = max(1, (n - 1).bit_length())
        cb = min(32 - src_bits, 13)
        if cb < 2:
            raise ValueError(f"mirror: {n} units leave too few bits for a destination chunk")
        if chunk_bits is not None:
            if not 2 <= chunk_bits <= cb:
                raise ValueError(f"mirror: chunk_bits {chunk_bits} not in [2, {cb}] for {n} units")
            cb = int(chunk_bits)
        chunk = 1 << cb
        groups = (n + chunk - 1) // chunk
        frm, to = bucket["from_id"], bucket["to_id"]
        live = torch.nonzero(bucket["dead"] == 0).flatten()
        f, t = frm[live].long(), to[live].long()
        ok = (f >= 0) & (f < n) & (t >= 0) & (t < n)
        live, f, t = live[ok], f[ok], t[ok]
        g = t >> cb
        order = torch.sort(g, stable=True).indices  # group, then slot order
        live, f, t, g = live[order], f[order], t[order], g[order]
        counts = torch.bincount(g, minlength=groups)
        # the largest in-degree: the fixed-point sum's error bound grows with it
        self.max_in_degree = int(torch.bincount(t, minlength=n).max().item()) if t.numel() else 0
        counts_h = counts.cpu().numpy().astype(np.int64)
        spare = np.maximum(min_slack, np.ceil(counts_h * slack).astype(np.int64))
        tile = _lib.MIRROR_TILE
        gcap = (counts_h + spare + tile - 1) // tile * tile
        gbase = np.concatenate([[0], np.cumsum(gcap)]).astype(np.int64)
        entries = int(gbase[-1])
        starts = torch.from_numpy(np.concatenate([[0], np.cumsum(counts_h)[:-1]])).to(dev)
        rank = torch.arange(live.numel(), device=dev) - starts[g]
        pos = torch.from_numpy(gbase[:-1]).to(dev)[g] + rank
        word = torch.full((entries,), -1, dtype=torch.int32, device=dev)
        packed = (f << cb) | (t & (chunk - 1))
        packed = packed - (packed >= 2**31).long() * 2**32
        word[pos] = packed.to(torch.int32)
        weight = torch.zeros(entries, dtype=torch.float32, device=dev)
        weight[pos] = bucket["weight"][live]
        slot = torch.full((entries,), -1, dtype=torch.int32, device=dev)
        slot[pos] = live.to(torch.int32)
        del packed, pos, rank, f, t, g, live, order
        ib, ie, ig = [], [], []
        for grp in range(groups):
            lo, hi = int(gbase[grp]), int(gbase[grp + 1])
            step = max(8, item_entries // 8 * 8)
            for b in range(lo, hi, step):
                ib.append(b)
                ie.append(min(b + step, hi))
                ig.append(grp)
        self.chunk_bits, self.groups, self.entries, self.num_units = cb, groups, entries, n
        self.gbase = torch.from_numpy(gbase).to(dev)
        self.gfill = counts.to(torch.int32)
        self.word, self.weight, self.slot = word, weight, slot
        self.hstack = torch.zeros(max(entries, 4), dtype=torch.int32, device=dev)
        self.hcount = torch.zeros(groups, dtype=torch.int32, device=dev)
        self.item_begin = torch.tensor(ib, dtype=torch.int64, device=dev)
        self.item_end = torch.tensor(ie, dtype=torch.int64, device=dev)
        self.item_group = torch.tensor(ig, dtype=torch.int32, device=dev)
        self.ovf_cap = int(ovf_cap)
        self.ovf_count = torch.zeros(1, dtype=torch.int32, device=dev)
        self.ovf_src = torch.full((max(ovf_cap, 1),), -1, dtype=torch.int32, device=dev)
        self.ovf_dst = torch.zeros(max(ovf_cap, 1), dtype=torch.int32, device=dev)
        self.ovf_slot = torch.zeros(max(ovf_cap, 1), dtype=torch.int32, device=dev)
        self.ovf_weight = torch.zeros(max(ovf_cap, 1), dtype=torch.float32, device=dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self.ins_count = torch.zeros(groups, dtype=torch.int32, device=dev)
        # the sweep's deferred prunes: one segment per sweep CTA (up to 8 per
        # SM), together about one entry in 256 (a CTA whose segment fills up
        # writes the rest of its tombstones in place)
        from plastax_b200.kernels import sm_count

        self.defer_ctas = 8 * sm_count()
        self.defer_seg = max(256, entries // 256 // self.defer_ctas)
        self.defer_pos = torch.empty(self.defer_ctas * self.defer_seg, dtype=torch.int64, device=dev)
        self.defer_count = torch.zeros(self.defer_ctas, dtype=torch.int32, device=dev)
        # the sweep's fixed-point sum: 28 fractional bits while every unit's
        # in-degree leaves room for growth under the 1e-6 bound (F * 2^-29),
        # else 31 (F * 2^-32); 28 bits wrap the 32-bit words far less often
        if sum_frac_bits is None:
            sum_frac_bits = 28 if self.max_in_degree <= FAST_SUM_FAN_IN else 31
        if sum_frac_bits not in (28, 31):
            raise ValueError(f"mirror: sum_frac_bits must be 28 or 31, got {sum_frac_bits}")
        self.sum_frac_bits = int(sum_frac_bits)
        p = lambda x: x.data_ptr()  # noqa: E731
        self.struct = _lib.Mirror(
            n, cb, groups, entries, p(self.gbase), p(self.gfill), p(self.word), p(self.weight), p(self.slot),
            p(self.hstack), p(self.hcount), len(ib), p(self.item_begin), p(self.item_end), p(self.item_group),
            self.ovf_cap, p(self.ovf_count), p(self.ovf_src), p(self.ovf_dst), p(self.ovf_slot), p(self.ovf_weight),
            p(self.status), p(self.ins_count), p(self.defer_pos), p(self.defer_count), self.defer_seg,
            self.defer_ctas, self.sum_frac_bits)

    def healthy(self) -> bool:
        """False when an edge could not be mirrored (host read; synchronises)."""
        return int(self.status.item()) == 0

    def bytes_per_sweep(self) -> int:
        """Bytes the forward streams: word + weight of every used entry."""
        return int(self.gfill.clamp(max=None).sum().item()) * 8


__all__ = ["Mirror", "math"]
