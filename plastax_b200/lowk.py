"""The exact lowest-|w| prune fused into the mirror sweep (see csrc/lowk.cu).

`LowestK` owns the prune's device state for one StepFn: the coarse and fine
histograms of bits(|w|) (>> 15 and >> 7; 256 KB and 64 MB) over the live
non-NaN edges (the whole arena, replicated on every Scheme-A rank), the
plan the plan kernel writes before each
sweep, the double-buffered lists of the threshold bin's edges (inside the
peer region under Scheme-A, so every rank's selection reads every rank's
list) and running churn totals. Each firing is: `plan()` before the sweep,
`sweep()` (the forward with the prune), `select()` after every rank's sweep,
then the claim and `hist_add()` of its committed edges. The set pruned is
the one the lowest-magnitude prune phase chooses (src/plastax/phases.py:
1444-1498 with the k-th smallest |w| as the predicate's threshold,
examples/dst_sparse.py:88-140): exactly min(k, live non-NaN) edges, ties by
ascending global slot.
"""

from __future__ import annotations

import ctypes

import torch

from plastax_b200 import _lib
from plastax_b200.kernels import _stream, ptr

# status bits of the plan
STATUS_LIST_OVERFLOW = 1
STATUS_COUNTS = 2


class LowestK:
    def __init__(self, k: int, device: torch.device, *, list_cap: int | None = None, slot_base: int = 0,
                 peers=None) -> None:
        dev = torch.device(device)
        self.k = int(k)
        self.list_cap = int(list_cap) if list_cap is not None else max(1 << 16, self.k)
        if self.list_cap < 1:
            raise ValueError("lowest-|w| prune: list capacity must be >= 1")
        self.dev = dev
        self.hist = torch.zeros(_lib.LOWK_BINS, dtype=torch.int32, device=dev)
        self.fine = torch.zeros(_lib.LOWK_FINE_BINS, dtype=torch.int32, device=dev)
        # pxb_lowk_plan: 64 bytes (lo, hi | take | below | listed | parity, status | pruned | floor, zero_lo |
        # zero_hi, pad)
        self.plan = torch.zeros(8, dtype=torch.int64, device=dev)
        self.pos = torch.empty(2 * self.list_cap, dtype=torch.int64, device=dev)
        # the plan kernel's partial sums and arrival counter (zero between plans)
        self.plan_scratch = torch.zeros(_lib.LOWK_PLAN_SCRATCH, dtype=torch.int32, device=dev)
        # running {pruned by this rank, committed, overflowed, firings}
        self.totals = torch.zeros(4, dtype=torch.int64, device=dev)
        self.peers = peers
        if peers is None:
            self.key = torch.empty(2 * self.list_cap, dtype=torch.int64, device=dev)
            self.level = torch.empty(2 * self.list_cap, dtype=torch.int32, device=dev)
            self.count = torch.zeros(4, dtype=torch.int64, device=dev)
            rank, world, pk, pl, pc = 0, 1, None, None, None
        else:
            if peers.lowk_cap != self.list_cap:
                raise ValueError(f"peer region holds lists of {peers.lowk_cap}, the prune needs {self.list_cap}")
            self.key, self.level, self.count = peers.lowk_key, peers.lowk_level, peers.lowk_count
            rank, world = peers.rank, peers.world
            pk, pl, pc = peers.p_lkey.data_ptr(), peers.p_llevel.data_ptr(), peers.p_lcount.data_ptr()
        self.struct = _lib.Lowk(rank, world, self.k, self.list_cap, int(slot_base), self.hist.data_ptr(),
                                self.fine.data_ptr(), self.plan.data_ptr(), self.key.data_ptr(), self.level.data_ptr(),
                                self.count.data_ptr(), self.pos.data_ptr(), pk, pl, pc,
                                self.plan_scratch.data_ptr())

    # -- histogram -------------------------------------------------------------
    def build_hist(self, buckets, combine=None, combine_min=None) -> None:
        """Rebuild the histograms from the canonical columns (a bind, or any
        change of the arena outside the step); `combine(t)` sums a tensor
        over the Scheme-A ranks, `combine_min(t)` takes its minimum."""
        self.hist.zero_()
        self.fine.zero_()
        w = self.plan.view(torch.int32)
        w[12] = -1  # floor: no fine bin seen yet
        for b in buckets:
            cap = int(b["dead"].numel())
            _lib.call("pxb_lowk_hist_build", ctypes.byref(self.struct), ctypes.c_int64(cap), ptr(b["dead"]),
                      ptr(b["weight"]), _stream())
        if combine is not None:
            combine(self.hist)
            combine(self.fine)
            floor = w[12:13].to(torch.int64) & 0xFFFFFFFF
            combine_min(floor)
            w[12] = floor.to(torch.int32)[0]

    # -- one firing --------------------------------------------------------------
    def make_plan(self) -> None:
        _lib.call("pxb_lowk_make_plan", ctypes.byref(self.struct), _stream())

    def sweep(self, m, act: torch.Tensor, acc: torch.Tensor, acc_fixed: torch.Tensor | None, monoid: str,
              dead: torch.Tensor, free_bitmap: torch.Tensor | None, bitmap_level: torch.Tensor | None,
              flush: bool = True) -> None:
        """The forward sweep with the prune; with `flush` False the sweep's
        deferred tombstones are left for `flush()`."""
        name = "pxb_mirror_forward_lowk" if flush else "pxb_mirror_forward_lowk_deferred"
        _lib.call(name, ctypes.byref(m.struct), ptr(act), ctypes.c_int32(_lib.MONOID[monoid]),
                  ptr(acc), ptr(acc_fixed), ctypes.byref(self.struct), ptr(dead), ptr(free_bitmap),
                  ctypes.c_int64((dead.numel() + 31) // 32), ptr(bitmap_level), _stream())

    def flush(self, m, monoid: str, dead: torch.Tensor, free_bitmap: torch.Tensor | None,
              bitmap_level: torch.Tensor | None) -> None:
        """The deferred tombstones of the last `sweep(..., flush=False)`."""
        _lib.call("pxb_mirror_defer_flush", ctypes.byref(m.struct), ctypes.c_int32(_lib.MONOID[monoid]),
                  ctypes.byref(self.struct), ptr(dead), ptr(free_bitmap), ctypes.c_int64((dead.numel() + 31) // 32),
                  ptr(bitmap_level), _stream())

    def select(self, m, dead: torch.Tensor, free_bitmap: torch.Tensor | None, bitmap_level: torch.Tensor | None,
               *, num_levels: int = 0, level_before: torch.Tensor | None = None,
               level_totals: torch.Tensor | None = None) -> None:
        _lib.call("pxb_lowk_select", ctypes.byref(self.struct), ctypes.byref(m.struct), ptr(dead), ptr(free_bitmap),
                  ctypes.c_int64((dead.numel() + 31) // 32), ptr(bitmap_level), ctypes.c_int32(num_levels),
                  ptr(level_before), ptr(level_totals), _stream())

    def hist_add(self, weight: torch.Tensor, committed: torch.Tensor, claim_counts: torch.Tensor | None,
                 tally: bool = True) -> None:
        _lib.call("pxb_lowk_hist_add", ctypes.byref(self.struct), ctypes.c_int64(weight.numel()), ptr(weight),
                  ptr(committed), ptr(claim_counts), ptr(self.totals) if tally else None, _stream())

    # -- host reads ----------------------------------------------------------------
    @property
    def status(self) -> torch.Tensor:
        """Device word: bit 0 a list overflowed its capacity, bit 1 the swept
        counts disagreed with the histogram."""
        return self.plan.view(torch.int32)[9]

    def plan_host(self) -> dict:
        """The last plan's fields (host read; synchronises)."""
        p = self.plan.cpu()
        w = p.view(torch.int32)
        return {"lo_bits": int(w[0]) & 0xFFFFFFFF, "hi_bits": int(w[1]) & 0xFFFFFFFF, "take": int(p[1]),
                "below_expect": int(p[2]), "listed_expect": int(p[3]), "parity": int(w[8]), "status": int(w[9]),
                "pruned": int(p[5]), "floor": int(w[12]) & 0xFFFFFFFF, "zero_lo": int(w[13]) & 0xFFFFFFFF,
                "zero_hi": int(w[14]) & 0xFFFFFFFF}


__all__ = ["LowestK", "STATUS_LIST_OVERFLOW", "STATUS_COUNTS"]
