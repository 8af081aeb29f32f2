"""Scheme-A groups over NVLink peer memory (see csrc/peer.cu).

Every rank allocates one region with the same layout -- the int64
fixed-point partials, the float side partials, the activation column and two
rows of flags -- and maps every peer's region through CUDA IPC; the handles
travel once through torch.distributed. `scheme_a_apply` then reduces this
rank's slice of the units from every peer and writes the applied activations
into every peer, in one kernel per step (the all-reduce of
src/plastax/monoid.py:175-204 plus the apply of src/plastax/sweep.py:183-230).
"""

from __future__ import annotations

import ctypes

import torch

from plastax_b200 import _lib

_ALIGN = 256
# polls of one flag before a wait gives up (about a second with the kernel's
# back-off); a timeout sets status bit 0 instead of hanging the GPU
DEFAULT_WAIT_POLLS = 1 << 23


def _align(x: int) -> int:
    return (x + _ALIGN - 1) // _ALIGN * _ALIGN


class _Raw:
    """A device buffer described to torch without a copy."""

    def __init__(self, ptr: int, n: int, typestr: str) -> None:
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": typestr, "data": (ptr, False), "version": 3}


def _view(ptr: int, n: int, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
    typestr = {torch.int64: "<i8", torch.float32: "<f4", torch.int32: "<i4", torch.uint8: "|u1"}[dtype]
    return torch.as_tensor(_Raw(ptr, n, typestr), device=device)


class PeerGroup:
    """One rank's symmetric region and its peers' mappings (collective: every
    rank of `group` constructs it at the same point)."""

    def __init__(self, num_units: int, device: torch.device, group=None, lowk_cap: int = 0, win_k: int = 0,
                 win_blocks: int = 3) -> None:
        import torch.distributed as dist

        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.dev = torch.device(device)
        n = int(num_units)
        self.n = n
        self.off_fixed = 0
        self.off_side = _align(self.off_fixed + 8 * n)
        self.off_act = _align(self.off_side + 4 * n)
        self.off_flags = _align(self.off_act + 4 * n)
        self.off_counts = _align(self.off_flags + 4 * 2 * self.world)
        # the exact lowest-|w| prune's lists (keys, claim domains, counters),
        # double-buffered, read by every peer's selection
        self.lowk_cap = int(lowk_cap)
        self.off_lkey = _align(self.off_counts + 4 * self.world * _lib.PEER_MAX_LEVELS)
        self.off_llevel = _align(self.off_lkey + 8 * 2 * self.lowk_cap)
        self.off_lcount = _align(self.off_llevel + 4 * 2 * self.lowk_cap)
        # the growth selection's winner columns (src, dst, weight, growable),
        # `win_blocks` lists of `win_k` each, written by every rank's share of
        # the selection
        self.win_k, self.win_blocks = int(win_k), int(win_blocks)
        wn = self.win_k * self.win_blocks
        self.off_wsrc = _align(self.off_lcount + 8 * 4)
        self.off_wdst = _align(self.off_wsrc + 4 * wn)
        self.off_ww = _align(self.off_wdst + 4 * wn)
        self.off_wgrow = _align(self.off_ww + 4 * wn)
        self.bytes = _align(self.off_wgrow + wn)
        lib = _lib.lib()
        lib.pxb_set_device(self.dev.index)
        base = ctypes.c_void_p()
        handle = (ctypes.c_uint8 * 64)()
        _lib.call("pxb_peer_alloc", ctypes.c_size_t(self.bytes), ctypes.byref(base),
                  ctypes.cast(handle, ctypes.c_void_p))
        self.base = int(base.value)
        handles: list = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.bases: list[int] = []
        self.opened: list[int] = []
        for q, h in enumerate(handles):
            if q == self.rank:
                self.bases.append(self.base)
                continue
            hb = (ctypes.c_uint8 * 64).from_buffer_copy(h)
            p = ctypes.c_void_p()
            _lib.call("pxb_peer_open", ctypes.cast(hb, ctypes.c_void_p), ctypes.byref(p))
            self.bases.append(int(p.value))
            self.opened.append(int(p.value))
        mk = lambda off: torch.tensor([b + off for b in self.bases], dtype=torch.int64, device=self.dev)  # noqa: E731
        self.p_fixed, self.p_side, self.p_act, self.p_flags, self.p_counts = (
            mk(self.off_fixed), mk(self.off_side), mk(self.off_act), mk(self.off_flags), mk(self.off_counts))
        self.p_lkey, self.p_llevel, self.p_lcount = mk(self.off_lkey), mk(self.off_llevel), mk(self.off_lcount)
        self.words = torch.zeros(4, dtype=torch.int32, device=self.dev)  # epoch, done, status, pad
        w = self.words.data_ptr()
        self.struct = _lib.PeerGroup(self.rank, self.world, self.p_fixed.data_ptr(), self.p_side.data_ptr(),
                                     self.p_act.data_ptr(), self.p_flags.data_ptr(), self.p_counts.data_ptr(),
                                     w, w + 4, w + 8)
        # this rank's buffers as tensors (the region outlives them: close() last)
        self.acc_fixed = _view(self.base + self.off_fixed, n, torch.int64, self.dev)
        self.acc_side = _view(self.base + self.off_side, n, torch.float32, self.dev)
        self.act = _view(self.base + self.off_act, n, torch.float32, self.dev)
        if self.lowk_cap > 0:
            self.lowk_key = _view(self.base + self.off_lkey, 2 * self.lowk_cap, torch.int64, self.dev)
            self.lowk_level = _view(self.base + self.off_llevel, 2 * self.lowk_cap, torch.int32, self.dev)
            self.lowk_count = _view(self.base + self.off_lcount, 4, torch.int64, self.dev)
        self.win_cols = None
        if wn > 0:
            self.win_cols = (_view(self.base + self.off_wsrc, wn, torch.int32, self.dev),
                             _view(self.base + self.off_wdst, wn, torch.int32, self.dev),
                             _view(self.base + self.off_ww, wn, torch.float32, self.dev),
                             _view(self.base + self.off_wgrow, wn, torch.uint8, self.dev))
            # every rank's columns, as this rank addresses them
            self.win_ptrs = [(b + self.off_wsrc, b + self.off_wdst, b + self.off_ww, b + self.off_wgrow)
                             for b in self.bases]
        self.closed = False

    @property
    def status(self) -> torch.Tensor:
        """Device word: bit 0 set when a wait for a peer gave up."""
        return self.words[2]

    def close(self) -> None:
        """Unmap the peers and free the region once every rank is done with it."""
        if self.closed:
            return
        torch.cuda.synchronize(self.dev)
        self.dist.barrier(group=self.group)
        for p in self.opened:
            _lib.call("pxb_peer_close", ctypes.c_void_p(p))
        self.dist.barrier(group=self.group)
        self.acc_fixed = self.acc_side = self.act = None
        self.lowk_key = self.lowk_level = self.lowk_count = None
        self.win_cols = None
        _lib.call("pxb_peer_free", ctypes.c_void_p(self.base))
        self.closed = True


def scheme_a_apply(group: PeerGroup, act_kind: str, *, is_input: torch.Tensor | None = None,
                   pruned: torch.Tensor | None = None, level_counts: torch.Tensor | None = None,
                   level_before: torch.Tensor | None = None, level_totals: torch.Tensor | None = None,
                   wait_polls: int = DEFAULT_WAIT_POLLS) -> None:
    """The combine + apply; with `level_counts` (this rank's per-domain free
    counts) the counts of every rank ride on the barrier and `level_before` /
    `level_totals` receive the claim's Scheme-A inputs."""
    from plastax_b200.kernels import _stream, ptr

    nl = 0 if level_counts is None else level_counts.numel()
    _lib.call("pxb_scheme_a_apply", ctypes.byref(group.struct), ctypes.c_int32(group.n),
              ctypes.c_int32(_lib.act_code(act_kind)), ptr(is_input), ptr(pruned), ptr(level_counts),
              ctypes.c_int32(nl), ptr(level_before), ptr(level_totals), ctypes.c_uint32(wait_polls), _stream())


__all__ = ["PeerGroup", "scheme_a_apply", "DEFAULT_WAIT_POLLS"]
