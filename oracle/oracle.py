"""CPU oracle for the plastax edge-arena hot path (numpy front end of pxo.c).

TEST INFRASTRUCTURE ONLY: the checker the CUDA engine is compared against,
and the CPU baseline bench.py times. Only tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg import it; plastax_b200 never does.

Arrays are numpy; buckets are dicts of columns named as the reference names
them (``from_id``, ``to_id``, ``dead``, ``weight``, ``opt/...``). Every
function names the reference lines it restates (paths within the plastax
project); the C bodies in pxo.c carry the same citations.
"""

from __future__ import annotations

import ctypes
import functools
import pathlib
import subprocess

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
LIB = HERE / "_build" / "libpxo.so"

MONOID = {"sum": 0, "max": 1, "min": 2}
ACT = {"identity": 0, "tanh": 1, "relu": 2, "sigmoid": 3}
OPT = {"sgd": 0, "momentum": 1, "adam": 2, "rmsprop": 3}


class _Opt(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int32), ("lr", ctypes.c_float), ("b1", ctypes.c_float),
                ("b2", ctypes.c_float), ("eps", ctypes.c_float), ("wd", ctypes.c_float)]


class _Extra(ctypes.Structure):
    _fields_ = [("n_extra", ctypes.c_int32), ("cols", ctypes.c_void_p * 8), ("bytes", ctypes.c_int32 * 8),
                ("vals", ctypes.c_void_p * 8)]


def build() -> pathlib.Path:
    """Compile pxo.c into _build/libpxo.so (make, with the PATH gcc)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB


@functools.cache
def lib() -> ctypes.CDLL:
    if not LIB.exists():
        build()
    h = ctypes.CDLL(str(LIB))
    h.pxo_philox32.restype = ctypes.c_uint32
    h.pxo_philox32.argtypes = [ctypes.c_uint64, ctypes.c_uint64]
    h.pxo_site_seed.restype = ctypes.c_uint64
    h.pxo_site_seed.argtypes = [ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32]
    h.pxo_unit_float.restype = ctypes.c_float
    h.pxo_unit_float.argtypes = [ctypes.c_uint32]
    h.pxo_select_step.restype = ctypes.c_int64
    h.pxo_max_threads.restype = ctypes.c_int
    h.pxo_lowest_prune.restype = ctypes.c_int64
    return h


def _p(a: np.ndarray | None) -> ctypes.c_void_p | None:
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be contiguous"
    return ctypes.c_void_p(a.ctypes.data)


def _i64(v: int) -> ctypes.c_int64:
    return ctypes.c_int64(int(v))


# ---------------------------------------------------------------------------
# RNG (src/plastax/rng.py:1-57, :109-142, :207-246)
# ---------------------------------------------------------------------------
def philox32(seed: int, counter: int) -> int:
    return int(lib().pxo_philox32(seed & (2**64 - 1), counter & (2**64 - 1)))


def philox32_many(seed: np.ndarray, counter: np.ndarray) -> np.ndarray:
    s = np.ascontiguousarray(seed, np.uint64)
    c = np.ascontiguousarray(counter, np.uint64)
    out = np.empty(s.shape, np.uint32)
    lib().pxo_philox32_many(_i64(s.size), _p(s), _p(c), _p(out))
    return out


def site_seed(network_seed: int, step: int, stream: int, key: int) -> int:
    return int(lib().pxo_site_seed(network_seed, step, stream, key))


def unit_float(word: int) -> np.float32:
    return np.float32(lib().pxo_unit_float(word))


class SiteRng:
    """One proposal site's draw stream (src/plastax/rng.py:188-300)."""

    def __init__(self, seed: int, j: int) -> None:
        self.seed, self.j, self.sub = seed, j, 0

    def word(self) -> int:
        w = philox32(self.seed, (self.j << 16) | self.sub)
        self.sub += 1
        return w

    def uniform(self) -> np.float32:
        return unit_float(self.word())

    def uniform_int(self, n: int) -> int:
        u = self.uniform()
        return min(int(np.uint32(np.float32(u) * np.float32(n))), n - 1)


# ---------------------------------------------------------------------------
# propagation (src/plastax/sweep.py:113-232, phases.py:942-1104)
# ---------------------------------------------------------------------------
def forward_accumulate(b: dict, act: np.ndarray, n: int, monoid: str, acc: np.ndarray) -> None:
    work = np.empty(n, np.float64)
    lib().pxo_forward_accumulate(_i64(b["dead"].size), _p(b["from_id"]), _p(b["to_id"]), _p(b["dead"]),
                                 _p(b["weight"]), _p(act), ctypes.c_int32(n), MONOID[monoid], _p(acc), _p(work))


def backward_accumulate(b: dict, grad: np.ndarray, n: int, monoid: str, acc: np.ndarray) -> None:
    work = np.empty(n, np.float64)
    lib().pxo_backward_accumulate(_i64(b["dead"].size), _p(b["from_id"]), _p(b["to_id"]), _p(b["dead"]),
                                  _p(b["weight"]), _p(grad), ctypes.c_int32(n), MONOID[monoid], _p(acc),
                                  _p(work))


def prune(b: dict, n: int, kind: int, threshold: float, unit_threshold: np.ndarray | None = None,
          block_len: int = 0) -> np.ndarray | None:
    """dead |= predicate in place (src/plastax/phases.py:1444-1498); returns
    the per-block free counts when block_len > 0."""
    cap = b["dead"].size
    counts = np.zeros((cap + block_len - 1) // block_len, np.int32) if block_len else None
    lib().pxo_prune(_i64(cap), _p(b["to_id"]), _p(b["dead"]), _p(b["weight"]), ctypes.c_int32(n),
                    ctypes.c_int(kind), ctypes.c_float(threshold), _p(unit_threshold),
                    ctypes.c_int32(block_len), _p(counts))
    return counts


def _opt(kind: str, lr: float, b1: float = 0.0, b2: float = 0.0, eps: float = 0.0, wd: float = 0.0) -> _Opt:
    return _Opt(OPT[kind], lr, b1, b2, eps, wd)


def update_conn(b: dict, grad: np.ndarray, act: np.ndarray, n: int, opt: dict) -> None:
    """Incoming optimizer pass over one bucket (src/plastax/sweep.py:488-532)."""
    o = _opt(**opt)
    lib().pxo_update_conn(_i64(b["dead"].size), _p(b["from_id"]), _p(b["to_id"]), _p(b["dead"]),
                          _p(b["weight"]), _p(grad), _p(act), ctypes.c_int32(n), ctypes.byref(o),
                          _p(b.get("opt/m")), _p(b.get("opt/v")), _p(b.get("opt/t")))


def batched_update(b: dict, g: np.ndarray, a: np.ndarray, n: int, opt: dict) -> None:
    """Exact batch-mean update (src/plastax/phases.py:434-483); g, a are [n, B]."""
    o = _opt(**opt)
    lib().pxo_batched_update(_i64(b["dead"].size), _p(b["from_id"]), _p(b["to_id"]), _p(b["dead"]),
                             _p(b["weight"]), _p(g), _p(a), ctypes.c_int32(g.shape[1]), ctypes.c_int32(n),
                             ctypes.byref(o), _p(b.get("opt/m")), _p(b.get("opt/v")), _p(b.get("opt/t")))


def batched_product(b: dict, x: np.ndarray, n: int, backward: bool, out: np.ndarray) -> None:
    lib().pxo_batched_product(_i64(b["dead"].size), _p(b["from_id"]), _p(b["to_id"]), _p(b["dead"]),
                              _p(b["weight"]), _p(x), ctypes.c_int32(x.shape[1]), ctypes.c_int32(n),
                              ctypes.c_int(1 if backward else 0), _p(out))


def unit_apply(n: int, mode: int, act_kind: str, monoid: str, acc: np.ndarray, act: np.ndarray | None,
               seed: np.ndarray | None, level: np.ndarray | None, target_level: int,
               is_input: np.ndarray | None, pruned: np.ndarray | None, out: np.ndarray) -> None:
    lib().pxo_unit_apply(ctypes.c_int32(n), ctypes.c_int(mode), ctypes.c_int(ACT[act_kind]),
                         ctypes.c_int(MONOID[monoid]), _p(acc), _p(act), _p(seed), _p(level),
                         ctypes.c_int32(target_level), _p(is_input), _p(pruned), _p(out))


# ---------------------------------------------------------------------------
# growth (src/plastax/phases.py:3813-3860, :4041-4487)
# ---------------------------------------------------------------------------
def propose_per_unit(n: int, proposals: int, network_seed: int, step: int, dst_lo: int, dst_n: int,
                     score_kind: int, level: np.ndarray, *, grad: np.ndarray | None = None,
                     act: np.ndarray | None = None, pruned: np.ndarray | None = None, max_level_gap: int = 1,
                     direction: int = 0, allow_self_loops: bool = False, bucket_level: int = -1,
                     src_level_bound: int = 0, threads: int = 1) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Per-unit proposals; `threads` > 1 splits the units over host threads
    (the same output)."""
    total = n * proposals
    src = np.empty(total, np.int32)
    dst = np.empty(total, np.int32)
    score = np.empty(total, np.float32)
    args = [ctypes.c_int32(n), ctypes.c_int32(proposals), ctypes.c_uint64(network_seed),
            ctypes.c_int32(step), ctypes.c_int32(dst_lo), ctypes.c_int32(dst_n),
            ctypes.c_int(score_kind), _p(grad), _p(act), _p(level), _p(pruned),
            ctypes.c_int32(max_level_gap), ctypes.c_int(direction),
            ctypes.c_int(1 if allow_self_loops else 0), ctypes.c_int32(bucket_level),
            ctypes.c_int32(src_level_bound), _p(src), _p(dst), _p(score)]
    if threads > 1:
        lib().pxo_propose_per_unit_mt(*args, ctypes.c_int(threads))
    else:
        lib().pxo_propose_per_unit(*args)
    return src, dst, score


def total_order(score: np.ndarray, src: np.ndarray, dst: np.ndarray, threads: int = 1) -> np.ndarray:
    """The total order's permutation; `threads` > 1 sorts chunks on host
    threads and merges them (the same permutation)."""
    score = np.ascontiguousarray(score, np.float32)
    src = np.ascontiguousarray(src, np.int32)
    dst = np.ascontiguousarray(dst, np.int32)
    perm = np.empty(score.size, np.int32)
    if threads > 1:
        lib().pxo_total_order_mt(_i64(score.size), _p(score), _p(src), _p(dst), _p(perm), ctypes.c_int(threads))
    else:
        lib().pxo_total_order(_i64(score.size), _p(score), _p(src), _p(dst), _p(perm))
    return perm


def select_step(perm: np.ndarray, src: np.ndarray, level: np.ndarray, k: int) -> np.ndarray:
    win = np.empty(max(min(k, perm.size), 1), np.int32)
    kk = lib().pxo_select_step(_i64(perm.size), _p(perm), _p(src), _p(level), _i64(k), _p(win))
    return win[:kk]


def select_per_segment(perm: np.ndarray, segment: np.ndarray, num_seg: int, k: int
                       ) -> tuple[np.ndarray, np.ndarray]:
    win = np.zeros((num_seg, max(k, 1)), np.int32)
    filled = np.zeros(num_seg, np.int32)
    seg = np.ascontiguousarray(segment, np.int32)
    lib().pxo_select_per_segment(_i64(perm.size), _p(perm), _p(seg),
                                 ctypes.c_int32(num_seg), _i64(k), _p(win), _p(filled))
    return win[:, :k], filled


def _extra(cols: list[np.ndarray], vals: list[np.ndarray]) -> _Extra:
    e = _Extra()
    e.n_extra = len(cols)
    for i, (c, v) in enumerate(zip(cols, vals, strict=True)):
        e.cols[i] = c.ctypes.data
        e.bytes[i] = c.dtype.itemsize
        e.vals[i] = v.ctypes.data
    return e


def claim_pipeline(b: dict, level: np.ndarray, tail_start: int, src: np.ndarray, dst: np.ndarray,
                   weight: np.ndarray, growable: np.ndarray, *, max_new: int = -1,
                   extra: dict[str, np.ndarray] | None = None, threads: int = 1) -> tuple[np.ndarray, np.ndarray, int]:
    """Pipeline claim in place (src/plastax/phases.py:2985-3106). Returns
    (counts[4], overflowed[k], new tail_start); `threads` > 1 builds the
    free-slot lists on host threads (the same claim)."""
    k = src.size
    counts = np.zeros(4, np.int32)
    over = np.zeros(max(k, 1), np.uint8)
    tail = ctypes.c_int64(tail_start)
    grow = np.ascontiguousarray(growable, np.uint8)
    names = sorted(extra or {})
    ex = _extra([b[nm] for nm in names], [np.ascontiguousarray(extra[nm]) for nm in names]) if names else None
    args = [_i64(b["dead"].size), _p(b["from_id"]), _p(b["to_id"]), _p(b["dead"]), _p(b["weight"]), _p(level),
            ctypes.c_int32(level.size), ctypes.byref(tail), _i64(k), _p(src), _p(dst), _p(weight), _p(grow),
            _i64(max_new), ctypes.byref(ex) if ex else None, _p(counts), _p(over)]
    if threads > 1:
        lib().pxo_claim_pipeline_mt(*args, ctypes.c_int(threads))
    else:
        lib().pxo_claim_pipeline(*args)
    return counts, over[:k], int(tail.value)


def claim_topological(b: dict, level: np.ndarray, src: np.ndarray, dst: np.ndarray, weight: np.ndarray,
                      growable: np.ndarray, *, max_new: int = -1, extra: dict[str, np.ndarray] | None = None
                      ) -> tuple[np.ndarray, np.ndarray]:
    """Topological claim of one bucket in place (src/plastax/phases.py:2853-2982)."""
    k = src.size
    counts = np.zeros(4, np.int32)
    over = np.zeros(max(k, 1), np.uint8)
    grow = np.ascontiguousarray(growable, np.uint8)
    names = sorted(extra or {})
    ex = _extra([b[nm] for nm in names], [np.ascontiguousarray(extra[nm]) for nm in names]) if names else None
    lib().pxo_claim_topological(_i64(b["dead"].size), _p(b["from_id"]), _p(b["to_id"]), _p(b["dead"]),
                                _p(b["weight"]), _p(level), ctypes.c_int32(level.size), _i64(k), _p(src),
                                _p(dst), _p(weight), _p(grow), _i64(max_new),
                                ctypes.byref(ex) if ex else None, _p(counts), _p(over))
    return counts, over[:k]


# ---------------------------------------------------------------------------
# CPU baseline (timing only)
# ---------------------------------------------------------------------------
def forward_prune_mt(b: dict, act: np.ndarray, n: int, threshold: float, acc: np.ndarray, threads: int) -> None:
    work = np.empty(max(threads, 1) * n, np.float64)
    lib().pxo_forward_prune_mt(_i64(b["dead"].size), _p(b["from_id"]), _p(b["to_id"]), _p(b["dead"]),
                               _p(b["weight"]), _p(act), ctypes.c_int32(n), ctypes.c_float(threshold), _p(acc),
                               ctypes.c_int(threads), _p(work))


def lowest_prune(b: dict, k: int, threads: int = 1) -> int:
    """Tombstone the k live edges of lowest |w| of one bucket (ties by
    ascending slot, NaN never), in place; returns the number pruned
    (src/plastax/phases.py:1444-1498 with the k-th smallest |w| as the
    threshold, examples/dst_sparse.py:88-140)."""
    return int(lib().pxo_lowest_prune(_i64(b["dead"].size), _p(b["dead"]), _p(b["weight"]), _i64(k),
                                      ctypes.c_int(threads)))


def max_threads() -> int:
    return int(lib().pxo_max_threads())
