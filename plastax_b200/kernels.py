"""Typed torch-tensor front end of the C ABI (include/pxb.h).

Device memory and streams come from PyTorch (plumbing only); every call goes
straight to a libpxb.so entry point on the current CUDA stream. Arguments
are checked here (device, dtype, contiguity, length) before the C ABI checks
them again, so misuse raises a Python exception and never reaches a kernel.

A bucket is a dict of device columns named like the reference's SOA tags:
``from_id`` int32, ``to_id`` int32, ``dead`` uint8 (the reference's bool),
``weight`` float32 and any ``opt/...`` float32 optimizer column.
"""

from __future__ import annotations

import ctypes
from collections.abc import Mapping, Sequence

import torch

from plastax_b200 import _lib
from plastax_b200._lib import call, query_size

Bucket = Mapping[str, torch.Tensor]

_DTYPES = {
    "from_id": torch.int32,
    "to_id": torch.int32,
    "dead": torch.uint8,
    "weight": torch.float32,
}


_bound_device: list[int] = [-1]


def _stream() -> ctypes.c_void_p:
    """The current torch stream, after binding the library's runtime to the
    current torch device (libpxb links its own CUDA runtime)."""
    dev = torch.cuda.current_device()
    if dev != _bound_device[0]:
        call("pxb_set_device", ctypes.c_int32(dev))
        _bound_device[0] = dev
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def ptr(t: torch.Tensor | None) -> ctypes.c_void_p | None:
    """Device pointer of a contiguous CUDA tensor (None passes NULL)."""
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("engine tensors must live on a CUDA device")
    if not t.is_contiguous():
        raise ValueError("engine tensors must be contiguous")
    return ctypes.c_void_p(t.data_ptr())


def _check(t: torch.Tensor, dtype: torch.dtype, n: int | None, what: str) -> None:
    if t.dtype != dtype:
        raise TypeError(f"{what}: expected {dtype}, got {t.dtype}")
    if n is not None and t.numel() != n:
        raise ValueError(f"{what}: expected {n} elements, got {t.numel()}")


def _bucket(b: Bucket, names=None) -> int:
    """The bucket's capacity, after checking the columns a call reads
    (`names`, default every canonical column)."""
    cap = b["dead"].numel()
    for name, dt in _DTYPES.items():
        if names is None or name in names:
            _check(b[name], dt, cap, f"bucket column {name!r}")
    return cap


def clear_accumulators(acc: torch.Tensor, value: float, acc_fixed: torch.Tensor | None = None) -> None:
    """acc = value and acc_fixed = 0, one launch."""
    _check(acc, torch.float32, None, "accumulator")
    if acc_fixed is not None:
        _check(acc_fixed, torch.int64, acc.numel(), "fixed-point accumulator")
    call("pxb_clear_accumulators", ctypes.c_int64(acc.numel()), ctypes.c_float(value), ptr(acc), ptr(acc_fixed),
         _stream())


def fill(t: torch.Tensor, value: float) -> None:
    _check(t, torch.float32, None, "fill target")
    call("pxb_fill_f32", ctypes.c_int64(t.numel()), ctypes.c_float(value), ptr(t), _stream())


def sm_count() -> int:
    out = ctypes.c_int32(0)
    call("pxb_sm_count", ctypes.byref(out))
    return out.value


# ---------------------------------------------------------------------------
# propagation
# ---------------------------------------------------------------------------
def forward_accumulate(b: Bucket, act: torch.Tensor, acc: torch.Tensor, monoid: str = "sum") -> None:
    cap = _bucket(b)
    n = acc.numel()
    _check(act, torch.float32, n, "act")
    _check(acc, torch.float32, n, "acc")
    call("pxb_forward_accumulate", ctypes.c_int64(cap), ptr(b["from_id"]), ptr(b["to_id"]), ptr(b["dead"]),
         ptr(b["weight"]), ptr(act), ctypes.c_int32(n), _lib.MONOID[monoid], ptr(acc), _stream())


def forward_prune(b: Bucket, act: torch.Tensor, acc: torch.Tensor, *, monoid: str = "sum",
                  prune_kind: int = _lib.PRUNE_ABS_BELOW, threshold: float = 0.0,
                  unit_threshold: torch.Tensor | None = None, dead_out: torch.Tensor | None = None,
                  block_len: int = 0, block_free: torch.Tensor | None = None,
                  free_bitmap: torch.Tensor | None = None, bitmap_level: torch.Tensor | None = None) -> None:
    """Forward accumulate + prune predicate + per-block free counts, one pass."""
    cap = _bucket(b)
    n = acc.numel()
    _check(act, torch.float32, n, "act")
    _check(acc, torch.float32, n, "acc")
    out = b["dead"] if dead_out is None else dead_out
    _check(out, torch.uint8, cap, "dead_out")
    if block_free is not None:
        _check(block_free, torch.int32, (cap + block_len - 1) // block_len, "block_free")
    call("pxb_forward_prune", ctypes.c_int64(cap), ptr(b["from_id"]), ptr(b["to_id"]), ptr(b["dead"]),
         ptr(b["weight"]), ptr(act), ctypes.c_int32(n), _lib.MONOID[monoid], ptr(acc), ctypes.c_int32(prune_kind),
         ctypes.c_float(threshold), ptr(unit_threshold), ptr(out), ctypes.c_int32(block_len), ptr(block_free),
         ptr(free_bitmap), ptr(bitmap_level), _stream())


def prune_conn(b: Bucket, num_units: int, *, prune_kind: int = _lib.PRUNE_ABS_BELOW, threshold: float = 0.0,
               unit_threshold: torch.Tensor | None = None, block_len: int = 0,
               block_free: torch.Tensor | None = None, free_bitmap: torch.Tensor | None = None,
               bitmap_level: torch.Tensor | None = None) -> None:
    cap = _bucket(b)
    call("pxb_prune_conn", ctypes.c_int64(cap), ptr(b["from_id"]), ptr(b["to_id"]), ptr(b["dead"]),
         ptr(b["weight"]), ctypes.c_int32(num_units), ctypes.c_int32(prune_kind), ctypes.c_float(threshold),
         ptr(unit_threshold), ptr(b["dead"]), ctypes.c_int32(block_len), ptr(block_free), ptr(free_bitmap),
         ptr(bitmap_level), _stream())


def backward_accumulate(b: Bucket, grad: torch.Tensor, acc: torch.Tensor, monoid: str = "sum") -> None:
    cap = _bucket(b)
    n = acc.numel()
    _check(grad, torch.float32, n, "grad")
    _check(acc, torch.float32, n, "acc")
    call("pxb_backward_accumulate", ctypes.c_int64(cap), ptr(b["from_id"]), ptr(b["to_id"]), ptr(b["dead"]),
         ptr(b["weight"]), ptr(grad), ctypes.c_int32(n), _lib.MONOID[monoid], ptr(acc), _stream())


def optimizer_struct(kind: str, lr: float, b1: float = 0.0, b2: float = 0.0, eps: float = 0.0,
                     weight_decay: float = 0.0) -> _lib.Optimizer:
    return _lib.Optimizer(_lib.OPT[kind], lr, b1, b2, eps, weight_decay)


OPT_COLS = ("opt/m", "opt/v", "opt/t")


def backward_update(b: Bucket, grad: torch.Tensor, act: torch.Tensor, acc: torch.Tensor | None,
                    opt: _lib.Optimizer, cols: tuple[str, str, str] = OPT_COLS) -> None:
    """Backward accumulate (acc may be None) fused with the optimizer update;
    `cols` names the bucket's (m, v, t) state columns."""
    cap = _bucket(b)
    n = grad.numel()
    _check(act, torch.float32, n, "act")
    if acc is not None:
        _check(acc, torch.float32, n, "acc")
    call("pxb_backward_update", ctypes.c_int64(cap), ptr(b["from_id"]), ptr(b["to_id"]), ptr(b["dead"]),
         ptr(b["weight"]), ptr(grad), ptr(act), ctypes.c_int32(n), ptr(acc), ctypes.byref(opt),
         ptr(b.get(cols[0])), ptr(b.get(cols[1])), ptr(b.get(cols[2])), _stream())


def unit_apply(acc: torch.Tensor, out: torch.Tensor, *, mode: int, act_kind: str, monoid: str = "sum",
               act: torch.Tensor | None = None, seed: torch.Tensor | None = None,
               level: torch.Tensor | None = None, target_level: int = 0, is_input: torch.Tensor | None = None,
               pruned: torch.Tensor | None = None, acc_fixed: torch.Tensor | None = None) -> None:
    n = acc.numel()
    if acc_fixed is not None:
        _check(acc_fixed, torch.int64, n, "unit_apply acc_fixed")
    call("pxb_unit_apply", ctypes.c_int32(n), ctypes.c_int32(mode), ctypes.c_int32(_lib.act_code(act_kind)),
         ctypes.c_int32(_lib.MONOID[monoid]), ptr(acc), ptr(acc_fixed), ptr(act), ptr(seed), ptr(level),
         ctypes.c_int32(target_level), ptr(is_input), ptr(pruned), ptr(out), _stream())


def step_end(step: torch.Tensor, grown: torch.Tensor | None = None, overflow: torch.Tensor | None = None) -> None:
    """Clear the growth flags (when given) and advance the device step
    counter, one launch."""
    call("pxb_step_end", ptr(step), ptr(grown), ptr(overflow), _stream())


def pipeline_train(desc: _lib.PipelineTrain) -> None:
    """The fused pipeline training step (forward + backward accumulation,
    applies and seed, update) over the descriptor's bucket."""
    call("pxb_pipeline_train_step", ctypes.byref(desc), _stream())


def mse_loss(output_ids: torch.Tensor, act: torch.Tensor, target: torch.Tensor, seed: torch.Tensor,
             loss_out: torch.Tensor | None) -> None:
    call("pxb_mse_loss", ctypes.c_int32(output_ids.numel()), ptr(output_ids), ptr(act), ptr(target), ptr(seed),
         ptr(loss_out), _stream())


# ---------------------------------------------------------------------------
# batched products ([num_units, B] unit rows)
# ---------------------------------------------------------------------------
def batched_forward(b: Bucket, x: torch.Tensor, out: torch.Tensor) -> None:
    cap = _bucket(b)
    n, batch = x.shape
    call("pxb_batched_forward", ctypes.c_int64(cap), ptr(b["from_id"]), ptr(b["to_id"]), ptr(b["dead"]),
         ptr(b["weight"]), ptr(x), ctypes.c_int32(batch), ctypes.c_int32(n), ptr(out), _stream())


def batched_backward(b: Bucket, g: torch.Tensor, out: torch.Tensor) -> None:
    cap = _bucket(b)
    n, batch = g.shape
    call("pxb_batched_backward", ctypes.c_int64(cap), ptr(b["from_id"]), ptr(b["to_id"]), ptr(b["dead"]),
         ptr(b["weight"]), ptr(g), ctypes.c_int32(batch), ctypes.c_int32(n), ptr(out), _stream())


def batched_unit_apply(acc: torch.Tensor, out: torch.Tensor, *, mode: int, act_kind: str,
                       act: torch.Tensor | None = None, seed: torch.Tensor | None = None,
                       level: torch.Tensor | None = None, target_level: int = 0,
                       is_input: torch.Tensor | None = None) -> None:
    """Masked apply over [N, B] rows (sum monoid)."""
    n, batch = acc.shape
    call("pxb_batched_unit_apply", ctypes.c_int32(n), ctypes.c_int32(batch), ctypes.c_int32(mode),
         ctypes.c_int32(_lib.act_code(act_kind)), ptr(acc), ptr(act), ptr(seed), ptr(level), ctypes.c_int32(target_level),
         ptr(is_input), ptr(out), _stream())


def batched_loss(kind: int, output_ids: torch.Tensor, batch: int, act: torch.Tensor, target: torch.Tensor,
                 seed: torch.Tensor, loss_per_sample: torch.Tensor, loss_out: torch.Tensor) -> None:
    """Per-sample MSE or softmax cross-entropy; loss_out = the batch mean."""
    call("pxb_batched_loss", ctypes.c_int32(kind), ctypes.c_int32(output_ids.numel()), ptr(output_ids),
         ctypes.c_int32(batch), ptr(act), ptr(target), ptr(seed), ptr(loss_per_sample), ptr(loss_out), _stream())


def batch_mean(x: torch.Tensor, out: torch.Tensor) -> None:
    """out[u] = mean over the batch of x[u, :] (sample order)."""
    n, batch = x.shape
    call("pxb_batch_mean", ctypes.c_int32(n), ctypes.c_int32(batch), ptr(x), ptr(out), _stream())


def batched_update(b: Bucket, g: torch.Tensor, a: torch.Tensor, opt: _lib.Optimizer) -> None:
    cap = _bucket(b)
    n, batch = g.shape
    call("pxb_batched_update", ctypes.c_int64(cap), ptr(b["from_id"]), ptr(b["to_id"]), ptr(b["dead"]),
         ptr(b["weight"]), ptr(g), ptr(a), ctypes.c_int32(batch), ctypes.c_int32(n), ctypes.byref(opt),
         ptr(b.get("opt/m")), ptr(b.get("opt/v")), ptr(b.get("opt/t")), _stream())


# ---------------------------------------------------------------------------
# growth
# ---------------------------------------------------------------------------
def philox32(seed: torch.Tensor, counter: torch.Tensor) -> torch.Tensor:
    out = torch.empty(seed.shape, dtype=torch.int32, device=seed.device)
    call("pxb_philox32", ctypes.c_int64(seed.numel()), ptr(seed), ptr(counter), ptr(out), _stream())
    return out


def site_seed(network_seed: int, step: int, stream: int, key: int) -> int:
    return int(_lib.lib().pxb_site_seed(network_seed, step, stream, key))


def propose_per_unit(num_units: int, proposals: int, network_seed: int, step: int, *, dst_lo: int, dst_n: int,
                     score_kind: int, level: torch.Tensor, grad: torch.Tensor | None = None,
                     act: torch.Tensor | None = None, pruned: torch.Tensor | None = None, max_level_gap: int = 1,
                     direction: int = 0, allow_self_loops: bool = False, bucket_level: int = -1,
                     src_level_bound: int = 0, step_dev: torch.Tensor | None = None,
                     out: tuple[torch.Tensor, torch.Tensor, torch.Tensor] | None = None
                     ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    total = num_units * proposals
    dev = level.device
    if out is None:
        out = (torch.empty(total, dtype=torch.int32, device=dev), torch.empty(total, dtype=torch.int32, device=dev),
               torch.empty(total, dtype=torch.float32, device=dev))
    src, dst, score = out
    call("pxb_propose_per_unit", ctypes.c_int32(num_units), ctypes.c_int32(proposals),
         ctypes.c_uint64(network_seed), ctypes.c_int32(step), ctypes.c_int32(dst_lo), ctypes.c_int32(dst_n),
         ctypes.c_int32(score_kind), ptr(grad), ptr(act), ptr(level), ptr(pruned), ctypes.c_int32(max_level_gap),
         ctypes.c_int32(direction), ctypes.c_int32(1 if allow_self_loops else 0), ctypes.c_int32(bucket_level),
         ctypes.c_int32(src_level_bound), ptr(step_dev), ptr(src), ptr(dst), ptr(score), _stream())
    return src, dst, score


def _window_args(level, pruned, max_level_gap, direction, allow_self_loops, bucket_level, src_level_bound):
    return (ptr(level), ptr(pruned), ctypes.c_int32(max_level_gap), ctypes.c_int32(direction),
            ctypes.c_int32(1 if allow_self_loops else 0), ctypes.c_int32(bucket_level), ctypes.c_int32(src_level_bound))


def propose_global(proposals: int, network_seed: int, step: int, num_units: int, *, src_lo: int, src_n: int,
                   dst_lo: int, dst_n: int, score_kind: int, level: torch.Tensor, grad: torch.Tensor | None = None,
                   act: torch.Tensor | None = None, pruned: torch.Tensor | None = None, max_level_gap: int = 1,
                   direction: int = 0, allow_self_loops: bool = False, bucket_level: int = -1,
                   src_level_bound: int = 0, step_dev: torch.Tensor | None = None,
                   out: tuple | None = None) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    dev = level.device
    if out is None:
        out = (torch.empty(proposals, dtype=torch.int32, device=dev),
               torch.empty(proposals, dtype=torch.int32, device=dev),
               torch.empty(proposals, dtype=torch.float32, device=dev))
    src, dst, score = out
    call("pxb_propose_global", ctypes.c_int32(proposals), ctypes.c_uint64(network_seed), ctypes.c_int32(step),
         ctypes.c_int32(num_units), ctypes.c_int32(src_lo), ctypes.c_int32(src_n), ctypes.c_int32(dst_lo),
         ctypes.c_int32(dst_n), ctypes.c_int32(score_kind), ptr(grad), ptr(act),
         *_window_args(level, pruned, max_level_gap, direction, allow_self_loops, bucket_level, src_level_bound),
         ptr(step_dev), ptr(src), ptr(dst), ptr(score), _stream())
    return src, dst, score


def pair_score(form: int, *, x_src: torch.Tensor | None = None, x_dst: torch.Tensor | None = None, a: int = 0,
               b: int = 0, m: int = 1, c: int = 0, scale: float = 1.0) -> _lib.PairScore:
    """A `pxb_pair_score` (the caller keeps x_src / x_dst alive)."""
    return _lib.PairScore(form, ptr(x_src), ptr(x_dst), a, b, m, c, scale)


def unit_importance(num_units: int, form: _lib.PairScore, *, pruned: torch.Tensor | None = None,
                    level: torch.Tensor | None = None, mask_kind: int = 0, bucket: int = 0, max_level_gap: int = 1,
                    direction: int = 0, out: torch.Tensor | None = None, device=None) -> torch.Tensor:
    if out is None:
        out = torch.empty(num_units, dtype=torch.float32, device=device if device is not None else level.device)
    call("pxb_unit_importance", ctypes.c_int32(num_units), ctypes.byref(form), ptr(pruned), ptr(level),
         ctypes.c_int32(mask_kind), ctypes.c_int32(bucket), ctypes.c_int32(max_level_gap), ctypes.c_int32(direction),
         ptr(out), _stream())
    return out


def propose_grid(num_units: int, grids: int, rows: int, cols: int, score: _lib.PairScore, *, level: torch.Tensor,
                 row_ids: torch.Tensor | None = None, col_ids: torch.Tensor | None = None,
                 per_grid_bucket: bool = False, pruned: torch.Tensor | None = None, max_level_gap: int = 1,
                 direction: int = 0, allow_self_loops: bool = False, src_level_bound: int = 0,
                 out: tuple | None = None) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    n = grids * rows * cols
    dev = level.device
    if out is None:
        out = (torch.empty(n, dtype=torch.int32, device=dev), torch.empty(n, dtype=torch.int32, device=dev),
               torch.empty(n, dtype=torch.float32, device=dev))
    src, dst, sc = out
    call("pxb_propose_grid", ctypes.c_int32(num_units), ctypes.c_int32(grids), ctypes.c_int32(rows),
         ctypes.c_int32(cols), ptr(row_ids), ptr(col_ids), ctypes.c_int32(1 if per_grid_bucket else 0),
         ctypes.byref(score), ptr(level), ptr(pruned), ctypes.c_int32(max_level_gap), ctypes.c_int32(direction),
         ctypes.c_int32(1 if allow_self_loops else 0), ctypes.c_int32(src_level_bound), ptr(src), ptr(dst), ptr(sc),
         _stream())
    return src, dst, sc


def lowest_keys(b: Bucket, base: int, score: torch.Tensor, slot: torch.Tensor) -> None:
    cap = _bucket(b)
    call("pxb_lowest_keys", ctypes.c_int64(cap), ptr(b["dead"]), ptr(b["weight"]), ctypes.c_int64(base), ptr(score),
         ptr(slot), _stream())


def prune_selected(b: Bucket, k: int, idx: torch.Tensor, score: torch.Tensor, base: int, num_units: int, *,
                   free_bitmap: torch.Tensor | None = None, bitmap_level: torch.Tensor | None = None) -> None:
    cap = _bucket(b)
    call("pxb_prune_selected", ctypes.c_int64(k), ptr(idx), ptr(score), ctypes.c_int64(base), ctypes.c_int64(cap),
         ptr(b["from_id"]), ptr(b["dead"]), ctypes.c_int32(num_units), ptr(free_bitmap), ptr(bitmap_level), _stream())


# -- unit lifecycle --------------------------------------------------------
def unit_columns(cols: Sequence[tuple[torch.Tensor, float | int | bool]]) -> _lib.UnitColumns:
    """A `pxb_unit_columns` of (column, default) pairs (4-byte float/int32
    or 1-byte columns); the caller keeps the columns alive."""
    import struct as _struct

    if len(cols) > _lib.MAX_UNIT_COLUMNS:
        raise ValueError(f"unit_columns: at most {_lib.MAX_UNIT_COLUMNS} columns, got {len(cols)}")
    out = _lib.UnitColumns()
    out.count = len(cols)
    for k, (col, default) in enumerate(cols):
        out.cols[k] = col.data_ptr()
        if col.dtype == torch.float32:
            out.bytes[k], out.defaults[k] = 4, _struct.unpack("<I", _struct.pack("<f", float(default)))[0]
        elif col.dtype == torch.int32:
            out.bytes[k], out.defaults[k] = 4, int(default) & 0xFFFFFFFF
        elif col.dtype in (torch.uint8, torch.bool, torch.int8):
            out.bytes[k], out.defaults[k] = 1, int(default) & 0xFF
        else:
            raise ValueError(f"unit_columns: unsupported column dtype {col.dtype}")
    return out


def unit_update(kind: int, field: torch.Tensor, *, src: torch.Tensor | None = None, a: float = 1.0, b: float = 0.0,
                pruned: torch.Tensor | None = None) -> None:
    call("pxb_unit_update", ctypes.c_int32(field.numel()), ctypes.c_int32(kind), ptr(field), ptr(src), ctypes.c_float(a),
         ctypes.c_float(b), ptr(pruned), _stream())


def unit_quantile_scratch(n: int) -> int:
    return query_size("pxb_unit_quantile_scratch_bytes", ctypes.c_int32(n))


def unit_quantile(field: torch.Tensor, q: float, out: torch.Tensor, *, pruned: torch.Tensor | None = None,
                  exempt: torch.Tensor | None = None, scratch: torch.Tensor | None = None) -> torch.Tensor:
    n = field.numel()
    need = unit_quantile_scratch(n)
    if scratch is None or scratch.numel() < need:
        scratch = torch.empty(max(need, 1), dtype=torch.uint8, device=field.device)
    call("pxb_unit_quantile", ctypes.c_int32(n), ptr(field), ptr(pruned), ptr(exempt), ctypes.c_float(q), ptr(out),
         ptr(scratch), ctypes.c_size_t(scratch.numel()), _stream())
    return out


def unit_prune(field: torch.Tensor, threshold: torch.Tensor, pruned: torch.Tensor, doomed: torch.Tensor,
               reset: _lib.UnitColumns, *, exempt: torch.Tensor | None = None) -> None:
    call("pxb_unit_prune", ctypes.c_int32(field.numel()), ptr(field), ptr(threshold), ptr(exempt), ptr(pruned),
         ptr(doomed), ctypes.byref(reset), _stream())


def kill_unit_edges(b: Bucket, doomed: torch.Tensor, *, free_bitmap: torch.Tensor | None = None,
                    bitmap_level: torch.Tensor | None = None) -> None:
    cap = _bucket(b)
    call("pxb_kill_unit_edges", ctypes.c_int64(cap), ptr(b["from_id"]), ptr(b["to_id"]), ptr(b["dead"]),
         ctypes.c_int32(doomed.numel()), ptr(doomed), ptr(free_bitmap), ptr(bitmap_level), _stream())


def unit_add(spawn: _lib.UnitSpawn, pruned: torch.Tensor, level: torch.Tensor, reset: _lib.UnitColumns,
             scratch: torch.Tensor, units_added: torch.Tensor, unit_overflow: torch.Tensor) -> None:
    call("pxb_unit_add", ctypes.c_int32(pruned.numel()), ctypes.byref(spawn), ptr(pruned), ptr(level),
         ctypes.byref(reset), ptr(scratch), ptr(units_added), ptr(unit_overflow), _stream())


def conn_rank_scratch(cap: int, num_units: int) -> int:
    return query_size("pxb_conn_rank_scratch_bytes", ctypes.c_int64(cap), ctypes.c_int32(num_units))


def propose_per_conn(b: Bucket, proposals: int, network_seed: int, step: int, num_units: int, *, dst_lo: int,
                     dst_n: int, score_kind: int, level: torch.Tensor, grad: torch.Tensor | None = None,
                     act: torch.Tensor | None = None, pruned: torch.Tensor | None = None, max_level_gap: int = 1,
                     direction: int = 0, allow_self_loops: bool = False, bucket_level: int = -1,
                     src_level_bound: int = 0, step_dev: torch.Tensor | None = None,
                     scratch: torch.Tensor | None = None,
                     out: tuple | None = None) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Per-connection proposals over one (bucket-major) arena `b` (its
    from_id, to_id and dead columns)."""
    cap = _bucket(b, ("from_id", "to_id", "dead"))
    dev = level.device
    total = cap * proposals
    if out is None:
        out = (torch.empty(total, dtype=torch.int32, device=dev), torch.empty(total, dtype=torch.int32, device=dev),
               torch.empty(total, dtype=torch.float32, device=dev))
    if scratch is None:
        scratch = torch.empty(max(conn_rank_scratch(cap, num_units), 1), dtype=torch.uint8, device=dev)
    src, dst, score = out
    call("pxb_propose_per_conn", ctypes.c_int64(cap), ptr(b["from_id"]), ptr(b["to_id"]), ptr(b["dead"]),
         ctypes.c_int32(proposals), ctypes.c_uint64(network_seed), ctypes.c_int32(step), ctypes.c_int32(num_units),
         ctypes.c_int32(dst_lo), ctypes.c_int32(dst_n), ctypes.c_int32(score_kind), ptr(grad), ptr(act),
         *_window_args(level, pruned, max_level_gap, direction, allow_self_loops, bucket_level, src_level_bound),
         ptr(step_dev), ptr(src), ptr(dst), ptr(score), ptr(scratch), ctypes.c_size_t(scratch.numel()), _stream())
    return src, dst, score


def cap_per_level(idx: torch.Tensor, src: torch.Tensor, level: torch.Tensor, num_levels: int, k: int,
                  out: torch.Tensor, count: torch.Tensor, scratch: torch.Tensor) -> None:
    """First k of every level's run of the level-major list `idx` (out filled
    with -1 beyond the winners; count = their number, device)."""
    out.fill_(-1)
    call("pxb_cap_per_level", ctypes.c_int64(idx.numel()), ptr(idx), ptr(src), ptr(level), ctypes.c_int32(num_levels),
         ctypes.c_int64(k), ptr(out), ptr(count), ptr(scratch), _stream())


def resort_order(b: Bucket, num_units: int) -> torch.Tensor:
    """The bucket's slots stably ordered by dead * num_units + from_id."""
    cap = _bucket(b)
    perm = torch.empty(max(cap, 1), dtype=torch.int32, device=b["dead"].device)
    scratch = torch.empty(max(query_size("pxb_resort_order_scratch_bytes", ctypes.c_int64(cap)), 1),
                          dtype=torch.uint8, device=b["dead"].device)
    call("pxb_resort_order", ctypes.c_int64(cap), ptr(b["dead"]), ptr(b["from_id"]), ctypes.c_int32(num_units),
         ptr(perm), ptr(scratch), ctypes.c_size_t(scratch.numel()), _stream())
    return perm[:cap]


def total_order_scratch(n: int, id_bound: int) -> int:
    return query_size("pxb_total_order_scratch_bytes", ctypes.c_int64(n), ctypes.c_int32(id_bound))


def total_order(score: torch.Tensor, src: torch.Tensor, dst: torch.Tensor, id_bound: int,
                perm: torch.Tensor | None = None, scratch: torch.Tensor | None = None) -> torch.Tensor:
    n = score.numel()
    if perm is None:
        perm = torch.empty(n, dtype=torch.int32, device=score.device)
    need = total_order_scratch(n, id_bound)
    if scratch is None or scratch.numel() < need:
        scratch = torch.empty(max(need, 1), dtype=torch.uint8, device=score.device)
    call("pxb_total_order", ctypes.c_int64(n), ptr(score), ptr(src), ptr(dst), ctypes.c_int32(id_bound), ptr(perm),
         ptr(scratch), ctypes.c_size_t(scratch.numel()), _stream())
    return perm


def topk_unique_scratch(n: int, k: int, id_bound: int) -> int:
    return query_size("pxb_topk_unique_scratch_bytes", ctypes.c_int64(n), ctypes.c_int64(k), ctypes.c_int32(id_bound))


def topk_unique(score: torch.Tensor, src: torch.Tensor, id_bound: int, k: int, out: torch.Tensor | None = None,
                scratch: torch.Tensor | None = None) -> torch.Tensor:
    """First min(k, n) of the total order for candidates with distinct src."""
    n = score.numel()
    kk = min(k, n)
    if out is None:
        out = torch.empty(max(kk, 1), dtype=torch.int32, device=score.device)
    need = topk_unique_scratch(n, k, id_bound)
    if scratch is None or scratch.numel() < need:
        scratch = torch.empty(max(need, 1), dtype=torch.uint8, device=score.device)
    call("pxb_topk_unique", ctypes.c_int64(n), ptr(score), ptr(src), ctypes.c_int32(id_bound), ctypes.c_int64(k),
         ptr(out), ptr(scratch), ctypes.c_size_t(scratch.numel()), _stream())
    return out[:kk]


def select_unique_scratch(num_units: int, k: int, num_levels: int, score_kind: int) -> int:
    return query_size("pxb_select_unique_scratch_bytes", ctypes.c_int32(num_units), ctypes.c_int64(k),
                      ctypes.c_int32(num_levels), ctypes.c_int32(score_kind))


def propose_select_unique(num_units: int, network_seed: int, step: int, *, dst_lo: int, dst_n: int, score_kind: int,
                          level: torch.Tensor, k: int, num_levels: int, init_kind: int, init_a: float = 0.0,
                          init_b: float = 0.0, init_salt: int = 0, pruned: torch.Tensor | None = None,
                          max_level_gap: int = 1, direction: int = 0, allow_self_loops: bool = False,
                          src_level_bound: int = 0, step_dev: torch.Tensor | None = None,
                          status: torch.Tensor | None = None, scratch: torch.Tensor | None = None,
                          out: tuple | None = None, shard=None) -> tuple[torch.Tensor, ...] | None:
    """One proposal per unit scored by the site RNG: proposals, the first k of
    the total order listed levels ascending, gathered as the claim's inputs
    (src, dst, init weight, growable). With `shard` (a `_lib.SelectShard`)
    this rank ranks its share of the full bins and stores their winners into
    every rank's columns (`out` is then unused and None is returned)."""
    dev = level.device
    if scratch is None:
        need = select_unique_scratch(num_units, k, num_levels, score_kind)
        scratch = torch.empty(max(need, 1), dtype=torch.uint8, device=dev)
    head = (ctypes.c_int32(num_units), ctypes.c_uint64(network_seed), ctypes.c_int32(step), ctypes.c_int32(dst_lo),
            ctypes.c_int32(dst_n), ctypes.c_int32(score_kind), ptr(level), ptr(pruned),
            ctypes.c_int32(max_level_gap), ctypes.c_int32(direction), ctypes.c_int32(1 if allow_self_loops else 0),
            ctypes.c_int32(src_level_bound), ptr(step_dev), ctypes.c_int64(k), ctypes.c_int32(num_levels),
            ctypes.c_int32(init_kind), ctypes.c_float(init_a), ctypes.c_float(init_b), ctypes.c_uint32(init_salt))
    if shard is not None:
        call("pxb_propose_select_unique_sharded", *head, ctypes.byref(shard), ptr(status), ptr(scratch),
             ctypes.c_size_t(scratch.numel()), _stream())
        return None
    if out is None:
        out = (torch.empty(k, dtype=torch.int32, device=dev), torch.empty(k, dtype=torch.int32, device=dev),
               torch.empty(k, dtype=torch.float32, device=dev), torch.empty(k, dtype=torch.uint8, device=dev))
    s, d, w, g = out
    call("pxb_propose_select_unique", *head, ptr(s), ptr(d), ptr(w), ptr(g), ptr(status), ptr(scratch),
         ctypes.c_size_t(scratch.numel()), _stream())
    return s, d, w, g


def select_shard(rank: int, world: int, blocks: int, columns: list) -> "_lib.SelectShard":
    """The `pxb_select_shard` of a shared selection: `columns[q]` is rank q's
    (src, dst, weight, growable) device pointers, each column holding
    `blocks` lists of k entries."""
    if not 1 <= world <= _lib.SELECT_MAX_WORLD or len(columns) != world:
        raise ValueError(f"a shared selection takes 1..{_lib.SELECT_MAX_WORLD} ranks' columns, got {len(columns)}")
    sh = _lib.SelectShard()
    sh.rank, sh.world, sh.blocks = int(rank), int(world), int(blocks)
    for q, (s, d, w, g) in enumerate(columns):
        sh.src_out[q], sh.dst_out[q], sh.weight_out[q], sh.growable_out[q] = int(s), int(d), int(w), int(g)
    return sh


def select_take(k: int, blocks: int, step_dev: torch.Tensor | None, cols: tuple, out: tuple) -> None:
    """List (step mod blocks) of the four columns `cols` (blocks * k entries
    each) copied into `out` (the claim's inputs), in one launch."""
    s, d, w, g = cols
    so, do, wo, go = out
    call("pxb_select_take", ctypes.c_int64(k), ctypes.c_int32(blocks), ptr(step_dev), ptr(s), ptr(d), ptr(w), ptr(g),
         ptr(so), ptr(do), ptr(wo), ptr(go), _stream())


def select_step_scratch(n: int, k: int) -> int:
    return query_size("pxb_select_step_scratch_bytes", ctypes.c_int64(n), ctypes.c_int64(k))


def select_step(perm: torch.Tensor, score: torch.Tensor, src: torch.Tensor, level: torch.Tensor, k: int,
                win: torch.Tensor | None = None, scratch: torch.Tensor | None = None,
                num_levels: int | None = None) -> torch.Tensor:
    n = perm.numel()
    kk = min(k, n)
    if win is None:
        win = torch.empty(max(kk, 1), dtype=torch.int32, device=perm.device)
    need = select_step_scratch(n, k)
    if scratch is None or scratch.numel() < need:
        scratch = torch.empty(max(need, 1), dtype=torch.uint8, device=perm.device)
    if num_levels is None:
        num_levels = int(level.max().item()) + 1 if level.numel() else 1
    call("pxb_select_step", ctypes.c_int64(n), ptr(perm), ptr(score), ptr(src), ptr(level),
         ctypes.c_int32(num_levels), ctypes.c_int64(k), ptr(win), None, ptr(scratch), ctypes.c_size_t(scratch.numel()),
         _stream())
    return win[:kk]


def gather_winners(win: torch.Tensor, count: int, k: int, src: torch.Tensor, dst: torch.Tensor,
                   score: torch.Tensor, *, init_kind: int, init_a: float = 0.0, init_b: float = 0.0,
                   init_salt: int = 0, out: tuple | None = None) -> tuple[torch.Tensor, ...]:
    dev = src.device
    if out is None:
        out = (torch.empty(k, dtype=torch.int32, device=dev), torch.empty(k, dtype=torch.int32, device=dev),
               torch.empty(k, dtype=torch.float32, device=dev), torch.empty(k, dtype=torch.uint8, device=dev))
    s, d, w, g = out
    call("pxb_gather_winners", ctypes.c_int64(k), ctypes.c_int64(count), ptr(win), ptr(src), ptr(dst), ptr(score),
         ctypes.c_int32(init_kind), ctypes.c_float(init_a), ctypes.c_float(init_b), ctypes.c_uint32(init_salt),
         ptr(s), ptr(d), ptr(w), ptr(g), _stream())
    return s, d, w, g


# ---------------------------------------------------------------------------
# slot claim
# ---------------------------------------------------------------------------
def claim_scratch(cap: int, k: int, num_levels: int) -> int:
    return query_size("pxb_claim_scratch_bytes", ctypes.c_int64(cap), ctypes.c_int64(k), ctypes.c_int32(num_levels))


class ClaimWorkspace:
    """Caller-owned scratch for one claim (allocated once, reused per step)."""

    def __init__(self, cap: int, k: int, num_levels: int, device: torch.device) -> None:
        self.cap, self.k, self.num_levels = cap, k, num_levels
        self.scratch = torch.empty(max(claim_scratch(cap, k, num_levels), 1), dtype=torch.uint8, device=device)
        self.level_counts = torch.zeros(num_levels, dtype=torch.int32, device=device)
        self.counts = torch.zeros(4, dtype=torch.int32, device=device)
        self.overflowed = torch.zeros(max(k, 1), dtype=torch.uint8, device=device)


def claim_prepare(mode: int, b: Bucket, unit_level: torch.Tensor, tail_start: torch.Tensor | None,
                  ws: ClaimWorkspace, *, shard_base: int = 0, free_bitmap: torch.Tensor | None = None
                  ) -> torch.Tensor:
    cap = _bucket(b)
    call("pxb_claim_prepare", ctypes.c_int32(mode), ctypes.c_int64(cap), ptr(b["from_id"]), ptr(b["dead"]),
         ptr(unit_level), ctypes.c_int32(unit_level.numel()), ctypes.c_int32(ws.num_levels),
         ctypes.c_int64(shard_base), ptr(tail_start), ptr(free_bitmap), ctypes.c_int64(ws.k), ptr(ws.level_counts),
         ptr(ws.scratch), ctypes.c_size_t(ws.scratch.numel()), _stream())
    return ws.level_counts


def claim_commit(mode: int, b: Bucket, unit_level: torch.Tensor, tail_start: torch.Tensor | None,
                 ws: ClaimWorkspace, src: torch.Tensor, dst: torch.Tensor, weight: torch.Tensor,
                 growable: torch.Tensor, *, max_new: int = -1, shard_base: int = 0, global_cap: int | None = None,
                 level_before: torch.Tensor | None = None, level_totals: torch.Tensor | None = None,
                 extra: Mapping[str, torch.Tensor] | None = None, free_bitmap: torch.Tensor | None = None,
                 placed: torch.Tensor | None = None, committed: torch.Tensor | None = None) -> None:
    cap = _bucket(b)
    k = src.numel()
    if k != ws.k:
        raise ValueError(f"claim workspace sized for {ws.k} candidates, got {k}")
    names = sorted(extra or {})
    n_extra = len(names)
    cols = (ctypes.c_void_p * 8)(*[b[nm].data_ptr() for nm in names])
    nbytes = (ctypes.c_int32 * 8)(*[b[nm].element_size() for nm in names])
    vals = (ctypes.c_void_p * 8)(*[extra[nm].data_ptr() for nm in names])  # type: ignore[index]
    call("pxb_claim_commit", ctypes.c_int32(mode), ctypes.c_int64(cap), ptr(b["from_id"]), ptr(b["to_id"]),
         ptr(b["dead"]), ptr(b["weight"]), ptr(unit_level), ctypes.c_int32(unit_level.numel()),
         ctypes.c_int32(ws.num_levels), ctypes.c_int64(shard_base),
         ctypes.c_int64(cap + shard_base if global_cap is None else global_cap), ptr(tail_start), ctypes.c_int64(k),
         ptr(src), ptr(dst), ptr(weight), ptr(growable), ctypes.c_int64(max_new), ptr(level_before),
         ptr(level_totals), ptr(free_bitmap), ctypes.c_int32(n_extra),
         ctypes.cast(cols, ctypes.c_void_p) if n_extra else None,
         ctypes.cast(nbytes, ctypes.c_void_p) if n_extra else None,
         ctypes.cast(vals, ctypes.c_void_p) if n_extra else None, ptr(ws.counts), ptr(ws.overflowed), ptr(placed),
         ptr(committed), ptr(ws.scratch), ctypes.c_size_t(ws.scratch.numel()), _stream())


def growth_flags(counts: torch.Tensor, *, reset: bool, grown: torch.Tensor | None,
                 overflow: torch.Tensor | None, needs_resort: torch.Tensor | None) -> None:
    """grown (+)= counts[0]; overflow |= counts[1] > 0; needs_resort |= counts[3] > 0."""
    for t, dt in ((grown, torch.int32), (overflow, torch.bool), (needs_resort, torch.bool)):
        if t is not None:
            _check(t, dt, 1, "growth_flags")
    call("pxb_growth_flags", ptr(counts), ctypes.c_int32(1 if reset else 0), ptr(grown), ptr(overflow),
         ptr(needs_resort), _stream())


def dedupe_scratch(n: int) -> int:
    return query_size("pxb_dedupe_scratch_bytes", ctypes.c_int64(n))


def dedupe(src: torch.Tensor, dst: torch.Tensor, score: torch.Tensor, *, buckets: Sequence[Bucket] = (),
           step_repeats: bool = False, live_hit: torch.Tensor | None = None, scratch: torch.Tensor | None = None,
           combine_hits=None) -> None:
    """Veto (score = -inf) candidates whose pair is live in any of `buckets`
    and, with `step_repeats`, every copy of a pair but its first in the
    stable order of -score. `combine_hits(live_hit)` may OR the live marks
    across ranks between the marks and the veto (Scheme-A)."""
    n = src.numel()
    if scratch is None:
        scratch = torch.empty(max(dedupe_scratch(n), 1), dtype=torch.uint8, device=src.device)
    call("pxb_pair_table_build", ctypes.c_int64(n), ptr(src), ptr(dst), ptr(scratch),
         ctypes.c_size_t(scratch.numel()), _stream())
    if buckets:
        if live_hit is None:
            live_hit = torch.empty(n, dtype=torch.uint8, device=src.device)
        for b in buckets:
            call("pxb_pair_table_mark", ctypes.c_int64(n), ctypes.c_int64(_bucket(b)), ptr(b["from_id"]),
                 ptr(b["to_id"]), ptr(b["dead"]), ptr(live_hit), ptr(scratch), ctypes.c_size_t(scratch.numel()),
                 _stream())
        if combine_hits is not None:
            combine_hits(live_hit)
    call("pxb_dedupe_apply", ctypes.c_int64(n), ptr(score), ptr(live_hit if buckets else None),
         ctypes.c_int32(1 if step_repeats else 0), ptr(scratch), ctypes.c_size_t(scratch.numel()), _stream())


def count_dead(b: Bucket, out: torch.Tensor) -> None:
    cap = _bucket(b)
    call("pxb_count_dead", ctypes.c_int64(cap), ptr(b["dead"]), ptr(out), _stream())


def free_bitmap_build(mode: int, b: Bucket, unit_level: torch.Tensor, tail_start: torch.Tensor | None,
                      num_levels: int, *, shard_base: int = 0, out: torch.Tensor | None = None) -> torch.Tensor:
    """Per-domain free-slot bitmaps of a bucket (int32 view of uint32 words)."""
    cap = _bucket(b)
    rows = 1 if (mode & ~_lib.CLAIM_LEVEL_MAJOR) == _lib.CLAIM_TOPOLOGICAL else num_levels
    words = (cap + 31) // 32
    if out is None:
        out = torch.zeros(rows * max(words, 1), dtype=torch.int32, device=b["dead"].device)
    call("pxb_free_bitmap_build", ctypes.c_int32(mode), ctypes.c_int64(cap), ptr(b["from_id"]), ptr(b["dead"]),
         ptr(unit_level), ctypes.c_int32(unit_level.numel()), ctypes.c_int32(num_levels), ctypes.c_int64(shard_base),
         ptr(tail_start), ptr(out), _stream())
    return out


def mirror_forward(m, act: torch.Tensor, acc: torch.Tensor, *, acc_fixed: torch.Tensor | None = None,
                   monoid: str = "sum", prune_kind: int = 0,
                   threshold: float = 0.0, unit_threshold: torch.Tensor | None = None,
                   dead: torch.Tensor | None = None, free_bitmap: torch.Tensor | None = None, bitmap_words: int = 0,
                   bitmap_level: torch.Tensor | None = None, pruned_count: torch.Tensor | None = None) -> None:
    """Mirror sweep; for sum, `acc_fixed` (int64, zeroed) receives the exact
    fixed-point sum and `acc` only non-finite or huge products."""
    if acc_fixed is not None:
        _check(acc_fixed, torch.int64, acc.numel(), "mirror_forward acc_fixed")
    call("pxb_mirror_forward", ctypes.byref(m.struct), ptr(act), ctypes.c_int32(_lib.MONOID[monoid]), ptr(acc),
         ptr(acc_fixed), ctypes.c_int32(prune_kind), ctypes.c_float(threshold), ptr(unit_threshold), ptr(dead), ptr(free_bitmap),
         ctypes.c_int64(bitmap_words), ptr(bitmap_level), ptr(pruned_count), _stream())


def mirror_insert(m, src: torch.Tensor, dst: torch.Tensor, weight: torch.Tensor, placed: torch.Tensor) -> None:
    call("pxb_mirror_insert", ctypes.byref(m.struct), ctypes.c_int64(src.numel()), ptr(src), ptr(dst), ptr(weight),
         ptr(placed), _stream())


def host_device_pointer(t: torch.Tensor) -> int:
    """The device address of a pinned host tensor (kernels read and write it
    over the bus)."""
    out = ctypes.c_void_p()
    try:
        call("pxb_host_device_pointer", ctypes.c_void_p(t.data_ptr()), ctypes.byref(out))
    except _lib.PxbError:
        # a block of the caching host allocator: under unified addressing
        # the host address is the device address
        return int(t.data_ptr())
    return int(out.value)


def scatter_inputs(ids: torch.Tensor, src_ptr: int, act: torch.Tensor) -> None:
    """act[ids[i]] = src[i], src a device address (pinned host memory through
    `host_device_pointer`, or device memory)."""
    call("pxb_scatter_inputs", ctypes.c_int32(ids.numel()), ptr(ids), ctypes.c_void_p(src_ptr), ptr(act), _stream())


def flags_out(grown: torch.Tensor | None, overflow: torch.Tensor | None, out_ptr: int) -> None:
    """out[0] = grown, out[1] = overflow as int32, out a device address."""
    call("pxb_flags_out", ptr(grown), ptr(overflow), ctypes.c_void_p(out_ptr), _stream())
