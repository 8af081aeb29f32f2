"""ctypes binding of libpxb.so (the C ABI declared in include/pxb.h).

Every entry point is wrapped so a non-zero status raises `PxbError` with the
library's own message. Loading fails loudly: there is no CPU fallback behind
these calls, so a missing or unbuildable library is an error, never a silent
switch to another implementation.
"""

from __future__ import annotations

import ctypes
import functools
import os
import pathlib
from collections.abc import Callable
from typing import Any

_PKG = pathlib.Path(__file__).resolve().parent
# the in-tree build, or another build of the same sources (PLASTAX_B200_LIB)
LIB_PATH = pathlib.Path(os.environ.get("PLASTAX_B200_LIB", str(_PKG / "libpxb.so")))

c_i32 = ctypes.c_int32
c_i64 = ctypes.c_int64
c_u32 = ctypes.c_uint32
c_u64 = ctypes.c_uint64
c_f32 = ctypes.c_float
c_size = ctypes.c_size_t
c_ptr = ctypes.c_void_p

# constants of include/pxb.h
MONOID = {"sum": 0, "max": 1, "min": 2}
ACT = {"identity": 0, "tanh": 1, "relu": 2, "sigmoid": 3}
PRUNE_NONE, PRUNE_ABS_BELOW, PRUNE_ABS_BELOW_DST, PRUNE_LOWEST_K = 0, 1, 2, 3
LOWK_BINS, LOWK_SHIFT = 65536, 15
LOWK_FINE_BINS, LOWK_FINE_SHIFT = 1 << 24, 7
LOWK_PLAN_SCRATCH = 256
OPT = {"sgd": 0, "momentum": 1, "adam": 2, "rmsprop": 3, "upgd": 4}
SCORE_UNIFORM, SCORE_UNIFORM_Q256, SCORE_GRAD_ACT = 0, 1, 2
INIT_CONST, INIT_DYADIC, INIT_HASH_UNIFORM = 0, 1, 2
CLAIM_PIPELINE, CLAIM_TOPOLOGICAL = 0, 1
CLAIM_LEVEL_MAJOR = 0x100
LOSS_MSE, LOSS_SOFTMAX_CE = 0, 1
MIRROR_TILE = 2048
PEER_MAX_LEVELS = 8
FIXED_FRAC_BITS = 31
PAIR_ABS_PRODUCT, PAIR_PRODUCT, PAIR_MODULAR, PAIR_MODULAR_PREDICATE = 0, 1, 2, 3
UNIT_UPDATE_AFFINE, UNIT_UPDATE_TRACE_ABS, UNIT_UPDATE_TRACE = 0, 1, 2
SPAWN_FIELD_AT_LEAST, SPAWN_ARGMAX = 0, 1
MAX_UNIT_COLUMNS = 16


def act_code(kind) -> int:
    """An apply entry point's activation code: a kind name, or a (kind,
    output kind) pair whose second kind applies to the output units."""
    if isinstance(kind, tuple):
        base, out = kind
        return ACT[base] if out is None else ACT[base] | ((ACT[out] + 1) << 8)
    return ACT[kind]


class Mirror(ctypes.Structure):
    """`pxb_mirror`: the destination-grouped index of one bucket."""

    _fields_ = [
        ("num_units", c_i32), ("chunk_bits", c_i32), ("groups", c_i64), ("entries", c_i64),
        ("gbase", c_ptr), ("gfill", c_ptr), ("word", c_ptr), ("weight", c_ptr), ("slot", c_ptr),
        ("hstack", c_ptr), ("hcount", c_ptr), ("items", c_i64), ("item_begin", c_ptr), ("item_end", c_ptr),
        ("item_group", c_ptr), ("ovf_cap", c_i64), ("ovf_count", c_ptr), ("ovf_src", c_ptr), ("ovf_dst", c_ptr),
        ("ovf_slot", c_ptr), ("ovf_weight", c_ptr), ("status", c_ptr), ("ins_count", c_ptr),
        ("defer_pos", c_ptr), ("defer_count", c_ptr), ("defer_seg", c_i64), ("defer_ctas", c_i32),
        ("sum_frac_bits", c_i32),
    ]


class PeerGroup(ctypes.Structure):
    """`pxb_peer_group`: one rank's view of a Scheme-A group."""

    _fields_ = [
        ("rank", c_i32), ("world", c_i32), ("acc_fixed", c_ptr), ("acc_side", c_ptr), ("act", c_ptr),
        ("flags", c_ptr), ("counts", c_ptr), ("epoch", c_ptr), ("done", c_ptr), ("status", c_ptr),
    ]


class Lowk(ctypes.Structure):
    """`pxb_lowk`: the exact lowest-|w| prune's histogram, plan and lists."""

    _fields_ = [
        ("rank", c_i32), ("world", c_i32), ("k", c_i64), ("list_cap", c_i64), ("slot_base", c_i64),
        ("hist", c_ptr), ("fine", c_ptr), ("plan", c_ptr), ("key", c_ptr), ("level", c_ptr), ("count", c_ptr),
        ("pos", c_ptr),
        ("peer_key", c_ptr), ("peer_level", c_ptr), ("peer_count", c_ptr), ("plan_scratch", c_ptr),
    ]


SELECT_MAX_WORLD = 8


class SelectShard(ctypes.Structure):
    """`pxb_select_shard`: the ranks' winner columns of a shared selection."""

    _fields_ = [
        ("rank", c_i32), ("world", c_i32), ("blocks", c_i32), ("pad", c_i32),
        ("src_out", c_ptr * SELECT_MAX_WORLD), ("dst_out", c_ptr * SELECT_MAX_WORLD),
        ("weight_out", c_ptr * SELECT_MAX_WORLD), ("growable_out", c_ptr * SELECT_MAX_WORLD),
    ]


class PairScore(ctypes.Structure):
    """`pxb_pair_score`: a ScoreAddConn rule's lowered score or importance."""

    _fields_ = [
        ("form", c_i32), ("x_src", c_ptr), ("x_dst", c_ptr), ("a", c_i32), ("b", c_i32), ("m", c_i32),
        ("c", c_i32), ("scale", c_f32),
    ]


class LoopDesc(ctypes.Structure):
    """`pxb_loop_desc`: the buffers of a device-side chunk loop."""

    _fields_ = [
        ("counter", c_ptr), ("count", c_i32), ("in_chunk", c_ptr), ("in_cols", c_i32), ("in_buf", c_ptr),
        ("tgt_chunk", c_ptr), ("tgt_cols", c_i32), ("tgt_buf", c_ptr), ("loss", c_ptr), ("loss_rec", c_ptr),
        ("act", c_ptr), ("out_ids", c_ptr), ("n_out", c_i32), ("out_rec", c_ptr), ("overflow", c_ptr),
        ("needs_resort", c_ptr), ("resorts", c_i32), ("status", c_ptr),
    ]


class UnitColumns(ctypes.Structure):
    """`pxb_unit_columns`: unit columns with their default bit patterns."""

    _fields_ = [("count", c_i32), ("cols", c_ptr * 16), ("bytes", c_i32 * 16), ("defaults", ctypes.c_uint32 * 16)]


class UnitSpawn(ctypes.Structure):
    """`pxb_unit_spawn`: an add_unit rule's lowered form."""

    _fields_ = [("kind", c_i32), ("field", c_ptr), ("threshold", c_f32), ("offset", c_i32), ("max_level", c_i32),
                ("init_dst", c_ptr), ("init_src", c_ptr), ("init_scale", c_f32)]


class PxbError(RuntimeError):
    """A libpxb entry point returned a non-zero status."""


class Optimizer(ctypes.Structure):
    """`pxb_optimizer`: the optimizer bundle's kind and hyper-parameters."""

    _fields_ = [
        ("kind", c_i32),
        ("lr", c_f32),
        ("b1", c_f32),
        ("b2", c_f32),
        ("eps", c_f32),
        ("weight_decay", c_f32),
        ("unit_scale", c_ptr),
    ]


class PipelineTrain(ctypes.Structure):
    """`pxb_pipeline_train`: the fused pipeline training step's bucket, unit
    columns, loss and optimizer."""

    _fields_ = [
        ("cap", c_i64),
        ("from_id", c_ptr),
        ("to_id", c_ptr),
        ("dead", c_ptr),
        ("weight", c_ptr),
        ("opt_m", c_ptr),
        ("opt_v", c_ptr),
        ("opt_t", c_ptr),
        ("num_units", c_i32),
        ("act", c_ptr),
        ("grad", c_ptr),
        ("seed", c_ptr),
        ("roles", c_ptr),
        ("pruned", c_ptr),
        ("fwd_act", c_i32),
        ("bwd_act", c_i32),
        ("num_outputs", c_i32),
        ("target_of", c_ptr),
        ("output_ids", c_ptr),
        ("target", c_ptr),
        ("loss", c_ptr),
        ("update_grad", c_ptr),
        ("opt", Optimizer),
        ("scratch", c_ptr),
        ("tail_start", c_ptr),
    ]


# name -> (restype, argtypes); every int-returning entry point is checked.
_SIGNATURES: dict[str, tuple[Any, list[Any]]] = {
    "pxb_abi_version": (c_i32, []),
    "pxb_last_error": (ctypes.c_char_p, []),
    "pxb_sm_count": (c_i32, [c_ptr]),
    "pxb_set_device": (c_i32, [c_i32]),
    "pxb_get_device": (c_i32, [c_ptr]),
    "pxb_clear_accumulators": (c_i32, [c_i64, c_f32, c_ptr, c_ptr, c_ptr]),
    "pxb_fill_f32": (c_i32, [c_i64, c_f32, c_ptr, c_ptr]),
    "pxb_forward_accumulate": (c_i32, [c_i64, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_i32, c_i32, c_ptr, c_ptr]),
    "pxb_forward_prune": (
        c_i32,
        [c_i64, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_i32, c_i32, c_ptr, c_i32, c_f32, c_ptr, c_ptr, c_i32, c_ptr,
         c_ptr, c_ptr, c_ptr],
    ),
    "pxb_prune_conn": (
        c_i32, [c_i64, c_ptr, c_ptr, c_ptr, c_ptr, c_i32, c_i32, c_f32, c_ptr, c_ptr, c_i32, c_ptr, c_ptr, c_ptr, c_ptr]),
    "pxb_backward_accumulate": (c_i32, [c_i64, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_i32, c_i32, c_ptr, c_ptr]),
    "pxb_backward_update": (
        c_i32,
        [c_i64, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_i32, c_ptr, ctypes.POINTER(Optimizer), c_ptr, c_ptr,
         c_ptr, c_ptr],
    ),
    "pxb_unit_apply": (
        c_i32,
        [c_i32, c_i32, c_i32, c_i32, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_i32, c_ptr, c_ptr, c_ptr, c_ptr],
    ),
    "pxb_mse_loss": (c_i32, [c_i32, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr]),
    "pxb_batched_forward": (c_i32, [c_i64, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_i32, c_i32, c_ptr, c_ptr]),
    "pxb_batched_backward": (c_i32, [c_i64, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_i32, c_i32, c_ptr, c_ptr]),
    "pxb_batched_update": (
        c_i32,
        [c_i64, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_i32, c_i32, ctypes.POINTER(Optimizer), c_ptr, c_ptr,
         c_ptr, c_ptr],
    ),
    "pxb_philox32": (c_i32, [c_i64, c_ptr, c_ptr, c_ptr, c_ptr]),
    "pxb_site_seed": (c_u64, [c_u64, c_u32, c_u32, c_u32]),
    "pxb_propose_per_unit": (
        c_i32,
        [c_i32, c_i32, c_u64, c_i32, c_i32, c_i32, c_i32, c_ptr, c_ptr, c_ptr, c_ptr, c_i32, c_i32, c_i32, c_i32,
         c_i32, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr],
    ),
    "pxb_total_order_scratch_bytes": (c_i32, [c_i64, c_i32, ctypes.POINTER(c_size)]),
    "pxb_total_order": (c_i32, [c_i64, c_ptr, c_ptr, c_ptr, c_i32, c_ptr, c_ptr, c_size, c_ptr]),
    "pxb_total_order_noalloc": (c_i32, [c_i64, c_ptr, c_ptr, c_ptr, c_i32, c_ptr, c_ptr]),
    "pxb_topk_unique_scratch_bytes": (c_i32, [c_i64, c_i64, c_i32, ctypes.POINTER(c_size)]),
    "pxb_topk_unique": (c_i32, [c_i64, c_ptr, c_ptr, c_i32, c_i64, c_ptr, c_ptr, c_size, c_ptr]),
    "pxb_select_step_scratch_bytes": (c_i32, [c_i64, c_i64, ctypes.POINTER(c_size)]),
    "pxb_select_step": (c_i32, [c_i64, c_ptr, c_ptr, c_ptr, c_ptr, c_i32, c_i64, c_ptr, c_ptr, c_ptr, c_size, c_ptr]),
    "pxb_gather_winners": (
        c_i32,
        [c_i64, c_i64, c_ptr, c_ptr, c_ptr, c_ptr, c_i32, c_f32, c_f32, c_u32, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr],
    ),
    "pxb_claim_scratch_bytes": (c_i32, [c_i64, c_i64, c_i32, ctypes.POINTER(c_size)]),
    "pxb_claim_prepare": (
        c_i32,
        [c_i32, c_i64, c_ptr, c_ptr, c_ptr, c_i32, c_i32, c_i64, c_ptr, c_ptr, c_i64, c_ptr, c_ptr, c_size, c_ptr],
    ),
    "pxb_claim_commit": (
        c_i32,
        [c_i32, c_i64, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_i32, c_i32, c_i64, c_i64, c_ptr, c_i64, c_ptr, c_ptr,
         c_ptr, c_ptr, c_i64, c_ptr, c_ptr, c_ptr, c_i32, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr,
         c_size, c_ptr],
    ),
    "pxb_free_bitmap_build": (c_i32, [c_i32, c_i64, c_ptr, c_ptr, c_ptr, c_i32, c_i32, c_i64, c_ptr, c_ptr, c_ptr]),
    "pxb_propose_global": (c_i32, [c_i32, ctypes.c_uint64, c_i32, c_i32, c_i32, c_i32, c_i32, c_i32, c_i32, c_ptr,
                                   c_ptr, c_ptr, c_ptr, c_i32, c_i32, c_i32, c_i32, c_i32, c_ptr, c_ptr, c_ptr,
                                   c_ptr, c_ptr]),
    "pxb_conn_rank_scratch_bytes": (c_i32, [c_i64, c_i32, ctypes.POINTER(c_size)]),
    "pxb_propose_per_conn": (c_i32, [c_i64, c_ptr, c_ptr, c_ptr, c_i32, ctypes.c_uint64, c_i32, c_i32, c_i32, c_i32,
                                     c_i32, c_ptr, c_ptr, c_ptr, c_ptr, c_i32, c_i32, c_i32, c_i32, c_i32, c_ptr,
                                     c_ptr, c_ptr, c_ptr, c_ptr, c_size, c_ptr]),
    "pxb_cap_per_level": (c_i32, [c_i64, c_ptr, c_ptr, c_ptr, c_i32, c_i64, c_ptr, c_ptr, c_ptr, c_ptr]),
    "pxb_resort_order_scratch_bytes": (c_i32, [c_i64, ctypes.POINTER(c_size)]),
    "pxb_resort_order": (c_i32, [c_i64, c_ptr, c_ptr, c_i32, c_ptr, c_ptr, c_size, c_ptr]),
    "pxb_select_unique_scratch_bytes": (c_i32, [c_i32, c_i64, c_i32, c_i32, ctypes.POINTER(c_size)]),
    "pxb_propose_select_unique": (
        c_i32, [c_i32, ctypes.c_uint64, c_i32, c_i32, c_i32, c_i32, c_ptr, c_ptr, c_i32, c_i32, c_i32, c_i32,
                c_ptr, c_i64, c_i32, c_i32, c_f32, c_f32, ctypes.c_uint32, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr,
                c_ptr, c_size, c_ptr]),
    "pxb_propose_select_unique_sharded": (
        c_i32, [c_i32, ctypes.c_uint64, c_i32, c_i32, c_i32, c_i32, c_ptr, c_ptr, c_i32, c_i32, c_i32, c_i32,
                c_ptr, c_i64, c_i32, c_i32, c_f32, c_f32, ctypes.c_uint32, c_ptr, c_ptr, c_ptr, c_size, c_ptr]),
    "pxb_scatter_inputs": (c_i32, [c_i32, c_ptr, c_ptr, c_ptr, c_ptr]),
    "pxb_flags_out": (c_i32, [c_ptr, c_ptr, c_ptr, c_ptr]),
    "pxb_host_device_pointer": (c_i32, [c_ptr, ctypes.POINTER(c_ptr)]),
    "pxb_select_take": (c_i32, [c_i64, c_i32, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr]),
    "pxb_mirror_forward": (
        c_i32, [c_ptr, c_ptr, c_i32, c_ptr, c_ptr, c_i32, c_f32, c_ptr, c_ptr, c_ptr, c_i64, c_ptr, c_ptr, c_ptr]),
    "pxb_mirror_insert": (c_i32, [c_ptr, c_i64, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr]),
    "pxb_lowk_hist_build": (c_i32, [c_ptr, c_i64, c_ptr, c_ptr, c_ptr]),
    "pxb_lowk_make_plan": (c_i32, [c_ptr, c_ptr]),
    "pxb_mirror_forward_lowk": (c_i32, [c_ptr, c_ptr, c_i32, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_i64, c_ptr, c_ptr]),
    "pxb_mirror_forward_lowk_deferred": (c_i32, [c_ptr, c_ptr, c_i32, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_i64, c_ptr,
                                                 c_ptr]),
    "pxb_mirror_defer_flush": (c_i32, [c_ptr, c_i32, c_ptr, c_ptr, c_ptr, c_i64, c_ptr, c_ptr]),
    "pxb_lowk_select": (c_i32, [c_ptr, c_ptr, c_ptr, c_ptr, c_i64, c_ptr, c_i32, c_ptr, c_ptr, c_ptr]),
    "pxb_lowk_hist_add": (c_i32, [c_ptr, c_i64, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr]),
    "pxb_step_end": (c_i32, [c_ptr, c_ptr, c_ptr, c_ptr]),
    "pxb_growth_flags": (c_i32, [c_ptr, c_i32, c_ptr, c_ptr, c_ptr, c_ptr]),
    "pxb_peer_alloc": (c_i32, [c_size, ctypes.POINTER(c_ptr), c_ptr]),
    "pxb_peer_open": (c_i32, [c_ptr, ctypes.POINTER(c_ptr)]),
    "pxb_peer_close": (c_i32, [c_ptr]),
    "pxb_peer_free": (c_i32, [c_ptr]),
    "pxb_scheme_a_apply": (c_i32, [c_ptr, c_i32, c_i32, c_ptr, c_ptr, c_ptr, c_i32, c_ptr, c_ptr, ctypes.c_uint32,
                                   c_ptr]),
    "pxb_dedupe_scratch_bytes": (c_i32, [c_i64, ctypes.POINTER(c_size)]),
    "pxb_pair_table_build": (c_i32, [c_i64, c_ptr, c_ptr, c_ptr, c_size, c_ptr]),
    "pxb_pair_table_mark": (c_i32, [c_i64, c_i64, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_size, c_ptr]),
    "pxb_dedupe_apply": (c_i32, [c_i64, c_ptr, c_ptr, c_i32, c_ptr, c_size, c_ptr]),
    "pxb_batched_unit_apply": (c_i32, [c_i32, c_i32, c_i32, c_i32, c_ptr, c_ptr, c_ptr, c_ptr, c_i32, c_ptr, c_ptr,
                                       c_ptr]),
    "pxb_batched_loss": (c_i32, [c_i32, c_i32, c_ptr, c_i32, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr]),
    "pxb_batch_mean": (c_i32, [c_i32, c_i32, c_ptr, c_ptr, c_ptr]),
    "pxb_count_dead": (c_i32, [c_i64, c_ptr, c_ptr, c_ptr]),
    "pxb_loop_build": (c_i32, [c_ptr, c_ptr, ctypes.POINTER(c_ptr)]),
    "pxb_loop_launch": (c_i32, [c_ptr, c_ptr]),
    "pxb_loop_destroy": (c_i32, [c_ptr]),
    "pxb_graph_instantiate": (c_i32, [c_ptr, c_i32, ctypes.POINTER(c_ptr)]),
    "pxb_graph_launch": (c_i32, [c_ptr, c_ptr]),
    "pxb_graph_exec_destroy": (c_i32, [c_ptr]),
    "pxb_lowest_keys": (c_i32, [c_i64, c_ptr, c_ptr, c_i64, c_ptr, c_ptr, c_ptr]),
    "pxb_prune_selected": (c_i32, [c_i64, c_ptr, c_ptr, c_i64, c_i64, c_ptr, c_ptr, c_i32, c_ptr, c_ptr, c_ptr]),
    "pxb_unit_update": (c_i32, [c_i32, c_i32, c_ptr, c_ptr, c_f32, c_f32, c_ptr, c_ptr]),
    "pxb_unit_quantile_scratch_bytes": (c_i32, [c_i32, ctypes.POINTER(c_size)]),
    "pxb_unit_quantile": (c_i32, [c_i32, c_ptr, c_ptr, c_ptr, c_f32, c_ptr, c_ptr, c_size, c_ptr]),
    "pxb_unit_prune": (c_i32, [c_i32, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr]),
    "pxb_kill_unit_edges": (c_i32, [c_i64, c_ptr, c_ptr, c_ptr, c_i32, c_ptr, c_ptr, c_ptr, c_ptr]),
    "pxb_unit_add": (c_i32, [c_i32, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr]),
    "pxb_unit_importance": (c_i32, [c_i32, c_ptr, c_ptr, c_ptr, c_i32, c_i32, c_i32, c_i32, c_ptr, c_ptr]),
    "pxb_pipeline_train_max_units": (c_i32, [c_i32]),
    "pxb_pipeline_train_scratch_bytes": (c_i32, [c_i32, ctypes.POINTER(c_size)]),
    "pxb_pipeline_train_step": (c_i32, [c_ptr, c_ptr]),
    "pxb_propose_grid": (c_i32, [c_i32, c_i32, c_i32, c_i32, c_ptr, c_ptr, c_i32, c_ptr, c_ptr, c_ptr, c_i32, c_i32,
                                 c_i32, c_i32, c_ptr, c_ptr, c_ptr, c_ptr]),
}


@functools.cache
def lib() -> ctypes.CDLL:
    """Load libpxb.so (once) and declare every entry point's signature."""
    if not LIB_PATH.exists():
        raise PxbError(
            f"{LIB_PATH} is missing: build it with `python -m plastax_b200.build` "
            "(the engine has no CPU fallback)"
        )
    handle = ctypes.CDLL(str(LIB_PATH))
    for name, (res, args) in _SIGNATURES.items():
        fn = getattr(handle, name)
        fn.restype = res
        fn.argtypes = args
    return handle


def exported_names() -> list[str]:
    """Every entry point this binding declares (the header's function set)."""
    return list(_SIGNATURES)


def last_error() -> str:
    raw = lib().pxb_last_error()
    return raw.decode() if raw else ""


def call(name: str, *args: Any) -> None:
    """Call a status-returning entry point; raise PxbError on failure."""
    fn: Callable[..., int] = getattr(lib(), name)
    rc = fn(*args)
    if rc != 0:
        raise PxbError(f"{name} failed (status {rc}): {last_error()}")


def query_size(name: str, *args: Any) -> int:
    """Call a `*_scratch_bytes` entry point and return the byte count."""
    out = c_size(0)
    call(name, *args, ctypes.byref(out))
    return int(out.value)
