"""Policy traits and the Network base (mirrors src/plastax/traits.py).

The reference's policies are arbitrary JAX callables traced under vmap; a
native engine can only run the forms it recognises. Each trait here is that
recognised form, with the reference's names, attributes and defaults, and
`Network` validates a subclass's slots the way the reference's
`__init_subclass__` does, raising at class-definition time for a policy the
engine cannot run (there is no fallback path).

Recognised forms:
- ForwardPass: map = weight * activation[src] (the linear_input map of
  src/plastax/phases.py:535-556), combine = sum/max/min, apply =
  activation(acc) written into ACTIVATION (identity, tanh, relu, sigmoid),
  optionally another activation for the output units (a linear readout).
- BackwardPass: map = weight * grad_field[dst], combine = sum, apply:
  grad_field = (acc + seed_field) * activation'(ACTIVATION)
  (scripts/parity/golden_rules.py relu_mlp_v1 generalised).
- Loss: MSELoss (scripts/parity/reference.py:338-352) and
  SoftmaxCrossEntropyLoss (src/plastax/traits.py:205-250).
- batch_reduction: MeanFloatFirstRest for a batched step.
- update_conn: an optimizer bundle from plastax_b200.optim (sgd, momentum,
  adam, adamw, rmsprop; src/plastax/optim).
- PruneConn: |weight| < threshold (MagnitudePrune) or |weight| <
  unit[field, dst] (DestinationThresholdPrune).
- ProposeAddConn: proposer "per_unit" (dst = dst_lo + uniform_int(dst_n)
  [sub 0], score [sub 1]), "global" (src = src_lo + uniform_int(src_n) [sub
  0], dst [sub 1], score [sub 2]) or "per_connection" (src = the proposing
  connection's source, dst [sub 0], score [sub 1]); score uniform /
  floor(u*256)/256 or |grad[dst]*act[src]|; selection top_k, threshold (a
  constant) or all, capped per source level or per step;
  init weight constant / dyadic / hashed uniform; dedupe_live (a candidate
  equal to a live edge is vetoed) and dedupe_step (a pair's copies after the
  first in score order are vetoed).
- ScoreAddConn: the exhaustive grid, the importance shortlist or the
  per-level shortlists, scored by a lowered pair score (|x[src]*y[dst]|,
  x[src]*y[dst], |grad[dst]*act[src]|, the modular conformance rules) with
  the same selection, caps, dedupes and init as ProposeAddConn;
  predicate_add_conn for a boolean rule.
"""

from __future__ import annotations

import dataclasses
from typing import Any, ClassVar

from plastax_b200 import monoid as _monoid
from plastax_b200.types import FieldSpec, Propagation, ShardSpec

ACTIVATIONS = ("identity", "tanh", "relu", "sigmoid")

GRAD_PRE_ACT = FieldSpec.float32("grad_pre_act")
LOSS_GRAD = FieldSpec.float32("loss_grad")


class ForwardPass:
    """Forward propagation policy (src/plastax/traits.py:39-90)."""

    combine: _monoid.Monoid = _monoid.sum_
    activation: str = "tanh"
    # the output units' activation, when it differs (a linear readout)
    output_activation: str | None = None

    def __init__(self, activation: str | None = None, combine: _monoid.Monoid | None = None,
                 output_activation: str | None = None) -> None:
        if activation is not None:
            self.activation = activation
        if combine is not None:
            self.combine = combine
        if output_activation is not None:
            self.output_activation = output_activation


class BackwardPass:
    """Backward propagation policy (src/plastax/traits.py:92-152)."""

    combine: _monoid.Monoid = _monoid.sum_
    activation: str = "tanh"
    grad_field: FieldSpec = GRAD_PRE_ACT
    seed_field: FieldSpec = LOSS_GRAD
    # the output units' activation derivative (None: the forward pass's
    # output_activation, else `activation`)
    output_activation: str | None = None

    def __init__(self, activation: str | None = None, grad_field: FieldSpec | None = None,
                 seed_field: FieldSpec | None = None, output_activation: str | None = None) -> None:
        if output_activation is not None:
            self.output_activation = output_activation
        if activation is not None:
            self.activation = activation
        if grad_field is not None:
            self.grad_field = grad_field
        if seed_field is not None:
            self.seed_field = seed_field


class MSELoss:
    """L = 0.5 * sum (act - t)^2 over the outputs; seed = act - t
    (scripts/parity/reference.py:338-352)."""

    def __init__(self, seed_field: FieldSpec = LOSS_GRAD) -> None:
        self.seed_field = seed_field


class SoftmaxCrossEntropyLoss:
    """Softmax over the output activations, cross-entropy against a target
    distribution (src/plastax/traits.py:205-250): z = a - max(a), s = sum
    exp(z), loss = sum t * (log s - z), seed = exp(z) / s - t."""

    def __init__(self, seed_field: FieldSpec = LOSS_GRAD) -> None:
        self.seed_field = seed_field


class MeanFloatFirstRest:
    """Batch reduction (src/plastax/traits.py:811-838): the batch mean of every
    floating unit column, sample 0 of any other, LEVEL and PRUNED not batched."""

    def reduction(self, field: FieldSpec) -> str:
        if field.name in ("level", "pruned"):
            return "not_batched"
        return "mean" if field.dtype.kind == "f" else "first"


class PruneConn:
    """Connection prune policy (src/plastax/traits.py:352-375)."""


class MagnitudePrune(PruneConn):
    """Prune a connection when |weight| < threshold."""

    def __init__(self, threshold: float) -> None:
        self.threshold = float(threshold)


class DestinationThresholdPrune(PruneConn):
    """Prune a connection when |weight| < unit[field, dst] (the per-unit
    magnitude threshold of examples/dst_sparse.py:189-199)."""

    def __init__(self, field: FieldSpec) -> None:
        self.field = field


class LowestMagnitudePrune(PruneConn):
    """Prune the k live connections of lowest |weight| (ties by ascending
    slot, buckets in order), on the steps `every` divides: the
    lowest-magnitude churn of the dynamic-sparse-training configurations
    (the reference states it as a predicate against a threshold the host
    computes into the globals; here the selection runs on the device and
    prunes exactly min(k, live) edges). A NaN weight is never selected.

    On an arena with a destination-grouped mirror (no weight-rewriting
    phase, one bucket) the prune rides on the forward sweep: only the edges
    whose |w| shares the k-th smallest's histogram bin (the top 16 bits of
    |w|) are listed and selected apart; `list_capacity` bounds that list
    per rank (default max(65536, k)), and a firing whose threshold bin
    holds more live edges than that raises an error instead of pruning
    fewer than k."""

    def __init__(self, k: int, every: int = 1, list_capacity: int | None = None) -> None:
        if int(k) < 0 or int(every) < 1:
            raise ValueError("LowestMagnitudePrune: k must be >= 0 and every >= 1")
        if list_capacity is not None and int(list_capacity) < 1:
            raise ValueError("LowestMagnitudePrune: list_capacity must be >= 1")
        self.k = int(k)
        self.every = int(every)
        self.list_capacity = None if list_capacity is None else int(list_capacity)


class ResetGlobal:
    """Globals reset (src/plastax/traits.py:686-703); host-side, O(1)."""

    def reset(self, g: Any) -> Any:
        return g


@dataclasses.dataclass
class ProposeAddConn:
    """Proposal growth (src/plastax/traits.py:577-684) in its recognised form."""

    proposals_per_proposer: int
    max_new_per_level: int
    dst_lo: int = 0
    dst_n: int | None = None
    src_lo: int = 0  # the global proposer's source range
    src_n: int | None = None
    score: str = "uniform"  # "uniform", "uniform_q256" or "grad_act"
    init: tuple = ("const", 0.0)  # ("const", a) | ("dyadic",) | ("hash_uniform", a)
    proposer: str = "per_unit"
    selection: str = "top_k"
    level_cap_scope: str = "source_level"
    max_level_gap: int = 1
    direction: str = "any"
    allow_self_loops: bool = False
    dedupe_live: bool = False
    dedupe_step: bool = False
    max_new_per_step: int | None = None
    trigger: Any = "every_step"
    on_overflow: str = "flag"
    grad_field: FieldSpec = GRAD_PRE_ACT
    threshold: float | None = None  # selection "threshold": keep scores >= threshold

    def validate(self) -> None:
        if self.proposer not in ("per_unit", "global", "per_connection"):
            raise ValueError(f"unknown proposer {self.proposer!r}")
        if self.selection not in ("top_k", "threshold", "all"):
            raise ValueError(f"unknown selection {self.selection!r}")
        if self.selection == "threshold" and self.threshold is None:
            raise ValueError("selection 'threshold' needs ProposeAddConn.threshold")
        if self.level_cap_scope not in ("source_level", "step"):
            raise ValueError(f"unknown level_cap_scope {self.level_cap_scope!r}")
        if self.direction not in ("any", "deeper", "same_or_deeper"):
            raise ValueError(f"unknown direction {self.direction!r}")
        if self.score not in ("uniform", "uniform_q256", "grad_act"):
            raise ValueError(f"unknown proposal score {self.score!r}")
        if self.init[0] not in ("const", "dyadic", "hash_uniform"):
            raise ValueError(f"unknown init rule {self.init!r}")
        if self.proposals_per_proposer < 1 or self.max_new_per_level < 0:
            raise ValueError("proposals_per_proposer must be >= 1 and max_new_per_level >= 0")
        if self.on_overflow not in ("flag", "error"):
            raise ValueError(f"unknown on_overflow {self.on_overflow!r}")


def _field_name(f) -> str:
    return f if isinstance(f, str) else f.name


class UpdateUnit:
    """Unit update policy (src/plastax/traits.py:254-278): one write per live
    unit, inputs and outputs included, after the backward pass and before
    the connection update."""


@dataclasses.dataclass(frozen=True)
class AffineUnitUpdate(UpdateUnit):
    """field = field * scale + shift (scripts/parity/golden_rules.py:
    unit_update_v1 is AffineUnitUpdate("activation", 1.0, 0.125))."""

    field: Any
    scale: float = 1.0
    shift: float = 0.0


@dataclasses.dataclass(frozen=True)
class TraceUnitUpdate(UpdateUnit):
    """field = (1 - rate) * field + rate * |source| (or source when
    `absolute` is False): a running trace such as the examples' activation
    EMA (examples/upgd.py:113-128)."""

    field: Any
    source: Any
    rate: float
    absolute: bool = True


class PruneUnit:
    """Unit prune policy (src/plastax/traits.py:377-406): the predicate on
    the pre-phase state; inputs and outputs are never pruned; a pruned unit's
    columns reset to their defaults (LEVEL kept) and every incident
    connection is tombstoned."""


@dataclasses.dataclass(frozen=True)
class FieldBelowPrune(PruneUnit):
    """Prune a unit when u[field] < threshold: a constant, or (quantile q)
    the value at rank floor(q * m) of the m live non-I/O units' values
    ascending, computed on the device before the phase
    (scripts/parity/golden_rules.py: unit_prune_v1 is
    FieldBelowPrune("activation", threshold=-0.5))."""

    field: Any
    threshold: float | None = None
    quantile: float | None = None


class AddUnit:
    """Unit addition policy (src/plastax/traits.py:409-465): live parents
    spawn one child each into the lowest free slots, ascending parent id; the
    child's level is clamp(level(parent) + offset, 1, max_levels - 1)."""


@dataclasses.dataclass(frozen=True)
class FieldSpawn(AddUnit):
    """Every live unit with u[field] >= threshold spawns; `init` is None or
    ("scale_parent", child_field, parent_field, scale): child_field of the
    child = parent_field of the parent * scale (golden rules unit_spawn_v1 =
    FieldSpawn("activation", 0.5, 1), unit_child_init_v1 = ("scale_parent",
    "activation", "activation", 0.5))."""

    field: Any
    threshold: float
    offset: int = 1
    init: tuple | None = None


@dataclasses.dataclass(frozen=True)
class ArgmaxSpawn(AddUnit):
    """The live unit with the largest u[field] (lowest id on ties) spawns
    one child: with structural_interval N, one unit every N steps."""

    field: Any
    offset: int = 1
    init: tuple | None = None


_SCORE_FORMS = {"abs_product": 3, "product": 3, "grad_act": 1, "modular": 6, "modular_predicate": 5}
_IMPORTANCE_FORMS = {"abs_field": 2, "field": 2, "modular": 5}


@dataclasses.dataclass
class ScoreAddConn:
    """Scored-candidate growth (src/plastax/traits.py:467-575) in its
    recognised form.

    `candidates`: "exhaustive" (every ordered unit pair, index src * N +
    dst), "shortlist" (the M x M grid over the top-M units by importance,
    ties by ascending id; M = shortlist_size) or "shortlist_per_level"
    (TOPOLOGICAL only: per source level, its top-M sources x the top-M
    destinations inside its window). A shortlist with M >= num_units is the
    exhaustive grid, as in the reference.

    `score` (the rule's score(u, src, dst, g)), one of
    ("abs_product", src_field, dst_field): |u[src_field][src] * u[dst_field][dst]|;
    ("product", src_field, dst_field): u[src_field][src] * u[dst_field][dst];
    ("grad_act",): |grad_field[dst] * activation[src]|;
    ("modular", a, b, m, c, scale): (((a*src + b*dst) mod m) - c) * scale;
    ("modular_predicate", a, b, m, r): 0 if (a*src + b*dst) mod m == r else -inf.
    `importance` (importance(u, i, g)): ("abs_field", field), ("field",
    field) or ("modular", a, m, c, scale) = (((a*i) mod m) - c) * scale.
    A non-finite score vetoes the candidate. The modular forms are the
    reference's versioned conformance rules (scripts/parity/golden_rules.py:
    grid_score_v1 = ("modular", 3, 5, 17, 8, 0.125), importance_v1 =
    ("modular", 7, 13, 0, 0.25), predicate_v1 = ("modular_predicate", 1, 1, 2, 0)).
    """

    score: tuple
    max_new_per_level: int | None = None
    candidates: str = "exhaustive"
    shortlist_size: int | None = None
    importance: tuple | None = None
    init: tuple = ("const", 0.0)
    selection: str = "top_k"
    threshold: float | None = None
    level_cap_scope: str = "source_level"
    max_new_per_step: int | None = None
    max_level_gap: int = 1
    direction: str = "any"
    allow_self_loops: bool = False
    dedupe_live: bool = False
    dedupe_step: bool = False
    trigger: Any = "every_step"
    on_overflow: str = "flag"
    grad_field: FieldSpec = GRAD_PRE_ACT

    def validate(self) -> None:
        """The reference's knob checks (src/plastax/traits.py:1390-1520),
        TypeError as there, plus the lowered forms' own."""
        if self.candidates not in ("exhaustive", "shortlist", "shortlist_per_level"):
            raise TypeError(f"add_conn.candidates must be exhaustive / shortlist / shortlist_per_level; got "
                            f"{self.candidates!r}")
        if self.candidates != "exhaustive":
            size = self.shortlist_size
            if not isinstance(size, int) or isinstance(size, bool) or size < 1:
                raise TypeError(f"add_conn.shortlist_size must be an int >= 1 for candidates = "
                                f"{self.candidates!r}; got {size!r}")
            if self.importance is None:
                raise TypeError(f"add_conn: candidates = {self.candidates!r} requires an importance form")
        if self.selection not in ("top_k", "threshold", "all"):
            raise TypeError(f"add_conn.selection must be top_k / threshold / all; got {self.selection!r}")
        mnpl = self.max_new_per_level
        if self.selection != "all" or mnpl is not None:
            if not isinstance(mnpl, int) or isinstance(mnpl, bool) or mnpl < 1:
                raise TypeError(f"add_conn.max_new_per_level must be an int >= 1 (required unless selection = "
                                f"'all'); got {mnpl!r}")
        if self.selection == "threshold" and self.threshold is None:
            raise TypeError("add_conn: selection = 'threshold' requires a threshold")
        if self.level_cap_scope not in ("source_level", "step"):
            raise TypeError(f"add_conn.level_cap_scope must be source_level / step; got {self.level_cap_scope!r}")
        mnps = self.max_new_per_step
        if mnps is not None and (not isinstance(mnps, int) or isinstance(mnps, bool) or mnps < 1):
            raise TypeError(f"add_conn.max_new_per_step must be an int >= 1 or None; got {mnps!r}")
        if self.direction not in ("any", "deeper", "same_or_deeper"):
            raise TypeError(f"add_conn.direction must be any / deeper / same_or_deeper; got {self.direction!r}")
        if self.on_overflow not in ("flag", "error"):
            raise TypeError(f"add_conn.on_overflow must be 'flag' or 'error'; got {self.on_overflow!r}")
        for flag in ("dedupe_live", "dedupe_step", "allow_self_loops"):
            if not isinstance(getattr(self, flag), bool):
                raise TypeError(f"add_conn.{flag} must be a bool")
        form = self.score
        if not isinstance(form, tuple) or not form or form[0] not in _SCORE_FORMS \
                or len(form) != _SCORE_FORMS[form[0]]:
            raise NotImplementedError(f"add_conn.score form {form!r} has no engine lowering")
        if self.importance is not None:
            imp = self.importance
            if not isinstance(imp, tuple) or not imp or imp[0] not in _IMPORTANCE_FORMS \
                    or len(imp) != _IMPORTANCE_FORMS[imp[0]]:
                raise NotImplementedError(f"add_conn.importance form {imp!r} has no engine lowering")
        if self.init[0] not in ("const", "dyadic", "hash_uniform"):
            raise NotImplementedError(f"add_conn.init rule {self.init!r} has no engine lowering")


def predicate_add_conn(should_add: tuple, init: tuple = ("const", 0.0), **params: Any) -> ScoreAddConn:
    """A boolean growth predicate as a ScoreAddConn (src/plastax/traits.py:
    1523-1580): score 0 (grow) or -inf (veto), selection "all" and
    dedupe_step True unless `params` override them. `should_add` is
    ("modular_predicate", a, b, m, r)."""
    params.setdefault("selection", "all")
    params.setdefault("dedupe_step", True)
    return ScoreAddConn(score=should_add, init=init, **params)


class Network:
    """A network's trait slots (src/plastax/traits.py:874-1072).

    Subclasses set class attributes; a slot left None is elided from the
    step, as in the reference's phase assembly (src/plastax/phases.py:87-176).
    """

    forward_pass: ClassVar[ForwardPass]
    loss: ClassVar[MSELoss | SoftmaxCrossEntropyLoss | None] = None
    backward_pass: ClassVar[BackwardPass | None] = None
    update_unit: ClassVar[UpdateUnit | None] = None
    update_conn: ClassVar[Any] = None  # an optimizer bundle (plastax_b200.optim)
    prune_unit: ClassVar[PruneUnit | None] = None
    prune_conn: ClassVar[PruneConn | None] = None
    add_unit: ClassVar[AddUnit | None] = None
    add_conn: ClassVar[ProposeAddConn | ScoreAddConn | None] = None
    reset_global: ClassVar[ResetGlobal | None] = None
    propagation: ClassVar[Propagation] = Propagation.TOPOLOGICAL
    seed: ClassVar[int] = 0
    extra_conn_fields: ClassVar[tuple[FieldSpec, ...]] = ()
    extra_unit_fields: ClassVar[tuple[FieldSpec, ...]] = ()
    unit_capacity: ClassVar[int | None] = None
    max_levels: ClassVar[int] = 1024  # a child's level is clamped to [1, max_levels - 1]
    structural_interval: ClassVar[int] = 1
    sharding: ClassVar[ShardSpec | None] = None
    kahn_max_depth: ClassVar[int | None] = None
    batch_reduction: ClassVar[Any] = None  # e.g. MeanFloatFirstRest(), required by a batched step

    def __init_subclass__(cls, **kwargs: Any) -> None:
        super().__init_subclass__(**kwargs)
        fp = getattr(cls, "forward_pass", None)
        if fp is None or not isinstance(fp, ForwardPass):
            raise TypeError(f"{cls.__name__}: forward_pass must be a ForwardPass")
        if fp.activation not in ACTIVATIONS:
            raise ValueError(f"{cls.__name__}: unknown activation {fp.activation!r}")
        if fp.output_activation is not None and fp.output_activation not in ACTIVATIONS:
            raise ValueError(f"{cls.__name__}: unknown output activation {fp.output_activation!r}")
        bp_out = getattr(cls.backward_pass, "output_activation", None)
        if bp_out is not None and bp_out not in ACTIVATIONS:
            raise ValueError(f"{cls.__name__}: unknown backward output activation {bp_out!r}")
        fp.combine.lowered()
        if cls.backward_pass is not None:
            bp = cls.backward_pass
            if bp.activation not in ACTIVATIONS:
                raise ValueError(f"{cls.__name__}: unknown backward activation {bp.activation!r}")
            if bp.combine.lowered() != "sum":
                raise NotImplementedError(f"{cls.__name__}: the backward combine must be sum")
        if cls.prune_conn is not None and not isinstance(cls.prune_conn, (MagnitudePrune, DestinationThresholdPrune,
                                                                          LowestMagnitudePrune)):
            raise NotImplementedError(f"{cls.__name__}: prune_conn form has no engine lowering")
        if cls.add_conn is not None:
            cls.add_conn.validate()
            if (isinstance(cls.add_conn, ScoreAddConn) and cls.add_conn.candidates == "shortlist_per_level"
                    and cls.propagation is Propagation.PIPELINE):
                raise ValueError('candidates = "shortlist_per_level" is levels-based and so topological-only; '
                                 "PIPELINE networks use the global shortlist")
        if cls.update_unit is not None and not isinstance(cls.update_unit, (AffineUnitUpdate, TraceUnitUpdate)):
            raise NotImplementedError(f"{cls.__name__}: update_unit form has no engine lowering")
        if cls.prune_unit is not None:
            pu = cls.prune_unit
            if not isinstance(pu, FieldBelowPrune):
                raise NotImplementedError(f"{cls.__name__}: prune_unit form has no engine lowering")
            if (pu.threshold is None) == (pu.quantile is None):
                raise ValueError(f"{cls.__name__}: FieldBelowPrune takes exactly one of threshold and quantile")
            if pu.quantile is not None and not 0.0 <= pu.quantile <= 1.0:
                raise ValueError(f"{cls.__name__}: FieldBelowPrune quantile must be in [0, 1]")
        if cls.add_unit is not None:
            au = cls.add_unit
            if not isinstance(au, (FieldSpawn, ArgmaxSpawn)):
                raise NotImplementedError(f"{cls.__name__}: add_unit form has no engine lowering")
            if au.init is not None and (len(au.init) != 4 or au.init[0] != "scale_parent"):
                raise NotImplementedError(f"{cls.__name__}: add_unit init {au.init!r} has no engine lowering")
        if (cls.prune_unit is not None or cls.add_unit is not None) and cls.unit_capacity is None:
            raise TypeError(f"{cls.__name__}: prune_unit and add_unit require Network.unit_capacity")
        if int(cls.max_levels) < 2:
            raise ValueError(f"{cls.__name__}: max_levels must be >= 2")

    @classmethod
    def unit_fields(cls) -> tuple[FieldSpec, ...]:
        from plastax_b200.types import ACTIVATION, LEVEL, PRUNED

        fields: list[FieldSpec] = [ACTIVATION, LEVEL]
        if cls.backward_pass is not None:
            fields += [cls.backward_pass.grad_field]
        if cls.loss is not None:
            fields += [cls.loss.seed_field]
        if isinstance(cls.prune_conn, DestinationThresholdPrune):
            fields += [cls.prune_conn.field]
        fields += list(cls.extra_unit_fields)
        if cls.update_conn is not None:
            fields += list(getattr(cls.update_conn, "unit_fields", ()))
        if cls.unit_capacity is not None:
            fields += [PRUNED]
        out: list[FieldSpec] = []
        for f in fields:
            if f.name not in {o.name for o in out}:
                out.append(f)
        return tuple(out)

    @classmethod
    def conn_fields(cls) -> tuple[FieldSpec, ...]:
        from plastax_b200.types import BUILTIN_CONN_FIELDS

        extra = list(cls.extra_conn_fields)
        if cls.update_conn is not None:
            extra += list(cls.update_conn.state_fields)
        out = list(BUILTIN_CONN_FIELDS)
        for f in extra:
            if f.name not in {o.name for o in out}:
                out.append(f)
        return tuple(out)
