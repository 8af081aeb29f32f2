"""plastax_b200: a B200-native engine for plastax's edge-arena hot path.

The public surface mirrors the parts of `plastax` that sit on the hot path
(the SOA arena, the Network traits in their recognised forms, NetworkBuilder
and make_step); the work runs in hand-written sm_100a kernels behind the C ABI
in include/pxb.h (libpxb.so), with PyTorch providing device memory, streams
and torch.distributed (NCCL) for Scheme-A. There is no CPU execution path:
a missing libpxb.so is an error.
"""

from plastax_b200 import monoid, optim
from plastax_b200._lib import PxbError
from plastax_b200.builder import NetworkBuilder
from plastax_b200.state import NetworkState, NetworkStatic, live_conn_count, make_empty_state
from plastax_b200.state import grow_bucket
from plastax_b200.driver import Driver
from plastax_b200.step import GrowthRemainder, StepFn, StepInputs, StepResult, make_growth_retry, make_step
from plastax_b200.shortlist import ShortlistCoverage, recommended_shortlist, shortlist_coverage
from plastax_b200.topo import resort
from plastax_b200.traits import (
    GRAD_PRE_ACT,
    LOSS_GRAD,
    AddUnit,
    LowestMagnitudePrune,
    AffineUnitUpdate,
    ArgmaxSpawn,
    FieldBelowPrune,
    FieldSpawn,
    PruneUnit,
    TraceUnitUpdate,
    UpdateUnit,
    BackwardPass,
    DestinationThresholdPrune,
    ForwardPass,
    MagnitudePrune,
    MeanFloatFirstRest,
    MSELoss,
    Network,
    ProposeAddConn,
    PruneConn,
    ResetGlobal,
    ScoreAddConn,
    SoftmaxCrossEntropyLoss,
    predicate_add_conn,
)
from plastax_b200.types import (
    ACTIVATION,
    DEAD,
    FROM_ID,
    LEVEL,
    PRUNED,
    TO_ID,
    WEIGHT,
    FieldSpec,
    Propagation,
    ShardSpec,
)

__all__ = [
    "AddUnit", "AffineUnitUpdate", "LowestMagnitudePrune", "ArgmaxSpawn", "FieldBelowPrune", "FieldSpawn", "PruneUnit", "TraceUnitUpdate",
    "UpdateUnit",
    "ACTIVATION", "DEAD", "FROM_ID", "GRAD_PRE_ACT", "LEVEL", "LOSS_GRAD", "PRUNED", "TO_ID", "WEIGHT",
    "BackwardPass", "DestinationThresholdPrune", "Driver", "FieldSpec", "ForwardPass", "GrowthRemainder", "MSELoss",
    "MagnitudePrune", "MeanFloatFirstRest", "Network", "NetworkBuilder", "NetworkState", "NetworkStatic", "Propagation", "ProposeAddConn",
    "PruneConn", "PxbError", "ResetGlobal", "ScoreAddConn", "ShardSpec", "SoftmaxCrossEntropyLoss", "StepFn", "StepInputs", "StepResult", "live_conn_count",
    "grow_bucket", "make_empty_state", "make_growth_retry", "make_step", "monoid", "optim", "predicate_add_conn",
    "recommended_shortlist", "resort", "shortlist_coverage", "ShortlistCoverage",
]
