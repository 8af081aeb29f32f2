"""Optimizer bundles (mirrors src/plastax/optim/__init__.py:1-77).

A bundle names the per-connection update the engine runs (fused into the
backward sweep where legal) and the extra SOA columns its state needs; the
columns shard with the connections under Scheme-A. The update rules follow
src/plastax/optim/_sgd.py:121-127, _momentum.py:136-139, _adam.py:157-172 and
_rmsprop.py:135-140; the delta-rule gradient is grad_field[dst] *
activation[src].
"""

from __future__ import annotations

import dataclasses

from plastax_b200.types import FieldSpec
from plastax_b200.traits import GRAD_PRE_ACT

_M = FieldSpec.float32("opt/m")
_V = FieldSpec.float32("opt/v")
_T = FieldSpec.float32("opt/t")


UPGD_UTIL = FieldSpec.float32("upgd/util")
UPGD_T = FieldSpec.float32("upgd/t")
UPGD_ETA = FieldSpec.float32("upgd/eta")


@dataclasses.dataclass(frozen=True)
class Optimizer:
    kind: str
    lr: float
    grad_field: FieldSpec = GRAD_PRE_ACT
    b1: float = 0.0
    b2: float = 0.0
    eps: float = 0.0
    weight_decay: float = 0.0
    state_fields: tuple[FieldSpec, ...] = ()
    needs_step_counter: bool = False
    # the bucket columns the kernel reads as (m, v, t)
    cols: tuple[str, str, str] = ("opt/m", "opt/v", "opt/t")
    unit_fields: tuple[FieldSpec, ...] = ()
    # upgd: the unit column of the utility scale, and who writes it: "local"
    # (the step, as the max of each destination's incoming utilities) or
    # "global" (the caller, e.g. upgd_global_eta)
    scale_field: FieldSpec | None = None
    eta: str = "local"

    def struct(self, unit_scale=None):
        from plastax_b200._lib import OPT, Optimizer as COpt

        scale = None if unit_scale is None else unit_scale.data_ptr()
        return COpt(OPT[self.kind], self.lr, self.b1, self.b2, self.eps, self.weight_decay, scale)

    def oracle_args(self) -> dict:
        return dict(kind=self.kind, lr=self.lr, b1=self.b1, b2=self.b2, eps=self.eps, wd=self.weight_decay)


def sgd(lr: float, grad_field: FieldSpec = GRAD_PRE_ACT) -> Optimizer:
    return Optimizer("sgd", lr, grad_field)


def momentum(lr: float, momentum: float = 0.9, grad_field: FieldSpec = GRAD_PRE_ACT) -> Optimizer:
    return Optimizer("momentum", lr, grad_field, b1=momentum, state_fields=(_V,))


def adam(lr: float, grad_field: FieldSpec = GRAD_PRE_ACT, b1: float = 0.9, b2: float = 0.999,
         eps: float = 1e-8) -> Optimizer:
    return Optimizer("adam", lr, grad_field, b1=b1, b2=b2, eps=eps, state_fields=(_M, _V, _T))


def adamw(lr: float, grad_field: FieldSpec = GRAD_PRE_ACT, weight_decay: float = 1e-4, b1: float = 0.9,
          b2: float = 0.999, eps: float = 1e-8) -> Optimizer:
    return Optimizer("adam", lr, grad_field, b1=b1, b2=b2, eps=eps, weight_decay=weight_decay,
                     state_fields=(_M, _V, _T))


def rmsprop(lr: float, grad_field: FieldSpec = GRAD_PRE_ACT, decay: float = 0.9, eps: float = 1e-8) -> Optimizer:
    return Optimizer("rmsprop", lr, grad_field, b1=decay, eps=eps, state_fields=(_V,))


def upgd(lr: float = 0.01, beta: float = 0.999, sigma: float = 0.001, eps: float = 1e-8,
         grad_field: FieldSpec = GRAD_PRE_ACT, eta: str = "local") -> Optimizer:
    """Utility-based perturbed gradient descent (examples/upgd.py:135-208):
    per-edge utility trace `upgd/util` and step `upgd/t`, the utility scale
    per destination in the unit column `upgd/eta` -- the max of its incoming
    edges' stored utilities, computed by the step before the update
    (eta="local", the example's v1), or written by the caller between steps
    (eta="global", v0: see upgd_global_eta)."""
    if eta not in ("local", "global"):
        raise ValueError(f"upgd: eta must be 'local' or 'global', got {eta!r}")
    return Optimizer("upgd", lr, grad_field, b1=beta, b2=sigma, eps=eps, state_fields=(UPGD_UTIL, UPGD_T),
                     cols=(UPGD_UTIL.name, "", UPGD_T.name), unit_fields=(UPGD_ETA,), scale_field=UPGD_ETA, eta=eta)


def upgd_global_eta(state) -> None:
    """v0's scale (examples/upgd.py:211-230): max(1e-8, max(0, every live
    edge's utility)) broadcast into `upgd/eta`, in place (device reductions,
    one host read)."""
    import torch

    best = torch.zeros((), dtype=torch.float32, device=state.units[UPGD_ETA.name].device)
    for b in state.conns:
        live = b["dead"] == 0
        if bool(live.any()):
            best = torch.maximum(best, b[UPGD_UTIL.name][live].max())
    state.units[UPGD_ETA.name].fill_(max(float(best.item()), 1e-8))
