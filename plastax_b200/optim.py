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

    def struct(self):
        from plastax_b200._lib import OPT, Optimizer as COpt

        return COpt(OPT[self.kind], self.lr, self.b1, self.b2, self.eps, self.weight_decay)

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
