"""Named combine monoids (mirrors src/plastax/monoid.py:27-218).

sum/max/min lower to the engine's atomic / warp-segmented combines and to
the matching NCCL all-reduce under Scheme-A; `prod` and generic monoids have
no lowering and raise `UnsupportedMonoidError`, as the reference's collective
does for them (src/plastax/monoid.py:175-204).
"""

from __future__ import annotations

import dataclasses
import math


class UnsupportedMonoidError(NotImplementedError):
    """Raised when a monoid without an engine lowering reaches a phase."""


@dataclasses.dataclass(frozen=True)
class Monoid:
    name: str

    @property
    def identity(self) -> float:
        return {"sum": 0.0, "prod": 1.0, "max": -math.inf, "min": math.inf}[self.name]

    def lowered(self) -> str:
        """The engine's monoid name; raises for monoids it cannot run."""
        if self.name not in ("sum", "max", "min"):
            raise UnsupportedMonoidError(
                f"monoid {self.name!r} has no engine lowering; only sum/max/min map to the "
                "device combine and its all-reduce"
            )
        return self.name

    def torch_reduce_op(self):
        """The torch.distributed ReduceOp of the Scheme-A partial combine."""
        import torch.distributed as dist

        return {"sum": dist.ReduceOp.SUM, "max": dist.ReduceOp.MAX, "min": dist.ReduceOp.MIN}[self.lowered()]


sum_ = Monoid("sum")
prod = Monoid("prod")
max_ = Monoid("max")
min_ = Monoid("min")
