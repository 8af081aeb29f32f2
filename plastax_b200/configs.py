"""Synthetic instances of the benchmark configurations.

Every input is seeded; no dataset is involved. Shapes follow the reference's
configurations: `reservoir_churn` is the Scheme-A large reservoir (1,048,576
tanh units, fan-in 256, 16 inputs, 0.1% churn per step), built like
examples/reservoir.py:126-187 (recurrent weights N(0, (rho/sqrt(fan_in))^2),
input weights U(-1, 1), every reservoir unit fed by every input).

The churn rule, frozen here so the oracle and the engine run the same
network:
- PruneConn: |w| < tau with tau = 0.0012533 * sigma, the threshold that
  removes 0.1% of N(0, sigma^2) weights (the half-normal 0.1% quantile);
- ProposeAddConn(per_unit, P=1): src = proposing unit, dst = a uniform
  reservoir unit [sub 0], score = uniform() [sub 1], the step's
  max_new_per_level = 0.1% of the recurrent edges under
  level_cap_scope="step", init weight = sigma*sqrt(3)*(2u - 1) with u a
  hash of (src, dst) (the variance of the recurrent weights; a pure function
  of the endpoints, as growth init rules are in the reference).
"""

from __future__ import annotations

import dataclasses
import math

import torch

from plastax_b200 import monoid
from plastax_b200.builder import NetworkBuilder
from plastax_b200.traits import ForwardPass, MagnitudePrune, Network, ProposeAddConn
from plastax_b200.types import Propagation, ShardSpec


@dataclasses.dataclass(frozen=True)
class ReservoirConfig:
    num_units: int = 1 << 20  # reservoir units
    num_inputs: int = 16
    fan_in: int = 256
    rho: float = 0.95
    churn: float = 0.001
    capacity_align: int = 8192
    capacity_headroom: float = 0.01
    seed: int = 0

    @property
    def sigma(self) -> float:
        return self.rho / math.sqrt(self.fan_in)

    @property
    def recurrent_edges(self) -> int:
        return self.num_units * self.fan_in

    @property
    def input_edges(self) -> int:
        return self.num_units * self.num_inputs

    @property
    def live_edges(self) -> int:
        return self.recurrent_edges + self.input_edges

    @property
    def tau(self) -> float:
        return 0.0012533 * self.sigma

    @property
    def k(self) -> int:
        return int(round(self.churn * self.recurrent_edges))


C5 = ReservoirConfig()


def reservoir_net(cfg: ReservoirConfig, sharding: ShardSpec | None = None) -> type[Network]:
    class ReservoirChurn(Network):
        forward_pass = ForwardPass("tanh", monoid.sum_)
        prune_conn = MagnitudePrune(cfg.tau)
        add_conn = ProposeAddConn(
            proposals_per_proposer=1, max_new_per_level=cfg.k, dst_lo=cfg.num_inputs, dst_n=cfg.num_units,
            score="uniform", init=("hash_uniform", cfg.sigma * math.sqrt(3.0)), level_cap_scope="step")
        propagation = Propagation.PIPELINE
        seed = cfg.seed

    ReservoirChurn.sharding = sharding
    return ReservoirChurn


def reservoir_edges(cfg: ReservoirConfig, device: torch.device | str):
    """(src, dst, weight) device tensors of the reservoir, seeded."""
    dev = torch.device(device)
    g = torch.Generator(device=dev)
    g.manual_seed(cfg.seed)
    n_in, n_res = cfg.num_inputs, cfg.num_units
    res = torch.arange(n_res, dtype=torch.int32, device=dev) + n_in
    rec_dst = res.repeat_interleave(cfg.fan_in)
    rec_src = torch.randint(0, n_res, (cfg.recurrent_edges,), generator=g, device=dev, dtype=torch.int32) + n_in
    rec_w = torch.randn(cfg.recurrent_edges, generator=g, device=dev, dtype=torch.float32) * cfg.sigma
    in_dst = res.repeat_interleave(n_in)
    in_src = torch.arange(n_in, dtype=torch.int32, device=dev).repeat(n_res)
    in_w = torch.rand(cfg.input_edges, generator=g, device=dev, dtype=torch.float32) * 2.0 - 1.0
    src = torch.cat([rec_src, in_src])
    del rec_src, in_src
    dst = torch.cat([rec_dst, in_dst])
    del rec_dst, in_dst
    w = torch.cat([rec_w, in_w])
    return src, dst, w


def build_reservoir(cfg: ReservoirConfig, device: torch.device | str = "cuda", *, sharding: ShardSpec | None = None,
                    shard_rank: int = 0):
    net = reservoir_net(cfg, sharding)
    src, dst, w = reservoir_edges(cfg, device)
    total = cfg.num_inputs + cfg.num_units
    static, state = NetworkBuilder.from_edges(
        net, total, src, dst, weights=w, input_ids=tuple(range(cfg.num_inputs)), output_ids=(),
        capacity_headroom=cfg.capacity_headroom, capacity_align=cfg.capacity_align, sharding=sharding,
        shard_rank=shard_rank, device=device)
    del src, dst, w
    return net, static, state
