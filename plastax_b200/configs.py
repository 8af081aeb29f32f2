"""Synthetic instances of the benchmark configurations.

Every input is seeded; no dataset is involved. Shapes follow the reference's
configurations: `reservoir_churn` is the Scheme-A large reservoir (1,048,576
tanh units, fan-in 256, 16 inputs, 0.1% churn per step), built like
examples/reservoir.py:126-187 (recurrent weights N(0, (rho/sqrt(fan_in))^2),
input weights U(-1, 1), every reservoir unit fed by every input).

The churn rule, frozen here so the oracle and the engine run the same
network:
- PruneConn: the k = 0.1% x recurrent-edge-count live edges of lowest |w|,
  every step (the k-th smallest |w| of the state before the step as the
  threshold, as the reference's churn recomputes it from the current
  weights, examples/dst_sparse.py:88-140; ties by ascending slot, so
  exactly k go and the live-edge count stays constant under regrowth).
  `prune="threshold"` keeps the older fixed rule |w| < tau with
  tau = 0.0012533 * sigma (the half-normal 0.1% quantile of the initial
  weights), which prunes 0.1% only on the first step;
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
from plastax_b200.traits import ForwardPass, LowestMagnitudePrune, MagnitudePrune, Network, ProposeAddConn
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
    prune: str = "lowest_k"  # or "threshold"

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
        prune_conn = LowestMagnitudePrune(cfg.k) if cfg.prune == "lowest_k" else MagnitudePrune(cfg.tau)
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


@dataclasses.dataclass(frozen=True)
class EsnConfig:
    """The streaming echo-state reservoir (the reference's CPU-runnable
    configuration; examples/echo_state_network.py): one input unit, `units`
    tanh reservoir units with recurrent fan-in 16 from uniform sources
    without self-loops, weights N(0, 1/16) rescaled to spectral radius `rho`,
    every reservoir unit fed by the input with weight U(-1, 1), and one
    linear readout unit fed by every reservoir unit (weights start at 0),
    trained online by LMS (SGD on the MSE seed) to reproduce the input
    delayed `delay` steps."""

    units: int = 1024
    fan_in: int = 16
    rho: float = 0.9
    lr: float = 1e-3
    delay: int = 5
    seed: int = 0


C1 = EsnConfig()


def esn_net(cfg: EsnConfig) -> type[Network]:
    from plastax_b200 import optim
    from plastax_b200.traits import LOSS_GRAD, MSELoss

    class EchoStateNetwork(Network):
        forward_pass = ForwardPass("tanh", monoid.sum_, output_activation="identity")
        loss = MSELoss()
        update_conn = optim.sgd(cfg.lr, grad_field=LOSS_GRAD)
        propagation = Propagation.PIPELINE
        seed = cfg.seed

    return EchoStateNetwork


def esn_edges(cfg: EsnConfig):
    """(src, dst, weight) numpy arrays of the ESN, seeded (the spectral
    radius from the dense eigenvalues of the recurrent matrix)."""
    import numpy as np

    rng = np.random.default_rng(cfg.seed)
    n = cfg.units
    res = np.arange(n) + 1  # unit 0 is the input, n + 1 the readout
    rec_dst = np.repeat(res, cfg.fan_in)
    off = rng.integers(1, n, rec_dst.size)  # a uniform source other than the destination
    rec_src = (rec_dst - 1 + off) % n + 1
    rec_w = rng.standard_normal(rec_dst.size) / math.sqrt(cfg.fan_in)
    dense = np.zeros((n, n))
    np.add.at(dense, (rec_dst - 1, rec_src - 1), rec_w)
    radius = float(np.max(np.abs(np.linalg.eigvals(dense))))
    rec_w = rec_w * (cfg.rho / radius)
    in_w = rng.uniform(-1.0, 1.0, n)
    src = np.concatenate([rec_src, np.zeros(n, np.int64), res])
    dst = np.concatenate([rec_dst, res, np.full(n, n + 1)])
    w = np.concatenate([rec_w, in_w, np.zeros(n)]).astype(np.float32)
    return src.astype(np.int32), dst.astype(np.int32), w


def build_esn(cfg: EsnConfig = C1, device: torch.device | str = "cuda"):
    net = esn_net(cfg)
    src, dst, w = esn_edges(cfg)
    static, state = NetworkBuilder.from_edges(net, cfg.units + 2, src, dst, weights=w, input_ids=(0,),
                                              output_ids=(cfg.units + 1,), device=device)
    return net, static, state
