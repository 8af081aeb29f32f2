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


# ---------------------------------------------------------------------------
# The training configurations: the sparse MLP (batched), dynamic sparse
# training and the unit lifecycle. Every input, target and weight is seeded;
# no dataset is involved (the MLP's images and labels are N(0, 1) inputs and
# uniform labels of the same shapes).
# ---------------------------------------------------------------------------
@dataclasses.dataclass(frozen=True)
class MlpConfig:
    """Topological sparse MLP trained with make_step(batch_size=B): layers
    784-1000-1000-10, each layer pair's connections drawn with probability
    `density` (0.1: 179,400 edges; 0.5: ~897,000), Kaiming-uniform weights
    U(+-sqrt(6 / fan_in)) with the destination's actual fan-in, ReLU hidden
    units, linear logits, softmax cross-entropy against one-hot labels, SGD,
    MeanFloatFirstRest batch reduction."""

    layers: tuple = (784, 1000, 1000, 10)
    density: float = 0.1
    batch: int = 256
    lr: float = 0.01
    seed: int = 0

    @property
    def num_units(self) -> int:
        return int(sum(self.layers))


C2 = MlpConfig()


def mlp_net(cfg: MlpConfig) -> type[Network]:
    from plastax_b200 import optim
    from plastax_b200.traits import BackwardPass, MeanFloatFirstRest, SoftmaxCrossEntropyLoss

    class SparseMLP(Network):
        forward_pass = ForwardPass("relu", monoid.sum_, output_activation="identity")
        backward_pass = BackwardPass("relu")
        loss = SoftmaxCrossEntropyLoss()
        update_conn = optim.sgd(cfg.lr)
        batch_reduction = MeanFloatFirstRest()
        propagation = Propagation.TOPOLOGICAL
        seed = cfg.seed

    return SparseMLP


def mlp_edges(cfg: MlpConfig):
    """(src, dst, weight) numpy arrays of the MLP, seeded."""
    import numpy as np

    rng = np.random.default_rng(cfg.seed)
    off = np.concatenate([[0], np.cumsum(cfg.layers)])
    src, dst = [], []
    for layer in range(len(cfg.layers) - 1):
        a = np.arange(off[layer], off[layer + 1], dtype=np.int32)
        b = np.arange(off[layer + 1], off[layer + 2], dtype=np.int32)
        keep = rng.random((a.size, b.size)) < cfg.density
        s, d = np.nonzero(keep)
        src.append(a[s])
        dst.append(b[d])
    src, dst = np.concatenate(src), np.concatenate(dst)
    fan_in = np.bincount(dst, minlength=cfg.num_units).astype(np.float64)
    bound = np.sqrt(6.0 / np.maximum(fan_in[dst], 1.0))
    w = (rng.uniform(-1.0, 1.0, src.size) * bound).astype(np.float32)
    return src, dst, w


def build_mlp(cfg: MlpConfig = C2, device: torch.device | str = "cuda"):
    net = mlp_net(cfg)
    src, dst, w = mlp_edges(cfg)
    n = cfg.num_units
    static, state = NetworkBuilder.from_edges(net, n, src, dst, weights=w, input_ids=tuple(range(cfg.layers[0])),
                                              output_ids=tuple(range(n - cfg.layers[-1], n)), device=device)
    return net, static, state


def mlp_batch(cfg: MlpConfig, rng):
    """One batch: N(0, 1) inputs (B, 784) and one-hot uniform labels (B, 10)."""
    import numpy as np

    x = rng.standard_normal((cfg.batch, cfg.layers[0])).astype(np.float32)
    labels = rng.integers(0, cfg.layers[-1], cfg.batch)
    t = np.zeros((cfg.batch, cfg.layers[-1]), np.float32)
    t[np.arange(cfg.batch), labels] = 1.0
    return x, t


@dataclasses.dataclass(frozen=True)
class DstConfig:
    """Dynamic sparse training, streaming (PIPELINE): 64 inputs, 4,096 tanh
    hidden units and 8 linear outputs; 2^20 live edges with uniform sources
    (any unit) and uniform non-input destinations, no self-loops, weights
    N(0, 1 / fan_in(dst)), capacity 2^21; MSE against a fixed random teacher
    MLP 64-256-8 (tanh hidden, seed 1) on N(0, 1) inputs; SGD. Every `every`
    steps the 1% live edges of lowest |w| are pruned (ties by slot) and as
    many regrown from 64 per-unit proposals (src = the unit, dst uniform over
    the non-input units) scored |grad[dst] * act[src]|, new weights 0."""

    num_inputs: int = 64
    hidden: int = 4096
    num_outputs: int = 8
    live: int = 1 << 20
    teacher_hidden: int = 256
    lr: float = 1e-3
    churn: float = 0.01
    every: int = 100
    proposals: int = 64
    seed: int = 0

    @property
    def num_units(self) -> int:
        return self.num_inputs + self.hidden + self.num_outputs

    @property
    def k(self) -> int:
        return int(round(self.churn * self.live))


C3 = DstConfig()


def dst_net(cfg: DstConfig) -> type[Network]:
    from plastax_b200 import optim
    from plastax_b200.traits import BackwardPass, MSELoss

    class DynamicSparseTraining(Network):
        forward_pass = ForwardPass("tanh", monoid.sum_, output_activation="identity")
        backward_pass = BackwardPass("tanh")
        loss = MSELoss()
        update_conn = optim.sgd(cfg.lr)
        prune_conn = LowestMagnitudePrune(cfg.k, every=cfg.every)
        add_conn = ProposeAddConn(proposals_per_proposer=cfg.proposals, max_new_per_level=cfg.k,
                                  dst_lo=cfg.num_inputs, score="grad_act", level_cap_scope="step",
                                  trigger=("every", cfg.every))
        propagation = Propagation.PIPELINE
        seed = cfg.seed

    return DynamicSparseTraining


def dst_edges(cfg: DstConfig):
    import numpy as np

    rng = np.random.default_rng(cfg.seed)
    n = cfg.num_units
    dst = rng.integers(cfg.num_inputs, n, cfg.live).astype(np.int32)
    src = rng.integers(0, n - 1, cfg.live).astype(np.int32)
    src = src + (src >= dst)  # uniform over every unit but the destination
    fan_in = np.bincount(dst, minlength=n).astype(np.float64)
    w = (rng.standard_normal(cfg.live) / np.sqrt(np.maximum(fan_in[dst], 1.0))).astype(np.float32)
    return src.astype(np.int32), dst, w


def dst_teacher(cfg: DstConfig):
    """The teacher MLP's weights (seed 1): W1 (256, 64) N(0, 1/64), W2 (8, 256)
    N(0, 1/256); targets = W2 tanh(W1 x)."""
    import numpy as np

    rng = np.random.default_rng(1)
    w1 = (rng.standard_normal((cfg.teacher_hidden, cfg.num_inputs)) / np.sqrt(cfg.num_inputs)).astype(np.float32)
    w2 = (rng.standard_normal((cfg.num_outputs, cfg.teacher_hidden)) / np.sqrt(cfg.teacher_hidden)).astype(np.float32)
    return w1, w2


def build_dst(cfg: DstConfig = C3, device: torch.device | str = "cuda"):
    net = dst_net(cfg)
    src, dst, w = dst_edges(cfg)
    n = cfg.num_units
    static, state = NetworkBuilder.from_edges(net, n, src, dst, weights=w, input_ids=tuple(range(cfg.num_inputs)),
                                              output_ids=tuple(range(n - cfg.num_outputs, n)),
                                              capacity_headroom=0.01, device=device)
    return net, static, state


@dataclasses.dataclass(frozen=True)
class UnitsConfig:
    """Unit addition and pruning (TOPOLOGICAL, single device): 32 inputs, 8,159
    ReLU hidden units and 1 linear output live at start (8,192 of 65,536 unit
    slots); every hidden unit fed by every input, the output by every hidden
    unit (fan-in 32 into the hidden layer), weights N(0, 0.1^2), edge capacity
    2^22; MSE against a random linear map of the inputs, resampled every
    5,000 steps; UPGD connection updates; a utility trace per unit; every 10
    steps one unit spawns from the highest-utility parent and the units below
    the 1st utility percentile are pruned; per-unit proposals (8 per unit,
    deeper, uniform score) regrow up to 256 edges per source level."""

    num_inputs: int = 32
    live_units: int = 8192
    unit_capacity: int = 65536
    edge_capacity_log2: int = 22
    lr: float = 0.01
    beta: float = 0.99
    sigma: float = 0.001
    interval: int = 10
    proposals: int = 8
    max_new: int = 256
    resample: int = 5000
    seed: int = 0


C4 = UnitsConfig()


def units_net(cfg: UnitsConfig) -> type[Network]:
    from plastax_b200 import optim
    from plastax_b200.traits import ArgmaxSpawn, BackwardPass, FieldBelowPrune, MSELoss, TraceUnitUpdate
    from plastax_b200.types import FieldSpec

    trace = FieldSpec.float32("utility")

    class UnitLifecycle(Network):
        forward_pass = ForwardPass("relu", monoid.sum_, output_activation="identity")
        backward_pass = BackwardPass("relu")
        loss = MSELoss()
        update_conn = optim.upgd(lr=cfg.lr, beta=cfg.beta, sigma=cfg.sigma)
        update_unit = TraceUnitUpdate(trace, "activation", 0.05)
        prune_unit = FieldBelowPrune(trace, quantile=0.01)
        add_unit = ArgmaxSpawn(trace, offset=1)
        add_conn = ProposeAddConn(proposals_per_proposer=cfg.proposals, max_new_per_level=cfg.max_new,
                                  dst_lo=cfg.num_inputs, score="uniform", max_level_gap=2, direction="deeper")
        extra_unit_fields = (trace,)
        unit_capacity = cfg.unit_capacity
        structural_interval = cfg.interval
        propagation = Propagation.TOPOLOGICAL
        seed = cfg.seed

    return UnitLifecycle


def units_edges(cfg: UnitsConfig):
    import numpy as np

    rng = np.random.default_rng(cfg.seed)
    n = cfg.live_units
    hidden = np.arange(cfg.num_inputs, n - 1, dtype=np.int32)
    src = np.concatenate([np.tile(np.arange(cfg.num_inputs, dtype=np.int32), hidden.size), hidden])
    dst = np.concatenate([np.repeat(hidden, cfg.num_inputs), np.full(hidden.size, n - 1, np.int32)])
    w = (rng.standard_normal(src.size) * 0.1).astype(np.float32)
    return src, dst, w


def build_units(cfg: UnitsConfig = C4, device: torch.device | str = "cuda"):
    net = units_net(cfg)
    src, dst, w = units_edges(cfg)
    n = cfg.live_units
    cap = 1 << cfg.edge_capacity_log2
    static, state = NetworkBuilder.from_edges(net, n, src, dst, weights=w, input_ids=tuple(range(cfg.num_inputs)),
                                              output_ids=(n - 1,), capacity_headroom=cap / src.size - 1.0,
                                              device=device)
    return net, static, state


def units_target_map(cfg: UnitsConfig, phase: int):
    """The linear target map of the inputs for steps [phase * resample, ...)."""
    import numpy as np

    rng = np.random.default_rng(1000 + phase)
    return (rng.standard_normal(cfg.num_inputs) / np.sqrt(cfg.num_inputs)).astype(np.float32)
