// The fused pipeline training step: forward + backward accumulation in one
// pass over the arena, the unit applies and the MSE seed, then the update.
//
// In a PIPELINE step both propagation sums read only the previous step's
// unit columns (src/plastax/sweep.py:300-340, :402-450): the forward sums
// w * act[src] into destinations, the backward sums w * grad[dst] into
// sources, and neither reads what the other writes. So one pass over the
// bucket feeds both, and the canonical source-major order costs nothing:
// every CTA holds all units' accumulators for both sums in shared memory
// (exact fixed point, fixed.cuh), so no edge issues a global atomic. A
// thread-block cluster then reduces its CTAs' accumulators through
// distributed shared memory into one int64 row per cluster. The second
// kernel sums the rows per unit and applies; the third applies the
// optimizer to every live edge (src/plastax/phases.py:488-532).
#include <cooperative_groups.h>

#include "fixed.cuh"
#include "optim.cuh"

namespace cg = cooperative_groups;

namespace pxb {
namespace {

constexpr int kTrainFrac = 31;        // fractional bits of the shared words
constexpr int kAccThreads = 1024;     // accumulate kernel: one CTA per SM
constexpr int kMaxRows = 40;          // clusters (int64 rows) at most
constexpr int kApplyThreads = 256;
constexpr int kUpdateThreads = 512;
constexpr int64_t kSmemCap = 227 * 1024;

static_assert(PXB_FIXED_FRAC_BITS == kTrainFrac, "the rows are in the global accumulator's unit");

struct Scratch {
  int64_t *rows;   // [kMaxRows][2N]: forward sums, then backward sums
  float *side;     // [2N]: the float side of each sum (kept zero between steps)
};

inline Scratch scratch_of(void *base, int32_t n) {
  char *p = static_cast<char *>(base);
  Scratch s;
  s.rows = reinterpret_cast<int64_t *>(p);
  p += sizeof(int64_t) * kMaxRows * 2 * static_cast<int64_t>(n);
  s.side = reinterpret_cast<float *>(p);
  return s;
}

inline int64_t scratch_bytes(int32_t n) {
  return sizeof(int64_t) * kMaxRows * 2 * static_cast<int64_t>(n) + sizeof(float) * 2 * static_cast<int64_t>(n) +
         64;
}

// The edge's liveness exactly as the canonical sweeps test it.
__device__ __forceinline__ bool live_edge(uint8_t dead, int32_t f, int32_t t, uint32_t n) {
  return !dead && static_cast<uint32_t>(f) < n && static_cast<uint32_t>(t) < n;
}

template <bool BWD>
__device__ __forceinline__ void acc_edge(int32_t *fwd, int32_t *bwd, float *side_f, float *side_b, int32_t n,
                                         const float *__restrict__ act, const float *__restrict__ grad, uint8_t d,
                                         int32_t f, int32_t t, float w) {
  if (!live_edge(d, f, t, static_cast<uint32_t>(n))) return;
  fixed_add<kTrainFrac>(fwd + t, fwd + n + t, side_f + t, __fmul_rn(w, __ldg(act + f)));
  if (BWD) fixed_add<kTrainFrac>(bwd + f, bwd + n + f, side_b + f, __fmul_rn(w, __ldg(grad + t)));
}

// One CTA's sweep of slots [lo, hi) into its shared accumulators (lo a
// multiple of four slots, so the column bases stay 16-byte aligned).
template <bool BWD>
__device__ __forceinline__ void sweep_slots(int32_t *fwd, int32_t *bwd, float *side_f, float *side_b, int32_t n,
                                            const float *__restrict__ act, const float *__restrict__ grad,
                                            const int32_t *__restrict__ from, const int32_t *__restrict__ to,
                                            const uint8_t *__restrict__ dead, const float *__restrict__ weight,
                                            int64_t lo, int64_t hi) {
  // 16-byte loads of four slots (per_cta and the column bases are multiples
  // of four slots / 16 bytes), two groups in flight per thread
  const int64_t vec_end = lo + ((hi > lo ? hi - lo : 0) & ~int64_t(3));
  const int64_t step = 4 * static_cast<int64_t>(blockDim.x);
  for (int64_t s = lo + 4 * threadIdx.x; s < vec_end; s += 2 * step) {
    const bool two = s + step < vec_end;
    const int4 f0 = *reinterpret_cast<const int4 *>(from + s);
    const int4 t0 = *reinterpret_cast<const int4 *>(to + s);
    const float4 w0 = *reinterpret_cast<const float4 *>(weight + s);
    const uint32_t d0 = *reinterpret_cast<const uint32_t *>(dead + s);
    int4 f1 = make_int4(-1, -1, -1, -1), t1 = f1;
    float4 w1 = make_float4(0.f, 0.f, 0.f, 0.f);
    uint32_t d1 = 0x01010101u;
    if (two) {
      f1 = *reinterpret_cast<const int4 *>(from + s + step);
      t1 = *reinterpret_cast<const int4 *>(to + s + step);
      w1 = *reinterpret_cast<const float4 *>(weight + s + step);
      d1 = *reinterpret_cast<const uint32_t *>(dead + s + step);
    }
    // every gather of the eight slots issued before the first atomic
    const int32_t ff[8] = {f0.x, f0.y, f0.z, f0.w, f1.x, f1.y, f1.z, f1.w};
    const int32_t tt[8] = {t0.x, t0.y, t0.z, t0.w, t1.x, t1.y, t1.z, t1.w};
    const float ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
    bool lv[8];
    float pa[8], pg[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t dj = ((j < 4 ? d0 : d1) >> (8 * (j & 3))) & 0xffu;
      lv[j] = live_edge(static_cast<uint8_t>(dj), ff[j], tt[j], static_cast<uint32_t>(n));
      pa[j] = lv[j] ? __ldg(act + ff[j]) : 0.0f;
      pg[j] = (BWD && lv[j]) ? __ldg(grad + tt[j]) : 0.0f;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (!lv[j]) continue;
      fixed_add<kTrainFrac>(fwd + tt[j], fwd + n + tt[j], side_f + tt[j], __fmul_rn(ww[j], pa[j]));
      if (BWD) fixed_add<kTrainFrac>(bwd + ff[j], bwd + n + ff[j], side_b + ff[j], __fmul_rn(ww[j], pg[j]));
    }
  }
  for (int64_t s = vec_end + threadIdx.x; s < hi; s += blockDim.x)
    acc_edge<BWD>(fwd, bwd, side_f, side_b, n, act, grad, dead[s], from[s], to[s], weight[s]);

}

// Kernel 1: every CTA sweeps a contiguous slot range into its shared
// accumulators (forward lo[N] hi[N], backward lo[N] hi[N]); the cluster's
// CTAs then split the units and each sums its share over every CTA of the
// cluster (distributed shared memory) into the cluster's int64 row.
template <bool BWD>
__global__ void __launch_bounds__(kAccThreads, 1)
    train_accumulate_kernel(int64_t cap, const int32_t *__restrict__ from, const int32_t *__restrict__ to,
                            const uint8_t *__restrict__ dead, const float *__restrict__ weight,
                            const float *__restrict__ act, const float *__restrict__ grad, int32_t n,
                            const int64_t *__restrict__ tail, Scratch sc) {
  extern __shared__ int32_t smem[];
  int32_t *fwd = smem;              // lo[n], hi[n]
  int32_t *bwd = smem + 2 * n;      // lo[n], hi[n] (BWD)
  const int words = (BWD ? 4 : 2) * n;
  for (int i = threadIdx.x; i < words; i += blockDim.x) smem[i] = 0;
  __syncthreads();
  float *side_f = sc.side, *side_b = sc.side + n;

  // the swept slots: the capacity, or up to the arena's tail
  int64_t limit = cap;
  if (tail != nullptr) {
    const int64_t ts = *tail;
    limit = ts < 0 ? 0 : (ts < cap ? ts : cap);
  }
  const int64_t per_cta = ((limit + gridDim.x - 1) / gridDim.x + 3) & ~int64_t(3);
  const int64_t lo = static_cast<int64_t>(blockIdx.x) * per_cta;
  const int64_t hi = lo + per_cta < limit ? lo + per_cta : limit;
  sweep_slots<BWD>(fwd, bwd, side_f, side_b, n, act, grad, from, to, dead, weight, lo, hi);

  cg::cluster_group cluster = cg::this_cluster();
  cluster.sync();  // every CTA of the cluster has swept
  const int cs = static_cast<int>(cluster.num_blocks());
  const int rank = static_cast<int>(cluster.block_rank());
  const int64_t row = blockIdx.x / cs;
  int64_t *out = sc.rows + row * 2 * static_cast<int64_t>(n);
  const int32_t share = (n + cs - 1) / cs;
  const int32_t u0 = rank * share;
  const int32_t u1 = u0 + share < n ? u0 + share : n;
  for (int32_t u = u0 + threadIdx.x; u < u1; u += blockDim.x) {
    long long tf = 0, tb = 0;
#pragma unroll
    for (int q = 0; q < 8; ++q) {  // cluster sizes 2, 4 or 8: every peer's loads in flight at once
      if (q >= cs) break;
      const int32_t *peer = cluster.map_shared_rank(smem, q);
      tf += (static_cast<long long>(peer[n + u]) << kTrainFrac) + peer[u];
      if (BWD) tb += (static_cast<long long>(peer[3 * n + u]) << kTrainFrac) + peer[2 * n + u];
    }
    out[u] = tf;
    out[n + u] = tb;
  }
  cluster.sync();  // no CTA leaves while a peer reads its shared memory
}

struct ApplyArgs {
  int32_t n, rows, num_outputs;
  float *act, *grad, *seed;
  const uint8_t *roles, *pruned;
  int32_t fwd_act, bwd_act;
  const int32_t *target_of, *output_ids;
  const float *target;
  float *loss;
};

struct LossArgs {
  int32_t num_outputs;
  const int32_t *output_ids;
  const float *seed;
  float *loss;
};

constexpr int kRowLanes = 8;  // lanes summing one unit's rows
constexpr int kApplyUnits = kApplyThreads / kRowLanes;

// A unit's exact sum over the cluster rows, read by kRowLanes lanes at once
// (rows lane, lane + 8, ...), combined by shuffles: every lane returns it.
__device__ __forceinline__ long long rows_sum(const int64_t *rows, int32_t rows_n, int64_t stride, int64_t u,
                                              int lane, bool in) {
  long long f = 0;
  if (in) {
#pragma unroll 4
    for (int r = lane; r < rows_n; r += kRowLanes) f += rows[r * stride + u];
  }
#pragma unroll
  for (int o = kRowLanes / 2; o > 0; o >>= 1) f += __shfl_xor_sync(0xffffffffu, f, o);
  return f;
}

// The exact sum rounded once plus the float side (read and reset), as
// pxb_unit_apply rounds a fixed-point accumulator.
__device__ __forceinline__ float round_sum(long long f, float *side) {
  float a = *side;
  if (a != 0.0f) *side = 0.0f;
  if (f != 0) a = __fadd_rn(__fmul_rn(__ll2float_rn(f), 1.0f / float(1ll << kTrainFrac)), a);
  return a;
}

// One unit's applies from its exact sums (ff forward, fb backward): the
// forward apply (inputs and pruned kept, src/plastax/sweep.py:332-338), the
// MSE seed of an output, the backward apply (every unit but the pruned,
// :444-449). side_f / side_b are the unit's float sides (read and reset).
template <bool BWD>
__device__ __forceinline__ void apply_unit(const ApplyArgs &a, int32_t u, long long ff, long long fb, float *side_f,
                                           float *side_b) {
  const uint8_t role = a.roles ? a.roles[u] : 0;
  const bool pr = a.pruned != nullptr && a.pruned[u];
  const float fa = round_sum(ff, side_f);
  float act = a.act[u];
  if (role != 1 && !pr) {
    act = act_fn(unit_act_kind(a.fwd_act, role), fa);
    a.act[u] = act;
  }
  float s = 0.0f;
  if (a.seed != nullptr) {
    const int32_t j = a.target_of[u];
    if (j >= 0 && a.target != nullptr) {
      s = __fsub_rn(act, a.target[j]);
      a.seed[u] = s;
    } else {
      s = a.seed[u];
    }
  }
  if (BWD) {
    const float ba = round_sum(fb, side_b);
    if (!pr) {
      const uint8_t brole = role == 1 ? 0 : role;
      a.grad[u] = __fmul_rn(__fadd_rn(ba, s), act_prime_from_act(unit_act_kind(a.bwd_act, brole), act));
    }
  }
}

// Kernel 2: per unit the forward apply (inputs and pruned kept,
// src/plastax/sweep.py:332-338), the MSE seed of an output, the backward
// apply (every unit but the pruned, :444-449).
template <bool BWD>
__global__ void __launch_bounds__(kApplyThreads) train_apply_kernel(ApplyArgs a, Scratch sc) {
  const int lane = threadIdx.x % kRowLanes;
  const int32_t u = blockIdx.x * kApplyUnits + threadIdx.x / kRowLanes;
  const bool in = u < a.n;
  const int64_t stride = 2 * static_cast<int64_t>(a.n);
  const long long ff = rows_sum(sc.rows, a.rows, stride, u, lane, in);
  long long fb = 0;
  if (BWD) fb = rows_sum(sc.rows + a.n, a.rows, stride, u, lane, in);
  if (in && lane == 0) apply_unit<BWD>(a, u, ff, fb, sc.side + u, sc.side + a.n + u);
}

// COHERENT: the unit columns were written earlier in the same kernel (by
// other CTAs of its cluster), so they are read through L2, not the
// read-only path.
template <bool COHERENT = false>
__device__ __forceinline__ void update_edge(const OptParams &p, float *__restrict__ weight, float *m_col,
                                            float *v_col, float *t_col, const float *__restrict__ act,
                                            const float *__restrict__ ug, uint32_t n, int64_t s, uint8_t d,
                                            int32_t f, int32_t t, float w) {
  if (!live_edge(d, f, t, n)) return;
  const float g = COHERENT ? __fmul_rn(__ldcg(ug + t), __ldcg(act + f)) : __fmul_rn(__ldg(ug + t), __ldg(act + f));
  opt_step(p, g, w, m_col, v_col, t_col, s, f, t);
  weight[s] = w;
}

// The MSE loss in output order (as pxb_mse_loss), by one warp: the seeds
// loaded 32 at a time, summed in order by lane 0.
__device__ __forceinline__ void loss_warp(const LossArgs &l) {
  const int lane = threadIdx.x & 31;
  float total = 0.0f;
  for (int32_t base = 0; base < l.num_outputs; base += 32) {
    const int32_t i = base + lane;
    const float d = i < l.num_outputs ? __ldcg(l.seed + l.output_ids[i]) : 0.0f;  // through L2: written by other CTAs
    const float sq = __fmul_rn(__fmul_rn(0.5f, d), d);
    const int cnt = l.num_outputs - base < 32 ? l.num_outputs - base : 32;
    for (int j = 0; j < cnt; ++j) {
      const float v = __shfl_sync(0xffffffffu, sq, j);
      if (lane == 0) total = __fadd_rn(total, v);
    }
  }
  if (lane == 0) l.loss[0] = total;
}

// Kernel 3: the optimizer on every live edge below the tail, grid-stride
// over 4-slot groups with 16-byte loads, two groups in flight per thread;
// block 0's first warp also sums the loss (the seeds are final: the apply
// kernel has completed).
__global__ void __launch_bounds__(kUpdateThreads, 2)
    train_update_kernel(int64_t cap, const int32_t *__restrict__ from, const int32_t *__restrict__ to,
                        const uint8_t *__restrict__ dead, float *__restrict__ weight, float *m_col, float *v_col,
                        float *t_col, const float *__restrict__ act, const float *__restrict__ ug, uint32_t n,
                        const int64_t *__restrict__ tail, OptParams p, LossArgs l) {
  if (l.loss != nullptr && blockIdx.x == 0 && threadIdx.x < 32) loss_warp(l);
  if (tail != nullptr) {
    const int64_t ts = *tail;
    cap = ts < 0 ? 0 : (ts < cap ? ts : cap);
  }
  const int64_t groups = cap >> 2;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t g = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; g < groups; g += 2 * stride) {
    const bool two = g + stride < groups;
    const int64_t s0 = g << 2, s1 = (g + stride) << 2;
    const int4 f0 = *reinterpret_cast<const int4 *>(from + s0);
    const int4 t0 = *reinterpret_cast<const int4 *>(to + s0);
    const float4 w0 = *reinterpret_cast<const float4 *>(weight + s0);
    const uint32_t d0 = *reinterpret_cast<const uint32_t *>(dead + s0);
    int4 f1 = make_int4(-1, -1, -1, -1), t1 = f1;
    float4 w1 = make_float4(0.f, 0.f, 0.f, 0.f);
    uint32_t d1 = 0x01010101u;
    if (two) {
      f1 = *reinterpret_cast<const int4 *>(from + s1);
      t1 = *reinterpret_cast<const int4 *>(to + s1);
      w1 = *reinterpret_cast<const float4 *>(weight + s1);
      d1 = *reinterpret_cast<const uint32_t *>(dead + s1);
    }
    update_edge(p, weight, m_col, v_col, t_col, act, ug, n, s0, d0 & 0xff, f0.x, t0.x, w0.x);
    update_edge(p, weight, m_col, v_col, t_col, act, ug, n, s0 + 1, (d0 >> 8) & 0xff, f0.y, t0.y, w0.y);
    update_edge(p, weight, m_col, v_col, t_col, act, ug, n, s0 + 2, (d0 >> 16) & 0xff, f0.z, t0.z, w0.z);
    update_edge(p, weight, m_col, v_col, t_col, act, ug, n, s0 + 3, d0 >> 24, f0.w, t0.w, w0.w);
    update_edge(p, weight, m_col, v_col, t_col, act, ug, n, s1, d1 & 0xff, f1.x, t1.x, w1.x);
    update_edge(p, weight, m_col, v_col, t_col, act, ug, n, s1 + 1, (d1 >> 8) & 0xff, f1.y, t1.y, w1.y);
    update_edge(p, weight, m_col, v_col, t_col, act, ug, n, s1 + 2, (d1 >> 16) & 0xff, f1.z, t1.z, w1.z);
    update_edge(p, weight, m_col, v_col, t_col, act, ug, n, s1 + 3, d1 >> 24, f1.w, t1.w, w1.w);
  }
  const int64_t rest = groups << 2;
  const int64_t s = rest + blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (s < cap) update_edge(p, weight, m_col, v_col, t_col, act, ug, n, s, dead[s], from[s], to[s], weight[s]);
}

// The whole step in one launch for a small arena: one cluster of
// kSmallCluster CTAs. Each CTA sweeps its slot range into its shared
// accumulators; after a cluster barrier each CTA applies its share of the
// units, summing every CTA's accumulators through distributed shared memory;
// after a second barrier (its release / acquire orders the unit columns'
// global writes for the whole cluster) each CTA updates the slots it swept
// and one warp sums the loss. The barriers are the cluster's hardware
// barrier: every thread of every CTA takes both.
constexpr int kSmallCluster = 8;
constexpr int64_t kSmallSlots = 1 << 16;  // the arenas this path takes

template <bool BWD>
__global__ void __launch_bounds__(kAccThreads, 1)
    train_cluster_kernel(int64_t cap, const int32_t *__restrict__ from, const int32_t *__restrict__ to,
                         const uint8_t *__restrict__ dead, float *__restrict__ weight, float *m_col, float *v_col,
                         float *t_col, const int64_t *__restrict__ tail, ApplyArgs a, const float *ug, OptParams p,
                         LossArgs l, Scratch sc) {
  extern __shared__ int32_t smem[];
  const int32_t n = a.n;
  int32_t *fwd = smem;
  int32_t *bwd = smem + 2 * n;
  const int words = (BWD ? 4 : 2) * n;
  for (int i = threadIdx.x; i < words; i += blockDim.x) smem[i] = 0;
  __syncthreads();
  int64_t limit = cap;
  if (tail != nullptr) {
    const int64_t ts = *tail;
    limit = ts < 0 ? 0 : (ts < cap ? ts : cap);
  }
  cg::cluster_group cluster = cg::this_cluster();
  const int cs = static_cast<int>(cluster.num_blocks());
  const int rank = static_cast<int>(cluster.block_rank());
  const int64_t per = ((limit + cs - 1) / cs + 3) & ~int64_t(3);
  const int64_t lo = rank * per;
  const int64_t hi = lo + per < limit ? lo + per : limit;
  sweep_slots<BWD>(fwd, bwd, sc.side, sc.side + n, n, a.act, a.grad, from, to, dead, weight, lo, hi);
  cluster.sync();  // every CTA has swept
  const int32_t share = (n + cs - 1) / cs;
  const int32_t u0 = rank * share;
  const int32_t u1 = u0 + share < n ? u0 + share : n;
  for (int32_t u = u0 + threadIdx.x; u < u1; u += blockDim.x) {
    long long ff = 0, fb = 0;
#pragma unroll
    for (int q = 0; q < kSmallCluster; ++q) {
      if (q >= cs) break;
      const int32_t *peer = cluster.map_shared_rank(smem, q);
      ff += (static_cast<long long>(peer[n + u]) << kTrainFrac) + peer[u];
      if (BWD) fb += (static_cast<long long>(peer[3 * n + u]) << kTrainFrac) + peer[2 * n + u];
    }
    apply_unit<BWD>(a, u, ff, fb, sc.side + u, sc.side + n + u);
  }
  cluster.sync();  // every unit is applied; no CTA reads a peer's shared memory after this
  if (l.loss != nullptr && rank == 0 && threadIdx.x < 32) loss_warp(l);
  for (int64_t s = lo + threadIdx.x; s < hi; s += blockDim.x)
    update_edge<true>(p, weight, m_col, v_col, t_col, a.act, ug, static_cast<uint32_t>(n), s, dead[s], from[s],
                      to[s], weight[s]);
}

int32_t max_units(bool bwd) {
  return static_cast<int32_t>((kSmemCap - 1024) / ((bwd ? 4 : 2) * sizeof(int32_t)));
}

// The cluster size and count of the accumulate launch: the largest number
// of co-resident CTAs (fewer rows to sum on ties), at most kMaxRows rows.
struct AccShape {
  int cs, clusters;
};

template <typename K>
int occupancy_shape(K kern, size_t smem, cudaStream_t st, int32_t n, AccShape *out) {
  AccShape best{1, 1};
  int best_ctas = 0;
  for (int cs : {8, 4, 2}) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(cs * kMaxRows);
    cfg.blockDim = dim3(kAccThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = cs;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess) {
      cudaGetLastError();
      continue;
    }
    clusters = clusters < kMaxRows ? clusters : kMaxRows;
    if (clusters * cs > best_ctas) {
      best_ctas = clusters * cs;
      best = AccShape{cs, clusters};
    }
  }
  PXB_REQUIRE(best_ctas > 0, "pxb_pipeline_train_step: no cluster shape fits the accumulators of %d units", n);
  *out = best;
  return PXB_OK;
}

template <bool BWD>
int acc_shape(int64_t cap, int32_t n, size_t smem, cudaStream_t st, AccShape *out) {
  // the shape depends only on the shared memory size and the device: kept
  // for the last (device, size) so a step launches without queries
  static thread_local int cached_dev = -1;
  static thread_local size_t cached_smem = 0;
  static thread_local AccShape cached{0, 0};
  int dev = 0;
  PXB_CUDA(cudaGetDevice(&dev));
  auto kern = train_accumulate_kernel<BWD>;
  if (dev != cached_dev || smem != cached_smem) {
    PXB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
    AccShape s{0, 0};
    int rc = occupancy_shape(kern, smem, st, n, &s);
    if (rc) return rc;
    cached_dev = dev;
    cached_smem = smem;
    cached = s;
  }
  AccShape best = cached;
  // no more CTAs than slots to keep each one busy (>= 2048 slots per CTA)
  const int64_t want = (cap + 2047) / 2048;
  while (best.clusters > 1 && static_cast<int64_t>(best.clusters - 1) * best.cs >= want) --best.clusters;
  *out = best;
  return PXB_OK;
}

template <bool BWD>
int launch_accumulate(const pxb_pipeline_train *t, const Scratch &sc, cudaStream_t st, int *rows) {
  const size_t smem = static_cast<size_t>(BWD ? 4 : 2) * t->num_units * sizeof(int32_t);
  AccShape sh;
  int rc = acc_shape<BWD>(t->cap, t->num_units, smem, st, &sh);
  if (rc) return rc;
  const int ctas = sh.cs * sh.clusters;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ctas);
  cfg.blockDim = dim3(kAccThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = sh.cs;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  PXB_CUDA(cudaLaunchKernelEx(&cfg, train_accumulate_kernel<BWD>, t->cap, t->from_id, t->to_id, t->dead,
                              static_cast<const float *>(t->weight), static_cast<const float *>(t->act),
                              static_cast<const float *>(t->grad), t->num_units, t->tail_start, sc));
  *rows = sh.clusters;
  return PXB_OK;
}

}  // namespace
}  // namespace pxb

using namespace pxb;

extern "C" int32_t pxb_pipeline_train_max_units(int32_t with_backward) { return max_units(with_backward != 0); }

extern "C" int pxb_pipeline_train_scratch_bytes(int32_t num_units, size_t *bytes) {
  PXB_REQUIRE(bytes != nullptr, "pxb_pipeline_train_scratch_bytes: NULL output");
  PXB_REQUIRE(num_units >= 0, "pxb_pipeline_train_scratch_bytes: negative num_units");
  *bytes = static_cast<size_t>(scratch_bytes(num_units));
  return PXB_OK;
}

extern "C" int pxb_pipeline_train_step(const pxb_pipeline_train *t, void *stream) {
  PXB_REQUIRE(t != nullptr, "pxb_pipeline_train_step: NULL descriptor");
  const bool bwd = t->grad != nullptr;
  const int32_t n = t->num_units;
  PXB_REQUIRE(n > 0 && n <= max_units(bwd), "pxb_pipeline_train_step: num_units %d outside [1, %d]", n,
              max_units(bwd));
  PXB_REQUIRE(t->cap >= 0 && t->cap < (int64_t(1) << 40), "pxb_pipeline_train_step: capacity out of range");
  PXB_REQUIRE(t->from_id && t->to_id && t->dead && t->weight && t->act && t->update_grad && t->scratch,
              "pxb_pipeline_train_step: a column or the scratch is NULL");
  PXB_REQUIRE(aligned16(t->from_id) && aligned16(t->to_id) && aligned16(t->weight) &&
                  (reinterpret_cast<uintptr_t>(t->dead) & 3u) == 0 && aligned16(t->scratch),
              "pxb_pipeline_train_step: the bucket columns need 16-byte aligned bases (dead: 4-byte)");
  PXB_REQUIRE(act_code_ok(t->fwd_act) && (!bwd || act_code_ok(t->bwd_act)),
              "pxb_pipeline_train_step: unknown activation code");
  const pxb_optimizer &o = t->opt;
  PXB_REQUIRE(o.kind >= PXB_OPT_SGD && o.kind <= PXB_OPT_RMSPROP,
              "pxb_pipeline_train_step: optimizer kind %d is not fused (UPGD needs its scale sweep)", o.kind);
  PXB_REQUIRE(o.kind != PXB_OPT_MOMENTUM || t->opt_v, "pxb_pipeline_train_step: momentum needs opt_v");
  PXB_REQUIRE(o.kind != PXB_OPT_ADAM || (t->opt_m && t->opt_v && t->opt_t),
              "pxb_pipeline_train_step: adam needs opt_m, opt_v and opt_t");
  PXB_REQUIRE(o.kind != PXB_OPT_RMSPROP || t->opt_v, "pxb_pipeline_train_step: rmsprop needs opt_v");
  PXB_REQUIRE(!t->seed || (t->target_of && (t->num_outputs == 0 || t->output_ids)),
              "pxb_pipeline_train_step: a loss needs target_of and output_ids");
  PXB_REQUIRE(!t->loss || t->seed, "pxb_pipeline_train_step: the loss needs the seed column");
  cudaStream_t st = as_stream(stream);
  const Scratch sc = scratch_of(t->scratch, n);
  const OptParams p{o.kind, o.lr, o.b1, o.b2, o.eps, o.weight_decay, nullptr};
  const LossArgs l{t->num_outputs, t->output_ids, t->seed, t->loss};
  if (t->cap <= kSmallSlots) {
    // a small arena: the whole step as one cluster
    ApplyArgs a{n,         0,          t->num_outputs, t->act,     t->grad,       t->seed,
                t->roles,  t->pruned,  t->fwd_act,     t->bwd_act, t->target_of,  t->output_ids,
                t->target, t->loss};
    const size_t smem = static_cast<size_t>(bwd ? 4 : 2) * n * sizeof(int32_t);
    auto kern = bwd ? train_cluster_kernel<true> : train_cluster_kernel<false>;
    PXB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kSmallCluster);
    cfg.blockDim = dim3(kAccThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = kSmallCluster;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    PXB_CUDA(cudaLaunchKernelEx(&cfg, kern, t->cap, t->from_id, t->to_id, t->dead, t->weight, t->opt_m, t->opt_v,
                                t->opt_t, t->tail_start, a, static_cast<const float *>(t->update_grad), p, l, sc));
    PXB_LAUNCHED("train_cluster_kernel");
    return PXB_OK;
  }
  int rows = 0;
  int rc = bwd ? launch_accumulate<true>(t, sc, st, &rows) : launch_accumulate<false>(t, sc, st, &rows);
  if (rc) return rc;
  PXB_LAUNCHED("train_accumulate_kernel");
  ApplyArgs a{n,         rows,       t->num_outputs, t->act,    t->grad,         t->seed,
              t->roles,  t->pruned,  t->fwd_act,     t->bwd_act, t->target_of,   t->output_ids,
              t->target, t->loss};
  const int agrid = (n + kApplyUnits - 1) / kApplyUnits;
  if (bwd) train_apply_kernel<true><<<agrid, kApplyThreads, 0, st>>>(a, sc);
  else train_apply_kernel<false><<<agrid, kApplyThreads, 0, st>>>(a, sc);
  PXB_LAUNCHED("train_apply_kernel");
  const int64_t groups = (t->cap + 3) / 4;
  int ugrid = static_cast<int>((groups + 2 * kUpdateThreads - 1) / (2 * kUpdateThreads));
  const int cap_grid = sm_count() * 2;  // one wave: two CTAs per SM
  if (ugrid > cap_grid) ugrid = cap_grid;
  if (ugrid < 1) ugrid = 1;
  train_update_kernel<<<ugrid, kUpdateThreads, 0, st>>>(t->cap, t->from_id, t->to_id, t->dead, t->weight, t->opt_m,
                                                        t->opt_v, t->opt_t, t->act, t->update_grad,
                                                        static_cast<uint32_t>(n), t->tail_start, p, l);
  PXB_LAUNCHED("train_update_kernel");
  return PXB_OK;
}
