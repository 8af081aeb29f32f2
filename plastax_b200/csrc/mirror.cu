// Destination-grouped mirror of a bucket: the index the forward sweep reads
// instead of the canonical source-major columns.
//
// The canonical arena keeps the reference's slot order (it is the state the
// claim's slot indices and every parity check refer to); its forward would
// scatter one atomic per edge to a random destination, which binds on L2.
// The mirror groups a bucket's live edges by destination chunk (2^chunk_bits
// consecutive units): entry = one packed 32-bit word (src << chunk_bits |
// dst - chunk base) + the weight + the canonical slot. A CTA sweeps a
// contiguous run of one group's entries, accumulates into the chunk's
// accumulators in shared memory, and flushes them to global memory once per
// run, so the forward streams 8 B per edge with no global atomics per edge.
//
// Maintenance under churn, all on the device:
// - the fused prune tombstones the mirror entry (word = EMPTY), the canonical
//   dead byte and the free bitmap bit, and pushes the entry position on its
//   group's hole stack;
// - the claim's placed edges are inserted by pxb_mirror_insert: a hole of
//   the destination's group if one is left, else the group's never-used
//   slack, else an overflow list that the forward sweeps with atomics.
#include "fixed.cuh"
#include "mirror.cuh"

namespace pxb {

// The sum is accumulated exactly in fixed point, independent of order. A
// chunk's shared accumulator is two 32-bit words per unit: lo in units of
// 2^-F and hi in units of 1.0 (2^F lo units), F = 28 or 31 fractional bits
// (the mirror's choice, by its largest in-degree); shared-memory integer
// atomics are native, where a float add is a compare-and-swap loop at a
// third of the rate. A product of magnitude < 1 is rounded to the nearest
// unit (exact when its 24-bit mantissa ends at or above 2^-F, i.e. when it is
// >= 2^(23-F); an error of at most 2^-(F+1) below) and added to lo; the
// adding thread sees a signed wrap of lo exactly, from the value its atomic
// returns, and carries 2^(32-F) (2^32 units) into hi. With F = 28 the word
// holds +-8 and wraps rarely; with F = 31 it holds +-1 and wraps (a carry)
// more often, for an error bound 8x tighter. A product in [1, 2^20) is a
// multiple of 2^-23, so its fixed value is exact: the part above 2^F units
// goes to hi, the rest to lo. A product that is not finite or >= 2^20 goes
// to the float side accumulator. The flush adds (hi * 2^F + lo) * 2^(31-F)
// to the unit's int64 global accumulator, always in units of
// 2^-PXB_FIXED_FRAC_BITS; one rounding to float happens in the unit apply.
constexpr int kFixBits = PXB_FIXED_FRAC_BITS;  // the global accumulator's unit
static_assert(kFixBits == 31, "the flush's shift and fix_scale assume a global unit of 2^-31");

// The same contribution straight into the global accumulators (the
// overflow list's edges), in their unit of 2^-31, rounded as the mirror's
// shared words round it (to 2^-frac): an edge sums to the same value
// whether it sits in a group or in the overflow list.
__device__ __forceinline__ void fixed_add_global(int64_t *af, float *gf, float p, int frac) {
  if (fabsf(p) < 1048576.0f) {
    const float scale = frac == 28 ? fix_scale<28>() : fix_scale<31>();
    const long long v = __float2ll_rn(p * scale) * (1ll << (kFixBits - frac));
    atomicAdd(reinterpret_cast<unsigned long long *>(af), static_cast<unsigned long long>(v));
  } else {
    atomicAdd(gf, p);
  }
}

template <int MONOID, int F>
__device__ __forceinline__ void smem_combine(float *acc_s, int chunk, float *acc_g, uint32_t dl, float v) {
  if (MONOID == PXB_MONOID_SUM) {
    int32_t *lo = reinterpret_cast<int32_t *>(acc_s);
    fixed_add<F>(lo + dl, lo + chunk + dl, acc_g + dl, v);
  } else if (MONOID == PXB_MONOID_MAX) {
    atomic_max_f32(acc_s + dl, v);
  } else {
    atomic_min_f32(acc_s + dl, v);
  }
}

// ---------------------------------------------------------------------------
// The sweep: a persistent, warp-specialised kernel. The entry arrays are cut
// into tiles of kTile entries; group bases are multiples of kTile, so a tile
// lies in one group. CTA c owns a contiguous run of tiles. One producer thread
// streams each tile's words and weights (only its used prefix) into a ring of
// kStages shared-memory stages with cp.async.bulk, completing on the stage's
// `full` mbarrier; kConsWarps consumer warps gather the activations, combine
// into the chunk's shared accumulators and release the stage on its `empty`
// mbarrier. A change of group between two tiles flushes the accumulators to
// global memory (float4 atomics for sum). Every mbarrier wait is bounded: on
// timeout the kernel records status bit 1 and stops touching the stage data,
// while still taking every consumer barrier, so it always terminates.
// ---------------------------------------------------------------------------
// Launch shape (overridable at compile time for tuning sweeps).
#ifndef PXB_SWEEP_STAGES
#define PXB_SWEEP_STAGES 2
#endif
#ifndef PXB_SWEEP_CONS_WARPS
#define PXB_SWEEP_CONS_WARPS 8
#endif
#ifndef PXB_SWEEP_MIN_CTAS
#define PXB_SWEEP_MIN_CTAS 3
#endif
#ifndef PXB_SWEEP_TILE
#define PXB_SWEEP_TILE PXB_MIRROR_TILE
#endif

constexpr int kTile = PXB_SWEEP_TILE;  // divides PXB_MIRROR_TILE: a tile lies in one group
static_assert(PXB_MIRROR_TILE % kTile == 0 && kTile % 4 == 0, "the sweep tile must divide the mirror tile");
constexpr int kStages = PXB_SWEEP_STAGES;
constexpr int kConsWarps = PXB_SWEEP_CONS_WARPS;
constexpr int kConsThreads = kConsWarps * 32;
constexpr int kSweepThreads = kConsThreads + 32;
constexpr uint32_t kWaitPolls = 1u << 24;

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}
// Wait for the phase of `parity` to complete, giving up after kWaitPolls polls.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
  for (uint32_t i = 0; i < kWaitPolls; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}
// Bulk copy global -> this CTA's shared memory, completing on `bar`; the
// source is marked evict-first in L2 (it is streamed once per sweep, while
// the activations it indexes should stay resident).
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar,
                                          uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
          "r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kConsThreads) : "memory"); }

// The group a sweep is in, with its bounds and fill held in registers.
struct GroupCursor {
  int64_t g, base, next, fill;
};

__device__ __forceinline__ void cursor_load(const MirrorK &m, GroupCursor &c) {
  c.base = __ldg(m.gbase + c.g);
  c.next = c.g + 1 < m.groups ? __ldg(m.gbase + c.g + 1) : INT64_MAX;
  c.fill = __ldg(m.gfill + c.g);
}

// Advance t to the next tile of [t, t_hi) with used entries; the cursor
// tracks its group. Producer and consumers walk the same sequence (gfill is
// not written during the sweep).
__device__ __forceinline__ bool next_tile(const MirrorK &m, int64_t &t, int64_t t_hi, GroupCursor &c,
                                          int32_t &used) {
  for (; t < t_hi; ++t) {
    const int64_t e0 = t * kTile;
    while (e0 >= c.next) {
      ++c.g;
      cursor_load(m, c);
    }
    const int64_t u = c.fill - (e0 - c.base);
    if (u > 0) {
      used = static_cast<int32_t>(u < kTile ? u : kTile);
      return true;
    }
  }
  return false;
}

// One tile of one group, staged in shared memory: each consumer thread takes
// two quads (8 entries). The gathers of all 8 entries are issued before any
// combine (an empty word reads a clamped, unused activation instead of
// branching); the prune predicate only sets a bit per entry, and the rare
// tombstones are written after the combines. Mirror words are written only
// by the build and the insert, which keep src < n and dst < n, so the loop
// carries no range checks (an accumulator past n is dropped at the flush).
// A pruned entry: its position goes on this CTA's deferred list (the
// tombstone is written by mirror_defer_flush_kernel after the sweep), or,
// when the list is full or absent, the tombstone is written here.
__device__ __forceinline__ void prune_entry(const MirrorK &m, const MPrune &p, int64_t pos, int32_t src, int64_t g,
                                            int64_t gb, int *defer_n, int64_t seg) {
  if (defer_n != nullptr) {
    const int i = atomicAdd(defer_n, 1);
    if (i < seg) {
      m.defer_pos[blockIdx.x * seg + i] = pos;
      return;
    }
  }
  tombstone(p, m.slot[pos], src);
  empty_entry(m, pos, g, gb);
}

template <int MONOID, int PK, int F>
__device__ __forceinline__ void sweep_tile(const MirrorK &m, const MPrune &p, const LowkCut &cut,
                                           const float *__restrict__ act, const uint32_t *word_t, const float *w_t,
                                           int used, float *acc_s, float *acc_g, int32_t g, int64_t gb, int64_t e0,
                                           int &pruned_here, int *defer_n, int64_t seg) {
  const uint32_t mask = (1u << m.cb) - 1u;
  const int chunk = 1 << m.cb;
  const uint32_t last = static_cast<uint32_t>(m.n - 1);
  const int nq = (used + 3) >> 2;
  const uint4 *wq = reinterpret_cast<const uint4 *>(word_t);
  const float4 *fq = reinterpret_cast<const float4 *>(w_t);
  for (int q = threadIdx.x; q < nq; q += 2 * kConsThreads) {
    const int q2 = q + kConsThreads;
    const bool two = q2 < nq;
    const uint4 wa = wq[q];
    const float4 fa = fq[q];
    const uint4 wb = two ? wq[q2] : make_uint4(kEmpty, kEmpty, kEmpty, kEmpty);
    const float4 fb = two ? fq[q2] : make_float4(0.f, 0.f, 0.f, 0.f);
    uint32_t ws[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
    float fs[8] = {fa.x, fa.y, fa.z, fa.w, fb.x, fb.y, fb.z, fb.w};
    if (used < kTile) {  // the group's used prefix ends inside this tile
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (((j < 4 ? q : q2) * 4 + (j & 3)) >= used) {
          ws[j] = kEmpty;
          fs[j] = 0.0f;
        }
    }
    float av[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) av[j] = __ldg(act + min(ws[j] >> m.cb, last));
    if (MONOID == PXB_MONOID_SUM) {
      // branch-free common case: every product of the eight below 1 in
      // magnitude (a NaN fails the test). An empty entry's weight is 0 (the
      // prune zeroes it, the build and the tail mask leave 0), so it adds an
      // exact 0 into the chunk's last unit (kEmpty & mask); a non-finite
      // activation behind it fails the test and the slow path skips it
      float pv[8];
      bool small = true;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        pv[j] = __fmul_rn(fs[j], av[j]);
        small &= fabsf(pv[j]) < 1.0f;
      }
      int32_t *lo = reinterpret_cast<int32_t *>(acc_s);
      if (small) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint32_t dl = ws[j] & mask;
          lo_add<F>(lo + dl, lo + chunk + dl, __float2int_rn(pv[j] * fix_scale<F>()));
        }
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (ws[j] != kEmpty)
            fixed_add<F>(lo + (ws[j] & mask), lo + chunk + (ws[j] & mask), acc_g + (ws[j] & mask), pv[j]);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (ws[j] != kEmpty) smem_combine<MONOID, F>(acc_s, chunk, acc_g, ws[j] & mask, __fmul_rn(fs[j], av[j]));
    }
    if (PK != PXB_PRUNE_NONE) {
      // the predicate is rare: one test of the smallest |w| (fminf drops a
      // NaN, which no predicate prunes) or of any below its destination's
      // threshold, then the per-entry pass only when it passes
      bool any;
      if (PK == PXB_PRUNE_ABS_BELOW) {
        float mn = fabsf(fs[0]);
#pragma unroll
        for (int j = 1; j < 8; ++j) mn = fminf(mn, fabsf(fs[j]));
        any = mn < p.thr;
      } else if (PK == PXB_PRUNE_LOWEST_K) {
        // below the threshold bin's end (an empty entry's zero weight
        // passes and is skipped below; fminf drops a NaN, which is never
        // pruned or listed)
        float mn = fabsf(fs[0]);
#pragma unroll
        for (int j = 1; j < 8; ++j) mn = fminf(mn, fabsf(fs[j]));
        any = mn <= cut.hi_le;
      } else {
        any = false;
#pragma unroll
        for (int j = 0; j < 8; ++j)
          any |= ws[j] != kEmpty && fabsf(fs[j]) < __ldg(p.unit_thr + ((g << m.cb) | (ws[j] & mask)));
      }
      if (any) {
        for (int j = 0; j < 8; ++j) {
          if (ws[j] == kEmpty) continue;
          const int64_t pos = e0 + (j < 4 ? q : q2) * 4 + (j & 3);
          if (PK == PXB_PRUNE_LOWEST_K) {
            const uint32_t b = abs_bits(fs[j]);
            if (b >= cut.hi) continue;
            if (b >= cut.lo) {  // the threshold bin: listed, selected after every sweep
              lowk_list(p, cut.parity, b, m.slot[pos], static_cast<int32_t>(ws[j] >> m.cb), pos);
              continue;
            }
            ++pruned_here;
          } else {
            const float thr = PK == PXB_PRUNE_ABS_BELOW ? p.thr : __ldg(p.unit_thr + ((g << m.cb) | (ws[j] & mask)));
            if (!(fabsf(fs[j]) < thr)) continue;
          }
          prune_entry(m, p, pos, static_cast<int32_t>(ws[j] >> m.cb), g, gb, defer_n, seg);
        }
      }
    }
  }
}

// Flush (unless g < 0) and reset the chunk accumulators; each consumer thread
// flushes and resets the same indices, so one barrier before and one after.
template <int MONOID, int F>
__device__ __forceinline__ void flush_reset(const MirrorK &m, float *acc_s, float *__restrict__ acc,
                                            int64_t *__restrict__ acc_fixed, int64_t g) {
  const int chunk = 1 << m.cb;
  const int32_t base = static_cast<int32_t>(g) << m.cb;
  if (MONOID == PXB_MONOID_SUM) {
    int4 *lo4 = reinterpret_cast<int4 *>(acc_s);
    int4 *hi4 = lo4 + chunk / 4;
    const int4 z = make_int4(0, 0, 0, 0);
    for (int u = threadIdx.x; u < chunk / 4; u += kConsThreads) {
      if (g >= 0) {
        const int4 l = lo4[u], h = hi4[u];
        const int32_t ls[4] = {l.x, l.y, l.z, l.w}, hs[4] = {h.x, h.y, h.z, h.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const long long tot = ((static_cast<long long>(hs[j]) << F) + ls[j]) * (1ll << (kFixBits - F));
          if (tot != 0 && base + 4 * u + j < m.n)
            atomicAdd(reinterpret_cast<unsigned long long *>(acc_fixed + base + 4 * u + j),
                      static_cast<unsigned long long>(tot));
        }
      }
      lo4[u] = z;
      hi4[u] = z;
    }
    return;
  }
  const float ident = monoid_identity(MONOID);
  float4 *s4 = reinterpret_cast<float4 *>(acc_s);
  const float4 id4 = make_float4(ident, ident, ident, ident);
  for (int u = threadIdx.x; u < chunk / 4; u += kConsThreads) {
    if (g >= 0) {
      const float4 v = s4[u];
      const float vs[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (vs[j] != ident && base + 4 * u + j < m.n) atomic_combine<MONOID>(acc + base + 4 * u + j, vs[j]);
    }
    s4[u] = id4;
  }
}

template <int MONOID, int PK, int F>
__global__ void __launch_bounds__(kSweepThreads, PXB_SWEEP_MIN_CTAS) mirror_sweep_kernel(MirrorK m, const float *__restrict__ act,
                                                                        float *__restrict__ acc,
                                                                        int64_t *__restrict__ acc_fixed, MPrune p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  uint64_t *full = reinterpret_cast<uint64_t *>(smem_raw);
  uint64_t *empty = full + kStages;
  uint32_t *word_s = reinterpret_cast<uint32_t *>(smem_raw + 128);
  float *w_s = reinterpret_cast<float *>(word_s + kStages * kTile);
  float *acc_s = w_s + kStages * kTile;

  __shared__ int s_defer;
  const bool defer = PK != PXB_PRUNE_NONE && m.defer_pos != nullptr && gridDim.x <= m.defer_ctas;
  const int64_t seg = defer ? m.defer_total / gridDim.x : 0;
  const int64_t tiles = m.entries / kTile;
  const int64_t per = (tiles + gridDim.x - 1) / gridDim.x;
  const int64_t t_lo = blockIdx.x * per;
  const int64_t t_hi = t_lo + per < tiles ? t_lo + per : tiles;
  if (t_lo >= t_hi) {
    if (defer && threadIdx.x == 0) m.defer_count[blockIdx.x] = 0;
    return;
  }
  if (threadIdx.x == 0) {
    s_defer = 0;
    for (int s = 0; s < kStages; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, kConsWarps);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  // the group of tile t_lo: the last g with gbase[g] <= t_lo * kTile
  int64_t lo = 0, hi = m.groups - 1;
  while (lo < hi) {
    const int64_t mid = (lo + hi + 1) / 2;
    if (__ldg(m.gbase + mid) <= t_lo * kTile) lo = mid; else hi = mid - 1;
  }
  __syncthreads();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == kConsWarps) {
    // producer: one thread issues the ring's bulk copies
    if (lane != 0) return;
    uint64_t policy;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
    int64_t t = t_lo;
    GroupCursor c{lo, 0, 0, 0};
    cursor_load(m, c);
    int32_t used;
    uint32_t i = 0;
    bool ok = true;
    while (next_tile(m, t, t_hi, c, used)) {
      const int s = static_cast<int>(i % kStages);
      if (i >= kStages && !mbar_wait(empty + s, ((i / kStages) - 1) & 1)) {
        ok = false;
        break;
      }
      const uint32_t bytes = static_cast<uint32_t>((used + 3) / 4 * 16);
      mbar_arrive_expect_tx(full + s, 2 * bytes);
      bulk_load(word_s + s * kTile, m.word + t * kTile, bytes, full + s, policy);
      bulk_load(w_s + s * kTile, m.w + t * kTile, bytes, full + s, policy);
      ++t;
      ++i;
    }
    // never leave with a copy in flight: wait for the last issued stages
    const uint32_t first = i > kStages ? i - kStages : 0;
    for (uint32_t j = first; j < i; ++j)
      if (!mbar_wait(full + (j % kStages), (j / kStages) & 1)) ok = false;
    if (!ok) atomicOr(m.status, 2);
    return;
  }

  // consumers
  const LowkCut cut = lowk_cut(p);
  int pruned_here = 0;
  int64_t t = t_lo, cur = -1;
  GroupCursor c{lo, 0, 0, 0};
  cursor_load(m, c);
  int32_t used;
  uint32_t i = 0;
  bool ok = true;
  while (next_tile(m, t, t_hi, c, used)) {
    const int64_t g = c.g;
    if (g != cur) {
      consumer_sync();
      flush_reset<MONOID, F>(m, acc_s, acc, acc_fixed, cur);
      consumer_sync();
      cur = g;
    }
    const int s = static_cast<int>(i % kStages);
    if (ok && !mbar_wait(full + s, (i / kStages) & 1)) ok = false;
    if (ok)
      sweep_tile<MONOID, PK, F>(m, p, cut, act, word_s + s * kTile, w_s + s * kTile, used, acc_s,
                             acc + (static_cast<int64_t>(g) << m.cb), static_cast<int32_t>(g), c.base, t * kTile,
                             pruned_here, defer ? &s_defer : nullptr, seg);
    __syncwarp();
    if (lane == 0) mbar_arrive(empty + s);
    ++t;
    ++i;
  }
  if (cur >= 0) {
    consumer_sync();
    flush_reset<MONOID, F>(m, acc_s, acc, acc_fixed, cur);
  }
  if (defer) {
    consumer_sync();  // every consumer's deferred prunes are listed
    if (threadIdx.x == 0) m.defer_count[blockIdx.x] = s_defer < seg ? s_defer : static_cast<int>(seg);
  }
  if (!ok && lane == 0) atomicOr(m.status, 2);
  if (PK == PXB_PRUNE_LOWEST_K) {
    const int w_pruned = __reduce_add_sync(0xffffffffu, pruned_here);
    if (lane == 0 && w_pruned) atomicAdd(p.lk.count + 2 * cut.parity + 1, static_cast<unsigned long long>(w_pruned));
  }
}

// Edges the mirror had no room for: swept with global atomics.
template <int MONOID, int PK>
__global__ void mirror_overflow_kernel(MirrorK m, const float *__restrict__ act, float *__restrict__ acc,
                                       int64_t *__restrict__ acc_fixed, MPrune p) {
  const int64_t cnt = *m.ovf_count < m.ovf_cap ? *m.ovf_count : m.ovf_cap;
  const LowkCut cut = lowk_cut(p);
  int pruned_here = 0;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < cnt;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int32_t s = m.ovf_src[i], d = m.ovf_dst[i];
    if (s < 0 || s >= m.n || d < 0 || d >= m.n) continue;
    const float w = m.ovf_w[i];
    if (MONOID == PXB_MONOID_SUM) fixed_add_global(acc_fixed + d, acc + d, __fmul_rn(w, act[s]), m.sum_frac);
    else atomic_combine<MONOID>(acc + d, __fmul_rn(w, act[s]));
    if (PK == PXB_PRUNE_LOWEST_K) {
      const uint32_t b = abs_bits(w);
      if (b >= cut.hi) continue;
      if (b >= cut.lo) {
        lowk_list(p, cut.parity, b, m.ovf_slot[i], s, -1 - i);
        continue;
      }
      ++pruned_here;
      m.ovf_src[i] = -1;
      tombstone(p, m.ovf_slot[i], s);
    } else if (PK != PXB_PRUNE_NONE && mprune_pred(p, w, d)) {
      m.ovf_src[i] = -1;
      tombstone(p, m.ovf_slot[i], s);
    }
  }
  if (PK == PXB_PRUNE_LOWEST_K) {
    const int w_pruned = __reduce_add_sync(0xffffffffu, pruned_here);
    if ((threadIdx.x & 31) == 0 && w_pruned)
      atomicAdd(p.lk.count + 2 * cut.parity + 1, static_cast<unsigned long long>(w_pruned));
  }
}

// The sweep's deferred prunes: CTA c of the sweep listed defer_count[c]
// entry positions (all inside its contiguous run of tiles, so in a few
// groups); each gets its tombstone (canonical dead byte, free bitmap bit)
// and leaves the mirror (emptied, pushed on its group's hole stack). The
// pushes are counted per group in shared memory first and each group's run
// of the stack reserved with one atomic, as one counter per group would
// take every push of the run otherwise.
constexpr int kFlushThreads = 256;
constexpr int kFlushPer = 8;
constexpr int kFlushGroups = 64;
__global__ void __launch_bounds__(kFlushThreads) mirror_defer_flush_kernel(MirrorK m, MPrune p, int sweep_ctas) {
  __shared__ int32_t s_cnt[kFlushGroups];
  const int64_t seg = m.defer_total / sweep_ctas;
  const int64_t tiles = m.entries / kTile;
  const int64_t per = (tiles + sweep_ctas - 1) / sweep_ctas;
  for (int c = blockIdx.x; c < sweep_ctas; c += gridDim.x) {
    const int n = m.defer_count[c];
    if (n == 0) continue;  // uniform over the CTA
    const int64_t t_lo = c * per, t_hi = min(t_lo + per, tiles);
    const int64_t g0 = group_of(m, t_lo * kTile), g1 = group_of(m, t_hi * kTile - 1);
    const bool local = g1 - g0 < kFlushGroups;
    for (int chunk = 0; chunk < n; chunk += kFlushThreads * kFlushPer) {
      if (threadIdx.x < kFlushGroups) s_cnt[threadIdx.x] = 0;
      __syncthreads();
      int64_t pos[kFlushPer], grp[kFlushPer];
      int rank[kFlushPer];
#pragma unroll
      for (int j = 0; j < kFlushPer; ++j) {
        const int i = chunk + j * kFlushThreads + threadIdx.x;
        pos[j] = -1;
        if (i >= n) continue;
        pos[j] = m.defer_pos[c * seg + i];
        if (local) {
          int64_t g = g0;  // the CTA's run spans a few groups
          while (g < g1 && __ldg(m.gbase + g + 1) <= pos[j]) ++g;
          grp[j] = g;
          rank[j] = atomicAdd(&s_cnt[g - g0], 1);
        } else {
          grp[j] = group_of(m, pos[j]);
        }
      }
      __syncthreads();
      if (local && threadIdx.x < kFlushGroups && g0 + threadIdx.x <= g1) {
        const int32_t cnt = s_cnt[threadIdx.x];
        if (cnt) s_cnt[threadIdx.x] = atomicAdd(m.hcount + g0 + threadIdx.x, cnt);  // the run's first hole
      }
      __syncthreads();
      // every load first (a store to word may alias a later entry's load,
      // which would serialise the entries), then the writes
      int32_t src[kFlushPer], slot[kFlushPer], row[kFlushPer];
#pragma unroll
      for (int j = 0; j < kFlushPer; ++j) {
        if (pos[j] < 0) continue;
        src[j] = static_cast<int32_t>(m.word[pos[j]] >> m.cb);
        slot[j] = m.slot[pos[j]];
      }
#pragma unroll
      for (int j = 0; j < kFlushPer; ++j)
        if (pos[j] >= 0) row[j] = p.bm_level ? __ldg(p.bm_level + src[j]) : 0;
#pragma unroll
      for (int j = 0; j < kFlushPer; ++j) {
        if (pos[j] < 0) continue;
        p.dead[slot[j]] = 1;
        if (p.bm != nullptr)
          atomicOr(p.bm + static_cast<int64_t>(row[j]) * p.bm_words + (slot[j] >> 5), 1u << (slot[j] & 31));
        if (p.pruned) atomicAdd(p.pruned, 1);
        const int64_t gb = m.gbase[grp[j]];
        m.word[pos[j]] = kEmpty;
        m.w[pos[j]] = 0.0f;
        const int32_t h = local ? s_cnt[grp[j] - g0] + rank[j] : atomicAdd(m.hcount + grp[j], 1);
        m.hstack[gb + h] = static_cast<int32_t>(pos[j] - gb);
      }
      __syncthreads();
    }
  }
}

// Insert, phase 1: each placed edge takes rank r in its destination group;
// the r-th insert of a group takes the group's r-th hole from the top of its
// stack, then its unused slack, then the overflow list. Phase 2 retires the
// used holes and slack.
__device__ __forceinline__ void insert_at(const MirrorK &m, int32_t a, int32_t d, float w, int32_t s, int32_t g,
                                          int32_t r) {
  const int64_t gb = m.gbase[g], gcap = m.gbase[g + 1] - gb;
  const int32_t holes = m.hcount[g];
  int64_t pos = -1;
  if (r < holes) {
    pos = gb + m.hstack[gb + holes - 1 - r];
  } else {
    const int64_t f = static_cast<int64_t>(m.gfill[g]) + (r - holes);
    if (f < gcap) pos = gb + f;
  }
  if (pos >= 0) {
    m.word[pos] = (static_cast<uint32_t>(a) << m.cb) | (static_cast<uint32_t>(d) & ((1u << m.cb) - 1u));
    m.w[pos] = w;
    m.slot[pos] = s;
  } else {
    const int32_t o = atomicAdd(m.ovf_count, 1);
    if (o < m.ovf_cap) {
      m.ovf_src[o] = a;
      m.ovf_dst[o] = d;
      m.ovf_w[o] = w;
      m.ovf_slot[o] = s;
    } else {
      atomicOr(m.status, 1);  // an edge is missing from the mirror: rebuild it
    }
  }
}

// One global counter per destination group takes every placed edge's rank
// (the path for meshes of many groups).
__global__ void mirror_insert_kernel(MirrorK m, int64_t k, const int32_t *__restrict__ src,
                                     const int32_t *__restrict__ dst, const float *__restrict__ w,
                                     const int32_t *__restrict__ placed, int32_t *__restrict__ ins_count) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < k;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int32_t s = placed[i];
    if (s < 0) continue;
    const int32_t a = src[i], d = dst[i];
    if (a < 0 || a >= m.n || d < 0 || d >= m.n) continue;
    const int32_t g = d >> m.cb;
    insert_at(m, a, d, w[i], s, g, atomicAdd(ins_count + g, 1));
  }
}

// The same ranks with the groups counted per CTA first: each CTA takes
// kInsertPer edges per thread, ranks them in shared memory, reserves each
// group's run with one global atomic, then inserts (a global counter per
// edge would serialise on the few hundred group counters).
constexpr int kInsertThreads = 1024;
constexpr int kInsertPer = 2;
constexpr int kInsertMaxGroups = 8192;
__global__ void __launch_bounds__(kInsertThreads) mirror_insert_grouped_kernel(
    MirrorK m, int64_t k, const int32_t *__restrict__ src, const int32_t *__restrict__ dst,
    const float *__restrict__ w, const int32_t *__restrict__ placed, int32_t *__restrict__ ins_count) {
  __shared__ int32_t s_cnt[kInsertMaxGroups];
  for (int64_t g = threadIdx.x; g < m.groups; g += kInsertThreads) s_cnt[g] = 0;
  __syncthreads();
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kInsertThreads * kInsertPer;
  int32_t grp[kInsertPer], rank[kInsertPer];
#pragma unroll
  for (int j = 0; j < kInsertPer; ++j) {
    const int64_t i = base + j * kInsertThreads + threadIdx.x;
    grp[j] = -1;
    if (i >= k || placed[i] < 0) continue;
    const int32_t a = src[i], d = dst[i];
    if (a < 0 || a >= m.n || d < 0 || d >= m.n) continue;
    grp[j] = d >> m.cb;
    rank[j] = atomicAdd(&s_cnt[grp[j]], 1);
  }
  __syncthreads();
  for (int64_t g = threadIdx.x; g < m.groups; g += kInsertThreads) {
    const int32_t c = s_cnt[g];
    if (c) s_cnt[g] = atomicAdd(ins_count + g, c);  // the CTA's first rank in group g
  }
  __syncthreads();
#pragma unroll
  for (int j = 0; j < kInsertPer; ++j) {
    if (grp[j] < 0) continue;
    const int64_t i = base + j * kInsertThreads + threadIdx.x;
    insert_at(m, src[i], dst[i], w[i], placed[i], grp[j], s_cnt[grp[j]] + rank[j]);
  }
}

__global__ void mirror_insert_finish_kernel(MirrorK m, int32_t *__restrict__ ins_count) {
  for (int64_t g = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; g < m.groups;
       g += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int32_t ins = ins_count[g];
    if (ins == 0) continue;
    const int32_t holes = m.hcount[g];
    const int64_t gcap = m.gbase[g + 1] - m.gbase[g];
    if (ins <= holes) {
      m.hcount[g] = holes - ins;
    } else {
      m.hcount[g] = 0;
      const int64_t f = static_cast<int64_t>(m.gfill[g]) + (ins - holes);
      m.gfill[g] = static_cast<int32_t>(f < gcap ? f : gcap);
    }
    ins_count[g] = 0;
  }
}

int check_mirror(const char *fn, const pxb_mirror *m) {
  PXB_REQUIRE(m != nullptr, "%s: mirror is NULL", fn);
  PXB_REQUIRE(m->chunk_bits >= 2 && m->chunk_bits <= 13, "%s: chunk_bits %d not in [2, 13]", fn, m->chunk_bits);
  PXB_REQUIRE(m->num_units > 0, "%s: num_units must be > 0", fn);
  PXB_REQUIRE(m->groups == ((int64_t(m->num_units) + (int64_t(1) << m->chunk_bits) - 1) >> m->chunk_bits),
              "%s: groups does not match num_units and chunk_bits", fn);
  PXB_REQUIRE(m->entries % PXB_MIRROR_TILE == 0, "%s: entries must be a multiple of %d", fn, PXB_MIRROR_TILE);
  int bits = 0;
  while ((int64_t(1) << bits) < m->num_units) ++bits;
  PXB_REQUIRE(bits + m->chunk_bits <= 32, "%s: unit ids need %d bits, too many for %d chunk bits", fn, bits,
              m->chunk_bits);
  PXB_REQUIRE(m->gbase && m->gfill && m->word && m->weight && m->slot && m->hstack && m->hcount && m->status,
              "%s: a mirror array is NULL", fn);
  PXB_REQUIRE(m->items == 0 || (m->item_begin && m->item_end && m->item_group), "%s: work items are NULL", fn);
  PXB_REQUIRE(aligned16(m->word) && aligned16(m->weight), "%s: mirror word/weight must be 16-byte aligned", fn);
  PXB_REQUIRE(m->ovf_cap == 0 || (m->ovf_count && m->ovf_src && m->ovf_dst && m->ovf_slot && m->ovf_weight),
              "%s: overflow list is NULL", fn);
  return PXB_OK;
}

}  // namespace pxb

using namespace pxb;

namespace pxb {

// The sweep and the overflow pass of one mirror, for any monoid and prune.
// The sweep's grid for (monoid, prune kind): every CTA resident at once, no
// more CTAs than tiles. The deferred tombstones are segmented by it, so the
// flush recomputes it the same way.
template <int M, int P>
static int sweep_grid_of(const MirrorK &m, int *grid) {
  const size_t acc_bytes = (M == PXB_MONOID_SUM ? 2 * sizeof(int32_t) : sizeof(float)) << m.cb;
  const size_t smem = 128 + size_t(kStages) * kTile * 8 + acc_bytes;
  auto fn = (M == PXB_MONOID_SUM && m.sum_frac == 28) ? mirror_sweep_kernel<M, P, 28> : mirror_sweep_kernel<M, P, 31>;
  PXB_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
  int per_sm = 0;
  PXB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kSweepThreads, smem));
  const int64_t full = int64_t(sm_count()) * (per_sm > 0 ? per_sm : 1);
  const int64_t tiles = m.entries / kTile;
  *grid = static_cast<int>(tiles < full ? tiles : full);
  return PXB_OK;
}

// The lowest-|w| sweep's deferred tombstones (the sweep of the same mirror
// and monoid ran before on the stream).
static int lowk_flush_launch(const MirrorK &m, int32_t monoid, const MPrune &p, cudaStream_t st) {
  if (m.entries <= 0 || m.defer_pos == nullptr) return PXB_OK;
  int grid = 0;
  int rc = monoid == PXB_MONOID_SUM   ? sweep_grid_of<PXB_MONOID_SUM, PXB_PRUNE_LOWEST_K>(m, &grid)
           : monoid == PXB_MONOID_MAX ? sweep_grid_of<PXB_MONOID_MAX, PXB_PRUNE_LOWEST_K>(m, &grid)
                                      : sweep_grid_of<PXB_MONOID_MIN, PXB_PRUNE_LOWEST_K>(m, &grid);
  if (rc) return rc;
  if (grid > 0 && grid <= m.defer_ctas) {
    mirror_defer_flush_kernel<<<grid, kFlushThreads, 0, st>>>(m, p, grid);
    PXB_LAUNCHED("mirror_defer_flush_kernel");
  }
  return PXB_OK;
}

static int mirror_forward_launch(const MirrorK &m, const float *act, int32_t monoid, float *acc, int64_t *acc_fixed,
                                 const MPrune &p, cudaStream_t st, bool flush = true) {
  const int32_t prune_kind = p.kind;
  int sweep_grid = 0;
  if (m.entries > 0) {
    const size_t acc_bytes = (monoid == PXB_MONOID_SUM ? 2 * sizeof(int32_t) : sizeof(float)) << m.cb;
    const size_t smem = 128 + size_t(kStages) * kTile * 8 + acc_bytes;
    const int threads = kSweepThreads;
    const int64_t tiles = m.entries / kTile;
#define PXB_MS(M, P)                                                                              \
  do {                                                                                            \
    auto fn = (M == PXB_MONOID_SUM && m.sum_frac == 28) ? mirror_sweep_kernel<M, P, 28>           \
                                                        : mirror_sweep_kernel<M, P, 31>;          \
    PXB_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));   \
    int per_sm = 0;                                                                               \
    PXB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, threads, smem));          \
    const int64_t full = int64_t(sm_count()) * (per_sm > 0 ? per_sm : 1);                        \
    sweep_grid = static_cast<int>(tiles < full ? tiles : full);                                   \
    fn<<<sweep_grid, threads, smem, st>>>(m, act, acc, acc_fixed, p);                             \
  } while (0)
#define PXB_MS_K(M)                                                                               \
  do {                                                                                            \
    if (prune_kind == PXB_PRUNE_ABS_BELOW) PXB_MS(M, PXB_PRUNE_ABS_BELOW);                        \
    else if (prune_kind == PXB_PRUNE_ABS_BELOW_DST) PXB_MS(M, PXB_PRUNE_ABS_BELOW_DST);           \
    else if (prune_kind == PXB_PRUNE_LOWEST_K) PXB_MS(M, PXB_PRUNE_LOWEST_K);                     \
    else PXB_MS(M, PXB_PRUNE_NONE);                                                               \
  } while (0)
    if (monoid == PXB_MONOID_SUM) PXB_MS_K(PXB_MONOID_SUM);
    else if (monoid == PXB_MONOID_MAX) PXB_MS_K(PXB_MONOID_MAX);
    else PXB_MS_K(PXB_MONOID_MIN);
#undef PXB_MS_K
#undef PXB_MS
    PXB_LAUNCHED("mirror_sweep_kernel");
    if (flush && prune_kind != PXB_PRUNE_NONE && m.defer_pos != nullptr && sweep_grid <= m.defer_ctas) {
      mirror_defer_flush_kernel<<<sweep_grid, kFlushThreads, 0, st>>>(m, p, sweep_grid);
      PXB_LAUNCHED("mirror_defer_flush_kernel");
    }
  }
  if (m.ovf_cap > 0) {
#define PXB_MO(M, P) mirror_overflow_kernel<M, P><<<sm_count(), 256, 0, st>>>(m, act, acc, acc_fixed, p)
#define PXB_MO_K(M)                                                                               \
  do {                                                                                            \
    if (prune_kind == PXB_PRUNE_ABS_BELOW) PXB_MO(M, PXB_PRUNE_ABS_BELOW);                        \
    else if (prune_kind == PXB_PRUNE_ABS_BELOW_DST) PXB_MO(M, PXB_PRUNE_ABS_BELOW_DST);           \
    else if (prune_kind == PXB_PRUNE_LOWEST_K) PXB_MO(M, PXB_PRUNE_LOWEST_K);                     \
    else PXB_MO(M, PXB_PRUNE_NONE);                                                               \
  } while (0)
    if (monoid == PXB_MONOID_SUM) PXB_MO_K(PXB_MONOID_SUM);
    else if (monoid == PXB_MONOID_MAX) PXB_MO_K(PXB_MONOID_MAX);
    else PXB_MO_K(PXB_MONOID_MIN);
#undef PXB_MO_K
#undef PXB_MO
    PXB_LAUNCHED("mirror_overflow_kernel");
  }
  return PXB_OK;
}

static int mirror_forward_checks(const char *fn, const pxb_mirror *mirror, const float *act, int32_t monoid,
                                 float *acc, int64_t *acc_fixed) {
  int rc = check_mirror(fn, mirror);
  if (rc) return rc;
  PXB_REQUIRE(monoid >= 0 && monoid <= 2, "%s: unknown monoid %d", fn, monoid);
  PXB_REQUIRE(act && acc, "%s: act/acc is NULL", fn);
  PXB_REQUIRE(monoid != PXB_MONOID_SUM || acc_fixed != nullptr,
              "%s: the sum needs its fixed-point accumulator acc_fixed", fn);
  PXB_REQUIRE((reinterpret_cast<uintptr_t>(acc_fixed) & 7u) == 0, "%s: acc_fixed must be 8-byte aligned", fn);
  return PXB_OK;
}

}  // namespace pxb

extern "C" int pxb_mirror_forward(const pxb_mirror *mirror, const float *act, int32_t monoid, float *acc,
                                  int64_t *acc_fixed, int32_t prune_kind, float prune_threshold, const float *unit_threshold,
                                  uint8_t *dead, uint32_t *free_bitmap, int64_t bitmap_words,
                                  const int32_t *bitmap_level, int32_t *pruned_count, void *stream) {
  int rc = mirror_forward_checks("pxb_mirror_forward", mirror, act, monoid, acc, acc_fixed);
  if (rc) return rc;
  PXB_REQUIRE(prune_kind >= 0 && prune_kind <= 2, "pxb_mirror_forward: unknown prune kind %d", prune_kind);
  PXB_REQUIRE(prune_kind == PXB_PRUNE_NONE || dead, "pxb_mirror_forward: pruning needs the canonical dead column");
  PXB_REQUIRE(prune_kind != PXB_PRUNE_ABS_BELOW_DST || unit_threshold,
              "pxb_mirror_forward: per-destination threshold column is NULL");
  MPrune p{prune_kind, prune_threshold, unit_threshold, dead, free_bitmap, bitmap_words, bitmap_level, pruned_count,
           LowkSweep{}};
  return mirror_forward_launch(to_k(mirror), act, monoid, acc, acc_fixed, p, as_stream(stream));
}

static int forward_lowk(const pxb_mirror *mirror, const float *act, int32_t monoid, float *acc, int64_t *acc_fixed,
                        const pxb_lowk *lowk, uint8_t *dead, uint32_t *free_bitmap, int64_t bitmap_words,
                        const int32_t *bitmap_level, int flush, void *stream) {
  int rc = mirror_forward_checks("pxb_mirror_forward_lowk", mirror, act, monoid, acc, acc_fixed);
  if (rc) return rc;
  PXB_REQUIRE(lowk != nullptr && lowk->plan && lowk->key && lowk->level && lowk->count && lowk->pos,
              "pxb_mirror_forward_lowk: a lowk array is NULL");
  PXB_REQUIRE(lowk->list_cap > 0, "pxb_mirror_forward_lowk: list_cap must be > 0");
  PXB_REQUIRE(dead != nullptr, "pxb_mirror_forward_lowk: pruning needs the canonical dead column");
  PXB_REQUIRE(lowk->slot_base >= 0 && lowk->slot_base < (int64_t(1) << 31),
              "pxb_mirror_forward_lowk: slot_base out of range (global slots are keyed in 32 bits)");
  MPrune p{PXB_PRUNE_LOWEST_K, 0.0f, nullptr, dead, free_bitmap, bitmap_words, bitmap_level, nullptr,
           LowkSweep{lowk->plan, lowk->key, lowk->level, lowk->count, lowk->pos, lowk->list_cap, lowk->slot_base}};
  return mirror_forward_launch(to_k(mirror), act, monoid, acc, acc_fixed, p, as_stream(stream), flush != 0);
}

extern "C" int pxb_mirror_defer_flush(const pxb_mirror *mirror, int32_t monoid, const pxb_lowk *lowk, uint8_t *dead,
                                      uint32_t *free_bitmap, int64_t bitmap_words, const int32_t *bitmap_level,
                                      void *stream) {
  int rc = check_mirror("pxb_mirror_defer_flush", mirror);
  if (rc) return rc;
  PXB_REQUIRE(monoid >= 0 && monoid <= 2, "pxb_mirror_defer_flush: unknown monoid %d", monoid);
  PXB_REQUIRE(lowk != nullptr && lowk->plan && lowk->key && lowk->level && lowk->count && lowk->pos,
              "pxb_mirror_defer_flush: a lowk array is NULL");
  PXB_REQUIRE(dead != nullptr, "pxb_mirror_defer_flush: dead is NULL");
  MPrune p{PXB_PRUNE_LOWEST_K, 0.0f, nullptr, dead, free_bitmap, bitmap_words, bitmap_level, nullptr,
           LowkSweep{lowk->plan, lowk->key, lowk->level, lowk->count, lowk->pos, lowk->list_cap, lowk->slot_base}};
  return lowk_flush_launch(to_k(mirror), monoid, p, as_stream(stream));
}

extern "C" int pxb_mirror_forward_lowk(const pxb_mirror *mirror, const float *act, int32_t monoid, float *acc,
                                       int64_t *acc_fixed, const pxb_lowk *lowk, uint8_t *dead, uint32_t *free_bitmap,
                                       int64_t bitmap_words, const int32_t *bitmap_level, void *stream) {
  return forward_lowk(mirror, act, monoid, acc, acc_fixed, lowk, dead, free_bitmap, bitmap_words, bitmap_level, 1,
                      stream);
}

extern "C" int pxb_mirror_forward_lowk_deferred(const pxb_mirror *mirror, const float *act, int32_t monoid,
                                                float *acc, int64_t *acc_fixed, const pxb_lowk *lowk, uint8_t *dead,
                                                uint32_t *free_bitmap, int64_t bitmap_words,
                                                const int32_t *bitmap_level, void *stream) {
  return forward_lowk(mirror, act, monoid, acc, acc_fixed, lowk, dead, free_bitmap, bitmap_words, bitmap_level, 0,
                      stream);
}

extern "C" int pxb_mirror_insert(const pxb_mirror *mirror, int64_t k, const int32_t *src, const int32_t *dst,
                                 const float *weight, const int32_t *placed, void *stream) {
  int rc = check_mirror("pxb_mirror_insert", mirror);
  if (rc) return rc;
  PXB_REQUIRE(k >= 0, "pxb_mirror_insert: negative k");
  if (k == 0) return PXB_OK;
  PXB_REQUIRE(src && dst && weight && placed, "pxb_mirror_insert: a pointer is NULL");
  PXB_REQUIRE(mirror->ins_count != nullptr, "pxb_mirror_insert: ins_count is NULL");
  cudaStream_t st = as_stream(stream);
  const MirrorK m = to_k(mirror);
  if (m.groups <= kInsertMaxGroups) {
    const int64_t per_cta = int64_t(kInsertThreads) * kInsertPer;
    mirror_insert_grouped_kernel<<<static_cast<int>((k + per_cta - 1) / per_cta), kInsertThreads, 0, st>>>(
        m, k, src, dst, weight, placed, mirror->ins_count);
    PXB_LAUNCHED("mirror_insert_grouped_kernel");
  } else {
    mirror_insert_kernel<<<grid_for(k, 256, 8), 256, 0, st>>>(m, k, src, dst, weight, placed, mirror->ins_count);
    PXB_LAUNCHED("mirror_insert_kernel");
  }
  mirror_insert_finish_kernel<<<grid_for(m.groups, 256, 4), 256, 0, st>>>(m, mirror->ins_count);
  PXB_LAUNCHED("mirror_insert_finish_kernel");
  return PXB_OK;
}
