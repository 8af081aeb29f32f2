// Free-slot claim for growth: the i-th growable candidate of a claim domain
// takes that domain's i-th free slot in slot order.
//
// PIPELINE (src/plastax/phases.py:2985-3106): a dead slot below the bucket's
//   high-water mark belongs to the level of its former occupant's source
//   (unit_level[from_id]); each candidate level first takes its own domain's
//   slots, the rest spill to the never-used tail, levels ascending, in claim
//   order within a level. A spill past the global capacity overflows.
// TOPOLOGICAL (src/plastax/phases.py:2853-2982): one domain, every dead slot
//   of the bucket, candidates in claim order; no tail.
//
// Scheme-A: this rank holds global positions [shard_base, shard_base + cap).
// The per-domain free counts of the ranks before it (`level_before`) and the
// global totals (`level_totals`) come from an all-gather on the host side, so
// every rank takes identical decisions and writes only the slots it owns.
//
// Device work, no host synchronisation:
//   prepare: one warp per tile of slots counts the tile's free slots per
//            domain (level-major matrix), one exclusive scan over the matrix
//            gives each (domain, tile) its rank offset;
//   commit:  the candidates are stably sorted by level (radix), ranked within
//            their level and among the spills (scan), then the tiles that
//            hold a needed slot write it into a per-level list and one thread
//            per candidate writes its columns at the chosen slot.
#include <cub/cub.cuh>

#include "pxb_common.cuh"

namespace pxb {

static inline size_t align_up_c(size_t v, size_t a) { return (v + a - 1) / a * a; }

// The level-major commit (candidates listed levels ascending, no per-step
// cap) in four launches: per-block level counts, one plan block, the slot
// lists, the placement. A claiming candidate's position, its level's run
// and its spill rank all follow from the level counts, so no partition,
// run or scan pass over the candidates is needed.
constexpr int kLmThreads = 512;
constexpr int kLmMaxLevels = 64;
constexpr int kLmMaxBlocks = 1024;
// [blocks][levels] counts, [blocks] offsets, [levels] spill bases
static inline int64_t lm_words(int32_t num_levels) {
  const int64_t l = num_levels < kLmMaxLevels ? num_levels : kLmMaxLevels;
  return int64_t(kLmMaxBlocks) * l + kLmMaxBlocks + l;
}

constexpr int kClaimWarps = 8;         // warps per CTA in the tile kernels
constexpr int kMaxLevels = 1024;       // per-warp shared counters
constexpr int64_t kMaxMatrix = int64_t(1) << 24;

struct ClaimGeom {
  int64_t cap;
  int32_t num_levels;
  int tile_shift;  // log2(slots per tile)
  int64_t tiles;
};

static ClaimGeom geom_of(int64_t cap, int32_t num_levels, bool bitmap = false) {
  ClaimGeom g;
  g.cap = cap;
  g.num_levels = num_levels;
  g.tile_shift = bitmap ? 13 : 10;
  for (;;) {
    g.tiles = (cap + (int64_t(1) << g.tile_shift) - 1) >> g.tile_shift;
    if (g.tiles < 1) g.tiles = 1;
    if (g.tiles * num_levels <= kMaxMatrix || g.tile_shift >= 30) break;
    ++g.tile_shift;
  }
  return g;
}

struct ClaimScratch {
  int32_t *tile_counts, *tile_offsets;    // [num_levels * tiles]
  int32_t *level_local, *level_base;      // [num_levels]
  int32_t *level_first, *level_end;       // [num_levels + 1]
  int32_t *need, *need_off;               // [num_levels], [num_levels + 1]
  int32_t *list;                          // [k]
  uint32_t *ckey_in, *ckey_out;           // [k]
  int32_t *cidx_in, *cidx_out;            // [k]
  int32_t *flag, *rank;                   // [k]
  int32_t *counts;                        // [8]
  int32_t *lm;                            // level-major path: per-block level counts, offsets, spill bases
  void *cub_tmp;
  size_t cub_bytes, total;
};

static int claim_scratch(const ClaimGeom &g, int64_t k, char *base, ClaimScratch *o) {
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t at = off;
    off = align_up_c(off + (bytes ? bytes : 1), 256);
    return base ? base + at : nullptr;
  };
  const int64_t m = g.tiles * g.num_levels;
  const int64_t kk = k > 0 ? k : 1;
  o->tile_counts = reinterpret_cast<int32_t *>(take(m * 4));
  o->tile_offsets = reinterpret_cast<int32_t *>(take(m * 4));
  o->level_local = reinterpret_cast<int32_t *>(take(g.num_levels * 4));
  o->level_base = reinterpret_cast<int32_t *>(take(g.num_levels * 4));
  o->level_first = reinterpret_cast<int32_t *>(take((g.num_levels + 1) * 4));
  o->level_end = reinterpret_cast<int32_t *>(take((g.num_levels + 1) * 4));
  o->need = reinterpret_cast<int32_t *>(take(g.num_levels * 4));
  o->need_off = reinterpret_cast<int32_t *>(take((g.num_levels + 1) * 4));
  o->list = reinterpret_cast<int32_t *>(take(kk * 4));
  o->ckey_in = reinterpret_cast<uint32_t *>(take(kk * 4));
  o->ckey_out = reinterpret_cast<uint32_t *>(take(kk * 4));
  o->cidx_in = reinterpret_cast<int32_t *>(take(kk * 4));
  o->cidx_out = reinterpret_cast<int32_t *>(take(kk * 4));
  o->flag = reinterpret_cast<int32_t *>(take(kk * 4));
  o->rank = reinterpret_cast<int32_t *>(take(kk * 4));
  o->counts = reinterpret_cast<int32_t *>(take(8 * 4));
  o->lm = reinterpret_cast<int32_t *>(take(lm_words(g.num_levels) * 4));
  size_t t1 = 0, t2 = 0, t3 = 0, t4 = 0;
  if (cub::DeviceScan::ExclusiveSum(nullptr, t1, o->tile_counts, o->tile_offsets, static_cast<int>(m)) !=
      cudaSuccess)
    return PXB_ECUDA;
  if (cub::DevicePartition::Flagged(nullptr, t4, cub::CountingInputIterator<int32_t>(0), o->ckey_in, o->cidx_out,
                                    o->counts, static_cast<int>(kk)) != cudaSuccess)
    return PXB_ECUDA;
  if (cub::DeviceRadixSort::SortPairs(nullptr, t2, o->ckey_in, o->ckey_out, o->cidx_in, o->cidx_out,
                                      static_cast<int>(kk), 0, 32) != cudaSuccess)
    return PXB_ECUDA;
  if (cub::DeviceScan::ExclusiveSum(nullptr, t3, o->flag, o->rank, static_cast<int>(kk)) != cudaSuccess)
    return PXB_ECUDA;
  o->cub_bytes = t1 > t2 ? t1 : t2;
  if (t3 > o->cub_bytes) o->cub_bytes = t3;
  if (t4 > o->cub_bytes) o->cub_bytes = t4;
  o->cub_tmp = take(o->cub_bytes);
  o->total = off;
  return PXB_OK;
}

struct DomainArgs {
  int topo;  // 1: one domain of every dead slot, no tail
  int64_t cap;
  const int32_t *from;
  const uint8_t *dead;
  const int32_t *level;
  int32_t num_units, num_levels;
  int64_t shard_base;
  const int64_t *tail_start;  // device scalar (global position)
  const uint32_t *bm;         // per-domain free bitmaps [num_levels][bm_words], or NULL
  int64_t bm_words;
};

// Domain of slot s, or -1 when it is not a claimable free slot.
__device__ __forceinline__ int32_t slot_domain(const DomainArgs &a, int64_t s, int64_t tail) {
  if (s >= a.cap || !a.dead[s]) return -1;
  if (a.topo) return 0;
  if (a.shard_base + s >= tail) return -1;
  int32_t owner = a.from[s];
  owner = owner < 0 ? 0 : (owner >= a.num_units ? a.num_units - 1 : owner);
  const int32_t d = a.level[owner];
  return (d >= 0 && d < a.num_levels) ? d : -1;
}

// prepare: per-(domain, tile) free counts.
__global__ void __launch_bounds__(kClaimWarps * 32) tile_count_kernel(DomainArgs a, ClaimGeom g,
                                                                      int32_t *__restrict__ tile_counts) {
  __shared__ int32_t cnt[kClaimWarps][kMaxLevels];
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  const int64_t tail = a.topo ? 0 : *a.tail_start;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * kClaimWarps;
  const int64_t tile_slots = int64_t(1) << g.tile_shift;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * kClaimWarps + wib; t < g.tiles; t += warps) {
    for (int l = lane; l < g.num_levels; l += 32) cnt[wib][l] = 0;
    __syncwarp();
    const int64_t first = t * tile_slots;
    for (int64_t it = 0; it < tile_slots; it += 32) {
      const int64_t s = first + it + lane;
      if (first + it >= a.cap) break;
      const int32_t dom = slot_domain(a, s, tail);
      const unsigned active = __ballot_sync(0xffffffffu, dom >= 0);
      if (active == 0) continue;
      if (dom >= 0) {
        const unsigned peers = __match_any_sync(active, dom);
        if (lane == __ffs(peers) - 1) cnt[wib][dom] += __popc(peers);
      }
      __syncwarp();
    }
    __syncwarp();
    for (int l = lane; l < g.num_levels; l += 32) tile_counts[static_cast<int64_t>(l) * g.tiles + t] = cnt[wib][l];
    __syncwarp();
  }
}

// prepare from the per-domain bitmaps: a tile of 2^tile_shift slots is
// 2^(tile_shift-5) words; one warp per (tile, domain) pops its words.
__global__ void __launch_bounds__(kClaimWarps * 32) tile_count_bm_kernel(DomainArgs a, ClaimGeom g,
                                                                         int32_t *__restrict__ tile_counts) {
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * kClaimWarps;
  const int64_t words_per_tile = int64_t(1) << (g.tile_shift - 5);
  const int64_t jobs = g.tiles * g.num_levels;
  for (int64_t j = static_cast<int64_t>(blockIdx.x) * kClaimWarps + wib; j < jobs; j += warps) {
    const int64_t l = j / g.tiles, t = j - l * g.tiles;
    const uint32_t *row = a.bm + l * a.bm_words;
    int c = 0;
    const int64_t w_end = (t + 1) * words_per_tile < a.bm_words ? (t + 1) * words_per_tile : a.bm_words;
#pragma unroll 8
    for (int64_t w = t * words_per_tile + lane; w < w_end; w += 32) c += __popc(__ldg(row + w));
    c = __reduce_add_sync(0xffffffffu, c);
    if (lane == 0) tile_counts[j] = c;
  }
}

// level_local[L] = free slots of domain L on this rank; level_base[L] = its
// start in the level-major scan.
__global__ void level_totals_kernel(ClaimGeom g, const int32_t *__restrict__ tile_counts,
                                    const int32_t *__restrict__ tile_offsets, int32_t *__restrict__ level_local,
                                    int32_t *__restrict__ level_base, int32_t *__restrict__ out) {
  for (int l = blockIdx.x * blockDim.x + threadIdx.x; l < g.num_levels; l += gridDim.x * blockDim.x) {
    const int64_t lo = static_cast<int64_t>(l) * g.tiles, hi = lo + g.tiles - 1;
    const int32_t base = tile_offsets[lo];
    const int32_t n = tile_offsets[hi] + tile_counts[hi] - base;
    level_base[l] = base;
    level_local[l] = n;
    if (out) out[l] = n;
  }
}

// The (domain, tile) matrix's exclusive scan and the per-domain totals in
// one block, for a matrix of at most kPrepScanMax entries (one launch where
// the library scan takes two and the totals a third). Each thread reads a
// contiguous run, so the loads of a warp spread over as many lines as it
// has lanes: past a few entries per thread the library's multi-block scan
// is faster (64 per thread measured 30 us against its 6).
constexpr int kPrepScanThreads = 1024;
constexpr int64_t kPrepScanMax = int64_t(kPrepScanThreads) * 4;
__global__ void __launch_bounds__(kPrepScanThreads) prep_scan_kernel(ClaimGeom g, const int32_t *__restrict__ counts,
                                                                     int32_t *__restrict__ offsets,
                                                                     int32_t *__restrict__ level_local,
                                                                     int32_t *__restrict__ level_base,
                                                                     int32_t *__restrict__ out) {
  using Scan = cub::BlockScan<int32_t, kPrepScanThreads>;
  __shared__ typename Scan::TempStorage ts;
  const int64_t m = g.tiles * g.num_levels;
  const int64_t per = (m + kPrepScanThreads - 1) / kPrepScanThreads;
  const int64_t lo = threadIdx.x * per, hi = lo + per < m ? lo + per : m;
  int32_t mine = 0;
  for (int64_t j = lo; j < hi; ++j) mine += counts[j];
  int32_t ex, agg;
  Scan(ts).ExclusiveSum(mine, ex, agg);
  for (int64_t j = lo; j < hi; ++j) {
    offsets[j] = ex;
    ex += counts[j];
  }
  __syncthreads();  // the offsets are written
  for (int l = threadIdx.x; l < g.num_levels; l += blockDim.x) {
    const int64_t a = static_cast<int64_t>(l) * g.tiles, z = a + g.tiles - 1;
    const int32_t base = offsets[a];
    const int32_t n = offsets[z] + counts[z] - base;
    level_base[l] = base;
    level_local[l] = n;
    if (out) out[l] = n;
  }
}

struct CandArgs {
  int topo;
  int64_t k;
  const int32_t *src, *dst;
  const uint8_t *growable;
  const int32_t *level;
  int32_t num_units, num_levels;
  int64_t max_new;
};

__device__ __forceinline__ int32_t cand_level(const CandArgs &c, int64_t i) {
  if (c.topo) return 0;
  int32_t s = c.src[i];
  s = s < 0 ? 0 : (s >= c.num_units ? c.num_units - 1 : s);
  int32_t l = c.level[s];
  return l < 0 ? 0 : (l >= c.num_levels ? c.num_levels - 1 : l);
}

__global__ void growable_flag_kernel(CandArgs c, int32_t *__restrict__ flag) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < c.k;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    flag[i] = c.growable[i] ? 1 : 0;
}

// Sort keys: the candidate's level when it may claim (growable and under the
// per-step cap), the sentinel num_levels otherwise.
__global__ void cand_key_kernel(CandArgs c, const int32_t *__restrict__ grow_rank, uint32_t *__restrict__ key,
                                int32_t *__restrict__ idx) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < c.k;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    bool g = c.growable[i] != 0;
    if (g && c.max_new >= 0 && grow_rank != nullptr) g = grow_rank[i] < c.max_new;
    key[i] = g ? static_cast<uint32_t>(cand_level(c, i)) : static_cast<uint32_t>(c.num_levels);
    idx[i] = static_cast<int32_t>(i);
  }
}

// Level-major lists: the stable partition's flag (a claiming candidate), then
// the sort key of each partitioned position (its level, or the sentinel for
// the non-claiming tail, whose order no later stage reads).
__global__ void claim_flag_kernel(CandArgs c, const int32_t *__restrict__ grow_rank, uint32_t *__restrict__ flag) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < c.k;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    bool g = c.growable[i] != 0;
    if (g && c.max_new >= 0 && grow_rank != nullptr) g = grow_rank[i] < c.max_new;
    flag[i] = g ? 1u : 0u;
  }
}

__global__ void partition_key_kernel(CandArgs c, const int32_t *__restrict__ num_sel, const int32_t *__restrict__ idx,
                                     uint32_t *__restrict__ key) {
  const int64_t sel = *num_sel;
  for (int64_t p = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; p < c.k;
       p += static_cast<int64_t>(gridDim.x) * blockDim.x)
    key[p] = p < sel ? static_cast<uint32_t>(cand_level(c, idx[p])) : static_cast<uint32_t>(c.num_levels);
}

__global__ void level_runs_kernel(int64_t k, const uint32_t *__restrict__ key, int32_t *__restrict__ first,
                                  int32_t *__restrict__ end) {
  for (int64_t p = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; p < k;
       p += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint32_t kp = key[p];
    if (p == 0 || key[p - 1] != kp) first[kp] = static_cast<int32_t>(p);
    if (p == k - 1 || key[p + 1] != kp) end[kp] = static_cast<int32_t>(p + 1);
  }
}

struct TotalsArgs {
  const int32_t *level_local, *level_before, *level_totals;
};

__device__ __forceinline__ int32_t total_of(const TotalsArgs &t, int l) {
  return t.level_totals ? t.level_totals[l] : t.level_local[l];
}
__device__ __forceinline__ int32_t before_of(const TotalsArgs &t, int l) {
  return t.level_before ? t.level_before[l] : 0;
}

// spill flag per sorted position: a claiming candidate past its level's
// global free count.
__global__ void spill_flag_kernel(int64_t k, int32_t num_levels, const uint32_t *__restrict__ key,
                                  const int32_t *__restrict__ first, TotalsArgs t, int32_t *__restrict__ flag) {
  for (int64_t p = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; p < k;
       p += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint32_t l = key[p];
    int32_t f = 0;
    if (l < static_cast<uint32_t>(num_levels)) f = (p - first[l]) >= total_of(t, l) ? 1 : 0;
    flag[p] = f;
  }
}

// need[L]: this rank's domain-L slots that own claims take; need_off: their
// offsets in the list (one thread: the level count is small).
__global__ void need_kernel(int32_t num_levels, const int32_t *__restrict__ first, const int32_t *__restrict__ end,
                            TotalsArgs t, int32_t *__restrict__ need, int32_t *__restrict__ need_off) {
  if (blockIdx.x != 0 || threadIdx.x != 0) return;
  int32_t acc = 0;
  for (int l = 0; l < num_levels; ++l) {
    const int32_t kl = end[l] - first[l];
    const int32_t tot = total_of(t, l);
    int32_t own = kl < tot ? kl : tot;
    int32_t n = own - before_of(t, l);
    if (n < 0) n = 0;
    if (n > t.level_local[l]) n = t.level_local[l];
    need[l] = n;
    need_off[l] = acc;
    acc += n;
  }
  need_off[num_levels] = acc;
}

struct LmGeom {
  int64_t chunk;   // candidates per block, a multiple of kLmThreads
  int32_t blocks;  // <= kLmMaxBlocks
};

static LmGeom lm_geom(int64_t k) {
  LmGeom lg;
  int64_t chunk = int64_t(kLmThreads) * 4;
  if ((k + chunk - 1) / chunk > kLmMaxBlocks) chunk = (k + kLmMaxBlocks - 1) / kLmMaxBlocks;
  chunk = (chunk + kLmThreads - 1) / kLmThreads * kLmThreads;
  lg.chunk = chunk;
  lg.blocks = static_cast<int32_t>((k + chunk - 1) / chunk);
  if (lg.blocks < 1) lg.blocks = 1;
  return lg;
}

// Pass 1: each block's claiming candidates per level (a warp adds each
// level it saw once).
__global__ void __launch_bounds__(kLmThreads) lm_count_kernel(CandArgs c, LmGeom lg, int32_t *__restrict__ lm) {
  __shared__ int32_t cnt[kLmMaxLevels];
  const int L = c.num_levels;
  for (int l = threadIdx.x; l < L; l += blockDim.x) cnt[l] = 0;
  __syncthreads();
  const int64_t lo = static_cast<int64_t>(blockIdx.x) * lg.chunk;
  const int64_t hi = lo + lg.chunk < c.k ? lo + lg.chunk : c.k;
  for (int64_t base = lo; base < hi; base += blockDim.x) {
    const int64_t i = base + threadIdx.x;
    const bool g = i < hi && c.growable[i] != 0;
    const int32_t l = g ? cand_level(c, i) : -1;
    const unsigned active = __ballot_sync(0xffffffffu, g);
    if (g) {
      const unsigned peers = __match_any_sync(active, l);
      if ((threadIdx.x & 31) == __ffs(peers) - 1) atomicAdd(&cnt[l], __popc(peers));
    }
  }
  __syncthreads();
  for (int l = threadIdx.x; l < L; l += blockDim.x) lm[static_cast<int64_t>(blockIdx.x) * L + l] = cnt[l];
}

// One block: each block's first claiming position, the level runs, this
// rank's needs per level and the spill bases; the commit's counters cleared.
__global__ void __launch_bounds__(1024) lm_plan_kernel(CandArgs c, LmGeom lg, TotalsArgs t, int32_t *__restrict__ lm,
                                                       int32_t *__restrict__ first, int32_t *__restrict__ end,
                                                       int32_t *__restrict__ need, int32_t *__restrict__ need_off,
                                                       int32_t *__restrict__ counts) {
  using Scan = cub::BlockScan<int32_t, 1024>;
  __shared__ typename Scan::TempStorage ts;
  __shared__ int32_t cnt[kLmMaxLevels];
  const int L = c.num_levels;
  const int b = threadIdx.x;
  int32_t *off = lm + static_cast<int64_t>(kLmMaxBlocks) * L;
  int32_t *spill_base = off + kLmMaxBlocks;
  for (int l = threadIdx.x; l < L; l += blockDim.x) cnt[l] = 0;
  if (threadIdx.x < 8) counts[threadIdx.x] = 0;
  __syncthreads();
  int32_t tot = 0;
  for (int l = 0; l < L; ++l) {
    const int32_t v = b < lg.blocks ? lm[static_cast<int64_t>(b) * L + l] : 0;
    tot += v;
    const int32_t w = __reduce_add_sync(0xffffffffu, v);
    if ((threadIdx.x & 31) == 0 && w) atomicAdd(&cnt[l], w);
  }
  int32_t ex, agg;
  Scan(ts).ExclusiveSum(tot, ex, agg);
  if (b < lg.blocks) off[b] = ex;
  __syncthreads();
  if (threadIdx.x == 0) {
    int32_t run = 0, acc = 0, spill = 0;
    for (int l = 0; l < L; ++l) {
      const int32_t kl = cnt[l], total = total_of(t, l);
      first[l] = run;
      end[l] = run + kl;
      run += kl;
      int32_t own = kl < total ? kl : total;
      int32_t n = own - before_of(t, l);
      if (n < 0) n = 0;
      if (n > t.level_local[l]) n = t.level_local[l];
      need[l] = n;
      need_off[l] = acc;
      acc += n;
      spill_base[l] = spill;
      if (kl > total) spill += kl - total;
    }
    need_off[L] = acc;
  }
}

// list fill: the needed free slots of each domain, in slot order.
__global__ void __launch_bounds__(kClaimWarps * 32) list_fill_kernel(
    DomainArgs a, ClaimGeom g, const int32_t *__restrict__ tile_offsets, const int32_t *__restrict__ level_base,
    const int32_t *__restrict__ need, const int32_t *__restrict__ need_off, int32_t *__restrict__ list) {
  __shared__ int32_t run[kClaimWarps][kMaxLevels];
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  const int64_t tail = a.topo ? 0 : *a.tail_start;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * kClaimWarps;
  const int64_t tile_slots = int64_t(1) << g.tile_shift;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * kClaimWarps + wib; t < g.tiles; t += warps) {
    // Skip a tile none of whose domains still needs a slot at its rank.
    bool useful = false;
    for (int l = lane; l < g.num_levels; l += 32) {
      const int32_t r0 = tile_offsets[static_cast<int64_t>(l) * g.tiles + t] - level_base[l];
      run[wib][l] = r0;
      useful = useful || r0 < need[l];
    }
    if (!__any_sync(0xffffffffu, useful)) continue;
    __syncwarp();
    const int64_t first = t * tile_slots;
    for (int64_t it = 0; it < tile_slots; it += 32) {
      if (first + it >= a.cap) break;
      const int64_t s = first + it + lane;
      const int32_t dom = slot_domain(a, s, tail);
      const unsigned active = __ballot_sync(0xffffffffu, dom >= 0);
      if (active == 0) continue;
      if (dom >= 0) {
        const unsigned peers = __match_any_sync(active, dom);
        const int32_t r = run[wib][dom] + __popc(peers & ((1u << lane) - 1u));
        if (r < need[dom]) list[need_off[dom] + r] = static_cast<int32_t>(s);
        __syncwarp(peers);
        if (lane == __ffs(peers) - 1) run[wib][dom] += __popc(peers);
      }
      __syncwarp();
    }
    __syncwarp();
  }
}

// list fill from the bitmaps: one warp per (tile, domain) that still owes
// needed ranks. A tile is read 256 words at a time, eight consecutive words
// per lane issued together (one memory round trip per 256 words, not one
// per 32); a warp scan of the lanes' popcounts gives each set bit its rank
// in slot order.
__global__ void __launch_bounds__(kClaimWarps * 32) list_fill_bm_kernel(
    DomainArgs a, ClaimGeom g, const int32_t *__restrict__ tile_offsets, const int32_t *__restrict__ level_base,
    const int32_t *__restrict__ need, const int32_t *__restrict__ need_off, int32_t *__restrict__ list) {
  constexpr int kWordsPerLane = 8;
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * kClaimWarps;
  const int64_t words_per_tile = int64_t(1) << (g.tile_shift - 5);
  const int64_t jobs = g.tiles * g.num_levels;
  for (int64_t j = static_cast<int64_t>(blockIdx.x) * kClaimWarps + wib; j < jobs; j += warps) {
    const int64_t l = j / g.tiles, t = j - l * g.tiles;
    int32_t run = tile_offsets[j] - level_base[l];
    const int32_t nl = need[l];
    if (run >= nl) continue;
    const uint32_t *row = a.bm + l * a.bm_words;
    const int32_t off = need_off[l];
    const int64_t w_end = (t + 1) * words_per_tile < a.bm_words ? (t + 1) * words_per_tile : a.bm_words;
    for (int64_t w0 = t * words_per_tile; w0 < w_end && run < nl; w0 += 32 * kWordsPerLane) {
      const int64_t wl = w0 + lane * kWordsPerLane;
      uint32_t bits[kWordsPerLane];
      int pc = 0;
#pragma unroll
      for (int q = 0; q < kWordsPerLane; ++q) {
        bits[q] = wl + q < w_end ? __ldg(row + wl + q) : 0u;
        pc += __popc(bits[q]);
      }
      int incl = pc;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      int r = run + incl - pc;
#pragma unroll
      for (int q = 0; q < kWordsPerLane; ++q) {
        uint32_t b = bits[q];
        while (b && r < nl) {
          list[off + r] = static_cast<int32_t>((wl + q) * 32 + (__ffs(b) - 1));
          b &= b - 1;
          ++r;
        }
      }
      run += __shfl_sync(0xffffffffu, incl, 31);
    }
  }
}

struct WriteArgs {
  int topo;
  int64_t cap, shard_base, global_cap;
  const int64_t *tail_start;
  int32_t *from, *to;
  uint8_t *dead;
  float *weight;
  int32_t n_extra;
  void *extra_cols[8];
  int32_t extra_bytes[8];
  const void *extra_vals[8];
  uint32_t *bm;  // per-domain free bitmaps to clear at placed own slots, or NULL
  int64_t bm_words;
  int32_t *placed;  // per candidate: the local slot written, -1 when none
  uint8_t *committed;  // per candidate: 1 when committed on any rank, or NULL
};

struct PlaceTally {
  int committed = 0, over = 0, tail = 0, resort = 0;
};

// Claiming candidate i of level l, own_rank-th of its level: its slot (its
// level's own domain, else the tail at its spill rank), the columns written
// when this rank holds the slot, the tallies. `spill_rank(i)` is read only
// past the level's free count.
template <class SpillRank>
__device__ __forceinline__ void place_one(const CandArgs &c, const WriteArgs &w, const TotalsArgs &t, int64_t tail,
                                          int64_t tail_free, int32_t i, uint32_t l, int32_t own_rank,
                                          SpillRank spill_rank, const int32_t *__restrict__ need,
                                          const int32_t *__restrict__ need_off, const int32_t *__restrict__ list,
                                          const float *__restrict__ cand_w, uint8_t *__restrict__ overflowed,
                                          PlaceTally &tl) {
  int n_committed = 0, n_over = 0, n_tail = 0, n_resort = 0;
  {
    int64_t slot = -1;
    bool committed = false, to_tail = false;
    if (own_rank < total_of(t, l)) {
      committed = true;
      const int32_t r = own_rank - before_of(t, l);
      if (r >= 0 && r < need[l]) slot = list[need_off[l] + r];
    } else {
      const int64_t sr = spill_rank();
      if (sr < tail_free) {
        committed = true;
        to_tail = true;
        const int64_t pos = tail + sr;
        if (pos >= w.shard_base && pos < w.shard_base + w.cap) slot = pos - w.shard_base;
      } else if (overflowed) {
        overflowed[i] = 1;
      }
    }
    if (committed) {
      if (w.committed) w.committed[i] = 1;
      ++n_committed;
      if (to_tail) ++n_tail;
      const int32_t s = c.src[i], d = c.dst[i];
      const bool in = s >= 0 && s < c.num_units && d >= 0 && d < c.num_units;
      if (in && c.level[d] <= c.level[s]) ++n_resort;
    } else {
      ++n_over;
    }
    if (slot >= 0 && slot < w.cap) {
      w.from[slot] = c.src[i];
      w.to[slot] = c.dst[i];
      w.weight[slot] = cand_w[i];
      for (int e = 0; e < w.n_extra; ++e) {
        if (w.extra_bytes[e] == 4)
          reinterpret_cast<int32_t *>(w.extra_cols[e])[slot] = reinterpret_cast<const int32_t *>(w.extra_vals[e])[i];
        else
          reinterpret_cast<uint8_t *>(w.extra_cols[e])[slot] = reinterpret_cast<const uint8_t *>(w.extra_vals[e])[i];
      }
      w.dead[slot] = 0;
      if (w.bm != nullptr && !to_tail)
        atomicAnd(w.bm + static_cast<int64_t>(l) * w.bm_words + (slot >> 5), ~(1u << (slot & 31)));
      if (w.placed) w.placed[i] = static_cast<int32_t>(slot);
    }
  }
  tl.committed += n_committed;
  tl.over += n_over;
  tl.tail += n_tail;
  tl.resort += n_resort;
}

// The tallies added once per warp, then once per block (one address takes
// every candidate's increment otherwise).
__device__ __forceinline__ void add_tallies(PlaceTally tl, int32_t *__restrict__ counts) {
  __shared__ int s_counts[4];
  if (threadIdx.x < 4) s_counts[threadIdx.x] = 0;
  __syncthreads();
  const int n_committed = __reduce_add_sync(0xffffffffu, tl.committed);
  const int n_over = __reduce_add_sync(0xffffffffu, tl.over);
  const int n_tail = __reduce_add_sync(0xffffffffu, tl.tail);
  const int n_resort = __reduce_add_sync(0xffffffffu, tl.resort);
  if ((threadIdx.x & 31) == 0) {
    if (n_committed) atomicAdd(&s_counts[0], n_committed);
    if (n_over) atomicAdd(&s_counts[1], n_over);
    if (n_tail) atomicAdd(&s_counts[2], n_tail);
    if (n_resort) atomicAdd(&s_counts[3], n_resort);
  }
  __syncthreads();
  if (threadIdx.x < 4 && s_counts[threadIdx.x]) atomicAdd(counts + threadIdx.x, s_counts[threadIdx.x]);
}

// One thread per sorted claim position: choose the slot and write.
__global__ void place_kernel(CandArgs c, WriteArgs w, const uint32_t *__restrict__ key,
                             const int32_t *__restrict__ idx, const int32_t *__restrict__ first, TotalsArgs t,
                             const int32_t *__restrict__ spill_rank, const int32_t *__restrict__ need,
                             const int32_t *__restrict__ need_off, const int32_t *__restrict__ list,
                             const float *__restrict__ cand_w, int32_t *__restrict__ counts,
                             uint8_t *__restrict__ overflowed) {
  const int64_t tail = w.topo ? 0 : *w.tail_start;
  const int64_t tail_free = w.topo ? 0 : w.global_cap - tail;
  PlaceTally tl;
  for (int64_t p = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; p < c.k;
       p += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint32_t l = key[p];
    const int32_t i = idx[p];
    if (overflowed) overflowed[i] = 0;
    if (w.placed) w.placed[i] = -1;
    if (w.committed) w.committed[i] = 0;
    if (l >= static_cast<uint32_t>(c.num_levels)) continue;
    place_one(c, w, t, tail, tail_free, i, l, static_cast<int32_t>(p) - first[l],
              [&] { return static_cast<int64_t>(spill_rank[p]); }, need, need_off, list, cand_w, overflowed, tl);
  }
  add_tallies(tl, counts);
}

// The level-major placement: candidate i's position among the claiming
// candidates is its block's offset plus its rank inside the block (a block
// scan per 512), its level's run starts at first[l], and past the level's
// free count its spill rank is the spill base of its level plus its rank
// among the level's spills.
__global__ void __launch_bounds__(kLmThreads) lm_place_kernel(CandArgs c, WriteArgs w, LmGeom lg,
                                                              const int32_t *__restrict__ lm,
                                                              const int32_t *__restrict__ first, TotalsArgs t,
                                                              const int32_t *__restrict__ need,
                                                              const int32_t *__restrict__ need_off,
                                                              const int32_t *__restrict__ list,
                                                              const float *__restrict__ cand_w,
                                                              int32_t *__restrict__ counts,
                                                              uint8_t *__restrict__ overflowed) {
  using Scan = cub::BlockScan<int32_t, kLmThreads>;
  __shared__ typename Scan::TempStorage ts;
  const int L = c.num_levels;
  const int32_t *off = lm + static_cast<int64_t>(kLmMaxBlocks) * L;
  const int32_t *spill_base = off + kLmMaxBlocks;
  const int64_t tail = w.topo ? 0 : *w.tail_start;
  const int64_t tail_free = w.topo ? 0 : w.global_cap - tail;
  const int64_t lo = static_cast<int64_t>(blockIdx.x) * lg.chunk;
  const int64_t hi = lo + lg.chunk < c.k ? lo + lg.chunk : c.k;
  int32_t carry = off[blockIdx.x];
  PlaceTally tl;
  for (int64_t base = lo; base < hi; base += blockDim.x) {
    const int64_t i = base + threadIdx.x;
    const bool in = i < hi;
    const bool g = in && c.growable[i] != 0;
    int32_t ex, agg;
    Scan(ts).ExclusiveSum(g ? 1 : 0, ex, agg);
    if (in) {
      if (overflowed) overflowed[i] = 0;
      if (w.placed) w.placed[i] = -1;
      if (w.committed) w.committed[i] = 0;
    }
    if (g) {
      const int32_t l = cand_level(c, i);
      const int32_t own_rank = carry + ex - first[l];
      place_one(c, w, t, tail, tail_free, static_cast<int32_t>(i), static_cast<uint32_t>(l), own_rank,
                [&] { return static_cast<int64_t>(spill_base[l]) + (own_rank - total_of(t, l)); }, need, need_off,
                list, cand_w, overflowed, tl);
    }
    carry += agg;
    __syncthreads();  // the scan's storage is reused
  }
  add_tallies(tl, counts);
}

__global__ void finish_kernel(int topo, int64_t *tail_start, const int32_t *__restrict__ counts,
                              int32_t *__restrict__ out) {
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    if (!topo && tail_start) *tail_start += counts[2];
    if (out)
      for (int j = 0; j < 4; ++j) out[j] = counts[j];
  }
}

// The step's growth flags from a claim's counts (committed, overflowed,
// tail used, resort): grown (+)= committed, overflow |= overflowed > 0,
// needs_resort |= resort > 0; reset starts grown and overflow afresh.
__global__ void growth_flags_kernel(const int32_t *__restrict__ counts, int32_t reset, int32_t *grown,
                                    uint8_t *overflow, uint8_t *needs_resort) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  if (grown) *grown = (reset ? 0 : *grown) + counts[0];
  if (overflow) *overflow = static_cast<uint8_t>((reset ? 0 : *overflow) | (counts[1] > 0 ? 1 : 0));
  if (needs_resort) *needs_resort = static_cast<uint8_t>(*needs_resort | (counts[3] > 0 ? 1 : 0));
}

// The commit's counters and level runs cleared in one launch (a memset
// node per array costs a gap of microseconds before the next kernel).
__global__ void claim_reset_kernel(int32_t *counts, int32_t *level_first, int32_t *level_end, int32_t levels) {
  for (int i = threadIdx.x; i < 8; i += blockDim.x) counts[i] = 0;
  if (level_first != nullptr)
    for (int i = threadIdx.x; i <= levels; i += blockDim.x) {
      level_first[i] = 0;
      level_end[i] = 0;
    }
}

// The end of a step: the growth flags of a step that claimed nothing
// cleared (when given) and the device step counter advanced, in one launch.
__global__ void step_end_kernel(int32_t *step, int32_t *grown, uint8_t *overflow) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  if (grown) *grown = 0;
  if (overflow) *overflow = 0;
  if (step) *step += 1;
}

}  // namespace pxb

using namespace pxb;

extern "C" int pxb_step_end(int32_t *step, int32_t *grown, uint8_t *overflow, void *stream) {
  step_end_kernel<<<1, 32, 0, as_stream(stream)>>>(step, grown, overflow);
  PXB_LAUNCHED("step_end_kernel");
  return PXB_OK;
}

extern "C" int pxb_growth_flags(const int32_t *counts, int32_t reset, int32_t *grown, uint8_t *overflow,
                                uint8_t *needs_resort, void *stream) {
  PXB_REQUIRE(counts != nullptr, "pxb_growth_flags: counts is NULL");
  growth_flags_kernel<<<1, 32, 0, as_stream(stream)>>>(counts, reset, grown, overflow, needs_resort);
  PXB_LAUNCHED("growth_flags_kernel");
  return PXB_OK;
}

extern "C" int pxb_claim_scratch_bytes(int64_t cap, int64_t k, int32_t num_levels, size_t *bytes) {
  PXB_REQUIRE(bytes != nullptr, "pxb_claim_scratch_bytes: bytes is NULL");
  PXB_REQUIRE(cap >= 0 && cap < (int64_t(1) << 31) && k >= 0 && k < (int64_t(1) << 31),
              "pxb_claim_scratch_bytes: sizes out of range");
  PXB_REQUIRE(num_levels >= 1 && num_levels <= kMaxLevels, "pxb_claim_scratch_bytes: num_levels %d not in [1, %d]",
              num_levels, kMaxLevels);
  ClaimScratch o;
  if (claim_scratch(geom_of(cap, num_levels), k, nullptr, &o) != PXB_OK) {
    set_error("pxb_claim_scratch_bytes: CUB size query failed");
    return PXB_ECUDA;
  }
  *bytes = o.total;
  return PXB_OK;
}

static int claim_common_checks(const char *fn, int32_t mode, int64_t cap, int32_t num_levels) {
  PXB_REQUIRE(mode == PXB_CLAIM_PIPELINE || mode == PXB_CLAIM_TOPOLOGICAL, "%s: unknown mode %d", fn, mode);
  PXB_REQUIRE(cap >= 0 && cap < (int64_t(1) << 31), "%s: capacity out of range", fn);
  PXB_REQUIRE(num_levels >= 1 && num_levels <= kMaxLevels, "%s: num_levels %d not in [1, %d]", fn, num_levels,
              kMaxLevels);
  return PXB_OK;
}

extern "C" int pxb_claim_prepare(int32_t mode, int64_t cap, const int32_t *from_id, const uint8_t *dead,
                                 const int32_t *unit_level, int32_t num_units, int32_t num_levels,
                                 int64_t shard_base, const int64_t *tail_start, const uint32_t *free_bitmap,
                                 int64_t k, int32_t *level_counts, void *scratch, size_t scratch_bytes,
                                 void *stream) {
  mode &= ~PXB_CLAIM_LEVEL_MAJOR;  // the list's order does not concern the domains' counts
  int rc = claim_common_checks("pxb_claim_prepare", mode, cap, num_levels);
  if (rc) return rc;
  const int topo = mode == PXB_CLAIM_TOPOLOGICAL;
  if (topo) num_levels = 1;
  PXB_REQUIRE(scratch != nullptr, "pxb_claim_prepare: scratch is NULL");
  PXB_REQUIRE(free_bitmap || topo || (from_id && unit_level && tail_start && num_units > 0),
              "pxb_claim_prepare: pipeline mode needs from_id, unit_level, num_units and tail_start");
  PXB_REQUIRE(free_bitmap || cap == 0 || dead, "pxb_claim_prepare: dead is NULL");
  const ClaimGeom g = geom_of(cap, num_levels, free_bitmap != nullptr);
  ClaimScratch o;
  if (claim_scratch(g, k, static_cast<char *>(scratch), &o) != PXB_OK) {
    set_error("pxb_claim_prepare: CUB size query failed");
    return PXB_ECUDA;
  }
  PXB_REQUIRE(o.total <= scratch_bytes, "pxb_claim_prepare: scratch has %zu bytes, needs %zu", scratch_bytes,
              o.total);
  cudaStream_t st = as_stream(stream);
  const int64_t m = g.tiles * g.num_levels;
  // the bitmap count writes every (domain, tile) entry; the byte count and
  // an empty band need the zeros
  if (free_bitmap == nullptr || cap == 0) PXB_CUDA(cudaMemsetAsync(o.tile_counts, 0, m * 4, st));
  if (cap > 0) {
    DomainArgs a{topo, cap, from_id, dead, unit_level, num_units, num_levels, shard_base, tail_start,
                 free_bitmap, (cap + 31) / 32};
    if (free_bitmap != nullptr) {
      tile_count_bm_kernel<<<grid_for(m, kClaimWarps, 4), kClaimWarps * 32, 0, st>>>(a, g, o.tile_counts);
      PXB_LAUNCHED("tile_count_bm_kernel");
    } else {
      tile_count_kernel<<<grid_for(g.tiles, kClaimWarps, 4), kClaimWarps * 32, 0, st>>>(a, g, o.tile_counts);
      PXB_LAUNCHED("tile_count_kernel");
    }
  }
  if (m <= kPrepScanMax) {
    prep_scan_kernel<<<1, kPrepScanThreads, 0, st>>>(g, o.tile_counts, o.tile_offsets, o.level_local, o.level_base,
                                                     level_counts);
    PXB_LAUNCHED("prep_scan_kernel");
    return PXB_OK;
  }
  size_t tb = o.cub_bytes;
  PXB_CUDA(cub::DeviceScan::ExclusiveSum(o.cub_tmp, tb, o.tile_counts, o.tile_offsets, static_cast<int>(m), st));
  level_totals_kernel<<<(num_levels + 255) / 256, 256, 0, st>>>(g, o.tile_counts, o.tile_offsets, o.level_local,
                                                               o.level_base, level_counts);
  PXB_LAUNCHED("level_totals_kernel");
  return PXB_OK;
}

extern "C" int pxb_claim_commit(int32_t mode, int64_t cap, int32_t *from_id, int32_t *to_id, uint8_t *dead,
                                float *weight, const int32_t *unit_level, int32_t num_units, int32_t num_levels,
                                int64_t shard_base, int64_t global_cap, int64_t *tail_start, int64_t k,
                                const int32_t *cand_src, const int32_t *cand_dst, const float *cand_weight,
                                const uint8_t *growable, int64_t max_new, const int32_t *level_before,
                                const int32_t *level_totals, uint32_t *free_bitmap, int32_t n_extra,
                                void *const *extra_cols, const int32_t *extra_bytes, const void *const *extra_vals,
                                int32_t *counts_out, uint8_t *overflowed_out, int32_t *placed_out,
                                uint8_t *committed_out, void *scratch, size_t scratch_bytes, void *stream) {
  const bool level_major = (mode & PXB_CLAIM_LEVEL_MAJOR) != 0;
  mode &= ~PXB_CLAIM_LEVEL_MAJOR;
  int rc = claim_common_checks("pxb_claim_commit", mode, cap, num_levels);
  if (rc) return rc;
  const int topo = mode == PXB_CLAIM_TOPOLOGICAL;
  if (topo) num_levels = 1;
  PXB_REQUIRE(k >= 0 && k < (int64_t(1) << 31), "pxb_claim_commit: k out of range");
  PXB_REQUIRE(n_extra >= 0 && n_extra <= 8, "pxb_claim_commit: at most 8 extra columns");
  PXB_REQUIRE(scratch != nullptr, "pxb_claim_commit: scratch is NULL");
  PXB_REQUIRE(unit_level && num_units > 0, "pxb_claim_commit: unit_level/num_units required");
  PXB_REQUIRE(topo || tail_start, "pxb_claim_commit: pipeline mode needs tail_start");
  PXB_REQUIRE(cap == 0 || (from_id && to_id && dead && weight), "pxb_claim_commit: a bucket column is NULL");
  PXB_REQUIRE(k == 0 || (cand_src && cand_dst && cand_weight && growable), "pxb_claim_commit: candidates are NULL");
  PXB_REQUIRE(global_cap >= shard_base + cap, "pxb_claim_commit: global_cap below this rank's band");
  const ClaimGeom g = geom_of(cap, num_levels, free_bitmap != nullptr);
  ClaimScratch o;
  if (claim_scratch(g, k, static_cast<char *>(scratch), &o) != PXB_OK) {
    set_error("pxb_claim_commit: CUB size query failed");
    return PXB_ECUDA;
  }
  PXB_REQUIRE(o.total <= scratch_bytes, "pxb_claim_commit: scratch has %zu bytes, needs %zu", scratch_bytes,
              o.total);
  WriteArgs w;
  w.topo = topo;
  w.cap = cap;
  w.shard_base = shard_base;
  w.global_cap = global_cap;
  w.tail_start = tail_start;
  w.from = from_id;
  w.to = to_id;
  w.dead = dead;
  w.weight = weight;
  w.n_extra = n_extra;
  w.bm = free_bitmap;
  w.bm_words = (cap + 31) / 32;
  w.placed = placed_out;
  w.committed = committed_out;
  for (int e = 0; e < n_extra; ++e) {
    PXB_REQUIRE(extra_cols && extra_bytes && extra_vals && extra_cols[e] && extra_vals[e],
                "pxb_claim_commit: extra column %d is NULL", e);
    PXB_REQUIRE(extra_bytes[e] == 1 || extra_bytes[e] == 4, "pxb_claim_commit: extra column %d has %d-byte elements",
                e, extra_bytes[e]);
    w.extra_cols[e] = extra_cols[e];
    w.extra_bytes[e] = extra_bytes[e];
    w.extra_vals[e] = extra_vals[e];
  }
  cudaStream_t st = as_stream(stream);
  if (k > 0 && level_major && max_new < 0 && num_levels <= kLmMaxLevels) {
    // the level-major list without a per-step cap: four launches (the
    // plan clears the counters)
    CandArgs c{topo, k, cand_src, cand_dst, growable, unit_level, num_units, num_levels, max_new};
    const LmGeom lg = lm_geom(k);
    TotalsArgs t{o.level_local, level_before, level_totals};
    lm_count_kernel<<<lg.blocks, kLmThreads, 0, st>>>(c, lg, o.lm);
    PXB_LAUNCHED("lm_count_kernel");
    lm_plan_kernel<<<1, 1024, 0, st>>>(c, lg, t, o.lm, o.level_first, o.level_end, o.need, o.need_off, o.counts);
    PXB_LAUNCHED("lm_plan_kernel");
    if (cap > 0) {
      DomainArgs a{topo, cap, from_id, dead, unit_level, num_units, num_levels, shard_base, tail_start,
                   free_bitmap, (cap + 31) / 32};
      if (free_bitmap != nullptr) {
        list_fill_bm_kernel<<<grid_for(g.tiles * g.num_levels, kClaimWarps, 4), kClaimWarps * 32, 0, st>>>(
            a, g, o.tile_offsets, o.level_base, o.need, o.need_off, o.list);
        PXB_LAUNCHED("list_fill_bm_kernel");
      } else {
        list_fill_kernel<<<grid_for(g.tiles, kClaimWarps, 4), kClaimWarps * 32, 0, st>>>(
            a, g, o.tile_offsets, o.level_base, o.need, o.need_off, o.list);
        PXB_LAUNCHED("list_fill_kernel");
      }
    }
    lm_place_kernel<<<lg.blocks, kLmThreads, 0, st>>>(c, w, lg, o.lm, o.level_first, t, o.need, o.need_off, o.list,
                                                       cand_weight, o.counts, overflowed_out);
    PXB_LAUNCHED("lm_place_kernel");
    finish_kernel<<<1, 32, 0, st>>>(topo, tail_start, o.counts, counts_out);
    PXB_LAUNCHED("finish_kernel");
    return PXB_OK;
  }
  claim_reset_kernel<<<1, 128, 0, st>>>(o.counts, k > 0 ? o.level_first : nullptr, o.level_end, num_levels);
  PXB_LAUNCHED("claim_reset_kernel");
  if (k > 0) {
    CandArgs c{topo, k, cand_src, cand_dst, growable, unit_level, num_units, num_levels, max_new};
    const int grid = grid_for(k, 256, 8);
    const int32_t *grow_rank = nullptr;
    size_t tb;
    if (max_new >= 0) {
      growable_flag_kernel<<<grid, 256, 0, st>>>(c, o.flag);
      PXB_LAUNCHED("growable_flag_kernel");
      tb = o.cub_bytes;
      PXB_CUDA(cub::DeviceScan::ExclusiveSum(o.cub_tmp, tb, o.flag, o.rank, static_cast<int>(k), st));
      grow_rank = o.rank;
    }
    if (level_major) {
      // claiming candidates already ascend by level: a stable partition
      // gives the order the level sort would
      claim_flag_kernel<<<grid, 256, 0, st>>>(c, grow_rank, o.ckey_in);
      PXB_LAUNCHED("claim_flag_kernel");
      tb = o.cub_bytes;
      PXB_CUDA(cub::DevicePartition::Flagged(o.cub_tmp, tb, cub::CountingInputIterator<int32_t>(0), o.ckey_in,
                                             o.cidx_out, o.counts + 7, static_cast<int>(k), st));
      partition_key_kernel<<<grid, 256, 0, st>>>(c, o.counts + 7, o.cidx_out, o.ckey_out);
      PXB_LAUNCHED("partition_key_kernel");
    } else {
      cand_key_kernel<<<grid, 256, 0, st>>>(c, grow_rank, o.ckey_in, o.cidx_in);
      PXB_LAUNCHED("cand_key_kernel");
      int key_bits = 1;
      while ((1u << key_bits) <= static_cast<uint32_t>(num_levels)) ++key_bits;
      tb = o.cub_bytes;
      PXB_CUDA(cub::DeviceRadixSort::SortPairs(o.cub_tmp, tb, o.ckey_in, o.ckey_out, o.cidx_in, o.cidx_out,
                                               static_cast<int>(k), 0, key_bits, st));
    }
    level_runs_kernel<<<grid, 256, 0, st>>>(k, o.ckey_out, o.level_first, o.level_end);
    PXB_LAUNCHED("level_runs_kernel");
    TotalsArgs t{o.level_local, level_before, level_totals};
    spill_flag_kernel<<<grid, 256, 0, st>>>(k, num_levels, o.ckey_out, o.level_first, t, o.flag);
    PXB_LAUNCHED("spill_flag_kernel");
    tb = o.cub_bytes;
    PXB_CUDA(cub::DeviceScan::ExclusiveSum(o.cub_tmp, tb, o.flag, o.rank, static_cast<int>(k), st));
    need_kernel<<<1, 1, 0, st>>>(num_levels, o.level_first, o.level_end, t, o.need, o.need_off);
    PXB_LAUNCHED("need_kernel");
    if (cap > 0) {
      DomainArgs a{topo, cap, from_id, dead, unit_level, num_units, num_levels, shard_base, tail_start,
                   free_bitmap, (cap + 31) / 32};
      if (free_bitmap != nullptr) {
        list_fill_bm_kernel<<<grid_for(g.tiles * g.num_levels, kClaimWarps, 4), kClaimWarps * 32, 0, st>>>(
            a, g, o.tile_offsets, o.level_base, o.need, o.need_off, o.list);
        PXB_LAUNCHED("list_fill_bm_kernel");
      } else {
        list_fill_kernel<<<grid_for(g.tiles, kClaimWarps, 4), kClaimWarps * 32, 0, st>>>(
            a, g, o.tile_offsets, o.level_base, o.need, o.need_off, o.list);
        PXB_LAUNCHED("list_fill_kernel");
      }
    }
    place_kernel<<<grid, 256, 0, st>>>(c, w, o.ckey_out, o.cidx_out, o.level_first, t, o.rank, o.need, o.need_off,
                                       o.list, cand_weight, o.counts, overflowed_out);
    PXB_LAUNCHED("place_kernel");
  }
  finish_kernel<<<1, 32, 0, st>>>(topo, tail_start, o.counts, counts_out);
  PXB_LAUNCHED("finish_kernel");
  return PXB_OK;
}

__global__ void count_dead_kernel(int64_t cap, const uint8_t *__restrict__ dead, int32_t *__restrict__ out) {
  int c = 0;
  for (int64_t s = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; s < cap;
       s += static_cast<int64_t>(gridDim.x) * blockDim.x)
    c += dead[s] ? 1 : 0;
  c = __reduce_add_sync(0xffffffffu, c);
  if ((threadIdx.x & 31) == 0 && c) atomicAdd(out, c);
}

extern "C" int pxb_count_dead(int64_t cap, const uint8_t *dead, int32_t *out, void *stream) {
  PXB_REQUIRE(cap >= 0 && out, "pxb_count_dead: bad arguments");
  cudaStream_t st = as_stream(stream);
  PXB_CUDA(cudaMemsetAsync(out, 0, sizeof(int32_t), st));
  if (cap == 0) return PXB_OK;
  PXB_REQUIRE(dead, "pxb_count_dead: dead is NULL");
  count_dead_kernel<<<grid_for(cap, 256, 8), 256, 0, st>>>(cap, dead, out);
  PXB_LAUNCHED("count_dead_kernel");
  return PXB_OK;
}

// Per-domain free bitmaps of a bucket (bit s of domain d set iff slot s is a
// claimable free slot of domain d, as slot_domain() defines it).
__global__ void bitmap_build_kernel(DomainArgs a, uint32_t *__restrict__ bm) {
  const int64_t tail = a.topo ? 0 : *a.tail_start;
  for (int64_t s = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; s < a.cap;
       s += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int32_t d = slot_domain(a, s, tail);
    if (d >= 0) atomicOr(bm + static_cast<int64_t>(d) * a.bm_words + (s >> 5), 1u << (s & 31));
  }
}

extern "C" int pxb_free_bitmap_build(int32_t mode, int64_t cap, const int32_t *from_id, const uint8_t *dead,
                                     const int32_t *unit_level, int32_t num_units, int32_t num_levels,
                                     int64_t shard_base, const int64_t *tail_start, uint32_t *bitmap,
                                     void *stream) {
  int rc = claim_common_checks("pxb_free_bitmap_build", mode, cap, num_levels);
  if (rc) return rc;
  const int topo = mode == PXB_CLAIM_TOPOLOGICAL;
  if (topo) num_levels = 1;
  PXB_REQUIRE(bitmap != nullptr, "pxb_free_bitmap_build: bitmap is NULL");
  PXB_REQUIRE(topo || (from_id && unit_level && tail_start && num_units > 0),
              "pxb_free_bitmap_build: pipeline mode needs from_id, unit_level, num_units and tail_start");
  const int64_t words = (cap + 31) / 32;
  cudaStream_t st = as_stream(stream);
  PXB_CUDA(cudaMemsetAsync(bitmap, 0, static_cast<size_t>(words) * num_levels * 4, st));
  if (cap == 0) return PXB_OK;
  PXB_REQUIRE(dead != nullptr, "pxb_free_bitmap_build: dead is NULL");
  DomainArgs a{topo, cap, from_id, dead, unit_level, num_units, num_levels, shard_base, tail_start, bitmap, words};
  bitmap_build_kernel<<<grid_for(cap, 256, 8), 256, 0, st>>>(a, bitmap);
  PXB_LAUNCHED("bitmap_build_kernel");
  return PXB_OK;
}
