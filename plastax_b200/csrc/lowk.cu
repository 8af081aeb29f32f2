// The exact lowest-|w| prune fused into the mirror sweep: the k live edges
// of lowest |w| (ties by ascending global slot, a NaN weight never) leave
// the arena every firing, the same set pxb_lowest_keys + pxb_topk_unique +
// pxb_prune_selected would choose, without a selection over every slot.
//
// An edge's order key is (bits(|w|), global slot): bits(|w|) of a float
// without its sign is monotone in |w|. A histogram of the key's top 16 bits
// over the live non-NaN edges is kept current on the device, so the plan
// before each sweep knows the threshold bin b*: every edge in a lower bin is
// pruned by the sweep itself; the sweep lists the edges of bin b* (a few
// thousand at the benchmark's size, out of 285 M), and one CTA
// radix-selects the `take` smallest of them afterwards. The histogram is
// then cut by the plan and raised by every committed growth edge, which
// keeps it equal to the arena's (checked every firing: the counts the
// sweeps saw must equal the counts the plan expected).
//
// Under Scheme-A the lists sit in every rank's peer region and the select
// reads every rank's list after the peer barrier of the forward's combine;
// each rank tombstones its own selected edges and adds every rank's to the
// claim's per-domain counts that rode on that barrier. The lists are
// double-buffered by the plan's parity, so a rank a step ahead never
// overwrites a list a peer still reads.
#include <cub/block/block_reduce.cuh>
#include <cub/block/block_scan.cuh>

#include "mirror.cuh"

namespace pxb {

constexpr int kLowkShift = PXB_LOWK_SHIFT;
constexpr int kLowkBins = PXB_LOWK_BINS;
constexpr int kFineShift = PXB_LOWK_FINE_SHIFT;
constexpr int kFinePer = 1 << (kLowkShift - kFineShift);  // fine bins per coarse bin
constexpr uint32_t kFineBins = PXB_LOWK_FINE_BINS;
constexpr uint32_t kInfBits = 0x7f800000u;  // +inf; anything above is a NaN
constexpr uint32_t kAllBits = kInfBits + 1;   // a cut that prunes every non-NaN edge
constexpr int kPlanThreads = 256;
constexpr int kBinsPerCta = 4 * kPlanThreads;  // one uint4 of coarse bins per plan thread
constexpr int kPlanCtas = kLowkBins / kBinsPerCta;
static_assert(2 * kPlanCtas + 1 <= PXB_LOWK_PLAN_SCRATCH, "the plan's partials and arrival counter fit its scratch");
static_assert(kPlanCtas <= kPlanThreads, "one last-CTA thread per partial");
constexpr int kSelectThreads = 1024;
constexpr int kMaxWorld = 64;
constexpr int kMaxLevels = PXB_PEER_MAX_LEVELS;
static_assert(kLowkBins == (1 << (31 - kLowkShift)), "the coarse bins cover bits(|w|) >> PXB_LOWK_SHIFT");
static_assert(kFineBins == (1u << (31 - kFineShift)), "the fine bins cover bits(|w|) >> PXB_LOWK_FINE_SHIFT");
static_assert(kFinePer <= kPlanThreads, "one plan thread per fine bin of the threshold's coarse bin");

__global__ void lowk_hist_build_kernel(int64_t cap, const uint8_t *__restrict__ dead,
                                       const float *__restrict__ weight, uint32_t *__restrict__ hist,
                                       uint32_t *__restrict__ fine, pxb_lowk_plan *plan) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t span = (cap + stride - 1) / stride * stride;  // every lane of a warp runs every iteration
  uint32_t lowest = 0xffffffffu;
  for (int64_t s = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; s < span; s += stride) {
    uint32_t b = 0xffffffffu;
    if (s < cap && dead[s] == 0) {
      b = abs_bits(weight[s]);
      if (b > kInfBits) b = 0xffffffffu;
    }
    const uint32_t bin = b == 0xffffffffu ? b : b >> kLowkShift;
    // lanes of one coarse bin add once (the weights crowd a few hundred bins)
    const uint32_t same = __match_any_sync(0xffffffffu, bin);
    if (bin != 0xffffffffu && (threadIdx.x & 31) == __ffs(same) - 1) atomicAdd(hist + bin, __popc(same));
    if (b != 0xffffffffu) {
      atomicAdd(fine + (b >> kFineShift), 1u);
      lowest = min(lowest, b >> kFineShift);
    }
  }
  lowest = __reduce_min_sync(0xffffffffu, lowest);
  if ((threadIdx.x & 31) == 0 && lowest != 0xffffffffu) atomicMin(&plan->floor, lowest);
}

// The plan: the fine threshold bin of the k-th smallest key, the coarse
// histogram's cut and the fine bin's part; the fine bins wholly pruned are
// emptied by lowk_zero_kernel from the plan's [zero_lo, zero_hi). This
// rank's list counters of the new parity are reset.
//
// kPlanCtas CTAs each sum 1024 coarse bins (one 16-byte load per thread)
// into a partial; the last CTA to arrive scans the partials, then the 1024
// bins of the range holding the k-th key, then that coarse bin's fine bins.
// One CTA reading the whole 256 KB histogram is bound by the loads a single
// SM keeps in flight; here each CTA reads 4 KB and the last one 9 KB more.
__global__ void __launch_bounds__(kPlanThreads) lowk_plan_kernel(uint32_t *__restrict__ hist,
                                                                 uint32_t *__restrict__ fine, pxb_lowk_plan *plan,
                                                                 int64_t k, unsigned long long *count,
                                                                 uint32_t *scratch) {
  using Scan = cub::BlockScan<long long, kPlanThreads>;
  using Reduce = cub::BlockReduce<long long, kPlanThreads>;
  __shared__ union {
    typename Scan::TempStorage scan;
    typename Reduce::TempStorage reduce;
  } tmp;
  __shared__ int s_last, s_range, s_bin, s_fbin;
  __shared__ long long s_range_excl, s_below_c, s_below, s_in_bin;
  unsigned long long *part = reinterpret_cast<unsigned long long *>(scratch);
  unsigned int *arrived = scratch + 2 * kPlanCtas;
  const int t = threadIdx.x;
  {
    const uint4 v = reinterpret_cast<const uint4 *>(hist)[blockIdx.x * kPlanThreads + t];
    const long long mine = static_cast<long long>(v.x) + v.y + v.z + v.w;
    const long long sum = Reduce(tmp.reduce).Sum(mine);
    if (t == 0) {
      part[blockIdx.x] = static_cast<unsigned long long>(sum);
      __threadfence();
      s_last = atomicAdd(arrived, 1u) == kPlanCtas - 1;
    }
    __syncthreads();
    if (!s_last) return;
  }
  // the last CTA: every partial is visible (fence before each arrival)
  __threadfence();
  if (t == 0) {
    *arrived = 0u;  // ready for the next plan
    s_range = -1;
    s_bin = -1;
    s_fbin = -1;
  }
  const long long p = t < kPlanCtas ? static_cast<long long>(__ldcg(part + t)) : 0;
  long long excl, total;
  __syncthreads();
  Scan(tmp.scan).ExclusiveSum(p, excl, total);
  if (k > 0 && total > k && t < kPlanCtas && excl < k && excl + p >= k) {
    s_range = t;
    s_range_excl = excl;
  }
  __syncthreads();
  const int rg = s_range;
  if (rg >= 0) {
    // the range's 1024 coarse bins, four per thread
    const uint4 v = __ldcg(reinterpret_cast<const uint4 *>(hist) + rg * kPlanThreads + t);
    const long long mine = static_cast<long long>(v.x) + v.y + v.z + v.w;
    long long bex, btot;
    Scan(tmp.scan).ExclusiveSum(mine, bex, btot);
    const long long before = s_range_excl + bex;
    if (before < k && before + mine >= k) {
      const uint32_t h[4] = {v.x, v.y, v.z, v.w};
      long long run = before;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (run < k && run + h[j] >= k) {
          s_bin = rg * kBinsPerCta + 4 * t + j;
          s_below_c = run;
        }
        run += h[j];
      }
    }
    __syncthreads();
  }
  const int b = s_bin;
  if (b >= 0) {
    // the coarse bin's fine bins, one per thread
    const uint32_t f = t < kFinePer ? __ldcg(fine + static_cast<int64_t>(b) * kFinePer + t) : 0u;
    long long fexcl, ftotal;
    __syncthreads();  // the scan's storage is reused
    Scan(tmp.scan).ExclusiveSum(static_cast<long long>(f), fexcl, ftotal);
    const long long want = k - s_below_c;  // the rank inside the coarse bin, 1-based
    if (t < kFinePer && fexcl < want && fexcl + f >= want) {
      s_fbin = b * kFinePer + t;
      s_below = s_below_c + fexcl;
      s_in_bin = f;
    }
    __syncthreads();
  }
  const int fb = s_fbin;
  const uint32_t old_floor = plan->floor;
  // the fine bins of the coarse bin must hold its count; if they do not,
  // the histograms are stale: prune nothing and report it
  const bool stale = b >= 0 && fb < 0;
  if (stale) k = 0;
  long long take = 0;
  bool whole = false;
  uint32_t cut;  // fine bins below `cut` are emptied
  if (k <= 0) {
    cut = 0u;
  } else if (fb < 0) {
    cut = kFineBins;  // k >= every counted edge: all of them go
  } else {
    take = k - s_below;
    whole = take == s_in_bin;
    cut = whole ? static_cast<uint32_t>(fb) + 1u : static_cast<uint32_t>(fb);
    if (whole) take = 0;
  }
  __syncthreads();  // every thread has read plan->floor
  if (t == 0) {
    pxb_lowk_plan pl = *plan;
    pl.parity ^= 1;
    if (k <= 0) {
      pl.lo_bits = pl.hi_bits = 0u;
      pl.below_expect = 0;
    } else if (fb < 0) {
      pl.lo_bits = pl.hi_bits = kAllBits;
      pl.below_expect = total;
    } else {
      const uint32_t end = static_cast<uint32_t>(fb + 1) << kFineShift;
      const uint32_t hi = end < kAllBits ? end : kAllBits;
      pl.lo_bits = whole ? hi : static_cast<uint32_t>(fb) << kFineShift;
      pl.hi_bits = hi;
      pl.below_expect = whole ? k : s_below;
    }
    pl.take = take;
    pl.listed_expect = take > 0 ? s_in_bin : 0;
    pl.pruned = 0;
    if (stale) pl.status |= 2;
    pl.zero_lo = old_floor < cut ? old_floor : cut;
    pl.zero_hi = cut;
    if (k > 0) pl.floor = cut > old_floor ? cut : old_floor;
    *plan = pl;
    count[2 * pl.parity] = 0ull;
    count[2 * pl.parity + 1] = 0ull;
    if (fb >= 0 && !whole) fine[fb] -= static_cast<uint32_t>(take);
  }
  // the coarse cut: bins wholly below the threshold's emptied (those from
  // the floor's up: none below it holds an edge), its own bin loses what
  // its fine bins lose
  if (k > 0) {
    const int cb = fb < 0 ? kLowkBins : b;
    const int cfloor = static_cast<int>(min(old_floor >> (kLowkShift - kFineShift), static_cast<uint32_t>(kLowkBins)));
    for (int bin = cfloor + t; bin < cb; bin += kPlanThreads) hist[bin] = 0u;
    const long long removed_in_b = fb < 0 ? 0 : (s_below - s_below_c) + (whole ? s_in_bin : take);
    if (t == 0 && cb < kLowkBins && removed_in_b > 0) hist[cb] -= static_cast<uint32_t>(removed_in_b);
  }
}

// The fine bins the plan prunes wholly: [zero_lo, zero_hi) (between the
// lowest bin that may hold an edge and the threshold bin).
__global__ void lowk_zero_kernel(uint32_t *__restrict__ fine, const pxb_lowk_plan *plan) {
  const uint32_t lo = plan->zero_lo, hi = plan->zero_hi;
  for (int64_t i = lo + blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < hi;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    fine[i] = 0u;
}

struct SelectArgs {
  pxb_lowk_plan *plan;
  int32_t rank, world;
  int64_t cap, slot_base;
  const uint64_t *my_key;
  const int32_t *my_level;
  const int64_t *my_pos;
  const unsigned long long *my_count;
  uint64_t *const *peer_key;
  int32_t *const *peer_level;
  unsigned long long *const *peer_count;
  uint8_t *dead;
  uint32_t *bm;
  int64_t bm_words;
  const int32_t *bm_level;
  int32_t num_levels;
  int32_t *level_before, *level_totals;
};

__device__ __forceinline__ const uint64_t *keys_of(const SelectArgs &a, int q) {
  return a.world == 1 ? a.my_key : a.peer_key[q];
}

// The select's keys and claim domains staged in shared memory when every
// rank's list fits.
constexpr int kStageKeys = 12288;  // 96 KB of keys + 48 KB of domains
constexpr int kDigitBits = 10;
constexpr int kDigits = 1 << kDigitBits;
static_assert(kDigits == kSelectThreads, "one select thread per digit value");

// One CTA: every rank's listed keys of this firing, the take-th smallest by
// an MSD radix select, this rank's listed edges up to it tombstoned. The
// listed keys share their fine bin, i.e. key bits 63..39 (bits(|w|) >> 7
// above the 32-bit slot), so four 10-bit digits over bits 38..0 decide; the
// keys are read from shared memory when every rank's list fits there.
__global__ void __launch_bounds__(kSelectThreads) lowk_select_kernel(SelectArgs a, MirrorK m) {
  using Scan = cub::BlockScan<int, kSelectThreads>;
  __shared__ typename Scan::TempStorage scan_tmp;
  __shared__ unsigned int digit_hist[kDigits];
  __shared__ int64_t s_n[kMaxWorld], s_off[kMaxWorld + 1];
  __shared__ unsigned long long s_prefix;
  __shared__ int s_want;
  __shared__ int s_sel[kMaxWorld * kMaxLevels];
  __shared__ int s_pruned;
  __shared__ long long s_below[kMaxWorld];
  extern __shared__ unsigned long long s_keys[];
  int32_t *s_levels = reinterpret_cast<int32_t *>(s_keys + kStageKeys);
  const int t = threadIdx.x;
  const int parity = a.plan->parity;
  const long long take = a.plan->take;
  const int64_t base = static_cast<int64_t>(parity) * a.cap;
  // every rank's counters read at once (one thread per rank: remote loads
  // one after another would each take a full NVLink round trip)
  if (t < a.world) {
    const unsigned long long *cnt = a.world == 1 ? a.my_count : a.peer_count[t];
    s_n[t] = static_cast<int64_t>(cnt[2 * parity]);
    s_below[t] = static_cast<long long>(cnt[2 * parity + 1]);
  }
  __syncthreads();
  if (t == 0) {
    long long listed = 0, below = 0;
    int status = 0;
    s_off[0] = 0;
    for (int q = 0; q < a.world; ++q) {
      if (s_n[q] > a.cap) {
        status |= 1;
        s_n[q] = a.cap;
      }
      s_off[q + 1] = s_off[q] + s_n[q];
      listed += s_n[q];
      below += s_below[q];
    }
    if (listed != a.plan->listed_expect || below != a.plan->below_expect) status |= 2;
    if (status) atomicOr(&a.plan->status, status);
    s_pruned = 0;
  }
  for (int i = t; i < kMaxWorld * kMaxLevels; i += kSelectThreads) s_sel[i] = 0;
  __syncthreads();
  const int64_t listed_total = s_off[a.world];
  if (take <= 0) {
    if (t == 0) a.plan->pruned = static_cast<int64_t>(a.my_count[2 * parity + 1]);
    return;
  }
  const bool staged = listed_total <= kStageKeys;
  if (staged) {
    // one flattened pass over every rank's list: each thread's loads are
    // independent of one another, so they are in flight together
    const int32_t *levels0 = a.world == 1 ? a.my_level : nullptr;
    for (int64_t j = t; j < listed_total; j += kSelectThreads) {
      int q = 0;
      while (j >= s_off[q + 1]) ++q;
      const int64_t i = j - s_off[q];
      s_keys[j] = keys_of(a, q)[base + i];
      s_levels[j] = (levels0 != nullptr ? levels0 : a.peer_level[q])[base + i];
    }
    __syncthreads();
  }
  unsigned long long kstar = ~0ull;  // take >= every listed key: all of them
  if (take < listed_total) {
    // every listed key lies in the plan's fine bin: its bits 63..39
    unsigned long long prefix = static_cast<unsigned long long>(a.plan->lo_bits >> kFineShift) << 39;
    unsigned long long mask = ~0ull << 39;
    int want = static_cast<int>(take);
    for (int shift = 39 - kDigitBits; shift > -kDigitBits; shift -= kDigitBits) {
      const int sh = shift > 0 ? shift : 0;
      const int width = shift > 0 ? kDigitBits : kDigitBits + shift;
      const unsigned long long dmask = (1ull << width) - 1ull;
      digit_hist[t] = 0u;
      __syncthreads();
      for (int q = 0; q < a.world; ++q) {
        const uint64_t *keys = keys_of(a, q) + base;
        for (int64_t i = t; i < s_n[q]; i += kSelectThreads) {
          const unsigned long long key = staged ? s_keys[s_off[q] + i] : keys[i];
          if ((key & mask) == prefix) atomicAdd(&digit_hist[(key >> sh) & dmask], 1u);
        }
      }
      __syncthreads();
      const int h = static_cast<int>(digit_hist[t]);
      int excl;
      Scan(scan_tmp).ExclusiveSum(h, excl);
      if (excl < want && excl + h >= want) {
        s_prefix = prefix | (static_cast<unsigned long long>(t) << sh);
        s_want = want - excl;
      }
      __syncthreads();
      prefix = s_prefix;
      want = s_want;
      mask |= dmask << sh;
    }
    kstar = prefix;  // the keys are unique: exactly `take` of them are <= kstar
  }
  // this rank's selected edges leave the arena and the mirror
  int mine = 0;
  const uint64_t *my_keys = a.my_key + base;
  for (int64_t i = t; i < s_n[a.rank]; i += kSelectThreads) {
    const unsigned long long key = staged ? s_keys[s_off[a.rank] + i] : my_keys[i];
    if (key > kstar) continue;
    const int32_t slot = static_cast<int32_t>(static_cast<uint32_t>(key) - static_cast<uint32_t>(a.slot_base));
    const int64_t pos = a.my_pos[base + i];
    int32_t src;
    if (pos >= 0) {
      src = static_cast<int32_t>(m.word[pos] >> m.cb);
      const int64_t g = group_of(m, pos);
      empty_entry(m, pos, g, m.gbase[g]);
    } else {
      const int64_t o = -1 - pos;
      src = m.ovf_src[o];
      m.ovf_src[o] = -1;
    }
    a.dead[slot] = 1;
    if (a.bm != nullptr) {
      const int64_t row = a.bm_level ? a.bm_level[src] : 0;
      atomicOr(a.bm + row * a.bm_words + (slot >> 5), 1u << (slot & 31));
    }
    ++mine;
  }
  // every rank's selected edges per claim domain, for the Scheme-A counts
  if (a.level_totals != nullptr) {
    for (int q = 0; q < a.world; ++q) {
      const uint64_t *keys = keys_of(a, q) + base;
      const int32_t *lv = a.world == 1 ? a.my_level : a.peer_level[q];
      for (int64_t i = t; i < s_n[q]; i += kSelectThreads) {
        const unsigned long long key = staged ? s_keys[s_off[q] + i] : keys[i];
        if (key > kstar) continue;
        const int l = staged ? s_levels[s_off[q] + i] : lv[base + i];
        if (l >= 0 && l < a.num_levels) atomicAdd(&s_sel[q * kMaxLevels + l], 1);
      }
    }
  }
  mine = __reduce_add_sync(0xffffffffu, mine);
  if ((t & 31) == 0 && mine) atomicAdd(&s_pruned, mine);
  __syncthreads();
  if (a.level_totals != nullptr && t < a.num_levels) {
    int before = 0, total = 0;
    for (int q = 0; q < a.world; ++q) {
      const int v = s_sel[q * kMaxLevels + t];
      if (q < a.rank) before += v;
      total += v;
    }
    a.level_totals[t] += total;
    if (a.level_before != nullptr) a.level_before[t] += before;
  }
  if (t == 0) a.plan->pruned = static_cast<int64_t>(a.my_count[2 * parity + 1]) + s_pruned;
}

// The committed growth edges into both histograms. Their weights crowd a
// few hundred coarse bins, so each CTA counts its edges' coarse bins in
// shared memory (16-bit halves of 32-bit words) and adds each touched bin
// once; the fine bins are spread thin and take their atomics directly.
constexpr int kAddThreads = 1024;
constexpr int kAddPer = 4;  // edges per thread: a CTA's count per bin stays below 2^16
__global__ void __launch_bounds__(kAddThreads) lowk_hist_add_kernel(uint32_t *__restrict__ hist,
                                                                   uint32_t *__restrict__ fine, int64_t k,
                                                                   const float *__restrict__ weight,
                                                                   const uint8_t *__restrict__ committed,
                                                                   pxb_lowk_plan *plan, const int32_t *claim_counts,
                                                                   long long *totals) {
  extern __shared__ uint32_t s_half[];  // kLowkBins / 2 words
  __shared__ uint32_t s_lowest;
  if (totals != nullptr && blockIdx.x == 0 && threadIdx.x == 0) {
    atomicAdd(reinterpret_cast<unsigned long long *>(totals + 0), static_cast<unsigned long long>(plan->pruned));
    if (claim_counts != nullptr) {
      atomicAdd(reinterpret_cast<unsigned long long *>(totals + 1), static_cast<unsigned long long>(claim_counts[0]));
      atomicAdd(reinterpret_cast<unsigned long long *>(totals + 2), static_cast<unsigned long long>(claim_counts[1]));
    }
    atomicAdd(reinterpret_cast<unsigned long long *>(totals + 3), 1ull);
  }
  for (int i = threadIdx.x; i < kLowkBins / 2; i += kAddThreads) s_half[i] = 0u;
  if (threadIdx.x == 0) s_lowest = 0xffffffffu;
  __syncthreads();
  uint32_t lowest = 0xffffffffu;
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kAddThreads * kAddPer;
#pragma unroll
  for (int j = 0; j < kAddPer; ++j) {
    const int64_t i = base + j * kAddThreads + threadIdx.x;
    if (i >= k || !committed[i]) continue;
    const uint32_t b = abs_bits(weight[i]);
    if (b > kInfBits) continue;
    const uint32_t cbin = b >> kLowkShift;
    atomicAdd(&s_half[cbin >> 1], (cbin & 1u) ? 0x10000u : 1u);
    atomicAdd(fine + (b >> kFineShift), 1u);
    lowest = min(lowest, b >> kFineShift);
  }
  // the floor: one atomic per CTA (one address takes them all)
  lowest = __reduce_min_sync(0xffffffffu, lowest);
  if ((threadIdx.x & 31) == 0 && lowest != 0xffffffffu) atomicMin(&s_lowest, lowest);
  __syncthreads();
  if (threadIdx.x == 0 && s_lowest != 0xffffffffu) atomicMin(&plan->floor, s_lowest);
  for (int i = threadIdx.x; i < kLowkBins / 2; i += kAddThreads) {
    const uint32_t v = s_half[i];
    if (v & 0xffffu) atomicAdd(hist + 2 * i, v & 0xffffu);
    if (v >> 16) atomicAdd(hist + 2 * i + 1, v >> 16);
  }
}

static int check_lowk(const char *fn, const pxb_lowk *lk) {
  PXB_REQUIRE(lk != nullptr, "%s: lowk is NULL", fn);
  PXB_REQUIRE(lk->hist && lk->fine && lk->plan && lk->key && lk->level && lk->count && lk->pos && lk->plan_scratch,
              "%s: a lowk array is NULL", fn);
  PXB_REQUIRE(lk->world >= 1 && lk->world <= kMaxWorld && lk->rank >= 0 && lk->rank < lk->world,
              "%s: rank %d / world %d out of range (world <= %d)", fn, lk->rank, lk->world, kMaxWorld);
  PXB_REQUIRE(lk->world == 1 || (lk->peer_key && lk->peer_level && lk->peer_count),
              "%s: the peer lists are NULL", fn);
  PXB_REQUIRE(lk->list_cap > 0, "%s: list_cap must be > 0", fn);
  PXB_REQUIRE(lk->k >= 0, "%s: negative k", fn);
  return PXB_OK;
}

}  // namespace pxb

using namespace pxb;

extern "C" int pxb_lowk_hist_build(const pxb_lowk *lowk, int64_t cap, const uint8_t *dead, const float *weight,
                                   void *stream) {
  int rc = check_lowk("pxb_lowk_hist_build", lowk);
  if (rc) return rc;
  PXB_REQUIRE(cap >= 0, "pxb_lowk_hist_build: negative cap");
  if (cap == 0) return PXB_OK;
  PXB_REQUIRE(dead && weight, "pxb_lowk_hist_build: dead/weight is NULL");
  lowk_hist_build_kernel<<<grid_for(cap, 256, 8), 256, 0, as_stream(stream)>>>(cap, dead, weight, lowk->hist,
                                                                               lowk->fine, lowk->plan);
  PXB_LAUNCHED("lowk_hist_build_kernel");
  return PXB_OK;
}

extern "C" int pxb_lowk_make_plan(const pxb_lowk *lowk, void *stream) {
  int rc = check_lowk("pxb_lowk_make_plan", lowk);
  if (rc) return rc;
  cudaStream_t st = as_stream(stream);
  lowk_plan_kernel<<<kPlanCtas, kPlanThreads, 0, st>>>(lowk->hist, lowk->fine, lowk->plan, lowk->k, lowk->count,
                                                        lowk->plan_scratch);
  PXB_LAUNCHED("lowk_plan_kernel");
  lowk_zero_kernel<<<grid_for(int64_t(1) << 20, 256, 4), 256, 0, st>>>(lowk->fine, lowk->plan);
  PXB_LAUNCHED("lowk_zero_kernel");
  return PXB_OK;
}

extern "C" int pxb_lowk_select(const pxb_lowk *lowk, const pxb_mirror *mirror, uint8_t *dead, uint32_t *free_bitmap,
                               int64_t bitmap_words, const int32_t *bitmap_level, int32_t num_levels,
                               int32_t *level_before, int32_t *level_totals, void *stream) {
  int rc = check_lowk("pxb_lowk_select", lowk);
  if (rc) return rc;
  rc = check_mirror("pxb_lowk_select", mirror);
  if (rc) return rc;
  PXB_REQUIRE(dead != nullptr, "pxb_lowk_select: dead is NULL");
  PXB_REQUIRE(level_totals == nullptr || (num_levels >= 1 && num_levels <= kMaxLevels),
              "pxb_lowk_select: 1..%d claim domains when level_totals is given", kMaxLevels);
  SelectArgs a;
  a.plan = lowk->plan;
  a.rank = lowk->rank;
  a.world = lowk->world;
  a.cap = lowk->list_cap;
  a.slot_base = lowk->slot_base;
  a.my_key = lowk->key;
  a.my_level = lowk->level;
  a.my_pos = lowk->pos;
  a.my_count = lowk->count;
  a.peer_key = lowk->peer_key;
  a.peer_level = lowk->peer_level;
  a.peer_count = lowk->peer_count;
  a.dead = dead;
  a.bm = free_bitmap;
  a.bm_words = bitmap_words;
  a.bm_level = bitmap_level;
  a.num_levels = num_levels;
  a.level_before = level_before;
  a.level_totals = level_totals;
  const size_t smem = kStageKeys * (sizeof(unsigned long long) + sizeof(int32_t));
  PXB_CUDA(cudaFuncSetAttribute(lowk_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
  lowk_select_kernel<<<1, kSelectThreads, smem, as_stream(stream)>>>(a, to_k(mirror));
  PXB_LAUNCHED("lowk_select_kernel");
  return PXB_OK;
}

extern "C" int pxb_lowk_hist_add(const pxb_lowk *lowk, int64_t k, const float *weight, const uint8_t *committed,
                                 const int32_t *claim_counts, int64_t *totals, void *stream) {
  int rc = check_lowk("pxb_lowk_hist_add", lowk);
  if (rc) return rc;
  PXB_REQUIRE(k >= 0, "pxb_lowk_hist_add: negative k");
  PXB_REQUIRE(k == 0 || (weight && committed), "pxb_lowk_hist_add: weight/committed is NULL");
  const size_t smem = kLowkBins / 2 * sizeof(uint32_t);
  PXB_CUDA(cudaFuncSetAttribute(lowk_hist_add_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
  const int64_t per_cta = int64_t(kAddThreads) * kAddPer;
  const int grid = static_cast<int>(k > 0 ? (k + per_cta - 1) / per_cta : 1);
  lowk_hist_add_kernel<<<grid, kAddThreads, smem, as_stream(stream)>>>(
      lowk->hist, lowk->fine, k, weight, committed, lowk->plan, claim_counts, reinterpret_cast<long long *>(totals));
  PXB_LAUNCHED("lowk_hist_add_kernel");
  return PXB_OK;
}
