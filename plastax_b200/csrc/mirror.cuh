// Device view of the destination-grouped mirror and the prune records its
// sweep writes; shared by the sweep (mirror.cu) and the exact lowest-|w|
// prune's selection (lowk.cu).
#pragma once

#include "pxb_common.cuh"

namespace pxb {

constexpr uint32_t kEmpty = 0xffffffffu;

struct MirrorK {
  int64_t entries;
  int32_t n;
  int cb;  // chunk bits
  int64_t groups;
  const int64_t *gbase;
  int32_t *gfill;
  uint32_t *word;
  float *w;
  int32_t *slot;
  int32_t *hstack, *hcount;
  int64_t items;
  const int64_t *ib, *ie;
  const int32_t *ig;
  int64_t ovf_cap;
  int32_t *ovf_count, *ovf_src, *ovf_dst, *ovf_slot;
  float *ovf_w;
  int32_t *status;
  int64_t *defer_pos;  // the sweep's deferred prunes (NULL: in place)
  int32_t *defer_count;
  int64_t defer_total;
  int32_t defer_ctas;
  int32_t sum_frac;  // fractional bits of the sweep's shared sum words: 28 or 31
};

inline MirrorK to_k(const pxb_mirror *m) {
  MirrorK k;
  k.entries = m->entries;
  k.n = m->num_units;
  k.cb = m->chunk_bits;
  k.groups = m->groups;
  k.gbase = m->gbase;
  k.gfill = m->gfill;
  k.word = m->word;
  k.w = m->weight;
  k.slot = m->slot;
  k.hstack = m->hstack;
  k.hcount = m->hcount;
  k.items = m->items;
  k.ib = m->item_begin;
  k.ie = m->item_end;
  k.ig = m->item_group;
  k.ovf_cap = m->ovf_cap;
  k.ovf_count = m->ovf_count;
  k.ovf_src = m->ovf_src;
  k.ovf_dst = m->ovf_dst;
  k.ovf_slot = m->ovf_slot;
  k.ovf_w = m->ovf_weight;
  k.status = m->status;
  const bool defer = m->defer_pos != nullptr && m->defer_count != nullptr && m->defer_seg > 0 && m->defer_ctas > 0;
  k.defer_pos = defer ? m->defer_pos : nullptr;
  k.defer_count = defer ? m->defer_count : nullptr;
  k.defer_total = defer ? m->defer_seg * m->defer_ctas : 0;
  k.defer_ctas = defer ? m->defer_ctas : 0;
  k.sum_frac = m->sum_frac_bits == 28 ? 28 : 31;
  return k;
}

// The group holding mirror position pos: the last g with gbase[g] <= pos.
__device__ __forceinline__ int64_t group_of(const MirrorK &m, int64_t pos) {
  int64_t lo = 0, hi = m.groups - 1;
  while (lo < hi) {
    const int64_t mid = (lo + hi + 1) / 2;
    if (m.gbase[mid] <= pos) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

int check_mirror(const char *fn, const pxb_mirror *m);

// The lowest-|w| prune's lists as the sweep writes them (this rank's).
struct LowkSweep {
  const pxb_lowk_plan *plan;
  uint64_t *key;
  int32_t *level;
  unsigned long long *count;
  int64_t *pos;
  int64_t cap, slot_base;
};

struct MPrune {
  int kind;
  float thr;
  const float *unit_thr;
  uint8_t *dead;
  uint32_t *bm;
  int64_t bm_words;
  const int32_t *bm_level;
  int32_t *pruned;
  LowkSweep lk;
};

// The plan's cut as one sweep reads it. hi_le is the float whose bits are
// hi - 1: for a non-NaN w, bits(|w|) < hi exactly when |w| <= hi_le (the
// bit order of non-negative floats is their value order; hi - 1 = +inf's
// bits takes every non-NaN, and hi = 0 gives a NaN that takes none), so the
// fast test is one float min over the entries with the free |.| modifier.
struct LowkCut {
  uint32_t lo, hi;
  float hi_le;
  int parity;
};

__device__ __forceinline__ LowkCut lowk_cut(const MPrune &p) {
  LowkCut c{0u, 0u, 0.0f, 0};
  if (p.kind == PXB_PRUNE_LOWEST_K) {
    c.lo = p.lk.plan->lo_bits;
    c.hi = p.lk.plan->hi_bits;
    c.hi_le = __uint_as_float(c.hi - 1u);
    c.parity = p.lk.plan->parity;
  }
  return c;
}

// bits(|w|): the non-negative float's bit pattern, monotone in |w| (a NaN
// lies above +inf).
__device__ __forceinline__ uint32_t abs_bits(float w) { return __float_as_uint(w) & 0x7fffffffu; }

__device__ __forceinline__ bool mprune_pred(const MPrune &p, float w, int32_t dst) {
  if (p.kind == PXB_PRUNE_ABS_BELOW) return fabsf(w) < p.thr;
  if (p.kind == PXB_PRUNE_ABS_BELOW_DST) return fabsf(w) < __ldg(p.unit_thr + dst);
  return false;
}

// The canonical record of a tombstone: dead byte, free bitmap bit, counter.
__device__ __forceinline__ void tombstone(const MPrune &p, int32_t slot, int32_t src) {
  p.dead[slot] = 1;
  if (p.bm != nullptr) {
    const int64_t row = p.bm_level ? p.bm_level[src] : 0;
    atomicOr(p.bm + row * p.bm_words + (slot >> 5), 1u << (slot & 31));
  }
  if (p.pruned) atomicAdd(p.pruned, 1);
}

// Empty mirror entry `pos` of group g (base gb) and push it on the group's
// hole stack.
__device__ __forceinline__ void empty_entry(const MirrorK &m, int64_t pos, int64_t g, int64_t gb) {
  m.word[pos] = kEmpty;
  m.w[pos] = 0.0f;
  const int32_t h = atomicAdd(m.hcount + g, 1);
  m.hstack[gb + h] = static_cast<int32_t>(pos - gb);
}

// List an edge of the plan's threshold bin (this rank's list of the plan's
// parity): its key, claim domain and mirror position. An index past the
// list's capacity is dropped here and reported by the selection.
__device__ __forceinline__ void lowk_list(const MPrune &p, int parity, uint32_t bits, int32_t slot, int32_t src,
                                          int64_t pos) {
  const unsigned long long i = atomicAdd(p.lk.count + 2 * parity, 1ull);
  if (i < static_cast<unsigned long long>(p.lk.cap)) {
    const int64_t j = parity * p.lk.cap + static_cast<int64_t>(i);
    p.lk.key[j] = (static_cast<uint64_t>(bits) << 32) | static_cast<uint32_t>(p.lk.slot_base + slot);
    p.lk.level[j] = p.bm_level ? p.bm_level[src] : 0;
    p.lk.pos[j] = pos;
  }
}

}  // namespace pxb
