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
};

static MirrorK to_k(const pxb_mirror *m) {
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
  return k;
}

struct MPrune {
  int kind;
  float thr;
  const float *unit_thr;
  uint8_t *dead;
  uint32_t *bm;
  int64_t bm_words;
  const int32_t *bm_level;
  int32_t *pruned;
};

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

template <int MONOID>
__device__ __forceinline__ void smem_combine(float *a, float v) {
  if (MONOID == PXB_MONOID_SUM) atomicAdd(a, v);
  else if (MONOID == PXB_MONOID_MAX) atomic_max_f32(a, v);
  else atomic_min_f32(a, v);
}

// One entry of the sweep: gather, shared-memory combine, fused prune.
template <int MONOID, bool PRUNE>
__device__ __forceinline__ void sweep_entry(const MirrorK &m, const MPrune &p, float *acc_s, int32_t g, int64_t gb,
                                            uint32_t mask, uint32_t word, float w, float a, int64_t pos) {
  if (word == kEmpty) return;
  const uint32_t src = word >> m.cb;
  if (src >= static_cast<uint32_t>(m.n)) return;
  const uint32_t dl = word & mask;
  smem_combine<MONOID>(acc_s + dl, __fmul_rn(w, a));
  if (PRUNE) {
    const int32_t dst = (g << m.cb) | static_cast<int32_t>(dl);
    if (dst < m.n && mprune_pred(p, w, dst)) {
      m.word[pos] = kEmpty;
      tombstone(p, m.slot[pos], static_cast<int32_t>(src));
      const int32_t h = atomicAdd(m.hcount + g, 1);
      m.hstack[gb + h] = static_cast<int32_t>(pos - gb);
    }
  }
}

// Each CTA sweeps an equal contiguous range of the entry array (balanced by
// construction), accumulating into shared memory and flushing the chunk's
// accumulators whenever its range crosses into the next group. Two quads
// (8 entries, 2 x 32 B of loads) per thread per iteration keep enough bytes
// in flight to cover the HBM latency.
template <int MONOID, bool PRUNE>
__global__ void __launch_bounds__(256) mirror_forward_kernel(MirrorK m, const float *__restrict__ act,
                                                             float *__restrict__ acc, MPrune p) {
  extern __shared__ float acc_s[];
  const int chunk = 1 << m.cb;
  const uint32_t mask = static_cast<uint32_t>(chunk - 1);
  const float ident = monoid_identity(MONOID);
  const int64_t quads = m.entries / 4;
  const int64_t per = (quads + gridDim.x - 1) / gridDim.x;
  const int64_t q_lo = blockIdx.x * per;
  const int64_t q_hi = q_lo + per < quads ? q_lo + per : quads;
  if (q_lo >= q_hi) return;
  // first group whose region holds quad q_lo: the last g with gbase[g] <= 4*q_lo
  int64_t lo = 0, hi = m.groups - 1;
  while (lo < hi) {
    const int64_t mid = (lo + hi + 1) / 2;
    if (m.gbase[mid] <= q_lo * 4) lo = mid; else hi = mid - 1;
  }
  const uint4 *w4 = reinterpret_cast<const uint4 *>(m.word);
  const float4 *f4 = reinterpret_cast<const float4 *>(m.w);
  for (int64_t g = lo; g < m.groups && m.gbase[g] < q_hi * 4; ++g) {
    const int64_t gb = m.gbase[g], gcap = m.gbase[g + 1] - gb;
    int64_t fill = m.gfill[g];
    fill = fill < gcap ? fill : gcap;
    const int64_t a_q = gb / 4 > q_lo ? gb / 4 : q_lo;
    const int64_t e_used = (gb + fill + 3) / 4;
    const int64_t b_q = e_used < q_hi ? e_used : q_hi;
    if (a_q >= b_q) continue;
    for (int u = threadIdx.x; u < chunk; u += blockDim.x) acc_s[u] = ident;
    __syncthreads();
    const int gi = static_cast<int>(g);
    int64_t q = a_q + threadIdx.x;
    for (; q + blockDim.x < b_q; q += 2 * blockDim.x) {
      const int64_t q2 = q + blockDim.x;
      const uint4 wa = __ldcs(w4 + q), wb = __ldcs(w4 + q2);
      const float4 fa = __ldcs(f4 + q), fb = __ldcs(f4 + q2);
      const uint32_t ws[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
      const float fs[8] = {fa.x, fa.y, fa.z, fa.w, fb.x, fb.y, fb.z, fb.w};
      float av[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint32_t src = ws[i] >> m.cb;
        av[i] = (ws[i] != kEmpty && src < static_cast<uint32_t>(m.n)) ? __ldg(act + src) : 0.0f;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i)
        sweep_entry<MONOID, PRUNE>(m, p, acc_s, gi, gb, mask, ws[i], fs[i], av[i], (i < 4 ? q : q2) * 4 + (i & 3));
    }
    if (q < b_q) {
      const uint4 wa = __ldcs(w4 + q);
      const float4 fa = __ldcs(f4 + q);
      const uint32_t ws[4] = {wa.x, wa.y, wa.z, wa.w};
      const float fs[4] = {fa.x, fa.y, fa.z, fa.w};
      float av[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t src = ws[i] >> m.cb;
        av[i] = (ws[i] != kEmpty && src < static_cast<uint32_t>(m.n)) ? __ldg(act + src) : 0.0f;
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) sweep_entry<MONOID, PRUNE>(m, p, acc_s, gi, gb, mask, ws[i], fs[i], av[i], q * 4 + i);
    }
    __syncthreads();
    const int32_t base = gi << m.cb;
    if (MONOID == PXB_MONOID_SUM && base + chunk <= m.n) {
      float4 *acc4 = reinterpret_cast<float4 *>(acc + base);
      const float4 *s4 = reinterpret_cast<const float4 *>(acc_s);
      for (int u = threadIdx.x; u < chunk / 4; u += blockDim.x) {
        const float4 v = s4[u];
        if (v.x != 0.0f || v.y != 0.0f || v.z != 0.0f || v.w != 0.0f) atomicAdd(acc4 + u, v);
      }
    } else {
      for (int u = threadIdx.x; u < chunk; u += blockDim.x) {
        const float v = acc_s[u];
        if (v != ident && base + u < m.n) atomic_combine<MONOID>(acc + base + u, v);
      }
    }
    __syncthreads();
  }
}

// Edges the mirror had no room for: swept with global atomics.
template <int MONOID, bool PRUNE>
__global__ void mirror_overflow_kernel(MirrorK m, const float *__restrict__ act, float *__restrict__ acc, MPrune p) {
  const int64_t cnt = *m.ovf_count < m.ovf_cap ? *m.ovf_count : m.ovf_cap;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < cnt;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int32_t s = m.ovf_src[i], d = m.ovf_dst[i];
    if (s < 0 || s >= m.n || d < 0 || d >= m.n) continue;
    const float w = m.ovf_w[i];
    atomic_combine<MONOID>(acc + d, __fmul_rn(w, act[s]));
    if (PRUNE && mprune_pred(p, w, d)) {
      m.ovf_src[i] = -1;
      tombstone(p, m.ovf_slot[i], s);
    }
  }
}

// Insert, phase 1: each placed edge takes rank r in its destination group
// (one atomicAdd on the group's insert counter); the r-th insert of a group
// takes the group's r-th hole from the top of its stack, then its unused
// slack, then the overflow list. Phase 2 retires the used holes and slack.
__global__ void mirror_insert_kernel(MirrorK m, int64_t k, const int32_t *__restrict__ src,
                                     const int32_t *__restrict__ dst, const float *__restrict__ w,
                                     const int32_t *__restrict__ placed, int32_t *__restrict__ ins_count) {
  const uint32_t mask = (1u << m.cb) - 1u;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < k;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int32_t s = placed[i];
    if (s < 0) continue;
    const int32_t a = src[i], d = dst[i];
    if (a < 0 || a >= m.n || d < 0 || d >= m.n) continue;
    const int32_t g = d >> m.cb;
    const int64_t gb = m.gbase[g], gcap = m.gbase[g + 1] - gb;
    const int32_t r = atomicAdd(ins_count + g, 1);
    const int32_t holes = m.hcount[g];
    int64_t pos = -1;
    if (r < holes) {
      pos = gb + m.hstack[gb + holes - 1 - r];
    } else {
      const int64_t f = static_cast<int64_t>(m.gfill[g]) + (r - holes);
      if (f < gcap) pos = gb + f;
    }
    if (pos >= 0) {
      m.word[pos] = (static_cast<uint32_t>(a) << m.cb) | (static_cast<uint32_t>(d) & mask);
      m.w[pos] = w[i];
      m.slot[pos] = s;
    } else {
      const int32_t o = atomicAdd(m.ovf_count, 1);
      if (o < m.ovf_cap) {
        m.ovf_src[o] = a;
        m.ovf_dst[o] = d;
        m.ovf_w[o] = w[i];
        m.ovf_slot[o] = s;
      } else {
        atomicOr(m.status, 1);  // an edge is missing from the mirror: rebuild it
      }
    }
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

static int check_mirror(const char *fn, const pxb_mirror *m) {
  PXB_REQUIRE(m != nullptr, "%s: mirror is NULL", fn);
  PXB_REQUIRE(m->chunk_bits >= 2 && m->chunk_bits <= 13, "%s: chunk_bits %d not in [2, 13]", fn, m->chunk_bits);
  PXB_REQUIRE(m->num_units > 0, "%s: num_units must be > 0", fn);
  PXB_REQUIRE(m->groups == ((int64_t(m->num_units) + (int64_t(1) << m->chunk_bits) - 1) >> m->chunk_bits),
              "%s: groups does not match num_units and chunk_bits", fn);
  PXB_REQUIRE(m->entries % 8 == 0, "%s: entries must be a multiple of 8", fn);
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

extern "C" int pxb_mirror_forward(const pxb_mirror *mirror, const float *act, int32_t monoid, float *acc,
                                  int32_t prune_kind, float prune_threshold, const float *unit_threshold,
                                  uint8_t *dead, uint32_t *free_bitmap, int64_t bitmap_words,
                                  const int32_t *bitmap_level, int32_t *pruned_count, void *stream) {
  int rc = check_mirror("pxb_mirror_forward", mirror);
  if (rc) return rc;
  PXB_REQUIRE(monoid >= 0 && monoid <= 2, "pxb_mirror_forward: unknown monoid %d", monoid);
  PXB_REQUIRE(prune_kind >= 0 && prune_kind <= 2, "pxb_mirror_forward: unknown prune kind %d", prune_kind);
  PXB_REQUIRE(act && acc, "pxb_mirror_forward: act/acc is NULL");
  PXB_REQUIRE(prune_kind == PXB_PRUNE_NONE || dead, "pxb_mirror_forward: pruning needs the canonical dead column");
  PXB_REQUIRE(prune_kind != PXB_PRUNE_ABS_BELOW_DST || unit_threshold,
              "pxb_mirror_forward: per-destination threshold column is NULL");
  PXB_REQUIRE(monoid != PXB_MONOID_SUM || aligned16(acc), "pxb_mirror_forward: acc must be 16-byte aligned");
  MirrorK m = to_k(mirror);
  MPrune p{prune_kind, prune_threshold, unit_threshold, dead, free_bitmap, bitmap_words, bitmap_level, pruned_count};
  cudaStream_t st = as_stream(stream);
  const size_t smem = sizeof(float) << m.cb;
  if (m.entries > 0) {
    const int64_t full = int64_t(sm_count()) * 8;
    const int64_t want = (m.entries / 4 + 1023) / 1024;  // at least 4 K entries per CTA
    const int grid = static_cast<int>(want < full ? (want > 0 ? want : 1) : full);
#define PXB_MF(M, P) mirror_forward_kernel<M, P><<<grid, 256, smem, st>>>(m, act, acc, p)
    const bool pr = prune_kind != PXB_PRUNE_NONE;
    if (monoid == PXB_MONOID_SUM) { if (pr) PXB_MF(PXB_MONOID_SUM, true); else PXB_MF(PXB_MONOID_SUM, false); }
    else if (monoid == PXB_MONOID_MAX) { if (pr) PXB_MF(PXB_MONOID_MAX, true); else PXB_MF(PXB_MONOID_MAX, false); }
    else { if (pr) PXB_MF(PXB_MONOID_MIN, true); else PXB_MF(PXB_MONOID_MIN, false); }
#undef PXB_MF
    PXB_LAUNCHED("mirror_forward_kernel");
  }
  if (m.ovf_cap > 0) {
    const bool pr = prune_kind != PXB_PRUNE_NONE;
#define PXB_MO(M, P) mirror_overflow_kernel<M, P><<<sm_count(), 256, 0, st>>>(m, act, acc, p)
    if (monoid == PXB_MONOID_SUM) { if (pr) PXB_MO(PXB_MONOID_SUM, true); else PXB_MO(PXB_MONOID_SUM, false); }
    else if (monoid == PXB_MONOID_MAX) { if (pr) PXB_MO(PXB_MONOID_MAX, true); else PXB_MO(PXB_MONOID_MAX, false); }
    else { if (pr) PXB_MO(PXB_MONOID_MIN, true); else PXB_MO(PXB_MONOID_MIN, false); }
#undef PXB_MO
    PXB_LAUNCHED("mirror_overflow_kernel");
  }
  return PXB_OK;
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
  mirror_insert_kernel<<<grid_for(k, 256, 8), 256, 0, st>>>(m, k, src, dst, weight, placed, mirror->ins_count);
  PXB_LAUNCHED("mirror_insert_kernel");
  mirror_insert_finish_kernel<<<grid_for(m.groups, 256, 4), 256, 0, st>>>(m, mirror->ins_count);
  PXB_LAUNCHED("mirror_insert_finish_kernel");
  return PXB_OK;
}
