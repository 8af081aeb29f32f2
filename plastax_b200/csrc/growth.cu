// Growth candidates and their selection: Philox per-unit proposals with the
// framework validity window, the total candidate order as two stable radix
// passes (CUB, header-only), the step-scoped top-k relisted levels ascending,
// and the winners' gather with the growth rule's init values.
#include <cub/cub.cuh>

#include "pxb_common.cuh"

namespace pxb {

static inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

static inline int bits_for(int64_t bound) {
  int b = 1;
  while (b < 62 && (int64_t(1) << b) < bound) ++b;
  return b;
}

// ---------------------------------------------------------------------------
// raw Philox words
// ---------------------------------------------------------------------------
__global__ void philox_kernel(int64_t n, const uint64_t *__restrict__ seed, const uint64_t *__restrict__ ctr,
                              uint32_t *__restrict__ out) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    out[i] = philox32(seed[i], ctr[i]);
}

// ---------------------------------------------------------------------------
// per-unit proposals + validity (src/plastax/phases.py:3813-3860,
// :4041-4108; rng.py:207-246)
// ---------------------------------------------------------------------------
struct ProposeArgs {
  int32_t num_units, proposals;
  uint64_t keyed_hi;  // philox32(network_seed, (step << 8) | 1): the site seed's high limb
  uint64_t network_seed;
  const int32_t *step_dev;  // when set, the step is read here (graph replay) and keyed_hi derived from it
  int32_t dst_lo, dst_n, score_kind;
  const float *grad, *act;
  const int32_t *level;
  const uint8_t *pruned;
  int32_t max_level_gap, direction, allow_self_loops, bucket_level, src_level_bound;
};

// The site seed's high limb for this launch: philox32(network_seed,
// (step << 8) | 1), the step read from step_dev when set (graph replay).
__device__ __forceinline__ uint64_t keyed_hi_of(const ProposeArgs &a) {
  __shared__ uint64_t keyed;
  if (a.step_dev == nullptr) return a.keyed_hi;
  if (threadIdx.x == 0)
    keyed = philox32(a.network_seed, (static_cast<uint64_t>(static_cast<uint32_t>(*a.step_dev)) << 8) | 1u);
  __syncthreads();
  return keyed;
}

// The framework's validity window (src/plastax/phases.py:4041-4108): an
// out-of-range id is vetoed and clamped to 0 (_clamp_proposals); pruned
// endpoints, self-loops, the level gap, the direction, the bucket's source
// level and a non-finite score veto the candidate (score -inf), as does a
// dead proposing connection.
__device__ __forceinline__ void apply_window(const ProposeArgs &a, int32_t &src, int32_t &dst, float &score,
                                             bool proposer_live) {
  bool valid = proposer_live && src >= 0 && src < a.num_units && dst >= 0 && dst < a.num_units;
  if (!(src >= 0 && src < a.num_units && dst >= 0 && dst < a.num_units)) {
    src = 0;
    dst = 0;
  }
  if (valid && a.pruned != nullptr) valid = !a.pruned[src] && !a.pruned[dst];
  if (valid) {
    const int32_t ls = a.level[src], ld = a.level[dst];
    const int32_t gap = ld > ls ? ld - ls : ls - ld;
    valid = gap <= a.max_level_gap;
    if (!a.allow_self_loops) valid = valid && src != dst;
    if (a.direction == 1) valid = valid && ld > ls;
    else if (a.direction == 2) valid = valid && ld >= ls;
    if (a.bucket_level >= 0) valid = valid && ls == a.bucket_level;
    if (a.src_level_bound > 0) valid = valid && ls < a.src_level_bound;
  }
  if (!valid || !isfinite(score)) score = -__int_as_float(0x7f800000);
}

// A proposal's score at draw `sub` of its site: uniform, floor(u*256)/256,
// or |grad[dst] * act[src]| (no draw).
__device__ __forceinline__ float proposal_score(const ProposeArgs &a, uint64_t seed, uint32_t j, uint32_t sub,
                                                int32_t src, int32_t dst) {
  if (a.score_kind == PXB_SCORE_UNIFORM) return unit_float(site_draw(seed, j, sub));
  if (a.score_kind == PXB_SCORE_UNIFORM_Q256) {
    const float u = unit_float(site_draw(seed, j, sub));
    return static_cast<float>(static_cast<int32_t>(__fmul_rn(u, 256.0f))) * (1.0f / 256.0f);
  }
  const bool in = dst >= 0 && dst < a.num_units && src >= 0 && src < a.num_units;
  return in ? fabsf(__fmul_rn(a.grad[dst], a.act[src])) : 0.0f;
}

// Candidate c = i * proposals + j of unit i: its endpoints and score, the
// score -inf when the framework's validity window vetoes it.
__device__ __forceinline__ void propose_one(const ProposeArgs &a, uint64_t keyed_hi, int64_t c, int32_t &src_o,
                                            int32_t &dst_o, float &score_o) {
  const int32_t i = static_cast<int32_t>(c / a.proposals);
  const uint32_t j = static_cast<uint32_t>(c - static_cast<int64_t>(i) * a.proposals);
  const uint64_t seed = (keyed_hi << 32) | static_cast<uint32_t>(i);
  int32_t src = i;
  int32_t dst = a.dst_lo + static_cast<int32_t>(uniform_int(unit_float(site_draw(seed, j, 0)), a.dst_n));
  float score = proposal_score(a, seed, j, 1, src, dst);
  apply_window(a, src, dst, score, true);
  src_o = src;
  dst_o = dst;
  score_o = score;
}

__global__ void propose_per_unit_kernel(ProposeArgs a, int32_t *__restrict__ src_out,
                                        int32_t *__restrict__ dst_out, float *__restrict__ score_out) {
  const int64_t total = static_cast<int64_t>(a.num_units) * a.proposals;
  const uint64_t keyed_hi = keyed_hi_of(a);
  for (int64_t c = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; c < total;
       c += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int32_t src, dst;
    float score;
    propose_one(a, keyed_hi, c, src, dst, score);
    src_out[c] = src;
    dst_out[c] = dst;
    score_out[c] = score;
  }
}

// ---------------------------------------------------------------------------
// total order (src/plastax/phases.py:4208-4321)
// ---------------------------------------------------------------------------
// Order-preserving uint32 image of the leading key: -score, NaN -> +inf,
// -0 -> +0.
__device__ __forceinline__ uint32_t score_key(float s) {
  float neg = isnan(s) ? __int_as_float(0x7f800000) : -s;
  if (neg == 0.0f) neg = 0.0f;
  const uint32_t u = __float_as_uint(neg);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__global__ void pair_key_kernel(int64_t n, const int32_t *__restrict__ src, const int32_t *__restrict__ dst,
                                int bits, uint64_t *__restrict__ keys, int32_t *__restrict__ vals) {
  const uint64_t mask = (uint64_t(1) << bits) - 1;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    keys[i] = ((static_cast<uint64_t>(static_cast<uint32_t>(src[i])) & mask) << bits) |
              (static_cast<uint64_t>(static_cast<uint32_t>(dst[i])) & mask);
    vals[i] = static_cast<int32_t>(i);
  }
}

__global__ void score_key_kernel(int64_t n, const float *__restrict__ score, const int32_t *__restrict__ perm,
                                 uint32_t *__restrict__ keys) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    keys[i] = score_key(score[perm[i]]);
}

struct OrderScratch {
  uint64_t *pair_in, *pair_out;
  uint32_t *skey_in, *skey_out;
  int32_t *val_a, *val_b;
  void *cub_tmp;
  size_t cub_bytes;
  size_t total;
};

static int order_scratch(int64_t n, int bits, char *base, OrderScratch *o) {
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t at = off;
    off = align_up(off + bytes, 256);
    return base ? base + at : nullptr;
  };
  o->pair_in = reinterpret_cast<uint64_t *>(take(n * sizeof(uint64_t)));
  o->pair_out = reinterpret_cast<uint64_t *>(take(n * sizeof(uint64_t)));
  o->skey_in = reinterpret_cast<uint32_t *>(take(n * sizeof(uint32_t)));
  o->skey_out = reinterpret_cast<uint32_t *>(take(n * sizeof(uint32_t)));
  o->val_a = reinterpret_cast<int32_t *>(take(n * sizeof(int32_t)));
  o->val_b = reinterpret_cast<int32_t *>(take(n * sizeof(int32_t)));
  size_t t1 = 0, t2 = 0;
  if (cub::DeviceRadixSort::SortPairs(nullptr, t1, o->pair_in, o->pair_out, o->val_a, o->val_b,
                                      static_cast<int>(n), 0, 2 * bits) != cudaSuccess)
    return PXB_ECUDA;
  if (cub::DeviceRadixSort::SortPairs(nullptr, t2, o->skey_in, o->skey_out, o->val_b, o->val_a,
                                      static_cast<int>(n), 0, 32) != cudaSuccess)
    return PXB_ECUDA;
  o->cub_bytes = t1 > t2 ? t1 : t2;
  o->cub_tmp = take(o->cub_bytes);
  o->total = off;
  return PXB_OK;
}

// ---------------------------------------------------------------------------
// step-scoped selection (src/plastax/phases.py:4891-4903, level_major
// :4469-4487): the first k of the total order, relisted levels ascending.
// ---------------------------------------------------------------------------
__global__ void winner_level_kernel(int64_t kk, const int32_t *__restrict__ perm, const int32_t *__restrict__ src,
                                    const int32_t *__restrict__ level, uint32_t *__restrict__ keys,
                                    int32_t *__restrict__ vals) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < kk;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int32_t c = perm[i];
    keys[i] = static_cast<uint32_t>(level[src[c]]);
    vals[i] = c;
  }
}

__global__ void set_i32_kernel(int32_t *p, int32_t v) { *p = v; }

struct SelectScratch {
  uint32_t *key_in, *key_out;
  int32_t *val_in;
  void *cub_tmp;
  size_t cub_bytes, total;
};

static int select_scratch(int64_t kk, char *base, SelectScratch *o, int32_t *val_out_probe) {
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t at = off;
    off = align_up(off + bytes, 256);
    return base ? base + at : nullptr;
  };
  o->key_in = reinterpret_cast<uint32_t *>(take(kk * sizeof(uint32_t)));
  o->key_out = reinterpret_cast<uint32_t *>(take(kk * sizeof(uint32_t)));
  o->val_in = reinterpret_cast<int32_t *>(take(kk * sizeof(int32_t)));
  size_t t = 0;
  if (cub::DeviceRadixSort::SortPairs(nullptr, t, o->key_in, o->key_out, o->val_in, val_out_probe,
                                      static_cast<int>(kk), 0, 32) != cudaSuccess)
    return PXB_ECUDA;
  o->cub_bytes = t;
  o->cub_tmp = take(t);
  o->total = off;
  return PXB_OK;
}

// ---------------------------------------------------------------------------
// winners' gather: (src, dst, init weight, growable) per selected candidate
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t lowbias32(uint32_t x) {
  x ^= x >> 16;
  x *= 0x7FEB352Du;
  x ^= x >> 15;
  x *= 0x846CA68Bu;
  return x ^ (x >> 16);
}

struct InitArgs {
  int32_t kind;  // PXB_INIT_*
  float a, b;
  uint32_t salt;
};

__device__ __forceinline__ float init_weight(const InitArgs &ia, int32_t src, int32_t dst) {
  switch (ia.kind) {
    case PXB_INIT_CONST: return ia.a;
    case PXB_INIT_DYADIC: {
      const int32_t r = ((3 * src + 5 * dst) % 16) - 8;
      return static_cast<float>(r) / 8.0f;
    }
    case PXB_INIT_HASH_UNIFORM: {
      uint32_t h = lowbias32(0x9E3779B9u ^ static_cast<uint32_t>(src));
      h = lowbias32(h ^ static_cast<uint32_t>(dst));
      h = lowbias32(h ^ ia.salt);
      const float u = unit_float(h);
      return __fmul_rn(ia.a, __fsub_rn(__fmul_rn(2.0f, u), 1.0f));
    }
    default: return 0.0f;
  }
}

__global__ void gather_winners_kernel(int64_t k, int64_t count, const int32_t *__restrict__ win,
                                      const int32_t *__restrict__ src, const int32_t *__restrict__ dst,
                                      const float *__restrict__ score, InitArgs ia, int32_t *__restrict__ s_out,
                                      int32_t *__restrict__ d_out, float *__restrict__ w_out,
                                      uint8_t *__restrict__ growable) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < k;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    if (i < count && win[i] >= 0) {
      const int32_t c = win[i];
      const int32_t s = src[c], d = dst[c];
      s_out[i] = s;
      d_out[i] = d;
      w_out[i] = init_weight(ia, s, d);
      growable[i] = isfinite(score[c]) ? 1 : 0;
    } else {
      s_out[i] = 0;
      d_out[i] = 0;
      w_out[i] = 0.0f;
      growable[i] = 0;
    }
  }
}

// ---------------------------------------------------------------------------
// top-k by unique 64-bit keys: exact radix select of the k-th key, one
// compaction, a sort of the k winners only
// ---------------------------------------------------------------------------
constexpr int kSelBits = 11;
constexpr int kSelBins = 1 << kSelBits;

struct SelState {
  unsigned long long prefix;  // selected high digits so far
  long long remaining;        // rank still to find inside the prefix
  unsigned long long thr;     // final k-th key
  int count;                  // compaction cursor
};

__global__ void unique_key_kernel(int64_t n, const float *__restrict__ score, const int32_t *__restrict__ src,
                                  int src_bits, uint64_t *__restrict__ keys) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    keys[i] = (static_cast<uint64_t>(score_key(score[i])) << src_bits) |
              (static_cast<uint64_t>(static_cast<uint32_t>(src[i])) & ((uint64_t(1) << src_bits) - 1));
}

__global__ void sel_histogram_kernel(int64_t n, const uint64_t *__restrict__ keys, int shift, int width,
                                     int hi_shift, const SelState *__restrict__ st, unsigned int *__restrict__ hist) {
  __shared__ unsigned int h[kSelBins];
  for (int b = threadIdx.x; b < kSelBins; b += blockDim.x) h[b] = 0;
  __syncthreads();
  const unsigned long long prefix = st->prefix;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint64_t key = keys[i];
    if (hi_shift >= 64 || (key >> hi_shift) == prefix) atomicAdd(&h[(key >> shift) & ((1u << width) - 1u)], 1u);
  }
  __syncthreads();
  for (int b = threadIdx.x; b < kSelBins; b += blockDim.x)
    if (h[b]) atomicAdd(hist + b, h[b]);
}

// one block: find the bin holding rank `remaining`, extend the prefix
__global__ void sel_pick_kernel(unsigned int *__restrict__ hist, SelState *__restrict__ st, int last, int width) {
  __shared__ unsigned int part[1024];
  const int t = threadIdx.x;  // 1024 threads, 2 bins each
  const unsigned int a = hist[2 * t], b = hist[2 * t + 1];
  part[t] = a + b;
  __syncthreads();
  for (int off = 1; off < 1024; off <<= 1) {  // inclusive scan
    const unsigned int v = t >= off ? part[t - off] : 0u;
    __syncthreads();
    part[t] += v;
    __syncthreads();
  }
  const long long rem = st->remaining;
  const long long before = t ? part[t - 1] : 0;
  __syncthreads();
  if (before <= rem && rem < before + a + b) {
    int bin;
    long long below;
    if (rem < before + a) { bin = 2 * t; below = before; }
    else { bin = 2 * t + 1; below = before + a; }
    st->prefix = (st->prefix << width) | static_cast<unsigned long long>(bin);
    st->remaining = rem - below;
    if (last) st->thr = st->prefix;
  }
  hist[2 * t] = 0;
  hist[2 * t + 1] = 0;
}

__global__ void sel_compact_kernel(int64_t n, const uint64_t *__restrict__ keys, SelState *__restrict__ st,
                                   uint64_t *__restrict__ out_keys, int32_t *__restrict__ out_idx) {
  const unsigned long long thr = st->thr;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint64_t key = keys[i];
    const bool take = key <= thr;
    const unsigned mask = __ballot_sync(__activemask(), take);
    if (!take) continue;
    const int lane = threadIdx.x & 31;
    const int leader = __ffs(mask) - 1;
    int base = 0;
    if (lane == leader) base = atomicAdd(&st->count, __popc(mask));
    base = __shfl_sync(mask, base, leader);
    const int pos = base + __popc(mask & ((1u << lane) - 1u));
    out_keys[pos] = key;
    out_idx[pos] = static_cast<int32_t>(i);
  }
}

__global__ void sel_init_kernel(SelState *st, long long k) {
  st->prefix = 0;
  st->remaining = k - 1;  // rank of the k-th key (0-based)
  st->thr = 0;
  st->count = 0;
}

struct TopkScratch {
  uint64_t *keys, *ckeys, *skeys;
  int32_t *cidx;
  SelState *st;
  unsigned int *hist;
  void *cub_tmp;
  size_t cub_bytes, total;
};

static int topk_scratch(int64_t n, int64_t k, int key_bits, char *base, TopkScratch *o, int32_t *probe_out) {
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t at = off;
    off = align_up(off + (bytes ? bytes : 1), 256);
    return base ? base + at : nullptr;
  };
  const int64_t kk = k > 0 ? k : 1;
  o->keys = reinterpret_cast<uint64_t *>(take(n * 8));
  o->ckeys = reinterpret_cast<uint64_t *>(take(kk * 8));
  o->skeys = reinterpret_cast<uint64_t *>(take(kk * 8));
  o->cidx = reinterpret_cast<int32_t *>(take(kk * 4));
  o->st = reinterpret_cast<SelState *>(take(sizeof(SelState)));
  o->hist = reinterpret_cast<unsigned int *>(take(kSelBins * 4));
  size_t t = 0;
  if (cub::DeviceRadixSort::SortPairs(nullptr, t, o->ckeys, o->skeys, o->cidx, probe_out, static_cast<int>(kk), 0,
                                      key_bits) != cudaSuccess)
    return PXB_ECUDA;
  o->cub_bytes = t;
  o->cub_tmp = take(t);
  o->total = off;
  return PXB_OK;
}

}  // namespace pxb

using namespace pxb;

extern "C" int pxb_topk_unique_scratch_bytes(int64_t n, int64_t k, int32_t id_bound, size_t *bytes) {
  PXB_REQUIRE(bytes && n >= 0 && k >= 0 && n < (int64_t(1) << 31) && id_bound >= 1,
              "pxb_topk_unique_scratch_bytes: bad arguments");
  TopkScratch o;
  const int key_bits = 32 + bits_for(id_bound);
  if (topk_scratch(n, k < n ? k : n, key_bits, nullptr, &o, nullptr) != PXB_OK) {
    set_error("pxb_topk_unique_scratch_bytes: CUB size query failed");
    return PXB_ECUDA;
  }
  *bytes = o.total;
  return PXB_OK;
}

extern "C" int pxb_topk_unique(int64_t n, const float *score, const int32_t *src, int32_t id_bound, int64_t k,
                               int32_t *out_idx, void *scratch, size_t scratch_bytes, void *stream) {
  PXB_REQUIRE(n >= 0 && k >= 0 && n < (int64_t(1) << 31) && id_bound >= 1, "pxb_topk_unique: bad sizes");
  const int64_t kk = k < n ? k : n;
  if (kk == 0) return PXB_OK;
  PXB_REQUIRE(score && src && out_idx && scratch, "pxb_topk_unique: a pointer is NULL");
  const int src_bits = bits_for(id_bound);
  const int key_bits = 32 + src_bits;
  TopkScratch o;
  if (topk_scratch(n, kk, key_bits, static_cast<char *>(scratch), &o, out_idx) != PXB_OK) {
    set_error("pxb_topk_unique: CUB size query failed");
    return PXB_ECUDA;
  }
  PXB_REQUIRE(o.total <= scratch_bytes, "pxb_topk_unique: scratch has %zu bytes, needs %zu", scratch_bytes, o.total);
  cudaStream_t st = as_stream(stream);
  const int grid = grid_for(n, 256, 4);
  unique_key_kernel<<<grid, 256, 0, st>>>(n, score, src, src_bits, o.keys);
  PXB_LAUNCHED("unique_key_kernel");
  sel_init_kernel<<<1, 1, 0, st>>>(o.st, kk);
  PXB_LAUNCHED("sel_init_kernel");
  PXB_CUDA(cudaMemsetAsync(o.hist, 0, kSelBins * 4, st));
  // digits of up to 11 bits from the most significant end; a pass counts
  // the keys whose higher digits equal the prefix picked so far
  for (int rem_bits = key_bits; rem_bits > 0;) {
    const int width = rem_bits < kSelBits ? rem_bits : kSelBits;
    const int shift = rem_bits - width;
    const int hi_shift = rem_bits >= key_bits ? 64 : rem_bits;
    sel_histogram_kernel<<<grid, 256, 0, st>>>(n, o.keys, shift, width, hi_shift, o.st, o.hist);
    PXB_LAUNCHED("sel_histogram_kernel");
    sel_pick_kernel<<<1, 1024, 0, st>>>(o.hist, o.st, shift == 0, width);
    PXB_LAUNCHED("sel_pick_kernel");
    rem_bits = shift;
  }
  sel_compact_kernel<<<grid, 256, 0, st>>>(n, o.keys, o.st, o.ckeys, o.cidx);
  PXB_LAUNCHED("sel_compact_kernel");
  size_t tb = o.cub_bytes;
  PXB_CUDA(cub::DeviceRadixSort::SortPairs(o.cub_tmp, tb, o.ckeys, o.skeys, o.cidx, out_idx, static_cast<int>(kk), 0,
                                           key_bits, st));
  return PXB_OK;
}

extern "C" int pxb_philox32(int64_t n, const uint64_t *seed, const uint64_t *counter, uint32_t *out,
                            void *stream) {
  PXB_REQUIRE(n >= 0, "pxb_philox32: negative n");
  if (n == 0) return PXB_OK;
  PXB_REQUIRE(seed && counter && out, "pxb_philox32: a pointer is NULL");
  philox_kernel<<<grid_for(n, 256, 8), 256, 0, as_stream(stream)>>>(n, seed, counter, out);
  PXB_LAUNCHED("philox_kernel");
  return PXB_OK;
}

extern "C" uint64_t pxb_site_seed(uint64_t network_seed, uint32_t step, uint32_t stream_id, uint32_t key) {
  return site_seed(network_seed, step, stream_id, key);
}

extern "C" int pxb_propose_per_unit(int32_t num_units, int32_t proposals, uint64_t network_seed, int32_t step,
                                    int32_t dst_lo, int32_t dst_n, int32_t score_kind, const float *grad,
                                    const float *act, const int32_t *level, const uint8_t *pruned,
                                    int32_t max_level_gap, int32_t direction, int32_t allow_self_loops,
                                    int32_t bucket_level, int32_t src_level_bound, const int32_t *step_dev,
                                    int32_t *src_out, int32_t *dst_out, float *score_out, void *stream) {
  PXB_REQUIRE(num_units >= 0 && proposals >= 0, "pxb_propose_per_unit: negative sizes");
  PXB_REQUIRE(dst_n >= 1, "pxb_propose_per_unit: dst_n must be >= 1");
  PXB_REQUIRE(score_kind >= 0 && score_kind <= 2, "pxb_propose_per_unit: unknown score kind %d", score_kind);
  PXB_REQUIRE(direction >= 0 && direction <= 2, "pxb_propose_per_unit: unknown direction %d", direction);
  PXB_REQUIRE(score_kind != PXB_SCORE_GRAD_ACT || (grad && act), "pxb_propose_per_unit: grad/act is NULL");
  const int64_t total = static_cast<int64_t>(num_units) * proposals;
  if (total == 0) return PXB_OK;
  PXB_REQUIRE(total < (int64_t(1) << 31), "pxb_propose_per_unit: more than 2^31 candidates");
  PXB_REQUIRE(level && src_out && dst_out && score_out, "pxb_propose_per_unit: a pointer is NULL");
  ProposeArgs a;
  a.num_units = num_units;
  a.proposals = proposals;
  a.keyed_hi = philox32(network_seed, (static_cast<uint64_t>(static_cast<uint32_t>(step)) << 8) | 1u);
  a.network_seed = network_seed;
  a.step_dev = step_dev;
  a.dst_lo = dst_lo;
  a.dst_n = dst_n;
  a.score_kind = score_kind;
  a.grad = grad;
  a.act = act;
  a.level = level;
  a.pruned = pruned;
  a.max_level_gap = max_level_gap;
  a.direction = direction;
  a.allow_self_loops = allow_self_loops;
  a.bucket_level = bucket_level;
  a.src_level_bound = src_level_bound;
  propose_per_unit_kernel<<<grid_for(total, 256, 8), 256, 0, as_stream(stream)>>>(a, src_out, dst_out,
                                                                                  score_out);
  PXB_LAUNCHED("propose_per_unit_kernel");
  return PXB_OK;
}

extern "C" int pxb_total_order_scratch_bytes(int64_t n, int32_t id_bound, size_t *bytes) {
  PXB_REQUIRE(bytes != nullptr, "pxb_total_order_scratch_bytes: bytes is NULL");
  PXB_REQUIRE(n >= 0 && n < (int64_t(1) << 31), "pxb_total_order_scratch_bytes: n out of range");
  PXB_REQUIRE(id_bound >= 1, "pxb_total_order_scratch_bytes: id_bound must be >= 1");
  OrderScratch o;
  if (order_scratch(n, bits_for(id_bound), nullptr, &o) != PXB_OK) {
    set_error("pxb_total_order_scratch_bytes: CUB size query failed");
    return PXB_ECUDA;
  }
  *bytes = o.total;
  return PXB_OK;
}

namespace pxb {
// The total order over caller-provided scratch (shared by pxb_total_order
// and its allocation-free variant).
int total_order_impl(const char *fn, int64_t n, const float *score, const int32_t *src, const int32_t *dst,
                     int32_t id_bound, int32_t *perm_out, void *scratch, size_t scratch_bytes, cudaStream_t st) {
  PXB_REQUIRE(n >= 0 && n < (int64_t(1) << 31), "%s: n out of range", fn);
  PXB_REQUIRE(id_bound >= 1, "%s: id_bound must be >= 1", fn);
  if (n == 0) return PXB_OK;
  PXB_REQUIRE(score && src && dst && perm_out && scratch, "%s: a pointer is NULL", fn);
  const int bits = bits_for(id_bound);
  OrderScratch o;
  if (order_scratch(n, bits, static_cast<char *>(scratch), &o) != PXB_OK) {
    set_error("%s: CUB size query failed", fn);
    return PXB_ECUDA;
  }
  PXB_REQUIRE(o.total <= scratch_bytes, "%s: scratch has %zu bytes, needs %zu", fn, scratch_bytes, o.total);
  const int grid = grid_for(n, 256, 8);
  pair_key_kernel<<<grid, 256, 0, st>>>(n, src, dst, bits, o.pair_in, o.val_a);
  PXB_LAUNCHED("pair_key_kernel");
  size_t tb = o.cub_bytes;
  PXB_CUDA(cub::DeviceRadixSort::SortPairs(o.cub_tmp, tb, o.pair_in, o.pair_out, o.val_a, o.val_b,
                                           static_cast<int>(n), 0, 2 * bits, st));
  score_key_kernel<<<grid, 256, 0, st>>>(n, score, o.val_b, o.skey_in);
  PXB_LAUNCHED("score_key_kernel");
  tb = o.cub_bytes;
  PXB_CUDA(cub::DeviceRadixSort::SortPairs(o.cub_tmp, tb, o.skey_in, o.skey_out, o.val_b, perm_out,
                                           static_cast<int>(n), 0, 32, st));
  return PXB_OK;
}

size_t total_order_bytes(int64_t n, int32_t id_bound) {
  OrderScratch o;
  if (order_scratch(n, bits_for(id_bound), nullptr, &o) != PXB_OK) return ~size_t(0);
  return o.total;
}
// ---------------------------------------------------------------------------
// Fused selection for one Philox-scored proposal per unit (score uniform or
// uniform_q256): the proposals, the first k of the total order and their
// level-major listing, gathered into the claim's input columns.
//
// Each candidate gets a unique key whose order is the total order: a valid
// candidate 0 | (2^b - 1 - m) | src, with m the score's b-bit integer
// (score = m * 2^-b), an invalid one 1 | src | 0. The top bin_bits of the
// key name its bin; bins are sized for ~256 candidates (the score integers
// are Philox draws, and an invalid bin spans a fixed range of sources), so
// a bin is ordered by ranking its members in shared memory. The threshold
// bin is found from the (level, bin) histogram, the winners of full bins are
// scattered into level-major bins, and the threshold bin's best r are
// ranked apart. A bin larger than kFsRankCap is ranked from global memory
// (up to kFsSlowCap members; beyond that status bit 0 is set and the list
// is incomplete -- never reached by Philox-scored proposals in practice).
// ---------------------------------------------------------------------------
constexpr int kFsMaxLevels = 8;
constexpr int kFsRankCap = 4096;
constexpr int kFsSlowCap = 1 << 16;
constexpr int kFsThreads = 256;
constexpr int kFsMaxBinBits = 13;
constexpr int kFsMaxIpt = (1 << kFsMaxBinBits) / 1024;
// One (level, bin) counter per 32-byte sector: the propose pass's million
// returning atomics spread over every L2 slice instead of queueing on the
// few lines a packed array of counters occupies.
constexpr int kFsHistStride = 8;
__host__ __device__ __forceinline__ int64_t fs_hidx(int64_t lb) { return lb * kFsHistStride; }

struct FsGeom {
  int32_t n, L, nb;
  int64_t k;
  int src_bits, score_bits, key_bits, bin_bits;
};

struct FsInfo {
  int32_t tb, r, count, tcount;
  int32_t C[kFsMaxLevels], R[kFsMaxLevels], F[kFsMaxLevels], T[kFsMaxLevels];
};

struct FsScratch {
  uint64_t *keys, *tk, *bk;
  // byrank: each candidate's slot inside its (level, bin) from the propose
  // pass to the scatter, then the threshold bin's members by rank
  int32_t *dst, *ti, *bi, *byrank;
  uint32_t *hist, *toff;
  FsInfo *info;
  size_t total;
};

// Where the winners go: `world` ranks' columns of `blocks` lists of k
// entries each (one rank and one list for the plain selection). Rank `rank`
// ranks the full (level, bin) pairs q with q % world == rank and stores
// their winners into every rank's columns; the threshold bin and the zero
// fill are computed by every rank and stored into its own only.
constexpr int kSelMaxWorld = PXB_SELECT_MAX_WORLD;
struct FsOut {
  int32_t rank, world, blocks, step;  // step: the list's step when step_dev is NULL
  const int32_t *step_dev;
  int32_t *s[kSelMaxWorld];
  int32_t *d[kSelMaxWorld];
  float *w[kSelMaxWorld];
  uint8_t *g[kSelMaxWorld];
};

// Offset of this launch's list inside a column: (step mod blocks) * k.
__device__ __forceinline__ int64_t fs_list_base(const FsOut &out, int64_t k) {
  if (out.blocks <= 1) return 0;
  const int32_t st = out.step_dev != nullptr ? *out.step_dev : out.step;
  const int32_t b = ((st % out.blocks) + out.blocks) % out.blocks;
  return static_cast<int64_t>(b) * k;
}

__device__ __forceinline__ bool fs_owns(int32_t rank, int32_t world, int64_t pair) {
  return world <= 1 || pair % world == rank;
}

__device__ __forceinline__ uint64_t fs_key(const FsGeom &g, int kind, float score, int32_t src) {
  const uint64_t s = static_cast<uint32_t>(src);
  if (!(score >= 0.0f)) return (uint64_t(1) << (g.key_bits - 1)) | (s << g.score_bits);
  const uint32_t m = kind == PXB_SCORE_UNIFORM ? static_cast<uint32_t>(score * 16777216.0f)
                                                : static_cast<uint32_t>(score * 256.0f);
  const uint64_t d = ((uint64_t(1) << g.score_bits) - 1) - m;
  return (d << g.src_bits) | s;
}
__device__ __forceinline__ bool fs_valid(const FsGeom &g, uint64_t key) { return !(key >> (g.key_bits - 1)); }
__device__ __forceinline__ int32_t fs_src(const FsGeom &g, uint64_t key) {
  const uint64_t mask = (uint64_t(1) << g.src_bits) - 1;
  return static_cast<int32_t>(fs_valid(g, key) ? (key & mask) : ((key >> g.score_bits) & mask));
}
__device__ __forceinline__ int32_t fs_bin(const FsGeom &g, uint64_t key) {
  return static_cast<int32_t>(key >> (g.key_bits - g.bin_bits));
}
__device__ __forceinline__ int32_t fs_level(const FsGeom &g, const int32_t *level, int32_t src) {
  const int32_t l = level[src];
  return l < 0 ? 0 : (l >= g.L ? g.L - 1 : l);
}

__global__ void __launch_bounds__(kFsThreads) fs_propose_kernel(ProposeArgs a, FsGeom g, FsScratch o) {
  const uint64_t keyed_hi = keyed_hi_of(a);
  for (int64_t c = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; c < g.n;
       c += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int32_t src, dst;
    float score;
    propose_one(a, keyed_hi, c, src, dst, score);
    const uint64_t key = fs_key(g, a.score_kind, score, src);
    o.keys[c] = key;
    o.dst[c] = dst;
    // the count's old value is the candidate's slot inside its (level, bin):
    // the scatter needs no atomic of its own
    o.byrank[c] = static_cast<int32_t>(
        atomicAdd(o.hist + fs_hidx(static_cast<int64_t>(fs_level(g, a.level, src)) * g.nb + fs_bin(g, key)), 1u));
  }
}

// One block: the threshold bin, the level counts and the temp offsets of the
// full bins (level-major). Thread t owns the consecutive bins
// [t * ipt, (t + 1) * ipt): one block scan finds the threshold bin and one
// per level lays out the full bins.
__global__ void __launch_bounds__(1024) fs_threshold_kernel(FsGeom g, FsScratch o) {
  using Scan = cub::BlockScan<int32_t, 1024>;
  __shared__ typename Scan::TempStorage ts;
  __shared__ int32_t s_tb, s_excl;
  FsInfo *info = o.info;
  const int ipt = (g.nb + 1023) / 1024;  // <= kFsMaxIpt (bins are capped at 8192)
  const int b0 = threadIdx.x * ipt;
  if (threadIdx.x == 0) {
    s_tb = g.nb;
    s_excl = 0;
  }
  // this thread's bin totals over the levels, every load issued at once
  int32_t tot[kFsMaxIpt];
#pragma unroll
  for (int j = 0; j < kFsMaxIpt; ++j) tot[j] = 0;
  for (int l = 0; l < g.L; ++l) {
#pragma unroll
    for (int j = 0; j < kFsMaxIpt; ++j)
      if (j < ipt && b0 + j < g.nb) tot[j] += static_cast<int32_t>(o.hist[fs_hidx(l * g.nb + b0 + j)]);
  }
  int32_t mine = 0;
#pragma unroll
  for (int j = 0; j < kFsMaxIpt; ++j) mine += tot[j];
  int32_t ex, agg;
  Scan(ts).ExclusiveSum(mine, ex, agg);
  if (g.k < g.n && ex < g.k && ex + mine >= g.k) {  // the crossing lies in my bins
    int32_t cum = ex;
    bool found = false;
#pragma unroll
    for (int j = 0; j < kFsMaxIpt; ++j) {
      if (!found && j < ipt && cum + tot[j] >= g.k) {
        s_tb = b0 + j;
        s_excl = cum;
        found = true;
      }
      cum += tot[j];
    }
  }
  __syncthreads();
  const int32_t tb = s_tb;
  int32_t t_run = 0;
  for (int l = 0; l < g.L; ++l) {
    int32_t v[kFsMaxIpt];
    int32_t lm = 0;
#pragma unroll
    for (int j = 0; j < kFsMaxIpt; ++j) {
      v[j] = (j < ipt && b0 + j < tb) ? static_cast<int32_t>(o.hist[fs_hidx(l * g.nb + b0 + j)]) : 0;
      lm += v[j];
    }
    int32_t lex, lagg;
    __syncthreads();  // the scan storage is reused
    Scan(ts).ExclusiveSum(lm, lex, lagg);
    int32_t run = t_run + lex;
#pragma unroll
    for (int j = 0; j < kFsMaxIpt; ++j) {
      if (j < ipt && b0 + j < g.nb) {
        o.toff[l * g.nb + b0 + j] = static_cast<uint32_t>(run);
      }
      run += v[j];
    }
    if (threadIdx.x == 0) {
      info->C[l] = lagg;
      info->T[l] = t_run;
    }
    t_run += lagg;
  }
  if (threadIdx.x == 0) {
    info->tb = tb;
    info->r = tb < g.nb ? static_cast<int32_t>(g.k - s_excl) : 0;
    info->count = static_cast<int32_t>(g.k < g.n ? g.k : g.n);
    info->tcount = 0;
  }
}

__global__ void __launch_bounds__(kFsThreads) fs_scatter_kernel(FsGeom g, const int32_t *__restrict__ level,
                                                                 FsScratch o, int32_t rank, int32_t world) {
  const int32_t tb = o.info->tb;
  for (int64_t c = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; c < g.n;
       c += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint64_t key = o.keys[c];
    const int32_t b = fs_bin(g, key);
    if (b < tb) {
      const int32_t l = fs_level(g, level, fs_src(g, key));
      if (!fs_owns(rank, world, static_cast<int64_t>(l) * tb + b)) continue;  // another rank ranks this pair
      const int32_t slot = l * g.nb + b;
      const uint32_t pos = o.toff[slot] + static_cast<uint32_t>(o.byrank[c]);
      o.bk[pos] = key;
      o.bi[pos] = static_cast<int32_t>(c);
    } else if (b == tb) {
      const int32_t p = atomicAdd(&o.info->tcount, 1);
      o.tk[p] = key;
      o.ti[p] = static_cast<int32_t>(c);
    }
  }
}

// Rank of each of m unique keys (the number of smaller keys), from shared
// memory when they fit, else from global memory. Returns false (and ranks
// nothing) past kFsSlowCap.
__device__ __forceinline__ bool fs_rank(const uint64_t *keys_g, int32_t m, uint64_t *keys_s, int32_t *rank_out) {
  if (m > kFsSlowCap) return false;
  const bool in_smem = m <= kFsRankCap;
  if (in_smem) {
    for (int e = threadIdx.x; e < m; e += blockDim.x) keys_s[e] = keys_g[e];
    __syncthreads();
  }
  const uint64_t *src = in_smem ? keys_s : keys_g;
  for (int e = threadIdx.x; e < m; e += blockDim.x) {
    const uint64_t ke = src[e];
    int32_t r = 0;
    for (int f = 0; f < m; ++f) r += src[f] < ke ? 1 : 0;
    rank_out[e] = r;
  }
  __syncthreads();
  return true;
}

// Winner `key` (candidate c) at list position pos: into this rank's list,
// or into every rank's when `every` (a full bin this rank ranks).
__device__ __forceinline__ void fs_emit(const FsGeom &g, const FsScratch &o, const InitArgs &ia, uint64_t key,
                                        int32_t c, int64_t pos, const FsOut &out, bool every) {
  const int32_t s = fs_src(g, key), d = o.dst[c];
  const float w = init_weight(ia, s, d);
  const uint8_t grow = fs_valid(g, key) ? 1 : 0;
  const int q0 = every ? 0 : out.rank, q1 = every ? out.world : out.rank + 1;
  for (int q = q0; q < q1; ++q) {
    out.s[q][pos] = s;
    out.d[q][pos] = d;
    out.w[q][pos] = w;
    out.g[q][pos] = grow;
  }
}

// One block: the threshold bin's best r, their level counts, the level
// bases of the final list, and the zero fill past min(k, n).
__global__ void __launch_bounds__(1024) fs_threshold_bin_kernel(FsGeom g, const int32_t *__restrict__ level,
                                                                InitArgs ia, FsScratch o, FsOut out,
                                                                int32_t *status) {
  using Scan = cub::BlockScan<int32_t, 1024>;
  __shared__ typename Scan::TempStorage ts;
  __shared__ uint64_t keys_s[kFsRankCap];
  __shared__ int32_t s_carry;
  FsInfo *info = o.info;
  const int64_t list = fs_list_base(out, g.k);
  const int32_t m = info->tcount;
  int32_t r = info->r;
  int32_t *rank = o.ti + g.n;  // member ranks, then level positions (the scratch holds 3n)
  if (r > 0 && !fs_rank(o.tk, m, keys_s, rank)) {
    // unreachable for Philox scores; the list is flagged and the threshold
    // bin's winners are left out, every write staying in range
    if (threadIdx.x == 0 && status) atomicOr(status, 1);
    r = 0;
  }
  // winners by rank
  if (r > 0)
    for (int e = threadIdx.x; e < m; e += blockDim.x)
      if (rank[e] < r) o.byrank[rank[e]] = e;
  __syncthreads();
  int32_t R[kFsMaxLevels];
  for (int l = 0; l < g.L; ++l) {
    if (threadIdx.x == 0) s_carry = 0;
    __syncthreads();
    for (int base = 0; base < r; base += 1024) {
      const int p = base + threadIdx.x;
      int32_t f = 0;
      if (p < r) f = fs_level(g, level, fs_src(g, o.tk[o.byrank[p]])) == l ? 1 : 0;
      int32_t ex, agg;
      Scan(ts).ExclusiveSum(f, ex, agg);
      if (f) rank[g.n + p] = s_carry + ex;  // position among level-l winners (scratch after ranks)
      __syncthreads();
      if (threadIdx.x == 0) s_carry += agg;
      __syncthreads();
    }
    R[l] = s_carry;
    __syncthreads();
  }
  int32_t F[kFsMaxLevels];
  int32_t run = 0;
  for (int l = 0; l < g.L; ++l) {
    F[l] = run;
    run += info->C[l] + R[l];
  }
  for (int p = threadIdx.x; p < r; p += blockDim.x) {
    const int32_t e = o.byrank[p];
    const uint64_t key = o.tk[e];
    const int32_t l = fs_level(g, level, fs_src(g, key));
    fs_emit(g, o, ia, key, o.ti[e], list + F[l] + info->C[l] + rank[g.n + p], out, false);
  }
  const int64_t filled = r == info->r ? info->count : run;
  for (int64_t p = filled + threadIdx.x; p < g.k; p += blockDim.x) {
    out.s[out.rank][list + p] = 0;
    out.d[out.rank][list + p] = 0;
    out.w[out.rank][list + p] = 0.0f;
    out.g[out.rank][list + p] = 0;
  }
  if (threadIdx.x == 0)
    for (int l = 0; l < g.L; ++l) {
      info->R[l] = R[l];
      info->F[l] = F[l];
    }
}

// The full bins of at most kFsWarpCap members, one warp per (level, bin)
// pair: the bin's keys in the warp's shared memory, each lane ranking a
// quarter of them against all (broadcast reads), then emitting them at their
// final position. Eight bins are in flight per CTA (a CTA per bin would
// take them one after another, each a chain of loads and barriers).
constexpr int kFsWarpCap = 512;
constexpr int kFsWarps = kFsThreads / 32;
constexpr int kFsLaneKeys = 4;
__global__ void __launch_bounds__(kFsThreads) fs_bins_warp_kernel(FsGeom g, InitArgs ia, FsScratch o, FsOut out) {
  __shared__ uint64_t keys_s[kFsWarps][kFsWarpCap];
  const FsInfo *info = o.info;
  const int32_t tb = info->tb < g.nb ? info->tb : g.nb;
  const int64_t pairs = static_cast<int64_t>(g.L) * tb;
  const int64_t list = fs_list_base(out, g.k);
  const int32_t world = out.world > 1 ? out.world : 1, me = out.world > 1 ? out.rank : 0;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint64_t *ks = keys_s[w];
  bool stored = false;
  // this rank's pairs: q = me, me + world, ...
  for (int64_t j = static_cast<int64_t>(blockIdx.x) * kFsWarps + w; j * world + me < pairs;
       j += static_cast<int64_t>(gridDim.x) * kFsWarps) {
    const int64_t q = j * world + me;
    const int32_t l = static_cast<int32_t>(q / tb), b = static_cast<int32_t>(q % tb);
    const int32_t m = static_cast<int32_t>(o.hist[fs_hidx(static_cast<int64_t>(l) * g.nb + b)]);
    if (m == 0 || m > kFsWarpCap) continue;  // larger bins: fs_bins_kernel
    const uint32_t t0 = o.toff[l * g.nb + b];
    for (int e = lane; e < m; e += 32) ks[e] = o.bk[t0 + e];
    __syncwarp();
    const int64_t base = list + static_cast<int64_t>(info->F[l]) + (t0 - info->T[l]);
    // each lane ranks up to kFsLaneKeys of the bin's keys at once: one
    // shared-memory read of key f serves all of them
    for (int e0 = lane; e0 < m; e0 += 32 * kFsLaneKeys) {
      uint64_t ke[kFsLaneKeys];
      int32_t r[kFsLaneKeys];
#pragma unroll
      for (int i = 0; i < kFsLaneKeys; ++i) {
        const int e = e0 + 32 * i;
        ke[i] = e < m ? ks[e] : ~0ull;  // the keys are unique: a padding key is never emitted
        r[i] = 0;
      }
      for (int f = 0; f < m; ++f) {
        const uint64_t kf = ks[f];
#pragma unroll
        for (int i = 0; i < kFsLaneKeys; ++i) r[i] += kf < ke[i] ? 1 : 0;
      }
#pragma unroll
      for (int i = 0; i < kFsLaneKeys; ++i) {
        const int e = e0 + 32 * i;
        if (e < m) {
          fs_emit(g, o, ia, ke[i], o.bi[t0 + e], base + r[i], out, true);
          stored = true;
        }
      }
    }
    __syncwarp();
  }
  // the peers' stores are made visible before the kernel ends (a later
  // release on this GPU's stream publishes them); a thread that stored
  // nothing skips the system-wide fence
  if (world > 1 && stored) __threadfence_system();
}

// The full bins larger than a warp's share, each (level, bin) pair ranked
// by a CTA and emitted at its final position.
__global__ void __launch_bounds__(kFsThreads) fs_bins_kernel(FsGeom g, InitArgs ia, FsScratch o, FsOut out,
                                                             int32_t *rank_scratch, int32_t *status) {
  __shared__ uint64_t keys_s[kFsRankCap];
  const FsInfo *info = o.info;
  const int32_t tb = info->tb < g.nb ? info->tb : g.nb;
  const int64_t pairs = static_cast<int64_t>(g.L) * tb;
  const int64_t list = fs_list_base(out, g.k);
  const int32_t world = out.world > 1 ? out.world : 1, me = out.world > 1 ? out.rank : 0;
  bool stored = false;
  for (int64_t j = blockIdx.x; j * world + me < pairs; j += gridDim.x) {
    const int64_t q = j * world + me;
    const int32_t l = static_cast<int32_t>(q / tb), b = static_cast<int32_t>(q % tb);
    const int32_t m = static_cast<int32_t>(o.hist[fs_hidx(static_cast<int64_t>(l) * g.nb + b)]);
    if (m <= kFsWarpCap) continue;  // fs_bins_warp_kernel's
    const uint32_t t0 = o.toff[l * g.nb + b];
    int32_t *rank = rank_scratch + t0;
    if (!fs_rank(o.bk + t0, m, keys_s, rank)) {
      if (threadIdx.x == 0 && status) atomicOr(status, 1);
      continue;
    }
    const int64_t base = list + static_cast<int64_t>(info->F[l]) + (t0 - info->T[l]);
    for (int e = threadIdx.x; e < m; e += blockDim.x) {
      fs_emit(g, o, ia, o.bk[t0 + e], o.bi[t0 + e], base + rank[e], out, true);
      stored = true;
    }
    __syncthreads();
  }
  if (world > 1 && stored) __threadfence_system();
}

static int fs_geom(int32_t num_units, int64_t k, int32_t num_levels, int32_t score_kind, FsGeom *g) {
  g->n = num_units;
  g->k = k;
  g->L = num_levels;
  g->src_bits = bits_for(num_units);
  g->score_bits = score_kind == PXB_SCORE_UNIFORM ? 24 : 8;
  g->key_bits = 1 + g->score_bits + g->src_bits;
  int bb = 1;
  while (bb < kFsMaxBinBits && (int64_t(num_units) >> bb) > 128) ++bb;  // ~256 valid candidates per bin
  g->bin_bits = bb < g->key_bits ? bb : g->key_bits;
  g->nb = 1 << g->bin_bits;
  return g->key_bits <= 64 ? PXB_OK : PXB_EINVAL;
}

static void fs_layout(const FsGeom &g, char *base, FsScratch *o) {
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t at = off;
    off = align_up(off + (bytes ? bytes : 1), 256);
    return base ? base + at : nullptr;
  };
  const int64_t n = g.n, kk = g.k > 0 ? g.k : 1, hb = int64_t(g.L) * g.nb;
  o->keys = reinterpret_cast<uint64_t *>(take(n * 8));
  o->dst = reinterpret_cast<int32_t *>(take(n * 4));
  o->tk = reinterpret_cast<uint64_t *>(take(n * 8));
  o->ti = reinterpret_cast<int32_t *>(take(n * 4 * 3));  // members, their ranks, level positions
  o->bk = reinterpret_cast<uint64_t *>(take(kk * 8));
  o->bi = reinterpret_cast<int32_t *>(take(kk * 4 * 2));  // indices, then ranks
  o->byrank = reinterpret_cast<int32_t *>(take(n * 4));
  o->hist = reinterpret_cast<uint32_t *>(take(hb * 4 * kFsHistStride));
  o->toff = reinterpret_cast<uint32_t *>(take(hb * 4));
  o->info = reinterpret_cast<FsInfo *>(take(sizeof(FsInfo)));
  o->total = off;
}

// ---------------------------------------------------------------------------
// the global and per-connection proposers (src/plastax/phases.py:3766-3810,
// :3921-4039) and the per-source-level cap (:4324-4487)
// ---------------------------------------------------------------------------
// Global: proposal j at key 0: src [sub 0], dst [sub 1], score [sub 2];
// candidate index j.
__global__ void propose_global_kernel(ProposeArgs a, int32_t src_lo, int32_t src_n, int32_t *__restrict__ src_out,
                                      int32_t *__restrict__ dst_out, float *__restrict__ score_out) {
  const uint64_t keyed_hi = keyed_hi_of(a);
  const uint64_t seed = keyed_hi << 32;
  for (int64_t c = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; c < a.proposals;
       c += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint32_t j = static_cast<uint32_t>(c);
    int32_t src = src_lo + static_cast<int32_t>(uniform_int(unit_float(site_draw(seed, j, 0)), src_n));
    int32_t dst = a.dst_lo + static_cast<int32_t>(uniform_int(unit_float(site_draw(seed, j, 1)), a.dst_n));
    float score = proposal_score(a, seed, j, 2, src, dst);
    apply_window(a, src, dst, score, true);
    src_out[c] = src;
    dst_out[c] = dst;
    score_out[c] = score;
  }
}

// Live connections ranked ascending by (src, dst, slot), dead slots after
// them: the packed key of slot s (dead: every bit set), its slot as value.
__global__ void conn_key_kernel(int64_t cap, const int32_t *__restrict__ from, const int32_t *__restrict__ to,
                                const uint8_t *__restrict__ dead, int id_bits, uint64_t *__restrict__ key,
                                int32_t *__restrict__ val) {
  const uint64_t all = (id_bits >= 32) ? ~0ull : ((uint64_t(1) << (2 * id_bits)) - 1);
  for (int64_t s = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; s < cap;
       s += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    key[s] = dead[s] ? all
                     : ((static_cast<uint64_t>(static_cast<uint32_t>(from[s])) << id_bits) |
                        static_cast<uint32_t>(to[s]));
    val[s] = static_cast<int32_t>(s);
  }
}

// The run start of each sorted position (max-scan input): p where the key
// changes, 0 elsewhere.
__global__ void run_start_kernel(int64_t cap, const uint64_t *__restrict__ key, int32_t *__restrict__ start) {
  for (int64_t p = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; p < cap;
       p += static_cast<int64_t>(gridDim.x) * blockDim.x)
    start[p] = (p == 0 || key[p] != key[p - 1]) ? static_cast<int32_t>(p) : 0;
}

// Proposals of the connection at rank r = c / P: src = its source, dst
// [sub 0], score [sub 1] at key philox32((src << 32) | dst, occurrence); a
// dead proposer's candidates are vetoed.
__global__ void propose_per_conn_kernel(ProposeArgs a, int64_t cap, const int32_t *__restrict__ from,
                                        const int32_t *__restrict__ to, const uint8_t *__restrict__ dead,
                                        const int32_t *__restrict__ rank_slot, const int32_t *__restrict__ run_start,
                                        int32_t *__restrict__ src_out, int32_t *__restrict__ dst_out,
                                        float *__restrict__ score_out) {
  const uint64_t keyed_hi = keyed_hi_of(a);
  const int64_t total = cap * a.proposals;
  for (int64_t c = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; c < total;
       c += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = c / a.proposals;
    const uint32_t j = static_cast<uint32_t>(c - r * a.proposals);
    const int32_t slot = rank_slot[r];
    const uint32_t occ = static_cast<uint32_t>(r - run_start[r]);
    const int32_t cs = from[slot], cd = to[slot];
    const uint32_t key = philox32((static_cast<uint64_t>(static_cast<uint32_t>(cs)) << 32) | static_cast<uint32_t>(cd),
                                  occ);
    const uint64_t seed = (keyed_hi << 32) | key;
    int32_t src = cs;
    int32_t dst = a.dst_lo + static_cast<int32_t>(uniform_int(unit_float(site_draw(seed, j, 0)), a.dst_n));
    float score = proposal_score(a, seed, j, 1, src, dst);
    apply_window(a, src, dst, score, dead[slot] == 0);
    src_out[c] = src;
    dst_out[c] = dst;
    score_out[c] = score;
  }
}

// The per-level cap over a level-major ordered list (pxb_select_step with
// k = n): the first k of every level's run, listed levels ascending.
__global__ void level_bounds_kernel(int64_t n, const int32_t *__restrict__ idx, const int32_t *__restrict__ src,
                                    const int32_t *__restrict__ level, int32_t num_levels, int32_t *__restrict__ first,
                                    int32_t *__restrict__ end) {
  for (int64_t p = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; p < n;
       p += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    auto lv = [&](int64_t q) {
      const int32_t l = level[src[idx[q]]];
      return l < 0 ? 0 : (l >= num_levels ? num_levels - 1 : l);
    };
    const int32_t l = lv(p);
    if (p == 0 || lv(p - 1) != l) first[l] = static_cast<int32_t>(p);
    if (p == n - 1 || lv(p + 1) != l) end[l] = static_cast<int32_t>(p + 1);
  }
}

__global__ void level_caps_kernel(int32_t num_levels, int64_t k, const int32_t *__restrict__ first,
                                  const int32_t *__restrict__ end, int32_t *__restrict__ off, int32_t *count) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  int32_t acc = 0;
  for (int l = 0; l < num_levels; ++l) {
    off[l] = acc;
    const int64_t m = end[l] - first[l];
    acc += static_cast<int32_t>(m < k ? m : k);
  }
  off[num_levels] = acc;
  if (count) *count = acc;
}

__global__ void level_cap_compact_kernel(int64_t n, const int32_t *__restrict__ idx, const int32_t *__restrict__ src,
                                         const int32_t *__restrict__ level, int32_t num_levels, int64_t k,
                                         const int32_t *__restrict__ first, const int32_t *__restrict__ off,
                                         int32_t *__restrict__ out) {
  for (int64_t p = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; p < n;
       p += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int32_t l = level[src[idx[p]]];
    l = l < 0 ? 0 : (l >= num_levels ? num_levels - 1 : l);
    const int64_t r = p - first[l];
    if (r < k) out[off[l] + r] = idx[p];
  }
}

struct ConnRankScratch {
  uint64_t *key_in, *key_out;
  int32_t *val_in, *val_out, *start_in, *start_out;
  void *cub_tmp;
  size_t cub_bytes, total;
};

static int conn_rank_scratch(int64_t cap, int id_bits, char *base, ConnRankScratch *o) {
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t at = off;
    off = align_up(off + (bytes ? bytes : 1), 256);
    return base ? base + at : nullptr;
  };
  const int64_t c = cap > 0 ? cap : 1;
  o->key_in = reinterpret_cast<uint64_t *>(take(c * 8));
  o->key_out = reinterpret_cast<uint64_t *>(take(c * 8));
  o->val_in = reinterpret_cast<int32_t *>(take(c * 4));
  o->val_out = reinterpret_cast<int32_t *>(take(c * 4));
  o->start_in = reinterpret_cast<int32_t *>(take(c * 4));
  o->start_out = reinterpret_cast<int32_t *>(take(c * 4));
  size_t t1 = 0, t2 = 0;
  const int bits = 2 * id_bits < 64 ? 2 * id_bits : 64;
  if (cub::DeviceRadixSort::SortPairs(nullptr, t1, o->key_in, o->key_out, o->val_in, o->val_out,
                                      static_cast<int>(c), 0, bits) != cudaSuccess)
    return PXB_ECUDA;
  if (cub::DeviceScan::InclusiveScan(nullptr, t2, o->start_in, o->start_out, cub::Max(), static_cast<int>(c)) !=
      cudaSuccess)
    return PXB_ECUDA;
  o->cub_bytes = t1 > t2 ? t1 : t2;
  o->cub_tmp = take(o->cub_bytes);
  o->total = off;
  return PXB_OK;
}

// ---------------------------------------------------------------------------
// resort compaction order (src/plastax/topo.py:303-452): a stable order of a
// bucket's slots by dead * num_units + from_id
// ---------------------------------------------------------------------------
__global__ void resort_key_kernel(int64_t cap, const uint8_t *__restrict__ dead, const int32_t *__restrict__ from,
                                  int32_t num_units, uint32_t *__restrict__ key, int32_t *__restrict__ val) {
  for (int64_t s = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; s < cap;
       s += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int32_t f = from[s];
    f = f < 0 ? 0 : (f >= num_units ? num_units - 1 : f);
    key[s] = (dead[s] ? static_cast<uint32_t>(num_units) : 0u) + static_cast<uint32_t>(f);
    val[s] = static_cast<int32_t>(s);
  }
}

}  // namespace pxb

extern "C" int pxb_total_order(int64_t n, const float *score, const int32_t *src, const int32_t *dst,
                               int32_t id_bound, int32_t *perm_out, void *scratch, size_t scratch_bytes,
                               void *stream) {
  return total_order_impl("pxb_total_order", n, score, src, dst, id_bound, perm_out, scratch, scratch_bytes,
                          as_stream(stream));
}

extern "C" int pxb_select_step_scratch_bytes(int64_t n, int64_t k, size_t *bytes) {
  PXB_REQUIRE(bytes != nullptr, "pxb_select_step_scratch_bytes: bytes is NULL");
  PXB_REQUIRE(n >= 0 && k >= 0, "pxb_select_step_scratch_bytes: negative sizes");
  const int64_t kk = k < n ? k : n;
  SelectScratch o;
  if (select_scratch(kk, nullptr, &o, nullptr) != PXB_OK) {
    set_error("pxb_select_step_scratch_bytes: CUB size query failed");
    return PXB_ECUDA;
  }
  *bytes = o.total;
  return PXB_OK;
}

extern "C" int pxb_select_step(int64_t n, const int32_t *perm, const float *score, const int32_t *src,
                               const int32_t *level, int32_t num_levels, int64_t k, int32_t *win_idx,
                               int32_t *win_count, void *scratch, size_t scratch_bytes, void *stream) {
  (void)score;
  PXB_REQUIRE(n >= 0 && k >= 0 && n < (int64_t(1) << 31), "pxb_select_step: sizes out of range");
  const int64_t kk = k < n ? k : n;
  cudaStream_t st = as_stream(stream);
  if (win_count != nullptr) {
    set_i32_kernel<<<1, 1, 0, st>>>(win_count, static_cast<int32_t>(kk));
    PXB_LAUNCHED("set_i32_kernel");
  }
  if (kk == 0) return PXB_OK;
  PXB_REQUIRE(perm && src && level && win_idx && scratch, "pxb_select_step: a pointer is NULL");
  SelectScratch o;
  if (select_scratch(kk, static_cast<char *>(scratch), &o, win_idx) != PXB_OK) {
    set_error("pxb_select_step: CUB size query failed");
    return PXB_ECUDA;
  }
  PXB_REQUIRE(o.total <= scratch_bytes, "pxb_select_step: scratch has %zu bytes, needs %zu", scratch_bytes,
              o.total);
  PXB_REQUIRE(num_levels >= 1, "pxb_select_step: num_levels must be >= 1");
  winner_level_kernel<<<grid_for(kk, 256, 8), 256, 0, st>>>(kk, perm, src, level, o.key_in, o.val_in);
  PXB_LAUNCHED("winner_level_kernel");
  int key_bits = 1;
  while (key_bits < 32 && (int64_t(1) << key_bits) < num_levels) ++key_bits;
  size_t tb = o.cub_bytes;
  PXB_CUDA(cub::DeviceRadixSort::SortPairs(o.cub_tmp, tb, o.key_in, o.key_out, o.val_in, win_idx,
                                           static_cast<int>(kk), 0, key_bits, st));
  return PXB_OK;
}

extern "C" int pxb_gather_winners(int64_t k, int64_t count, const int32_t *win_idx, const int32_t *src,
                                  const int32_t *dst, const float *score, int32_t init_kind, float init_a,
                                  float init_b, uint32_t init_salt, int32_t *src_out, int32_t *dst_out,
                                  float *weight_out, uint8_t *growable_out, void *stream) {
  PXB_REQUIRE(k >= 0 && count >= 0 && count <= k, "pxb_gather_winners: sizes out of range");
  PXB_REQUIRE(init_kind >= 0 && init_kind <= 2, "pxb_gather_winners: unknown init kind %d", init_kind);
  if (k == 0) return PXB_OK;
  PXB_REQUIRE(src_out && dst_out && weight_out && growable_out, "pxb_gather_winners: an output is NULL");
  PXB_REQUIRE(count == 0 || (win_idx && src && dst && score), "pxb_gather_winners: an input is NULL");
  InitArgs ia{init_kind, init_a, init_b, init_salt};
  gather_winners_kernel<<<grid_for(k, 256, 8), 256, 0, as_stream(stream)>>>(
      k, count, win_idx, src, dst, score, ia, src_out, dst_out, weight_out, growable_out);
  PXB_LAUNCHED("gather_winners_kernel");
  return PXB_OK;
}

extern "C" int pxb_select_unique_scratch_bytes(int32_t num_units, int64_t k, int32_t num_levels, int32_t score_kind,
                                               size_t *bytes) {
  PXB_REQUIRE(bytes && num_units >= 1 && k >= 0 && num_levels >= 1 && num_levels <= kFsMaxLevels,
              "pxb_select_unique_scratch_bytes: bad arguments");
  PXB_REQUIRE(score_kind == PXB_SCORE_UNIFORM || score_kind == PXB_SCORE_UNIFORM_Q256,
              "pxb_select_unique_scratch_bytes: the score must be uniform or uniform_q256");
  FsGeom g;
  if (fs_geom(num_units, k, num_levels, score_kind, &g) != PXB_OK) {
    set_error("pxb_select_unique_scratch_bytes: %d units need too many key bits", num_units);
    return PXB_EINVAL;
  }
  FsScratch o;
  fs_layout(g, nullptr, &o);
  *bytes = o.total;
  return PXB_OK;
}

// The fused selection's launches (both entry points): the proposals and
// threshold bin on every rank, the full bins this rank ranks, the winners
// into `out`.
static int fs_run(const char *fn, int32_t num_units, uint64_t network_seed, int32_t step, int32_t dst_lo,
                  int32_t dst_n, int32_t score_kind, const int32_t *level, const uint8_t *pruned,
                  int32_t max_level_gap, int32_t direction, int32_t allow_self_loops, int32_t src_level_bound,
                  const int32_t *step_dev, int64_t k, int32_t num_levels, int32_t init_kind, float init_a,
                  float init_b, uint32_t init_salt, FsOut out, int32_t *status, void *scratch,
                  size_t scratch_bytes, void *stream) {
  PXB_REQUIRE(num_units >= 1 && k >= 0, "%s: bad sizes", fn);
  PXB_REQUIRE(num_levels >= 1 && num_levels <= kFsMaxLevels, "%s: num_levels %d not in [1, %d]", fn, num_levels,
              kFsMaxLevels);
  PXB_REQUIRE(score_kind == PXB_SCORE_UNIFORM || score_kind == PXB_SCORE_UNIFORM_Q256,
              "%s: the score must be uniform or uniform_q256", fn);
  PXB_REQUIRE(dst_n >= 1 && dst_lo >= 0 && int64_t(dst_lo) + dst_n <= num_units,
              "%s: destinations [%d, %lld) exceed the %d units", fn, dst_lo,
              static_cast<long long>(dst_lo) + dst_n, num_units);
  PXB_REQUIRE(init_kind >= 0 && init_kind <= 2, "%s: unknown init kind %d", fn, init_kind);
  if (k == 0) return PXB_OK;
  PXB_REQUIRE(level && scratch, "%s: a pointer is NULL", fn);
  for (int q = 0; q < out.world; ++q)
    PXB_REQUIRE(out.s[q] && out.d[q] && out.w[q] && out.g[q], "%s: rank %d's output column is NULL", fn, q);
  FsGeom g;
  if (fs_geom(num_units, k, num_levels, score_kind, &g) != PXB_OK) {
    set_error("%s: %d units need too many key bits", fn, num_units);
    return PXB_EINVAL;
  }
  FsScratch o;
  fs_layout(g, static_cast<char *>(scratch), &o);
  PXB_REQUIRE(o.total <= scratch_bytes, "%s: scratch has %zu bytes, needs %zu", fn, scratch_bytes, o.total);
  ProposeArgs a{num_units, 1, 0, network_seed, step_dev, dst_lo, dst_n, score_kind, nullptr, nullptr, level,
                pruned, max_level_gap, direction, allow_self_loops, -1, src_level_bound};
  if (step_dev == nullptr) a.keyed_hi = philox32(network_seed, (static_cast<uint64_t>(static_cast<uint32_t>(step)) << 8) | 1u);
  InitArgs ia{init_kind, init_a, init_b, init_salt};
  out.step = step;
  out.step_dev = step_dev;
  cudaStream_t st = as_stream(stream);
  PXB_CUDA(cudaMemsetAsync(o.hist, 0, size_t(g.L) * g.nb * 4 * kFsHistStride, st));
  const int grid = grid_for(num_units, kFsThreads, 8);
  fs_propose_kernel<<<grid, kFsThreads, 0, st>>>(a, g, o);
  PXB_LAUNCHED("fs_propose_kernel");
  fs_threshold_kernel<<<1, 1024, 0, st>>>(g, o);
  PXB_LAUNCHED("fs_threshold_kernel");
  fs_scatter_kernel<<<grid, kFsThreads, 0, st>>>(g, level, o, out.rank, out.world);
  PXB_LAUNCHED("fs_scatter_kernel");
  fs_threshold_bin_kernel<<<1, 1024, 0, st>>>(g, level, ia, o, out, status);
  PXB_LAUNCHED("fs_threshold_bin_kernel");
  fs_bins_warp_kernel<<<sm_count() * 8, kFsThreads, 0, st>>>(g, ia, o, out);
  PXB_LAUNCHED("fs_bins_warp_kernel");
  fs_bins_kernel<<<sm_count() * 2, kFsThreads, 0, st>>>(g, ia, o, out, o.bi + (g.k > 0 ? g.k : 1), status);
  PXB_LAUNCHED("fs_bins_kernel");
  return PXB_OK;
}

extern "C" int pxb_propose_select_unique(int32_t num_units, uint64_t network_seed, int32_t step, int32_t dst_lo,
                                         int32_t dst_n, int32_t score_kind, const int32_t *level,
                                         const uint8_t *pruned, int32_t max_level_gap, int32_t direction,
                                         int32_t allow_self_loops, int32_t src_level_bound,
                                         const int32_t *step_dev, int64_t k, int32_t num_levels, int32_t init_kind,
                                         float init_a, float init_b, uint32_t init_salt, int32_t *src_out,
                                         int32_t *dst_out, float *weight_out, uint8_t *growable_out,
                                         int32_t *status, void *scratch, size_t scratch_bytes, void *stream) {
  FsOut out{};
  out.rank = 0;
  out.world = 1;
  out.blocks = 1;
  out.s[0] = src_out;
  out.d[0] = dst_out;
  out.w[0] = weight_out;
  out.g[0] = growable_out;
  return fs_run("pxb_propose_select_unique", num_units, network_seed, step, dst_lo, dst_n, score_kind, level,
                pruned, max_level_gap, direction, allow_self_loops, src_level_bound, step_dev, k, num_levels,
                init_kind, init_a, init_b, init_salt, out, status, scratch, scratch_bytes, stream);
}

extern "C" int pxb_propose_select_unique_sharded(int32_t num_units, uint64_t network_seed, int32_t step,
                                                 int32_t dst_lo, int32_t dst_n, int32_t score_kind,
                                                 const int32_t *level, const uint8_t *pruned, int32_t max_level_gap,
                                                 int32_t direction, int32_t allow_self_loops,
                                                 int32_t src_level_bound, const int32_t *step_dev, int64_t k,
                                                 int32_t num_levels, int32_t init_kind, float init_a, float init_b,
                                                 uint32_t init_salt, const pxb_select_shard *shard, int32_t *status,
                                                 void *scratch, size_t scratch_bytes, void *stream) {
  PXB_REQUIRE(shard != nullptr, "pxb_propose_select_unique_sharded: shard is NULL");
  PXB_REQUIRE(shard->world >= 1 && shard->world <= kSelMaxWorld && shard->rank >= 0 && shard->rank < shard->world,
              "pxb_propose_select_unique_sharded: rank %d of world %d (at most %d ranks)", shard->rank, shard->world,
              kSelMaxWorld);
  PXB_REQUIRE(shard->blocks >= 1, "pxb_propose_select_unique_sharded: blocks %d < 1", shard->blocks);
  FsOut out{};
  out.rank = shard->rank;
  out.world = shard->world;
  out.blocks = shard->blocks;
  for (int q = 0; q < shard->world; ++q) {
    out.s[q] = shard->src_out[q];
    out.d[q] = shard->dst_out[q];
    out.w[q] = shard->weight_out[q];
    out.g[q] = shard->growable_out[q];
  }
  return fs_run("pxb_propose_select_unique_sharded", num_units, network_seed, step, dst_lo, dst_n, score_kind,
                level, pruned, max_level_gap, direction, allow_self_loops, src_level_bound, step_dev, k,
                num_levels, init_kind, init_a, init_b, init_salt, out, status, scratch, scratch_bytes, stream);
}

__global__ void select_take_kernel(int64_t k, int32_t blocks, const int32_t *__restrict__ step_dev,
                                   const int32_t *__restrict__ s_col, const int32_t *__restrict__ d_col,
                                   const float *__restrict__ w_col, const uint8_t *__restrict__ g_col,
                                   int32_t *__restrict__ s_out, int32_t *__restrict__ d_out, float *__restrict__ w_out,
                                   uint8_t *__restrict__ g_out) {
  int64_t base = 0;
  if (blocks > 1) {
    const int32_t st = *step_dev;
    base = static_cast<int64_t>(((st % blocks) + blocks) % blocks) * k;
  }
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < k;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    s_out[i] = s_col[base + i];
    d_out[i] = d_col[base + i];
    w_out[i] = w_col[base + i];
    g_out[i] = g_col[base + i];
  }
}

extern "C" int pxb_select_take(int64_t k, int32_t blocks, const int32_t *step_dev, const int32_t *src_col,
                               const int32_t *dst_col, const float *weight_col, const uint8_t *growable_col,
                               int32_t *src_out, int32_t *dst_out, float *weight_out, uint8_t *growable_out,
                               void *stream) {
  PXB_REQUIRE(k >= 0 && blocks >= 1, "pxb_select_take: bad sizes");
  if (k == 0) return PXB_OK;
  PXB_REQUIRE(blocks == 1 || step_dev != nullptr, "pxb_select_take: %d lists need step_dev", blocks);
  PXB_REQUIRE(src_col && dst_col && weight_col && growable_col && src_out && dst_out && weight_out && growable_out,
              "pxb_select_take: a pointer is NULL");
  select_take_kernel<<<grid_for(k, 256, 8), 256, 0, as_stream(stream)>>>(
      k, blocks, step_dev, src_col, dst_col, weight_col, growable_col, src_out, dst_out, weight_out, growable_out);
  PXB_LAUNCHED("select_take_kernel");
  return PXB_OK;
}

static ProposeArgs propose_args(int32_t num_units, int32_t proposals, uint64_t network_seed, int32_t step,
                                const int32_t *step_dev, int32_t dst_lo, int32_t dst_n, int32_t score_kind,
                                const float *grad, const float *act, const int32_t *level, const uint8_t *pruned,
                                int32_t max_level_gap, int32_t direction, int32_t allow_self_loops,
                                int32_t bucket_level, int32_t src_level_bound) {
  ProposeArgs a{num_units, proposals, 0, network_seed, step_dev, dst_lo, dst_n, score_kind, grad, act, level,
                pruned, max_level_gap, direction, allow_self_loops, bucket_level, src_level_bound};
  if (step_dev == nullptr)
    a.keyed_hi = philox32(network_seed, (static_cast<uint64_t>(static_cast<uint32_t>(step)) << 8) | 1u);
  return a;
}

extern "C" int pxb_propose_global(int32_t proposals, uint64_t network_seed, int32_t step, int32_t num_units,
                                  int32_t src_lo, int32_t src_n, int32_t dst_lo, int32_t dst_n, int32_t score_kind,
                                  const float *grad, const float *act, const int32_t *level, const uint8_t *pruned,
                                  int32_t max_level_gap, int32_t direction, int32_t allow_self_loops,
                                  int32_t bucket_level, int32_t src_level_bound, const int32_t *step_dev,
                                  int32_t *src_out, int32_t *dst_out, float *score_out, void *stream) {
  PXB_REQUIRE(proposals >= 0 && num_units >= 1 && src_n >= 1 && dst_n >= 1, "pxb_propose_global: bad sizes");
  PXB_REQUIRE(score_kind >= 0 && score_kind <= 2, "pxb_propose_global: unknown score kind %d", score_kind);
  if (proposals == 0) return PXB_OK;
  PXB_REQUIRE(level && src_out && dst_out && score_out, "pxb_propose_global: a pointer is NULL");
  PXB_REQUIRE(score_kind != PXB_SCORE_GRAD_ACT || (grad && act), "pxb_propose_global: grad_act needs grad and act");
  const ProposeArgs a = propose_args(num_units, proposals, network_seed, step, step_dev, dst_lo, dst_n, score_kind,
                                     grad, act, level, pruned, max_level_gap, direction, allow_self_loops, bucket_level,
                                     src_level_bound);
  propose_global_kernel<<<grid_for(proposals, 256, 4), 256, 0, as_stream(stream)>>>(a, src_lo, src_n, src_out,
                                                                                      dst_out, score_out);
  PXB_LAUNCHED("propose_global_kernel");
  return PXB_OK;
}

extern "C" int pxb_conn_rank_scratch_bytes(int64_t cap, int32_t num_units, size_t *bytes) {
  PXB_REQUIRE(bytes && cap >= 0 && cap < (int64_t(1) << 31) && num_units >= 1,
              "pxb_conn_rank_scratch_bytes: bad arguments");
  ConnRankScratch o;
  if (conn_rank_scratch(cap, bits_for(int64_t(num_units) + 1), nullptr, &o) != PXB_OK) {
    set_error("pxb_conn_rank_scratch_bytes: CUB size query failed");
    return PXB_ECUDA;
  }
  *bytes = o.total;
  return PXB_OK;
}

extern "C" int pxb_propose_per_conn(int64_t cap, const int32_t *from_id, const int32_t *to_id, const uint8_t *dead,
                                    int32_t proposals, uint64_t network_seed, int32_t step, int32_t num_units,
                                    int32_t dst_lo, int32_t dst_n, int32_t score_kind, const float *grad,
                                    const float *act, const int32_t *level, const uint8_t *pruned,
                                    int32_t max_level_gap, int32_t direction, int32_t allow_self_loops,
                                    int32_t bucket_level, int32_t src_level_bound, const int32_t *step_dev,
                                    int32_t *src_out, int32_t *dst_out, float *score_out, void *scratch,
                                    size_t scratch_bytes, void *stream) {
  PXB_REQUIRE(cap >= 0 && cap < (int64_t(1) << 31) && proposals >= 0 && num_units >= 1 && dst_n >= 1,
              "pxb_propose_per_conn: bad sizes");
  PXB_REQUIRE(cap * int64_t(proposals) < (int64_t(1) << 31), "pxb_propose_per_conn: too many candidates");
  PXB_REQUIRE(score_kind >= 0 && score_kind <= 2, "pxb_propose_per_conn: unknown score kind %d", score_kind);
  if (cap == 0 || proposals == 0) return PXB_OK;
  PXB_REQUIRE(from_id && to_id && dead && level && src_out && dst_out && score_out && scratch,
              "pxb_propose_per_conn: a pointer is NULL");
  PXB_REQUIRE(score_kind != PXB_SCORE_GRAD_ACT || (grad && act), "pxb_propose_per_conn: grad_act needs grad and act");
  const int id_bits = bits_for(int64_t(num_units) + 1);
  ConnRankScratch o;
  if (conn_rank_scratch(cap, id_bits, static_cast<char *>(scratch), &o) != PXB_OK) {
    set_error("pxb_propose_per_conn: CUB size query failed");
    return PXB_ECUDA;
  }
  PXB_REQUIRE(o.total <= scratch_bytes, "pxb_propose_per_conn: scratch has %zu bytes, needs %zu", scratch_bytes,
              o.total);
  cudaStream_t st = as_stream(stream);
  const int grid = grid_for(cap, 256, 8);
  conn_key_kernel<<<grid, 256, 0, st>>>(cap, from_id, to_id, dead, id_bits, o.key_in, o.val_in);
  PXB_LAUNCHED("conn_key_kernel");
  size_t tb = o.cub_bytes;
  const int bits = 2 * id_bits < 64 ? 2 * id_bits : 64;
  PXB_CUDA(cub::DeviceRadixSort::SortPairs(o.cub_tmp, tb, o.key_in, o.key_out, o.val_in, o.val_out,
                                           static_cast<int>(cap), 0, bits, st));
  run_start_kernel<<<grid, 256, 0, st>>>(cap, o.key_out, o.start_in);
  PXB_LAUNCHED("run_start_kernel");
  tb = o.cub_bytes;
  PXB_CUDA(cub::DeviceScan::InclusiveScan(o.cub_tmp, tb, o.start_in, o.start_out, cub::Max(), static_cast<int>(cap),
                                          st));
  const ProposeArgs a = propose_args(num_units, proposals, network_seed, step, step_dev, dst_lo, dst_n, score_kind,
                                     grad, act, level, pruned, max_level_gap, direction, allow_self_loops, bucket_level,
                                     src_level_bound);
  propose_per_conn_kernel<<<grid_for(cap * proposals, 256, 8), 256, 0, st>>>(
      a, cap, from_id, to_id, dead, o.val_out, o.start_out, src_out, dst_out, score_out);
  PXB_LAUNCHED("propose_per_conn_kernel");
  return PXB_OK;
}

extern "C" int pxb_cap_per_level(int64_t n, const int32_t *idx, const int32_t *src, const int32_t *level,
                                 int32_t num_levels, int64_t k, int32_t *out_idx, int32_t *out_count,
                                 int32_t *scratch, void *stream) {
  PXB_REQUIRE(n >= 0 && n < (int64_t(1) << 31) && k >= 0 && num_levels >= 1, "pxb_cap_per_level: bad sizes");
  PXB_REQUIRE(scratch && out_count, "pxb_cap_per_level: scratch / out_count is NULL");
  cudaStream_t st = as_stream(stream);
  int32_t *first = scratch, *end = scratch + num_levels, *off = scratch + 2 * num_levels;
  PXB_CUDA(cudaMemsetAsync(scratch, 0, sizeof(int32_t) * (3 * num_levels + 1), st));
  if (n > 0) {
    PXB_REQUIRE(idx && src && level && out_idx, "pxb_cap_per_level: a pointer is NULL");
    level_bounds_kernel<<<grid_for(n, 256, 8), 256, 0, st>>>(n, idx, src, level, num_levels, first, end);
    PXB_LAUNCHED("level_bounds_kernel");
  }
  level_caps_kernel<<<1, 32, 0, st>>>(num_levels, k, first, end, off, out_count);
  PXB_LAUNCHED("level_caps_kernel");
  if (n > 0) {
    level_cap_compact_kernel<<<grid_for(n, 256, 8), 256, 0, st>>>(n, idx, src, level, num_levels, k, first, off,
                                                                  out_idx);
    PXB_LAUNCHED("level_cap_compact_kernel");
  }
  return PXB_OK;
}

extern "C" int pxb_resort_order_scratch_bytes(int64_t cap, size_t *bytes) {
  PXB_REQUIRE(bytes && cap >= 0 && cap < (int64_t(1) << 31), "pxb_resort_order_scratch_bytes: bad arguments");
  const int64_t c = cap > 0 ? cap : 1;
  size_t t = 0;
  if (cub::DeviceRadixSort::SortPairs(nullptr, t, static_cast<uint32_t *>(nullptr), static_cast<uint32_t *>(nullptr),
                                      static_cast<int32_t *>(nullptr), static_cast<int32_t *>(nullptr),
                                      static_cast<int>(c), 0, 32) != cudaSuccess) {
    set_error("pxb_resort_order_scratch_bytes: CUB size query failed");
    return PXB_ECUDA;
  }
  *bytes = align_up(c * 4, 256) * 3 + align_up(t, 256);
  return PXB_OK;
}

extern "C" int pxb_resort_order(int64_t cap, const uint8_t *dead, const int32_t *from_id, int32_t num_units,
                                int32_t *perm_out, void *scratch, size_t scratch_bytes, void *stream) {
  PXB_REQUIRE(cap >= 0 && cap < (int64_t(1) << 31) && num_units >= 1 && num_units < (1 << 30),
              "pxb_resort_order: sizes out of range");
  if (cap == 0) return PXB_OK;
  PXB_REQUIRE(dead && from_id && perm_out && scratch, "pxb_resort_order: a pointer is NULL");
  size_t need = 0;
  int rc = pxb_resort_order_scratch_bytes(cap, &need);
  if (rc) return rc;
  PXB_REQUIRE(need <= scratch_bytes, "pxb_resort_order: scratch has %zu bytes, needs %zu", scratch_bytes, need);
  char *base = static_cast<char *>(scratch);
  const size_t col = align_up(cap * 4, 256);
  uint32_t *key_in = reinterpret_cast<uint32_t *>(base), *key_out = reinterpret_cast<uint32_t *>(base + col);
  int32_t *val_in = reinterpret_cast<int32_t *>(base + 2 * col);
  void *tmp = base + 3 * col;
  size_t tb = scratch_bytes - 3 * col;
  int bits = 1;
  while (bits < 32 && (int64_t(1) << bits) < 2 * int64_t(num_units)) ++bits;
  cudaStream_t st = as_stream(stream);
  resort_key_kernel<<<grid_for(cap, 256, 8), 256, 0, st>>>(cap, dead, from_id, num_units, key_in, val_in);
  PXB_LAUNCHED("resort_key_kernel");
  PXB_CUDA(cub::DeviceRadixSort::SortPairs(tmp, tb, key_in, key_out, val_in, perm_out, static_cast<int>(cap), 0, bits,
                                           st));
  return PXB_OK;
}

// ---------------------------------------------------------------------------
// ScoreAddConn candidates (src/plastax/phases.py:3640-3746, :4690-4790):
// the exhaustive grid, the importance shortlist and the per-level shortlists,
// each candidate scored by the rule's lowered pair score and passed through
// the validity window.
// ---------------------------------------------------------------------------
namespace pxb {

__device__ __forceinline__ int64_t floor_mod(int64_t x, int64_t m) {
  const int64_t r = x % m;
  return r < 0 ? r + m : r;
}

__device__ __forceinline__ float pair_score(const pxb_pair_score &f, int32_t src, int32_t dst) {
  switch (f.form) {
    case PXB_PAIR_ABS_PRODUCT:
      return fabsf(__fmul_rn(f.x_src[src], f.x_dst[dst]));
    case PXB_PAIR_PRODUCT:
      return __fmul_rn(f.x_src[src], f.x_dst[dst]);
    case PXB_PAIR_MODULAR: {
      const int64_t r = floor_mod(int64_t(f.a) * src + int64_t(f.b) * dst, f.m);
      return __fmul_rn(static_cast<float>(r - f.c), f.scale);
    }
    default: {  // PXB_PAIR_MODULAR_PREDICATE
      const int64_t r = floor_mod(int64_t(f.a) * src + int64_t(f.b) * dst, f.m);
      return r == f.c ? 0.0f : -__int_as_float(0x7f800000);
    }
  }
}

// Importance of unit i under the rule's lowered form; -inf for a pruned unit
// or one outside the mask (the per-level shortlist's source level or the
// level's destination window).
__global__ void unit_importance_kernel(int32_t n, pxb_pair_score f, const uint8_t *__restrict__ pruned,
                                       const int32_t *__restrict__ level, int32_t mask_kind, int32_t bucket,
                                       int32_t max_level_gap, int32_t direction, float *__restrict__ out) {
  for (int32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    float v;
    if (f.form == PXB_PAIR_ABS_PRODUCT) v = fabsf(f.x_src[i]);
    else if (f.form == PXB_PAIR_PRODUCT) v = f.x_src[i];
    else v = __fmul_rn(static_cast<float>(floor_mod(int64_t(f.a) * i, f.m) - f.c), f.scale);
    bool keep = pruned == nullptr || !pruned[i];
    if (mask_kind == 1) {
      keep = keep && level[i] == bucket;
    } else if (mask_kind == 2) {
      const int32_t ld = level[i], gap = ld > bucket ? ld - bucket : bucket - ld;
      keep = keep && gap <= max_level_gap;
      if (direction == 1) keep = keep && ld > bucket;
      else if (direction == 2) keep = keep && ld >= bucket;
    }
    out[i] = keep ? v : -__int_as_float(0x7f800000);
  }
}

// Candidate c of `grids` grids of rows x cols: grid g, row r, column q
// (row-major inside a grid, grids in order); src = row_ids[g * rows + r]
// (r itself without row_ids), dst likewise from col_ids.
__global__ void propose_grid_kernel(ProposeArgs a, int32_t grids, int32_t rows, int32_t cols,
                                    const int32_t *__restrict__ row_ids, const int32_t *__restrict__ col_ids,
                                    int32_t per_grid_bucket, pxb_pair_score f, int32_t *__restrict__ src_out,
                                    int32_t *__restrict__ dst_out, float *__restrict__ score_out) {
  const int64_t per = static_cast<int64_t>(rows) * cols, total = per * grids;
  for (int64_t c = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; c < total;
       c += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int32_t g = static_cast<int32_t>(c / per);
    const int64_t rc = c - static_cast<int64_t>(g) * per;
    const int32_t r = static_cast<int32_t>(rc / cols), q = static_cast<int32_t>(rc - static_cast<int64_t>(r) * cols);
    int32_t src = row_ids ? row_ids[static_cast<int64_t>(g) * rows + r] : r;
    int32_t dst = col_ids ? col_ids[static_cast<int64_t>(g) * cols + q] : q;
    const bool in = src >= 0 && src < a.num_units && dst >= 0 && dst < a.num_units;
    float score = in ? pair_score(f, src, dst) : 0.0f;
    ProposeArgs ag = a;
    if (per_grid_bucket) ag.bucket_level = g;
    apply_window(ag, src, dst, score, true);
    src_out[c] = src;
    dst_out[c] = dst;
    score_out[c] = score;
  }
}

static bool pair_score_ok(const pxb_pair_score *f, bool two_columns) {
  if (f == nullptr) return false;
  switch (f->form) {
    case PXB_PAIR_ABS_PRODUCT:
    case PXB_PAIR_PRODUCT:
      return f->x_src != nullptr && (!two_columns || f->x_dst != nullptr);
    case PXB_PAIR_MODULAR:
    case PXB_PAIR_MODULAR_PREDICATE:
      return f->m >= 1;
    default:
      return false;
  }
}

}  // namespace pxb

using namespace pxb;

extern "C" int pxb_unit_importance(int32_t num_units, const pxb_pair_score *form, const uint8_t *pruned,
                                   const int32_t *level, int32_t mask_kind, int32_t bucket, int32_t max_level_gap,
                                   int32_t direction, float *out, void *stream) {
  PXB_REQUIRE(num_units >= 0, "pxb_unit_importance: negative num_units");
  PXB_REQUIRE(pair_score_ok(form, false) && form->form != PXB_PAIR_MODULAR_PREDICATE,
              "pxb_unit_importance: unknown or incomplete importance form");
  PXB_REQUIRE(mask_kind >= 0 && mask_kind <= 2 && (mask_kind == 0 || level != nullptr),
              "pxb_unit_importance: mask kind %d needs the level column", mask_kind);
  PXB_REQUIRE(direction >= 0 && direction <= 2, "pxb_unit_importance: unknown direction %d", direction);
  if (num_units == 0) return PXB_OK;
  PXB_REQUIRE(out != nullptr, "pxb_unit_importance: out is NULL");
  unit_importance_kernel<<<grid_for(num_units, 256, 4), 256, 0, as_stream(stream)>>>(
      num_units, *form, pruned, level, mask_kind, bucket, max_level_gap, direction, out);
  PXB_LAUNCHED("unit_importance_kernel");
  return PXB_OK;
}

extern "C" int pxb_propose_grid(int32_t num_units, int32_t grids, int32_t rows, int32_t cols, const int32_t *row_ids,
                                const int32_t *col_ids, int32_t per_grid_bucket, const pxb_pair_score *score,
                                const int32_t *level, const uint8_t *pruned, int32_t max_level_gap, int32_t direction,
                                int32_t allow_self_loops, int32_t src_level_bound, int32_t *src_out, int32_t *dst_out,
                                float *score_out, void *stream) {
  PXB_REQUIRE(num_units >= 1 && grids >= 0 && rows >= 0 && cols >= 0, "pxb_propose_grid: bad sizes");
  const int64_t total = int64_t(grids) * rows * cols;
  PXB_REQUIRE(total < (int64_t(1) << 31), "pxb_propose_grid: %lld candidates exceed the int32 candidate index",
              static_cast<long long>(total));
  PXB_REQUIRE(pair_score_ok(score, true), "pxb_propose_grid: unknown or incomplete score form");
  PXB_REQUIRE(direction >= 0 && direction <= 2, "pxb_propose_grid: unknown direction %d", direction);
  if (total == 0) return PXB_OK;
  PXB_REQUIRE(level && src_out && dst_out && score_out, "pxb_propose_grid: a pointer is NULL");
  PXB_REQUIRE((row_ids != nullptr || rows <= num_units) && (col_ids != nullptr || cols <= num_units),
              "pxb_propose_grid: an identity axis longer than the units");
  ProposeArgs a{num_units, 1, 0, 0, nullptr, 0, num_units, PXB_SCORE_UNIFORM, nullptr, nullptr, level,
                pruned, max_level_gap, direction, allow_self_loops, -1, src_level_bound};
  propose_grid_kernel<<<grid_for(total, 256, 8), 256, 0, as_stream(stream)>>>(
      a, grids, rows, cols, row_ids, col_ids, per_grid_bucket, *score, src_out, dst_out, score_out);
  PXB_LAUNCHED("propose_grid_kernel");
  return PXB_OK;
}
