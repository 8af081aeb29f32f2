// Growth dedupe (src/plastax/phases.py:4111-4205, :2481-2575): veto a
// candidate whose (src, dst) is already a live edge of the bucket, and keep
// only the first copy of a pair repeated within the step.
//
// The reference sorts every live pair id of the bucket and binary-searches
// each candidate, and sorts the candidates for the within-step repeats. Here
// the step's candidate pairs go into an open-addressing hash table (keys,
// the best copy, a live mark; it stays in L2 for a million candidates): one
// streaming pass over the bucket marks the pairs that are live, and the
// survivor of a repeated pair is the copy with the least (score rank,
// candidate index), found with a 64-bit atomic minimum. The score rank
// orders as the reference's stable sort of -score does: descending scores,
// -inf after every finite score, NaN last.
#include "pxb_common.cuh"

namespace pxb {

constexpr unsigned long long kNoKey = ~0ull;

struct PairTable {
  int64_t size;  // power of two
  unsigned long long *keys, *best;
  uint32_t *live;
  int32_t *slot;  // per candidate: its pair's table slot
};

__device__ __forceinline__ unsigned long long pair_key(int32_t s, int32_t d) {
  return (static_cast<unsigned long long>(static_cast<uint32_t>(s)) << 32) | static_cast<uint32_t>(d);
}

__device__ __forceinline__ uint64_t mix64(uint64_t x) {
  x ^= x >> 33;
  x *= 0xff51afd7ed558ccdull;
  x ^= x >> 33;
  x *= 0xc4ceb9fe1a85ec53ull;
  return x ^ (x >> 33);
}

// Order-preserving image of a score under the reference's stable sort of
// -score: smaller first; -inf after the finite scores, NaN last.
__device__ __forceinline__ uint32_t dedupe_rank(float s) {
  if (isnan(s)) return 0xffffffffu;
  float neg = -s;
  if (neg == 0.0f) neg = 0.0f;
  const uint32_t u = __float_as_uint(neg);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__global__ void pair_insert_kernel(int64_t n, const int32_t *__restrict__ src, const int32_t *__restrict__ dst,
                                   PairTable t) {
  const uint64_t mask = static_cast<uint64_t>(t.size - 1);
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const unsigned long long key = pair_key(src[i], dst[i]);
    uint64_t h = mix64(key) & mask;
    for (int64_t probe = 0; probe < t.size; ++probe) {  // the table is at least twice the candidates
      const unsigned long long prev = atomicCAS(t.keys + h, kNoKey, key);
      if (prev == kNoKey || prev == key) break;
      h = (h + 1) & mask;
    }
    t.slot[i] = static_cast<int32_t>(h);
  }
}

// Mark the table pairs that are live edges of the bucket.
__global__ void live_mark_kernel(int64_t cap, const int32_t *__restrict__ from_id, const int32_t *__restrict__ to_id,
                                 const uint8_t *__restrict__ dead, PairTable t) {
  const uint64_t mask = static_cast<uint64_t>(t.size - 1);
  for (int64_t s = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; s < cap;
       s += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    if (dead[s]) continue;
    const unsigned long long key = pair_key(from_id[s], to_id[s]);
    uint64_t h = mix64(key) & mask;
    for (int64_t probe = 0; probe < t.size; ++probe) {
      const unsigned long long k = t.keys[h];
      if (k == kNoKey) break;
      if (k == key) {
        t.live[h] = 1u;
        break;
      }
      h = (h + 1) & mask;
    }
  }
}

__global__ void live_hit_kernel(int64_t n, PairTable t, uint8_t *__restrict__ hit) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    hit[i] = t.live[t.slot[i]] ? 1 : 0;
}

// Live veto, then each copy offers (rank, index) to its pair's minimum.
__global__ void dedupe_offer_kernel(int64_t n, float *__restrict__ score, const uint8_t *__restrict__ hit,
                                    int32_t step_repeats, PairTable t) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float s = score[i];
    if (hit != nullptr && hit[i]) {
      s = -__int_as_float(0x7f800000);
      score[i] = s;
    }
    if (step_repeats)
      atomicMin(t.best + t.slot[i],
                (static_cast<unsigned long long>(dedupe_rank(s)) << 32) | static_cast<uint32_t>(i));
  }
}

__global__ void dedupe_veto_kernel(int64_t n, float *__restrict__ score, PairTable t) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    if (static_cast<uint32_t>(t.best[t.slot[i]]) != static_cast<uint32_t>(i)) score[i] = -__int_as_float(0x7f800000);
}

static int64_t table_size(int64_t n) {
  int64_t t = 1024;
  while (t < 2 * n) t <<= 1;
  return t;
}

static size_t table_layout(int64_t n, char *base, PairTable *t) {
  t->size = table_size(n);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off = (off + bytes + 255) / 256 * 256;
    return base ? base + at : nullptr;
  };
  t->keys = reinterpret_cast<unsigned long long *>(take(t->size * 8));
  t->best = reinterpret_cast<unsigned long long *>(take(t->size * 8));
  t->live = reinterpret_cast<uint32_t *>(take(t->size * 4));
  t->slot = reinterpret_cast<int32_t *>(take((n > 0 ? n : 1) * 4));
  return off;
}

}  // namespace pxb

using namespace pxb;

extern "C" int pxb_dedupe_scratch_bytes(int64_t n, size_t *bytes) {
  PXB_REQUIRE(bytes && n >= 0 && n < (int64_t(1) << 30), "pxb_dedupe_scratch_bytes: bad arguments");
  PairTable t;
  *bytes = table_layout(n, nullptr, &t);
  return PXB_OK;
}

extern "C" int pxb_pair_table_build(int64_t n, const int32_t *src, const int32_t *dst, void *scratch,
                                    size_t scratch_bytes, void *stream) {
  PXB_REQUIRE(n >= 0 && n < (int64_t(1) << 30), "pxb_pair_table_build: n out of range");
  if (n == 0) return PXB_OK;
  PXB_REQUIRE(src && dst && scratch, "pxb_pair_table_build: a pointer is NULL");
  PairTable t;
  const size_t need = table_layout(n, static_cast<char *>(scratch), &t);
  PXB_REQUIRE(need <= scratch_bytes, "pxb_pair_table_build: scratch has %zu bytes, needs %zu", scratch_bytes, need);
  cudaStream_t st = as_stream(stream);
  PXB_CUDA(cudaMemsetAsync(t.keys, 0xff, t.size * 8, st));
  PXB_CUDA(cudaMemsetAsync(t.best, 0xff, t.size * 8, st));
  PXB_CUDA(cudaMemsetAsync(t.live, 0, t.size * 4, st));
  pair_insert_kernel<<<grid_for(n, 256, 8), 256, 0, st>>>(n, src, dst, t);
  PXB_LAUNCHED("pair_insert_kernel");
  return PXB_OK;
}

extern "C" int pxb_pair_table_mark(int64_t n, int64_t cap, const int32_t *from_id, const int32_t *to_id,
                                   const uint8_t *dead, uint8_t *live_hit, void *scratch, size_t scratch_bytes,
                                   void *stream) {
  PXB_REQUIRE(n >= 0 && n < (int64_t(1) << 30) && cap >= 0, "pxb_pair_table_mark: sizes out of range");
  if (n == 0) return PXB_OK;
  PXB_REQUIRE(live_hit && scratch && (cap == 0 || (from_id && to_id && dead)),
              "pxb_pair_table_mark: a pointer is NULL");
  PairTable t;
  const size_t need = table_layout(n, static_cast<char *>(scratch), &t);
  PXB_REQUIRE(need <= scratch_bytes, "pxb_pair_table_mark: scratch has %zu bytes, needs %zu", scratch_bytes, need);
  cudaStream_t st = as_stream(stream);
  if (cap > 0) {
    live_mark_kernel<<<grid_for(cap, 256, 8), 256, 0, st>>>(cap, from_id, to_id, dead, t);
    PXB_LAUNCHED("live_mark_kernel");
  }
  live_hit_kernel<<<grid_for(n, 256, 8), 256, 0, st>>>(n, t, live_hit);
  PXB_LAUNCHED("live_hit_kernel");
  return PXB_OK;
}

extern "C" int pxb_dedupe_apply(int64_t n, float *score, const uint8_t *live_hit, int32_t step_repeats,
                                void *scratch, size_t scratch_bytes, void *stream) {
  PXB_REQUIRE(n >= 0 && n < (int64_t(1) << 30), "pxb_dedupe_apply: n out of range");
  if (n == 0) return PXB_OK;
  PXB_REQUIRE(score && scratch, "pxb_dedupe_apply: a pointer is NULL");
  PairTable t;
  const size_t need = table_layout(n, static_cast<char *>(scratch), &t);
  PXB_REQUIRE(need <= scratch_bytes, "pxb_dedupe_apply: scratch has %zu bytes, needs %zu", scratch_bytes, need);
  cudaStream_t st = as_stream(stream);
  if (live_hit == nullptr && !step_repeats) return PXB_OK;
  dedupe_offer_kernel<<<grid_for(n, 256, 8), 256, 0, st>>>(n, score, live_hit, step_repeats, t);
  PXB_LAUNCHED("dedupe_offer_kernel");
  if (step_repeats) {
    dedupe_veto_kernel<<<grid_for(n, 256, 8), 256, 0, st>>>(n, score, t);
    PXB_LAUNCHED("dedupe_veto_kernel");
  }
  return PXB_OK;
}
