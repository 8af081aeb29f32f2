// The unit lifecycle (src/plastax/phases.py:1148-1193, :1245-1425):
// update_unit, prune_unit with the tombstoning of every incident connection,
// and add_unit (lowest free ids to the parents in ascending id order), for the
// rules' lowered forms. Unit-side work is O(num_units) (C4: 65,536 slots);
// the one arena pass is the incident-edge kill.
#include <cub/cub.cuh>

#include "pxb_common.cuh"

namespace pxb {

constexpr int kMaxUnitColumns = PXB_MAX_UNIT_COLUMNS;

// Reset slot i of every listed column to its default bit pattern.
__device__ __forceinline__ void reset_columns(const pxb_unit_columns &c, int32_t i) {
  for (int k = 0; k < c.count && k < kMaxUnitColumns; ++k) {
    if (c.bytes[k] == 4) static_cast<uint32_t *>(c.cols[k])[i] = c.defaults[k];
    else if (c.bytes[k] == 1) static_cast<uint8_t *>(c.cols[k])[i] = static_cast<uint8_t>(c.defaults[k]);
  }
}

__global__ void unit_update_kernel(int32_t n, int32_t kind, float *__restrict__ field, const float *__restrict__ src,
                                   float a, float b, const uint8_t *__restrict__ pruned) {
  for (int32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    if (pruned != nullptr && pruned[i]) continue;
    const float f = field[i];
    if (kind == PXB_UNIT_UPDATE_AFFINE) {
      field[i] = __fadd_rn(__fmul_rn(f, a), b);
    } else {
      const float s = kind == PXB_UNIT_UPDATE_TRACE_ABS ? fabsf(src[i]) : src[i];
      field[i] = __fadd_rn(__fmul_rn(__fsub_rn(1.0f, a), f), __fmul_rn(a, s));
    }
  }
}

__global__ void unit_prune_kernel(int32_t n, const float *__restrict__ field, const float *__restrict__ threshold,
                                  const uint8_t *__restrict__ exempt, uint8_t *__restrict__ pruned,
                                  uint8_t *__restrict__ doomed, pxb_unit_columns reset) {
  const float thr = *threshold;
  for (int32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const bool d = field[i] < thr && !pruned[i] && !(exempt != nullptr && exempt[i]);
    doomed[i] = d ? 1 : 0;
    if (d) {
      reset_columns(reset, i);
      pruned[i] = 1;
    }
  }
}

// Every live connection with a doomed endpoint is tombstoned and joins its
// claim domain's free bitmap (row bitmap_level[from] or 0).
__global__ void kill_unit_edges_kernel(int64_t cap, const int32_t *__restrict__ from, const int32_t *__restrict__ to,
                                       uint8_t *__restrict__ dead, uint32_t n, const uint8_t *__restrict__ doomed,
                                       uint32_t *__restrict__ bm, int64_t bm_words,
                                       const int32_t *__restrict__ bm_level) {
  for (int64_t s = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; s < cap;
       s += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    if (dead[s]) continue;
    const int32_t f = from[s], t = to[s];
    const bool kill = (static_cast<uint32_t>(f) < n && doomed[f]) || (static_cast<uint32_t>(t) < n && doomed[t]);
    if (!kill) continue;
    dead[s] = 1;
    if (bm != nullptr) {
      const int64_t row = bm_level != nullptr && static_cast<uint32_t>(f) < n ? bm_level[f] : 0;
      atomicOr(bm + row * bm_words + (s >> 5), 1u << (s & 31));
    }
  }
}

// Candidate values of the quantile: live, non-exempt units (+inf for the
// rest, so they sort last), counted per CTA into `count` (zeroed before).
__global__ void quantile_gather_kernel(int32_t n, const float *__restrict__ field, const uint8_t *__restrict__ pruned,
                                       const uint8_t *__restrict__ exempt, float *__restrict__ vals,
                                       int32_t *__restrict__ count) {
  __shared__ int32_t s_count;
  if (threadIdx.x == 0) s_count = 0;
  __syncthreads();
  int32_t local = 0;
  for (int32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const bool cand = !(pruned != nullptr && pruned[i]) && !(exempt != nullptr && exempt[i]);
    const float v = field[i];
    vals[i] = cand && !isnan(v) ? v : __int_as_float(0x7f800000);
    local += (cand && !isnan(v)) ? 1 : 0;
  }
  local = __reduce_add_sync(0xffffffffu, local);
  if ((threadIdx.x & 31) == 0 && local) atomicAdd(&s_count, local);
  __syncthreads();
  if (threadIdx.x == 0 && s_count) atomicAdd(count, s_count);
}

// The quantile by a radix select (one CTA): the floor(q * m)-th smallest of
// the m candidates (values with the order of their float bits: the
// order a radix sort of floats gives, -0 before +0), three digit passes of
// 11, 11 and 10 bits over every value, -inf without a candidate. Exactly
// the element a full sort would put at that position.
constexpr int kQsThreads = 1024;
__device__ __forceinline__ uint32_t float_order(float v) {
  const uint32_t b = __float_as_uint(v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float order_float(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

__global__ void __launch_bounds__(kQsThreads) quantile_select_kernel(int32_t n, const float *__restrict__ vals,
                                                                     const int32_t *__restrict__ count, float q,
                                                                     float *__restrict__ out) {
  using Scan = cub::BlockScan<uint32_t, kQsThreads>;
  __shared__ typename Scan::TempStorage scan_tmp;
  __shared__ uint32_t hist[2048];
  __shared__ uint32_t s_prefix, s_rank;
  const int32_t m = *count;
  if (m == 0) {
    if (threadIdx.x == 0) *out = -__int_as_float(0x7f800000);
    return;
  }
  if (threadIdx.x == 0) {
    int64_t r = static_cast<int64_t>(floor(static_cast<double>(q) * m));
    if (r > m - 1) r = m - 1;
    if (r < 0) r = 0;
    s_prefix = 0u;
    s_rank = static_cast<uint32_t>(r);
  }
  const int shifts[3] = {21, 10, 0}, widths[3] = {11, 11, 10};
  uint32_t known = 0u;  // the mask of the key bits fixed so far
  for (int pass = 0; pass < 3; ++pass) {
    const int sh = shifts[pass], wd = widths[pass];
    for (int i = threadIdx.x; i < 2048; i += kQsThreads) hist[i] = 0u;
    __syncthreads();
    const uint32_t prefix = s_prefix;
    for (int32_t i = threadIdx.x; i < n; i += kQsThreads) {
      const uint32_t k = float_order(vals[i]);
      if ((k & known) == prefix) atomicAdd(&hist[(k >> sh) & ((1u << wd) - 1u)], 1u);
    }
    __syncthreads();
    const uint32_t h0 = hist[2 * threadIdx.x], h1 = hist[2 * threadIdx.x + 1];
    uint32_t ex, total;
    Scan(scan_tmp).ExclusiveSum(h0 + h1, ex, total);
    const uint32_t rank = s_rank;
    __syncthreads();  // every thread has read s_rank
    if (rank >= ex && rank < ex + h0) {
      s_prefix = prefix | (static_cast<uint32_t>(2 * threadIdx.x) << sh);
      s_rank = rank - ex;
    } else if (rank >= ex + h0 && rank < ex + h0 + h1) {
      s_prefix = prefix | (static_cast<uint32_t>(2 * threadIdx.x + 1) << sh);
      s_rank = rank - ex - h0;
    }
    known |= ((1u << wd) - 1u) << sh;
    __syncthreads();
  }
  if (threadIdx.x == 0) *out = order_float(s_prefix);
}

// add_unit in one CTA: the free slots (PRUNED at the start of the phase,
// ascending) and the parents (live spawners, ascending) are ranked with
// block-wide scans over 1024-slot tiles; parent k takes free slot k.
constexpr int kAddThreads = 1024;

__device__ __forceinline__ bool spawns(int32_t kind, const float *field, float threshold, int32_t argmax, int32_t i) {
  return kind == PXB_SPAWN_FIELD_AT_LEAST ? field[i] >= threshold : i == argmax;
}

__global__ void __launch_bounds__(kAddThreads) unit_add_kernel(int32_t n, pxb_unit_spawn sp, uint8_t *__restrict__ pruned,
                                                               int32_t *__restrict__ level, int32_t *__restrict__ free_ids,
                                                               int32_t *__restrict__ parent_of,
                                                               pxb_unit_columns reset, int32_t *__restrict__ added,
                                                               uint8_t *__restrict__ overflow) {
  typedef cub::BlockScan<int32_t, kAddThreads> Scan;
  __shared__ typename Scan::TempStorage scan_tmp;
  __shared__ int32_t s_base;
  __shared__ float s_val[kAddThreads];
  __shared__ int32_t s_idx[kAddThreads];
  // 0. the argmax spawner: the largest non-NaN field among live units, the
  //    lowest id on ties (none when there is no such unit)
  int32_t argmax = -1;
  if (sp.kind == PXB_SPAWN_ARGMAX) {
    float best = 0.0f;
    int32_t arg = -1;
    for (int32_t i = threadIdx.x; i < n; i += kAddThreads) {
      if (pruned[i]) continue;
      const float v = sp.field[i];
      if (isnan(v)) continue;
      if (arg < 0 || v > best) {  // ascending i per thread: ties keep the lower id
        best = v;
        arg = i;
      }
    }
    s_val[threadIdx.x] = best;
    s_idx[threadIdx.x] = arg;
    __syncthreads();
    for (int off = kAddThreads / 2; off > 0; off >>= 1) {
      if (threadIdx.x < off) {
        const int32_t ia = s_idx[threadIdx.x], ib = s_idx[threadIdx.x + off];
        const float va = s_val[threadIdx.x], vb = s_val[threadIdx.x + off];
        if (ib >= 0 && (ia < 0 || vb > va || (vb == va && ib < ia))) {
          s_val[threadIdx.x] = vb;
          s_idx[threadIdx.x] = ib;
        }
      }
      __syncthreads();
    }
    argmax = s_idx[0];
  }
  // 1. free ids, ascending; and the parents' marks (pre-phase state)
  if (threadIdx.x == 0) s_base = 0;
  __syncthreads();
  for (int32_t tile = 0; tile < n; tile += kAddThreads) {
    const int32_t i = tile + threadIdx.x;
    const int32_t is_free = i < n && pruned[i] ? 1 : 0;
    int32_t pos, total;
    Scan(scan_tmp).ExclusiveSum(is_free, pos, total);
    if (is_free) free_ids[s_base + pos] = i;
    if (i < n) parent_of[i] = -1;
    __syncthreads();
    if (threadIdx.x == 0) s_base += total;
    __syncthreads();
  }
  const int32_t num_free = s_base;
  __syncthreads();
  // 2. parents in ascending id take the free slots in ascending id
  if (threadIdx.x == 0) s_base = 0;
  __syncthreads();
  int32_t dropped = 0;
  for (int32_t tile = 0; tile < n; tile += kAddThreads) {
    const int32_t i = tile + threadIdx.x;
    const int32_t is_parent = i < n && !pruned[i] && spawns(sp.kind, sp.field, sp.threshold, argmax, i) ? 1 : 0;
    int32_t pos, total;
    Scan(scan_tmp).ExclusiveSum(is_parent, pos, total);
    if (is_parent) {
      const int32_t rank = s_base + pos;
      if (rank < num_free) parent_of[free_ids[rank]] = i;
      else dropped = 1;
    }
    __syncthreads();
    if (threadIdx.x == 0) s_base += total;
    __syncthreads();
  }
  const int32_t parents = s_base;
  if (dropped) *overflow = 1;  // any thread: a benign same-value store
  __syncthreads();
  // 3. the children: defaults, live, clamped level, the init write
  for (int32_t c = threadIdx.x; c < n; c += kAddThreads) {
    const int32_t p = parent_of[c];
    if (p < 0) continue;
    reset_columns(reset, c);
    int64_t lv = static_cast<int64_t>(level[p]) + sp.offset;
    if (lv < 1) lv = 1;
    if (lv > sp.max_level) lv = sp.max_level;
    level[c] = static_cast<int32_t>(lv);
    if (sp.init_dst != nullptr) sp.init_dst[c] = __fmul_rn(sp.init_src[p], sp.init_scale);
  }
  __syncthreads();
  for (int32_t c = threadIdx.x; c < n; c += kAddThreads)
    if (parent_of[c] >= 0) pruned[c] = 0;
  if (threadIdx.x == 0) *added = parents < num_free ? parents : num_free;
}

}  // namespace pxb

using namespace pxb;

static int check_columns(const char *fn, const pxb_unit_columns *c) {
  PXB_REQUIRE(c != nullptr && c->count >= 0 && c->count <= kMaxUnitColumns, "%s: bad column list", fn);
  for (int k = 0; k < c->count; ++k)
    PXB_REQUIRE(c->cols[k] != nullptr && (c->bytes[k] == 1 || c->bytes[k] == 4),
                "%s: column %d must be a 1- or 4-byte column", fn, k);
  return PXB_OK;
}

extern "C" int pxb_unit_update(int32_t num_units, int32_t kind, float *field, const float *src, float a, float b,
                               const uint8_t *pruned, void *stream) {
  PXB_REQUIRE(num_units >= 0, "pxb_unit_update: negative num_units");
  PXB_REQUIRE(kind >= 0 && kind <= 2, "pxb_unit_update: unknown kind %d", kind);
  if (num_units == 0) return PXB_OK;
  PXB_REQUIRE(field && (kind == PXB_UNIT_UPDATE_AFFINE || src), "pxb_unit_update: a column is NULL");
  unit_update_kernel<<<grid_for(num_units, 256, 4), 256, 0, as_stream(stream)>>>(num_units, kind, field, src, a, b,
                                                                                 pruned);
  PXB_LAUNCHED("unit_update_kernel");
  return PXB_OK;
}

extern "C" int pxb_unit_quantile_scratch_bytes(int32_t num_units, size_t *bytes) {
  PXB_REQUIRE(bytes && num_units >= 0, "pxb_unit_quantile_scratch_bytes: bad arguments");
  const size_t col = (size_t(num_units > 0 ? num_units : 1) * 4 + 255) / 256 * 256;
  *bytes = col + 256;  // the candidates' values, their count
  return PXB_OK;
}

extern "C" int pxb_unit_quantile(int32_t num_units, const float *field, const uint8_t *pruned, const uint8_t *exempt,
                                 float q, float *out, void *scratch, size_t scratch_bytes, void *stream) {
  PXB_REQUIRE(num_units >= 0 && q >= 0.0f && q <= 1.0f, "pxb_unit_quantile: bad arguments");
  PXB_REQUIRE(field && out && scratch, "pxb_unit_quantile: a pointer is NULL");
  size_t need = 0;
  int rc = pxb_unit_quantile_scratch_bytes(num_units, &need);
  if (rc) return rc;
  PXB_REQUIRE(need <= scratch_bytes, "pxb_unit_quantile: scratch has %zu bytes, needs %zu", scratch_bytes, need);
  cudaStream_t st = as_stream(stream);
  const size_t col = (size_t(num_units > 0 ? num_units : 1) * 4 + 255) / 256 * 256;
  float *vals = static_cast<float *>(scratch);
  int32_t *count = reinterpret_cast<int32_t *>(static_cast<char *>(scratch) + col);
  PXB_CUDA(cudaMemsetAsync(count, 0, sizeof(int32_t), st));
  if (num_units > 0) {
    quantile_gather_kernel<<<grid_for(num_units, 256, 4), 256, 0, st>>>(num_units, field, pruned, exempt, vals,
                                                                       count);
    PXB_LAUNCHED("quantile_gather_kernel");
  }
  quantile_select_kernel<<<1, kQsThreads, 0, st>>>(num_units, vals, count, q, out);
  PXB_LAUNCHED("quantile_select_kernel");
  PXB_LAUNCHED("quantile_pick_kernel");
  return PXB_OK;
}

extern "C" int pxb_unit_prune(int32_t num_units, const float *field, const float *threshold, const uint8_t *exempt,
                              uint8_t *pruned, uint8_t *doomed, const pxb_unit_columns *reset, void *stream) {
  PXB_REQUIRE(num_units >= 0, "pxb_unit_prune: negative num_units");
  int rc = check_columns("pxb_unit_prune", reset);
  if (rc) return rc;
  if (num_units == 0) return PXB_OK;
  PXB_REQUIRE(field && threshold && pruned && doomed, "pxb_unit_prune: a pointer is NULL");
  unit_prune_kernel<<<grid_for(num_units, 256, 4), 256, 0, as_stream(stream)>>>(num_units, field, threshold, exempt,
                                                                                pruned, doomed, *reset);
  PXB_LAUNCHED("unit_prune_kernel");
  return PXB_OK;
}

extern "C" int pxb_kill_unit_edges(int64_t cap, const int32_t *from_id, const int32_t *to_id, uint8_t *dead,
                                   int32_t num_units, const uint8_t *doomed, uint32_t *free_bitmap,
                                   const int32_t *bitmap_level, void *stream) {
  PXB_REQUIRE(cap >= 0 && num_units >= 0, "pxb_kill_unit_edges: sizes out of range");
  if (cap == 0) return PXB_OK;
  PXB_REQUIRE(from_id && to_id && dead && doomed, "pxb_kill_unit_edges: a pointer is NULL");
  kill_unit_edges_kernel<<<grid_for(cap, 256, 8), 256, 0, as_stream(stream)>>>(
      cap, from_id, to_id, dead, static_cast<uint32_t>(num_units), doomed, free_bitmap, (cap + 31) / 32,
      bitmap_level);
  PXB_LAUNCHED("kill_unit_edges_kernel");
  return PXB_OK;
}

extern "C" int pxb_unit_add(int32_t num_units, const pxb_unit_spawn *spawn, uint8_t *pruned, int32_t *level,
                            const pxb_unit_columns *reset, int32_t *scratch, int32_t *units_added,
                            uint8_t *unit_overflow, void *stream) {
  PXB_REQUIRE(num_units >= 0 && spawn != nullptr, "pxb_unit_add: bad arguments");
  PXB_REQUIRE(spawn->kind == PXB_SPAWN_FIELD_AT_LEAST || spawn->kind == PXB_SPAWN_ARGMAX,
              "pxb_unit_add: unknown spawn kind %d", spawn->kind);
  PXB_REQUIRE(spawn->max_level >= 1, "pxb_unit_add: max_level must be >= 1");
  PXB_REQUIRE(spawn->init_dst == nullptr || spawn->init_src != nullptr, "pxb_unit_add: init needs its source");
  int rc = check_columns("pxb_unit_add", reset);
  if (rc) return rc;
  PXB_REQUIRE(units_added && unit_overflow, "pxb_unit_add: outputs are NULL");
  cudaStream_t st = as_stream(stream);
  PXB_CUDA(cudaMemsetAsync(units_added, 0, 4, st));
  PXB_CUDA(cudaMemsetAsync(unit_overflow, 0, 1, st));
  if (num_units == 0) return PXB_OK;
  PXB_REQUIRE(spawn->field && pruned && level && scratch, "pxb_unit_add: a pointer is NULL");
  unit_add_kernel<<<1, kAddThreads, 0, st>>>(num_units, *spawn, pruned, level, scratch, scratch + num_units, *reset,
                                             units_added, unit_overflow);
  PXB_LAUNCHED("unit_add_kernel");
  return PXB_OK;
}
