// Edge sweeps over one SOA bucket: forward accumulate (optionally fused with
// the prune predicate and per-block free counts), backward accumulate with
// warp-segmented reduction over source runs (optionally fused with the
// optimizer update), the unit-side apply, and the MSE loss seed.
//
// Every sweep is a grid-stride loop over the bucket in slot order with all
// column loads of an iteration issued before their first use, so each
// thread keeps several independent 16-byte (or 4-byte) loads in flight:
// the sweeps are HBM-bound streams of 13 B/slot (+4 B per optimizer column).
#include "optim.cuh"

namespace pxb {

// ---------------------------------------------------------------------------
// forward accumulate (+ prune + block free counts)
// ---------------------------------------------------------------------------
struct PruneArgs {
  int kind;
  float threshold;
  const float *unit_threshold;
  uint8_t *dead_out;
  bool in_place;       // dead_out == dead: write only the bytes that change
  int block_shift;     // log2(block_len), -1 when no counts
  int32_t *block_free;
  uint32_t *bm;        // per-domain free bitmaps, or NULL
  int64_t bm_words;
  const int32_t *bm_level;  // domain of a freed slot = bm_level[from_id]; NULL: domain 0
};

// A slot this sweep tombstoned joins its claim domain's free bitmap.
__device__ __forceinline__ void mark_free(const PruneArgs &pa, int64_t s, int32_t from, uint32_t n) {
  if (pa.bm == nullptr) return;
  int64_t row = 0;
  if (pa.bm_level != nullptr) {
    const int32_t o = from < 0 ? 0 : (static_cast<uint32_t>(from) >= n ? static_cast<int32_t>(n) - 1 : from);
    row = pa.bm_level[o];
  }
  atomicOr(pa.bm + row * pa.bm_words + (s >> 5), 1u << (s & 31));
}

__device__ __forceinline__ bool prune_pred(const PruneArgs &pa, float w, int32_t to, uint32_t n) {
  if (pa.kind == PXB_PRUNE_ABS_BELOW) return fabsf(w) < pa.threshold;
  if (pa.kind == PXB_PRUNE_ABS_BELOW_DST)
    return static_cast<uint32_t>(to) < n && fabsf(w) < __ldg(pa.unit_threshold + to);
  return false;
}

// Warp-level free count of the new tombstones, one atomic per warp into the
// counting block its slots lie in (a warp covers <= 128 consecutive slots and
// block_len >= 128 is a power of two, so they all share one block).
__device__ __forceinline__ void count_free(const PruneArgs &pa, int64_t first_slot, int freed) {
  const unsigned mask = __activemask();
  const int total = __reduce_add_sync(mask, freed);
  const int leader = __ffs(mask) - 1;
  if ((threadIdx.x & 31) == leader && total > 0)
    atomicAdd(pa.block_free + (first_slot >> pa.block_shift), total);
}

template <int MONOID, bool PRUNE>
__global__ void __launch_bounds__(256) forward_vec4_kernel(
    int64_t groups, const int4 *__restrict__ from4, const int4 *__restrict__ to4,
    const uint32_t *__restrict__ dead4, const float4 *__restrict__ w4,
    const float *__restrict__ act, float *__restrict__ acc, uint32_t n, PruneArgs pa) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t g = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; g < groups; g += stride) {
    const int4 f = __ldcs(from4 + g);
    const int4 t = __ldcs(to4 + g);
    const float4 w = __ldcs(w4 + g);
    const uint32_t d = dead4[g];
    const int32_t fs[4] = {f.x, f.y, f.z, f.w};
    const int32_t ts[4] = {t.x, t.y, t.z, t.w};
    const float ws[4] = {w.x, w.y, w.z, w.w};
    float a[4];
    bool live[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      live[i] = !((d >> (8 * i)) & 0xffu) && static_cast<uint32_t>(fs[i]) < n && static_cast<uint32_t>(ts[i]) < n;
#pragma unroll
    for (int i = 0; i < 4; ++i) a[i] = live[i] ? __ldg(act + fs[i]) : 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (live[i]) atomic_combine<MONOID>(acc + ts[i], __fmul_rn(ws[i], a[i]));
    if (PRUNE) {
      uint32_t nd = d;
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (prune_pred(pa, ws[i], ts[i], n)) {
          nd |= (1u << (8 * i));
          if (!((d >> (8 * i)) & 0xffu)) mark_free(pa, g * 4 + i, fs[i], n);
        }
      if (!pa.in_place || nd != d) reinterpret_cast<uint32_t *>(pa.dead_out)[g] = nd;
      if (pa.block_shift >= 0) count_free(pa, g * 4, __popc(nd & 0x01010101u));
    }
  }
}

template <int MONOID, bool PRUNE>
__global__ void __launch_bounds__(256) forward_scalar_kernel(
    int64_t cap, const int32_t *__restrict__ from, const int32_t *__restrict__ to,
    const uint8_t *__restrict__ dead, const float *__restrict__ w, const float *__restrict__ act,
    float *__restrict__ acc, uint32_t n, PruneArgs pa) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t s = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; s < cap; s += stride) {
    const uint8_t d = dead[s];
    const float ws = w[s];
    const int32_t ts = to[s];
    const int32_t fs = from[s];
    if (!d && static_cast<uint32_t>(fs) < n && static_cast<uint32_t>(ts) < n)
      atomic_combine<MONOID>(acc + ts, __fmul_rn(ws, __ldg(act + fs)));
    if (PRUNE) {
      const uint8_t nd = d | (prune_pred(pa, ws, ts, n) ? 1 : 0);
      if (nd && !d) mark_free(pa, s, fs, n);
      if (!pa.in_place || nd != d) pa.dead_out[s] = nd;
      if (pa.block_shift >= 0) count_free(pa, s, nd ? 1 : 0);
    }
  }
}

// Prune sweep without the forward: reads w (+ to for a per-dst threshold).
__global__ void __launch_bounds__(256) prune_kernel(int64_t cap, const int32_t *__restrict__ from,
                                                    const int32_t *__restrict__ to,
                                                    const uint8_t *__restrict__ dead,
                                                    const float *__restrict__ w, uint32_t n, PruneArgs pa) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t s = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; s < cap; s += stride) {
    const uint8_t d = dead[s];
    const int32_t ts = pa.kind == PXB_PRUNE_ABS_BELOW_DST ? to[s] : 0;
    const uint8_t nd = d | (prune_pred(pa, w[s], ts, n) ? 1 : 0);
    if (nd && !d) mark_free(pa, s, pa.bm_level ? from[s] : 0, n);
    if (!pa.in_place || nd != d) pa.dead_out[s] = nd;
    if (pa.block_shift >= 0) count_free(pa, s, nd ? 1 : 0);
  }
}

// ---------------------------------------------------------------------------
// backward accumulate (+ fused optimizer update)
// ---------------------------------------------------------------------------
// Inclusive segmented combine across the warp: a segment is a run of equal
// keys in lane order. Returns the segment-prefix value; `tail` is set on the
// last lane of each segment.
template <int MONOID>
__device__ __forceinline__ float warp_segmented(float val, int32_t key, bool &tail) {
  const unsigned full = 0xffffffffu;
  const int lane = threadIdx.x & 31;
  const int32_t prev_key = __shfl_up_sync(full, key, 1);
  const int32_t next_key = __shfl_down_sync(full, key, 1);
  bool flag = lane == 0 || prev_key != key;
  tail = lane == 31 || next_key != key;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const float ov = __shfl_up_sync(full, val, off);
    const bool of = __shfl_up_sync(full, flag, off);
    if (lane >= off && !flag) {
      val = combine2<MONOID>(ov, val);
      flag = of;
    }
  }
  return val;
}

constexpr int kBwdUnroll = 4;

template <int MONOID, bool ACCUM, bool UPDATE>
__global__ void __launch_bounds__(256) backward_kernel(
    int64_t cap, const int32_t *__restrict__ from, const int32_t *__restrict__ to,
    const uint8_t *__restrict__ dead, float *__restrict__ weight, const float *__restrict__ grad,
    const float *__restrict__ act, float *__restrict__ acc, uint32_t n, OptParams op,
    float *__restrict__ m_col, float *__restrict__ v_col, float *__restrict__ t_col) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  const int64_t warps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const int64_t chunk_slots = 32 * kBwdUnroll;
  const int64_t chunks = (cap + chunk_slots - 1) / chunk_slots;
  const float ident = monoid_identity(MONOID);
  for (int64_t c = warp; c < chunks; c += warps) {
    int32_t f[kBwdUnroll], t[kBwdUnroll];
    float w[kBwdUnroll], g[kBwdUnroll];
    bool live[kBwdUnroll];
#pragma unroll
    for (int u = 0; u < kBwdUnroll; ++u) {
      const int64_t s = c * chunk_slots + u * 32 + lane;
      const bool in = s < cap;
      f[u] = in ? from[s] : -1;
      t[u] = in ? to[s] : 0;
      w[u] = in ? weight[s] : 0.0f;
      live[u] = in && !dead[s] && static_cast<uint32_t>(f[u]) < n && static_cast<uint32_t>(t[u]) < n;
    }
#pragma unroll
    for (int u = 0; u < kBwdUnroll; ++u) g[u] = live[u] ? __ldg(grad + t[u]) : 0.0f;
    if (ACCUM) {
#pragma unroll
      for (int u = 0; u < kBwdUnroll; ++u) {
        const int32_t key = live[u] ? f[u] : -1;
        bool tail;
        const float part = warp_segmented<MONOID>(live[u] ? __fmul_rn(w[u], g[u]) : ident, key, tail);
        if (tail && key >= 0) atomic_combine<MONOID>(acc + key, part);
      }
    }
    if (UPDATE) {
#pragma unroll
      for (int u = 0; u < kBwdUnroll; ++u) {
        if (!live[u]) continue;
        const int64_t s = c * chunk_slots + u * 32 + lane;
        const float gr = __fmul_rn(g[u], __ldg(act + f[u]));
        float wn = w[u];
        opt_step(op, gr, wn, m_col, v_col, t_col, s, f[u], t[u]);
        weight[s] = wn;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// unit apply (src/plastax/sweep.py:183-230)
// ---------------------------------------------------------------------------
__global__ void unit_apply_kernel(int32_t n, int mode, int act_kind, int monoid, float *__restrict__ acc,
                                  int64_t *__restrict__ acc_fixed, const float *__restrict__ act,
                                  const float *__restrict__ seed,
                                  const int32_t *__restrict__ level, int32_t target_level,
                                  const uint8_t *__restrict__ is_input, const uint8_t *__restrict__ pruned,
                                  float *__restrict__ out) {
  const int32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  if (level != nullptr && level[i] != target_level) return;
  const uint8_t role = is_input != nullptr ? is_input[i] : 0;
  if (role == 1) return;
  if (pruned != nullptr && pruned[i]) return;
  float a = acc[i];
  if (acc_fixed != nullptr) {
    // the exact fixed-point sum, rounded to float once (the scale is a power
    // of two), plus the float side (non-finite or huge products, normally 0)
    const long long f = acc_fixed[i];
    if (f != 0) {
      a = __fadd_rn(__fmul_rn(__ll2float_rn(f), 1.0f / float(1ll << PXB_FIXED_FRAC_BITS)), a);
      acc_fixed[i] = 0;
    }
  }
  if (mode == 0) {
    out[i] = act_fn(unit_act_kind(act_kind, role), a);
  } else {
    const float s = seed != nullptr ? seed[i] : 0.0f;
    out[i] = __fmul_rn(__fadd_rn(a, s), act_prime_from_act(unit_act_kind(act_kind, role), act[i]));
  }
  acc[i] = monoid_identity(monoid);
}

// MSE seed and loss over the outputs; one block, the loss summed in output
// order by thread 0 after the seeds are staged.
__global__ void mse_loss_kernel(int32_t k, const int32_t *__restrict__ ids, const float *__restrict__ act,
                                const float *__restrict__ target, float *__restrict__ seed,
                                float *__restrict__ loss) {
  for (int32_t i = threadIdx.x; i < k; i += blockDim.x) {
    const int32_t u = ids[i];
    seed[u] = __fsub_rn(act[u], target[i]);
  }
  __syncthreads();
  if (threadIdx.x == 0 && loss != nullptr) {
    float total = 0.0f;
    for (int32_t i = 0; i < k; ++i) {
      const float d = seed[ids[i]];
      total = __fadd_rn(total, __fmul_rn(__fmul_rn(0.5f, d), d));
    }
    loss[0] = total;
  }
}

static int check_bucket(const char *fn, int64_t cap, const void *from, const void *to, const void *dead,
                        const void *w) {
  PXB_REQUIRE(cap >= 0, "%s: negative capacity", fn);
  PXB_REQUIRE(cap < (int64_t(1) << 40), "%s: capacity out of range", fn);
  if (cap == 0) return PXB_OK;
  PXB_REQUIRE(from && to && dead && w, "%s: a bucket column is NULL", fn);
  return PXB_OK;
}

static int block_shift_of(const char *fn, int32_t block_len, int32_t *block_free, int min_len, int *shift) {
  *shift = -1;
  if (block_free == nullptr) return PXB_OK;
  PXB_REQUIRE(block_len >= min_len && (block_len & (block_len - 1)) == 0,
              "%s: block_len %d must be a power of two >= %d", fn, block_len, min_len);
  int s = 0;
  while ((1 << s) < block_len) ++s;
  *shift = s;
  return PXB_OK;
}

template <bool PRUNE>
static int launch_forward(int64_t cap, const int32_t *from, const int32_t *to, const uint8_t *dead,
                          const float *w, const float *act, int32_t num_units, int32_t monoid, float *acc,
                          PruneArgs pa, cudaStream_t st) {
  const uint32_t n = static_cast<uint32_t>(num_units);
  const bool vec = (cap % 4 == 0) && aligned16(from) && aligned16(to) && aligned16(w) &&
                   (reinterpret_cast<uintptr_t>(dead) % 4 == 0) &&
                   (!PRUNE || reinterpret_cast<uintptr_t>(pa.dead_out) % 4 == 0);
  if (vec) {
    const int64_t groups = cap / 4;
    const int grid = grid_for(groups, 256, 8);
#define PXB_FWD_VEC(M)                                                                          \
  forward_vec4_kernel<M, PRUNE><<<grid, 256, 0, st>>>(                                          \
      groups, reinterpret_cast<const int4 *>(from), reinterpret_cast<const int4 *>(to),         \
      reinterpret_cast<const uint32_t *>(dead), reinterpret_cast<const float4 *>(w), act, acc, n, pa)
    if (monoid == PXB_MONOID_SUM) PXB_FWD_VEC(PXB_MONOID_SUM);
    else if (monoid == PXB_MONOID_MAX) PXB_FWD_VEC(PXB_MONOID_MAX);
    else PXB_FWD_VEC(PXB_MONOID_MIN);
#undef PXB_FWD_VEC
    PXB_LAUNCHED("forward_vec4_kernel");
  } else {
    const int grid = grid_for(cap, 256, 8);
#define PXB_FWD_SC(M) \
  forward_scalar_kernel<M, PRUNE><<<grid, 256, 0, st>>>(cap, from, to, dead, w, act, acc, n, pa)
    if (monoid == PXB_MONOID_SUM) PXB_FWD_SC(PXB_MONOID_SUM);
    else if (monoid == PXB_MONOID_MAX) PXB_FWD_SC(PXB_MONOID_MAX);
    else PXB_FWD_SC(PXB_MONOID_MIN);
#undef PXB_FWD_SC
    PXB_LAUNCHED("forward_scalar_kernel");
  }
  return PXB_OK;
}

static int zero_counts(int64_t cap, int shift, int32_t *block_free, cudaStream_t st) {
  if (shift < 0) return PXB_OK;
  const int64_t blocks = (cap + (int64_t(1) << shift) - 1) >> shift;
  PXB_CUDA(cudaMemsetAsync(block_free, 0, blocks * sizeof(int32_t), st));
  return PXB_OK;
}

}  // namespace pxb

using namespace pxb;

extern "C" int pxb_forward_accumulate(int64_t cap, const int32_t *from_id, const int32_t *to_id,
                                      const uint8_t *dead, const float *weight, const float *act,
                                      int32_t num_units, int32_t monoid, float *acc, void *stream) {
  int rc = check_bucket("pxb_forward_accumulate", cap, from_id, to_id, dead, weight);
  if (rc) return rc;
  PXB_REQUIRE(monoid >= 0 && monoid <= 2, "pxb_forward_accumulate: unknown monoid %d", monoid);
  PXB_REQUIRE(num_units >= 0, "pxb_forward_accumulate: negative num_units");
  if (cap == 0) return PXB_OK;
  PXB_REQUIRE(act && acc, "pxb_forward_accumulate: act/acc is NULL");
  PruneArgs pa{PXB_PRUNE_NONE, 0.0f, nullptr, nullptr, false, -1, nullptr, nullptr, 0, nullptr};
  return launch_forward<false>(cap, from_id, to_id, dead, weight, act, num_units, monoid, acc, pa,
                               as_stream(stream));
}

extern "C" int pxb_forward_prune(int64_t cap, const int32_t *from_id, const int32_t *to_id,
                                 const uint8_t *dead, const float *weight, const float *act,
                                 int32_t num_units, int32_t monoid, float *acc, int32_t prune_kind,
                                 float prune_threshold, const float *unit_threshold, uint8_t *dead_out,
                                 int32_t block_len, int32_t *block_free, uint32_t *free_bitmap,
                                 const int32_t *bitmap_level, void *stream) {
  int rc = check_bucket("pxb_forward_prune", cap, from_id, to_id, dead, weight);
  if (rc) return rc;
  PXB_REQUIRE(monoid >= 0 && monoid <= 2, "pxb_forward_prune: unknown monoid %d", monoid);
  PXB_REQUIRE(prune_kind >= 0 && prune_kind <= 2, "pxb_forward_prune: unknown prune kind %d", prune_kind);
  PXB_REQUIRE(prune_kind != PXB_PRUNE_ABS_BELOW_DST || unit_threshold,
              "pxb_forward_prune: per-destination threshold column is NULL");
  PXB_REQUIRE(num_units >= 0, "pxb_forward_prune: negative num_units");
  int shift;
  rc = block_shift_of("pxb_forward_prune", block_len, block_free, 128, &shift);
  if (rc) return rc;
  cudaStream_t st = as_stream(stream);
  rc = zero_counts(cap, shift, block_free, st);
  if (rc) return rc;
  if (cap == 0) return PXB_OK;
  PXB_REQUIRE(act && acc && dead_out, "pxb_forward_prune: act/acc/dead_out is NULL");
  PruneArgs pa{prune_kind, prune_threshold, unit_threshold, dead_out, dead_out == dead, shift, block_free,
               free_bitmap, (cap + 31) / 32, bitmap_level};
  return launch_forward<true>(cap, from_id, to_id, dead, weight, act, num_units, monoid, acc, pa, st);
}

extern "C" int pxb_prune_conn(int64_t cap, const int32_t *from_id, const int32_t *to_id, const uint8_t *dead,
                              const float *weight, int32_t num_units, int32_t prune_kind, float prune_threshold,
                              const float *unit_threshold, uint8_t *dead_out, int32_t block_len,
                              int32_t *block_free, uint32_t *free_bitmap, const int32_t *bitmap_level,
                              void *stream) {
  PXB_REQUIRE(cap >= 0, "pxb_prune_conn: negative capacity");
  PXB_REQUIRE(num_units >= 0, "pxb_prune_conn: negative num_units");
  PXB_REQUIRE(prune_kind >= 0 && prune_kind <= 2, "pxb_prune_conn: unknown prune kind %d", prune_kind);
  PXB_REQUIRE(prune_kind != PXB_PRUNE_ABS_BELOW_DST || (unit_threshold && to_id),
              "pxb_prune_conn: per-destination threshold needs to_id and the threshold column");
  int shift;
  int rc = block_shift_of("pxb_prune_conn", block_len, block_free, 32, &shift);
  if (rc) return rc;
  cudaStream_t st = as_stream(stream);
  rc = zero_counts(cap, shift, block_free, st);
  if (rc) return rc;
  if (cap == 0) return PXB_OK;
  PXB_REQUIRE(dead && weight && dead_out, "pxb_prune_conn: a column is NULL");
  PXB_REQUIRE(!bitmap_level || from_id, "pxb_prune_conn: the bitmap domains need from_id");
  PruneArgs pa{prune_kind, prune_threshold, unit_threshold, dead_out, dead_out == dead, shift, block_free,
               free_bitmap, (cap + 31) / 32, bitmap_level};
  prune_kernel<<<grid_for(cap, 256, 8), 256, 0, st>>>(cap, from_id, to_id, dead, weight,
                                                      static_cast<uint32_t>(num_units), pa);
  PXB_LAUNCHED("prune_kernel");
  return PXB_OK;
}

static int launch_backward(int64_t cap, const int32_t *from, const int32_t *to, const uint8_t *dead,
                           float *weight, const float *grad, const float *act, int32_t num_units,
                           int32_t monoid, float *acc, const pxb_optimizer *opt, float *m, float *v, float *t,
                           cudaStream_t st) {
  const uint32_t n = static_cast<uint32_t>(num_units);
  OptParams op{0, 0, 0, 0, 0, 0, nullptr};
  const bool update = opt != nullptr;
  if (update) op = OptParams{opt->kind, opt->lr, opt->b1, opt->b2, opt->eps, opt->weight_decay, opt->unit_scale};
  const bool accum = acc != nullptr;
  const int64_t chunks = (cap + 32 * kBwdUnroll - 1) / (32 * kBwdUnroll);
  const int grid = grid_for(chunks, 8, 8);  // 8 warps per CTA
#define PXB_BWD(M, A, U)                                                                                  \
  backward_kernel<M, A, U><<<grid, 256, 0, st>>>(cap, from, to, dead, weight, grad, act, acc, n, op, m, v, t)
  if (accum && update) {
    if (monoid == PXB_MONOID_SUM) PXB_BWD(PXB_MONOID_SUM, true, true);
    else if (monoid == PXB_MONOID_MAX) PXB_BWD(PXB_MONOID_MAX, true, true);
    else PXB_BWD(PXB_MONOID_MIN, true, true);
  } else if (accum) {
    if (monoid == PXB_MONOID_SUM) PXB_BWD(PXB_MONOID_SUM, true, false);
    else if (monoid == PXB_MONOID_MAX) PXB_BWD(PXB_MONOID_MAX, true, false);
    else PXB_BWD(PXB_MONOID_MIN, true, false);
  } else if (update) {
    PXB_BWD(PXB_MONOID_SUM, false, true);
  }
#undef PXB_BWD
  PXB_LAUNCHED("backward_kernel");
  return PXB_OK;
}

extern "C" int pxb_backward_accumulate(int64_t cap, const int32_t *from_id, const int32_t *to_id,
                                       const uint8_t *dead, const float *weight, const float *grad,
                                       int32_t num_units, int32_t monoid, float *acc, void *stream) {
  int rc = check_bucket("pxb_backward_accumulate", cap, from_id, to_id, dead, weight);
  if (rc) return rc;
  PXB_REQUIRE(monoid >= 0 && monoid <= 2, "pxb_backward_accumulate: unknown monoid %d", monoid);
  PXB_REQUIRE(num_units >= 0, "pxb_backward_accumulate: negative num_units");
  if (cap == 0) return PXB_OK;
  PXB_REQUIRE(grad && acc, "pxb_backward_accumulate: grad/acc is NULL");
  return launch_backward(cap, from_id, to_id, dead, const_cast<float *>(weight), grad, nullptr, num_units,
                         monoid, acc, nullptr, nullptr, nullptr, nullptr, as_stream(stream));
}

static int check_opt(const char *fn, const pxb_optimizer *opt, const float *m, const float *v, const float *t) {
  PXB_REQUIRE(opt != nullptr, "%s: optimizer is NULL", fn);
  PXB_REQUIRE(opt->kind >= 0 && opt->kind <= 4, "%s: unknown optimizer kind %d", fn, opt->kind);
  PXB_REQUIRE(opt->kind != PXB_OPT_UPGD || (m && t && opt->unit_scale),
              "%s: upgd needs its utility (opt_m) and step (opt_t) columns and the unit scale", fn);
  PXB_REQUIRE(opt->kind != PXB_OPT_MOMENTUM || v, "%s: momentum needs its velocity column (opt_v)", fn);
  PXB_REQUIRE(opt->kind != PXB_OPT_ADAM || (m && v && t), "%s: adam needs opt/m, opt/v and opt/t", fn);
  PXB_REQUIRE(opt->kind != PXB_OPT_RMSPROP || v, "%s: rmsprop needs its mean-square column (opt_v)", fn);
  return PXB_OK;
}

extern "C" int pxb_backward_update(int64_t cap, const int32_t *from_id, const int32_t *to_id,
                                   const uint8_t *dead, float *weight, const float *grad, const float *act,
                                   int32_t num_units, float *acc, const pxb_optimizer *opt, float *opt_m,
                                   float *opt_v, float *opt_t, void *stream) {
  int rc = check_bucket("pxb_backward_update", cap, from_id, to_id, dead, weight);
  if (rc) return rc;
  rc = check_opt("pxb_backward_update", opt, opt_m, opt_v, opt_t);
  if (rc) return rc;
  PXB_REQUIRE(num_units >= 0, "pxb_backward_update: negative num_units");
  if (cap == 0) return PXB_OK;
  PXB_REQUIRE(grad && act, "pxb_backward_update: grad/act is NULL");
  return launch_backward(cap, from_id, to_id, dead, weight, grad, act, num_units, PXB_MONOID_SUM, acc, opt,
                         opt_m, opt_v, opt_t, as_stream(stream));
}

extern "C" int pxb_unit_apply(int32_t num_units, int32_t mode, int32_t act_kind, int32_t monoid, float *acc,
                              int64_t *acc_fixed, const float *act, const float *seed, const int32_t *level,
                              int32_t target_level,
                              const uint8_t *is_input, const uint8_t *pruned, float *out, void *stream) {
  PXB_REQUIRE(num_units >= 0, "pxb_unit_apply: negative num_units");
  PXB_REQUIRE(mode == 0 || mode == 1, "pxb_unit_apply: mode must be 0 (forward) or 1 (backward)");
  PXB_REQUIRE(act_code_ok(act_kind), "pxb_unit_apply: unknown activation code %d", act_kind);
  PXB_REQUIRE(monoid >= 0 && monoid <= 2, "pxb_unit_apply: unknown monoid %d", monoid);
  if (num_units == 0) return PXB_OK;
  PXB_REQUIRE(acc && out, "pxb_unit_apply: acc/out is NULL");
  PXB_REQUIRE(acc_fixed == nullptr || monoid == PXB_MONOID_SUM, "pxb_unit_apply: acc_fixed is for the sum monoid");
  PXB_REQUIRE(mode == 0 || act, "pxb_unit_apply: backward apply needs the activation column");
  unit_apply_kernel<<<(num_units + 255) / 256, 256, 0, as_stream(stream)>>>(
      num_units, mode, act_kind, monoid, acc, acc_fixed, act, seed, level, target_level, is_input, pruned, out);
  PXB_LAUNCHED("unit_apply_kernel");
  return PXB_OK;
}

extern "C" int pxb_mse_loss(int32_t num_outputs, const int32_t *output_ids, const float *act,
                            const float *target, float *seed, float *loss_out, void *stream) {
  PXB_REQUIRE(num_outputs >= 0, "pxb_mse_loss: negative output count");
  if (num_outputs == 0) return PXB_OK;
  PXB_REQUIRE(output_ids && act && target && seed, "pxb_mse_loss: a pointer is NULL");
  mse_loss_kernel<<<1, 256, 0, as_stream(stream)>>>(num_outputs, output_ids, act, target, seed, loss_out);
  PXB_LAUNCHED("mse_loss_kernel");
  return PXB_OK;
}

// ---------------------------------------------------------------------------
// lowest-|w| prune: keys for the selection, then the selected slots
// ---------------------------------------------------------------------------
namespace pxb {

// Candidate s of the bucket at global slot base + s: score -|w| (a dead
// slot -inf), id its global slot, so the total order's first k are the k
// lowest |w| with ties by ascending slot.
__global__ void lowest_keys_kernel(int64_t cap, const uint8_t *__restrict__ dead, const float *__restrict__ w,
                                   int64_t base, float *__restrict__ score, int32_t *__restrict__ slot) {
  for (int64_t s = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; s < cap;
       s += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    score[base + s] = dead[s] ? -__int_as_float(0x7f800000) : -fabsf(w[s]);
    slot[base + s] = static_cast<int32_t>(base + s);
  }
}

__global__ void prune_selected_kernel(int64_t k, const int32_t *__restrict__ idx, const float *__restrict__ score,
                                      int64_t base, int64_t cap, const int32_t *__restrict__ from,
                                      uint8_t *__restrict__ dead, uint32_t n, PruneArgs pa) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < k;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t g = idx[i];
    if (g < base || g >= base + cap) continue;
    if (!(score[g] > -__int_as_float(0x7f800000))) continue;  // a dead slot (or NaN weight) is not selected
    const int64_t s = g - base;
    if (dead[s]) continue;
    dead[s] = 1;
    mark_free(pa, s, pa.bm_level ? from[s] : 0, n);
  }
}

}  // namespace pxb

extern "C" int pxb_lowest_keys(int64_t cap, const uint8_t *dead, const float *weight, int64_t base, float *score_out,
                               int32_t *slot_out, void *stream) {
  PXB_REQUIRE(cap >= 0 && base >= 0 && base + cap < (int64_t(1) << 31), "pxb_lowest_keys: slots out of range");
  if (cap == 0) return PXB_OK;
  PXB_REQUIRE(dead && weight && score_out && slot_out, "pxb_lowest_keys: a pointer is NULL");
  pxb::lowest_keys_kernel<<<pxb::grid_for(cap, 256, 8), 256, 0, pxb::as_stream(stream)>>>(cap, dead, weight, base,
                                                                                         score_out, slot_out);
  PXB_LAUNCHED("lowest_keys_kernel");
  return PXB_OK;
}

extern "C" int pxb_prune_selected(int64_t k, const int32_t *idx, const float *score, int64_t base, int64_t cap,
                                  const int32_t *from_id, uint8_t *dead, int32_t num_units, uint32_t *free_bitmap,
                                  const int32_t *bitmap_level, void *stream) {
  PXB_REQUIRE(k >= 0 && cap >= 0 && base >= 0, "pxb_prune_selected: sizes out of range");
  if (k == 0 || cap == 0) return PXB_OK;
  PXB_REQUIRE(idx && score && from_id && dead, "pxb_prune_selected: a pointer is NULL");
  pxb::PruneArgs pa{PXB_PRUNE_NONE, 0.0f, nullptr, dead, true, -1, nullptr, free_bitmap, (cap + 31) / 32, bitmap_level};
  pxb::prune_selected_kernel<<<pxb::grid_for(k, 256, 4), 256, 0, pxb::as_stream(stream)>>>(
      k, idx, score, base, cap, from_id, dead, static_cast<uint32_t>(num_units), pa);
  PXB_LAUNCHED("prune_selected_kernel");
  return PXB_OK;
}
