/*
 * pxo.c -- CPU oracle for the plastax edge-arena hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This file restates the reference's algorithm in
 * plain sequential C so the CUDA engine (plastax_b200/csrc, libpxb.so) can be
 * checked against it, and so the reference's CPU cost can be timed on the
 * GPU box's host cores. Only tests/, __graft_entry__.smoke() and bench.py's
 * CPU-baseline leg load it; the engine never calls it and has no CPU path.
 *
 * Float semantics follow the reference's float32 evaluation: every product
 * and division rounds to float32 (built with -ffp-contract=off), and a
 * bucket's segment reduction starts from the monoid identity before it is
 * folded into the carried accumulator (src/plastax/sweep.py:157-175). A
 * segment sum is accumulated in double and rounded to float32 once, i.e. it
 * is the correctly rounded sum of the float32 products: XLA's float32
 * summation order is not pinned by the reference, and every order is an
 * approximation of this value, so the engine's tolerance is measured
 * against it rather than against one arbitrary order's rounding.
 *
 * Each function cites the reference lines it restates (paths within the
 * plastax project).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define PXO_SUM 0
#define PXO_MAX 1
#define PXO_MIN 2

/* ------------------------------------------------------------------ */
/* Philox-4x32-10 and the site RNG (src/plastax/rng.py:1-57, :109-142,  */
/* :207-246; scripts/parity/reference.py:147-225)                       */
/* ------------------------------------------------------------------ */
uint32_t pxo_philox32(uint64_t seed, uint64_t counter) {
  uint32_t x0 = (uint32_t)counter, x1 = (uint32_t)(counter >> 32);
  uint32_t x2 = (uint32_t)seed, x3 = (uint32_t)(seed >> 32);
  uint32_t k0 = x2, k1 = x3;
  for (int r = 0; r < 10; ++r) {
    uint64_t p0 = (uint64_t)0xD2511F53u * x0;
    uint64_t p1 = (uint64_t)0xCD9E8D57u * x2;
    uint32_t nx0 = (uint32_t)(p1 >> 32) ^ x1 ^ k0;
    uint32_t nx1 = (uint32_t)p1;
    uint32_t nx2 = (uint32_t)(p0 >> 32) ^ x3 ^ k1;
    uint32_t nx3 = (uint32_t)p0;
    x0 = nx0; x1 = nx1; x2 = nx2; x3 = nx3;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return x0;
}

void pxo_philox32_many(int64_t n, const uint64_t *seed, const uint64_t *ctr, uint32_t *out) {
  for (int64_t i = 0; i < n; ++i) out[i] = pxo_philox32(seed[i], ctr[i]);
}

float pxo_unit_float(uint32_t w) { return (float)(w >> 8) * (1.0f / 16777216.0f); }

uint32_t pxo_uniform_int(float u, uint32_t n) {
  volatile float scaled = u * (float)n;
  uint32_t v = (uint32_t)scaled;
  return v < n - 1 ? v : n - 1;
}

uint64_t pxo_site_seed(uint64_t network_seed, uint32_t step, uint32_t stream, uint32_t key) {
  uint64_t ctr = ((uint64_t)step << 8) | (stream & 0xFFu);
  return ((uint64_t)pxo_philox32(network_seed, ctr) << 32) | key;
}

/* ------------------------------------------------------------------ */
/* propagation                                                          */
/* ------------------------------------------------------------------ */
static float ident(int m) { return m == PXO_SUM ? 0.0f : (m == PXO_MAX ? -INFINITY : INFINITY); }
static float pair(int m, float a, float b) {
  if (m == PXO_SUM) return a + b;
  if (m == PXO_MAX) return a > b ? a : (b > a ? b : a);
  return a < b ? a : (b < a ? b : a);
}

/* Forward accumulate of one bucket, linear map w * act[from]
 * (src/plastax/sweep.py:113-180 with target TO_ID; the map of
 * examples/reservoir.py:59-70): dead slots go to the dropped null segment,
 * live ones reduce in slot order from the identity, then fold into acc. */
static double dpair(int m, double a, double b) {
  if (m == PXO_SUM) return a + b;
  if (m == PXO_MAX) return a > b ? a : b;
  return a < b ? a : b;
}

void pxo_forward_accumulate(int64_t cap, const int32_t *from, const int32_t *to, const uint8_t *dead,
                            const float *w, const float *act, int32_t n, int monoid, float *acc,
                            double *work /* n doubles */) {
  for (int32_t i = 0; i < n; ++i) work[i] = ident(monoid);
  for (int64_t s = 0; s < cap; ++s) {
    if (dead[s]) continue;
    int32_t f = from[s], t = to[s];
    if (f < 0 || f >= n || t < 0 || t >= n) continue;
    float v = w[s] * act[f];
    work[t] = dpair(monoid, work[t], v);
  }
  for (int32_t i = 0; i < n; ++i) acc[i] = pair(monoid, acc[i], (float)work[i]);
}

/* Backward accumulate (the same primitive with target FROM_ID,
 * src/plastax/sweep.py:343-400): acc[from] (+)= w * grad[to]. */
void pxo_backward_accumulate(int64_t cap, const int32_t *from, const int32_t *to, const uint8_t *dead,
                             const float *w, const float *grad, int32_t n, int monoid, float *acc,
                             double *work /* n doubles */) {
  for (int32_t i = 0; i < n; ++i) work[i] = ident(monoid);
  for (int64_t s = 0; s < cap; ++s) {
    if (dead[s]) continue;
    int32_t f = from[s], t = to[s];
    if (f < 0 || f >= n || t < 0 || t >= n) continue;
    float v = w[s] * grad[t];
    work[f] = dpair(monoid, work[f], v);
  }
  for (int32_t i = 0; i < n; ++i) acc[i] = pair(monoid, acc[i], (float)work[i]);
}

/* Prune sweep (src/plastax/phases.py:1444-1498): dead |= predicate; kind 1
 * |w| < thr, kind 2 |w| < unit_thr[to]. Per-block free counts
 * (src/plastax/phases.py:2595-2623) when block_free != NULL. */
void pxo_prune(int64_t cap, const int32_t *to, uint8_t *dead, const float *w, int32_t n, int kind, float thr,
               const float *unit_thr, int32_t block_len, int32_t *block_free) {
  for (int64_t s = 0; s < cap; ++s) {
    int p = 0;
    if (kind == 1) p = fabsf(w[s]) < thr;
    else if (kind == 2) p = to[s] >= 0 && to[s] < n && fabsf(w[s]) < unit_thr[to[s]];
    dead[s] = dead[s] | (uint8_t)p;
  }
  if (block_free) {
    int64_t blocks = (cap + block_len - 1) / block_len;
    for (int64_t b = 0; b < blocks; ++b) block_free[b] = 0;
    for (int64_t s = 0; s < cap; ++s) block_free[s / block_len] += dead[s] ? 1 : 0;
  }
}

/* Optimizer step (src/plastax/optim/_sgd.py:124-127, _momentum.py:136-139,
 * _adam.py:157-172, _rmsprop.py:135-140). */
typedef struct {
  int32_t kind;
  float lr, b1, b2, eps, wd;
} pxo_opt;

static void opt_step(const pxo_opt *p, float g, float *w, float *m, float *v, float *t) {
  switch (p->kind) {
    case 0: *w = *w - p->lr * g; break;
    case 1: { float vel = p->b1 * *v + g; *v = vel; *w = *w - p->lr * vel; break; }
    case 2: {
      float step = *t + 1.0f;
      float mm = p->b1 * *m + (1.0f - p->b1) * g;
      float vv = p->b2 * *v + (1.0f - p->b2) * (g * g);
      float m_hat = mm / (1.0f - powf(p->b1, step));
      float v_hat = vv / (1.0f - powf(p->b2, step));
      float dir = m_hat / (sqrtf(v_hat) + p->eps);
      *w = *w - p->lr * (dir + p->wd * *w);
      *m = mm; *v = vv; *t = step;
      break;
    }
    case 3: {
      float ms = p->b1 * *v + (1.0f - p->b1) * (g * g);
      *v = ms;
      *w = *w - (p->lr * g) / sqrtf(ms + p->eps);
      break;
    }
    default: break;
  }
}

/* Incoming conn update of one bucket (src/plastax/sweep.py:488-532,
 * src/plastax/phases.py:1196-1242): live slots take one optimizer step on
 * the delta-rule gradient grad[to] * act[from]; dead slots keep their values. */
void pxo_update_conn(int64_t cap, const int32_t *from, const int32_t *to, const uint8_t *dead, float *w,
                     const float *grad, const float *act, int32_t n, const pxo_opt *opt, float *m, float *v,
                     float *t) {
  float dm = 0, dv = 0, dt = 0;
  for (int64_t s = 0; s < cap; ++s) {
    if (dead[s]) continue;
    int32_t f = from[s], tt = to[s];
    if (f < 0 || f >= n || tt < 0 || tt >= n) continue;
    float g = grad[tt] * act[f];
    opt_step(opt, g, w + s, m ? m + s : &dm, v ? v + s : &dv, t ? t + s : &dt);
  }
}

/* Batched exact update (src/plastax/phases.py:434-483): per live slot the
 * per-sample gradients are summed over b = 0..B-1 in order, divided by B,
 * then one optimizer step. g and a are [n, B]. */
void pxo_batched_update(int64_t cap, const int32_t *from, const int32_t *to, const uint8_t *dead, float *w,
                        const float *g, const float *a, int32_t batch, int32_t n, const pxo_opt *opt, float *m,
                        float *v, float *t) {
  float dm = 0, dv = 0, dt = 0;
  for (int64_t s = 0; s < cap; ++s) {
    if (dead[s]) continue;
    int32_t f = from[s], tt = to[s];
    if (f < 0 || f >= n || tt < 0 || tt >= n) continue;
    float total = 0.0f;
    for (int32_t b = 0; b < batch; ++b) total = total + g[(int64_t)tt * batch + b] * a[(int64_t)f * batch + b];
    float stat = total / (float)batch;
    opt_step(opt, stat, w + s, m ? m + s : &dm, v ? v + s : &dv, t ? t + s : &dt);
  }
}

/* Batched products: out[to, :] += w * x[from, :] (forward) or
 * out[from, :] += w * x[to, :] (backward), slot order. */
void pxo_batched_product(int64_t cap, const int32_t *from, const int32_t *to, const uint8_t *dead, const float *w,
                         const float *x, int32_t batch, int32_t n, int backward, float *out) {
  for (int64_t s = 0; s < cap; ++s) {
    if (dead[s]) continue;
    int32_t f = from[s], t = to[s];
    if (f < 0 || f >= n || t < 0 || t >= n) continue;
    int32_t src_row = backward ? t : f, dst_row = backward ? f : t;
    for (int32_t b = 0; b < batch; ++b)
      out[(int64_t)dst_row * batch + b] += w[s] * x[(int64_t)src_row * batch + b];
  }
}

static float act_fn(int k, float x) {
  if (k == 1) return tanhf(x);
  if (k == 2) return x > 0.0f ? x : 0.0f;
  if (k == 3) return 1.0f / (1.0f + expf(-x));
  return x;
}
static float act_prime(int k, float a) {
  if (k == 1) return 1.0f - a * a;
  if (k == 2) return a > 0.0f ? 1.0f : 0.0f;
  if (k == 3) return a * (1.0f - a);
  return 1.0f;
}

/* Masked apply (src/plastax/sweep.py:183-230): finalized units get the
 * apply write and an identity accumulator; others keep both. */
void pxo_unit_apply(int32_t n, int mode, int act_kind, int monoid, float *acc, const float *act, const float *seed,
                    const int32_t *level, int32_t target_level, const uint8_t *is_input, const uint8_t *pruned,
                    float *out) {
  for (int32_t i = 0; i < n; ++i) {
    if (level && level[i] != target_level) continue;
    if (is_input && is_input[i]) continue;
    if (pruned && pruned[i]) continue;
    if (mode == 0) out[i] = act_fn(act_kind, acc[i]);
    else out[i] = (acc[i] + (seed ? seed[i] : 0.0f)) * act_prime(act_kind, act[i]);
    acc[i] = ident(monoid);
  }
}

/* ------------------------------------------------------------------ */
/* growth                                                               */
/* ------------------------------------------------------------------ */

/* Per-unit proposals + validity (src/plastax/phases.py:3813-3860,
 * :4041-4108): candidate i*P+j from site (seed, step, 1, i, j);
 * dst = dst_lo + uniform_int(dst_n) at sub 0, score at sub 1 (kind 0
 * uniform, 1 floor(u*256)/256 as scripts/parity/golden_rules.py
 * hash_propose_v1, 2 |grad[dst]*act[src]|). */
static void propose_unit(int32_t i, int32_t n, int32_t P, uint64_t network_seed, int32_t step, int32_t dst_lo,
                         int32_t dst_n, int score_kind, const float *grad, const float *act, const int32_t *level,
                         const uint8_t *pruned, int32_t max_gap, int direction, int self_loops,
                         int32_t bucket_level, int32_t src_level_bound, int32_t *src_out, int32_t *dst_out,
                         float *score_out);

void pxo_propose_per_unit(int32_t n, int32_t P, uint64_t network_seed, int32_t step, int32_t dst_lo, int32_t dst_n,
                          int score_kind, const float *grad, const float *act, const int32_t *level,
                          const uint8_t *pruned, int32_t max_gap, int direction, int self_loops, int32_t bucket_level,
                          int32_t src_level_bound, int32_t *src_out, int32_t *dst_out, float *score_out) {
  for (int32_t i = 0; i < n; ++i)
    propose_unit(i, n, P, network_seed, step, dst_lo, dst_n, score_kind, grad, act, level, pruned, max_gap,
                 direction, self_loops, bucket_level, src_level_bound, src_out, dst_out, score_out);
}

/* The same proposals with the units split over `threads` threads (each
 * unit's candidates depend on the unit alone). */
void pxo_propose_per_unit_mt(int32_t n, int32_t P, uint64_t network_seed, int32_t step, int32_t dst_lo,
                             int32_t dst_n, int score_kind, const float *grad, const float *act,
                             const int32_t *level, const uint8_t *pruned, int32_t max_gap, int direction,
                             int self_loops, int32_t bucket_level, int32_t src_level_bound, int32_t *src_out,
                             int32_t *dst_out, float *score_out, int threads) {
  if (threads < 1) threads = 1;
#pragma omp parallel for schedule(static) num_threads(threads)
  for (int32_t i = 0; i < n; ++i)
    propose_unit(i, n, P, network_seed, step, dst_lo, dst_n, score_kind, grad, act, level, pruned, max_gap,
                 direction, self_loops, bucket_level, src_level_bound, src_out, dst_out, score_out);
}

static void propose_unit(int32_t i, int32_t n, int32_t P, uint64_t network_seed, int32_t step, int32_t dst_lo,
                         int32_t dst_n, int score_kind, const float *grad, const float *act, const int32_t *level,
                         const uint8_t *pruned, int32_t max_gap, int direction, int self_loops,
                         int32_t bucket_level, int32_t src_level_bound, int32_t *src_out, int32_t *dst_out,
                         float *score_out) {
  {
    uint64_t seed = pxo_site_seed(network_seed, (uint32_t)step, 1, (uint32_t)i);
    for (int32_t j = 0; j < P; ++j) {
      int64_t c = (int64_t)i * P + j;
      uint32_t w0 = pxo_philox32(seed, ((uint64_t)(uint32_t)j << 16) | 0u);
      int32_t src = i;
      int32_t dst = dst_lo + (int32_t)pxo_uniform_int(pxo_unit_float(w0), (uint32_t)dst_n);
      float score;
      if (score_kind == 0) {
        score = pxo_unit_float(pxo_philox32(seed, ((uint64_t)(uint32_t)j << 16) | 1u));
      } else if (score_kind == 1) {
        float u = pxo_unit_float(pxo_philox32(seed, ((uint64_t)(uint32_t)j << 16) | 1u));
        volatile float su = u * 256.0f;
        score = (float)(int32_t)su / 256.0f;
      } else {
        score = (dst >= 0 && dst < n) ? fabsf(grad[dst] * act[src]) : 0.0f;
      }
      int valid = dst >= 0 && dst < n;
      if (!valid) { src = 0; dst = 0; }
      if (valid && pruned) valid = !pruned[src] && !pruned[dst];
      if (valid) {
        int32_t ls = level[src], ld = level[dst];
        int32_t gap = ld > ls ? ld - ls : ls - ld;
        valid = gap <= max_gap;
        if (!self_loops) valid = valid && src != dst;
        if (direction == 1) valid = valid && ld > ls;
        else if (direction == 2) valid = valid && ld >= ls;
        if (bucket_level >= 0) valid = valid && ls == bucket_level;
        if (src_level_bound > 0) valid = valid && ls < src_level_bound;
      }
      if (!valid || !isfinite(score)) score = -INFINITY;
      src_out[c] = src;
      dst_out[c] = dst;
      score_out[c] = score;
    }
  }
}

/* Total order (src/plastax/phases.py:4208-4321): ascending by
 * (-score with NaN -> +inf and -0 == +0, src, dst, candidate index). */
typedef struct {
  float key;
  int32_t src, dst, idx;
} order_item;

static int order_cmp(const void *pa, const void *pb) {
  const order_item *a = (const order_item *)pa, *b = (const order_item *)pb;
  if (a->key < b->key) return -1;
  if (a->key > b->key) return 1;
  if (a->src != b->src) return a->src < b->src ? -1 : 1;
  if (a->dst != b->dst) return a->dst < b->dst ? -1 : 1;
  return a->idx < b->idx ? -1 : (a->idx > b->idx);
}

void pxo_total_order(int64_t n, const float *score, const int32_t *src, const int32_t *dst, int32_t *perm) {
  order_item *it = (order_item *)malloc(sizeof(order_item) * (n > 0 ? n : 1));
  for (int64_t i = 0; i < n; ++i) {
    float k = isnan(score[i]) ? INFINITY : -score[i];
    if (k == 0.0f) k = 0.0f;
    it[i].key = k;
    it[i].src = src[i];
    it[i].dst = dst[i];
    it[i].idx = (int32_t)i;
  }
  qsort(it, (size_t)n, sizeof(order_item), order_cmp);
  for (int64_t i = 0; i < n; ++i) perm[i] = it[i].idx;
  free(it);
}

/* The same order with the items sorted in `threads` chunks, then merged
 * pairwise (the order is total, so the result is the sequential one). */
void pxo_total_order_mt(int64_t n, const float *score, const int32_t *src, const int32_t *dst, int32_t *perm,
                        int threads) {
  if (threads < 1) threads = 1;
  if (n < 2 * (int64_t)threads || threads == 1) {
    pxo_total_order(n, score, src, dst, perm);
    return;
  }
  order_item *a = (order_item *)malloc(sizeof(order_item) * n);
  order_item *b = (order_item *)malloc(sizeof(order_item) * n);
  int64_t *bound = (int64_t *)malloc(sizeof(int64_t) * (threads + 1));
  for (int t = 0; t <= threads; ++t) bound[t] = n * t / threads;
#pragma omp parallel for schedule(static) num_threads(threads)
  for (int64_t i = 0; i < n; ++i) {
    float k = isnan(score[i]) ? INFINITY : -score[i];
    if (k == 0.0f) k = 0.0f;
    a[i].key = k;
    a[i].src = src[i];
    a[i].dst = dst[i];
    a[i].idx = (int32_t)i;
  }
#pragma omp parallel for schedule(static, 1) num_threads(threads)
  for (int t = 0; t < threads; ++t) qsort(a + bound[t], (size_t)(bound[t + 1] - bound[t]), sizeof(order_item), order_cmp);
  int runs = threads;
  int64_t *rb = bound;
  while (runs > 1) {
    int pairs = runs / 2;
#pragma omp parallel for schedule(static, 1) num_threads(threads)
    for (int q = 0; q < pairs; ++q) {
      int64_t i = rb[2 * q], mid = rb[2 * q + 1], end = rb[2 * q + 2], j = mid, o = rb[2 * q];
      while (i < mid && j < end) b[o++] = order_cmp(&a[j], &a[i]) < 0 ? a[j++] : a[i++];
      while (i < mid) b[o++] = a[i++];
      while (j < end) b[o++] = a[j++];
    }
    if (runs % 2) {  /* the odd run out is copied as it is */
      for (int64_t i = rb[runs - 1]; i < rb[runs]; ++i) b[i] = a[i];
    }
    for (int q = 0; q < pairs; ++q) rb[q + 1] = rb[2 * q + 2];
    if (runs % 2) rb[pairs + 1] = rb[runs];
    runs = pairs + runs % 2;
    order_item *tmp = a;
    a = b;
    b = tmp;
  }
  for (int64_t i = 0; i < n; ++i) perm[i] = a[i].idx;
  free(a);
  free(b);
  free(bound);
}

/* Step-scoped selection + level-major relisting (src/plastax/phases.py:
 * 4891-4903, 4469-4487): the first min(k, n) of perm, stable by level. */
int64_t pxo_select_step(int64_t n, const int32_t *perm, const int32_t *src, const int32_t *level, int64_t k,
                        int32_t *win) {
  int64_t kk = k < n ? k : n;
  int32_t maxl = 0;
  for (int64_t i = 0; i < kk; ++i) {
    int32_t l = level[src[perm[i]]];
    if (l > maxl) maxl = l;
  }
  int64_t o = 0;
  for (int32_t l = 0; l <= maxl; ++l)
    for (int64_t i = 0; i < kk; ++i)
      if (level[src[perm[i]]] == l) win[o++] = perm[i];
  return kk;
}

/* Per-segment selection (src/plastax/phases.py:4356-4423): each segment's
 * first k members of the total order. win is [num_seg, k], filled[num_seg]
 * gets the member count (capped at k). */
void pxo_select_per_segment(int64_t n, const int32_t *perm, const int32_t *segment, int32_t num_seg, int64_t k,
                            int32_t *win, int32_t *filled) {
  for (int32_t s = 0; s < num_seg; ++s) filled[s] = 0;
  for (int64_t i = 0; i < n; ++i) {
    int32_t sg = segment[perm[i]];
    if (sg < 0 || sg >= num_seg) continue;
    if (filled[sg] < k) win[(int64_t)sg * k + filled[sg]++] = perm[i];
  }
}

/* ------------------------------------------------------------------ */
/* slot claim                                                           */
/* ------------------------------------------------------------------ */
typedef struct {
  int32_t n_extra;
  void *cols[8];
  int32_t bytes[8];
  const void *vals[8];
} pxo_extra;

static void write_slot(int64_t slot, int64_t i, int32_t *from, int32_t *to, uint8_t *dead, float *w,
                       const int32_t *cs, const int32_t *cd, const float *cw, const pxo_extra *ex) {
  from[slot] = cs[i];
  to[slot] = cd[i];
  w[slot] = cw[i];
  if (ex)
    for (int e = 0; e < ex->n_extra; ++e) {
      if (ex->bytes[e] == 4) ((int32_t *)ex->cols[e])[slot] = ((const int32_t *)ex->vals[e])[i];
      else ((uint8_t *)ex->cols[e])[slot] = ((const uint8_t *)ex->vals[e])[i];
    }
  dead[slot] = 0;
}

/* Pipeline claim (src/plastax/phases.py:2985-3106), one device: candidates
 * stably ordered by level (non-growable last); each level's first
 * total[level] take the level's dead slots below tail_start in slot order
 * (domain = level[from_id]); the rest spill to tail_start + spill rank,
 * levels ascending, up to cap. counts = {committed, overflowed, tail used,
 * violating}. max_new >= 0 caps the growable candidates in claim order. */
static void claim_pipeline_assign(int64_t cap, int32_t *from, int32_t *to, uint8_t *dead, float *w,
                                  const int32_t *level, int32_t n, int32_t num_levels, int64_t *tail_start, int64_t k,
                                  const int32_t *cs, const int32_t *cd, const float *cw, const uint8_t *growable_in,
                                  int64_t max_new, const pxo_extra *ex, int32_t *counts, uint8_t *overflowed,
                                  int64_t *cnt, int64_t *start, int64_t *lists);

static inline int32_t slot_domain(const int32_t *from, const int32_t *level, int32_t n, int64_t s) {
  int32_t o = from[s] < 0 ? 0 : (from[s] >= n ? n - 1 : from[s]);
  return level[o];
}

void pxo_claim_pipeline(int64_t cap, int32_t *from, int32_t *to, uint8_t *dead, float *w, const int32_t *level,
                        int32_t n, int64_t *tail_start, int64_t k, const int32_t *cs, const int32_t *cd,
                        const float *cw, const uint8_t *growable_in, int64_t max_new, const pxo_extra *ex,
                        int32_t *counts, uint8_t *overflowed) {
  int32_t num_levels = 1;
  for (int32_t i = 0; i < n; ++i) if (level[i] + 1 > num_levels) num_levels = level[i] + 1;
  int64_t tail = *tail_start;
  /* per-level dead slot lists in slot order */
  int64_t *cnt = (int64_t *)calloc(num_levels, sizeof(int64_t));
  for (int64_t s = 0; s < cap && s < tail; ++s)
    if (dead[s]) cnt[slot_domain(from, level, n, s)]++;
  int64_t *start = (int64_t *)calloc(num_levels + 1, sizeof(int64_t));
  for (int32_t l = 0; l < num_levels; ++l) start[l + 1] = start[l] + cnt[l];
  int64_t *lists = (int64_t *)malloc(sizeof(int64_t) * (start[num_levels] > 0 ? start[num_levels] : 1));
  int64_t *fill = (int64_t *)calloc(num_levels, sizeof(int64_t));
  for (int64_t s = 0; s < cap && s < tail; ++s)
    if (dead[s]) {
      int32_t l = slot_domain(from, level, n, s);
      lists[start[l] + fill[l]++] = s;
    }
  free(fill);
  claim_pipeline_assign(cap, from, to, dead, w, level, n, num_levels, tail_start, k, cs, cd, cw, growable_in, max_new,
                        ex, counts, overflowed, cnt, start, lists);
}

/* The same claim with the per-domain dead-slot lists built by `threads`
 * threads over contiguous slot ranges (each range's entries land after the
 * ranges before it, so the lists keep slot order); the assignment of the
 * candidates, in list order, is the sequential one. */
void pxo_claim_pipeline_mt(int64_t cap, int32_t *from, int32_t *to, uint8_t *dead, float *w, const int32_t *level,
                           int32_t n, int64_t *tail_start, int64_t k, const int32_t *cs, const int32_t *cd,
                           const float *cw, const uint8_t *growable_in, int64_t max_new, const pxo_extra *ex,
                           int32_t *counts, uint8_t *overflowed, int threads) {
  if (threads < 1) threads = 1;
  int32_t num_levels = 1;
  for (int32_t i = 0; i < n; ++i) if (level[i] + 1 > num_levels) num_levels = level[i] + 1;
  const int64_t tail = *tail_start, lim = cap < tail ? cap : tail;
  int64_t *tc = (int64_t *)calloc((size_t)threads * num_levels, sizeof(int64_t));
#pragma omp parallel for schedule(static, 1) num_threads(threads)
  for (int t = 0; t < threads; ++t) {
    const int64_t lo = lim * t / threads, hi = lim * (t + 1) / threads;
    int64_t *mine = tc + (int64_t)t * num_levels;
    for (int64_t s = lo; s < hi; ++s)
      if (dead[s]) mine[slot_domain(from, level, n, s)]++;
  }
  int64_t *cnt = (int64_t *)calloc(num_levels, sizeof(int64_t));
  int64_t *start = (int64_t *)calloc(num_levels + 1, sizeof(int64_t));
  for (int32_t l = 0; l < num_levels; ++l)
    for (int t = 0; t < threads; ++t) cnt[l] += tc[(int64_t)t * num_levels + l];
  for (int32_t l = 0; l < num_levels; ++l) start[l + 1] = start[l] + cnt[l];
  /* each thread's first list position per domain */
  int64_t *toff = (int64_t *)calloc((size_t)threads * num_levels, sizeof(int64_t));
  for (int32_t l = 0; l < num_levels; ++l) {
    int64_t run = start[l];
    for (int t = 0; t < threads; ++t) {
      toff[(int64_t)t * num_levels + l] = run;
      run += tc[(int64_t)t * num_levels + l];
    }
  }
  int64_t *lists = (int64_t *)malloc(sizeof(int64_t) * (start[num_levels] > 0 ? start[num_levels] : 1));
#pragma omp parallel for schedule(static, 1) num_threads(threads)
  for (int t = 0; t < threads; ++t) {
    const int64_t lo = lim * t / threads, hi = lim * (t + 1) / threads;
    int64_t *pos = toff + (int64_t)t * num_levels;
    for (int64_t s = lo; s < hi; ++s)
      if (dead[s]) lists[pos[slot_domain(from, level, n, s)]++] = s;
  }
  free(tc);
  free(toff);
  claim_pipeline_assign(cap, from, to, dead, w, level, n, num_levels, tail_start, k, cs, cd, cw, growable_in, max_new,
                        ex, counts, overflowed, cnt, start, lists);
}

static void claim_pipeline_assign(int64_t cap, int32_t *from, int32_t *to, uint8_t *dead, float *w,
                                  const int32_t *level, int32_t n, int32_t num_levels, int64_t *tail_start, int64_t k,
                                  const int32_t *cs, const int32_t *cd, const float *cw, const uint8_t *growable_in,
                                  int64_t max_new, const pxo_extra *ex, int32_t *counts, uint8_t *overflowed,
                                  int64_t *cnt, int64_t *start, int64_t *lists) {
  const int64_t tail = *tail_start;
  uint8_t *grow = (uint8_t *)malloc(k > 0 ? k : 1);
  int64_t rank = 0;
  for (int64_t i = 0; i < k; ++i) {
    grow[i] = growable_in[i];
    if (grow[i]) {
      if (max_new >= 0 && rank >= max_new) grow[i] = 0;
      rank++;
    }
  }
  int64_t *taken = (int64_t *)calloc(num_levels, sizeof(int64_t));
  int64_t spill = 0, tail_free = cap - tail;
  counts[0] = counts[1] = counts[2] = counts[3] = 0;
  for (int64_t i = 0; i < k; ++i) overflowed[i] = 0;
  for (int32_t l = 0; l < num_levels; ++l) {
    for (int64_t i = 0; i < k; ++i) {
      if (!grow[i]) continue;
      int32_t sc = cs[i] < 0 ? 0 : (cs[i] >= n ? n - 1 : cs[i]);
      if (level[sc] != l) continue;
      int64_t slot = -1;
      if (taken[l] < cnt[l]) {
        slot = lists[start[l] + taken[l]++];
      } else if (spill < tail_free) {
        slot = tail + spill++;
        counts[2]++;
      } else {
        overflowed[i] = 1;
        counts[1]++;
        continue;
      }
      counts[0]++;
      if (level[cd[i]] <= level[cs[i]]) counts[3]++;
      write_slot(slot, i, from, to, dead, w, cs, cd, cw, ex);
    }
  }
  *tail_start = tail + counts[2];
  free(cnt); free(start); free(lists); free(grow); free(taken);
}

/* Topological claim of one bucket (src/plastax/phases.py:2853-2982): the
 * i-th growable candidate takes the i-th dead slot in slot order. */
void pxo_claim_topological(int64_t cap, int32_t *from, int32_t *to, uint8_t *dead, float *w, const int32_t *level,
                           int32_t n, int64_t k, const int32_t *cs, const int32_t *cd, const float *cw,
                           const uint8_t *growable, int64_t max_new, const pxo_extra *ex, int32_t *counts,
                           uint8_t *overflowed) {
  int64_t nfree = 0;
  for (int64_t s = 0; s < cap; ++s) nfree += dead[s] ? 1 : 0;
  int64_t *slots = (int64_t *)malloc(sizeof(int64_t) * (nfree > 0 ? nfree : 1));
  int64_t f = 0;
  for (int64_t s = 0; s < cap; ++s) if (dead[s]) slots[f++] = s;
  counts[0] = counts[1] = counts[2] = counts[3] = 0;
  int64_t rank = 0, grank = 0;
  for (int64_t i = 0; i < k; ++i) {
    overflowed[i] = 0;
    if (!growable[i]) continue;
    if (max_new >= 0 && grank++ >= max_new) continue;
    if (rank < nfree) {
      int64_t slot = slots[rank++];
      counts[0]++;
      if (level[cd[i]] <= level[cs[i]]) counts[3]++;
      write_slot(slot, i, from, to, dead, w, cs, cd, cw, ex);
    } else {
      overflowed[i] = 1;
      counts[1]++;
    }
  }
  free(slots);
}

/* ------------------------------------------------------------------ */
/* multi-threaded variant of the forward + prune sweep (the CPU        */
/* baseline): per-thread private double accumulators over contiguous   */
/* slot ranges, then a fold in double and one rounding per unit.       */
/* ------------------------------------------------------------------ */
void pxo_forward_prune_mt(int64_t cap, const int32_t *from, const int32_t *to, uint8_t *dead, const float *w,
                          const float *act, int32_t n, float thr, float *acc, int threads,
                          double *work /* threads*n */) {
#ifdef _OPENMP
  if (threads < 1) threads = 1;
#pragma omp parallel num_threads(threads)
  {
    int tid = omp_get_thread_num(), nt = omp_get_num_threads();
    double *mine = work + (int64_t)tid * n;
    for (int32_t i = 0; i < n; ++i) mine[i] = 0.0;
    int64_t lo = cap * tid / nt, hi = cap * (tid + 1) / nt;
    for (int64_t s = lo; s < hi; ++s) {
      uint8_t d = dead[s];
      if (!d) {
        int32_t f = from[s], t = to[s];
        if (f >= 0 && f < n && t >= 0 && t < n) {
          float v = w[s] * act[f];
          mine[t] += v;
        }
      }
      if (fabsf(w[s]) < thr) dead[s] = 1;
    }
#pragma omp barrier
#pragma omp for schedule(static)
    for (int32_t i = 0; i < n; ++i) {
      double v = 0.0;
      for (int q = 0; q < nt; ++q) v += work[(int64_t)q * n + i];
      acc[i] = acc[i] + (float)v;
    }
  }
#else
  (void)threads;
  for (int32_t i = 0; i < n; ++i) work[i] = 0.0;
  for (int64_t s = 0; s < cap; ++s) {
    if (!dead[s]) {
      int32_t f = from[s], t = to[s];
      if (f >= 0 && f < n && t >= 0 && t < n) {
        float v = w[s] * act[f];
        work[t] += v;
      }
    }
    if (fabsf(w[s]) < thr) dead[s] = 1;
  }
  for (int32_t i = 0; i < n; ++i) acc[i] = acc[i] + (float)work[i];
#endif
}

/* ------------------------------------------------------------------ */
/* The lowest-magnitude prune of the churn configurations: the k live   */
/* edges of lowest |w| (ties by ascending slot, a NaN weight never) are */
/* tombstoned -- the predicate prune of src/plastax/phases.py:1444-1498 */
/* with the k-th smallest |w| as its threshold, the one the reference's */
/* churn computes from the current weights before each firing           */
/* (examples/dst_sparse.py:88-140), ties cut by slot so exactly k go.   */
/* Found by a histogram of bits(|w|) >> 15 (|w|'s bit pattern is        */
/* monotone in |w|), then a sort of the threshold bin's (bits, slot).   */
/* Returns the number pruned.                                           */
/* ------------------------------------------------------------------ */
#define PXO_LOWK_BINS 65536
#define PXO_INF_BITS 0x7f800000u

static inline uint32_t abs_bits(float w) {
  uint32_t u;
  memcpy(&u, &w, 4);
  return u & 0x7fffffffu;
}

static int key_cmp(const void *pa, const void *pb) {
  const uint64_t a = *(const uint64_t *)pa, b = *(const uint64_t *)pb;
  return a < b ? -1 : (a > b ? 1 : 0);
}

int64_t pxo_lowest_prune(int64_t cap, uint8_t *dead, const float *w, int64_t k, int threads) {
  if (k <= 0 || cap <= 0) return 0;
  if (threads < 1) threads = 1;
  int64_t *hist = (int64_t *)calloc((size_t)threads * PXO_LOWK_BINS, sizeof(int64_t));
#ifdef _OPENMP
#pragma omp parallel num_threads(threads)
#endif
  {
#ifdef _OPENMP
    const int tid = omp_get_thread_num(), nt = omp_get_num_threads();
#else
    const int tid = 0, nt = 1;
#endif
    int64_t *mine = hist + (int64_t)tid * PXO_LOWK_BINS;
    const int64_t lo = cap * tid / nt, hi = cap * (tid + 1) / nt;
    for (int64_t s = lo; s < hi; ++s) {
      if (dead[s]) continue;
      const uint32_t b = abs_bits(w[s]);
      if (b <= PXO_INF_BITS) mine[b >> 15]++;
    }
  }
  for (int t = 1; t < threads; ++t)
    for (int j = 0; j < PXO_LOWK_BINS; ++j) hist[j] += hist[(int64_t)t * PXO_LOWK_BINS + j];
  int64_t below = 0, total = 0;
  int bin = -1;
  for (int j = 0; j < PXO_LOWK_BINS; ++j) total += hist[j];
  if (total > k) {
    for (int j = 0; j < PXO_LOWK_BINS; ++j) {
      if (below + hist[j] >= k) {
        bin = j;
        break;
      }
      below += hist[j];
    }
  }
  /* edges with bits < lo go; of [lo, hi) the `take` smallest (bits, slot) */
  uint32_t lo_bits, hi_bits;
  int64_t take = 0, in_bin = 0;
  if (bin < 0) {
    lo_bits = hi_bits = PXO_INF_BITS + 1;
  } else {
    take = k - below;
    in_bin = hist[bin];
    lo_bits = (uint32_t)bin << 15;
    hi_bits = (uint32_t)(bin + 1) << 15;
    if (hi_bits > PXO_INF_BITS + 1) hi_bits = PXO_INF_BITS + 1;
    if (take == in_bin) {
      lo_bits = hi_bits;
      take = 0;
    }
  }
  free(hist);
  uint64_t *ties = take > 0 ? (uint64_t *)malloc((size_t)in_bin * sizeof(uint64_t)) : NULL;
  int64_t n_ties = 0, pruned = 0;
#ifdef _OPENMP
#pragma omp parallel for schedule(static) num_threads(threads) reduction(+ : pruned)
#endif
  for (int64_t s = 0; s < cap; ++s) {
    if (dead[s]) continue;
    const uint32_t b = abs_bits(w[s]);
    if (b < lo_bits) {
      dead[s] = 1;
      ++pruned;
    } else if (b < hi_bits && ties != NULL) {
      int64_t i;
#ifdef _OPENMP
#pragma omp atomic capture
#endif
      i = n_ties++;
      if (i < in_bin) ties[i] = ((uint64_t)b << 32) | (uint64_t)(uint32_t)s;
    }
  }
  if (ties != NULL) {
    if (n_ties > in_bin) n_ties = in_bin;
    qsort(ties, (size_t)n_ties, sizeof(uint64_t), key_cmp);
    for (int64_t i = 0; i < take && i < n_ties; ++i) {
      dead[(int64_t)(uint32_t)ties[i]] = 1;
      ++pruned;
    }
    free(ties);
  }
  return pruned;
}

int pxo_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* Stable counting sort of slots by an integer key in [0, num_keys): the
 * source-major order NetworkBuilder.from_edges gives a bucket whose edges
 * were generated in ascending-destination order per source
 * (src/plastax/builder.py:569-580). Used only to build CPU-baseline arenas. */
void pxo_stable_order_by_key(int64_t n, const int32_t *key, int32_t num_keys, int64_t *perm) {
  int64_t *start = (int64_t *)calloc((size_t)num_keys + 1, sizeof(int64_t));
  for (int64_t i = 0; i < n; ++i) start[key[i] + 1]++;
  for (int32_t k = 0; k < num_keys; ++k) start[k + 1] += start[k];
  for (int64_t i = 0; i < n; ++i) perm[start[key[i]]++] = i;
  free(start);
}
