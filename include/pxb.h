/*
 * pxb.h -- C ABI of the B200 edge-arena engine (libpxb.so).
 *
 * Every entry point takes plain device pointers, element counts and an
 * opaque CUDA stream (`void *stream`, a `cudaStream_t`; NULL = legacy
 * default stream). Nothing here allocates device memory: scratch is passed
 * in by the caller (sizes come from the matching `*_scratch_bytes` query),
 * and outputs the reference zero-fills are cleared by the callee on the
 * stream. No call synchronises the host with the device.
 *
 * Return value: 0 on success, otherwise a PXB_E* code. `pxb_last_error()`
 * returns a thread-local message for the last failing call on the calling
 * host thread. Argument errors are detected on the host before any launch.
 *
 * Arena layout (one bucket; every column has `cap` entries, struct of
 * arrays, slot order = the reference's slot order):
 *   from_id  int32   source unit of the slot
 *   to_id    int32   destination unit of the slot
 *   dead     uint8   1 = tombstoned / never used, 0 = live
 *   weight   float32
 *   opt[0..2] float32 optimizer columns (opt/m, opt/v, opt/t ...), optional
 *
 * Citations name the reference function (path within the plastax project)
 * each entry point stands in for.
 */
#ifndef PXB_H_
#define PXB_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PXB_ABI_VERSION 1

/* exported from libpxb.so (built with hidden default visibility) */
#if defined(__GNUC__)
#define PXB_API __attribute__((visibility("default")))
#else
#define PXB_API
#endif

/* status codes */
#define PXB_OK 0
#define PXB_EINVAL 1     /* bad argument (null pointer, size, enum)      */
#define PXB_ECUDA 2      /* a CUDA runtime call failed                   */
#define PXB_ESCRATCH 3   /* scratch buffer too small                     */
#define PXB_EUNSUPPORTED 4

/* monoids: src/plastax/monoid.py:27-59 (identities sum 0, max -inf, min +inf) */
#define PXB_MONOID_SUM 0
#define PXB_MONOID_MAX 1
#define PXB_MONOID_MIN 2

/* unit-side apply and its derivative from the activation */
#define PXB_ACT_IDENTITY 0
#define PXB_ACT_TANH 1
#define PXB_ACT_RELU 2
#define PXB_ACT_SIGMOID 3

/* connection prune predicates recognised by the fused sweep */
#define PXB_PRUNE_NONE 0
#define PXB_PRUNE_ABS_BELOW 1      /* |w| <  threshold                    */
#define PXB_PRUNE_ABS_BELOW_DST 2  /* |w| <  unit_threshold[to_id]        */

/* optimizer bundles: src/plastax/optim/_sgd.py:121-127, _momentum.py:136-139,
 * _adam.py:157-172, _rmsprop.py:135-140 */
#define PXB_OPT_SGD 0
#define PXB_OPT_MOMENTUM 1
#define PXB_OPT_ADAM 2
#define PXB_OPT_RMSPROP 3
/* Utility-based perturbed gradient descent (examples/upgd.py:135-208), per
 * live edge with g = grad[dst] * act[src], U = opt_m (utility), t = opt_t:
 *   t' = t + 1;  U' = b1*U + (1 - b1)*(-g * w)
 *   gate = sigmoid((U' / max(1 - b1^t', eps)) / max(unit_scale[dst], eps))
 *   noise = b2 * sqrt(-2 ln max(h(src, dst, t'), 1e-7)) * cos(2 pi h(dst, src, t'))
 *   w' = w - lr * (g + noise) * (1 - gate)
 * with h the three-word integer hash to [0, 1) of examples/dst_sparse.py:77-85
 * and t' truncated to int32 as its third word (b1 = beta, b2 = sigma). */
#define PXB_OPT_UPGD 4

typedef struct pxb_optimizer {
  int32_t kind;        /* PXB_OPT_* */
  float lr;
  float b1;            /* momentum: mu; adam: beta1; rmsprop: decay; upgd: beta */
  float b2;            /* adam: beta2; upgd: sigma */
  float eps;           /* adam: outside sqrt; rmsprop: inside sqrt; upgd: floors */
  float weight_decay;  /* adamw */
  const float *unit_scale; /* upgd: the utility scale (eta) per destination unit */
} pxb_optimizer;

/* growth score rules for per-unit proposals */
#define PXB_SCORE_UNIFORM 0       /* score = uniform()                         */
#define PXB_SCORE_UNIFORM_Q256 1  /* score = floor(uniform() * 256) / 256      */
#define PXB_SCORE_GRAD_ACT 2      /* score = |grad[dst] * act[src]| (no draw)  */

/* ------------------------------------------------------------------ */
/* library                                                             */
/* ------------------------------------------------------------------ */
PXB_API int pxb_abi_version(void);
PXB_API const char *pxb_last_error(void);
/* Number of SMs of the current device (grid sizing). */
PXB_API int pxb_sm_count(int32_t *out);
/* The library links the CUDA runtime statically: these set / read ITS
 * current device for the calling host thread. A host that switches devices
 * (one process driving several GPUs, or a device other than 0) binds the
 * device it launches on before calling the entry points. */
PXB_API int pxb_set_device(int32_t device);
PXB_API int pxb_get_device(int32_t *device);

/* ------------------------------------------------------------------ */
/* propagation                                                         */
/* ------------------------------------------------------------------ */

/* Forward accumulate of one bucket with the linear map w * act[from]:
 *   acc[to[s]] = acc[to[s]] (+) weight[s] * act[from[s]]   for live s.
 * `acc` is the carried accumulator (combine_pairwise semantics).
 * Replaces src/plastax/sweep.py:113-180 (_accumulate_into, target TO_ID)
 * with the linear_input map of src/plastax/phases.py:535-556. */
PXB_API int pxb_forward_accumulate(int64_t cap, const int32_t *from_id,
                           const int32_t *to_id, const uint8_t *dead,
                           const float *weight, const float *act,
                           int32_t num_units, int32_t monoid, float *acc,
                           void *stream);

/* Forward accumulate fused with a prune predicate and the per-block free
 * counts of the new tombstone mask (one read of every slot).
 *   accumulate as pxb_forward_accumulate over the PRE-prune dead mask;
 *   dead_out[s] = dead[s] | pred(s)   (dead_out may alias dead);
 *   block_free[b] = #dead_out slots in [b*block_len, (b+1)*block_len).
 * block_free may be NULL; block_len must be a power of two >= 128 when
 * given. free_bitmap (may be NULL): each slot pruned here sets its bit in
 * the domain row of pxb_free_bitmap_build (row level[from_id] when
 * bitmap_level is given, the PIPELINE domains; row 0 when it is NULL, the
 * TOPOLOGICAL claim). Replaces src/plastax/phases.py:2240-2319
 * (triton_forward_prune) and :2595 (free_block_counts). */
PXB_API int pxb_forward_prune(int64_t cap, const int32_t *from_id,
                      const int32_t *to_id, const uint8_t *dead,
                      const float *weight, const float *act,
                      int32_t num_units, int32_t monoid, float *acc,
                      int32_t prune_kind, float prune_threshold,
                      const float *unit_threshold, uint8_t *dead_out,
                      int32_t block_len, int32_t *block_free,
                      uint32_t *free_bitmap, const int32_t *bitmap_level,
                      void *stream);

/* Prune sweep on its own: dead_out = dead | pred, plus block counts.
 * Replaces src/plastax/phases.py:1444-1498 (build_prune_conn_phase). */
PXB_API int pxb_prune_conn(int64_t cap, const int32_t *from_id, const int32_t *to_id,
                   const uint8_t *dead, const float *weight, int32_t num_units,
                   int32_t prune_kind, float prune_threshold,
                   const float *unit_threshold, uint8_t *dead_out,
                   int32_t block_len, int32_t *block_free,
                   uint32_t *free_bitmap, const int32_t *bitmap_level,
                   void *stream);

/* The k-lowest-|w| prune (the lowest-magnitude churn of the benchmark
 * configurations, as a prune phase): every bucket writes its candidates at
 * global slots [base, base + cap) of one list -- score -|w| (-inf for a dead
 * slot), id the global slot -- so the first k of the total order
 * (pxb_topk_unique with id_bound = the arena's slots) are the k lowest |w|
 * live edges, ties by ascending slot; pxb_prune_selected then tombstones
 * those of the bucket (skipping the -inf ones, a NaN weight included) and
 * adds them to its claim domain's free bitmap. */
PXB_API int pxb_lowest_keys(int64_t cap, const uint8_t *dead, const float *weight, int64_t base,
                            float *score_out, int32_t *slot_out, void *stream);
PXB_API int pxb_prune_selected(int64_t k, const int32_t *idx, const float *score, int64_t base,
                               int64_t cap, const int32_t *from_id, uint8_t *dead,
                               int32_t num_units, uint32_t *free_bitmap,
                               const int32_t *bitmap_level, void *stream);

/* Backward accumulate of one bucket: acc[from[s]] (+)= w[s] * grad[to[s]].
 * Source-major buckets give long source runs: reduced by warp-segmented
 * shuffles, one atomic per run. Replaces src/plastax/sweep.py:113-180
 * (target FROM_ID). */
PXB_API int pxb_backward_accumulate(int64_t cap, const int32_t *from_id,
                            const int32_t *to_id, const uint8_t *dead,
                            const float *weight, const float *grad,
                            int32_t num_units, int32_t monoid, float *acc,
                            void *stream);

/* Backward accumulate fused with the optimizer's incoming update, one read
 * of every slot. Reads the OLD weight for the accumulate, then writes
 *   g = grad[to] * act[from];  weight, opt columns <- optimizer step(g).
 * Legal only where grad[to] is final when the bucket is swept (the
 * topological reverse walk) and no update_unit phase intervenes.
 * Replaces src/plastax/phases.py:1049-1104 + :1196-1242 for the optimizer
 * bundles (src/plastax/optim). opt_m/opt_v/opt_t may be NULL when the
 * optimizer keeps no such column; acc may be NULL (update only). */
PXB_API int pxb_backward_update(int64_t cap, const int32_t *from_id,
                        const int32_t *to_id, const uint8_t *dead,
                        float *weight, const float *grad, const float *act,
                        int32_t num_units, float *acc,
                        const pxb_optimizer *opt, float *opt_m, float *opt_v,
                        float *opt_t, void *stream);

/* Fractional bits of the exact fixed-point sum accumulators (int64, units
 * of 2^-PXB_FIXED_FRAC_BITS) that pxb_mirror_forward fills and
 * pxb_unit_apply reads. With the mirror's 31-bit sum a product of
 * magnitude >= 2^-7 adds exactly and a smaller one is rounded, an error of
 * at most 2^-32 each (a destination with F in-edges sums within F * 2^-32 of
 * the exact sum of its float32 products before the one final rounding:
 * under 1e-6 for F <= 4294); with its 28-bit sum, >= 2^-4 exact and at most
 * 2^-29 each (under 1e-6 for F <= 536). */
#define PXB_FIXED_FRAC_BITS 31

/* Activation codes of the apply entry points: the low byte is a
 * PXB_ACT_* kind; a non-zero second byte, kind + 1, is the kind of the
 * output units instead (a linear readout under tanh units: PXB_ACT_TANH |
 * ((PXB_ACT_IDENTITY + 1) << 8)). The `is_input` argument of the apply
 * entry points is a unit role column: 0 hidden, 1 input (skipped), 2
 * output. */
#define PXB_ACT_CODE(kind, output_kind) ((kind) | (((output_kind) + 1) << 8))

/* Unit apply with masked merge (src/plastax/sweep.py:183-230):
 * a unit i is finalized iff (level == NULL || level[i] == target_level)
 *   && (is_input == NULL || is_input[i] != 1) && (pruned == NULL || !pruned[i]).
 * The accumulated value x[i] = acc[i], or, when acc_fixed is not NULL,
 * acc_fixed[i] rounded to float and scaled by 2^-PXB_FIXED_FRAC_BITS (one
 * rounding), plus acc[i] as a float (the side accumulator, 0 unless a
 * product was not finite or huge).
 * forward (mode 0):  out[i] = act_fn(x[i])
 * backward (mode 1): out[i] = (x[i] + (seed ? seed[i] : 0)) * act_fn'(act[i])
 * Finalized units have acc[i] reset to the monoid identity (and
 * acc_fixed[i] to 0). */
PXB_API int pxb_unit_apply(int32_t num_units, int32_t mode, int32_t act_kind,
                   int32_t monoid, float *acc, int64_t *acc_fixed, const float *act,
                   const float *seed, const int32_t *level,
                   int32_t target_level, const uint8_t *is_input,
                   const uint8_t *pruned, float *out, void *stream);

/* Fill n floats with a value (accumulator identity reset). */
PXB_API int pxb_fill_f32(int64_t n, float value, float *out, void *stream);
/* A forward's accumulators before a sweep, in one launch: acc[0..n) = value
 * (the monoid's identity) and acc_fixed[0..n) = 0 when acc_fixed is given
 * (the identity_accumulator of src/plastax/sweep.py:334). */
PXB_API int pxb_clear_accumulators(int64_t n, float value, float *acc, int64_t *acc_fixed, void *stream);

/* A step's host traffic without copies (a step graph's first and last
 * kernels): act[ids[i]] = src[i] for i < n, and out[0] = *grown,
 * out[1] = *overflow (0 for a NULL flag). src and out may be pinned host
 * memory, through the device pointer pxb_host_device_pointer returns. */
PXB_API int pxb_scatter_inputs(int32_t n, const int64_t *ids, const float *src, float *act, void *stream);
PXB_API int pxb_flags_out(const int32_t *grown, const uint8_t *overflow, int32_t *out, void *stream);
PXB_API int pxb_host_device_pointer(void *host, void **dev_out);

/* Mean-squared-error loss over the outputs (scripts/parity/reference.py:338):
 * seed[out[k]] = act[out[k]] - target[k]; loss_out[0] = 0.5 * sum diff^2
 * (summed in output order). */
PXB_API int pxb_mse_loss(int32_t num_outputs, const int32_t *output_ids,
                 const float *act, const float *target, float *seed,
                 float *loss_out, void *stream);

/* ------------------------------------------------------------------ */
/* batched (make_step(batch_size=B)), unit columns laid out [N, B]     */
/* ------------------------------------------------------------------ */

/* out[to[s], b] += w[s] * x[from[s], b] for live s, all b < B
 * (B % 4 == 0, B <= 1024, rows 16-byte aligned).
 * Replaces src/plastax/phases.py:643-705 / :812-840 (bucket_product). */
PXB_API int pxb_batched_forward(int64_t cap, const int32_t *from_id,
                        const int32_t *to_id, const uint8_t *dead,
                        const float *weight, const float *x, int32_t batch,
                        int32_t num_units, float *out, void *stream);
/* out[from[s], b] += w[s] * g[to[s], b] (the transpose product). */
PXB_API int pxb_batched_backward(int64_t cap, const int32_t *from_id,
                         const int32_t *to_id, const uint8_t *dead,
                         const float *weight, const float *g, int32_t batch,
                         int32_t num_units, float *out, void *stream);
/* Losses of pxb_batched_loss. */
#define PXB_LOSS_MSE 0        /* scripts/parity/reference.py:338-352 */
#define PXB_LOSS_SOFTMAX_CE 1 /* src/plastax/traits.py:205-250 */

/* pxb_unit_apply (sum monoid) for every (unit, sample) of [N, B] rows:
 * acc, act, seed and out are [N, B]; level / is_input are per unit. */
PXB_API int pxb_batched_unit_apply(int32_t num_units, int32_t batch, int32_t mode,
                                   int32_t act_kind, float *acc, const float *act,
                                   const float *seed, const int32_t *level,
                                   int32_t target_level, const uint8_t *is_input,
                                   float *out, void *stream);
/* Per-sample loss over the outputs (act and seed [N, B], target [B,
 * num_outputs] row-major): seed rows of the outputs, loss_per_sample[b], and
 * loss_out[0] = their sum in sample order / B (StepResult.loss of a batched
 * step, src/plastax/step.py:76-237). MSE: seed = a - t, L = sum 0.5 d^2;
 * softmax cross-entropy: z = a - max(a), s = sum exp(z), seed = exp(z)/s - t,
 * L = sum t * (log s - z); sums in output order. */
PXB_API int pxb_batched_loss(int32_t kind, int32_t num_outputs,
                             const int32_t *output_ids, int32_t batch,
                             const float *act, const float *target, float *seed,
                             float *loss_per_sample, float *loss_out, void *stream);
/* out[u] = (sum_b x[u, b] in sample order) / B: the batch mean of a float
 * unit column (MeanFloatFirstRest, src/plastax/traits.py BatchReduction). */
PXB_API int pxb_batch_mean(int32_t num_units, int32_t batch, const float *x,
                           float *out, void *stream);

/* Exact batch-mean update (src/plastax/phases.py:434-483):
 *   stat[s] = (sum_b g[to,b] * a[from,b]) / B, then one optimizer step. */
PXB_API int pxb_batched_update(int64_t cap, const int32_t *from_id,
                       const int32_t *to_id, const uint8_t *dead,
                       float *weight, const float *g, const float *a,
                       int32_t batch, int32_t num_units,
                       const pxb_optimizer *opt, float *opt_m, float *opt_v,
                       float *opt_t, void *stream);

/* ------------------------------------------------------------------ */
/* growth                                                              */
/* ------------------------------------------------------------------ */

/* Philox-4x32-10 first word for n (seed, counter) pairs (src/plastax/rng.py:109). */
PXB_API int pxb_philox32(int64_t n, const uint64_t *seed, const uint64_t *counter,
                 uint32_t *out, void *stream);

/* The 64-bit seed of one proposal site (src/plastax/rng.py:207-246):
 * (philox32(network_seed, (step << 8) | stream) << 32) | key. Host-side. */
PXB_API uint64_t pxb_site_seed(uint64_t network_seed, uint32_t step, uint32_t stream,
                       uint32_t key);

/* Per-unit proposals (src/plastax/phases.py:3813-3860, rng.py:207-246):
 * candidate c = i * P + j for unit i < num_units, j < P, drawn from the site
 * (network_seed, step, stream 1, key i, j):
 *   src = i; dst = dst_lo + uniform_int(dst_n) [sub 0];
 *   score per score_kind [sub 1 when it draws];
 * then the framework validity (src/plastax/phases.py:4041-4108): ids in
 * range (else clamped to 0 and vetoed), endpoints live (pruned may be NULL),
 * no self loop unless allow_self_loops, |level gap| <= max_level_gap,
 * direction (0 any, 1 deeper, 2 same_or_deeper), and the topological
 * source-level checks: level[src] == bucket_level when bucket_level >= 0,
 * level[src] < src_level_bound (a bucket exists for it) when the bound is
 * > 0. Invalid or non-finite -> -inf. step_dev (may be NULL): when given,
 * the step is read from this device int32 instead of `step`, so the same
 * launch stays valid when replayed from a CUDA graph. */
PXB_API int pxb_propose_per_unit(int32_t num_units, int32_t proposals,
                         uint64_t network_seed, int32_t step, int32_t dst_lo,
                         int32_t dst_n, int32_t score_kind, const float *grad,
                         const float *act, const int32_t *level,
                         const uint8_t *pruned, int32_t max_level_gap,
                         int32_t direction, int32_t allow_self_loops,
                         int32_t bucket_level, int32_t src_level_bound,
                         const int32_t *step_dev, int32_t *src_out,
                         int32_t *dst_out, float *score_out, void *stream);

/* Scratch bytes for pxb_total_order over n candidates with ids < id_bound. */
PXB_API int pxb_total_order_scratch_bytes(int64_t n, int32_t id_bound, size_t *bytes);

/* Permutation of the candidates in the total order (-score, src, dst, index)
 * ascending; NaN sorts as -score = +inf, -0 ties +0. Two stable radix
 * passes: (src, dst) packed into 2*ceil(log2(id_bound)) bits, then the
 * score key (src/plastax/phases.py:4208-4321). */
PXB_API int pxb_total_order(int64_t n, const float *score, const int32_t *src,
                    const int32_t *dst, int32_t id_bound, int32_t *perm_out,
                    void *scratch, size_t scratch_bytes, void *stream);

/* Allocation-free pxb_total_order, for callers that cannot allocate device
 * memory for the scratch (an FFI handler running under CUDA-graph capture,
 * a plugin whose host process owns every device allocation): the scratch
 * is a 16 MiB array inside this library, held on every GPU that loads it
 * until the process exits. At most 262,144 candidates; larger n is
 * rejected with PXB_EINVAL. The first call on a device looks the array up
 * (call it once before any stream capture) and keeps its address for the
 * life of the process, so it is not valid after a reset of that device;
 * all calls share the array, so calls that overlap on the GPU race. No
 * counterpart in the reference. */
PXB_API int pxb_total_order_noalloc(int64_t n, const float *score,
                                    const int32_t *src, const int32_t *dst,
                                    int32_t id_bound, int32_t *perm_out,
                                    void *stream);

/* Step-scoped selection (level_cap_scope = "step",
 * src/plastax/phases.py:4891-4903 and level_major :4469-4487): the first
 * min(k, n) candidates of `perm`, relisted by source level ascending
 * (stable); every level is below num_levels. Writes win_idx[min(k, n)]
 * and win_count[0]. */
PXB_API int pxb_select_step_scratch_bytes(int64_t n, int64_t k, size_t *bytes);
PXB_API int pxb_select_step(int64_t n, const int32_t *perm, const float *score,
                    const int32_t *src, const int32_t *level,
                    int32_t num_levels, int64_t k, int32_t *win_idx,
                    int32_t *win_count, void *scratch, size_t scratch_bytes,
                    void *stream);

/* The first min(k, n) candidates of the total order when (score, src)
 * already orders them, i.e. src is distinct per candidate (per-unit
 * proposals with one proposal per unit): out_idx lists them in the total
 * order. Exact radix select of the k-th unique key (score key, src) in
 * 11-bit digits, one compaction, one sort of the winners. Same output as
 * the first k of pxb_total_order on such candidates. */
PXB_API int pxb_topk_unique_scratch_bytes(int64_t n, int64_t k, int32_t id_bound,
                                  size_t *bytes);
PXB_API int pxb_topk_unique(int64_t n, const float *score, const int32_t *src,
                    int32_t id_bound, int64_t k, int32_t *out_idx,
                    void *scratch, size_t scratch_bytes, void *stream);

/* growth init rules for a committed edge's weight (the rule's `init`) */
#define PXB_INIT_CONST 0         /* w = a                                      */
#define PXB_INIT_DYADIC 1        /* w = (((3*src + 5*dst) mod 16) - 8) / 8     */
#define PXB_INIT_HASH_UNIFORM 2  /* w = a * (2u - 1), u = unit_float(h(src, dst, salt)) */

/* Winners' claim inputs (src/plastax/phases.py:4953-4995): for i < count,
 * src/dst of candidate win_idx[i], its init weight, and growable =
 * isfinite(score); entries count..k-1 are not growable. */
PXB_API int pxb_gather_winners(int64_t k, int64_t count, const int32_t *win_idx,
                       const int32_t *src, const int32_t *dst,
                       const float *score, int32_t init_kind, float init_a,
                       float init_b, uint32_t init_salt, int32_t *src_out,
                       int32_t *dst_out, float *weight_out,
                       uint8_t *growable_out, void *stream);

/* The global proposer (src/plastax/phases.py:3766-3810): proposal j at key
 * 0, src = src_lo + uniform_int(src_n) [sub 0], dst = dst_lo +
 * uniform_int(dst_n) [sub 1], score [sub 2] (kinds as pxb_propose_per_unit),
 * candidate index j; the same validity window. */
PXB_API int pxb_propose_global(int32_t proposals, uint64_t network_seed, int32_t step,
                               int32_t num_units, int32_t src_lo, int32_t src_n,
                               int32_t dst_lo, int32_t dst_n, int32_t score_kind,
                               const float *grad, const float *act,
                               const int32_t *level, const uint8_t *pruned,
                               int32_t max_level_gap, int32_t direction,
                               int32_t allow_self_loops, int32_t bucket_level,
                               int32_t src_level_bound, const int32_t *step_dev,
                               int32_t *src_out, int32_t *dst_out,
                               float *score_out, void *stream);

/* The per-connection proposer (src/plastax/phases.py:3921-4039) over one
 * bucket-major arena of cap slots: the live connections ranked ascending by
 * (src, dst, occurrence in slot order), dead slots after them in slot order;
 * connection rank r proposes candidates r * P + j: src = its source, dst =
 * dst_lo + uniform_int(dst_n) [sub 0], score [sub 1], at the site key
 * philox32((src << 32) | dst, occurrence); a dead proposer's candidates are
 * vetoed. cap * P candidates; scratch of pxb_conn_rank_scratch_bytes. */
PXB_API int pxb_conn_rank_scratch_bytes(int64_t cap, int32_t num_units, size_t *bytes);
PXB_API int pxb_propose_per_conn(int64_t cap, const int32_t *from_id,
                                 const int32_t *to_id, const uint8_t *dead,
                                 int32_t proposals, uint64_t network_seed,
                                 int32_t step, int32_t num_units, int32_t dst_lo,
                                 int32_t dst_n, int32_t score_kind,
                                 const float *grad, const float *act,
                                 const int32_t *level, const uint8_t *pruned,
                                 int32_t max_level_gap, int32_t direction,
                                 int32_t allow_self_loops, int32_t bucket_level,
                                 int32_t src_level_bound, const int32_t *step_dev,
                                 int32_t *src_out, int32_t *dst_out,
                                 float *score_out, void *scratch,
                                 size_t scratch_bytes, void *stream);

/* ScoreAddConn's lowered pair scores and importances
 * (src/plastax/traits.py:467-560; the rule's score(u, src, dst, g) and
 * importance(u, i, g)):
 *   ABS_PRODUCT  |x_src[src] * x_dst[dst]|   (importance: |x_src[i]|)
 *   PRODUCT      x_src[src] * x_dst[dst]     (importance: x_src[i])
 *   MODULAR      (((a*src + b*dst) mod m) - c) * scale, floor mod
 *                (importance: (((a*i) mod m) - c) * scale)
 *   MODULAR_PREDICATE  0 when ((a*src + b*dst) mod m) == c, else -inf
 *                (the should_add predicate adapter)
 * The modular forms are the versioned conformance rules of the reference's
 * goldens (scripts/parity/golden_rules.py:57-77: grid_score_v1 =
 * MODULAR(3, 5, 17, 8, 1/8), importance_v1 = MODULAR(7, -, 13, 0, 1/4),
 * predicate_v1 = MODULAR_PREDICATE(1, 1, 2, 0)). */
#define PXB_PAIR_ABS_PRODUCT 0
#define PXB_PAIR_PRODUCT 1
#define PXB_PAIR_MODULAR 2
#define PXB_PAIR_MODULAR_PREDICATE 3

typedef struct pxb_pair_score {
  int32_t form;
  const float *x_src, *x_dst; /* unit columns of the product forms */
  int32_t a, b, m, c;
  float scale;
} pxb_pair_score;

/* Per-unit importance (src/plastax/phases.py:3640-3665) under `form`, -inf
 * for a pruned unit (the live mask of :4705-4712) and, with mask_kind 1,
 * for a unit whose level is not `bucket` (the per-level shortlist's
 * sources), with mask_kind 2 for one outside the bucket's destination
 * window (level gap <= max_level_gap and the direction 0 any / 1 deeper /
 * 2 same_or_deeper; src/plastax/phases.py:3704-3746). */
PXB_API int pxb_unit_importance(int32_t num_units, const pxb_pair_score *form,
                                const uint8_t *pruned, const int32_t *level,
                                int32_t mask_kind, int32_t bucket,
                                int32_t max_level_gap, int32_t direction,
                                float *out, void *stream);

/* ScoreAddConn candidates (src/plastax/phases.py:3668-3746, :4760-4860):
 * `grids` grids of rows x cols, listed grid after grid, row-major inside;
 * candidate (g, r, q): src = row_ids[g * rows + r] (r when row_ids is NULL:
 * the exhaustive grid, index src * num_units + dst), dst = col_ids[g * cols
 * + q] (q when NULL); its score from `score`, then the validity window of
 * pxb_propose_per_unit (with per_grid_bucket, grid g admits only sources at
 * level g: the per-level shortlist). grids * rows * cols < 2^31. */
PXB_API int pxb_propose_grid(int32_t num_units, int32_t grids, int32_t rows,
                             int32_t cols, const int32_t *row_ids,
                             const int32_t *col_ids, int32_t per_grid_bucket,
                             const pxb_pair_score *score, const int32_t *level,
                             const uint8_t *pruned, int32_t max_level_gap,
                             int32_t direction, int32_t allow_self_loops,
                             int32_t src_level_bound, int32_t *src_out,
                             int32_t *dst_out, float *score_out, void *stream);

/* A chunk of steps as one device-side loop (src/plastax/driver.py:170-317,
 * Driver.scan). `step_graph` is the cudaGraph_t of one captured step; the
 * loop runs it as the body of a conditional WHILE node: before each step
 * row *counter of in_chunk [count, in_cols] (and tgt_chunk) is copied into
 * the step's input buffers; after it the loss goes to loss_rec[row], the
 * activations of out_ids to out_rec[row, :], *counter advances and the
 * loop stops when it reaches `count` or right after a step whose *overflow
 * (or, with resorts, *needs_resort) is set. *status = rows done * 2 +
 * halted. Launch with pxb_loop_launch after setting *counter to the first
 * row; the graph is cloned, so step_graph may be released afterwards. */
typedef struct pxb_loop_desc {
  int32_t *counter;
  int32_t count;
  const float *in_chunk;
  int32_t in_cols;
  float *in_buf;
  const float *tgt_chunk; /* or NULL */
  int32_t tgt_cols;
  float *tgt_buf;
  const float *loss;      /* the step's loss scalar, or NULL */
  float *loss_rec;        /* [count], or NULL */
  const float *act;       /* the activation column, for out_rec */
  const int32_t *out_ids; /* [n_out] */
  int32_t n_out;
  float *out_rec;         /* [count, n_out], or NULL */
  const uint8_t *overflow;
  const uint8_t *needs_resort;
  int32_t resorts;
  int32_t *status;
} pxb_loop_desc;

PXB_API int pxb_loop_build(void *step_graph, const pxb_loop_desc *desc, void **loop_out);
PXB_API int pxb_loop_launch(void *loop, void *stream);
PXB_API int pxb_loop_destroy(void *loop);

/* A captured step graph (a cudaGraph_t) instantiated for replay, with
 * node_priority != 0 honouring each kernel node's priority (the priority of
 * the stream it was captured on), so low-priority side-stream work yields
 * SMs to the step's main stream; launch it on a stream, destroy it once.
 * The reference replays a jitted step (src/plastax/step.py:226-237); these
 * replace its dispatch, not a computation. */
PXB_API int pxb_graph_instantiate(void *graph, int32_t node_priority, void **exec_out);
PXB_API int pxb_graph_launch(void *exec, void *stream);
PXB_API int pxb_graph_exec_destroy(void *exec);

/* ------------------------------------------------------------------ */
/* unit lifecycle (src/plastax/phases.py:1148-1193, :1245-1425)        */
/* ------------------------------------------------------------------ */
/* Unit columns reset to their declared defaults (a pruned unit's, a new
 * child's): up to PXB_MAX_UNIT_COLUMNS columns of 1 or 4 bytes, each with
 * its default's bit pattern. LEVEL and PRUNED are never listed. */
#define PXB_MAX_UNIT_COLUMNS 16
typedef struct pxb_unit_columns {
  int32_t count;
  void *cols[PXB_MAX_UNIT_COLUMNS];
  int32_t bytes[PXB_MAX_UNIT_COLUMNS];
  uint32_t defaults[PXB_MAX_UNIT_COLUMNS];
} pxb_unit_columns;

/* update_unit's lowered forms, on every live unit (inputs and outputs
 * included; pruned slots skipped), each unit reading only its own slot:
 *   AFFINE     field = field * a + b
 *   TRACE_ABS  field = (1 - a) * field + a * |src|
 *   TRACE      field = (1 - a) * field + a * src */
#define PXB_UNIT_UPDATE_AFFINE 0
#define PXB_UNIT_UPDATE_TRACE_ABS 1
#define PXB_UNIT_UPDATE_TRACE 2
PXB_API int pxb_unit_update(int32_t num_units, int32_t kind, float *field, const float *src,
                            float a, float b, const uint8_t *pruned, void *stream);

/* The q-quantile of `field` over the live non-exempt units (NaN values
 * excluded): the value at rank floor(q * m) (0-based, clamped to m - 1) of
 * the m values ascending, into *out (device); -inf when m == 0. */
PXB_API int pxb_unit_quantile_scratch_bytes(int32_t num_units, size_t *bytes);
PXB_API int pxb_unit_quantile(int32_t num_units, const float *field, const uint8_t *pruned,
                              const uint8_t *exempt, float q, float *out, void *scratch,
                              size_t scratch_bytes, void *stream);

/* prune_unit (src/plastax/phases.py:1245-1307) for the predicate
 * field[i] < *threshold (device scalar): a live unit that is not exempt
 * (inputs and outputs) and that the predicate selects is doomed: doomed[i]
 * = 1, pruned[i] = 1, its `reset` columns back to their defaults (LEVEL
 * kept). Then pxb_kill_unit_edges over every bucket. */
PXB_API int pxb_unit_prune(int32_t num_units, const float *field, const float *threshold,
                           const uint8_t *exempt, uint8_t *pruned, uint8_t *doomed,
                           const pxb_unit_columns *reset, void *stream);

/* Tombstone every live connection with a doomed endpoint; each joins its
 * claim domain's free bitmap (row bitmap_level[from_id], or 0 when
 * bitmap_level is NULL; no bitmap when free_bitmap is NULL). */
PXB_API int pxb_kill_unit_edges(int64_t cap, const int32_t *from_id, const int32_t *to_id,
                                uint8_t *dead, int32_t num_units, const uint8_t *doomed,
                                uint32_t *free_bitmap, const int32_t *bitmap_level,
                                void *stream);

/* add_unit (src/plastax/phases.py:1310-1425). Spawners, from the pre-phase
 * state: FIELD_AT_LEAST every live unit with field >= threshold; ARGMAX the
 * live unit with the largest non-NaN field (lowest id on ties). Parents in
 * ascending id take the free slots (PRUNED at the start of the phase) in
 * ascending id; a parent past the last free slot is dropped
 * (*unit_overflow = 1). A child's slot takes its `reset` defaults, becomes
 * live, gets level clamp(level[parent] + offset, 1, max_level), and, with
 * init_dst, init_dst[child] = init_src[parent] * init_scale.
 * *units_added = children placed. scratch: 2 * num_units int32. One CTA. */
#define PXB_SPAWN_FIELD_AT_LEAST 0
#define PXB_SPAWN_ARGMAX 1
typedef struct pxb_unit_spawn {
  int32_t kind;
  const float *field;
  float threshold;
  int32_t offset;
  int32_t max_level;
  float *init_dst;
  const float *init_src;
  float init_scale;
} pxb_unit_spawn;
PXB_API int pxb_unit_add(int32_t num_units, const pxb_unit_spawn *spawn, uint8_t *pruned,
                         int32_t *level, const pxb_unit_columns *reset, int32_t *scratch,
                         int32_t *units_added, uint8_t *unit_overflow, void *stream);

/* The per-source-level cap (level_cap_scope "source_level",
 * src/plastax/phases.py:4324-4487): over a level-major list idx of n
 * candidates (pxb_select_step with k = n), the first k of every level's
 * run, listed levels ascending into out_idx (capacity num_levels * k; fill
 * it with -1 first, pxb_gather_winners treats -1 as no candidate);
 * out_count (device) = their number. scratch: 3 * num_levels + 1 int32. */
PXB_API int pxb_cap_per_level(int64_t n, const int32_t *idx, const int32_t *src,
                              const int32_t *level, int32_t num_levels, int64_t k,
                              int32_t *out_idx, int32_t *out_count, int32_t *scratch,
                              void *stream);

/* Fused growth selection for one proposal per unit scored by the site RNG
 * (score_kind PXB_SCORE_UNIFORM or PXB_SCORE_UNIFORM_Q256): the proposals
 * of every unit (as pxb_propose_per_unit with proposals = 1, bucket_level
 * -1), the first k of the total order, listed levels ascending with the
 * total order inside a level, gathered into the claim's input columns (as
 * pxb_gather_winners) -- the same k rows as pxb_propose_per_unit +
 * pxb_topk_unique + pxb_select_step + pxb_gather_winners. The keys' bins are
 * ranked in shared memory, with no sort pass (the score integers are Philox
 * draws). Requires dst_lo + dst_n <= num_units and num_levels <= 8.
 * status (device, may be NULL) gets bit 0 when a bin held more than 65,536
 * keys and the list is incomplete (not reached by RNG scores). Replaces
 * src/plastax/phases.py:3813-3860 + :4208-4487 + :5043-5058 for this form. */
PXB_API int pxb_select_unique_scratch_bytes(int32_t num_units, int64_t k,
                                            int32_t num_levels, int32_t score_kind,
                                            size_t *bytes);
PXB_API int pxb_propose_select_unique(
    int32_t num_units, uint64_t network_seed, int32_t step, int32_t dst_lo,
    int32_t dst_n, int32_t score_kind, const int32_t *level,
    const uint8_t *pruned, int32_t max_level_gap, int32_t direction,
    int32_t allow_self_loops, int32_t src_level_bound,
    const int32_t *step_dev, int64_t k, int32_t num_levels, int32_t init_kind,
    float init_a, float init_b, uint32_t init_salt, int32_t *src_out,
    int32_t *dst_out, float *weight_out, uint8_t *growable_out,
    int32_t *status, void *scratch, size_t scratch_bytes, void *stream);

/* The same selection with the ranking of the full bins shared out over the
 * ranks of a Scheme-A group (replaces the claim all-gather's replicated
 * selection, src/plastax/phases.py:3046-3053, for this form). Every rank
 * draws every proposal and finds the same threshold bin; rank r ranks the
 * full (level, bin) pairs q = level * threshold_bin + bin with
 * q % world == r and stores each of their winners into every rank's columns
 * (peer memory, e.g. pxb_peer_open mappings), and each rank stores the
 * threshold bin's winners and the zero fill past min(k, n) into its own.
 * After every rank's call has completed and a barrier has ordered it before
 * the reads (the combine's flags of pxb_scheme_a_apply, for a selection a
 * step ahead), every rank's columns hold the list pxb_propose_select_unique
 * returns. Each column holds `blocks` lists of k entries; a call fills list
 * (step mod blocks), the step read from step_dev when it is set, so a
 * captured graph rotates through them (three lists let a rank select step
 * t + 1's while a slower peer still claims step t - 1's).
 * pxb_select_take copies one list out. */
#define PXB_SELECT_MAX_WORLD 8
typedef struct pxb_select_shard {
  int32_t rank, world; /* 1 <= world <= PXB_SELECT_MAX_WORLD */
  int32_t blocks;      /* lists per column, >= 1 */
  int32_t pad;
  int32_t *src_out[PXB_SELECT_MAX_WORLD]; /* rank q's columns, blocks * k entries */
  int32_t *dst_out[PXB_SELECT_MAX_WORLD];
  float *weight_out[PXB_SELECT_MAX_WORLD];
  uint8_t *growable_out[PXB_SELECT_MAX_WORLD];
} pxb_select_shard;
PXB_API int pxb_propose_select_unique_sharded(
    int32_t num_units, uint64_t network_seed, int32_t step, int32_t dst_lo,
    int32_t dst_n, int32_t score_kind, const int32_t *level,
    const uint8_t *pruned, int32_t max_level_gap, int32_t direction,
    int32_t allow_self_loops, int32_t src_level_bound,
    const int32_t *step_dev, int64_t k, int32_t num_levels, int32_t init_kind,
    float init_a, float init_b, uint32_t init_salt, const pxb_select_shard *shard,
    int32_t *status, void *scratch, size_t scratch_bytes, void *stream);

/* List (step mod blocks) of four columns of `blocks` lists of k entries
 * (the step read from step_dev) copied into the claim's input columns, in
 * one launch. */
PXB_API int pxb_select_take(int64_t k, int32_t blocks, const int32_t *step_dev,
                            const int32_t *src_col, const int32_t *dst_col,
                            const float *weight_col, const uint8_t *growable_col,
                            int32_t *src_out, int32_t *dst_out, float *weight_out,
                            uint8_t *growable_out, void *stream);

/* Growth dedupe (src/plastax/phases.py:4111-4205): the step's candidate
 * pairs in a hash table (scratch of pxb_dedupe_scratch_bytes(n), reset by
 * every pxb_pair_table_build). pxb_pair_table_mark passes over a bucket,
 * marks the table pairs that are live edges there and writes live_hit[i]
 * for every candidate (marks accumulate over calls, one per bucket;
 * live_pair_member, :2481-2537; under Scheme-A OR the marks across ranks
 * before applying). pxb_dedupe_apply then sets score = -inf where live_hit
 * (may be NULL) is set and, with step_repeats, for every copy of a pair but
 * the first in the stable order of -score (dedupe_step / repeats_earlier,
 * :4156, :2540-2575; NaN scores order last). One table: build, mark, apply. */
PXB_API int pxb_dedupe_scratch_bytes(int64_t n, size_t *bytes);
PXB_API int pxb_pair_table_build(int64_t n, const int32_t *src, const int32_t *dst,
                                 void *scratch, size_t scratch_bytes, void *stream);
PXB_API int pxb_pair_table_mark(int64_t n, int64_t cap, const int32_t *from_id,
                                const int32_t *to_id, const uint8_t *dead,
                                uint8_t *live_hit, void *scratch,
                                size_t scratch_bytes, void *stream);
PXB_API int pxb_dedupe_apply(int64_t n, float *score, const uint8_t *live_hit,
                             int32_t step_repeats, void *scratch,
                             size_t scratch_bytes, void *stream);

/* The resort's compaction order (src/plastax/topo.py:303-452): perm_out =
 * the bucket's slots stably ordered by dead * num_units + from_id (live
 * edges grouped by source, old relative order kept within a source, dead
 * slots last); the caller gathers every column through it. */
PXB_API int pxb_resort_order_scratch_bytes(int64_t cap, size_t *bytes);
PXB_API int pxb_resort_order(int64_t cap, const uint8_t *dead, const int32_t *from_id,
                             int32_t num_units, int32_t *perm_out, void *scratch,
                             size_t scratch_bytes, void *stream);

/* ------------------------------------------------------------------ */
/* slot claim                                                          */
/* ------------------------------------------------------------------ */
#define PXB_CLAIM_PIPELINE 0     /* src/plastax/phases.py:2985-3106 */
#define PXB_CLAIM_TOPOLOGICAL 1  /* src/plastax/phases.py:2853-2982 */
/* pxb_claim_commit mode flag: the candidate list is level-major (the level
 * of every claiming candidate's source ascends along the list, as the
 * growth listing makes it), so the claim partitions instead of sorting. */
#define PXB_CLAIM_LEVEL_MAJOR 0x100

/* Scratch bytes for one claim over `cap` local slots, k candidates and
 * num_levels (<= 1024) claim domains (1 for the topological claim). */
PXB_API int pxb_claim_scratch_bytes(int64_t cap, int64_t k, int32_t num_levels,
                            size_t *bytes);

/* Claim, step 1: count this rank's free slots per domain. PIPELINE: a dead
 * slot at global position shard_base + s < *tail_start belongs to domain
 * unit_level[from_id[s]]; TOPOLOGICAL: every dead slot, one domain.
 * Writes level_counts[num_levels] (device) for the Scheme-A all-gather and
 * keeps the per-tile counts in `scratch` for step 2. With `free_bitmap`
 * (the per-domain bitmaps of pxb_free_bitmap_build, kept current by the
 * prune sweeps and the claim) the counts come from the bitmaps and neither
 * from_id nor dead is read. */
PXB_API int pxb_claim_prepare(int32_t mode, int64_t cap, const int32_t *from_id,
                      const uint8_t *dead, const int32_t *unit_level,
                      int32_t num_units, int32_t num_levels,
                      int64_t shard_base, const int64_t *tail_start,
                      const uint32_t *free_bitmap, int64_t k,
                      int32_t *level_counts, void *scratch,
                      size_t scratch_bytes, void *stream);

/* Claim, step 2: the k candidates in claim order (levels ascending, total
 * order within a level) with growable[i]; max_new >= 0 caps the growable
 * ones in claim order (max_new_per_step). Each candidate level's growable
 * candidates take that domain's free slots in slot order, global rank by
 * global rank; PIPELINE spills the rest to the tail (global positions
 * *tail_start + spill rank, levels ascending); past the global capacity a
 * candidate overflows. Writes from_id/to_id/weight and each extra column
 * (1- or 4-byte elements, k values each) at the placed slots this rank
 * owns, clears dead there, advances *tail_start (PIPELINE), and writes
 * counts_out[4] = {committed, overflowed, tail slots used, committed with
 * level[dst] <= level[src]} and overflowed_out[k] (either may be NULL).
 * level_before / level_totals: Scheme-A per-domain counts of the ranks
 * before this one and of all ranks (device; NULL on one GPU). `scratch`
 * must hold step 1's results. With `free_bitmap` (as in step 1) the claimed
 * own-domain slots are found in and cleared from the bitmaps.
 * placed_out[k] (may be NULL): the local slot each candidate was written
 * to on this rank, -1 when none. committed_out[k] (may be NULL): 1 for a
 * candidate committed on any rank (the same on every rank), else 0. */
PXB_API int pxb_claim_commit(int32_t mode, int64_t cap, int32_t *from_id,
                     int32_t *to_id, uint8_t *dead, float *weight,
                     const int32_t *unit_level, int32_t num_units,
                     int32_t num_levels, int64_t shard_base,
                     int64_t global_cap, int64_t *tail_start, int64_t k,
                     const int32_t *cand_src, const int32_t *cand_dst,
                     const float *cand_weight, const uint8_t *growable,
                     int64_t max_new, const int32_t *level_before,
                     const int32_t *level_totals, uint32_t *free_bitmap,
                     int32_t n_extra, void *const *extra_cols,
                     const int32_t *extra_bytes, const void *const *extra_vals,
                     int32_t *counts_out, uint8_t *overflowed_out,
                     int32_t *placed_out, uint8_t *committed_out,
                     void *scratch, size_t scratch_bytes, void *stream);

/* Per-domain free-slot bitmaps of a bucket: num_levels rows of
 * ceil(cap / 32) words; bit s of row d is set iff slot s is a claimable free
 * slot of domain d (PIPELINE: dead, below *tail_start, d = level[from_id];
 * TOPOLOGICAL: dead, d = 0). */
PXB_API int pxb_free_bitmap_build(int32_t mode, int64_t cap, const int32_t *from_id,
                          const uint8_t *dead, const int32_t *unit_level,
                          int32_t num_units, int32_t num_levels,
                          int64_t shard_base, const int64_t *tail_start,
                          uint32_t *bitmap, void *stream);

/* The end of a step (device values, each may be NULL): *grown = 0 and
 * *overflow = 0 for a step that claimed nothing (src/plastax/phases.py:
 * 4953-5132 report zero then), and the device step counter the proposals
 * read under graph replay advanced by one (src/plastax/step.py:226-229). */
PXB_API int pxb_step_end(int32_t *step, int32_t *grown, uint8_t *overflow, void *stream);

/* The step's growth flags from a claim's counts_out (device): grown (+)=
 * counts[0], overflow |= counts[1] > 0, needs_resort |= counts[3] > 0; with
 * reset != 0 grown and overflow start from 0 (the step's first bucket).
 * grown, overflow and needs_resort may each be NULL. The flags of
 * src/plastax/phases.py:4953-5132 (StepResult.overflow, grown,
 * needs_resort). */
PXB_API int pxb_growth_flags(const int32_t *counts, int32_t reset, int32_t *grown,
                             uint8_t *overflow, uint8_t *needs_resort, void *stream);

/* Count the dead slots of a bucket into out[0] (device). */
PXB_API int pxb_count_dead(int64_t cap, const uint8_t *dead, int32_t *out,
                   void *stream);

/* ------------------------------------------------------------------ */
/* destination-grouped mirror (the forward sweep's index)              */
/* ------------------------------------------------------------------ */
/* Entries per tile of the mirror sweep: group bases and the entry count
 * are multiples of it. */
#define PXB_MIRROR_TILE 2048

/* A bucket's live edges grouped by destination chunk (2^chunk_bits
 * consecutive units, chunk_bits <= 13, ceil(log2 num_units) + chunk_bits
 * <= 32). Group g owns entries [gbase[g], gbase[g+1]) (multiples of
 * PXB_MIRROR_TILE), of which the first gfill[g] have ever been used. Entry e: word[e] = src <<
 * chunk_bits | (dst - g * 2^chunk_bits), or 0xffffffff when empty;
 * weight[e]; slot[e] = the canonical (local) slot it mirrors. hstack at
 * gbase[g] holds hcount[g] free entry offsets of group g. items /
 * item_begin / item_end / item_group describe runs of entries for callers
 * that split the sweep themselves (the sweep here does not read them).
 * Edges a full group cannot take go to the overflow list (ovf_*); status[0]
 * bit 0 is set when that list is full too (the mirror must be rebuilt), bit
 * 1 when a sweep's pipeline wait timed out (its result is incomplete). All
 * arrays are device memory owned by the caller; word and weight 16-byte
 * aligned. defer_pos / defer_count (may be NULL): the sweep's deferred
 * prunes -- sweep CTA c lists up to defer_seg entry positions it pruned at
 * defer_pos[c * defer_seg ...] and their count at defer_count[c] (for c <
 * defer_ctas), and a second pass writes their tombstones, so the sweep's
 * pipeline never waits on the scattered writes of a tombstone; a CTA past
 * defer_ctas, or past its segment, writes them in place. */
typedef struct pxb_mirror {
  int32_t num_units;
  int32_t chunk_bits;
  int64_t groups;
  int64_t entries;
  const int64_t *gbase;
  int32_t *gfill;
  uint32_t *word;
  float *weight;
  int32_t *slot;
  int32_t *hstack;
  int32_t *hcount;
  int64_t items;
  const int64_t *item_begin;
  const int64_t *item_end;
  const int32_t *item_group;
  int64_t ovf_cap;
  int32_t *ovf_count;
  int32_t *ovf_src;
  int32_t *ovf_dst;
  int32_t *ovf_slot;
  float *ovf_weight;
  int32_t *status;
  int32_t *ins_count; /* [groups] zeroed scratch of pxb_mirror_insert */
  int64_t *defer_pos;
  int32_t *defer_count;
  int64_t defer_seg;
  int32_t defer_ctas;
  int32_t sum_frac_bits; /* the sweep's shared-memory sum: 28 fractional bits
                            (each product below 2^-4 rounded to 2^-28, an error
                            of at most 2^-29; the words rarely wrap) or any
                            other value for 31 (below 2^-7 to 2^-31, at most
                            2^-32); acc_fixed is in 2^-31 units either way */
} pxb_mirror;

/* Forward accumulate of the mirrored bucket (w * act[src] combined per
 * destination) fused with the prune predicate. For sum the products are
 * accumulated exactly, independent of order: acc_fixed (int64, units of
 * 2^-PXB_FIXED_FRAC_BITS, non-NULL) += each float32 product rounded to that
 * unit (exact for |w * act| >= 2^-4), and a product that is not finite or
 * of magnitude >= 2^20 is added to acc as a float instead; the sum is then
 * acc_fixed * 2^-PXB_FIXED_FRAC_BITS + acc (pxb_unit_apply reads both).
 * For max / min, acc (+)= as pxb_forward_accumulate does and acc_fixed is
 * unused. The prune: a pruned edge still
 * contributes (the forward reads the pre-prune state), then its mirror entry
 * is emptied and pushed on its group's hole stack, and the canonical record
 * is written: dead[slot] = 1, its free-bitmap bit (row bitmap_level[src],
 * or row 0 when bitmap_level is NULL), pruned_count += 1 (may be NULL).
 * Replaces src/plastax/phases.py:2240-2319 and sweep.py:113-180 for a
 * bucket that has a mirror. */
PXB_API int pxb_mirror_forward(const pxb_mirror *mirror, const float *act,
                               int32_t monoid, float *acc, int64_t *acc_fixed,
                               int32_t prune_kind,
                               float prune_threshold,
                               const float *unit_threshold, uint8_t *dead,
                               uint32_t *free_bitmap, int64_t bitmap_words,
                               const int32_t *bitmap_level,
                               int32_t *pruned_count, void *stream);

/* Insert the claim's placed edges into the mirror: candidate i with
 * placed[i] >= 0 (pxb_claim_commit's placed_out) goes to a hole of its
 * destination's group, else the group's unused slack, else the overflow
 * list. */
PXB_API int pxb_mirror_insert(const pxb_mirror *mirror, int64_t k,
                              const int32_t *src, const int32_t *dst,
                              const float *weight, const int32_t *placed,
                              void *stream);

/* ------------------------------------------------------------------ */
/* exact lowest-|w| prune fused into the mirror sweep                  */
/* ------------------------------------------------------------------ */
/* The k live edges of lowest |w| (ties by ascending global slot, a NaN
 * weight never) are pruned every firing, as pxb_lowest_keys +
 * pxb_topk_unique + pxb_prune_selected do, but without a selection over
 * every slot: the order key of an edge is (bits(|w|), global slot), and two
 * histograms of bits(|w|) over the live non-NaN edges are kept current on
 * the device -- coarse bins (bits >> PXB_LOWK_SHIFT, 2^16) and fine bins
 * (bits >> PXB_LOWK_FINE_SHIFT, 2^24; a fine bin spans 2^-16 of its
 * value) -- built once (pxb_lowk_hist_build), cut by every plan (the bins a
 * plan prunes are emptied) and raised by every committed growth edge
 * (pxb_lowk_hist_add). Under Scheme-A every rank holds the same whole-arena
 * histograms: each plan and each committed edge is the same on every rank.
 *
 * One firing:
 *   1. pxb_lowk_make_plan: from the histograms, the fine threshold bin b* of
 *      the k-th smallest key -- every edge in a bin below b* is pruned; of
 *      the bin itself the `take` smallest keys, unless the whole bin is
 *      needed (two launches: 64 CTAs sum the coarse bins and the last to
 *      finish plans, a grid empties the fine bins the plan prunes);
 *   2. pxb_mirror_forward_lowk: the forward sweep; an edge below the bin is
 *      tombstoned there (as the fused threshold prune does), an edge in the
 *      bin is listed (key, source level, mirror position);
 *   3. pxb_lowk_select (after every rank's sweep has finished: after
 *      pxb_scheme_a_apply's barrier under Scheme-A): one CTA radix-selects
 *      the take-th smallest key over every rank's list and tombstones this
 *      rank's listed edges up to it; under Scheme-A it also adds every
 *      rank's selected edges to level_before / level_totals (their claim
 *      domains), so the per-domain counts that rode on the barrier stay
 *      exact.
 * The lists are double-buffered by the plan's parity, so a rank one step
 * ahead never overwrites a list a peer still reads. plan->status: bit 0 a
 * list overflowed list_cap (the threshold bin held more edges than the
 * list -- only when that many live edges share a |w| to 2^-16; the step's
 * prune is incomplete), bit 1 the swept counts disagree with the histogram
 * (the histogram is stale: rebuild it). Replaces the lowest-magnitude prune
 * phase (src/plastax/phases.py:1444-1498, with the k-th smallest |w| as the
 * predicate's threshold, examples/dst_sparse.py:88-140) for a single-bucket
 * arena with a mirror. */
#define PXB_PRUNE_LOWEST_K 3
#define PXB_LOWK_SHIFT 15
#define PXB_LOWK_BINS 65536
#define PXB_LOWK_FINE_SHIFT 7
#define PXB_LOWK_FINE_BINS 16777216
#define PXB_LOWK_PLAN_SCRATCH 256

typedef struct pxb_lowk_plan { /* device memory, written by pxb_lowk_make_plan */
  uint32_t lo_bits;     /* every live edge with bits(|w|) < lo_bits is pruned  */
  uint32_t hi_bits;     /* lo_bits <= bits(|w|) < hi_bits: listed              */
  int64_t take;         /* the listed edges pruned (smallest keys, all ranks)  */
  int64_t below_expect; /* edges below lo_bits, all ranks (from the histogram) */
  int64_t listed_expect;/* edges in [lo_bits, hi_bits), all ranks             */
  int32_t parity;       /* the list buffer this firing writes                   */
  int32_t status;       /* bit 0 list overflow, bit 1 counts disagree          */
  int64_t pruned;       /* edges this rank pruned in the last firing           */
  uint32_t floor;       /* no fine bin below this one holds an edge            */
  uint32_t zero_lo;     /* fine bins [zero_lo, zero_hi) the last plan emptied  */
  uint32_t zero_hi;
  uint32_t pad;
} pxb_lowk_plan;

typedef struct pxb_lowk {
  int32_t rank, world;
  int64_t k;            /* edges pruned per firing (whole arena)               */
  int64_t list_cap;     /* entries per list buffer                             */
  int64_t slot_base;    /* this rank's first global slot                       */
  uint32_t *hist;       /* [PXB_LOWK_BINS] coarse bins                         */
  uint32_t *fine;       /* [PXB_LOWK_FINE_BINS] fine bins                      */
  pxb_lowk_plan *plan;  /* device; zero it, then set floor = 0xFFFFFFFF, before
                           the first pxb_lowk_hist_build                      */
  /* this rank's lists (device; under Scheme-A inside its peer region) */
  uint64_t *key;        /* [2 * list_cap] (bits(|w|) << 32) | global slot      */
  int32_t *level;       /* [2 * list_cap] the listed slot's claim domain       */
  unsigned long long *count; /* [4]: per parity {listed, pruned below lo_bits} */
  int64_t *pos;         /* [2 * list_cap] mirror positions (-1 - i for the
                           mirror's overflow entry i); never read by a peer    */
  /* every rank's key / level / count (device arrays of `world` pointers,
   * peers mapped into this rank's address space); NULL when world == 1 */
  uint64_t *const *peer_key;
  int32_t *const *peer_level;
  unsigned long long *const *peer_count;
  uint32_t *plan_scratch; /* [PXB_LOWK_PLAN_SCRATCH] device words for the plan's
                             partial sums; zero them once before the first plan */
} pxb_lowk;

/* Both histograms += every live slot of a bucket whose weight is not NaN,
 * and plan->floor lowered to the lowest fine bin seen (the caller zeroes the
 * histograms and sets the plan first). */
PXB_API int pxb_lowk_hist_build(const pxb_lowk *lowk, int64_t cap,
                                const uint8_t *dead, const float *weight,
                                void *stream);
/* Step 1 above (64 CTAs; the last one to finish plans). */
PXB_API int pxb_lowk_make_plan(const pxb_lowk *lowk, void *stream);
/* Step 2 above: pxb_mirror_forward with the plan's prune; bitmap_level
 * (PIPELINE, else NULL) names the claim domain of a pruned or listed slot. */
PXB_API int pxb_mirror_forward_lowk(const pxb_mirror *mirror, const float *act,
                                    int32_t monoid, float *acc,
                                    int64_t *acc_fixed, const pxb_lowk *lowk,
                                    uint8_t *dead, uint32_t *free_bitmap,
                                    int64_t bitmap_words,
                                    const int32_t *bitmap_level, void *stream);
/* Step 2 in two parts, so the tombstones of the edges below the bin can be
 * written beside step 3 on one GPU: pxb_mirror_forward_lowk_deferred runs the
 * sweep and the mirror's overflow pass and leaves the sweep's deferred
 * tombstones, which pxb_mirror_defer_flush (same mirror, monoid and lowk;
 * any stream ordered after the sweep) writes. Together they do what
 * pxb_mirror_forward_lowk does. */
PXB_API int pxb_mirror_forward_lowk_deferred(const pxb_mirror *mirror,
                                             const float *act, int32_t monoid,
                                             float *acc, int64_t *acc_fixed,
                                             const pxb_lowk *lowk, uint8_t *dead,
                                             uint32_t *free_bitmap,
                                             int64_t bitmap_words,
                                             const int32_t *bitmap_level,
                                             void *stream);
PXB_API int pxb_mirror_defer_flush(const pxb_mirror *mirror, int32_t monoid,
                                   const pxb_lowk *lowk, uint8_t *dead,
                                   uint32_t *free_bitmap, int64_t bitmap_words,
                                   const int32_t *bitmap_level, void *stream);
/* Step 3 above; one CTA. level_before / level_totals ([num_levels], may be
 * NULL) receive every rank's selected edges per claim domain. */
PXB_API int pxb_lowk_select(const pxb_lowk *lowk, const pxb_mirror *mirror,
                            uint8_t *dead, uint32_t *free_bitmap,
                            int64_t bitmap_words, const int32_t *bitmap_level,
                            int32_t num_levels, int32_t *level_before,
                            int32_t *level_totals, void *stream);
/* hist[bin(weight[i])] += 1 for every committed[i] (pxb_claim_commit's
 * committed_out) whose weight is not NaN: the growth edges of a firing.
 * totals ([4] int64, may be NULL) accumulate {edges this rank pruned in
 * the firing, claim_counts[0] committed, claim_counts[1] overflowed,
 * firings} (claim_counts: pxb_claim_commit's counts_out, may be NULL). */
PXB_API int pxb_lowk_hist_add(const pxb_lowk *lowk, int64_t k,
                              const float *weight, const uint8_t *committed,
                              const int32_t *claim_counts, int64_t *totals,
                              void *stream);

/* ------------------------------------------------------------------ */
/* Scheme-A reduction over NVLink peer memory                          */
/* ------------------------------------------------------------------ */
/* Device memory shared with peer processes through CUDA IPC: alloc returns
 * a zeroed region and its 64-byte IPC handle; a peer opens the handle to map
 * the region (close before the owner frees it). */
PXB_API int pxb_peer_alloc(size_t bytes, void **ptr_out, uint8_t *ipc_handle_out);
PXB_API int pxb_peer_open(const uint8_t *ipc_handle, void **ptr_out);
PXB_API int pxb_peer_close(void *ptr);
PXB_API int pxb_peer_free(void *ptr);

/* Levels a Scheme-A group's counts area holds per rank. */
#define PXB_PEER_MAX_LEVELS 8

/* One rank's view of a Scheme-A group: device arrays of `world` pointers
 * (entry q = rank q's buffer, mapped here; entry rank = this rank's own):
 * the int64 fixed-point partials (units of 2^-PXB_FIXED_FRAC_BITS, as
 * pxb_mirror_forward fills them), the float side partials, the activation
 * column, each rank's flag rows ([2][world] uint32, zero at creation) and
 * each rank's counts area ([world][PXB_PEER_MAX_LEVELS] int32; may be NULL
 * when no counts ride on the barrier). epoch, done and status are this
 * rank's device words (zero at creation). */
typedef struct pxb_peer_group {
  int32_t rank;
  int32_t world;
  int64_t *const *acc_fixed;
  float *const *acc_side;
  float *const *act;
  uint32_t *const *flags;
  int32_t *const *counts;
  uint32_t *epoch;
  uint32_t *done;
  int32_t *status;
} pxb_peer_group;

/* The forward's Scheme-A combine and apply in one kernel: waits until every
 * rank's partials are complete, reduces this rank's slice of the units from
 * every rank (exact int64 sum rounded once, plus the float side in rank
 * order), applies act_kind (units not input and not pruned, as
 * pxb_unit_apply) and stores the activation into every rank's activation
 * column, then waits until every rank is done. Every rank calls it once per
 * step. A wait gives up after wait_polls polls and sets status bit 0.
 * With level_counts (this rank's per-domain free counts from
 * pxb_claim_prepare, device, [num_levels]) the counts of every rank ride on
 * the first barrier, and level_before / level_totals receive the sums over
 * the ranks before this one and over all ranks (pxb_claim_commit's
 * Scheme-A inputs; the all-gather of src/plastax/phases.py:3046-3053).
 * Replaces the all-reduce of src/plastax/monoid.py:175-204 plus
 * src/plastax/sweep.py:183-230 for the pipeline sweep's sum. */
PXB_API int pxb_scheme_a_apply(const pxb_peer_group *group, int32_t num_units,
                               int32_t act_kind, const uint8_t *is_input,
                               const uint8_t *pruned,
                               const int32_t *level_counts, int32_t num_levels,
                               int32_t *level_before, int32_t *level_totals,
                               uint32_t wait_polls, void *stream);

/* ------------------------------------------------------------------ */
/* The fused pipeline training step                                     */
/* ------------------------------------------------------------------ */
/* One PIPELINE step of a single-device net whose forward and backward sum
 * over one bucket, as three kernels: (1) one pass over the arena
 * accumulating both the forward (into destinations, from the previous
 * activations) and the backward (into sources, from the previous
 * gradients) in exact fixed point in shared memory, each CTA holding
 * every unit's two accumulators; a thread-block cluster reduces its CTAs'
 * accumulators through distributed shared memory into one int64 row per
 * cluster; (2) per unit: the rows summed (exact) and rounded once, the
 * forward apply (inputs and pruned units kept), the MSE seed of the outputs
 * (act - target), the backward apply (every unit but the pruned, inputs
 * included); (3) one pass over the arena applying the optimizer to every
 * live edge with the edge gradient update_grad[dst] * act[src] (the new
 * columns), one warp of it summing the loss in output order.
 * Replaces, for such nets, src/plastax/sweep.py:300-340 (forward sweep),
 * :402-450 (backward sweep), src/plastax/phases.py:488-532 (update_conn) and
 * the MSE seed of scripts/parity/reference.py:338-352, in the order of
 * src/plastax/step.py:45-237. Every value equals the unfused passes' within
 * the fixed-point sum's bound (each product rounded to 2^-32 at most). An
 * arena of at most 65,536 slots takes all three phases in one launch of one
 * thread-block cluster (its hardware barrier between them). */
typedef struct pxb_pipeline_train {
  int64_t cap;                 /* the bucket */
  const int32_t *from_id, *to_id;
  const uint8_t *dead;
  float *weight;
  float *opt_m, *opt_v, *opt_t; /* optimizer columns (NULL where unused) */
  int32_t num_units;
  float *act;          /* in: previous activations, inputs scattered; out: new */
  float *grad;         /* in: previous gradients; out: new (NULL: no backward) */
  float *seed;         /* the loss seed column (NULL: no loss) */
  const uint8_t *roles;    /* 1 input, 2 output (own activation), 0 hidden */
  const uint8_t *pruned;   /* or NULL */
  int32_t fwd_act, bwd_act; /* PXB_ACT_CODE codes; bwd_act ignored without grad */
  int32_t num_outputs;
  const int32_t *target_of; /* [num_units]: output index of a unit, -1 if none */
  const int32_t *output_ids; /* [num_outputs], the loss's summation order */
  const float *target;       /* [num_outputs], device (NULL: no loss) */
  float *loss;               /* device scalar, or NULL */
  float *update_grad;        /* the column the edge gradient reads at dst */
  pxb_optimizer opt;         /* any kind but PXB_OPT_UPGD */
  void *scratch;             /* pxb_pipeline_train_scratch_bytes(num_units) */
  const int64_t *tail_start; /* device: slots at or past it are never live (a
                                PIPELINE arena's tail), so neither pass reads
                                them; NULL: the whole capacity */
} pxb_pipeline_train;

/* The largest num_units the step takes (every CTA holds every unit's
 * accumulators in shared memory), with or without a backward. */
PXB_API int32_t pxb_pipeline_train_max_units(int32_t with_backward);
/* Device scratch the step needs (*bytes); zero it once before the first
 * call (the step leaves it zeroed where it must be). */
PXB_API int pxb_pipeline_train_scratch_bytes(int32_t num_units, size_t *bytes);
PXB_API int pxb_pipeline_train_step(const pxb_pipeline_train *t, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* PXB_H_ */
