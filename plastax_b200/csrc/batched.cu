// Batched edge products for make_step(batch_size=B): unit columns are laid
// out [num_units, B] (one 4B*B row per unit), so each edge moves whole rows.
// A warp owns 32 consecutive slots per iteration: lane l loads slot l's
// (from, to, dead, w) once, then the warp walks the 32 slots, broadcasting
// each slot's ids by shuffle and moving its rows as float4 (B % 4 == 0).
//
// forward  out[to, :]   += w * x[from, :]   (vector atomics, sm_90+ RED.v4)
// backward out[from, :] += w * g[to, :]     (source-major runs are summed in
//                                             registers, one atomic per run)
// update   stat = (sum_b g[to, b] * a[from, b]) / B, then one optimizer step
//          (src/plastax/phases.py:434-483, the exact batch-mean update).
#include "pxb_common.cuh"

namespace pxb {

struct BOpt {
  int kind;
  float lr, b1, b2, eps, wd;
};

// Same float32 operation order as the streaming sweep's optimizer step.
__device__ __forceinline__ void bopt_step(const BOpt &p, float grad, float &w, float *m_col, float *v_col,
                                          float *t_col, int64_t s) {
  switch (p.kind) {
    case PXB_OPT_SGD: w = __fsub_rn(w, __fmul_rn(p.lr, grad)); break;
    case PXB_OPT_MOMENTUM: {
      const float vel = __fadd_rn(__fmul_rn(p.b1, v_col[s]), grad);
      v_col[s] = vel;
      w = __fsub_rn(w, __fmul_rn(p.lr, vel));
      break;
    }
    case PXB_OPT_ADAM: {
      const float step = __fadd_rn(t_col[s], 1.0f);
      const float m = __fadd_rn(__fmul_rn(p.b1, m_col[s]), __fmul_rn(__fsub_rn(1.0f, p.b1), grad));
      const float v = __fadd_rn(__fmul_rn(p.b2, v_col[s]), __fmul_rn(__fsub_rn(1.0f, p.b2), __fmul_rn(grad, grad)));
      const float m_hat = __fdiv_rn(m, __fsub_rn(1.0f, powf(p.b1, step)));
      const float v_hat = __fdiv_rn(v, __fsub_rn(1.0f, powf(p.b2, step)));
      const float dir = __fdiv_rn(m_hat, __fadd_rn(__fsqrt_rn(v_hat), p.eps));
      w = __fsub_rn(w, __fmul_rn(p.lr, __fadd_rn(dir, __fmul_rn(p.wd, w))));
      m_col[s] = m;
      v_col[s] = v;
      t_col[s] = step;
      break;
    }
    case PXB_OPT_RMSPROP: {
      const float ms = __fadd_rn(__fmul_rn(p.b1, v_col[s]), __fmul_rn(__fsub_rn(1.0f, p.b1), __fmul_rn(grad, grad)));
      v_col[s] = ms;
      w = __fsub_rn(w, __fdiv_rn(__fmul_rn(p.lr, grad), __fsqrt_rn(__fadd_rn(ms, p.eps))));
      break;
    }
    default: break;
  }
}

__device__ __forceinline__ float4 axpy4(float a, float4 x, float4 y) {
  return make_float4(__fadd_rn(y.x, __fmul_rn(a, x.x)), __fadd_rn(y.y, __fmul_rn(a, x.y)),
                     __fadd_rn(y.z, __fmul_rn(a, x.z)), __fadd_rn(y.w, __fmul_rn(a, x.w)));
}

constexpr int kMaxQ = 8;  // float4 per lane: B <= 32 * 4 * kMaxQ = 1024

template <int Q>
__global__ void __launch_bounds__(256) batched_forward_kernel(int64_t cap, const int32_t *__restrict__ from,
                                                              const int32_t *__restrict__ to,
                                                              const uint8_t *__restrict__ dead,
                                                              const float *__restrict__ weight,
                                                              const float4 *__restrict__ x, int32_t q4,
                                                              float4 *__restrict__ out, uint32_t n) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  const int64_t warps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t base = warp * 32; base < cap; base += warps * 32) {
    const int64_t s = base + lane;
    int32_t f = 0, t = 0;
    float w = 0.0f;
    bool live = false;
    if (s < cap) {
      f = from[s];
      t = to[s];
      w = weight[s];
      live = !dead[s] && static_cast<uint32_t>(f) < n && static_cast<uint32_t>(t) < n;
    }
    unsigned todo = __ballot_sync(0xffffffffu, live);
    while (todo) {
      const int j = __ffs(todo) - 1;
      todo &= todo - 1;
      const int32_t fj = __shfl_sync(0xffffffffu, f, j);
      const int32_t tj = __shfl_sync(0xffffffffu, t, j);
      const float wj = __shfl_sync(0xffffffffu, w, j);
      const float4 *xr = x + static_cast<int64_t>(fj) * q4;
      float4 *orow = out + static_cast<int64_t>(tj) * q4;
#pragma unroll
      for (int u = 0; u < Q; ++u) {
        const int q = lane + 32 * u;
        if (q < q4) {
          const float4 v = __ldg(xr + q);
          atomicAdd(orow + q, make_float4(__fmul_rn(wj, v.x), __fmul_rn(wj, v.y), __fmul_rn(wj, v.z),
                                          __fmul_rn(wj, v.w)));
        }
      }
    }
  }
}

template <int Q>
__global__ void __launch_bounds__(256) batched_backward_kernel(int64_t cap, const int32_t *__restrict__ from,
                                                               const int32_t *__restrict__ to,
                                                               const uint8_t *__restrict__ dead,
                                                               const float *__restrict__ weight,
                                                               const float4 *__restrict__ g, int32_t q4,
                                                               float4 *__restrict__ out, uint32_t n) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  const int64_t warps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t base = warp * 32; base < cap; base += warps * 32) {
    const int64_t s = base + lane;
    int32_t f = -1, t = 0;
    float w = 0.0f;
    bool live = false;
    if (s < cap) {
      f = from[s];
      t = to[s];
      w = weight[s];
      live = !dead[s] && static_cast<uint32_t>(f) < n && static_cast<uint32_t>(t) < n;
    }
    unsigned todo = __ballot_sync(0xffffffffu, live);
    float4 run[Q];
    int32_t run_src = -1;
    while (todo) {
      const int j = __ffs(todo) - 1;
      todo &= todo - 1;
      const int32_t fj = __shfl_sync(0xffffffffu, f, j);
      const int32_t tj = __shfl_sync(0xffffffffu, t, j);
      const float wj = __shfl_sync(0xffffffffu, w, j);
      if (fj != run_src) {
        if (run_src >= 0) {
          float4 *orow = out + static_cast<int64_t>(run_src) * q4;
#pragma unroll
          for (int u = 0; u < Q; ++u)
            if (lane + 32 * u < q4) atomicAdd(orow + lane + 32 * u, run[u]);
        }
#pragma unroll
        for (int u = 0; u < Q; ++u) run[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        run_src = fj;
      }
      const float4 *gr = g + static_cast<int64_t>(tj) * q4;
#pragma unroll
      for (int u = 0; u < Q; ++u)
        if (lane + 32 * u < q4) run[u] = axpy4(wj, __ldg(gr + lane + 32 * u), run[u]);
    }
    if (run_src >= 0) {
      float4 *orow = out + static_cast<int64_t>(run_src) * q4;
#pragma unroll
      for (int u = 0; u < Q; ++u)
        if (lane + 32 * u < q4) atomicAdd(orow + lane + 32 * u, run[u]);
    }
  }
}

template <int Q>
__global__ void __launch_bounds__(256) batched_update_kernel(int64_t cap, const int32_t *__restrict__ from,
                                                             const int32_t *__restrict__ to,
                                                             const uint8_t *__restrict__ dead,
                                                             float *__restrict__ weight,
                                                             const float4 *__restrict__ g,
                                                             const float4 *__restrict__ a, int32_t q4, float nb,
                                                             BOpt op, float *m_col, float *v_col, float *t_col,
                                                             uint32_t n) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  const int64_t warps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t base = warp * 32; base < cap; base += warps * 32) {
    const int64_t s = base + lane;
    int32_t f = 0, t = 0;
    bool live = false;
    if (s < cap) {
      f = from[s];
      t = to[s];
      live = !dead[s] && static_cast<uint32_t>(f) < n && static_cast<uint32_t>(t) < n;
    }
    float mine = 0.0f;
    unsigned todo = __ballot_sync(0xffffffffu, live);
    while (todo) {
      const int j = __ffs(todo) - 1;
      todo &= todo - 1;
      const int32_t fj = __shfl_sync(0xffffffffu, f, j);
      const int32_t tj = __shfl_sync(0xffffffffu, t, j);
      const float4 *gr = g + static_cast<int64_t>(tj) * q4;
      const float4 *ar = a + static_cast<int64_t>(fj) * q4;
      float part = 0.0f;
#pragma unroll
      for (int u = 0; u < Q; ++u) {
        const int q = lane + 32 * u;
        if (q < q4) {
          const float4 gv = __ldg(gr + q), av = __ldg(ar + q);
          part = __fadd_rn(part, __fmul_rn(gv.x, av.x));
          part = __fadd_rn(part, __fmul_rn(gv.y, av.y));
          part = __fadd_rn(part, __fmul_rn(gv.z, av.z));
          part = __fadd_rn(part, __fmul_rn(gv.w, av.w));
        }
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) part = __fadd_rn(part, __shfl_xor_sync(0xffffffffu, part, off));
      if (lane == j) mine = part;
    }
    if (live) {
      float w = weight[s];
      bopt_step(op, __fdiv_rn(mine, nb), w, m_col, v_col, t_col, s);
      weight[s] = w;
    }
  }
}

static int check_batch(const char *fn, int64_t cap, const void *from, const void *to, const void *dead,
                       const void *w, const void *x, int32_t batch, const void *out) {
  PXB_REQUIRE(cap >= 0, "%s: negative capacity", fn);
  PXB_REQUIRE(batch > 0 && batch % 4 == 0 && batch <= 32 * 4 * kMaxQ,
              "%s: batch %d must be a positive multiple of 4 up to %d", fn, batch, 32 * 4 * kMaxQ);
  if (cap == 0) return PXB_OK;
  PXB_REQUIRE(from && to && dead && w && x && out, "%s: a pointer is NULL", fn);
  PXB_REQUIRE(aligned16(x) && aligned16(out), "%s: unit rows must be 16-byte aligned", fn);
  return PXB_OK;
}


// ---------------------------------------------------------------------------
// the batched step's unit side: masked apply, per-sample loss, batch mean
// ---------------------------------------------------------------------------
// As pxb_unit_apply (sum monoid) for every (unit, sample) of [N, B] rows.
__global__ void batched_apply_kernel(int32_t n, int32_t batch, int mode, int act_kind, float *__restrict__ acc,
                                     const float *__restrict__ act, const float *__restrict__ seed,
                                     const int32_t *__restrict__ level, int32_t target_level,
                                     const uint8_t *__restrict__ is_input, float *__restrict__ out) {
  const int64_t total = static_cast<int64_t>(n) * batch;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int32_t u = static_cast<int32_t>(i / batch);
    if (level != nullptr && level[u] != target_level) continue;
    const uint8_t role = is_input != nullptr ? is_input[u] : 0;
    if (role == 1) continue;
    const int kind = unit_act_kind(act_kind, role);
    const float a = acc[i];
    if (mode == 0) {
      out[i] = act_fn(kind, a);
    } else {
      const float sd = seed != nullptr ? seed[i] : 0.0f;
      out[i] = __fmul_rn(__fadd_rn(a, sd), act_prime_from_act(kind, act[i]));
    }
    acc[i] = 0.0f;
  }
}

// One block per sample b: the loss of sample b and the seed rows of the
// outputs. MSE: seed = a - t, L = sum 0.5 d^2 in output order
// (scripts/parity/reference.py:338-352). Softmax cross-entropy
// (src/plastax/traits.py:205-250): m = max(a), z = a - m, s = sum exp(z) in
// output order, seed = exp(z) / s - t, L = sum t * (log(s) - z).
__global__ void batched_loss_kernel(int kind, int32_t k, const int32_t *__restrict__ ids, int32_t batch,
                                    const float *__restrict__ act, const float *__restrict__ target,
                                    float *__restrict__ seed, float *__restrict__ loss_b) {
  extern __shared__ float ez[];  // exp(z) per output
  __shared__ float s_max, s_sum;
  const int32_t b = blockIdx.x;
  const float *t = target + static_cast<int64_t>(b) * k;
  if (kind == PXB_LOSS_MSE) {
    for (int32_t j = threadIdx.x; j < k; j += blockDim.x)
      seed[static_cast<int64_t>(ids[j]) * batch + b] = __fsub_rn(act[static_cast<int64_t>(ids[j]) * batch + b], t[j]);
    __syncthreads();
    if (threadIdx.x == 0) {
      float total = 0.0f;
      for (int32_t j = 0; j < k; ++j) {
        const float d = seed[static_cast<int64_t>(ids[j]) * batch + b];
        total = __fadd_rn(total, __fmul_rn(__fmul_rn(0.5f, d), d));
      }
      loss_b[b] = total;
    }
    return;
  }
  if (threadIdx.x == 0) {
    float m = act[static_cast<int64_t>(ids[0]) * batch + b];
    for (int32_t j = 1; j < k; ++j) m = fmaxf(m, act[static_cast<int64_t>(ids[j]) * batch + b]);
    s_max = m;
  }
  __syncthreads();
  for (int32_t j = threadIdx.x; j < k; j += blockDim.x)
    ez[j] = expf(__fsub_rn(act[static_cast<int64_t>(ids[j]) * batch + b], s_max));
  __syncthreads();
  if (threadIdx.x == 0) {
    float total = 0.0f;
    for (int32_t j = 0; j < k; ++j) total = __fadd_rn(total, ez[j]);
    s_sum = total;
  }
  __syncthreads();
  for (int32_t j = threadIdx.x; j < k; j += blockDim.x)
    seed[static_cast<int64_t>(ids[j]) * batch + b] = __fsub_rn(__fdiv_rn(ez[j], s_sum), t[j]);
  if (threadIdx.x == 0) {
    const float lse = logf(s_sum);
    float total = 0.0f;
    for (int32_t j = 0; j < k; ++j) {
      const float z = __fsub_rn(act[static_cast<int64_t>(ids[j]) * batch + b], s_max);
      total = __fadd_rn(total, __fmul_rn(t[j], __fsub_rn(lse, z)));
    }
    loss_b[b] = total;
  }
}

// loss = (sum of the per-sample losses in sample order) / B.
__global__ void batch_mean_scalar_kernel(int32_t batch, const float *__restrict__ loss_b, float *__restrict__ loss) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  float total = 0.0f;
  for (int32_t b = 0; b < batch; ++b) total = __fadd_rn(total, loss_b[b]);
  loss[0] = __fdiv_rn(total, static_cast<float>(batch));
}

// out[u] = (sum_b x[u, b] in sample order) / B, one warp per unit: the row
// read 32 samples at a time (coalesced), the sum still taken one sample
// after another (every lane adds the broadcast values in order).
__global__ void batch_mean_rows_kernel(int32_t n, int32_t batch, const float *__restrict__ x, float *__restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t u = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5; u < n; u += warps) {
    const float *row = x + u * batch;
    float total = 0.0f;
    for (int32_t b0 = 0; b0 < batch; b0 += 32) {
      const float v = b0 + lane < batch ? row[b0 + lane] : 0.0f;
      const int cnt = batch - b0 < 32 ? batch - b0 : 32;
      for (int j = 0; j < cnt; ++j) total = __fadd_rn(total, __shfl_sync(0xffffffffu, v, j));
    }
    if (lane == 0) out[u] = __fdiv_rn(total, static_cast<float>(batch));
  }
}

}  // namespace pxb

using namespace pxb;

extern "C" int pxb_batched_forward(int64_t cap, const int32_t *from_id, const int32_t *to_id, const uint8_t *dead,
                                   const float *weight, const float *x, int32_t batch, int32_t num_units,
                                   float *out, void *stream) {
  int rc = check_batch("pxb_batched_forward", cap, from_id, to_id, dead, weight, x, batch, out);
  if (rc || cap == 0) return rc;
  const int32_t q4 = batch / 4;
  const int grid = grid_for((cap + 31) / 32, 8, 8);
  cudaStream_t st = as_stream(stream);
  const int q = (q4 + 31) / 32;
  const float4 *x4 = reinterpret_cast<const float4 *>(x);
  float4 *o4 = reinterpret_cast<float4 *>(out);
  const uint32_t n = static_cast<uint32_t>(num_units);
  if (q <= 1) batched_forward_kernel<1><<<grid, 256, 0, st>>>(cap, from_id, to_id, dead, weight, x4, q4, o4, n);
  else if (q <= 2) batched_forward_kernel<2><<<grid, 256, 0, st>>>(cap, from_id, to_id, dead, weight, x4, q4, o4, n);
  else if (q <= 4) batched_forward_kernel<4><<<grid, 256, 0, st>>>(cap, from_id, to_id, dead, weight, x4, q4, o4, n);
  else batched_forward_kernel<8><<<grid, 256, 0, st>>>(cap, from_id, to_id, dead, weight, x4, q4, o4, n);
  PXB_LAUNCHED("batched_forward_kernel");
  return PXB_OK;
}

extern "C" int pxb_batched_backward(int64_t cap, const int32_t *from_id, const int32_t *to_id, const uint8_t *dead,
                                    const float *weight, const float *g, int32_t batch, int32_t num_units,
                                    float *out, void *stream) {
  int rc = check_batch("pxb_batched_backward", cap, from_id, to_id, dead, weight, g, batch, out);
  if (rc || cap == 0) return rc;
  const int32_t q4 = batch / 4;
  const int grid = grid_for((cap + 31) / 32, 8, 8);
  cudaStream_t st = as_stream(stream);
  const int q = (q4 + 31) / 32;
  const float4 *g4 = reinterpret_cast<const float4 *>(g);
  float4 *o4 = reinterpret_cast<float4 *>(out);
  const uint32_t n = static_cast<uint32_t>(num_units);
  if (q <= 1) batched_backward_kernel<1><<<grid, 256, 0, st>>>(cap, from_id, to_id, dead, weight, g4, q4, o4, n);
  else if (q <= 2) batched_backward_kernel<2><<<grid, 256, 0, st>>>(cap, from_id, to_id, dead, weight, g4, q4, o4, n);
  else if (q <= 4) batched_backward_kernel<4><<<grid, 256, 0, st>>>(cap, from_id, to_id, dead, weight, g4, q4, o4, n);
  else batched_backward_kernel<8><<<grid, 256, 0, st>>>(cap, from_id, to_id, dead, weight, g4, q4, o4, n);
  PXB_LAUNCHED("batched_backward_kernel");
  return PXB_OK;
}

extern "C" int pxb_batched_update(int64_t cap, const int32_t *from_id, const int32_t *to_id, const uint8_t *dead,
                                  float *weight, const float *g, const float *a, int32_t batch, int32_t num_units,
                                  const pxb_optimizer *opt, float *opt_m, float *opt_v, float *opt_t,
                                  void *stream) {
  int rc = check_batch("pxb_batched_update", cap, from_id, to_id, dead, weight, g, batch, a);
  if (rc || cap == 0) return rc;
  PXB_REQUIRE(opt != nullptr && opt->kind >= 0 && opt->kind <= 3, "pxb_batched_update: bad optimizer");
  PXB_REQUIRE(opt->kind == PXB_OPT_SGD || opt_v, "pxb_batched_update: optimizer state column is NULL");
  PXB_REQUIRE(opt->kind != PXB_OPT_ADAM || (opt_m && opt_t), "pxb_batched_update: adam needs opt/m and opt/t");
  BOpt op{opt->kind, opt->lr, opt->b1, opt->b2, opt->eps, opt->weight_decay};
  const int32_t q4 = batch / 4;
  const int grid = grid_for((cap + 31) / 32, 8, 8);
  cudaStream_t st = as_stream(stream);
  const int q = (q4 + 31) / 32;
  const float4 *g4 = reinterpret_cast<const float4 *>(g);
  const float4 *a4 = reinterpret_cast<const float4 *>(a);
  const float nb = static_cast<float>(batch);
  const uint32_t n = static_cast<uint32_t>(num_units);
#define PXB_BU(QQ)                                                                                             \
  batched_update_kernel<QQ><<<grid, 256, 0, st>>>(cap, from_id, to_id, dead, weight, g4, a4, q4, nb, op,    \
                                                  opt_m, opt_v, opt_t, n)
  if (q <= 1) PXB_BU(1);
  else if (q <= 2) PXB_BU(2);
  else if (q <= 4) PXB_BU(4);
  else PXB_BU(8);
#undef PXB_BU
  PXB_LAUNCHED("batched_update_kernel");
  return PXB_OK;
}

extern "C" int pxb_batched_unit_apply(int32_t num_units, int32_t batch, int32_t mode, int32_t act_kind, float *acc,
                                      const float *act, const float *seed, const int32_t *level,
                                      int32_t target_level, const uint8_t *is_input, float *out, void *stream) {
  PXB_REQUIRE(num_units >= 0 && batch >= 1, "pxb_batched_unit_apply: bad sizes");
  PXB_REQUIRE(mode == 0 || mode == 1, "pxb_batched_unit_apply: mode must be 0 (forward) or 1 (backward)");
  PXB_REQUIRE(act_code_ok(act_kind), "pxb_batched_unit_apply: unknown activation code %d", act_kind);
  if (num_units == 0) return PXB_OK;
  PXB_REQUIRE(acc && out && (mode == 0 || act), "pxb_batched_unit_apply: a pointer is NULL");
  const int64_t total = int64_t(num_units) * batch;
  batched_apply_kernel<<<grid_for(total, 256, 8), 256, 0, as_stream(stream)>>>(
      num_units, batch, mode, act_kind, acc, act, seed, level, target_level, is_input, out);
  PXB_LAUNCHED("batched_apply_kernel");
  return PXB_OK;
}

extern "C" int pxb_batched_loss(int32_t kind, int32_t num_outputs, const int32_t *output_ids, int32_t batch,
                                const float *act, const float *target, float *seed, float *loss_per_sample,
                                float *loss_out, void *stream) {
  PXB_REQUIRE(kind == PXB_LOSS_MSE || kind == PXB_LOSS_SOFTMAX_CE, "pxb_batched_loss: unknown loss %d", kind);
  PXB_REQUIRE(num_outputs >= 1 && num_outputs <= 8192 && batch >= 1, "pxb_batched_loss: bad sizes");
  PXB_REQUIRE(output_ids && act && target && seed && loss_per_sample && loss_out, "pxb_batched_loss: a pointer is NULL");
  cudaStream_t st = as_stream(stream);
  batched_loss_kernel<<<batch, 256, num_outputs * sizeof(float), st>>>(kind, num_outputs, output_ids, batch, act,
                                                                      target, seed, loss_per_sample);
  PXB_LAUNCHED("batched_loss_kernel");
  batch_mean_scalar_kernel<<<1, 32, 0, st>>>(batch, loss_per_sample, loss_out);
  PXB_LAUNCHED("batch_mean_scalar_kernel");
  return PXB_OK;
}

extern "C" int pxb_batch_mean(int32_t num_units, int32_t batch, const float *x, float *out, void *stream) {
  PXB_REQUIRE(num_units >= 0 && batch >= 1, "pxb_batch_mean: bad sizes");
  if (num_units == 0) return PXB_OK;
  PXB_REQUIRE(x && out, "pxb_batch_mean: a pointer is NULL");
  batch_mean_rows_kernel<<<grid_for(num_units, 8, 8), 256, 0, as_stream(stream)>>>(num_units, batch, x, out);
  PXB_LAUNCHED("batch_mean_rows_kernel");
  return PXB_OK;
}
