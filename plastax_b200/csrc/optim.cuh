// The per-connection optimizer step, shared by the backward sweep
// (sweep.cu) and the fused pipeline training step (train.cu).
#pragma once

#include "pxb_common.cuh"

namespace pxb {

// ---------------------------------------------------------------------------
// optimizer step (src/plastax/optim/_sgd.py:124-127, _momentum.py:136-139,
// _adam.py:157-172, _rmsprop.py:135-140), one connection, rounding kept
// per operation (no contraction) so it follows the reference's float32 order.
// ---------------------------------------------------------------------------
struct OptParams {
  int kind;
  float lr, b1, b2, eps, wd;
  const float *scale;  // upgd: eta per destination unit
};

// examples/dst_sparse.py:77-85: three words hashed to a float in [0, 1).
__device__ __forceinline__ float hash01(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t h = (a + 0x9E3779B1u) * 0x85EBCA77u;
  h = (h ^ b) * 0xC2B2AE3Du;
  h = (h ^ c) * 0x27D4EB2Fu;
  h ^= h >> 15;
  h *= 0x2C1B3C6Du;
  h ^= h >> 13;
  return __fdiv_rn(static_cast<float>(h >> 8), 16777216.0f);
}

// examples/upgd.py:160-199, float32 operation by operation.
__device__ __forceinline__ void upgd_step(const OptParams &p, float grad, float &w, float *u_col, float *t_col,
                                          int64_t s, int32_t src, int32_t dst) {
  const float inst = __fmul_rn(-grad, w);
  const float step = __fadd_rn(t_col[s], 1.0f);
  const float util = __fadd_rn(__fmul_rn(p.b1, u_col[s]), __fmul_rn(__fsub_rn(1.0f, p.b1), inst));
  const float corrected = __fdiv_rn(util, fmaxf(__fsub_rn(1.0f, powf(p.b1, step)), p.eps));
  const float scale = fmaxf(p.scale[dst], p.eps);
  const float gated = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-__fdiv_rn(corrected, scale))));
  const uint32_t salt = static_cast<uint32_t>(static_cast<int32_t>(step));
  const float u1 = fmaxf(hash01(static_cast<uint32_t>(src), static_cast<uint32_t>(dst), salt), 1e-7f);
  const float u2 = hash01(static_cast<uint32_t>(dst), static_cast<uint32_t>(src), salt);
  const float gauss = __fmul_rn(__fsqrt_rn(__fmul_rn(-2.0f, logf(u1))), cosf(__fmul_rn(6.2831855f, u2)));
  const float noise = __fmul_rn(p.b2, gauss);
  w = __fsub_rn(w, __fmul_rn(__fmul_rn(p.lr, __fadd_rn(grad, noise)), __fsub_rn(1.0f, gated)));
  u_col[s] = util;
  t_col[s] = step;
}

__device__ __forceinline__ void opt_step(const OptParams &p, float grad, float &w, float *m_col,
                                         float *v_col, float *t_col, int64_t s, int32_t src = 0,
                                         int32_t dst = 0) {
  switch (p.kind) {
    case PXB_OPT_UPGD:
      upgd_step(p, grad, w, m_col, t_col, s, src, dst);
      break;
    case PXB_OPT_SGD:
      w = __fsub_rn(w, __fmul_rn(p.lr, grad));
      break;
    case PXB_OPT_MOMENTUM: {
      const float vel = __fadd_rn(__fmul_rn(p.b1, v_col[s]), grad);
      v_col[s] = vel;
      w = __fsub_rn(w, __fmul_rn(p.lr, vel));
      break;
    }
    case PXB_OPT_ADAM: {
      const float step = __fadd_rn(t_col[s], 1.0f);
      const float m = __fadd_rn(__fmul_rn(p.b1, m_col[s]), __fmul_rn(__fsub_rn(1.0f, p.b1), grad));
      const float v = __fadd_rn(__fmul_rn(p.b2, v_col[s]),
                                __fmul_rn(__fsub_rn(1.0f, p.b2), __fmul_rn(grad, grad)));
      const float m_hat = __fdiv_rn(m, __fsub_rn(1.0f, powf(p.b1, step)));
      const float v_hat = __fdiv_rn(v, __fsub_rn(1.0f, powf(p.b2, step)));
      const float dir = __fdiv_rn(m_hat, __fadd_rn(__fsqrt_rn(v_hat), p.eps));
      const float upd = __fmul_rn(p.lr, __fadd_rn(dir, __fmul_rn(p.wd, w)));
      w = __fsub_rn(w, upd);
      m_col[s] = m;
      v_col[s] = v;
      t_col[s] = step;
      break;
    }
    case PXB_OPT_RMSPROP: {
      const float ms = __fadd_rn(__fmul_rn(p.b1, v_col[s]),
                                 __fmul_rn(__fsub_rn(1.0f, p.b1), __fmul_rn(grad, grad)));
      v_col[s] = ms;
      const float upd = __fdiv_rn(__fmul_rn(p.lr, grad), __fsqrt_rn(__fadd_rn(ms, p.eps)));
      w = __fsub_rn(w, upd);
      break;
    }
    default:
      break;
  }
}

}  // namespace pxb
