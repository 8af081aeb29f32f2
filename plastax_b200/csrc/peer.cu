// Scheme-A reduction of the forward's per-unit partials over NVLink peer
// memory, fused with the unit apply.
//
// Under Scheme-A every rank sweeps its band of the arena and holds a partial
// sum for every unit (src/plastax/monoid.py:175-204, an all-reduce in the
// reference). Here each rank owns a symmetric region (same layout on every
// rank, mapped into every peer through CUDA IPC): the int64 fixed-point
// partials, the float side partials, the activation column and two rows of
// flags. One kernel per step:
//   1. signals "my partials are complete" into every peer's flag row A and
//      waits until every peer has signalled (the sweep ran before it on the
//      stream, so its writes precede the release);
//   2. reduces its slice of the units, [rank * ceil(n / G), ...), by loading
//      every peer's partials (exact int64 sum, the float side added in rank
//      order), applies the activation once and stores it into every peer's
//      activation column;
//   3. the last block to finish signals row B ("done reading your partials,
//      done writing your activations") to every peer and waits for theirs,
//      so no rank clears its partials or reads activations early.
// The epoch (a device counter) makes the kernel replayable from a CUDA graph.
// Every wait is bounded: after `wait_polls` polls it gives up, sets status bit
// 0 and goes on (the step's result is then incomplete and the host can see
// it), so a rank that never arrives cannot hang the GPU.
#include "pxb_common.cuh"

namespace pxb {

struct PeerK {
  int32_t rank, world;
  int64_t *const *acc_fixed;
  float *const *acc_side;
  float *const *act;
  uint32_t *const *flags;
  int32_t *const *counts;
  uint32_t *epoch, *done;
  int32_t *status;
};

// The claim's per-domain free counts riding on the barrier: this rank's
// counts go into row `rank` of every peer's counts area before the release.
struct CountsK {
  const int32_t *local;  // [num_levels], or NULL
  int32_t num_levels;
  int32_t *before, *totals;  // [num_levels] out
};

__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Wait until row[q] has reached `epoch` for every rank q; false after
// `polls` unsuccessful polls of one flag.
__device__ bool wait_row(const uint32_t *row, int world, uint32_t epoch, uint32_t polls) {
  for (int q = 0; q < world; ++q) {
    uint32_t i = 0;
    while (static_cast<int32_t>(ld_acquire_sys(row + q) - epoch) < 0) {
      if (++i >= polls) return false;
      __nanosleep(128);
    }
  }
  return true;
}

constexpr float kFixUnitP = 1.0f / float(1ll << PXB_FIXED_FRAC_BITS);
constexpr int kPeerMaxLevels = PXB_PEER_MAX_LEVELS;

__global__ void __launch_bounds__(256) scheme_a_apply_kernel(PeerK g, int32_t n, int32_t act_kind,
                                                            const uint8_t *__restrict__ is_input,
                                                            const uint8_t *__restrict__ pruned, uint32_t polls,
                                                            CountsK c) {
  __shared__ int s_ok;
  const uint32_t epoch = *g.epoch + 1u;
  if (blockIdx.x == 0) {
    if (c.local != nullptr)
      for (int i = threadIdx.x; i < g.world * c.num_levels; i += blockDim.x) {
        const int q = i / c.num_levels, l = i - q * c.num_levels;
        g.counts[q][g.rank * kPeerMaxLevels + l] = c.local[l];
      }
    __syncthreads();
    if (threadIdx.x < static_cast<unsigned>(g.world)) {
      __threadfence_system();
      st_release_sys(g.flags[threadIdx.x] + g.rank, epoch);  // row A of peer threadIdx.x
    }
  }
  if (threadIdx.x == 0) {
    s_ok = wait_row(g.flags[g.rank], g.world, epoch, polls) ? 1 : 0;
    // a block that gave up skips its share of the units: the step is
    // incomplete whichever block finishes last
    if (!s_ok) atomicOr(g.status, 1);
  }
  __syncthreads();
  if (blockIdx.x == 0 && c.local != nullptr && threadIdx.x < static_cast<unsigned>(c.num_levels)) {
    // every rank's counts are here now: the ranks before this one and the total
    const int32_t *rows = g.counts[g.rank];
    int32_t before = 0, total = 0;
    for (int q = 0; q < g.world; ++q) {
      const int32_t v = rows[q * kPeerMaxLevels + threadIdx.x];
      if (q < g.rank) before += v;
      total += v;
    }
    c.before[threadIdx.x] = before;
    c.totals[threadIdx.x] = total;
  }
  if (s_ok) {
    const int32_t per = (n + g.world - 1) / g.world;
    const int32_t lo = g.rank * per;
    const int32_t hi = lo + per < n ? lo + per : n;
    const int32_t stride = gridDim.x * blockDim.x;
    // kUnits units per thread at a time, every rank's partials of all of
    // them (kRanks ranks at a time) loaded before any is used: a remote load
    // is a round trip over NVLink, so the loads of one thread overlap
    constexpr int kUnits = 4, kRanks = 4;
    for (int32_t u0 = lo + blockIdx.x * blockDim.x + threadIdx.x; u0 < hi; u0 += kUnits * stride) {
      long long f[kUnits];
      float side[kUnits];
      uint8_t role[kUnits], gone[kUnits];
#pragma unroll
      for (int i = 0; i < kUnits; ++i) {
        const int32_t u = u0 + i * stride;
        const bool in = u < hi;
        role[i] = in && is_input != nullptr ? is_input[u] : 0;
        gone[i] = in && pruned != nullptr ? pruned[u] : 0;
        f[i] = 0;
        side[i] = 0.0f;
      }
      for (int q0 = 0; q0 < g.world; q0 += kRanks) {
        long long fq[kUnits][kRanks];
        float sq[kUnits][kRanks];
#pragma unroll
        for (int i = 0; i < kUnits; ++i) {
          const int32_t u = u0 + i * stride;
#pragma unroll
          for (int j = 0; j < kRanks; ++j) {
            const bool v = u < hi && q0 + j < g.world;
            fq[i][j] = v ? g.acc_fixed[q0 + j][u] : 0;
            sq[i][j] = v ? g.acc_side[q0 + j][u] : 0.0f;
          }
        }
        // combined in rank order (the float side partials' order is fixed)
#pragma unroll
        for (int i = 0; i < kUnits; ++i)
#pragma unroll
          for (int j = 0; j < kRanks; ++j)
            if (q0 + j < g.world) {
              f[i] += fq[i][j];
              side[i] = __fadd_rn(side[i], sq[i][j]);
            }
      }
#pragma unroll
      for (int i = 0; i < kUnits; ++i) {
        const int32_t u = u0 + i * stride;
        if (u >= hi || role[i] == 1 || gone[i]) continue;
        const float x = f[i] != 0 ? __fadd_rn(__fmul_rn(__ll2float_rn(f[i]), kFixUnitP), side[i]) : side[i];
        const float a = act_fn(unit_act_kind(act_kind, role[i]), x);
        for (int q = 0; q < g.world; ++q) g.act[q][u] = a;
      }
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t prev = atomicAdd(g.done, 1u);
    if (prev == gridDim.x - 1) {  // the last block: every read and write of this rank is done
      *g.done = 0;
      __threadfence_system();
      for (int q = 0; q < g.world; ++q) st_release_sys(g.flags[q] + g.world + g.rank, epoch);  // row B
      const bool ok_b = wait_row(g.flags[g.rank] + g.world, g.world, epoch, polls);
      if (!s_ok || !ok_b) atomicOr(g.status, 1);
      *g.epoch = epoch;
    }
  }
}

}  // namespace pxb

using namespace pxb;

extern "C" int pxb_peer_alloc(size_t bytes, void **ptr_out, uint8_t *ipc_handle_out) {
  PXB_REQUIRE(ptr_out && ipc_handle_out && bytes > 0, "pxb_peer_alloc: bad arguments");
  void *p = nullptr;
  PXB_CUDA(cudaMalloc(&p, bytes));
  cudaError_t e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) {
    cudaIpcMemHandle_t h;
    e = cudaIpcGetMemHandle(&h, p);
    if (e == cudaSuccess) memcpy(ipc_handle_out, &h, sizeof(h));
  }
  if (e != cudaSuccess) {
    cudaFree(p);
    set_error("pxb_peer_alloc: %s", cudaGetErrorString(e));
    return PXB_ECUDA;
  }
  *ptr_out = p;
  return PXB_OK;
}

extern "C" int pxb_peer_open(const uint8_t *ipc_handle, void **ptr_out) {
  PXB_REQUIRE(ipc_handle && ptr_out, "pxb_peer_open: bad arguments");
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  PXB_CUDA(cudaIpcOpenMemHandle(ptr_out, h, cudaIpcMemLazyEnablePeerAccess));
  return PXB_OK;
}

extern "C" int pxb_peer_close(void *ptr) {
  PXB_REQUIRE(ptr != nullptr, "pxb_peer_close: ptr is NULL");
  PXB_CUDA(cudaIpcCloseMemHandle(ptr));
  return PXB_OK;
}

extern "C" int pxb_peer_free(void *ptr) {
  PXB_REQUIRE(ptr != nullptr, "pxb_peer_free: ptr is NULL");
  PXB_CUDA(cudaFree(ptr));
  return PXB_OK;
}

extern "C" int pxb_scheme_a_apply(const pxb_peer_group *group, int32_t num_units, int32_t act_kind,
                                  const uint8_t *is_input, const uint8_t *pruned, const int32_t *level_counts,
                                  int32_t num_levels, int32_t *level_before, int32_t *level_totals,
                                  uint32_t wait_polls, void *stream) {
  PXB_REQUIRE(group != nullptr, "pxb_scheme_a_apply: group is NULL");
  PXB_REQUIRE(group->world >= 1 && group->world <= 64 && group->rank >= 0 && group->rank < group->world,
              "pxb_scheme_a_apply: rank %d / world %d out of range", group->rank, group->world);
  PXB_REQUIRE(group->acc_fixed && group->acc_side && group->act && group->flags && group->epoch && group->done &&
                  group->status,
              "pxb_scheme_a_apply: a group array is NULL");
  PXB_REQUIRE(num_units >= 0, "pxb_scheme_a_apply: negative num_units");
  PXB_REQUIRE(act_code_ok(act_kind), "pxb_scheme_a_apply: unknown activation code %d", act_kind);
  PXB_REQUIRE(wait_polls >= 1, "pxb_scheme_a_apply: wait_polls must be >= 1");
  PXB_REQUIRE(level_counts == nullptr ||
                  (group->counts && level_before && level_totals && num_levels >= 1 && num_levels <= kPeerMaxLevels),
              "pxb_scheme_a_apply: level counts need the group's counts areas, outputs and 1..%d levels",
              kPeerMaxLevels);
  PeerK g{group->rank,   group->world,  group->acc_fixed, group->acc_side, group->act, group->flags,
          group->counts, group->epoch,  group->done,      group->status};
  CountsK c{level_counts, num_levels, level_before, level_totals};
  const int32_t per = (num_units + group->world - 1) / group->world;
  const int grid = grid_for(per > 0 ? per : 1, 256, 2);
  scheme_a_apply_kernel<<<grid, 256, 0, as_stream(stream)>>>(g, num_units, act_kind, is_input, pruned, wait_polls,
                                                               c);
  PXB_LAUNCHED("scheme_a_apply_kernel");
  return PXB_OK;
}
