// A chunk of steps as one device-side loop (src/plastax/driver.py:170-317,
// Driver.scan): the step's captured CUDA graph becomes the body of a
// conditional WHILE node, so a launch runs up to `count` steps with no host
// round trip between them and stops itself right after a step that
// overflowed (or, with `resorts`, that needs a resort).
//
//   head:   cond = (i < count)
//   WHILE cond:
//     fetch:  the chunk's row i of inputs (and targets) into the step's buffers
//     step:   the captured step graph (a child graph node)
//     tail:   record row i (loss, output activations); i += 1;
//             halted = overflow | (resorts & needs_resort);
//             status = i * 2 + halted; cond = (i < count) & !halted
//
// The condition is reset to 0 at every launch and i grows by one per
// iteration, so the loop ends after at most count - i0 iterations.
#include "pxb_common.cuh"

namespace pxb {

struct LoopK {
  int32_t *i;
  int32_t count;
  const float *in_chunk;
  int32_t in_cols;
  float *in_buf;
  const float *tgt_chunk;
  int32_t tgt_cols;
  float *tgt_buf;
  const float *loss;
  float *loss_rec;
  const float *act;
  const int32_t *out_ids;
  int32_t n_out;
  float *out_rec;
  const uint8_t *overflow;
  const uint8_t *needs_resort;
  int32_t resorts;
  int32_t *status;
  cudaGraphConditionalHandle cond;
};

__global__ void loop_head_kernel(LoopK k) {
  if (threadIdx.x == 0) {
    const int32_t i = *k.i;
    *k.status = i * 2;
    cudaGraphSetConditional(k.cond, i < k.count ? 1u : 0u);
  }
}

__global__ void loop_fetch_kernel(LoopK k) {
  const int64_t i = *k.i;
  for (int t = threadIdx.x; t < k.in_cols; t += blockDim.x) k.in_buf[t] = k.in_chunk[i * k.in_cols + t];
  if (k.tgt_chunk != nullptr)
    for (int t = threadIdx.x; t < k.tgt_cols; t += blockDim.x) k.tgt_buf[t] = k.tgt_chunk[i * k.tgt_cols + t];
}

__global__ void loop_tail_kernel(LoopK k) {
  const int32_t i = *k.i;
  if (k.out_rec != nullptr)
    for (int t = threadIdx.x; t < k.n_out; t += blockDim.x)
      k.out_rec[static_cast<int64_t>(i) * k.n_out + t] = k.act[k.out_ids[t]];
  __syncthreads();
  if (threadIdx.x == 0) {
    if (k.loss_rec != nullptr) k.loss_rec[i] = *k.loss;
    const bool halted = (k.overflow != nullptr && *k.overflow) ||
                        (k.resorts && k.needs_resort != nullptr && *k.needs_resort);
    const int32_t next = i + 1;
    *k.i = next;
    *k.status = next * 2 + (halted ? 1 : 0);
    cudaGraphSetConditional(k.cond, (next < k.count && !halted) ? 1u : 0u);
  }
}

struct LoopHandle {
  cudaGraph_t graph;
  cudaGraphExec_t exec;
};

static cudaError_t add_kernel(cudaGraphNode_t *node, cudaGraph_t g, const cudaGraphNode_t *deps, size_t ndeps,
                              void *func, LoopK *k) {
  cudaKernelNodeParams p = {};
  p.func = func;
  p.gridDim = dim3(1);
  p.blockDim = dim3(256);
  p.sharedMemBytes = 0;
  void *args[] = {k};
  p.kernelParams = args;
  p.extra = nullptr;
  return cudaGraphAddKernelNode(node, g, deps, ndeps, &p);
}

}  // namespace pxb

using namespace pxb;

extern "C" int pxb_loop_build(void *step_graph, const pxb_loop_desc *d, void **loop_out) {
  PXB_REQUIRE(step_graph && d && loop_out, "pxb_loop_build: a pointer is NULL");
  PXB_REQUIRE(d->counter && d->status && d->in_chunk && d->in_buf && d->in_cols >= 0 && d->count >= 0,
              "pxb_loop_build: the counter, status and input chunk are required");
  PXB_REQUIRE(d->tgt_chunk == nullptr || (d->tgt_buf && d->tgt_cols >= 0), "pxb_loop_build: targets need a buffer");
  PXB_REQUIRE(d->out_rec == nullptr || (d->act && d->out_ids && d->n_out >= 0),
              "pxb_loop_build: output records need the activation column and the output ids");
  LoopK k{d->counter, d->count,     d->in_chunk, d->in_cols,  d->in_buf,       d->tgt_chunk, d->tgt_cols,
          d->tgt_buf, d->loss,      d->loss_rec, d->act,      d->out_ids,      d->n_out,     d->out_rec,
          d->overflow, d->needs_resort, d->resorts, d->status, 0};
  auto *h = new LoopHandle{nullptr, nullptr};
  cudaError_t e = cudaGraphCreate(&h->graph, 0);
  cudaGraphNode_t head = nullptr, loop = nullptr, fetch = nullptr, step = nullptr, tail = nullptr;
  cudaGraph_t body = nullptr;
  if (e == cudaSuccess) e = cudaGraphConditionalHandleCreate(&k.cond, h->graph, 0, cudaGraphCondAssignDefault);
  if (e == cudaSuccess) e = add_kernel(&head, h->graph, nullptr, 0, reinterpret_cast<void *>(loop_head_kernel), &k);
  if (e == cudaSuccess) {
    cudaGraphNodeParams cp = {};
    cp.type = cudaGraphNodeTypeConditional;
    cp.conditional.handle = k.cond;
    cp.conditional.type = cudaGraphCondTypeWhile;
    cp.conditional.size = 1;
    e = cudaGraphAddNode(&loop, h->graph, &head, 1, &cp);
    if (e == cudaSuccess) body = cp.conditional.phGraph_out[0];
  }
  if (e == cudaSuccess) e = add_kernel(&fetch, body, nullptr, 0, reinterpret_cast<void *>(loop_fetch_kernel), &k);
  if (e == cudaSuccess) e = cudaGraphAddChildGraphNode(&step, body, &fetch, 1, static_cast<cudaGraph_t>(step_graph));
  if (e == cudaSuccess) e = add_kernel(&tail, body, &step, 1, reinterpret_cast<void *>(loop_tail_kernel), &k);
  if (e == cudaSuccess) e = cudaGraphInstantiate(&h->exec, h->graph, 0);
  if (e != cudaSuccess) {
    if (h->graph) cudaGraphDestroy(h->graph);
    delete h;
    set_error("pxb_loop_build: %s", cudaGetErrorString(e));
    return PXB_ECUDA;
  }
  *loop_out = h;
  return PXB_OK;
}

extern "C" int pxb_loop_launch(void *loop, void *stream) {
  PXB_REQUIRE(loop != nullptr, "pxb_loop_launch: loop is NULL");
  PXB_CUDA(cudaGraphLaunch(static_cast<LoopHandle *>(loop)->exec, as_stream(stream)));
  return PXB_OK;
}

extern "C" int pxb_loop_destroy(void *loop) {
  PXB_REQUIRE(loop != nullptr, "pxb_loop_destroy: loop is NULL");
  auto *h = static_cast<LoopHandle *>(loop);
  cudaError_t e1 = h->exec ? cudaGraphExecDestroy(h->exec) : cudaSuccess;
  cudaError_t e2 = h->graph ? cudaGraphDestroy(h->graph) : cudaSuccess;
  delete h;
  if (e1 != cudaSuccess || e2 != cudaSuccess) {
    set_error("pxb_loop_destroy: %s", cudaGetErrorString(e1 != cudaSuccess ? e1 : e2));
    return PXB_ECUDA;
  }
  return PXB_OK;
}

// A captured step graph instantiated with the kernels' own priorities: the
// side stream's selection (captured at low priority) then yields SMs to the
// main stream's kernels whenever both have CTAs waiting.
extern "C" int pxb_graph_instantiate(void *graph, int32_t node_priority, void **exec_out) {
  PXB_REQUIRE(graph && exec_out, "pxb_graph_instantiate: a pointer is NULL");
  cudaGraphExec_t exec = nullptr;
  const unsigned long long flags = node_priority ? cudaGraphInstantiateFlagUseNodePriority : 0;
  PXB_CUDA(cudaGraphInstantiateWithFlags(&exec, static_cast<cudaGraph_t>(graph), flags));
  *exec_out = exec;
  return PXB_OK;
}

extern "C" int pxb_graph_launch(void *exec, void *stream) {
  PXB_REQUIRE(exec != nullptr, "pxb_graph_launch: exec is NULL");
  PXB_CUDA(cudaGraphLaunch(static_cast<cudaGraphExec_t>(exec), as_stream(stream)));
  return PXB_OK;
}

extern "C" int pxb_graph_exec_destroy(void *exec) {
  PXB_REQUIRE(exec != nullptr, "pxb_graph_exec_destroy: exec is NULL");
  PXB_CUDA(cudaGraphExecDestroy(static_cast<cudaGraphExec_t>(exec)));
  return PXB_OK;
}
