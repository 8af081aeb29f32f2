// Library-level entry points: ABI version, error text, device facts, fills.
#include <mutex>
#include <vector>

#include "pxb_common.cuh"

namespace pxb {

static thread_local std::string g_last_error;

void set_error(const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
}

const char *last_error() { return g_last_error.c_str(); }

int sm_count() {
  static std::mutex mu;
  static std::vector<int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  std::lock_guard<std::mutex> lock(mu);
  if (dev >= static_cast<int>(cache.size())) cache.resize(dev + 1, 0);
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

// A forward's accumulators reset in one pass: the float column to the
// monoid's identity and the fixed-point column to zero.
// A step's inputs scattered into the activation column straight from the
// caller's buffer (pinned host memory, read over the bus, or device memory).
__global__ void scatter_inputs_kernel(int32_t n, const int64_t *__restrict__ ids, const float *__restrict__ src,
                                      float *__restrict__ act) {
  for (int i = threadIdx.x; i < n; i += blockDim.x) act[ids[i]] = src[i];
}

// A step's growth flags (grown, overflow) as two int32 into the caller's
// buffer (pinned host memory, written over the bus, or device memory).
__global__ void flags_out_kernel(const int32_t *grown, const uint8_t *overflow, int32_t *out) {
  if (threadIdx.x == 0) {
    out[0] = grown != nullptr ? *grown : 0;
    out[1] = overflow != nullptr ? static_cast<int32_t>(*overflow) : 0;
  }
}

__global__ void clear_acc_kernel(int64_t n, float v, float *__restrict__ acc, int64_t *__restrict__ fixed) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n; i += stride) {
    acc[i] = v;
    if (fixed != nullptr) fixed[i] = 0;
  }
}

__global__ void fill_f32_kernel(int64_t n, float v, float *__restrict__ out) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    out[i] = v;
}

}  // namespace pxb

extern "C" int pxb_abi_version(void) { return PXB_ABI_VERSION; }

extern "C" const char *pxb_last_error(void) { return pxb::last_error(); }

extern "C" int pxb_sm_count(int32_t *out) {
  PXB_REQUIRE(out != nullptr, "pxb_sm_count: out is NULL");
  *out = pxb::sm_count();
  return PXB_OK;
}

extern "C" int pxb_set_device(int32_t device) {
  PXB_CUDA(cudaSetDevice(device));
  return PXB_OK;
}

extern "C" int pxb_get_device(int32_t *device) {
  PXB_REQUIRE(device != nullptr, "pxb_get_device: device is NULL");
  int d = -1;
  PXB_CUDA(cudaGetDevice(&d));
  *device = d;
  return PXB_OK;
}

extern "C" int pxb_fill_f32(int64_t n, float value, float *out, void *stream) {
  PXB_REQUIRE(n >= 0, "pxb_fill_f32: negative n");
  if (n == 0) return PXB_OK;
  PXB_REQUIRE(out != nullptr, "pxb_fill_f32: out is NULL");
  pxb::fill_f32_kernel<<<pxb::grid_for(n, 1024, 4), 256, 0, pxb::as_stream(stream)>>>(n, value, out);
  PXB_LAUNCHED("fill_f32_kernel");
  return PXB_OK;
}

extern "C" int pxb_clear_accumulators(int64_t n, float value, float *acc, int64_t *acc_fixed, void *stream) {
  PXB_REQUIRE(n >= 0, "pxb_clear_accumulators: negative n");
  if (n == 0) return PXB_OK;
  PXB_REQUIRE(acc != nullptr, "pxb_clear_accumulators: acc is NULL");
  pxb::clear_acc_kernel<<<pxb::grid_for(n, 1024, 4), 256, 0, pxb::as_stream(stream)>>>(n, value, acc, acc_fixed);
  PXB_LAUNCHED("clear_acc_kernel");
  return PXB_OK;
}

extern "C" int pxb_scatter_inputs(int32_t n, const int64_t *ids, const float *src, float *act, void *stream) {
  PXB_REQUIRE(n >= 0, "pxb_scatter_inputs: negative n");
  if (n == 0) return PXB_OK;
  PXB_REQUIRE(ids && src && act, "pxb_scatter_inputs: a pointer is NULL");
  pxb::scatter_inputs_kernel<<<1, 256, 0, pxb::as_stream(stream)>>>(n, ids, src, act);
  PXB_LAUNCHED("scatter_inputs_kernel");
  return PXB_OK;
}

extern "C" int pxb_flags_out(const int32_t *grown, const uint8_t *overflow, int32_t *out, void *stream) {
  PXB_REQUIRE(out != nullptr, "pxb_flags_out: out is NULL");
  pxb::flags_out_kernel<<<1, 32, 0, pxb::as_stream(stream)>>>(grown, overflow, out);
  PXB_LAUNCHED("flags_out_kernel");
  return PXB_OK;
}

extern "C" int pxb_host_device_pointer(void *host, void **dev_out) {
  PXB_REQUIRE(host && dev_out, "pxb_host_device_pointer: a pointer is NULL");
  const cudaError_t e = cudaHostGetDevicePointer(dev_out, host, 0);
  if (e != cudaSuccess) {
    cudaGetLastError();  // not a sticky error: the next launch must not see it
    pxb::set_error("pxb_host_device_pointer: %s", cudaGetErrorString(e));
    return PXB_ECUDA;
  }
  return PXB_OK;
}
