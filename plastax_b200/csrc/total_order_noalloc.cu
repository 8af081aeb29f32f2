// Allocation-free variant of the total order, for callers that cannot
// allocate device memory (and so cannot provide pxb_total_order's scratch).
//
// Who needs it: a host that calls the engine from inside a region where any
// cudaMalloc is forbidden or unavailable -- an XLA/JAX FFI handler running
// under command-buffer (CUDA graph) capture, a plugin loaded into a process
// whose allocator owns all device memory and hands out none, or a real-time
// loop that must not hit the driver's allocator. Such callers still pass
// their inputs and output; the sort's scratch lives in a fixed device array
// of this library instead.
//
// The array (kNoAllocBytes, 16 MiB) is a file-scope __device__ variable:
// every GPU that loads libpxb.so holds it until the process exits. Its host
// name is only a stand-in for the symbol, so the device address is fetched
// once per device with cudaGetSymbolAddress (with that device current) and
// cached; the first call on a device does that set-up, so it should come
// before any stream capture. Every call on a device shares the array and it
// keeps the last call's contents; nothing in it needs to start at zero (the
// keys are written before they are read and CUB initialises its own
// temporary storage). Calls that overlap on the GPU (two streams, or two
// host threads on one device) race on the array: serialise them. The cached
// address belongs to the device's context as it was at the first call: after
// cudaDeviceReset (or anything else that replaces the primary context) it no
// longer names the array, so a process that resets a device must not call
// this entry point on that device again.
#include <mutex>

#include "pxb_common.cuh"

namespace pxb {

int total_order_impl(const char *fn, int64_t n, const float *score, const int32_t *src, const int32_t *dst,
                     int32_t id_bound, int32_t *perm_out, void *scratch, size_t scratch_bytes, cudaStream_t st);
size_t total_order_bytes(int64_t n, int32_t id_bound);

constexpr size_t kNoAllocBytes = size_t(16) << 20;
constexpr int64_t kNoAllocMaxN = int64_t(1) << 18;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

static std::mutex g_noalloc_mu;
static void *g_noalloc_ptr[kMaxDevices];

// The array's device address on the current device (fetched once per device).
static int noalloc_scratch(void **out) {
  int dev = -1;
  PXB_CUDA(cudaGetDevice(&dev));
  PXB_REQUIRE(dev >= 0 && dev < kMaxDevices, "pxb_total_order_noalloc: device %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void *p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      set_error("pxb_total_order_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
      return PXB_ECUDA;
    }
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return PXB_OK;
}

}  // namespace pxb

using namespace pxb;

extern "C" int pxb_total_order_noalloc(int64_t n, const float *score, const int32_t *src, const int32_t *dst,
                                       int32_t id_bound, int32_t *perm_out, void *stream) {
  PXB_REQUIRE(n >= 0, "pxb_total_order_noalloc: negative n");
  PXB_REQUIRE(n <= kNoAllocMaxN, "pxb_total_order_noalloc: n = %lld candidates exceeds the maximum %lld",
              static_cast<long long>(n), static_cast<long long>(kNoAllocMaxN));
  PXB_REQUIRE(id_bound >= 1, "pxb_total_order_noalloc: id_bound must be >= 1");
  if (n == 0) return PXB_OK;
  const size_t need = total_order_bytes(n, id_bound);
  PXB_REQUIRE(need <= kNoAllocBytes, "pxb_total_order_noalloc: n = %lld needs %zu scratch bytes, over the %zu held",
              static_cast<long long>(n), need, kNoAllocBytes);
  void *scratch = nullptr;
  const int rc = noalloc_scratch(&scratch);
  if (rc != PXB_OK) return rc;
  return total_order_impl("pxb_total_order_noalloc", n, score, src, dst, id_bound, perm_out, scratch, kNoAllocBytes,
                          as_stream(stream));
}
