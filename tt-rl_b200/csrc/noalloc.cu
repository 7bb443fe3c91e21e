// ttrl_linear_fwd_noalloc: the Linear forward GEMM with its split-K scratch
// taken from a fixed array compiled into this library instead of from a
// caller workspace.
//
// Who needs it: host code that cannot allocate device memory. Examples are
// an actor-side C host (an environment loop or an engine plugin) that links
// only this library and owns no memory pool to hand out workspace from, and
// a caller in a latency-critical loop, where cudaMalloc/cudaFree are ruled
// out because they can synchronise the device and stall work in flight on
// other streams. This entry point reaches no cudaMalloc, cudaFree or other
// allocating routine; it enqueues a 64 KB memset and the GEMM kernel(s), or
// nothing at all when it refuses the shape.
//
// The array is shared by every call on a device and keeps the previous
// call's contents. Calls whose GPU work overlaps (two streams, or two host
// threads on different streams) race on it and may produce wrong results.
// Calls issued to one stream are ordered and safe.
#include <mutex>

#include "internal.h"

namespace ttrl {

int linear_fwd(const float*, const float*, const float*, float*, int, int, int, int, int, float*,
               size_t, int*, cudaStream_t);
size_t linear_fwd_ws(int, int, int, int);

namespace {

constexpr int kMaxDevices = 64;

// [split-K arrival counters (kCounterBytes) | split-K partial sums].
__device__ __align__(256) unsigned char g_noalloc_scratch[TTRL_NOALLOC_SCRATCH_BYTES];

std::mutex g_setup_mutex;
float* g_scratch_ptr[kMaxDevices] = {};

// Once per device, with that device current: resolve the array's device
// address and set the GEMM kernels' shared-memory limits.
int scratch_for_current_device(float** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_cuda_error("ttrl_linear_fwd_noalloc: cudaGetDevice", e);
  if (dev < 0 || dev >= kMaxDevices)
    return set_error(TTRL_EUNSUPPORTED, "ttrl_linear_fwd_noalloc: device %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess)
      return set_cuda_error("ttrl_linear_fwd_noalloc: cudaGetSymbolAddress", e);
    const int rc = gemm_init_device();
    if (rc) return rc;
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_ptr[dev];
  return TTRL_OK;
}

}  // namespace

}  // namespace ttrl

using namespace ttrl;

extern "C" int ttrl_linear_fwd_noalloc(const float* x, const float* w, const float* b, float* y,
                                       int m, int k, int n, int relu, int precision, int* status,
                                       ttrl_stream_t stream) {
  if (m <= 0 || n <= 0 || k <= 0)
    return set_error(TTRL_EINVAL, "ttrl_linear_fwd_noalloc: bad extents m=%d k=%d n=%d", m, k, n);
  // The device set-up enqueues nothing; the split-K schedule (and so the
  // scratch it needs) depends on the cluster limit it records.
  float* scratch = nullptr;
  int rc = scratch_for_current_device(&scratch);
  if (rc) return rc;
  // Refuse an oversized shape before anything is enqueued: a refused call
  // must not touch the shared array, which a call on another stream may be
  // using.
  if (linear_fwd_ws(m, k, n, precision) > TTRL_NOALLOC_SCRATCH_BYTES)
    return set_error(TTRL_EWORKSPACE,
                     "ttrl_linear_fwd_noalloc: m=%d k=%d n=%d needs more split-K scratch than "
                     "the fixed %u bytes; use ttrl_linear_fwd with a caller workspace",
                     m, k, n, static_cast<unsigned>(TTRL_NOALLOC_SCRATCH_BYTES));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // The split-K kernels expect zeroed arrival counters. A completed call
  // leaves them zero, but a call that stopped early may not have, so clear
  // them every time. The partial sums are written before they are read.
  cudaError_t e = cudaMemsetAsync(scratch, 0, kCounterBytes, st);
  if (e != cudaSuccess) return set_cuda_error("ttrl_linear_fwd_noalloc: counter clear", e);
  return linear_fwd(x, w, b, y, m, k, n, relu, precision, scratch, TTRL_NOALLOC_SCRATCH_BYTES,
                    status, st);
}
