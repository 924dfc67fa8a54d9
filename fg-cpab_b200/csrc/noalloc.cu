// cpab_b200_order_points_static: cpab_b200_order_points without a scratch
// argument, for callers that cannot allocate device memory.
//
// Who needs it: a host that hands this library only the input and output
// buffers it already owns (a plugin framework or a language binding with no
// CUDA allocator of its own), code that must not call cudaMalloc/cudaFree
// because those calls can synchronize the whole device, and code that runs
// under a fixed device-memory budget decided up front.
//
// How: the per-cell counters that cpab_b200_order_points keeps in
// caller-provided scratch live instead in g_cell_counts, a fixed array
// compiled into this library.  Every GPU that loads the library holds it
// (kStaticCounts int32 = 4 MiB) until the process exits.  Each call clears the
// part it uses, so stale contents of the previous call do not matter -- but
// all calls on a device share the one array, so two calls whose work overlaps
// on the GPU (different streams, no ordering between them) race and both
// orders become wrong.  Nothing here calls cudaMalloc, cudaFree or any other
// allocating routine.
//
// In host code g_cell_counts names a host-side stand-in, not device memory, so
// it is never handed to a kernel directly: the first call on each device (with
// that device current) asks the runtime for the array's device address with
// cudaGetSymbolAddress and keeps it.  That first call should therefore come
// before any stream capture on that device.  The kept address belongs to the
// device's current context: after cudaDeviceReset (or anything else that
// destroys and recreates the primary context) it is stale, so this entry
// point must not be used on that device again in the same process.
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/cpab_b200.h"
#include "launch.h"

namespace {

constexpr int64_t kStaticCounts = int64_t(1) << 20;  // n_sets * nC must not exceed this

static __device__ __align__(256) int32_t g_cell_counts[kStaticCounts];

std::mutex g_mu;
int32_t *g_addr[64] = {};

// Device address of g_cell_counts on the current device (set up once per device).
cudaError_t static_counts(int32_t **out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_addr[dev] == nullptr) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_cell_counts);
    if (e != cudaSuccess) return e;
    g_addr[dev] = static_cast<int32_t *>(p);
  }
  *out = g_addr[dev];
  return cudaSuccess;
}

}  // namespace

extern "C" int cpab_b200_order_points_static(int ndim, const int32_t *nc, const float *points,
                                             int64_t nP, int n_sets, int32_t *order,
                                             cpab_stream_t stream) {
  // Sizes first (nothing touches the GPU before they pass); invalid shapes
  // (an axis outside [1, 2^20], as cpab_b200_order_points checks) leave nC at
  // 0 and are reported by cpab_b200_order_points itself below.  With every
  // axis at most 2^20, nC <= 5 * 2^60 fits int64; the limit is tested by
  // division so that n_sets * nC is never formed.
  int64_t nC = 0;
  if (ndim >= 1 && ndim <= 3 && nc != nullptr) {
    nC = ndim == 1 ? 1 : (ndim == 2 ? 4 : 5);
    for (int k = 0; k < ndim; ++k) {
      if (nc[k] < 1 || nc[k] > (1 << 20)) {
        nC = 0;
        break;
      }
      nC *= nc[k];
    }
  }
  if (nC > 0 && n_sets > 0 && nP > 0 && nC > kStaticCounts / n_sets)
    return cpab::report_error(CPAB_ERR_SIZE,
                              "order_points_static: n_sets (%d) * nC (%lld) exceeds the built-in "
                              "scratch of %lld counters; use cpab_b200_order_points",
                              n_sets, (long long)nC, (long long)kStaticCounts);
  int32_t *counts = nullptr;
  if (nC > 0 && n_sets > 0 && nP > 0) {
    const cudaError_t e = static_counts(&counts);
    if (e != cudaSuccess)
      return cpab::report_error(CPAB_ERR_CUDA, "order_points_static: cudaGetSymbolAddress: %s",
                                cudaGetErrorString(e));
  }
  return cpab_b200_order_points(ndim, nc, points, nP, n_sets, counts, order, stream);
}
