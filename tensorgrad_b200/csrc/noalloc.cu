// Column sums of a device matrix without any allocation.
//
// Some callers cannot allocate device memory: a host that hands all of the
// GPU's memory to its own pool or caching allocator and forbids other
// allocations, or a latency-critical loop that must not call cudaMalloc
// because it can synchronize the whole device. They may still need the
// deterministic column-sum reduction that the training step uses for bias
// and LayerNorm-gain gradients. This entry point runs the same two-pass
// kernel with its partial sums in a fixed device array that lives as long as
// the library is loaded, so the caller supplies only the input and the output.
//
// The first call on each device looks up that array's device address with
// the device current (cudaGetSymbolAddress); make that first call before any
// stream capture. All calls share the one array, so calls that overlap on the
// GPU (different streams, or different host threads without ordering) race.
#include <cstdio>
#include <mutex>
#include <string>

#include "../../include/tensorgrad_b200.h"
#include "kernels.cuh"

namespace tg {
int api_fail(const std::string& name, const std::string& msg);
int api_ok();
}  // namespace tg

// Partial sums of one call: 256 Ki floats = 1 MiB, held by every GPU that
// loads the library until the process exits.
#define TG_NOALLOC_SCRATCH_FLOATS (256 * 1024)
static __device__ __align__(256) float g_noalloc_scratch[TG_NOALLOC_SCRATCH_FLOATS];

namespace {
std::mutex g_mu;
float* g_scratch_ptr[64] = {};  // device address of g_noalloc_scratch, per device

// The array's name is only a host-side stand-in; its device address has to
// be looked up with the owning device current, once per device.
cudaError_t scratch_for_current_device(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_ptr[dev];
  return cudaSuccess;
}
}  // namespace

extern "C" int tg_colsum_noalloc(const float* x, float* out, int64_t outer, int64_t inner, void* stream) {
  if (!x || !out) return tg::api_fail("Error", "tg_colsum_noalloc: null input or output pointer");
  if (outer < 0 || inner <= 0) return tg::api_fail("Error", "tg_colsum_noalloc: outer must be >= 0 and inner > 0");
  const size_t need = tg::colsum_scratch_floats(outer, inner);
  if (need > (size_t)TG_NOALLOC_SCRATCH_FLOATS)
    return tg::api_fail("Error", "tg_colsum_noalloc: [" + std::to_string(outer) + ", " + std::to_string(inner) +
                                     "] needs " + std::to_string(need) + " partial sums, more than the fixed " +
                                     std::to_string(TG_NOALLOC_SCRATCH_FLOATS) + "-float scratch array");
  float* scratch = nullptr;
  if (need > 0) {
    cudaError_t e = scratch_for_current_device(&scratch);
    if (e != cudaSuccess)
      return tg::api_fail("CudaError", std::string("tg_colsum_noalloc: scratch lookup: ") + cudaGetErrorString(e));
  }
  // An error left pending by earlier, unrelated work on this thread is
  // reported as such, so the check after the launch covers only this call.
  cudaError_t pending = cudaGetLastError();
  if (pending != cudaSuccess)
    return tg::api_fail("CudaError", std::string("tg_colsum_noalloc: error pending from earlier work, not launched: ") +
                                         cudaGetErrorString(pending));
  // Every partial sum is written before it is read, so nothing in the array
  // needs clearing between calls.
  tg::launch_colsum(x, out, outer, inner, scratch, reinterpret_cast<cudaStream_t>(stream));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return tg::api_fail("CudaError", std::string("tg_colsum_noalloc: ") + cudaGetErrorString(e));
  return tg::api_ok();
}
