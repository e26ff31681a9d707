// Split-K W8A8 GEMM whose scratch is a fixed array inside this library, for
// callers that cannot allocate device memory.
//
// The split-K GEMM needs an int32 scratch of M x N partial sums plus arrival
// counters.  Some callers have no way to provide one: a plugin host whose
// enqueue call hands over no workspace pointer, a serving loop that froze its
// memory pool after warm-up and may not call cudaMalloc again, or a binding
// from another language with no device allocator of its own.  For them this
// file holds the scratch as a file-scope __device__ array of a fixed size
// (kStaticScratchBytes) and launches the same kernel as
// w8a8_gemm_dequant_splitk on it.  Nothing here allocates: no cudaMalloc,
// no cudaFree, no allocating library routine.
//
// Set-up: the first call on a device (with that device current) looks up the
// array's device address with cudaGetSymbolAddress and caches it per device;
// make that first call before any stream capture.  The cached address is not
// looked up again: after cudaDeviceReset in the host process it is stale, so
// a process that resets a device must not call this entry point again.
// Every call, from every thread and stream, shares the one array per device,
// so calls that overlap on the GPU race with each other.  Only calls whose
// GEMM splits use (and clear) the array; the others run without scratch.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "w8a8_internal.h"

static_assert(W8A8_SPLITK_STATIC_SCRATCH_BYTES % 256 == 0,
              "scratch size must keep 256-byte alignment");

// The scratch: int32 partial sums, then the arrival counters.
static __device__ __align__(256) uint8_t g_splitk_static_scratch[W8A8_SPLITK_STATIC_SCRATCH_BYTES];

namespace w8a8 {
namespace {

constexpr int64_t kStaticScratchBytes = W8A8_SPLITK_STATIC_SCRATCH_BYTES;

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of the array on the current device (looked up once per
// device).  Returns 0 or a W8A8_ERR_* code.
int static_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_error("cudaGetDevice failed: %s", cudaGetErrorString(e));
    return W8A8_ERR_ACCELERATOR;
  }
  if (dev < 0 || dev >= kMaxDevices) {
    set_error("device ordinal %d is beyond the %d devices the static scratch tracks", dev,
              kMaxDevices);
    return W8A8_ERR_INDEX;
  }
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (!g_scratch_ptr[dev]) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_splitk_static_scratch);
    if (e != cudaSuccess || !ptr) {
      set_error("cudaGetSymbolAddress of the static split-K scratch failed: %s",
                cudaGetErrorString(e));
      return W8A8_ERR_ACCELERATOR;
    }
    g_scratch_ptr[dev] = ptr;
  }
  *out = g_scratch_ptr[dev];
  return 0;
}

}  // namespace

int gemm_splitk_static_launch(GemmArgs g, cudaStream_t stream) {
  if (g.M == 0 || g.N == 0) return 0;
  // Plan first: a GEMM that does not split (split_k = 1, or a shape the
  // automatic policy runs whole) needs no scratch at all, whatever its size.
  GemmPlan plan{};
  if (int rc = plan_gemm(g, gemm_tc_ok(g), plan)) return rc;
  if (plan.splits <= 1) {
    g.split_k = 1;
    g.workspace = nullptr;
    g.workspace_bytes = 0;
    return gemm_launch(g, stream);
  }
  const int64_t need = plan.workspace_need;
  if (need > kStaticScratchBytes) {
    set_error("M=%lld x N=%lld split %d ways needs %lld bytes of split-K scratch; the static "
              "scratch holds %lld bytes (64 KiB per 128 x 128 output tile plus one counter per "
              "tile and epilogue warp)",
              static_cast<long long>(g.M), static_cast<long long>(g.N), plan.splits,
              static_cast<long long>(need), static_cast<long long>(kStaticScratchBytes));
    return W8A8_ERR_VALUE;
  }
  void* ptr = nullptr;
  if (int rc = static_scratch(&ptr)) return rc;
  // The partial sums and counters must start at zero.  A completed call
  // leaves them zero, but a call that gave up (device error) may not have,
  // so the part this call uses is cleared on its stream first.
  cudaError_t e = cudaMemsetAsync(ptr, 0, static_cast<size_t>(need), stream);
  if (e != cudaSuccess) {
    set_error("clearing the static split-K scratch failed: %s", cudaGetErrorString(e));
    return W8A8_ERR_ACCELERATOR;
  }
  g.workspace = ptr;
  g.workspace_bytes = kStaticScratchBytes;
  return gemm_launch(g, stream);
}

}  // namespace w8a8
