// RMSNorm backward without any memory allocation, for callers that cannot
// allocate: code that runs where cudaMalloc is forbidden or unsafe, such as
// inside a host callback, in a process whose device memory is owned by
// another allocator that must not be bypassed, or in a real-time loop where
// an allocation could block or fail at an arbitrary moment.
//
// The regular entry point (rmsnorm_bwd in kernels.cu, used by the framework)
// takes a caller-provided fp32 buffer for the per-block weight-gradient
// partials. This variant keeps those partials in a fixed array in device
// global memory instead, defined below at file scope. Properties:
//
//  * Size limits: the kernel handles up to kMaxCols (8192) columns; wider rows
//    are rejected with NMB_NOALLOC_BAD_ARGUMENT. The array holds
//    kScratchFloats fp32 values (4.6 MiB). A call needs
//    rmsnorm_bwd_blocks(rows, 296) * cols of them (at most 296 * cols), so every
//    `rows` works for cols <= 4096; larger requests are rejected with
//    NMB_NOALLOC_TOO_LARGE before anything is launched.
//  * The array lives in this library's device module. With eager module
//    loading every GPU the library is loaded on holds it until the process
//    exits; with CUDA_MODULE_LOADING=LAZY (the default of recent CUDA
//    runtimes) the driver places it on a device when the module is first used
//    there, which can be the set-up below.
//  * Set-up: the array's name in host code is only a host-side stand-in, not a
//    device address. nmb_noalloc_prepare() (with the device current) looks up
//    the device address with cudaGetSymbolAddress, which also loads the module
//    on that device, and caches it. Call it once per device before the region
//    that must not allocate, and again after cudaDeviceReset (the cached
//    address belongs to the old context). If it was not called, the first
//    call of the entry point on a device does it; make that first call before
//    any stream capture.
//  * All calls share the array, and a call leaves its partials in it. The
//    kernel writes every partial it later reads, so nothing needs clearing,
//    but two calls whose kernels overlap on the GPU (different streams
//    without ordering) race on the array and give wrong results.
//  * No cudaMalloc, cudaFree or allocating library routine is called.

#include <cuda_runtime.h>

#include <mutex>

#include "kernels.cuh"
#include "noalloc.h"

namespace {

constexpr int kPartialRows = 296;  // cap on the backward's blocks, i.e. on the partial rows
constexpr long kScratchFloats = (long)kPartialRows * 4096L;
constexpr int kMaxCols = 8192;  // 256 threads x 8 columns x 4 chunks in rmsnorm_bwd_kernel
constexpr int kMaxDevices = 64;

static __device__ __align__(256) float g_norm_partials[kScratchFloats];

float* g_scratch_ptr[kMaxDevices] = {nullptr};
thread_local int g_last_cuda_error = 0;  // cudaError_t of this thread's last failed launch
std::mutex g_setup_mutex;

float* scratch_for_current_device(int* code, bool refresh) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    *code = NMB_NOALLOC_SETUP_FAILED;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_scratch_ptr[dev] == nullptr || refresh) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_norm_partials) != cudaSuccess || p == nullptr) {
      *code = NMB_NOALLOC_SETUP_FAILED;
      return nullptr;
    }
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  return g_scratch_ptr[dev];
}

}  // namespace

extern "C" long nmb_rmsnorm_bwd_noalloc_scratch_floats(void) { return kScratchFloats; }

extern "C" int nmb_rmsnorm_bwd_noalloc_max_cols(void) { return kMaxCols; }

extern "C" int nmb_noalloc_prepare(void) {
  int code = NMB_NOALLOC_OK;
  return scratch_for_current_device(&code, /*refresh=*/true) != nullptr ? NMB_NOALLOC_OK : code;
}

extern "C" int nmb_rmsnorm_bwd_noalloc(const void* dy, const void* x, const float* w, const float* rstd, void* dx,
                                       float* dweight, int rows, int cols, int dtype, cudaStream_t stream) {
  if (!dy || !x || !w || !rstd || !dx || !dweight || rows <= 0 || cols <= 0 || cols % 8 != 0 ||
      cols > kMaxCols || (dtype != 0 && dtype != 1))
    return NMB_NOALLOC_BAD_ARGUMENT;
  const int blocks = nmb::rmsnorm_bwd_blocks(rows, kPartialRows);
  if ((long)blocks * cols > kScratchFloats) return NMB_NOALLOC_TOO_LARGE;
  int code = NMB_NOALLOC_OK;
  float* partials = scratch_for_current_device(&code, /*refresh=*/false);
  if (partials == nullptr) return code;
  cudaError_t err = nmb::rmsnorm_bwd(dy, x, w, rstd, dx, partials, rows, cols, dtype, stream, nullptr, kPartialRows);
  if (err == cudaSuccess) err = nmb::reduce_rows_add(partials, dweight, blocks, cols, stream);
  if (err != cudaSuccess) {
    g_last_cuda_error = static_cast<int>(err);
    return NMB_NOALLOC_LAUNCH_FAILED;
  }
  return NMB_NOALLOC_OK;
}

extern "C" int nmb_noalloc_last_cuda_error(void) { return g_last_cuda_error; }

extern "C" const char* nmb_noalloc_error_string(int code) {
  switch (code) {
    case NMB_NOALLOC_OK: return "ok";
    case NMB_NOALLOC_TOO_LARGE: return "rows/cols need more scratch than the fixed 296*4096-float array holds";
    case NMB_NOALLOC_BAD_ARGUMENT:
      return "null pointer, non-positive size, cols not a multiple of 8 or above 8192, or bad dtype";
    case NMB_NOALLOC_SETUP_FAILED: return "could not obtain the scratch array's device address on this device";
    case NMB_NOALLOC_LAUNCH_FAILED: return "a kernel launch failed";
    default: return "unknown code";
  }
}
