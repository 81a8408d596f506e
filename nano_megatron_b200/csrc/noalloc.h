// C entry point of the RMSNorm backward that allocates no memory.
//
// This entry point has no counterpart in the reference implementation; it is
// an addition for callers that cannot allocate device memory themselves: code
// that runs where cudaMalloc is forbidden or unsafe (a host callback, a
// process whose device memory belongs to another allocator, a real-time loop
// where an allocation could block or fail at an arbitrary moment).
//
// Rules for callers:
//  * Scratch: the weight-gradient partials live in one fixed device array of
//    nmb_rmsnorm_bwd_noalloc_scratch_floats() fp32 values per GPU, shared by
//    every call. Two calls whose kernels can overlap on the GPU (different
//    streams with no ordering between them) race on it and give wrong
//    results; order them on one stream or with events.
//  * Limits: cols must be a multiple of 8 and at most
//    nmb_rmsnorm_bwd_noalloc_max_cols() (8192), else NMB_NOALLOC_BAD_ARGUMENT;
//    rmsnorm_bwd_blocks(rows, 296) * cols (at most 296 * cols) must fit the array,
//    else NMB_NOALLOC_TOO_LARGE. Any row count fits for cols <= 4096.
//  * Set-up: call nmb_noalloc_prepare() once per device, with that device
//    current, before the region that must not allocate, and again after a
//    cudaDeviceReset. It looks up the array's device address and, under
//    CUDA_MODULE_LOADING=LAZY, makes the driver load this library's device
//    module (and place the array) on that device. Without it, the first call
//    of the entry point on a device does this set-up; that first call must
//    then come before any stream capture.
#pragma once

#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

// Return codes of nmb_rmsnorm_bwd_noalloc.
#define NMB_NOALLOC_OK 0
#define NMB_NOALLOC_TOO_LARGE 1      // rows/cols need more scratch than the fixed array holds
#define NMB_NOALLOC_BAD_ARGUMENT 2   // null pointer, non-positive size, cols % 8 != 0, cols > 8192, bad dtype
#define NMB_NOALLOC_SETUP_FAILED 3   // cudaGetSymbolAddress failed on this device
#define NMB_NOALLOC_LAUNCH_FAILED 4  // a kernel launch failed (see nmb_noalloc_last_cuda_error)

// Maximum number of fp32 scratch values: the fixed per-device array size.
long nmb_rmsnorm_bwd_noalloc_scratch_floats(void);

// Widest row (columns) the entry point accepts.
int nmb_rmsnorm_bwd_noalloc_max_cols(void);

// Per-device set-up (see the rules above); returns NMB_NOALLOC_OK or
// NMB_NOALLOC_SETUP_FAILED.
int nmb_noalloc_prepare(void);

// RMSNorm backward: dx = d(rmsnorm)/dx . dy, and dweight += sum over rows.
//   dy, x, dx : [rows][cols], dtype 1 = bf16, 0 = fp32
//   w         : [cols] fp32 norm weight; rstd : [rows] fp32 from the forward
//   dweight   : [cols] fp32, accumulated into (+=)
// Launches on `stream`; allocates nothing. On NMB_NOALLOC_LAUNCH_FAILED the
// CUDA error of the failed launch is returned by nmb_noalloc_last_cuda_error().
int nmb_rmsnorm_bwd_noalloc(const void* dy, const void* x, const float* w, const float* rstd, void* dx,
                            float* dweight, int rows, int cols, int dtype, cudaStream_t stream);

// cudaError_t value of the calling thread's last launch failure (0 if none).
int nmb_noalloc_last_cuda_error(void);

// Human-readable text of a return code.
const char* nmb_noalloc_error_string(int code);

#ifdef __cplusplus
}
#endif
