// C entry point of the RMSNorm backward that allocates no memory.
//
// This entry point has no counterpart in the reference implementation; it is
// an addition for callers that cannot allocate device memory themselves.
#pragma once

#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

// Return codes of nmb_rmsnorm_bwd_noalloc.
#define NMB_NOALLOC_OK 0
#define NMB_NOALLOC_TOO_LARGE 1      // rows/cols need more scratch than the fixed array holds
#define NMB_NOALLOC_BAD_ARGUMENT 2   // null pointer, non-positive size, cols % 8 != 0, bad dtype
#define NMB_NOALLOC_SETUP_FAILED 3   // cudaGetSymbolAddress failed on this device
#define NMB_NOALLOC_LAUNCH_FAILED 4  // a kernel launch failed (see cudaGetLastError)

// Maximum number of fp32 scratch values: the fixed per-device array size.
long nmb_rmsnorm_bwd_noalloc_scratch_floats(void);

// RMSNorm backward: dx = d(rmsnorm)/dx . dy, and dweight += sum over rows.
//   dy, x, dx : [rows][cols], dtype 1 = bf16, 0 = fp32
//   w         : [cols] fp32 norm weight; rstd : [rows] fp32 from the forward
//   dweight   : [cols] fp32, accumulated into (+=)
// Launches on `stream`; allocates nothing (see noalloc.cu for the rules).
int nmb_rmsnorm_bwd_noalloc(const void* dy, const void* x, const float* w, const float* rstd, void* dx,
                            float* dweight, int rows, int cols, int dtype, cudaStream_t stream);

// Human-readable text of a return code.
const char* nmb_noalloc_error_string(int code);

#ifdef __cplusplus
}
#endif
