// Host interface of the tcgen05 GEMM (gemm.cu).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace nmb {

// kSwiGLU: B is the fused gate|up weight [K][2F] (N-major, N = 2F); C = a =
// silu(X W_gate) * (X W_up) as bf16 [M][F]; optionally also the bf16
// pre-activation gu [M][2F] (gate | up halves) for the backward.
enum class OutMode : int { kBf16 = 0, kF32 = 1, kF32Accumulate = 2, kSwiGLU = 3 };

struct GemmArgs {
  const void* A;   // bf16; [M][lda] if !a_mn (K-major), [K][lda] if a_mn (M-major)
  const void* B;   // bf16; [N][ldb] if !b_mn (K-major), [K][ldb] if b_mn (N-major)
  void* C;         // [M][ldc], bf16 or fp32 per `out`
  long lda, ldb, ldc;  // row strides in elements
  int M, N, K;
  bool a_mn, b_mn;
  OutMode out;
  int* err;        // device error word (may be null)
  int num_sms;
  void* gu = nullptr;  // kSwiGLU only: [M][ldgu] bf16 pre-activation output, or null
  long ldgu = 0;
};

cudaError_t gemm_bf16(const GemmArgs& args, cudaStream_t stream);

// 2-D bf16 TMA descriptor with 128-byte swizzle; `inner` is the contiguous dim.
bool make_tmap_bf16_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_elems,
                       uint32_t box_inner, uint32_t box_outer);

// 2-D TMA descriptor of an output matrix [outer][inner] (row stride in bytes)
// for 128-byte-swizzled stores / reduce-adds: fp32 (box 32 x box_outer) or
// bf16 (box 64 x box_outer).
bool make_tmap_out_2d(CUtensorMap* map, const void* base, bool fp32, uint64_t inner, uint64_t outer,
                      uint64_t row_stride_bytes, uint32_t box_outer);

// 3-D bf16 TMA descriptor with 128-byte swizzle; dims[0] is contiguous, strides
// (bytes) of dims 1 and 2 must be multiples of 16.
bool make_tmap_bf16_3d(CUtensorMap* map, const void* base, const uint64_t dims[3], const uint64_t strides_bytes[2],
                       const uint32_t box[3]);

}  // namespace nmb
