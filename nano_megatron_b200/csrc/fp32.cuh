// Host interface of the exact-fp32 kernels (fp32.cu).
#pragma once

#include <cuda_runtime.h>

namespace nmb {

// C[m, n] = beta * C[m, n] + sum_k A[m*sam + k*sak] * B[k*sbk + n*sbn]
cudaError_t gemm_f32(int M, int N, int K, const float* A, long sam, long sak, const float* B, long sbk, long sbn,
                     float* C, long ldc, float beta, cudaStream_t stream);
// P = causal softmax of scale * S, S and P [n][n]
cudaError_t causal_softmax_f32(const float* S, float* P, int n, float scale, cudaStream_t stream);
// dS = scale * P * (dP - rowsum(P * dP)), all [n][n]
cudaError_t softmax_bwd_f32(const float* P, const float* dP, float* dS, int n, float scale, cudaStream_t stream);

}  // namespace nmb
