// Exact-fp32 kernels for the reference's fp32 training mode on CUDA
// (`--dtype float32`): a strided SIMT GEMM (fp32 FMA, no TF32) and the
// causal-softmax pieces of a materialized attention. They serve correctness
// (fp32 results within the oracle tests' 1e-4 tolerances), not speed; bf16 on
// the tensor-core kernels is the performance path. Reference ops: the fp32
// matmuls and SDPA of nano_megatron/model.py with compute_dtype "float32"
// (model.py:53-62).

#include <cuda_runtime.h>

#include <cfloat>
#include <cmath>

#include "fp32.cuh"

namespace nmb {

namespace {

constexpr int TM = 64, TN = 64, TK = 16;

// C[m, n] = beta * C[m, n] + sum_k A(m, k) * B(k, n) with element strides.
__global__ void __launch_bounds__(256)
gemm_f32_kernel(int M, int N, int K, const float* __restrict__ A, long sam, long sak, const float* __restrict__ B,
                long sbk, long sbn, float* __restrict__ C, long ldc, float beta) {
  __shared__ float As[TK][TM + 1];
  __shared__ float Bs[TK][TN + 1];
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int m0 = blockIdx.y * TM, n0 = blockIdx.x * TN;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += TK) {
    for (int i = threadIdx.x; i < TK * TM; i += 256) {
      const int kk = i / TM, mm = i % TM;
      const int m = m0 + mm, k = k0 + kk;
      As[kk][mm] = (m < M && k < K) ? A[m * sam + k * sak] : 0.f;
    }
    for (int i = threadIdx.x; i < TK * TN; i += 256) {
      const int kk = i / TN, nn = i % TN;
      const int n = n0 + nn, k = k0 + kk;
      Bs[kk][nn] = (n < N && k < K) ? B[k * sbk + n * sbn] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < TK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + ty * 4 + i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx * 4 + j;
      if (n < N) C[m * ldc + n] = beta == 0.f ? acc[i][j] : fmaf(beta, C[m * ldc + n], acc[i][j]);
    }
  }
}

// P = softmax(scale * S) over keys j <= i (row i); one block per row.
__global__ void causal_softmax_kernel(const float* __restrict__ S, float* __restrict__ P, int n, float scale) {
  const int row = blockIdx.x;
  const float* s = S + (long)row * n;
  float* p = P + (long)row * n;
  __shared__ float red[32];
  float mx = -FLT_MAX;
  for (int j = threadIdx.x; j <= row; j += blockDim.x) mx = fmaxf(mx, s[j] * scale);
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = mx;
  __syncthreads();
  mx = -FLT_MAX;
  for (int w = 0; w < (int)blockDim.x / 32; ++w) mx = fmaxf(mx, red[w]);
  __syncthreads();
  float sum = 0.f;
  for (int j = threadIdx.x; j <= row; j += blockDim.x) sum += expf(s[j] * scale - mx);
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = sum;
  __syncthreads();
  sum = 0.f;
  for (int w = 0; w < (int)blockDim.x / 32; ++w) sum += red[w];
  const float inv = 1.f / sum;
  for (int j = threadIdx.x; j < n; j += blockDim.x) p[j] = j <= row ? expf(s[j] * scale - mx) * inv : 0.f;
}

// dS = P * (dP - sum_j P dP) per row (softmax backward), times `scale`.
__global__ void softmax_bwd_kernel(const float* __restrict__ P, const float* __restrict__ dP, float* __restrict__ dS,
                                   int n, float scale) {
  const int row = blockIdx.x;
  const float* p = P + (long)row * n;
  const float* g = dP + (long)row * n;
  __shared__ float red[32];
  float dot = 0.f;
  for (int j = threadIdx.x; j < n; j += blockDim.x) dot += p[j] * g[j];
  for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = dot;
  __syncthreads();
  dot = 0.f;
  for (int w = 0; w < (int)blockDim.x / 32; ++w) dot += red[w];
  for (int j = threadIdx.x; j < n; j += blockDim.x) dS[(long)row * n + j] = p[j] * (g[j] - dot) * scale;
}

}  // namespace

cudaError_t gemm_f32(int M, int N, int K, const float* A, long sam, long sak, const float* B, long sbk, long sbn,
                     float* C, long ldc, float beta, cudaStream_t stream) {
  if (M <= 0 || N <= 0) return cudaSuccess;
  dim3 grid((N + TN - 1) / TN, (M + TM - 1) / TM);
  gemm_f32_kernel<<<grid, 256, 0, stream>>>(M, N, K, A, sam, sak, B, sbk, sbn, C, ldc, beta);
  return cudaGetLastError();
}

cudaError_t causal_softmax_f32(const float* S, float* P, int n, float scale, cudaStream_t stream) {
  causal_softmax_kernel<<<n, 256, 0, stream>>>(S, P, n, scale);
  return cudaGetLastError();
}

cudaError_t softmax_bwd_f32(const float* P, const float* dP, float* dS, int n, float scale, cudaStream_t stream) {
  softmax_bwd_kernel<<<n, 256, 0, stream>>>(P, dP, dS, n, scale);
  return cudaGetLastError();
}

}  // namespace nmb
