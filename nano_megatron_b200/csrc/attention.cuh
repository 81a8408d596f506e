// Host interface of the causal flash-attention kernels (attention.cu).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace nmb {

// qkv [S*batch, 3*heads*hd] -> out [S*batch, heads*hd], lse [batch*heads, S]
cudaError_t flash_attn_fwd(const __nv_bfloat16* qkv, __nv_bfloat16* out, float* lse, int S, int batch, int heads,
                           int head_dim, cudaStream_t stream);

// Same contract on tcgen05 tensor cores; S must be a multiple of 128.
cudaError_t flash_attn_fwd_tc(const __nv_bfloat16* qkv, __nv_bfloat16* out, float* lse, int S, int batch, int heads,
                              int head_dim, int* err, cudaStream_t stream);

// dqkv [S*batch, 3*heads*hd] (every element written); dvec [batch*heads*S] and
// dq_acc [batch*heads*S*hd] fp32 are scratch.
cudaError_t flash_attn_bwd(const __nv_bfloat16* dout, const __nv_bfloat16* qkv, const __nv_bfloat16* out,
                           const float* lse, float* dvec, float* dq_acc, __nv_bfloat16* dqkv, int S, int batch,
                           int heads, int head_dim, cudaStream_t stream);

// D[bh, s] = sum_d dO * O  (dvec [batch*heads*S])
cudaError_t flash_attn_bwd_dot(const __nv_bfloat16* dout, const __nv_bfloat16* out, float* dvec, int S, int batch,
                               int heads, cudaStream_t stream);

// tcgen05 backward (dK/dV kernel + dQ kernel, no atomics); dvec holds
// [2][batch*heads*S] floats: D from flash_attn_bwd_dot, then scratch for
// lse*log2(e); S must be a multiple of 128. With cosv/sinv ([S][head_dim/2]
// fp32) the inverse rotary embedding is applied to dQ and dK as they are
// stored; null leaves them unrotated.
cudaError_t flash_attn_bwd_tc(const __nv_bfloat16* dout, const __nv_bfloat16* qkv, const float* lse,
                              const float* dvec, __nv_bfloat16* dqkv, int S, int batch, int heads, int head_dim,
                              const float* cosv, const float* sinv, int* err, cudaStream_t stream);

}  // namespace nmb
