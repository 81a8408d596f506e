// Host interfaces of the memory-bound kernels (kernels.cu): RMSNorm, SwiGLU,
// RoPE, vocab-parallel embedding, cross-entropy statistics and gradient,
// AdamW over a flat buffer, weighted squared norm.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace nmb {

// dtype tags: 0 = fp32, 1 = bf16
cudaError_t rmsnorm_fwd(const void* x, const float* w, void* y, float* rstd, int rows, int cols, float eps,
                        int dtype, cudaStream_t s);
// Residual add fused with the norm that follows it: s = x + a (rounded to the
// dtype), y = rmsnorm(s) * w; cols <= 8192.
cudaError_t add_rmsnorm_fwd(const void* x, const void* a, void* s_out, const float* w, void* y, float* rstd,
                            int rows, int cols, float eps, int dtype, cudaStream_t s);
// Default cap on the blocks (and weight-gradient partial rows) of the backward:
// 2 per SM (4 per SM measured slower: twice the partial rows to reduce).
constexpr int kNormBwdMaxBlocks = 296;
// dx and per-block weight-gradient partials ([partial_rows, cols] fp32,
// partial_rows = rmsnorm_bwd_blocks(rows, max_blocks)); dx += dres when dres is given.
cudaError_t rmsnorm_bwd(const void* dy, const void* x, const float* w, const float* rstd, void* dx,
                        float* dw_partial, int rows, int cols, int dtype, cudaStream_t s, const void* dres = nullptr,
                        int max_blocks = kNormBwdMaxBlocks);
int rmsnorm_bwd_blocks(int rows, int max_blocks = kNormBwdMaxBlocks);
// out[c] += sum_b partial[b, c]
cudaError_t reduce_rows_add(const float* partial, float* out, int nrows, int cols, cudaStream_t s);

cudaError_t swiglu_fwd(const void* gu, void* a, long rows, int ffn, int dtype, cudaStream_t s);
cudaError_t swiglu_bwd(const void* da, const void* gu, void* dgu, long rows, int ffn, int dtype, cudaStream_t s);

// In-place NeoX rotation of the q and k sections of qkv [rows, 3*heads*hd];
// position = row / batch; sign = +1 forward, -1 inverse.
cudaError_t rope_inplace(void* qkv, const float* cos, const float* sin, long rows, int batch, int heads, int hd,
                         float sign, int dtype, cudaStream_t s);

cudaError_t embedding_fwd(const int64_t* ids, const float* w, void* out, long rows, int hidden, long vstart,
                          long vend, long vocab, int out_dtype, int* err, cudaStream_t s);
cudaError_t embedding_bwd(const void* dy, const int64_t* ids, float* wgrad, long rows, int hidden, long vstart,
                          long vend, int dtype, cudaStream_t s);

cudaError_t ce_stats(const void* logits, const int64_t* target, float* mx, float* se, float* tl, long rows, int vl,
                     long ld, long vstart, int dtype, cudaStream_t s);
cudaError_t ce_grad(const void* logits, const int64_t* target, const float* gmax, const float* gsum,
                    const float* gscale, float inv_n, void* dlogits, long rows, int vl, long ld, long vstart,
                    int dtype, cudaStream_t s);

cudaError_t adamw_flat(float* p, const float* g, float* m, float* v, __nv_bfloat16* compute, const float* scale,
                       long n, double lr, double beta1, double beta2, double eps, double wd, double bc1, double bc2_sqrt,
                       cudaStream_t s);

// out += sum_i weight[i] * ||seg_i||^2 (fp32 segments, fp64 result)
cudaError_t weighted_sq_norm(const int64_t* ptrs, const int64_t* numels, const double* weights, int nseg,
                             double* out, cudaStream_t s);

// Cycles of one tcgen05.mma (M=128, N = 64/128/256, A from TMEM when `ts`)
// in a chain of `iters` products on one SM: one CTA writes the chain's total
// cycles to out[0] (-1 if a wait ran out). tc_probe.cu.
cudaError_t tc_mma_cycles(int n, bool ts, int iters, long long* out, int* err, cudaStream_t stream);

}  // namespace nmb
