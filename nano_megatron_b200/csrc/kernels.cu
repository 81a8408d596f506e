// Memory-bound kernels of the training step. Each one moves its tensors once,
// with 16-byte vector accesses; fp32 math throughout, bf16 or fp32 storage.
//
//   RMSNorm fwd/bwd   one warp per row; backward also reduces the weight
//                     gradient per block in registers (deterministic order)
//   SwiGLU fwd/bwd    silu(gate) * up on the fused [gate | up] GEMM output
//   RoPE              in-place NeoX rotation of the q and k sections of qkv
//   embedding         vocab-shard gather with device-side id bounds check;
//                     backward is a vectorized fp32 atomic scatter-add
//   CE stats / grad   per-token (max, sum exp, target logit) over one vocab
//                     shard; softmax - onehot with the loss scale
//   AdamW             one pass over the flat fp32 master buffer, applies the
//                     clip coefficient on load and rewrites the bf16 copy
//   sq-norm           weighted sum of squares of many segments into fp64
//
// Reference ops (nano_megatron/): RMSNorm model.py:73-75; SwiGLU
// model.py:151-152; RoPE model.py:84-89; embedding tp_layers.py:112-127; CE
// cross_entropy.py:18-65; AdamW train.py:85 (torch.optim.AdamW defaults);
// squared norm grads.py:166-183.

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cfloat>

#include "kernels.cuh"
#include "ptx.cuh"

namespace nmb {

namespace {

// ---------------------------------------------------------- 8-wide vectors
template <typename T>
struct V8;

template <>
struct V8<float> {
  __device__ static void load(const float* p, float (&v)[8]) {
    const float4 a = *reinterpret_cast<const float4*>(p);
    const float4 b = *reinterpret_cast<const float4*>(p + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
  __device__ static void store(float* p, const float (&v)[8]) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
  }
  __device__ static float round(float x) { return x; }
};

template <>
struct V8<__nv_bfloat16> {
  __device__ static void load(const __nv_bfloat16* p, float (&v)[8]) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    float2 f;
    f = unpack_bf16x2(u.x); v[0] = f.x; v[1] = f.y;
    f = unpack_bf16x2(u.y); v[2] = f.x; v[3] = f.y;
    f = unpack_bf16x2(u.z); v[4] = f.x; v[5] = f.y;
    f = unpack_bf16x2(u.w); v[6] = f.x; v[7] = f.y;
  }
  __device__ static void store(__nv_bfloat16* p, const float (&v)[8]) {
    uint4 u;
    u.x = pack_bf16x2(v[0], v[1]);
    u.y = pack_bf16x2(v[2], v[3]);
    u.z = pack_bf16x2(v[4], v[5]);
    u.w = pack_bf16x2(v[6], v[7]);
    *reinterpret_cast<uint4*>(p) = u;
  }
  __device__ static float round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
};

__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ------------------------------------------------------------------ RMSNorm
template <typename T>
__global__ void rmsnorm_fwd_kernel(const T* __restrict__ x, const float* __restrict__ w, T* __restrict__ y,
                                   float* __restrict__ rstd, int rows, int cols, float eps) {
  const int warps = blockDim.x / 32;
  const int lane = threadIdx.x % 32;
  for (long row = (long)blockIdx.x * warps + threadIdx.x / 32; row < rows; row += (long)gridDim.x * warps) {
    const T* xr = x + row * cols;
    float ss = 0.f;
    for (int c = lane * 8; c < cols; c += 256) {
      float v[8];
      V8<T>::load(xr + c, v);
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += v[i] * v[i];
    }
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / cols + eps);
    if (lane == 0) rstd[row] = r;
    T* yr = y + row * cols;
    for (int c = lane * 8; c < cols; c += 256) {
      float v[8], wv[8];
      V8<T>::load(xr + c, v);
      V8<float>::load(w + c, wv);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = V8<T>::round(v[i] * r) * V8<T>::round(wv[i]);
      V8<T>::store(yr + c, v);
    }
  }
}

// One block per row (rows in a grid-stride loop): thread t holds columns
// (t + 256 j) * 8 .. + 8 for j < CH in registers, so the row is read once.
// With ADD the block first forms the residual sum s = x + a (rounded to the
// activation type, as a separate add would) and writes it, then normalizes s:
// the add and the norm that follows it cost one pass. The per-warp sums of
// squares alternate between two shared slots, one barrier per row.
constexpr int NORM_FWD_THREADS = 256;

template <typename T, int CH, bool ADD>
__global__ void __launch_bounds__(NORM_FWD_THREADS)
rmsnorm_fwd_row_kernel(const T* __restrict__ x, const T* __restrict__ a, T* __restrict__ s_out,
                       const float* __restrict__ w, T* __restrict__ y, float* __restrict__ rstd, int rows,
                       int cols, float eps) {
  __shared__ float red[2][NORM_FWD_THREADS / 32];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  int parity = 0;
  for (long row = blockIdx.x; row < rows; row += gridDim.x, parity ^= 1) {
    float v[CH][8];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < CH; ++j) {
      const int c = (threadIdx.x + j * NORM_FWD_THREADS) * 8;
      if (c < cols) {
        V8<T>::load(x + row * cols + c, v[j]);
        if (ADD) {
          float av[8];
          V8<T>::load(a + row * cols + c, av);
#pragma unroll
          for (int i = 0; i < 8; ++i) v[j][i] = V8<T>::round(v[j][i] + av[i]);
          V8<T>::store(s_out + row * cols + c, v[j]);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) ss += v[j][i] * v[j][i];
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[j][i] = 0.f;
      }
    }
    ss = warp_sum(ss);
    if (lane == 0) red[parity][warp] = ss;
    __syncthreads();
    float total = 0.f;
#pragma unroll
    for (int i = 0; i < NORM_FWD_THREADS / 32; ++i) total += red[parity][i];
    const float r = rsqrtf(total / cols + eps);
    if (threadIdx.x == 0) rstd[row] = r;
#pragma unroll
    for (int j = 0; j < CH; ++j) {
      const int c = (threadIdx.x + j * NORM_FWD_THREADS) * 8;
      if (c < cols) {
        float wv[8];
        V8<float>::load(w + c, wv);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[j][i] = V8<T>::round(v[j][i] * r) * V8<T>::round(wv[i]);
        V8<T>::store(y + row * cols + c, v[j]);
      }
    }
  }
}

constexpr int NORM_BWD_THREADS = 256;

// One block works on one row at a time with all its threads: thread t owns
// columns (t + 256 j) * 8 .. + 8 for j < CH, so the weight gradient of those
// columns accumulates in the thread's registers over all the block's rows
// (written once at the end, no shared-memory reduction) and the row's
// x / dy stay in registers between the dot product and dx. One barrier per
// pair of rows: the per-warp dot partials alternate between two shared slots.
// RES: dx also receives dres, the gradient that reaches the normalized input
// through the residual stream (x feeds both the norm and the next residual
// add), so the two gradient paths are summed in this pass.
template <typename T, int CH, bool RES>
__global__ void __launch_bounds__(NORM_BWD_THREADS)
rmsnorm_bwd_kernel(const T* __restrict__ dy, const T* __restrict__ x, const float* __restrict__ w,
                   const float* __restrict__ rstd, const T* __restrict__ dres, T* __restrict__ dx,
                   float* __restrict__ dw_partial, int rows, int cols) {
  __shared__ float red[2][2 * (NORM_BWD_THREADS / 32)];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  float wv[CH][8], acc[CH][8];
#pragma unroll
  for (int j = 0; j < CH; ++j) {
    const int c = (threadIdx.x + j * NORM_BWD_THREADS) * 8;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      acc[j][i] = 0.f;
      wv[j][i] = 0.f;
    }
    if (c < cols) V8<float>::load(w + c, wv[j]);
  }
  // two rows per iteration (rows r and r + gridDim.x): twice the loads in flight
  int parity = 0;
  for (long row0 = blockIdx.x; row0 < rows; row0 += 2L * gridDim.x, parity ^= 1) {
    float xh[2][CH][8], gv[2][CH][8], r[2], dot[2];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const long row = row0 + q * (long)gridDim.x;
      const bool live = row < rows;
      r[q] = live ? rstd[row] : 0.f;
#pragma unroll
      for (int j = 0; j < CH; ++j) {
        const int c = (threadIdx.x + j * NORM_BWD_THREADS) * 8;
        if (live && c < cols) {
          V8<T>::load(x + row * cols + c, xh[q][j]);
          V8<T>::load(dy + row * cols + c, gv[q][j]);
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) xh[q][j][i] = gv[q][j][i] = 0.f;
        }
      }
    }
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      dot[q] = 0.f;
#pragma unroll
      for (int j = 0; j < CH; ++j)
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          xh[q][j][i] *= r[q];
          acc[j][i] += gv[q][j][i] * V8<T>::round(xh[q][j][i]);
          dot[q] += gv[q][j][i] * wv[j][i] * xh[q][j][i];
        }
      dot[q] = warp_sum(dot[q]);
    }
    if (lane == 0) {
      red[parity][warp] = dot[0];
      red[parity][NORM_BWD_THREADS / 32 + warp] = dot[1];
    }
    __syncthreads();
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      float d = 0.f;
#pragma unroll
      for (int i = 0; i < NORM_BWD_THREADS / 32; ++i) d += red[parity][q * (NORM_BWD_THREADS / 32) + i];
      d /= cols;
      const long row = row0 + q * (long)gridDim.x;
      if (row >= rows) continue;
#pragma unroll
      for (int j = 0; j < CH; ++j) {
        const int c = (threadIdx.x + j * NORM_BWD_THREADS) * 8;
        if (c < cols) {
          float o[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) o[i] = r[q] * (gv[q][j][i] * wv[j][i] - xh[q][j][i] * d);
          if (RES) {
            float rv[8];
            V8<T>::load(dres + row * cols + c, rv);
#pragma unroll
            for (int i = 0; i < 8; ++i) o[i] += rv[i];
          }
          V8<T>::store(dx + row * cols + c, o);
        }
      }
    }
  }
#pragma unroll
  for (int j = 0; j < CH; ++j) {
    const int c = (threadIdx.x + j * NORM_BWD_THREADS) * 8;
    if (c < cols) V8<float>::store(dw_partial + (long)blockIdx.x * cols + c, acc[j]);
  }
}

__global__ void reduce_rows_add_kernel(const float* __restrict__ partial, float* __restrict__ out, int nrows,
                                       int cols) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= cols) return;
  float s = 0.f;
  for (int r = 0; r < nrows; ++r) s += partial[(long)r * cols + c];
  out[c] += s;
}

// ------------------------------------------------------------------- SwiGLU
template <typename T>
__global__ void swiglu_fwd_kernel(const T* __restrict__ gu, T* __restrict__ a, long rows, int ffn) {
  const long chunks = rows * (ffn / 8);
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < chunks; i += (long)gridDim.x * blockDim.x) {
    const long row = i / (ffn / 8);
    const int c = (int)(i - row * (ffn / 8)) * 8;
    float g[8], u[8], o[8];
    V8<T>::load(gu + row * 2 * ffn + c, g);
    V8<T>::load(gu + row * 2 * ffn + ffn + c, u);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float s = g[k] / (1.f + __expf(-g[k]));
      o[k] = V8<T>::round(s) * u[k];
    }
    V8<T>::store(a + row * ffn + c, o);
  }
}

template <typename T>
__global__ void swiglu_bwd_kernel(const T* __restrict__ da, const T* __restrict__ gu, T* __restrict__ dgu, long rows,
                                  int ffn) {
  const long chunks = rows * (ffn / 8);
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < chunks; i += (long)gridDim.x * blockDim.x) {
    const long row = i / (ffn / 8);
    const int c = (int)(i - row * (ffn / 8)) * 8;
    float d[8], g[8], u[8], dg[8], du[8];
    V8<T>::load(da + row * ffn + c, d);
    V8<T>::load(gu + row * 2 * ffn + c, g);
    V8<T>::load(gu + row * 2 * ffn + ffn + c, u);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float sig = 1.f / (1.f + __expf(-g[k]));
      du[k] = d[k] * g[k] * sig;
      dg[k] = d[k] * u[k] * sig * (1.f + g[k] * (1.f - sig));
    }
    V8<T>::store(dgu + row * 2 * ffn + c, dg);
    V8<T>::store(dgu + row * 2 * ffn + ffn + c, du);
  }
}

// --------------------------------------------------------------------- RoPE
template <typename T>
__global__ void rope_kernel(T* __restrict__ qkv, const float* __restrict__ cosv, const float* __restrict__ sinv,
                            long rows, int batch, int heads, int hd, float sign) {
  const int half = hd / 2;
  const int per_head = half / 8;             // 8-element chunks of the first half
  const long per_row = 2L * heads * per_head;  // q and k heads
  const long total = rows * per_row;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const long row = i / per_row;
    const int r = (int)(i - row * per_row);
    const int head = r / per_head;  // 0..2*heads-1 covers q then k
    const int c = (r - head * per_head) * 8;
    const long pos = row / batch;
    T* base = qkv + row * (3L * heads * hd) + (long)head * hd;
    float x1[8], x2[8], cs[8], sn[8], o1[8], o2[8];
    V8<T>::load(base + c, x1);
    V8<T>::load(base + half + c, x2);
    V8<float>::load(cosv + pos * half + c, cs);
    V8<float>::load(sinv + pos * half + c, sn);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float s = sn[k] * sign;
      o1[k] = x1[k] * cs[k] - x2[k] * s;
      o2[k] = x2[k] * cs[k] + x1[k] * s;
    }
    V8<T>::store(base + c, o1);
    V8<T>::store(base + half + c, o2);
  }
}

// ---------------------------------------------------------------- embedding
template <typename T>
__global__ void embedding_fwd_kernel(const int64_t* __restrict__ ids, const float* __restrict__ w, T* __restrict__ out,
                                     long rows, int hidden, long vstart, long vend, long vocab, int* err) {
  const int warps = blockDim.x / 32, lane = threadIdx.x % 32;
  for (long row = (long)blockIdx.x * warps + threadIdx.x / 32; row < rows; row += (long)gridDim.x * warps) {
    const long id = ids[row];
    if ((id < 0 || id >= vocab) && lane == 0) report_error(err, kBadToken);
    const bool own = id >= vstart && id < vend;
    const float* src = w + (own ? (id - vstart) : 0) * (long)hidden;
    T* dst = out + row * hidden;
    for (int c = lane * 8; c < hidden; c += 256) {
      float v[8];
      if (own) {
        V8<float>::load(src + c, v);
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = 0.f;
      }
      V8<T>::store(dst + c, v);
    }
  }
}

template <typename T>
__global__ void embedding_bwd_kernel(const T* __restrict__ dy, const int64_t* __restrict__ ids, float* wgrad,
                                     long rows, int hidden, long vstart, long vend) {
  const int warps = blockDim.x / 32, lane = threadIdx.x % 32;
  for (long row = (long)blockIdx.x * warps + threadIdx.x / 32; row < rows; row += (long)gridDim.x * warps) {
    const long id = ids[row];
    if (id < vstart || id >= vend) continue;
    float* dst = wgrad + (id - vstart) * (long)hidden;
    for (int c = lane * 8; c < hidden; c += 256) {
      float v[8];
      V8<T>::load(dy + row * hidden + c, v);
      atomicAdd(reinterpret_cast<float4*>(dst + c), make_float4(v[0], v[1], v[2], v[3]));
      atomicAdd(reinterpret_cast<float4*>(dst + c + 4), make_float4(v[4], v[5], v[6], v[7]));
    }
  }
}

// ------------------------------------------------------------ cross entropy
__device__ __forceinline__ void merge_ms(float& m, float& s, float m2, float s2) {
  const float mn = fmaxf(m, m2);
  s = (m == -FLT_MAX ? 0.f : s * __expf(m - mn)) + (m2 == -FLT_MAX ? 0.f : s2 * __expf(m2 - mn));
  m = mn;
}

template <typename T>
__global__ void ce_stats_kernel(const T* __restrict__ logits, const int64_t* __restrict__ target, float* mx,
                                float* se, float* tl, int vl, long ld, long vstart) {
  const long row = blockIdx.x;
  const T* lr = logits + row * ld;
  float m = -FLT_MAX, s = 0.f;
  for (int c = threadIdx.x * 8; c < vl; c += blockDim.x * 8) {
    float v[8];
    V8<T>::load(lr + c, v);
    float cm = v[0];
#pragma unroll
    for (int k = 1; k < 8; ++k) cm = fmaxf(cm, v[k]);
    float cs = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) cs += __expf(v[k] - cm);
    merge_ms(m, s, cm, cs);
  }
  __shared__ float sm[32], ss[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    merge_ms(m, s, m2, s2);
  }
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (lane == 0) { sm[warp] = m; ss[warp] = s; }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x / 32;
    m = lane < nw ? sm[lane] : -FLT_MAX;
    s = lane < nw ? ss[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
      const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
      merge_ms(m, s, m2, s2);
    }
    if (lane == 0) {
      mx[row] = m;
      se[row] = s;
      const long t = target[row] - vstart;
      tl[row] = (t >= 0 && t < vl) ? to_f32(lr[t]) : 0.f;
    }
  }
}

template <typename T>
// `logits` and `dlogits` may be the same buffer (each element is read, then
// written, by the same thread).
__global__ void ce_grad_kernel(const T* logits, const int64_t* __restrict__ target,
                               const float* __restrict__ gmax, const float* __restrict__ gsum,
                               const float* __restrict__ gscale, float inv_n, T* dlogits, long rows,
                               int vl, long ld, long vstart) {
  const long row = blockIdx.y;
  const float m = gmax[row];
  const float inv_s = 1.f / gsum[row];
  const float scale = gscale[0] * inv_n;
  const long t = target[row] - vstart;
  const T* lr = logits + row * ld;
  T* dr = dlogits + row * (long)vl;
  for (int c = (blockIdx.x * blockDim.x + threadIdx.x) * 8; c < vl; c += gridDim.x * blockDim.x * 8) {
    float v[8];
    V8<T>::load(lr + c, v);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float p = __expf(v[k] - m) * inv_s;
      if (c + k == t) p -= 1.f;
      v[k] = p * scale;
    }
    V8<T>::store(dr + c, v);
  }
}

// -------------------------------------------------------------------- AdamW
__global__ void adamw_kernel(float4* __restrict__ p, const float4* __restrict__ g, float4* __restrict__ m,
                             float4* __restrict__ v, uint2* __restrict__ compute, const float* __restrict__ scale_ptr,
                             long n4, float one_minus_b1, float beta2, float one_minus_b2, float eps, float decay,
                             float step, float bc2_sqrt) {
  const float scale = scale_ptr[0];
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n4; i += (long)gridDim.x * blockDim.x) {
    float4 pp = p[i], gg = g[i], mm = m[i], vv = v[i];
    float* pf = &pp.x; float* gf = &gg.x; float* mf = &mm.x; float* vf = &vv.x;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float gk = gf[k] * scale;
      pf[k] *= decay;
      mf[k] += (gk - mf[k]) * one_minus_b1;
      vf[k] = vf[k] * beta2 + one_minus_b2 * gk * gk;
      const float denom = sqrtf(vf[k]) / bc2_sqrt + eps;
      pf[k] -= step * (mf[k] / denom);
    }
    p[i] = pp; m[i] = mm; v[i] = vv;
    if (compute != nullptr) compute[i] = make_uint2(pack_bf16x2(pp.x, pp.y), pack_bf16x2(pp.z, pp.w));
  }
}

// ------------------------------------------------------------ squared norm
__global__ void weighted_sq_norm_kernel(const int64_t* __restrict__ ptrs, const int64_t* __restrict__ numels,
                                        const double* __restrict__ weights, int nseg, double* out) {
  const int seg = blockIdx.y;
  if (seg >= nseg) return;
  const float* x = reinterpret_cast<const float*>(ptrs[seg]);
  const long n = numels[seg];
  float acc = 0.f;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const float v = x[i];
    acc += v * v;
  }
  double d = acc;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
  __shared__ double red[32];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (lane == 0) red[warp] = d;
  __syncthreads();
  if (threadIdx.x == 0) {
    double s = 0.0;
    for (int i = 0; i < (int)(blockDim.x / 32); ++i) s += red[i];
    atomicAdd(out, s * weights[seg]);
  }
}

int grid_for(long work, int threads, int cap = 148 * 16) {
  long g = (work + threads - 1) / threads;
  if (g < 1) g = 1;
  return (int)(g < cap ? g : cap);
}

}  // namespace

// ====================================================================== host
template <typename T, int CH, bool ADD>
static void launch_norm_fwd(const void* x, const void* a, void* s_out, const float* w, void* y, float* rstd, int rows,
                            int cols, float eps, cudaStream_t s) {
  const int grid = rows < 148 * 8 ? rows : 148 * 8;
  rmsnorm_fwd_row_kernel<T, CH, ADD><<<grid, NORM_FWD_THREADS, 0, s>>>(
      static_cast<const T*>(x), static_cast<const T*>(a), static_cast<T*>(s_out), w, static_cast<T*>(y), rstd, rows,
      cols, eps);
}

template <bool ADD>
static cudaError_t norm_fwd_rows(const void* x, const void* a, void* s_out, const float* w, void* y, float* rstd,
                                 int rows, int cols, float eps, int dtype, cudaStream_t s) {
  const int chunks = (cols + 8 * NORM_FWD_THREADS - 1) / (8 * NORM_FWD_THREADS);
#define NMB_NF(CH)                                                                                          \
  {                                                                                                         \
    if (dtype == 1) launch_norm_fwd<__nv_bfloat16, CH, ADD>(x, a, s_out, w, y, rstd, rows, cols, eps, s);  \
    else launch_norm_fwd<float, CH, ADD>(x, a, s_out, w, y, rstd, rows, cols, eps, s);                     \
    return cudaGetLastError();                                                                              \
  }
  if (chunks <= 1) NMB_NF(1)
  if (chunks <= 2) NMB_NF(2)
  if (chunks <= 4) NMB_NF(4)
#undef NMB_NF
  return cudaErrorInvalidValue;
}

cudaError_t add_rmsnorm_fwd(const void* x, const void* a, void* s_out, const float* w, void* y, float* rstd,
                            int rows, int cols, float eps, int dtype, cudaStream_t s) {
  if (cols % 8 || cols > 8 * NORM_FWD_THREADS * 4) return cudaErrorInvalidValue;
  if (rows <= 0) return cudaSuccess;
  return norm_fwd_rows<true>(x, a, s_out, w, y, rstd, rows, cols, eps, dtype, s);
}

cudaError_t rmsnorm_fwd(const void* x, const float* w, void* y, float* rstd, int rows, int cols, float eps, int dtype,
                        cudaStream_t s) {
  if (cols % 8) return cudaErrorInvalidValue;
  if (rows <= 0) return cudaSuccess;
  if (cols <= 8 * NORM_FWD_THREADS * 4)  // rows of up to 8192 columns: one block per row, row in registers
    return norm_fwd_rows<false>(x, nullptr, nullptr, w, y, rstd, rows, cols, eps, dtype, s);
  const int threads = 256, warps = threads / 32;
  const int grid = grid_for((long)rows * 32, threads, 148 * 32);
  (void)warps;
  if (dtype == 1)
    rmsnorm_fwd_kernel<__nv_bfloat16><<<grid, threads, 0, s>>>(static_cast<const __nv_bfloat16*>(x), w,
                                                               static_cast<__nv_bfloat16*>(y), rstd, rows, cols, eps);
  else
    rmsnorm_fwd_kernel<float><<<grid, threads, 0, s>>>(static_cast<const float*>(x), w, static_cast<float*>(y), rstd,
                                                       rows, cols, eps);
  return cudaGetLastError();
}

int rmsnorm_bwd_blocks(int rows, int max_blocks) {
  int b = (rows + 7) / 8;  // >= 8 rows per block (one row at a time)
  return b < max_blocks ? (b < 1 ? 1 : b) : max_blocks;
}

template <typename T, int C, bool RES>
static cudaError_t launch_norm_bwd(const void* dy, const void* x, const float* w, const float* rstd, const void* dres,
                                   void* dx, float* part, int rows, int cols, int blocks, cudaStream_t s) {
  rmsnorm_bwd_kernel<T, C, RES><<<blocks, NORM_BWD_THREADS, 0, s>>>(
      static_cast<const T*>(dy), static_cast<const T*>(x), w, rstd, static_cast<const T*>(dres), static_cast<T*>(dx),
      part, rows, cols);
  return cudaGetLastError();
}

cudaError_t rmsnorm_bwd(const void* dy, const void* x, const float* w, const float* rstd, void* dx, float* part,
                        int rows, int cols, int dtype, cudaStream_t s, const void* dres, int max_blocks) {
  if (cols % 8) return cudaErrorInvalidValue;
  const int chunks = (cols + 8 * NORM_BWD_THREADS - 1) / (8 * NORM_BWD_THREADS);  // 8-column chunks per thread
  if (chunks > 4) return cudaErrorInvalidValue;  // up to 8192 columns
  const int blocks = rmsnorm_bwd_blocks(rows, max_blocks);
#define NMB_NORM_RES(C, RES)                                                                                   \
  return dtype == 1 ? launch_norm_bwd<__nv_bfloat16, C, RES>(dy, x, w, rstd, dres, dx, part, rows, cols, blocks, s) \
                    : launch_norm_bwd<float, C, RES>(dy, x, w, rstd, dres, dx, part, rows, cols, blocks, s);
#define NMB_NORM(C)            \
  if (dres != nullptr) {       \
    NMB_NORM_RES(C, true)      \
  } else {                     \
    NMB_NORM_RES(C, false)     \
  }
  if (chunks <= 1) { NMB_NORM(1) }
  if (chunks <= 2) { NMB_NORM(2) }
  NMB_NORM(4)
#undef NMB_NORM
#undef NMB_NORM_RES
}

cudaError_t reduce_rows_add(const float* partial, float* out, int nrows, int cols, cudaStream_t s) {
  reduce_rows_add_kernel<<<(cols + 255) / 256, 256, 0, s>>>(partial, out, nrows, cols);
  return cudaGetLastError();
}

cudaError_t swiglu_fwd(const void* gu, void* a, long rows, int ffn, int dtype, cudaStream_t s) {
  if (ffn % 8) return cudaErrorInvalidValue;
  const int grid = grid_for(rows * (ffn / 8), 256);
  if (dtype == 1)
    swiglu_fwd_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(gu),
                                                          static_cast<__nv_bfloat16*>(a), rows, ffn);
  else
    swiglu_fwd_kernel<float><<<grid, 256, 0, s>>>(static_cast<const float*>(gu), static_cast<float*>(a), rows, ffn);
  return cudaGetLastError();
}

cudaError_t swiglu_bwd(const void* da, const void* gu, void* dgu, long rows, int ffn, int dtype, cudaStream_t s) {
  if (ffn % 8) return cudaErrorInvalidValue;
  const int grid = grid_for(rows * (ffn / 8), 256);
  if (dtype == 1)
    swiglu_bwd_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(da),
                                                          static_cast<const __nv_bfloat16*>(gu),
                                                          static_cast<__nv_bfloat16*>(dgu), rows, ffn);
  else
    swiglu_bwd_kernel<float><<<grid, 256, 0, s>>>(static_cast<const float*>(da), static_cast<const float*>(gu),
                                                  static_cast<float*>(dgu), rows, ffn);
  return cudaGetLastError();
}

cudaError_t rope_inplace(void* qkv, const float* cosv, const float* sinv, long rows, int batch, int heads, int hd,
                         float sign, int dtype, cudaStream_t s) {
  if (hd % 16) return cudaErrorInvalidValue;
  const int grid = grid_for(rows * 2L * heads * (hd / 16), 256);
  if (dtype == 1)
    rope_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(static_cast<__nv_bfloat16*>(qkv), cosv, sinv, rows, batch, heads,
                                                    hd, sign);
  else
    rope_kernel<float><<<grid, 256, 0, s>>>(static_cast<float*>(qkv), cosv, sinv, rows, batch, heads, hd, sign);
  return cudaGetLastError();
}

cudaError_t embedding_fwd(const int64_t* ids, const float* w, void* out, long rows, int hidden, long vstart, long vend,
                          long vocab, int out_dtype, int* err, cudaStream_t s) {
  if (hidden % 8) return cudaErrorInvalidValue;
  const int grid = grid_for(rows * 32, 256);
  if (out_dtype == 1)
    embedding_fwd_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(ids, w, static_cast<__nv_bfloat16*>(out), rows, hidden,
                                                             vstart, vend, vocab, err);
  else
    embedding_fwd_kernel<float><<<grid, 256, 0, s>>>(ids, w, static_cast<float*>(out), rows, hidden, vstart, vend,
                                                     vocab, err);
  return cudaGetLastError();
}

cudaError_t embedding_bwd(const void* dy, const int64_t* ids, float* wgrad, long rows, int hidden, long vstart,
                          long vend, int dtype, cudaStream_t s) {
  if (hidden % 8) return cudaErrorInvalidValue;
  const int grid = grid_for(rows * 32, 256);
  if (dtype == 1)
    embedding_bwd_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(dy), ids, wgrad, rows,
                                                             hidden, vstart, vend);
  else
    embedding_bwd_kernel<float><<<grid, 256, 0, s>>>(static_cast<const float*>(dy), ids, wgrad, rows, hidden, vstart,
                                                     vend);
  return cudaGetLastError();
}

cudaError_t ce_stats(const void* logits, const int64_t* target, float* mx, float* se, float* tl, long rows, int vl,
                     long ld, long vstart, int dtype, cudaStream_t s) {
  if (vl % 8 || ld % 8) return cudaErrorInvalidValue;
  if (dtype == 1)
    ce_stats_kernel<__nv_bfloat16><<<rows, 512, 0, s>>>(static_cast<const __nv_bfloat16*>(logits), target, mx, se, tl,
                                                        vl, ld, vstart);
  else
    ce_stats_kernel<float><<<rows, 512, 0, s>>>(static_cast<const float*>(logits), target, mx, se, tl, vl, ld, vstart);
  return cudaGetLastError();
}

cudaError_t ce_grad(const void* logits, const int64_t* target, const float* gmax, const float* gsum,
                    const float* gscale, float inv_n, void* dlogits, long rows, int vl, long ld, long vstart,
                    int dtype, cudaStream_t s) {
  if (vl % 8 || ld % 8 || rows > 65535L) return cudaErrorInvalidValue;
  const int bx = (vl / 8 + 255) / 256;
  dim3 grid(bx < 8 ? bx : 8, (unsigned)rows);
  if (dtype == 1)
    ce_grad_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(logits), target, gmax, gsum,
                                                       gscale, inv_n, static_cast<__nv_bfloat16*>(dlogits), rows, vl,
                                                       ld, vstart);
  else
    ce_grad_kernel<float><<<grid, 256, 0, s>>>(static_cast<const float*>(logits), target, gmax, gsum, gscale, inv_n,
                                               static_cast<float*>(dlogits), rows, vl, ld, vstart);
  return cudaGetLastError();
}

cudaError_t adamw_flat(float* p, const float* g, float* m, float* v, __nv_bfloat16* compute, const float* scale, long n,
                       double lr, double beta1, double beta2, double eps, double wd, double bc1, double bc2_sqrt,
                       cudaStream_t s) {
  if (n % 4) return cudaErrorInvalidValue;
  const long n4 = n / 4;
  adamw_kernel<<<grid_for(n4, 256, 148 * 8), 256, 0, s>>>(
      reinterpret_cast<float4*>(p), reinterpret_cast<const float4*>(g), reinterpret_cast<float4*>(m),
      reinterpret_cast<float4*>(v), reinterpret_cast<uint2*>(compute), scale, n4, (float)(1.0 - beta1), (float)beta2,
      (float)(1.0 - beta2), (float)eps, (float)(1.0 - lr * wd), (float)(lr / bc1), (float)bc2_sqrt);
  return cudaGetLastError();
}

cudaError_t weighted_sq_norm(const int64_t* ptrs, const int64_t* numels, const double* weights, int nseg, double* out,
                             cudaStream_t s) {
  if (nseg <= 0) return cudaSuccess;
  dim3 grid(16, nseg);
  weighted_sq_norm_kernel<<<grid, 512, 0, s>>>(ptrs, numels, weights, nseg, out);
  return cudaGetLastError();
}

}  // namespace nmb
