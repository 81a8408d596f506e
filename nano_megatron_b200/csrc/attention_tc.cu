// Causal flash-attention forward on 5th-generation tensor cores (sm_100a),
// head_dim 128, bf16 in / out, fp32 softmax and accumulation.
//
// One CTA computes 128 query rows of one (batch, head); 6 warps:
//   warp 0     TMA loads: Q once, then K_j and V_j (128 keys each) into a
//              2-stage ring; all boxes come straight out of the fused QKV
//              buffer through one 3-D tensor map (cols, batch, position).
//   warp 1     MMA issue: S_j = Q K_j^T into one of two TMEM S buffers
//              (128 x 128 fp32), then O += P_{j-1} V_{j-1} into the TMEM O
//              accumulator once the softmax warps have published P_{j-1}.
//   warps 2-5  softmax, one query row per thread (TMEM lane = row):
//              tcgen05.ld the S row, online max / exp2 / row sum in fp32,
//              rescale the O row in TMEM only when a row maximum grew (warp
//              vote), write P (bf16) into 128-byte-swizzled shared memory as
//              the A operand of the next MMA, and finally normalize O and
//              write the output row and the log-sum-exp.
// S_{j+1} is computed while the softmax warps work on S_j; the PV product of
// block j overlaps the softmax of block j+1.
//
// TMEM: S0 columns [0,128), S1 [128,256), O [256,384) of a 512-column
// allocation. Shared memory: Q 32 KB, K 2x32 KB, V 2x32 KB, P 32 KB.
// Every mbarrier wait is bounded (error word + abort, never a trap).
//
// Output contract is the same as the mma.sync kernel of attention.cu (o and
// lse layouts), so the backward kernel consumes either.

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cmath>

#include "attention.cuh"
#include "gemm.cuh"
#include "ptx.cuh"

namespace nmb {

namespace {

constexpr int HD = 128, TQ = 128, TK = 128;
constexpr int HALF = TQ * 64 * 2;   // 16 KB: 128 rows x 64 bf16 (one swizzle atom column)
constexpr int TILE = 2 * HALF;      // 32 KB
constexpr int OFF_Q = 0, OFF_K = TILE, OFF_V = 3 * TILE, OFF_P = 5 * TILE, OFF_BAR = 6 * TILE;
constexpr int SMEM = 6 * TILE + 256 + 1024;
constexpr int THREADS = 192;

__device__ __forceinline__ uint64_t kmajor_desc(uint32_t base, int kk) { return nmb::kmajor_desc(base, kk, HALF); }

__global__ void __launch_bounds__(THREADS, 1)
flash_fwd_tc_kernel(const __grid_constant__ CUtensorMap tm_qkv, __nv_bfloat16* __restrict__ out,
                    float* __restrict__ lse, int S, int batch, int heads, float scale_log2, int* err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;    // [2]
  uint64_t* v_full = bars + 3;    // [2]
  uint64_t* kv_empty = bars + 5;  // [2]
  uint64_t* s_full = bars + 7;    // [2]
  uint64_t* s_free = bars + 9;    // [2]
  uint64_t* p_full = bars + 11;
  uint64_t* pv_done = bars + 12;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 13);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int nqb = S / TQ;
  const int qb = nqb - 1 - blockIdx.x;  // longest rows first
  const int bh = blockIdx.y, b = bh / heads, h = bh % heads;
  const int nkb = qb + 1;
  const int q_col = h * HD, k_col = heads * HD + h * HD, v_col = 2 * heads * HD + h * HD;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 128);
    }
    mbar_init(p_full, 128);
    mbar_init(pv_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t sbase = smem_u32(smem);

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------------ loads
    tma_prefetch_desc(&tm_qkv);
    int issued[2] = {-1, -1};
    mbar_arrive_expect_tx(q_full, TILE);
    tma_load_3d(smem + OFF_Q, &tm_qkv, q_full, q_col, b, qb * TQ);
    tma_load_3d(smem + OFF_Q + HALF, &tm_qkv, q_full, q_col + 64, b, qb * TQ);
    for (int j = 0; j < nkb; ++j) {
      const int st = j & 1;
      if (!lane_wait(&kv_empty[st], ((j >> 1) & 1) ^ 1, err, abort_flag)) break;
      uint8_t* kd = smem + OFF_K + st * TILE;
      uint8_t* vd = smem + OFF_V + st * TILE;
      mbar_arrive_expect_tx(&k_full[st], TILE);
      tma_load_3d(kd, &tm_qkv, &k_full[st], k_col, b, j * TK);
      tma_load_3d(kd + HALF, &tm_qkv, &k_full[st], k_col + 64, b, j * TK);
      mbar_arrive_expect_tx(&v_full[st], TILE);
      tma_load_3d(vd, &tm_qkv, &v_full[st], v_col, b, j * TK);
      tma_load_3d(vd + HALF, &tm_qkv, &v_full[st], v_col + 64, b, j * TK);
      issued[st] = (j >> 1) & 1;
    }
    // no copy may still be in flight at exit (matters only after an abort)
    mbar_wait(q_full, 0, nullptr, 1000000000ull);
    for (int st = 0; st < 2; ++st)
      if (issued[st] >= 0) {
        mbar_wait(&k_full[st], issued[st], nullptr, 1000000000ull);
        mbar_wait(&v_full[st], issued[st], nullptr, 1000000000ull);
      }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------------- MMA
    constexpr uint32_t idesc_s = idesc_bf16_f32(TQ, TK, false, false);
    constexpr uint32_t idesc_o = idesc_bf16_f32(TQ, HD, false, true);
    bool ok = lane_wait(q_full, 0, err, abort_flag);
    for (int j = 0; ok && j <= nkb; ++j) {
      if (j < nkb) {
        const int st = j & 1;
        if (!lane_wait(&k_full[st], (j >> 1) & 1, err, abort_flag)) break;
        if (!lane_wait(&s_free[st], ((j >> 1) & 1) ^ 1, err, abort_flag)) break;
        tc_fence_after();
        const uint32_t kb = sbase + OFF_K + st * TILE;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk)
          mma_bf16_ss(tmem + st * TK, kmajor_desc(sbase + OFF_Q, kk), kmajor_desc(kb, kk), idesc_s, kk > 0);
        mma_commit(&s_full[st]);
      }
      if (j >= 1) {
        const int i = j - 1, st = i & 1;
        if (!lane_wait(p_full, i & 1, err, abort_flag)) break;
        if (!lane_wait(&v_full[st], (i >> 1) & 1, err, abort_flag)) break;
        tc_fence_after();
        const uint32_t vb = sbase + OFF_V + st * TILE;
#pragma unroll
        for (int kk = 0; kk < TK / 16; ++kk)
          mma_bf16_ss(tmem + 256, kmajor_desc(sbase + OFF_P, kk), smem_desc_sw128(vb + kk * 2048, HALF, 1024),
                      idesc_o, (i > 0 || kk > 0));
        mma_commit(pv_done);
        mma_commit(&kv_empty[st]);
      }
    }
  } else if (warp >= 2) {
    // --------------------------------------------------------------- softmax
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // query row within the tile
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const int q = qb * TQ + r;
    float m = -INFINITY, l = 0.f;
    uint8_t* prow = smem + OFF_P + r * 128;
    bool ok = true;
    for (int j = 0; j < nkb && ok; ++j) {
      const int sb = j & 1;
      ok = warp_wait(&s_full[sb], (j >> 1) & 1, err, abort_flag);
      if (!ok) break;
      tc_fence_after();
      float s[TK];
#pragma unroll
      for (int c = 0; c < TK; c += 32) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tmem + lane_off + sb * TK + c, v);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) s[c + i] = __uint_as_float(v[i]);
      }
      tc_fence_before();
      mbar_arrive(&s_free[sb]);
      if (j == nkb - 1) {  // diagonal block: key index c > row r is in the future
#pragma unroll
        for (int c = 0; c < TK; ++c)
          if (c > r) s[c] = -INFINITY;
      }
      float mx0 = s[0], mx1 = s[1];
#pragma unroll
      for (int c = 2; c < TK; c += 2) {
        mx0 = fmaxf(mx0, s[c]);
        mx1 = fmaxf(mx1, s[c + 1]);
      }
      const float m_new = fmaxf(m, fmaxf(mx0, mx1));
      const float alpha = fast_exp2((m - m_new) * scale_log2);
      const float ms = m_new * scale_log2;
      float sum0 = 0.f, sum1 = 0.f;
#pragma unroll
      for (int c = 0; c < TK; c += 2) {
        s[c] = fast_exp2(fmaf(s[c], scale_log2, -ms));
        s[c + 1] = fast_exp2(fmaf(s[c + 1], scale_log2, -ms));
        sum0 += s[c];
        sum1 += s[c + 1];
      }
      const float sum = sum0 + sum1;
      l = l * alpha + sum;
      m = m_new;
      if (j > 0) {
        ok = warp_wait(pv_done, (j - 1) & 1, err, abort_flag);
        if (!ok) break;
        tc_fence_after();
        if (__any_sync(0xffffffffu, alpha < 1.f)) {
#pragma unroll
          for (int c = 0; c < HD; c += 32) {
            uint32_t v[32];
            tmem_ld_32x32b_x32(tmem + lane_off + 256 + c, v);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * alpha);
            tmem_st_32x32b_x32(tmem + lane_off + 256 + c, v);
          }
          tmem_wait_st();
        }
      }
      // P row -> shared memory, K-major 128-byte-swizzled layout
#pragma unroll
      for (int ch = 0; ch < TK / 8; ++ch) {
        uint4 u;
        u.x = pack_bf16x2(s[8 * ch + 0], s[8 * ch + 1]);
        u.y = pack_bf16x2(s[8 * ch + 2], s[8 * ch + 3]);
        u.z = pack_bf16x2(s[8 * ch + 4], s[8 * ch + 5]);
        u.w = pack_bf16x2(s[8 * ch + 6], s[8 * ch + 7]);
        *reinterpret_cast<uint4*>(prow + (ch >> 3) * HALF + (((ch & 7) ^ (r & 7)) << 4)) = u;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    if (ok) ok = warp_wait(pv_done, (nkb - 1) & 1, err, abort_flag);
    tc_fence_after();
    const float inv = 1.f / l;
    __nv_bfloat16* orow = out + ((long)q * batch + b) * heads * HD + h * HD;
#pragma unroll
    for (int c = 0; c < HD; c += 32) {
      uint32_t v[32];
      tmem_ld_32x32b_x32(tmem + lane_off + 256 + c, v);
      tmem_wait_ld();
      if (ok) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          uint4 u;
          u.x = pack_bf16x2(__uint_as_float(v[8 * k + 0]) * inv, __uint_as_float(v[8 * k + 1]) * inv);
          u.y = pack_bf16x2(__uint_as_float(v[8 * k + 2]) * inv, __uint_as_float(v[8 * k + 3]) * inv);
          u.z = pack_bf16x2(__uint_as_float(v[8 * k + 4]) * inv, __uint_as_float(v[8 * k + 5]) * inv);
          u.w = pack_bf16x2(__uint_as_float(v[8 * k + 6]) * inv, __uint_as_float(v[8 * k + 7]) * inv);
          *reinterpret_cast<uint4*>(orow + c + 8 * k) = u;
        }
      }
    }
    if (ok) lse[(long)bh * S + q] = (m * scale_log2 + log2f(l)) * 0.6931471805599453f;
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

cudaError_t flash_attn_fwd_tc(const __nv_bfloat16* qkv, __nv_bfloat16* out, float* lse, int S, int batch, int heads,
                              int head_dim, int* err, cudaStream_t stream) {
  if (head_dim != HD || S % TQ != 0) return cudaErrorInvalidValue;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(flash_fwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  // qkv viewed as [S][batch][3*heads*HD]; box = 64 columns x 1 batch x 128 positions
  const uint64_t cols = 3ull * heads * HD;
  const uint64_t dims[3] = {cols, (uint64_t)batch, (uint64_t)S};
  const uint64_t strides[2] = {cols * 2, cols * 2 * batch};
  const uint32_t box[3] = {64, 1, 128};
  CUtensorMap tm;
  if (!make_tmap_bf16_3d(&tm, qkv, dims, strides, box)) return cudaErrorInvalidValue;
  const float scale_log2 = (1.0f / sqrtf((float)HD)) * 1.4426950408889634f;
  dim3 grid(S / TQ, batch * heads);
  flash_fwd_tc_kernel<<<grid, THREADS, SMEM, stream>>>(tm, out, lse, S, batch, heads, scale_log2, err);
  return cudaGetLastError();
}

}  // namespace nmb
