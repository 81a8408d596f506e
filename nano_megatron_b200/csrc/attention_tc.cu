// Causal flash-attention forward on 5th-generation tensor cores (sm_100a),
// head_dim 128, bf16 in / out, fp32 softmax and accumulation.
//
// One CTA computes 256 query rows -- two 128-row tiles -- of one (batch,
// head). 16 warps in four warpgroups with separate register budgets
// (setmaxnreg):
//   WG0, WG1  softmax of tile 0 / tile 1, one query row per thread (TMEM lane
//             = row): tcgen05.ld the S row, row max, exp2, row sum, and the
//             probabilities P (bf16) written back into the same TMEM columns
//             with tcgen05.st, where the PV product reads them as its A
//             operand (no shared-memory round trip).
//   WG2       correction: when a row maximum grew, rescales that row of the
//             tile's O accumulator in TMEM; at the end normalizes O by the row
//             sum and writes the output rows.
//   WG3       warp 12 issues every tcgen05.mma; warp 13 issues the TMA loads
//             (Q once, K_j and V_j through two 2-slot rings, all boxes straight
//             out of the fused QKV buffer through one 3-D tensor map). A K slot
//             is released as soon as the last QK product reading it completes,
//             a V slot after the last PV product, so K_{j+2} and V_{j+1} load
//             while block j is still in flight.
//
// The tensor core alternates between the tiles:
//   ... PV_0(j-1)  QK_0(j)  PV_1(j-1)  QK_1(j)  PV_0(j)  QK_0(j+1) ...
// so the softmax of one tile runs while the MMAs of the other execute. S_t(j)
// is written over the TMEM columns that held P_t(j-1); the MMAs are issued by
// one thread and execute in issue order, so PV_t(j-1) has read P_t(j-1)
// before QK_t(j) overwrites it.
//
// The exponentials are split between the SFU (ex2.approx) and the FMA pipe
// (a cubic polynomial, see poly_exp2) so that neither unit alone bounds the
// softmax.
//
// Lazy rescaling: a row keeps its reference maximum until a block's maximum
// exceeds it by more than 2^8 (in exp2 units); only then are the row sum and
// the O row rescaled. Probabilities are at most 256 in between, which bf16
// and the fp32 sums hold without loss; the final O / l is exact either way.
//
// TMEM (512 columns): S0|P0 [0,128), S1|P1 [128,256), O0 [256,384), O1
// [384,512). Shared memory: Q 2 x 32 KB, K 2 x 32 KB, V 2 x 32 KB.
// Register budget (launch: 512 threads x 128): softmax warpgroups 192 each,
// correction 80, MMA/load 48 -- 128 x (192 + 192 + 80 + 48) = 65536.
// Every wait is bounded (error word + abort flag; never a trap).
//
// Output contract is the same as the mma.sync kernel of attention.cu (o and
// lse layouts), so the backward kernels consume either.

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
constexpr int HALF = TQ * 64 * 2;  // 16 KB: 128 rows x 64 bf16 (one swizzle atom column)
constexpr int TILE = 2 * HALF;     // 32 KB
constexpr int OFF_Q = 0, OFF_K = 2 * TILE, OFF_V = 4 * TILE;
constexpr int OFF_ALPHA = 6 * TILE;         // float [2][128]
constexpr int OFF_INVL = OFF_ALPHA + 1024;  // float [2][128]
constexpr int OFF_BAR = OFF_INVL + 1024;
constexpr int SMEM = OFF_BAR + 256 + 1024;
constexpr int THREADS = 512;
constexpr int REG_SOFTMAX = 192, REG_CORRECTION = 80, REG_ISSUE = 48;
static_assert(128 * (2 * REG_SOFTMAX + REG_CORRECTION + REG_ISSUE) == 65536, "register split must fill the launch");
constexpr float kRescaleThreshold = 8.0f;  // log2 units

template <int N>
__device__ __forceinline__ void reg_alloc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void reg_dealloc() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

__device__ __forceinline__ uint64_t kmajor_desc(uint32_t base, int kk) { return nmb::kmajor_desc(base, kk, HALF); }

// 2^x on the FMA pipe for x <= 127 (x below -126 clamps to a denormal, ~1e-38):
// x = n + f with n = rint(x) (adding and subtracting 1.5 * 2^23 rounds to an
// integer, and the low bits of the sum hold n) and f in [-0.5, 0.5]; 2^f is a
// cubic minimax polynomial (maximum relative error 7.5e-5, far below the bf16
// rounding of P; coefficients fitted for this kernel with the Remez exchange
// algorithm on [-0.5, 0.5]); 2^n is added into the exponent field.
__device__ __forceinline__ float poly_exp2(float x) {
  constexpr float kRound = 12582912.f;  // 1.5 * 2^23
  x = fmaxf(x, -126.f);  // n >= -126 keeps the exponent field of the result >= 0
  const float y = x + kRound;
  const float f = x - (y - kRound);
  const float p = fmaf(fmaf(fmaf(0.0551716685f, f, 0.2426111251f), f, 0.6932609677f), f, 0.9999280572f);
  return __uint_as_float(__float_as_uint(p) + (__float_as_uint(y) << 23));
}

// Pairs of columns (c, c+1) with (c / 2) % kPolyPeriod < kPolyPairs take the
// polynomial; the rest the SFU.
constexpr int kPolyPeriod = 4, kPolyPairs = 0;

__global__ void __launch_bounds__(THREADS, 1)
flash_fwd_tc_kernel(const __grid_constant__ CUtensorMap tm_qkv, __nv_bfloat16* __restrict__ out,
                    float* __restrict__ lse, int S, int batch, int heads, float scale_log2, int* err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* q_full = bars;           // 1
  uint64_t* k_full = bars + 1;       // [2] stages
  uint64_t* v_full = bars + 3;       // [2]
  uint64_t* k_empty = bars + 5;      // [2]
  uint64_t* s_full = bars + 7;       // [2] tiles
  uint64_t* p_full = bars + 9;       // [2]
  uint64_t* alpha_full = bars + 11;  // [2]
  uint64_t* o_ready = bars + 13;     // [2]
  uint64_t* pv_done = bars + 15;     // [2]
  uint64_t* fin = bars + 17;         // [2]
  uint64_t* mma_done = bars + 19;    // 1
  uint64_t* v_empty = bars + 20;     // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 22);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* alpha_s = reinterpret_cast<float*>(smem + OFF_ALPHA);
  float* invl_s = reinterpret_cast<float*>(smem + OFF_INVL);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int wg = warp / 4, quarter = warp % 4;
  const int nqt = S / TQ;                 // 128-row query tiles
  const int nblk = (nqt + 1) / 2;         // 256-row CTA blocks
  const int blk = nblk - 1 - blockIdx.x;  // longest rows first
  const int bh = blockIdx.y, b = bh / heads, h = bh % heads;
  int nkb[2];
#pragma unroll
  for (int t = 0; t < 2; ++t) nkb[t] = (2 * blk + t < nqt) ? 2 * blk + t + 1 : 0;
  const int nkb_max = nkb[0] > nkb[1] ? nkb[0] : nkb[1];
  const int q_col = h * HD, k_col = heads * HD + h * HD, v_col = 2 * heads * HD + h * HD;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
      mbar_init(&alpha_full[i], 128);
      mbar_init(&o_ready[i], 128);
      mbar_init(&pv_done[i], 1);
      mbar_init(&fin[i], 128);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 12) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t sbase = smem_u32(smem);
  const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;

  if (wg == 3) {
    reg_dealloc<REG_ISSUE>();
    if (warp == 13 && lane == 0) {
      // ---------------------------------------------------------------- loads
      tma_prefetch_desc(&tm_qkv);
      int issued[2] = {-1, -1};
      mbar_arrive_expect_tx(q_full, (nkb[1] > 0 ? 2 : 1) * TILE);
      for (int t = 0; t < 2; ++t) {
        if (nkb[t] == 0) continue;
        uint8_t* qd = smem + OFF_Q + t * TILE;
        tma_load_3d(qd, &tm_qkv, q_full, q_col, b, (2 * blk + t) * TQ);
        tma_load_3d(qd + HALF, &tm_qkv, q_full, q_col + 64, b, (2 * blk + t) * TQ);
      }
      int k_issued[2] = {-1, -1};
      for (int j = 0; j < nkb_max; ++j) {
        const int st = j & 1, par = (j >> 1) & 1;
        if (!lane_wait(&k_empty[st], par ^ 1, err, abort_flag)) break;
        uint8_t* kd = smem + OFF_K + st * TILE;
        mbar_arrive_expect_tx(&k_full[st], TILE);
        tma_load_3d(kd, &tm_qkv, &k_full[st], k_col, b, j * TK);
        tma_load_3d(kd + HALF, &tm_qkv, &k_full[st], k_col + 64, b, j * TK);
        k_issued[st] = par;
        if (!lane_wait(&v_empty[st], par ^ 1, err, abort_flag)) break;
        uint8_t* vd = smem + OFF_V + st * TILE;
        mbar_arrive_expect_tx(&v_full[st], TILE);
        tma_load_3d(vd, &tm_qkv, &v_full[st], v_col, b, j * TK);
        tma_load_3d(vd + HALF, &tm_qkv, &v_full[st], v_col + 64, b, j * TK);
        issued[st] = par;
      }
      // no copy may still be in flight at exit (matters only after an abort)
      mbar_wait(q_full, 0, nullptr, 1000000000ull);
      for (int st = 0; st < 2; ++st) {
        if (k_issued[st] >= 0) mbar_wait(&k_full[st], k_issued[st], nullptr, 1000000000ull);
        if (issued[st] >= 0) mbar_wait(&v_full[st], issued[st], nullptr, 1000000000ull);
      }
    } else if (warp == 12 && lane == 0) {
      // ------------------------------------------------------------------ MMA
      constexpr uint32_t idesc_s = idesc_bf16_f32(TQ, TK, false, false);
      constexpr uint32_t idesc_o = idesc_bf16_f32(TQ, HD, false, true);
      bool ok = lane_wait(q_full, 0, err, abort_flag) && lane_wait(&k_full[0], 0, err, abort_flag);
      if (ok) {
        tc_fence_after();
        for (int t = 0; t < 2; ++t) {
          if (nkb[t] == 0) continue;
          const uint32_t qb = sbase + OFF_Q + t * TILE, kb = sbase + OFF_K;
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk)
            mma_bf16_ss(tmem + t * TK, kmajor_desc(qb, kk), kmajor_desc(kb, kk), idesc_s, kk > 0);
          mma_commit(&s_full[t]);
        }
        mma_commit(&k_empty[0]);
      }
      for (int j = 1; ok && j <= nkb_max; ++j) {
        const int i = j - 1;  // the block whose PV products are issued now
        if (j < nkb_max && !(ok = lane_wait(&k_full[j & 1], (j >> 1) & 1, err, abort_flag))) break;
        if (!(ok = lane_wait(&v_full[i & 1], (i >> 1) & 1, err, abort_flag))) break;
        tc_fence_after();
        const uint32_t vb = sbase + OFF_V + (i & 1) * TILE;
        const uint32_t kb = sbase + OFF_K + (j & 1) * TILE;
        for (int t = 0; t < 2 && ok; ++t) {
          if (i < nkb[t]) {
            ok = lane_wait(&p_full[t], i & 1, err, abort_flag) &&
                 (i == 0 || lane_wait(&o_ready[t], (i - 1) & 1, err, abort_flag));
            if (!ok) break;
            tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < TK / 16; ++kk)
              mma_bf16_ts(tmem + 256 + t * HD, tmem + t * TK + kk * 8, smem_desc_sw128(vb + kk * 2048, HALF, 1024),
                          idesc_o, (i > 0 || kk > 0));
            mma_commit(&pv_done[t]);
          }
          if (t == 1) mma_commit(&v_empty[i & 1]);  // every PV of block i is issued
          if (j < nkb[t]) {
            const uint32_t qb = sbase + OFF_Q + t * TILE;
#pragma unroll
            for (int kk = 0; kk < HD / 16; ++kk)
              mma_bf16_ss(tmem + t * TK, kmajor_desc(qb, kk), kmajor_desc(kb, kk), idesc_s, kk > 0);
            mma_commit(&s_full[t]);
          }
        }
        if (ok && j < nkb_max) mma_commit(&k_empty[j & 1]);  // every QK of block j is issued
      }
      // TMEM is released only after the last MMA finished (matters after an abort)
      mma_commit(mma_done);
      mbar_wait(mma_done, 0, nullptr, 1000000000ull);
    }
  } else if (wg == 2) {
    reg_dealloc<REG_CORRECTION>();
    // ------------------------------------------------------------ correction
    const int r = quarter * 32 + lane;
    const uint32_t o_base = tmem + lane_off + 256;
    bool ok = true;
    for (int i = 1; i < nkb_max && ok; ++i) {
      for (int t = 0; t < 2; ++t) {
        if (i >= nkb[t]) continue;
        ok = warp_wait(&alpha_full[t], (i - 1) & 1, err, abort_flag) &&
             warp_wait(&pv_done[t], (i - 1) & 1, err, abort_flag);
        if (!ok) break;
        tc_fence_after();
        const float alpha = alpha_s[t * TQ + r];
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
          for (int c = 0; c < HD; c += 32) {
            uint32_t v[32];
            tmem_ld_32x32b_x32(o_base + t * HD + c, v);
            tmem_wait_ld();
#pragma unroll
            for (int k = 0; k < 32; ++k) v[k] = __float_as_uint(__uint_as_float(v[k]) * alpha);
            tmem_st_32x32b_x32(o_base + t * HD + c, v);
          }
          tmem_wait_st();
        }
        tc_fence_before();
        mbar_arrive(&o_ready[t]);
      }
    }
    // epilogue: O / l -> output rows
    for (int t = 0; t < 2 && ok; ++t) {
      if (nkb[t] == 0) continue;
      ok = warp_wait(&fin[t], 0, err, abort_flag) && warp_wait(&pv_done[t], (nkb[t] - 1) & 1, err, abort_flag);
      if (!ok) break;
      tc_fence_after();
      const float inv = invl_s[t * TQ + r];
      const int q = (2 * blk + t) * TQ + r;
      __nv_bfloat16* orow = out + ((long)q * batch + b) * heads * HD + h * HD;
#pragma unroll 1
      for (int c = 0; c < HD; c += 32) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(o_base + t * HD + c, v);
        tmem_wait_ld();
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
  } else {
    reg_alloc<REG_SOFTMAX>();
    // --------------------------------------------------------------- softmax
    const int t = wg;
    const int r = quarter * 32 + lane;  // query row within the tile
    const int q = (2 * blk + t) * TQ + r;
    const uint32_t s_addr = tmem + lane_off + t * TK;
    float m_ref = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nkb[t]; ++j) {
      if (!(ok = warp_wait(&s_full[t], j & 1, err, abort_flag))) break;
      tc_fence_after();
      uint32_t v[TK];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld_32x32b_x32(s_addr + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(&v[32 * c]));
      tmem_wait_ld();
      float* s = reinterpret_cast<float*>(v);
      if (j == nkb[t] - 1) {  // diagonal block: key index c > row r is in the future
#pragma unroll
        for (int c = 0; c < TK; ++c)
          if (c > r) s[c] = -INFINITY;
      }
      float mx0 = s[0], mx1 = s[1], mx2 = s[2], mx3 = s[3];
#pragma unroll
      for (int c = 4; c < TK; c += 4) {
        mx0 = fmaxf(mx0, s[c]);
        mx1 = fmaxf(mx1, s[c + 1]);
        mx2 = fmaxf(mx2, s[c + 2]);
        mx3 = fmaxf(mx3, s[c + 3]);
      }
      const float mb = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3));
      if (j == 0) {
        m_ref = mb;
      } else {
        float alpha = 1.f;
        if ((mb - m_ref) * scale_log2 > kRescaleThreshold) {
          alpha = fast_exp2((m_ref - mb) * scale_log2);
          l *= alpha;
          m_ref = mb;
        }
        alpha_s[t * TQ + r] = alpha;
        mbar_arrive(&alpha_full[t]);
      }
      const float ms = m_ref * scale_log2;
      float sum0 = 0.f, sum1 = 0.f;
      uint32_t p[TK / 2];
#pragma unroll
      for (int c = 0; c < TK; c += 2) {
        const bool poly = (c / 2) % kPolyPeriod < kPolyPairs;
        const float x0 = fmaf(s[c], scale_log2, -ms), x1 = fmaf(s[c + 1], scale_log2, -ms);
        const float e0 = poly ? poly_exp2(x0) : fast_exp2(x0);
        const float e1 = poly ? poly_exp2(x1) : fast_exp2(x1);
        sum0 += e0;
        sum1 += e1;
        p[c / 2] = pack_bf16x2(e0, e1);
      }
      l += sum0 + sum1;
      tmem_st_32x32b_x32(s_addr, *reinterpret_cast<uint32_t(*)[32]>(&p[0]));
      tmem_st_32x32b_x32(s_addr + 32, *reinterpret_cast<uint32_t(*)[32]>(&p[32]));
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_full[t]);
    }
    if (nkb[t] > 0) {
      if (ok) lse[(long)bh * S + q] = (m_ref * scale_log2 + log2f(l)) * 0.6931471805599453f;
      invl_s[t * TQ + r] = 1.f / l;
      mbar_arrive(&fin[t]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 12) {
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
  const int nblk = (S / TQ + 1) / 2;
  dim3 grid(nblk, batch * heads);
  flash_fwd_tc_kernel<<<grid, THREADS, SMEM, stream>>>(tm, out, lse, S, batch, heads, scale_log2, err);
  return cudaGetLastError();
}

}  // namespace nmb
