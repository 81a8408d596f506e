// Causal flash-attention forward on 5th-generation tensor cores (sm_100a),
// head_dim 128, bf16 in / out, fp32 softmax and accumulation.
// Reference op: F.scaled_dot_product_attention(q, k, v, is_causal=True),
// nano_megatron/model.py:126.
//
// One CTA computes 256 query rows -- two 128-row tiles -- of one (batch,
// head). 16 warps in four warpgroups with separate register budgets
// (setmaxnreg):
//   WG0, WG1  softmax of tile 0 / tile 1, one query row per thread (TMEM lane
//             = row). The S row streams out of TMEM in 32-column chunks (the
//             next chunk loads while the current one is exponentiated) and the
//             probabilities P (bf16) go back into the same TMEM columns, where
//             the PV product reads them as its A operand (no shared-memory
//             round trip). Rescaling of the O row, when needed, is done here
//             too (see below).
//   WG2       epilogue: normalizes O by the row sum and writes the output rows
//             of a tile while the other tile may still be running.
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
// before QK_t(j) overwrites it -- and once S_t(j) is complete, PV_t(j-1) has
// completed too, so the softmax may rescale O_t without further waiting.
//
// Lazy rescaling: a row exponentiates against a reference maximum that it
// keeps until a block's maximum exceeds it by more than 2^8 (in exp2 units).
// The common block therefore needs no maximum before its exponentials (they
// stream with the loads); the block maximum is checked at the end, and only
// then, rarely, does the warp reload S, move the reference, recompute the
// block and rescale the row sum and the O rows. Probabilities are at most 256
// in between, which bf16 and the fp32 sums hold without loss; O / l at the end
// is exact either way.
//
// TMEM (512 columns): S0|P0 [0,128), S1|P1 [128,256), O0 [256,384), O1
// [384,512). Shared memory: Q 2 x 32 KB, K 2 x 32 KB, V 2 x 32 KB.
// Register budget (launch: 512 threads x 128): softmax warpgroups 184 each,
// epilogue 88, MMA/load 56 -- 128 x (184 + 184 + 88 + 56) = 65536.
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
constexpr int OFF_INVL = 6 * TILE;  // float [2][128]
constexpr int OFF_BAR = OFF_INVL + 1024;
constexpr int SMEM = OFF_BAR + 256 + 1024;
constexpr int THREADS = 512;
constexpr int REG_SOFTMAX = 184, REG_EPILOGUE = 88, REG_ISSUE = 56;
static_assert(128 * (2 * REG_SOFTMAX + REG_EPILOGUE + REG_ISSUE) == 65536, "register split must fill the launch");
constexpr float kRescaleThreshold = 8.0f;  // log2 units

template <int N>
__device__ __forceinline__ void reg_alloc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void reg_dealloc() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}


__global__ void __launch_bounds__(THREADS, 1)
flash_fwd_tc_kernel(const __grid_constant__ CUtensorMap tm_qkv, __nv_bfloat16* __restrict__ out,
                    float* __restrict__ lse, int S, int batch, int heads, float scale_log2, int* err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* q_full = bars;         // 1
  uint64_t* k_full = bars + 1;     // [2] slots
  uint64_t* v_full = bars + 3;     // [2]
  uint64_t* k_empty = bars + 5;    // [2]
  uint64_t* v_empty = bars + 7;    // [2]
  uint64_t* s_full = bars + 9;     // [2] tiles
  uint64_t* p_full = bars + 11;    // [2]
  uint64_t* pv_done = bars + 13;   // [2]
  uint64_t* fin = bars + 15;       // [2]
  uint64_t* mma_done = bars + 17;  // 1
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 18);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* invl_s = reinterpret_cast<float*>(smem + OFF_INVL);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int wg = warp / 4, quarter = warp % 4;
  const int nqt = S / TQ;                 // 128-row query tiles
  const int nblk = (nqt + 1) / 2;         // 256-row CTA blocks
  // grid (batch*heads, blocks): heads vary fastest, so the hardware hands out
  // the longest (latest) query blocks of every head before any shorter one
  const int blk = nblk - 1 - blockIdx.y;
  const int bh = blockIdx.x, b = bh / heads, h = bh % heads;
  const int nkb0 = 2 * blk + 1;                             // tile 0 always exists
  const int nkb1 = (2 * blk + 1 < nqt) ? 2 * blk + 2 : 0;   // tile 1 may not (odd tile count)
  const int nkb_max = nkb1 > nkb0 ? nkb1 : nkb0;
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
      int k_issued[2] = {-1, -1}, v_issued[2] = {-1, -1};
      mbar_arrive_expect_tx(q_full, (nkb1 > 0 ? 2 : 1) * TILE);
      tma_load_3d(smem + OFF_Q, &tm_qkv, q_full, q_col, b, 2 * blk * TQ);
      tma_load_3d(smem + OFF_Q + HALF, &tm_qkv, q_full, q_col + 64, b, 2 * blk * TQ);
      if (nkb1 > 0) {
        tma_load_3d(smem + OFF_Q + TILE, &tm_qkv, q_full, q_col, b, (2 * blk + 1) * TQ);
        tma_load_3d(smem + OFF_Q + TILE + HALF, &tm_qkv, q_full, q_col + 64, b, (2 * blk + 1) * TQ);
      }
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
        v_issued[st] = par;
      }
      // no copy may still be in flight at exit (matters only after an abort)
      mbar_wait(q_full, 0, nullptr, 1000000000ull);
      for (int st = 0; st < 2; ++st) {
        if (k_issued[st] >= 0) mbar_wait(&k_full[st], k_issued[st], nullptr, 1000000000ull);
        if (v_issued[st] >= 0) mbar_wait(&v_full[st], v_issued[st], nullptr, 1000000000ull);
      }
    } else if (warp == 12 && lane == 0) {
      // ------------------------------------------------------------------ MMA
      constexpr uint32_t idesc_s = idesc_bf16_f32(TQ, TK, false, false);
      constexpr uint32_t idesc_o = idesc_bf16_f32(TQ, HD, false, true);
      // Two base descriptors (start address 0 of this CTA's tiles); a tile,
      // slot and k-step add a compile-time or small offset, in 16-byte units,
      // to the start-address field (which never carries into the next field:
      // shared addresses stay below 256 KB). K-major operands move 32 B inside
      // a swizzle row per k-step and switch 64-column halves at kk = 4; the
      // N-major V moves 16 rows of 128 B.
      const uint64_t kmaj = smem_desc_sw128(sbase, 0, 1024);
      const uint64_t nmaj = smem_desc_sw128(sbase, HALF, 1024);
      auto issue_qk = [&](int t, int slot) {
        const uint64_t qd = kmaj + (uint64_t)((OFF_Q + t * TILE) >> 4);
        const uint64_t kd = kmaj + (uint64_t)((OFF_K + slot * TILE) >> 4);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint64_t off = (uint64_t)(((kk >> 2) * HALF + (kk & 3) * 32) >> 4);
          mma_bf16_ss(tmem + t * TK, qd + off, kd + off, idesc_s, kk > 0);
        }
        mma_commit(&s_full[t]);
      };
      bool ok = lane_wait(q_full, 0, err, abort_flag) && lane_wait(&k_full[0], 0, err, abort_flag);
      if (ok) {
        tc_fence_after();
        issue_qk(0, 0);
        if (nkb1 > 0) issue_qk(1, 0);
        mma_commit(&k_empty[0]);
      }
      for (int j = 1; ok && j <= nkb_max; ++j) {
        const int i = j - 1;  // the block whose PV products are issued now
        if (j < nkb_max && !(ok = lane_wait(&k_full[j & 1], (j >> 1) & 1, err, abort_flag))) break;
        if (!(ok = lane_wait(&v_full[i & 1], (i >> 1) & 1, err, abort_flag))) break;
        for (int t = 0; t < 2 && ok; ++t) {
          const int nkb_t = t == 0 ? nkb0 : nkb1;
          if (i < nkb_t) {
            if (!(ok = lane_wait(&p_full[t], i & 1, err, abort_flag))) break;
            tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < TK / 16; ++kk)
              mma_bf16_ts(tmem + 256 + t * HD, tmem + t * TK + kk * 8,
                          nmaj + (uint64_t)((OFF_V + (i & 1) * TILE + kk * 2048) >> 4), idesc_o, (i > 0 || kk > 0));
            mma_commit(&pv_done[t]);
          }
          if (t == 1) mma_commit(&v_empty[i & 1]);  // every PV of block i is issued
          if (j < nkb_t) issue_qk(t, j & 1);
        }
        if (ok && j < nkb_max) mma_commit(&k_empty[j & 1]);  // every QK of block j is issued
      }
      // TMEM is released only after the last MMA finished (matters after an abort)
      mma_commit(mma_done);
      mbar_wait(mma_done, 0, nullptr, 1000000000ull);
    }
  } else if (wg == 2) {
    reg_dealloc<REG_EPILOGUE>();
    // -------------------------------------------------------------- epilogue
    const int r = quarter * 32 + lane;
    bool ok = true;
    for (int t = 0; t < 2 && ok; ++t) {
      const int nkb = t == 0 ? nkb0 : nkb1;
      if (nkb == 0) continue;
      // fin first: it implies every PV but the last completed (no parity aliasing)
      ok = warp_wait(&fin[t], 0, err, abort_flag) && warp_wait(&pv_done[t], (nkb - 1) & 1, err, abort_flag);
      if (!ok) break;
      tc_fence_after();
      const float inv = invl_s[t * TQ + r];
      const int q = (2 * blk + t) * TQ + r;
      __nv_bfloat16* orow = out + ((long)q * batch + b) * heads * HD + h * HD;
      const uint32_t o_addr = tmem + lane_off + 256 + t * HD;
#pragma unroll 1
      for (int c = 0; c < HD; c += 32) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(o_addr + c, v);
        tmem_wait_ld_regs(v);
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
    const int nkb = t == 0 ? nkb0 : nkb1;
    const int r = quarter * 32 + lane;  // query row within the tile
    const int q = (2 * blk + t) * TQ + r;
    const uint32_t s_addr = tmem + lane_off + t * TK;
    const uint32_t o_addr = tmem + lane_off + 256 + t * HD;
    const float2 scale2 = make_float2(scale_log2, scale_log2);
    float m_ref = -INFINITY, l = 0.f;
    uint32_t p[TK / 2];
    // One pass over the S row in 32-column chunks (the next chunk loads while
    // this one is processed): P = exp2(s * scale - m * scale) into p, returns
    // the row sum and the (masked) row maximum.
    auto exp_pass = [&](float m, bool diag, float& bmax) -> float {
      const float2 nms = make_float2(-m * scale_log2, -m * scale_log2);
      float2 acc = make_float2(0.f, 0.f);
      float mx = -INFINITY;
      uint32_t buf[2][32];
      tmem_ld_32x32b_x32(s_addr, buf[0]);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        tmem_wait_ld_regs(buf[c & 1]);
        if (c < 3) tmem_ld_32x32b_x32(s_addr + 32 * (c + 1), buf[(c + 1) & 1]);
#pragma unroll
        for (int k = 0; k < 32; k += 2) {
          float v0 = __uint_as_float(buf[c & 1][k]), v1 = __uint_as_float(buf[c & 1][k + 1]);
          if (diag) {
            if (32 * c + k > r) v0 = -INFINITY;
            if (32 * c + k + 1 > r) v1 = -INFINITY;
          }
          mx = fmaxf(mx, fmaxf(v0, v1));
          const float2 x = ffma2(make_float2(v0, v1), scale2, nms);
          const float e0 = fast_exp2(x.x), e1 = fast_exp2(x.y);
          acc = fadd2(acc, make_float2(e0, e1));
          p[16 * c + k / 2] = pack_bf16x2(e0, e1);
        }
      }
      bmax = mx;
      return acc.x + acc.y;
    };
    // Row maximum of the (masked) S row, chunk by chunk.
    auto max_pass = [&](bool diag) -> float {
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(s_addr + 32 * c, v);
        tmem_wait_ld_regs(v);
#pragma unroll
        for (int k = 0; k < 32; k += 2) {
          float v0 = __uint_as_float(v[k]), v1 = __uint_as_float(v[k + 1]);
          if (diag) {
            if (32 * c + k > r) v0 = -INFINITY;
            if (32 * c + k + 1 > r) v1 = -INFINITY;
          }
          mx0 = fmaxf(mx0, v0);
          mx1 = fmaxf(mx1, v1);
        }
      }
      return fmaxf(mx0, mx1);
    };
    bool ok = true;
    for (int j = 0; j < nkb; ++j) {
      if (!(ok = warp_wait(&s_full[t], j & 1, err, abort_flag))) break;
      tc_fence_after();
      const bool diag = j == nkb - 1;  // key index c > row r is in the future
      float alpha = 1.f, sum, bmax;
      if (j == 0) {
        m_ref = max_pass(diag);
        sum = exp_pass(m_ref, diag, bmax);
      } else {
        sum = exp_pass(m_ref, diag, bmax);
        const bool moved = (bmax - m_ref) * scale_log2 > kRescaleThreshold;
        if (__any_sync(0xffffffffu, moved)) {
          const float m_new = moved ? bmax : m_ref;
          alpha = fast_exp2((m_ref - m_new) * scale_log2);
          m_ref = m_new;
          sum = exp_pass(m_ref, diag, bmax);
#pragma unroll 1
          for (int c = 0; c < HD; c += 32) {
            uint32_t o[32];
            tmem_ld_32x32b_x32(o_addr + c, o);
            tmem_wait_ld_regs(o);
#pragma unroll
            for (int k = 0; k < 32; ++k) o[k] = __float_as_uint(__uint_as_float(o[k]) * alpha);
            tmem_st_32x32b_x32(o_addr + c, o);
          }
        }
      }
      l = l * alpha + sum;
      tmem_st_32x32b_x32(s_addr, *reinterpret_cast<uint32_t(*)[32]>(&p[0]));
      tmem_st_32x32b_x32(s_addr + 32, *reinterpret_cast<uint32_t(*)[32]>(&p[32]));
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_full[t]);
    }
    if (nkb > 0) {
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
  dim3 grid(batch * heads, nblk);
  flash_fwd_tc_kernel<<<grid, THREADS, SMEM, stream>>>(tm, out, lse, S, batch, heads, scale_log2, err);
  return cudaGetLastError();
}

}  // namespace nmb
