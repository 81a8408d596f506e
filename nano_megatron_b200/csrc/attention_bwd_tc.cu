// Causal flash-attention backward on 5th-generation tensor cores (sm_100a),
// head_dim 128, bf16 in / out, fp32 math. Two deterministic kernels, no atomics.
// Reference op: the autograd backward of the RoPE + causal SDPA of
// nano_megatron/model.py:124-126 (the inverse rotation is applied in the stores).
//
//   dK/dV kernel (one CTA = 128 keys of one (batch, head); loops over the
//   64-query blocks at or after it):
//     S^T = K Q^T and dP^T = V dO^T      (tcgen05, M=128 keys, N=64 queries)
//     P^T = exp(S^T*scale - lse[q]), dS^T = P^T (dP^T - D[q])   (one key row
//          per thread, causal mask on the diagonal blocks; P^T and dS^T go
//          back into TMEM as bf16)
//     dV += P^T dO and dK += dS^T Q      (tcgen05 with A from TMEM; the
//          accumulators stay in TMEM)
//   dQ kernel (one CTA = 128 queries; loops over the 128-key blocks up to it):
//     S = Q K^T, dP = dO V^T, dS = P (dP - D[q]) (back into TMEM), dQ += dS K.
//
// The dQ kernel recomputes S and dP instead of having the dK/dV kernel add
// dQ partials with atomics: two extra 128x64x128 products per block pair buy
// a fixed summation order and no fp32 atomic traffic.
//
// Both kernels: warp 0 issues TMA loads (tiles straight out of qkv / dO via
// 3-D tensor maps) through a ring, warp 1 issues the MMAs from an event loop,
// and two elementwise warpgroups (warps 2-5, 6-9) do the exp/convert work. In
// the dK/dV kernel the groups take alternate 64-query blocks, each with its
// own TMEM columns; in the dQ kernel both groups share every 128-key block
// (see there). The grid lists heads fastest, so the CTAs with the most blocks
// of every head are dispatched first. Every wait is bounded.
// D[q] = rowsum(dO * O) comes from flash_bwd_dot_kernel (attention.cu).

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cmath>

#include "attention.cuh"
#include "gemm.cuh"
#include "ptx.cuh"

namespace nmb {

namespace {

constexpr int HD = 128;
constexpr int BIG = 128, SMALL = 64;           // rows of the resident / streamed tiles
constexpr int HALF_BIG = BIG * 128;            // 16 KB: one 64-column half of a 128-row tile
constexpr int HALF_SMALL = SMALL * 128;        // 8 KB: one 64-column half of a 64-row tile
constexpr int TILE_BIG = 2 * HALF_BIG, TILE_SMALL = 2 * HALF_SMALL;
constexpr float LOG2E = 1.4426950408889634f;

// 64 values of a row as bf16 pairs into 32 TMEM columns at `taddr`.
__device__ __forceinline__ void st_row64(uint32_t taddr, const float (&v)[SMALL]) {
  uint32_t u[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) u[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
  tmem_st_32x32b_x32(taddr, u);
}

// Two 64-column fp32 TMEM rows (S and dP of one block): all four loads are in
// flight before the single wait.
__device__ __forceinline__ void ld_two_rows64(uint32_t ta, uint32_t tb, float (&x)[SMALL], float (&y)[SMALL]) {
  uint32_t u[4][32];
  tmem_ld_32x32b_x32(ta, u[0]);
  tmem_ld_32x32b_x32(ta + 32, u[1]);
  tmem_ld_32x32b_x32(tb, u[2]);
  tmem_ld_32x32b_x32(tb + 32, u[3]);
#pragma unroll
  for (int c = 0; c < 4; ++c) tmem_wait_ld_regs(u[c]);
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    x[i] = __uint_as_float(u[0][i]);
    x[32 + i] = __uint_as_float(u[1][i]);
    y[i] = __uint_as_float(u[2][i]);
    y[32 + i] = __uint_as_float(u[3][i]);
  }
}

// Write a 128-column fp32 TMEM row, times `scale`, as bf16 to global memory.
__device__ __forceinline__ void store_tmem_row(uint32_t taddr, __nv_bfloat16* dst, float scale, bool write) {
#pragma unroll
  for (int c = 0; c < HD; c += 32) {
    uint32_t v[32];
    tmem_ld_32x32b_x32(taddr + c, v);
    tmem_wait_ld();
    if (write) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        uint4 u;
        u.x = pack_bf16x2(__uint_as_float(v[8 * k + 0]) * scale, __uint_as_float(v[8 * k + 1]) * scale);
        u.y = pack_bf16x2(__uint_as_float(v[8 * k + 2]) * scale, __uint_as_float(v[8 * k + 3]) * scale);
        u.z = pack_bf16x2(__uint_as_float(v[8 * k + 4]) * scale, __uint_as_float(v[8 * k + 5]) * scale);
        u.w = pack_bf16x2(__uint_as_float(v[8 * k + 6]) * scale, __uint_as_float(v[8 * k + 7]) * scale);
        *reinterpret_cast<uint4*>(dst + c + 8 * k) = u;
      }
    }
  }
}


// Columns [c0, c0 + 32) and [c0 + 64, c0 + 96) of a 128-column fp32 TMEM row,
// times `scale`, as bf16 to the same columns of `dst`. With `cosv` set, the
// pairs (d, d + 64) are first turned back by the rotary angle of position
// `pos` (the inverse of the forward's NeoX rotation: x1 c + x2 s, x2 c - x1 s;
// cos/sin tables [S][64]), so no separate RoPE pass runs over the gradient.
__device__ __forceinline__ void store_tmem_pairs(uint32_t taddr, int c0, __nv_bfloat16* dst, float scale, bool write,
                                                 const float* cosv, const float* sinv, long pos) {
  uint32_t lo[32], hi[32];
  tmem_ld_32x32b_x32(taddr + c0, lo);
  tmem_ld_32x32b_x32(taddr + 64 + c0, hi);
  tmem_wait_ld_regs(lo);
  tmem_wait_ld_regs(hi);
  if (!write) return;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    float o1[8], o2[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      o1[e] = __uint_as_float(lo[8 * k + e]) * scale;
      o2[e] = __uint_as_float(hi[8 * k + e]) * scale;
    }
    if (cosv != nullptr) {
      const float4* cp = reinterpret_cast<const float4*>(cosv + pos * 64 + c0 + 8 * k);
      const float4* sp = reinterpret_cast<const float4*>(sinv + pos * 64 + c0 + 8 * k);
      const float4 ca = cp[0], cb = cp[1], sa = sp[0], sb = sp[1];
      const float cv[8] = {ca.x, ca.y, ca.z, ca.w, cb.x, cb.y, cb.z, cb.w};
      const float sv[8] = {sa.x, sa.y, sa.z, sa.w, sb.x, sb.y, sb.z, sb.w};
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float x1 = o1[e], x2 = o2[e];
        o1[e] = x1 * cv[e] + x2 * sv[e];
        o2[e] = x2 * cv[e] - x1 * sv[e];
      }
    }
    uint4 u1, u2;
    u1.x = pack_bf16x2(o1[0], o1[1]); u1.y = pack_bf16x2(o1[2], o1[3]);
    u1.z = pack_bf16x2(o1[4], o1[5]); u1.w = pack_bf16x2(o1[6], o1[7]);
    u2.x = pack_bf16x2(o2[0], o2[1]); u2.y = pack_bf16x2(o2[2], o2[3]);
    u2.z = pack_bf16x2(o2[4], o2[5]); u2.w = pack_bf16x2(o2[6], o2[7]);
    *reinterpret_cast<uint4*>(dst + c0 + 8 * k) = u1;
    *reinterpret_cast<uint4*>(dst + 64 + c0 + 8 * k) = u2;
  }
}

struct BwdArgs {
  const float* lse;   // [batch*heads, S]
  const float* lse2;  // lse * log2(e), [batch*heads, S]
  const float* dvec;  // [batch*heads, S]
  __nv_bfloat16* dqkv;
  const float* cosv;  // rotary tables [S][64] for dQ and dK, or null (no rotation)
  const float* sinv;
  int S, batch, heads;
  float scale;
  int* err;
};

// ============================================================ dK / dV kernel
// Two elementwise warpgroups (warps 2-5 and 6-9) take alternate 64-query
// blocks, each with its own S^T/dP^T TMEM columns, so one group's exp/convert
// work overlaps the tensor core's work for the other. P^T and dS^T go back
// into TMEM (bf16, over the S^T/dP^T columns just read) and are the A
// operands of the dV/dK products: no shared-memory round trip.
// smem: K 32K | V 32K | Q[4] 4x16K | dO[4] 4x16K | lse2,D[4]
// (lse2 = lse * log2(e) and D of a query block travel with its Q/dO stage)
constexpr int KV_THREADS = 320;
constexpr int KV_STAGES = 4;
constexpr int KV_OFF_K = 0, KV_OFF_V = TILE_BIG, KV_OFF_Q = 2 * TILE_BIG,
              KV_OFF_DO = KV_OFF_Q + KV_STAGES * TILE_SMALL,
              KV_OFF_LD = KV_OFF_DO + KV_STAGES * TILE_SMALL, KV_OFF_BAR = KV_OFF_LD + KV_STAGES * 2 * SMALL * 4;
constexpr int KV_SMEM = KV_OFF_BAR + 256 + 1024;

__global__ void __launch_bounds__(KV_THREADS, 1)
flash_bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tm_qkv_big, const __grid_constant__ CUtensorMap tm_qkv_small,
                      const __grid_constant__ CUtensorMap tm_do_small, const BwdArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + KV_OFF_BAR);
  uint64_t* kv_full = bars;                        // K and V
  uint64_t* qdo_full = bars + 1;                   // [KV_STAGES] Q/dO stage i % KV_STAGES
  uint64_t* qdo_empty = qdo_full + KV_STAGES;      // [KV_STAGES]
  uint64_t* st_full = qdo_empty + KV_STAGES;       // [2] per group: S^T and dP^T ready
  uint64_t* pds_full = st_full + 2;                // [2] per group: P^T and dS^T in TMEM
  uint64_t* acc_done = pds_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  // grid (batch*heads, key blocks): heads vary fastest, so the key blocks with
  // the most query blocks (low index) of every head are handed out first
  const int kb = blockIdx.y;  // key block of 128; low index = most query blocks
  const int bh = blockIdx.x, b = bh / a.heads, h = bh % a.heads;
  const int first_qb = 2 * kb, nqb = a.S / SMALL;
  const int nblk = nqb - first_qb;
  const int q_col = h * HD, k_col = a.heads * HD + h * HD, v_col = 2 * a.heads * HD + h * HD, do_col = h * HD;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < KV_STAGES; ++i) {
      mbar_init(&qdo_full[i], 1);
      mbar_init(&qdo_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&st_full[i], 1);
      mbar_init(&pds_full[i], 128);
    }
    mbar_init(acc_done, 1);
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
  // TMEM columns: S^T|P^T of group g at 64g, dP^T|dS^T of group g at 128 + 64g, dV 256, dK 384
  const uint32_t tmem = *tmem_slot;
  const uint32_t sbase = smem_u32(smem);

  if (warp == 0 && lane == 0) {
    int issued[KV_STAGES];
#pragma unroll
    for (int st = 0; st < KV_STAGES; ++st) issued[st] = -1;
    mbar_arrive_expect_tx(kv_full, 2 * TILE_BIG);
    tma_load_3d(smem + KV_OFF_K, &tm_qkv_big, kv_full, k_col, b, kb * BIG);
    tma_load_3d(smem + KV_OFF_K + HALF_BIG, &tm_qkv_big, kv_full, k_col + 64, b, kb * BIG);
    tma_load_3d(smem + KV_OFF_V, &tm_qkv_big, kv_full, v_col, b, kb * BIG);
    tma_load_3d(smem + KV_OFF_V + HALF_BIG, &tm_qkv_big, kv_full, v_col + 64, b, kb * BIG);
    for (int i = 0; i < nblk; ++i) {
      const int st = i % KV_STAGES;
      if (!lane_wait(&qdo_empty[st], ((i / KV_STAGES) & 1) ^ 1, a.err, abort_flag)) break;
      const int q0 = (first_qb + i) * SMALL;
      uint8_t* qd = smem + KV_OFF_Q + st * TILE_SMALL;
      uint8_t* dd = smem + KV_OFF_DO + st * TILE_SMALL;
      mbar_arrive_expect_tx(&qdo_full[st], 2 * TILE_SMALL + 2 * SMALL * 4);
      float* ld_dst = reinterpret_cast<float*>(smem + KV_OFF_LD) + st * 2 * SMALL;
      bulk_load(ld_dst, a.lse2 + (long)bh * a.S + q0, SMALL * 4, &qdo_full[st]);
      bulk_load(ld_dst + SMALL, a.dvec + (long)bh * a.S + q0, SMALL * 4, &qdo_full[st]);
      tma_load_3d(qd, &tm_qkv_small, &qdo_full[st], q_col, b, q0);
      tma_load_3d(qd + HALF_SMALL, &tm_qkv_small, &qdo_full[st], q_col + 64, b, q0);
      tma_load_3d(dd, &tm_do_small, &qdo_full[st], do_col, b, q0);
      tma_load_3d(dd + HALF_SMALL, &tm_do_small, &qdo_full[st], do_col + 64, b, q0);
      issued[st] = (i / KV_STAGES) & 1;
    }
    mbar_wait(kv_full, 0, nullptr, 1000000000ull);
    for (int st = 0; st < KV_STAGES; ++st)
      if (issued[st] >= 0) mbar_wait(&qdo_full[st], issued[st], nullptr, 1000000000ull);
  } else if (warp == 1 && lane == 0) {
    // Event loop: issue the S^T/dP^T products of block `ns` as soon as its
    // group's TMEM columns are free and its Q/dO stage has landed, and the
    // dV/dK products of block `na` as soon as its group has published P^T/dS^T,
    // whichever is ready first; never more than one block ahead per group.
    constexpr uint32_t idesc_t = idesc_bf16_f32(BIG, SMALL, false, false);  // S^T, dP^T
    constexpr uint32_t idesc_acc = idesc_bf16_f32(BIG, HD, false, true);    // dV, dK
    bool ok = lane_wait(kv_full, 0, a.err, abort_flag);
    int ns = 0, na = 0;
    uint64_t idle_since = 0;
    while (ok && na < nblk) {
      bool progressed = false;
      // S^T(ns) reuses the TMEM columns of block ns-2 of the same group, whose
      // dV/dK products (the readers of P^T/dS^T there) were issued before it.
      if (ns < nblk && ns < na + 2) {
        const int g = ns & 1, st = ns % KV_STAGES;
        if (mbar_try_wait(&qdo_full[st], (ns / KV_STAGES) & 1)) {
          tc_fence_after();
          const uint32_t qs = sbase + KV_OFF_Q + st * TILE_SMALL, ds = sbase + KV_OFF_DO + st * TILE_SMALL;
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk) {
            mma_bf16_ss(tmem + g * SMALL, kmajor_desc(sbase + KV_OFF_K, kk, HALF_BIG),
                        kmajor_desc(qs, kk, HALF_SMALL), idesc_t, kk > 0);
            mma_bf16_ss(tmem + 128 + g * SMALL, kmajor_desc(sbase + KV_OFF_V, kk, HALF_BIG),
                        kmajor_desc(ds, kk, HALF_SMALL), idesc_t, kk > 0);
          }
          mma_commit(&st_full[g]);
          ++ns;
          progressed = true;
        }
      }
      if (na < ns) {
        const int g = na & 1, st = na % KV_STAGES;
        if (mbar_try_wait(&pds_full[g], (na >> 1) & 1)) {
          tc_fence_after();
          const uint32_t qs = sbase + KV_OFF_Q + st * TILE_SMALL, ds = sbase + KV_OFF_DO + st * TILE_SMALL;
#pragma unroll
          for (int kk = 0; kk < SMALL / 16; ++kk) {
            // A = P^T / dS^T in TMEM (bf16 pairs, 8 columns per k-step);
            // B = dO / Q block viewed N-major: [2 d-halves][64 q rows][128 B]
            mma_bf16_ts(tmem + 256, tmem + g * SMALL + kk * 8, smem_desc_sw128(ds + kk * 2048, HALF_SMALL, 1024),
                        idesc_acc, (na > 0 || kk > 0));
            mma_bf16_ts(tmem + 384, tmem + 128 + g * SMALL + kk * 8,
                        smem_desc_sw128(qs + kk * 2048, HALF_SMALL, 1024), idesc_acc, (na > 0 || kk > 0));
          }
          mma_commit(&qdo_empty[st]);
          ++na;
          progressed = true;
        }
      }
      if (progressed) {
        idle_since = 0;
      } else {
        // nothing ready: back off briefly so the elementwise warps keep the issue slots
        if (idle_since == 0) {
          idle_since = globaltimer_ns();
        } else if (*abort_flag || globaltimer_ns() - idle_since > 2000000000ull) {
          report_error(a.err, kBarrierTimeout);
          *abort_flag = 1;
          ok = false;
        }
        __nanosleep(32);
      }
    }
    mma_commit(acc_done);
  } else if (warp >= 2) {
    const int g = (warp - 2) / 4;   // elementwise group
    const int quarter = warp & 3;   // TMEM lane quarter this warp may access
    const int r = quarter * 32 + lane;  // key row within the block
    const int key = kb * BIG + r;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const float sl2 = a.scale * LOG2E;
    bool ok = true;
    for (int i = g, n = 0; i < nblk && ok; i += 2, ++n) {
      const int q0 = (first_qb + i) * SMALL;
      // the block's lse2 and D arrived with its Q/dO stage (complete before S^T was issued)
      const float* lse_s = reinterpret_cast<const float*>(smem + KV_OFF_LD) + (i % KV_STAGES) * 2 * SMALL;
      const float* d_s = lse_s + SMALL;
      ok = warp_wait(&st_full[g], n & 1, a.err, abort_flag);
      if (!ok) break;
      tc_fence_after();
      float s[SMALL], dp[SMALL];
      const uint32_t s_addr = tmem + lane_off + g * SMALL, dp_addr = tmem + lane_off + 128 + g * SMALL;
      ld_two_rows64(s_addr, dp_addr, s, dp);
      const bool diagonal = q0 < kb * BIG + BIG;  // some key of this block is after some query
#pragma unroll
      for (int c = 0; c < SMALL; c += 4) {
        const float4 l4 = *reinterpret_cast<const float4*>(lse_s + c);
        const float4 d4 = *reinterpret_cast<const float4*>(d_s + c);
        const float lv[4] = {l4.x, l4.y, l4.z, l4.w}, dv[4] = {d4.x, d4.y, d4.z, d4.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          float pr = fast_exp2(fmaf(s[c + k], sl2, -lv[k]));
          if (diagonal && key > q0 + c + k) pr = 0.f;
          s[c + k] = pr;
          dp[c + k] = pr * (dp[c + k] - dv[k]);
        }
      }
      // P^T and dS^T (bf16) over the first half of the S^T / dP^T columns just read
      st_row64(s_addr, s);
      st_row64(dp_addr, dp);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&pds_full[g]);
    }
    if (ok) ok = warp_wait(acc_done, 0, a.err, abort_flag);
    tc_fence_after();
    const long ld = 3L * a.heads * HD;
    __nv_bfloat16* row = a.dqkv + ((long)key * a.batch + b) * ld;
    if (g == 0) store_tmem_row(tmem + lane_off + 256, row + v_col, 1.f, ok);      // dV
    else {                                                                         // dK
      store_tmem_pairs(tmem + lane_off + 384, 0, row + k_col, a.scale, ok, a.cosv, a.sinv, key);
      store_tmem_pairs(tmem + lane_off + 384, 32, row + k_col, a.scale, ok, a.cosv, a.sinv, key);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ================================================================= dQ kernel
// One CTA = 128 queries of one (batch, head), looping over the 128-key blocks
// up to the diagonal. Per block: S = Q K^T (A = Q held in TMEM) and dP = dO V^T,
// both M=128 x N=128; dS = P (dP - D[q]) goes back into TMEM as bf16 and is
// the A operand of dQ += dS K. Both elementwise warpgroups work on every
// block, group g on keys [64g, 64g + 64) of it. S and dP have barriers of
// their own: the groups load S and hand its columns back while dP is still on
// the tensor core, then load dP and hand those back while S of block j + 1
// runs, so each hand-off round trip (commit, load, release, issue) hides
// behind the other product instead of idling the tensor core. dS has columns
// of its own. At M=128 an MMA takes about max(N/2, 32 + N/4) cycles (the 128x16 A
// tile streams in 32 cycles, from TMEM or shared memory alike), so these
// N=128 products run at the full rate where N=64 ones reach two thirds of it.
// Warp 0 streams K/V through a 3-stage ring; Q is staged once in the V slot of
// stage 2 and copied into TMEM by group 0 before that slot is first filled.
// Warp 1 issues the MMAs from an event loop. dQ accumulates in TMEM in
// key-block order (deterministic).
// smem: dO 32K | [K 32K | V 32K] x 3
// TMEM columns: S 0 | dP 128 | dQ 256 | dS 384 (bf16 pairs) | Q 448 (bf16 pairs)
constexpr int Q_THREADS = 320;
constexpr int Q_STAGES = 3;
constexpr int Q_STAGE = 2 * TILE_BIG;
constexpr int Q_OFF_DO = 0, Q_OFF_KV = TILE_BIG, Q_OFF_BAR = Q_OFF_KV + Q_STAGES * Q_STAGE;
constexpr int Q_OFF_QSTAGE = Q_OFF_KV + 2 * Q_STAGE + TILE_BIG;  // V slot of stage 2
constexpr int Q_SMEM = Q_OFF_BAR + 256 + 1024;
constexpr uint32_t Q_TM_S = 0, Q_TM_DP = 128, Q_TM_DQ = 256, Q_TM_DS = 384, Q_TM_Q = 448;
static_assert(Q_SMEM <= 232448, "dQ kernel shared memory");

__global__ void __launch_bounds__(Q_THREADS, 1)
flash_bwd_dq_tc_kernel(const __grid_constant__ CUtensorMap tm_qkv_big, const __grid_constant__ CUtensorMap tm_do_big,
                       const BwdArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Q_OFF_BAR);
  uint64_t* qdo_full = bars;                 // Q (staged) and dO landed
  uint64_t* kv_full = bars + 1;              // [Q_STAGES]
  uint64_t* kv_empty = kv_full + Q_STAGES;   // [Q_STAGES]
  uint64_t* s_full = kv_empty + Q_STAGES;    // S of the block ready
  uint64_t* s_free = s_full + 1;             // S loaded by both groups
  uint64_t* dp_full = s_free + 1;            // dP of the block ready
  uint64_t* dp_free = dp_full + 1;           // dP loaded by both groups
  uint64_t* ds_full = dp_free + 1;           // dS in TMEM
  uint64_t* ds_empty = ds_full + 1;          // the dQ product that read dS is done
  uint64_t* q_tmem = ds_empty + 1;           // Q copied into TMEM (its staging slot is free)
  uint64_t* acc_done = q_tmem + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int nqb = a.S / BIG;
  const int qb = nqb - 1 - blockIdx.y;  // longest rows first (heads vary fastest in the grid)
  const int bh = blockIdx.x, b = bh / a.heads, h = bh % a.heads;
  const int nblk = qb + 1;              // 128-key blocks up to the diagonal
  const int q_col = h * HD, k_col = a.heads * HD + h * HD, v_col = 2 * a.heads * HD + h * HD, do_col = h * HD;

  if (threadIdx.x == 0) {
    mbar_init(qdo_full, 1);
    for (int i = 0; i < Q_STAGES; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, 256);
    mbar_init(dp_full, 1);
    mbar_init(dp_free, 256);
    mbar_init(ds_full, 256);
    mbar_init(ds_empty, 1);
    mbar_init(q_tmem, 128);
    mbar_init(acc_done, 1);
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
    int issued[Q_STAGES];
#pragma unroll
    for (int st = 0; st < Q_STAGES; ++st) issued[st] = -1;
    mbar_arrive_expect_tx(qdo_full, 2 * TILE_BIG);
    tma_load_3d(smem + Q_OFF_QSTAGE, &tm_qkv_big, qdo_full, q_col, b, qb * BIG);
    tma_load_3d(smem + Q_OFF_QSTAGE + HALF_BIG, &tm_qkv_big, qdo_full, q_col + 64, b, qb * BIG);
    tma_load_3d(smem + Q_OFF_DO, &tm_do_big, qdo_full, do_col, b, qb * BIG);
    tma_load_3d(smem + Q_OFF_DO + HALF_BIG, &tm_do_big, qdo_full, do_col + 64, b, qb * BIG);
    for (int j = 0; j < nblk; ++j) {
      const int st = j % Q_STAGES;
      if (!lane_wait(&kv_empty[st], ((j / Q_STAGES) & 1) ^ 1, a.err, abort_flag)) break;
      // stage 2's V slot held Q until group 0 copied it into TMEM
      if (j == 2 && !lane_wait(q_tmem, 0, a.err, abort_flag)) break;
      uint8_t* kd = smem + Q_OFF_KV + st * Q_STAGE;
      uint8_t* vd = kd + TILE_BIG;
      mbar_arrive_expect_tx(&kv_full[st], 2 * TILE_BIG);
      tma_load_3d(kd, &tm_qkv_big, &kv_full[st], k_col, b, j * BIG);
      tma_load_3d(kd + HALF_BIG, &tm_qkv_big, &kv_full[st], k_col + 64, b, j * BIG);
      tma_load_3d(vd, &tm_qkv_big, &kv_full[st], v_col, b, j * BIG);
      tma_load_3d(vd + HALF_BIG, &tm_qkv_big, &kv_full[st], v_col + 64, b, j * BIG);
      issued[st] = (j / Q_STAGES) & 1;
    }
    mbar_wait(qdo_full, 0, nullptr, 1000000000ull);
    for (int st = 0; st < Q_STAGES; ++st)
      if (issued[st] >= 0) mbar_wait(&kv_full[st], issued[st], nullptr, 1000000000ull);
  } else if (warp == 1 && lane == 0) {
    constexpr uint32_t idesc_s = idesc_bf16_f32(BIG, BIG, false, false);  // S, dP (N = 128 keys)
    constexpr uint32_t idesc_q = idesc_bf16_f32(BIG, HD, false, true);    // dQ
    bool ok = lane_wait(qdo_full, 0, a.err, abort_flag) && lane_wait(q_tmem, 0, a.err, abort_flag);
    int ns = 0, nd = 0, na = 0;  // next S, dP and dQ product to issue
    uint64_t idle_since = 0;
    // Every barrier here completes once per block in block order, and none
    // can complete twice before this loop has seen it, so the parity tests
    // never skip a phase.
    while (ok && na < nblk) {
      bool progressed = false;
      // S(ns) reuses the S columns once both groups have loaded S(ns-1)
      if (ns < nblk && ns <= nd && (ns == 0 || mbar_try_wait(s_free, (ns - 1) & 1))) {
        const int st = ns % Q_STAGES;
        if (mbar_try_wait(&kv_full[st], (ns / Q_STAGES) & 1)) {
          tc_fence_after();
          const uint32_t ks = sbase + Q_OFF_KV + st * Q_STAGE;
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk)
            // A = Q from TMEM (bf16 pairs, 8 columns per k-step), B = K
            mma_bf16_ts(tmem + Q_TM_S, tmem + Q_TM_Q + kk * 8, kmajor_desc(ks, kk, HALF_BIG), idesc_s, kk > 0);
          mma_commit(s_full);
          ++ns;
          progressed = true;
        }
      }
      // dP(nd) after S(nd), once both groups have loaded dP(nd-1)
      if (nd < ns && (nd == 0 || mbar_try_wait(dp_free, (nd - 1) & 1))) {
        const int st = nd % Q_STAGES;
        tc_fence_after();
        const uint32_t vs = sbase + Q_OFF_KV + st * Q_STAGE + TILE_BIG;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk)
          mma_bf16_ss(tmem + Q_TM_DP, kmajor_desc(sbase + Q_OFF_DO, kk, HALF_BIG), kmajor_desc(vs, kk, HALF_BIG),
                      idesc_s, kk > 0);
        mma_commit(dp_full);
        ++nd;
        progressed = true;
      }
      if (na < nd && mbar_try_wait(ds_full, na & 1)) {
        const int st = na % Q_STAGES;
        tc_fence_after();
        const uint32_t ks = sbase + Q_OFF_KV + st * Q_STAGE;
#pragma unroll
        for (int kk = 0; kk < BIG / 16; ++kk)
          // A = dS (bf16 pairs, 8 columns per 16 keys); B = the K block viewed
          // N-major: [2 d-halves][128 keys][128 B]
          mma_bf16_ts(tmem + Q_TM_DQ, tmem + Q_TM_DS + kk * 8, smem_desc_sw128(ks + kk * 2048, HALF_BIG, 1024),
                      idesc_q, (na > 0 || kk > 0));
        mma_commit(&kv_empty[st]);
        mma_commit(ds_empty);
        ++na;
        progressed = true;
      }
      if (progressed) {
        idle_since = 0;
      } else {
        // nothing ready: back off briefly so the elementwise warps keep the issue slots
        if (idle_since == 0) {
          idle_since = globaltimer_ns();
        } else if (*abort_flag || globaltimer_ns() - idle_since > 2000000000ull) {
          report_error(a.err, kBarrierTimeout);
          *abort_flag = 1;
          ok = false;
        }
        __nanosleep(32);
      }
    }
    mma_commit(acc_done);
  } else if (warp >= 2) {
    const int g = (warp - 2) / 4;       // elementwise group: keys [64g, 64g + 64) of each block
    const int quarter = warp & 3;       // TMEM lane quarter this warp may access
    const int r = quarter * 32 + lane;  // query row
    const int q = qb * BIG + r;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const float sl2 = a.scale * LOG2E;
    const float lse2 = a.lse2[(long)bh * a.S + q];
    const float dq = a.dvec[(long)bh * a.S + q];
    bool ok = true;
    if (g == 0) {
      // Q row r into TMEM as bf16 pairs (column c = elements 2c, 2c+1): the A
      // operand of S = Q K^T. Row r of a 128B-swizzled half keeps its 16-byte
      // chunk j at chunk j ^ (r & 7); the 8 rows a quarter-warp reads hit 8
      // different chunks, so the loads are free of bank conflicts.
      ok = warp_wait(qdo_full, 0, a.err, abort_flag);
      if (ok) {
        const uint8_t* qrow = smem + Q_OFF_QSTAGE + r * 128;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t u[32];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint4 v = *reinterpret_cast<const uint4*>(qrow + half * HALF_BIG + ((j ^ (r & 7)) << 4));
            u[4 * j + 0] = v.x;
            u[4 * j + 1] = v.y;
            u[4 * j + 2] = v.z;
            u[4 * j + 3] = v.w;
          }
          tmem_st_32x32b_x32(tmem + lane_off + Q_TM_Q + half * 32, u);
        }
        tmem_wait_st();
      }
      tc_fence_before();
      mbar_arrive(q_tmem);
    }
    for (int j = 0; j < nblk && ok; ++j) {
      const int k0 = j * BIG + g * SMALL;  // key of this group's first column
      const bool diagonal = j == qb;
      float p[SMALL];
      {
        ok = warp_wait(s_full, j & 1, a.err, abort_flag);
        if (!ok) break;
        tc_fence_after();
        uint32_t u[2][32];
        tmem_ld_32x32b_x32(tmem + lane_off + Q_TM_S + g * SMALL, u[0]);
        tmem_ld_32x32b_x32(tmem + lane_off + Q_TM_S + g * SMALL + 32, u[1]);
        tmem_wait_ld_regs(u[0]);
        tmem_wait_ld_regs(u[1]);
        tc_fence_before();
        mbar_arrive(s_free);  // the S columns may take block j + 1
#pragma unroll
        for (int c = 0; c < SMALL; ++c) {
          p[c] = fast_exp2(fmaf(__uint_as_float(u[c >> 5][c & 31]), sl2, -lse2));
          if (diagonal && k0 + c > q) p[c] = 0.f;
        }
      }
      uint32_t u[SMALL / 2];
      {
        ok = warp_wait(dp_full, j & 1, a.err, abort_flag);
        if (!ok) break;
        tc_fence_after();
        uint32_t v[2][32];
        tmem_ld_32x32b_x32(tmem + lane_off + Q_TM_DP + g * SMALL, v[0]);
        tmem_ld_32x32b_x32(tmem + lane_off + Q_TM_DP + g * SMALL + 32, v[1]);
        tmem_wait_ld_regs(v[0]);
        tmem_wait_ld_regs(v[1]);
        tc_fence_before();
        mbar_arrive(dp_free);  // the dP columns may take block j + 1
#pragma unroll
        for (int c = 0; c < SMALL; c += 2)
          u[c / 2] = pack_bf16x2(p[c] * (__uint_as_float(v[c >> 5][c & 31]) - dq),
                                 p[c + 1] * (__uint_as_float(v[(c + 1) >> 5][(c + 1) & 31]) - dq));
      }
      if (j > 0) {
        // dS of block j - 1 must have been read by its dQ product
        ok = warp_wait(ds_empty, (j - 1) & 1, a.err, abort_flag);
        if (!ok) break;
        tc_fence_after();
      }
      tmem_st_32x32b_x32(tmem + lane_off + Q_TM_DS + g * (SMALL / 2), u);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(ds_full);
    }
    if (ok) ok = warp_wait(acc_done, 0, a.err, abort_flag);
    tc_fence_after();
    // group g writes the column pairs (d, d + 64) for d in [32g, 32g + 32) of the dQ row
    __nv_bfloat16* dst = a.dqkv + ((long)q * a.batch + b) * 3L * a.heads * HD + q_col;
    store_tmem_pairs(tmem + lane_off + Q_TM_DQ, 32 * g, dst, a.scale, ok, a.cosv, a.sinv, q);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

__global__ void scale_kernel(const float* __restrict__ x, float* __restrict__ y, long n, float s) {
  const long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
  if (i < n) y[i] = x[i] * s;
}

bool qkv_map(CUtensorMap* m, const void* base, int S, int batch, long cols, uint32_t rows) {
  const uint64_t dims[3] = {(uint64_t)cols, (uint64_t)batch, (uint64_t)S};
  const uint64_t strides[2] = {(uint64_t)cols * 2, (uint64_t)cols * 2 * batch};
  const uint32_t box[3] = {64, 1, rows};
  return make_tmap_bf16_3d(m, base, dims, strides, box);
}

}  // namespace

cudaError_t flash_attn_bwd_tc(const __nv_bfloat16* dout, const __nv_bfloat16* qkv, const float* lse,
                              const float* dvec, __nv_bfloat16* dqkv, int S, int batch, int heads, int head_dim,
                              const float* cosv, const float* sinv, int* err, cudaStream_t stream) {
  if (head_dim != HD || S % BIG != 0) return cudaErrorInvalidValue;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(flash_bwd_dkdv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, KV_SMEM);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(flash_bwd_dq_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Q_SMEM);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  const long cols = 3L * heads * HD;
  CUtensorMap qkv_big, qkv_small, do_big, do_small;
  if (!qkv_map(&qkv_big, qkv, S, batch, cols, BIG) || !qkv_map(&qkv_small, qkv, S, batch, cols, SMALL) ||
      !qkv_map(&do_big, dout, S, batch, (long)heads * HD, BIG) ||
      !qkv_map(&do_small, dout, S, batch, (long)heads * HD, SMALL))
    return cudaErrorInvalidValue;
  // lse2 = lse * log2(e) is written into the second half of the dvec scratch
  // ([2][batch*heads*S] floats, allocated by the caller).
  const long rows = (long)batch * heads * S;
  float* lse2 = const_cast<float*>(dvec) + rows;
  scale_kernel<<<(int)((rows + 255) / 256), 256, 0, stream>>>(lse, lse2, rows, LOG2E);
  BwdArgs a{lse, lse2, dvec, dqkv, cosv, sinv, S, batch, heads, 1.0f / sqrtf((float)HD), err};
  dim3 grid_kv(batch * heads, S / BIG);
  flash_bwd_dkdv_kernel<<<grid_kv, KV_THREADS, KV_SMEM, stream>>>(qkv_big, qkv_small, do_small, a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  dim3 grid_q(batch * heads, S / BIG);
  flash_bwd_dq_tc_kernel<<<grid_q, Q_THREADS, Q_SMEM, stream>>>(qkv_big, do_big, a);
  return cudaGetLastError();
}

}  // namespace nmb
