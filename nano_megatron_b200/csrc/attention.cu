// Causal flash attention, forward and backward, head_dim 128 (bf16, fp32 math),
// reading q/k/v straight out of the fused QKV GEMM output.
//
// Layout: qkv is [T, 3*H*D] with token row t = s*batch + b (sequence-first),
// q of head h at columns [h*D, (h+1)*D), k at H*D + h*D, v at 2*H*D + h*D.
// o is [T, H*D]; lse is [batch*H, S] (natural log, of the scaled scores).
//
// Forward (one CTA = 64 query rows of one (batch, head), 4 warps x 16 rows):
//   S = Q K^T for 64-key blocks with mma.sync m16n8k16, online softmax in
//   registers, O += P V with P re-used from the S accumulators; K/V tiles are
//   double-buffered with cp.async into XOR-swizzled shared memory; key blocks
//   above the diagonal are skipped, the diagonal block is masked.
// Backward (one CTA = 64 keys, loops over the query blocks at or below it):
//   S^T = K Q^T, P^T = exp(S^T - lse), dV += P^T dO, dP^T = V dO^T,
//   dS^T = P^T (dP^T - D), dK += dS^T Q, dQ += dS K (fp32 vector atomics into
//   a [batch*H, S, D] accumulator), then a small kernel scales dQ into dqkv.
//   D = rowsum(dO * O) comes from a preprocessing kernel.
//
// This is the mma.sync path: it runs on the tensor cores of every sm_80+ GPU,
// sm_100a included, but not at tcgen05 throughput.
//
// Reference op: the causal F.scaled_dot_product_attention of
// nano_megatron/model.py:126 and its autograd backward.

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cfloat>

#include "attention.cuh"
#include "ptx.cuh"

namespace nmb {

namespace {

constexpr int D = 128;       // head dim
constexpr int BR = 64;       // query rows per forward CTA
constexpr int BC = 64;       // keys per block
constexpr int WARPS = 4;
constexpr int THREADS = WARPS * 32;
constexpr int TILE_BYTES = 64 * D * 2;  // 16 KB: 64 rows x 128 bf16

// ----------------------------------------------------------------- helpers
__device__ __forceinline__ uint32_t swz(int row, int col) {
  // byte offset of element (row, col) in a [64][128] bf16 tile, 16 B chunks XOR (row % 8)
  return row * 256 + ((((col >> 3) ^ (row & 7))) << 4) + ((col & 7) << 1);
}

__device__ __forceinline__ uint32_t swz64(int row, int col) {
  // [64][64] bf16 tile (128 B rows)
  return row * 128 + ((((col >> 3) ^ (row & 7))) << 4) + ((col & 7) << 1);
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Copy a 64 x 128 bf16 tile (row stride `ld` elements) into swizzled smem.
__device__ __forceinline__ void load_tile_async(uint32_t smem, const __nv_bfloat16* g, long ld, int tid) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int chunk = tid + i * THREADS;  // 1024 chunks of 16 B
    const int row = chunk >> 4, c = (chunk & 15) << 3;
    cp_async16(smem + swz(row, c), g + row * ld + c);
  }
}

// A fragments (16 rows x 16 k) of a row-major [rows][128] swizzled tile.
__device__ __forceinline__ void ld_a_frag(uint32_t tile, int m0, int k0, int lane, uint32_t (&a)[4]) {
  const int mi = lane >> 3;
  const int row = m0 + ((mi & 1) << 3) + (lane & 7);
  const int col = k0 + ((mi >> 1) << 3);
  ldsm_x4(tile + swz(row, col), a[0], a[1], a[2], a[3]);
}

// B fragments for two k-steps of B[k][n] = T[n][k] (T row-major, "col-major B"):
// returns (b0,b1) of k-step k0 and of k-step k0+16 for the n-tile at n0.
__device__ __forceinline__ void ld_b_nk(uint32_t tile, int n0, int k0, int lane, uint32_t (&b)[4]) {
  const int mi = lane >> 3;
  ldsm_x4(tile + swz(n0 + (lane & 7), k0 + (mi << 3)), b[0], b[1], b[2], b[3]);
}

// B fragments for B[k][n] = T[k][n] (T row-major over k): one k-step (16 rows
// at k0) for two n-tiles (n0, n0+8).
__device__ __forceinline__ void ld_b_kn(uint32_t tile, int k0, int n0, int lane, uint32_t (&b)[4]) {
  const int mi = lane >> 3;
  const int row = k0 + ((mi & 1) << 3) + (lane & 7);
  const int col = n0 + ((mi >> 1) << 3);
  ldsm_x4_t(tile + swz(row, col), b[0], b[1], b[2], b[3]);
}

__device__ __forceinline__ uint32_t pack2(float a, float b) { return pack_bf16x2(a, b); }

// ============================================================== forward
__global__ void __launch_bounds__(THREADS, 2)
flash_fwd_kernel(const __nv_bfloat16* __restrict__ qkv, __nv_bfloat16* __restrict__ out, float* __restrict__ lse,
                 int S, int batch, int heads, float scale_log2) {
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sK[2] = {sQ + TILE_BYTES, sQ + 2 * TILE_BYTES};
  const uint32_t sV[2] = {sQ + 3 * TILE_BYTES, sQ + 4 * TILE_BYTES};

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nqb = S / BR;
  const int qb = nqb - 1 - blockIdx.x;  // longest rows first
  const int bh = blockIdx.y;
  const int b = bh / heads, h = bh % heads;
  const long ld = 3L * heads * D;
  const long row_step = (long)batch * ld;  // stride between consecutive positions
  const __nv_bfloat16* qg = qkv + ((long)qb * BR * batch + b) * ld + h * D;
  const __nv_bfloat16* kg = qkv + (long)b * ld + heads * D + h * D;
  const __nv_bfloat16* vg = kg + heads * D;

  load_tile_async(sQ, qg, row_step, tid);
  load_tile_async(sK[0], kg, row_step, tid);
  load_tile_async(sV[0], vg, row_step, tid);
  cp_async_commit();

  uint32_t qf[8][4];
  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -FLT_MAX, m1 = -FLT_MAX, l0 = 0.f, l1 = 0.f;

  const int nkb = qb + 1;
  for (int kb = 0; kb < nkb; ++kb) {
    const int buf = kb & 1;
    if (kb + 1 < nkb) {
      load_tile_async(sK[buf ^ 1], kg + (long)(kb + 1) * BC * row_step, row_step, tid);
      load_tile_async(sV[buf ^ 1], vg + (long)(kb + 1) * BC * row_step, row_step, tid);
    }
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (kb == 0) {
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) ld_a_frag(sQ, warp * 16, ks * 16, lane, qf[ks]);
    }
    // S = Q K^T  (16 rows x 64 keys per warp)
    float s[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int ks = 0; ks < 8; ks += 2) {
        uint32_t bb[4];
        ld_b_nk(sK[buf], nt * 8, ks * 16, lane, bb);
        mma16816(s[nt], qf[ks], bb[0], bb[1]);
        mma16816(s[nt], qf[ks + 1], bb[2], bb[3]);
      }
    }
    // causal mask on the diagonal block
    const int qrow0 = qb * BR + warp * 16 + (lane >> 2);
    if (kb == qb) {
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const int key = kb * BC + nt * 8 + 2 * (lane & 3);
        if (key > qrow0) s[nt][0] = -FLT_MAX;
        if (key + 1 > qrow0) s[nt][1] = -FLT_MAX;
        if (key > qrow0 + 8) s[nt][2] = -FLT_MAX;
        if (key + 1 > qrow0 + 8) s[nt][3] = -FLT_MAX;
      }
    }
    // online softmax (rows r0 = lane/4, r1 = r0 + 8 of the warp's 16)
    float mx0 = m0, mx1 = m1;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      mx0 = fmaxf(mx0, fmaxf(s[nt][0], s[nt][1]));
      mx1 = fmaxf(mx1, fmaxf(s[nt][2], s[nt][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float c0 = exp2f((m0 - mx0) * scale_log2), c1 = exp2f((m1 - mx1) * scale_log2);
    m0 = mx0;
    m1 = mx1;
    const float ms0 = mx0 * scale_log2, ms1 = mx1 * scale_log2;
    float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      s[nt][0] = exp2f(s[nt][0] * scale_log2 - ms0);
      s[nt][1] = exp2f(s[nt][1] * scale_log2 - ms0);
      s[nt][2] = exp2f(s[nt][2] * scale_log2 - ms1);
      s[nt][3] = exp2f(s[nt][3] * scale_log2 - ms1);
      rs0 += s[nt][0] + s[nt][1];
      rs1 += s[nt][2] + s[nt][3];
    }
    l0 = l0 * c0 + rs0;
    l1 = l1 * c1 + rs1;
#pragma unroll
    for (int dt = 0; dt < 16; ++dt) {
      o[dt][0] *= c0; o[dt][1] *= c0; o[dt][2] *= c1; o[dt][3] *= c1;
    }
    // O += P V
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      uint32_t pa[4] = {pack2(s[2 * ks][0], s[2 * ks][1]), pack2(s[2 * ks][2], s[2 * ks][3]),
                        pack2(s[2 * ks + 1][0], s[2 * ks + 1][1]), pack2(s[2 * ks + 1][2], s[2 * ks + 1][3])};
#pragma unroll
      for (int dt = 0; dt < 16; dt += 2) {
        uint32_t bb[4];
        ld_b_kn(sV[buf], ks * 16, dt * 8, lane, bb);
        mma16816(o[dt], pa, bb[0], bb[1]);
        mma16816(o[dt + 1], pa, bb[2], bb[3]);
      }
    }
    __syncthreads();
  }
  // finalize
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float inv0 = 1.f / l0, inv1 = 1.f / l1;
  const int r0 = qb * BR + warp * 16 + (lane >> 2);
  const long ldo = (long)heads * D;
  __nv_bfloat16* o0 = out + ((long)r0 * batch + b) * ldo + h * D;
  __nv_bfloat16* o1 = out + ((long)(r0 + 8) * batch + b) * ldo + h * D;
#pragma unroll
  for (int dt = 0; dt < 16; ++dt) {
    const int c = dt * 8 + 2 * (lane & 3);
    *reinterpret_cast<uint32_t*>(o0 + c) = pack2(o[dt][0] * inv0, o[dt][1] * inv0);
    *reinterpret_cast<uint32_t*>(o1 + c) = pack2(o[dt][2] * inv1, o[dt][3] * inv1);
  }
  if ((lane & 3) == 0) {
    const float ln2 = 0.6931471805599453f;
    lse[(long)bh * S + r0] = (m0 * scale_log2 + log2f(l0)) * ln2;
    lse[(long)bh * S + r0 + 8] = (m1 * scale_log2 + log2f(l1)) * ln2;
  }
}

// ================================================================ backward
// D[bh, s] = sum_d dO * O
__global__ void flash_bwd_dot_kernel(const __nv_bfloat16* __restrict__ dout, const __nv_bfloat16* __restrict__ out,
                                     float* __restrict__ dvec, int S, int batch, int heads) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long idx = (long)blockIdx.x * (blockDim.x >> 5) + warp;  // (bh, s)
  if (idx >= (long)batch * heads * S) return;
  const int bh = idx / S, s = idx % S;
  const int b = bh / heads, h = bh % heads;
  const long off = ((long)s * batch + b) * heads * D + h * D + lane * 4;
  const uint2 x = *reinterpret_cast<const uint2*>(dout + off);
  const uint2 y = *reinterpret_cast<const uint2*>(out + off);
  const float2 x0 = unpack_bf16x2(x.x), x1 = unpack_bf16x2(x.y), y0 = unpack_bf16x2(y.x), y1 = unpack_bf16x2(y.y);
  float v = x0.x * y0.x + x0.y * y0.y + x1.x * y1.x + x1.y * y1.y;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if (lane == 0) dvec[idx] = v;
}

__global__ void __launch_bounds__(THREADS, 2)
flash_bwd_kernel(const __nv_bfloat16* __restrict__ qkv, const __nv_bfloat16* __restrict__ dout,
                 const float* __restrict__ lse, const float* __restrict__ dvec, float* __restrict__ dq_acc,
                 __nv_bfloat16* __restrict__ dqkv, int S, int batch, int heads, float scale) {
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sK = smem_u32(smem);
  const uint32_t sV = sK + TILE_BYTES;
  const uint32_t sQ[2] = {sK + 2 * TILE_BYTES, sK + 3 * TILE_BYTES};
  const uint32_t sdO[2] = {sK + 4 * TILE_BYTES, sK + 5 * TILE_BYTES};
  const uint32_t sdS = sK + 6 * TILE_BYTES;  // [64 keys][64 q] bf16 = 8 KB
  float* sL = reinterpret_cast<float*>(smem + 6 * TILE_BYTES + 8192);  // [2][64] lse
  float* sD = sL + 128;                                                // [2][64] D

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int kb = blockIdx.x;  // key block; low indices have the most work
  const int bh = blockIdx.y;
  const int b = bh / heads, h = bh % heads;
  const int nqb = S / BR;
  const long ld = 3L * heads * D;
  const long row_step = (long)batch * ld;
  const long ldo = (long)heads * D;
  const long do_step = (long)batch * ldo;
  const __nv_bfloat16* qg = qkv + (long)b * ld + h * D;
  const __nv_bfloat16* kg = qg + heads * D;
  const __nv_bfloat16* vg = kg + heads * D;
  const __nv_bfloat16* dog = dout + (long)b * ldo + h * D;
  const float scale_log2 = scale * 1.4426950408889634f;

  load_tile_async(sK, kg + (long)kb * BC * row_step, row_step, tid);
  load_tile_async(sV, vg + (long)kb * BC * row_step, row_step, tid);
  load_tile_async(sQ[0], qg + (long)kb * BR * row_step, row_step, tid);
  load_tile_async(sdO[0], dog + (long)kb * BR * do_step, do_step, tid);
  if (tid < 64) {
    sL[tid] = lse[(long)bh * S + kb * BR + tid];
    sD[tid] = dvec[(long)bh * S + kb * BR + tid];
  }
  cp_async_commit();

  float dk[16][4], dv[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    dk[i][0] = dk[i][1] = dk[i][2] = dk[i][3] = 0.f;
    dv[i][0] = dv[i][1] = dv[i][2] = dv[i][3] = 0.f;
  }
  const int key0 = kb * BC + warp * 16 + (lane >> 2);  // this thread's rows: key0, key0 + 8

  for (int qb = kb; qb < nqb; ++qb) {
    const int buf = (qb - kb) & 1;
    if (qb + 1 < nqb) {
      load_tile_async(sQ[buf ^ 1], qg + (long)(qb + 1) * BR * row_step, row_step, tid);
      load_tile_async(sdO[buf ^ 1], dog + (long)(qb + 1) * BR * do_step, do_step, tid);
      if (tid < 64) {
        sL[(buf ^ 1) * 64 + tid] = lse[(long)bh * S + (qb + 1) * BR + tid];
        sD[(buf ^ 1) * 64 + tid] = dvec[(long)bh * S + (qb + 1) * BR + tid];
      }
    }
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const float* L = sL + buf * 64;
    const float* Dv = sD + buf * 64;

    // S^T = K Q^T  (16 keys x 64 queries per warp)
    float st[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) st[nt][0] = st[nt][1] = st[nt][2] = st[nt][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ks += 2) {
      uint32_t ka[4], kc[4];
      ld_a_frag(sK, warp * 16, ks * 16, lane, ka);
      ld_a_frag(sK, warp * 16, ks * 16 + 16, lane, kc);
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        uint32_t bb[4];
        ld_b_nk(sQ[buf], nt * 8, ks * 16, lane, bb);
        mma16816(st[nt], ka, bb[0], bb[1]);
        mma16816(st[nt], kc, bb[2], bb[3]);
      }
    }
    // P^T = exp(S^T * scale - lse[q]), causal: key > q -> 0
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const int ql = nt * 8 + 2 * (lane & 3);
      const int q = qb * BR + ql;
      const float L0 = L[ql] * 1.4426950408889634f, L1 = L[ql + 1] * 1.4426950408889634f;
      st[nt][0] = (key0 > q) ? 0.f : exp2f(st[nt][0] * scale_log2 - L0);
      st[nt][1] = (key0 > q + 1) ? 0.f : exp2f(st[nt][1] * scale_log2 - L1);
      st[nt][2] = (key0 + 8 > q) ? 0.f : exp2f(st[nt][2] * scale_log2 - L0);
      st[nt][3] = (key0 + 8 > q + 1) ? 0.f : exp2f(st[nt][3] * scale_log2 - L1);
    }
    // dV += P^T dO
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      uint32_t pa[4] = {pack2(st[2 * ks][0], st[2 * ks][1]), pack2(st[2 * ks][2], st[2 * ks][3]),
                        pack2(st[2 * ks + 1][0], st[2 * ks + 1][1]), pack2(st[2 * ks + 1][2], st[2 * ks + 1][3])};
#pragma unroll
      for (int dt = 0; dt < 16; dt += 2) {
        uint32_t bb[4];
        ld_b_kn(sdO[buf], ks * 16, dt * 8, lane, bb);
        mma16816(dv[dt], pa, bb[0], bb[1]);
        mma16816(dv[dt + 1], pa, bb[2], bb[3]);
      }
    }
    // dP^T = V dO^T
    float dp[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) dp[nt][0] = dp[nt][1] = dp[nt][2] = dp[nt][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ks += 2) {
      uint32_t va[4], vc[4];
      ld_a_frag(sV, warp * 16, ks * 16, lane, va);
      ld_a_frag(sV, warp * 16, ks * 16 + 16, lane, vc);
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        uint32_t bb[4];
        ld_b_nk(sdO[buf], nt * 8, ks * 16, lane, bb);
        mma16816(dp[nt], va, bb[0], bb[1]);
        mma16816(dp[nt], vc, bb[2], bb[3]);
      }
    }
    // dS^T = P^T (dP^T - D[q])
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const int ql = nt * 8 + 2 * (lane & 3);
      dp[nt][0] = st[nt][0] * (dp[nt][0] - Dv[ql]);
      dp[nt][1] = st[nt][1] * (dp[nt][1] - Dv[ql + 1]);
      dp[nt][2] = st[nt][2] * (dp[nt][2] - Dv[ql]);
      dp[nt][3] = st[nt][3] * (dp[nt][3] - Dv[ql + 1]);
    }
    // dK += dS^T Q ; stash dS^T for the dQ product
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      uint32_t pa[4] = {pack2(dp[2 * ks][0], dp[2 * ks][1]), pack2(dp[2 * ks][2], dp[2 * ks][3]),
                        pack2(dp[2 * ks + 1][0], dp[2 * ks + 1][1]), pack2(dp[2 * ks + 1][2], dp[2 * ks + 1][3])};
      const int kr = warp * 16 + (lane >> 2);
      const int qc = ks * 16 + 2 * (lane & 3);
      asm volatile("st.shared.b32 [%0], %1;" ::"r"(sdS + swz64(kr, qc)), "r"(pa[0]));
      asm volatile("st.shared.b32 [%0], %1;" ::"r"(sdS + swz64(kr + 8, qc)), "r"(pa[1]));
      asm volatile("st.shared.b32 [%0], %1;" ::"r"(sdS + swz64(kr, qc + 8)), "r"(pa[2]));
      asm volatile("st.shared.b32 [%0], %1;" ::"r"(sdS + swz64(kr + 8, qc + 8)), "r"(pa[3]));
#pragma unroll
      for (int dt = 0; dt < 16; dt += 2) {
        uint32_t bb[4];
        ld_b_kn(sQ[buf], ks * 16, dt * 8, lane, bb);
        mma16816(dk[dt], pa, bb[0], bb[1]);
        mma16816(dk[dt + 1], pa, bb[2], bb[3]);
      }
    }
    __syncthreads();
    // dQ[q rows of this warp] += dS K  (dS read transposed from the stash)
    {
      float dqa[16][4];
#pragma unroll
      for (int i = 0; i < 16; ++i) dqa[i][0] = dqa[i][1] = dqa[i][2] = dqa[i][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        uint32_t a[4];
        const int mi = lane >> 3;
        const int key = ks * 16 + ((mi >> 1) << 3) + (lane & 7);
        const int qc = warp * 16 + ((mi & 1) << 3);
        ldsm_x4_t(sdS + swz64(key, qc), a[0], a[1], a[2], a[3]);
#pragma unroll
        for (int dt = 0; dt < 16; dt += 2) {
          uint32_t bb[4];
          ld_b_kn(sK, ks * 16, dt * 8, lane, bb);
          mma16816(dqa[dt], a, bb[0], bb[1]);
          mma16816(dqa[dt + 1], a, bb[2], bb[3]);
        }
      }
      const int q0 = qb * BR + warp * 16 + (lane >> 2);
      float* base0 = dq_acc + ((long)bh * S + q0) * D;
      float* base1 = base0 + 8L * D;
#pragma unroll
      for (int dt = 0; dt < 16; ++dt) {
        const int c = dt * 8 + 2 * (lane & 3);
        atomicAdd(reinterpret_cast<float2*>(base0 + c), make_float2(dqa[dt][0], dqa[dt][1]));
        atomicAdd(reinterpret_cast<float2*>(base1 + c), make_float2(dqa[dt][2], dqa[dt][3]));
      }
    }
    __syncthreads();
  }
  // write dK (scaled) and dV into the k / v sections of dqkv
  const long rk0 = (long)key0 * batch + b, rk1 = (long)(key0 + 8) * batch + b;
  __nv_bfloat16* dk0 = dqkv + rk0 * ld + heads * D + h * D;
  __nv_bfloat16* dk1 = dqkv + rk1 * ld + heads * D + h * D;
#pragma unroll
  for (int dt = 0; dt < 16; ++dt) {
    const int c = dt * 8 + 2 * (lane & 3);
    *reinterpret_cast<uint32_t*>(dk0 + c) = pack2(dk[dt][0] * scale, dk[dt][1] * scale);
    *reinterpret_cast<uint32_t*>(dk1 + c) = pack2(dk[dt][2] * scale, dk[dt][3] * scale);
    *reinterpret_cast<uint32_t*>(dk0 + heads * D + c) = pack2(dv[dt][0], dv[dt][1]);
    *reinterpret_cast<uint32_t*>(dk1 + heads * D + c) = pack2(dv[dt][2], dv[dt][3]);
  }
}

// dq (bf16, into dqkv's q section) = scale * dq_acc
__global__ void flash_bwd_dq_kernel(const float* __restrict__ dq_acc, __nv_bfloat16* __restrict__ dqkv, int S,
                                    int batch, int heads, float scale) {
  const long total = (long)batch * heads * S * (D / 8);
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const long row = i / (D / 8);  // (bh, s)
    const int c = (int)(i % (D / 8)) * 8;
    const int bh = row / S, s = row % S;
    const int b = bh / heads, h = bh % heads;
    const float4 x = *reinterpret_cast<const float4*>(dq_acc + row * D + c);
    const float4 y = *reinterpret_cast<const float4*>(dq_acc + row * D + c + 4);
    uint4 u;
    u.x = pack_bf16x2(x.x * scale, x.y * scale);
    u.y = pack_bf16x2(x.z * scale, x.w * scale);
    u.z = pack_bf16x2(y.x * scale, y.y * scale);
    u.w = pack_bf16x2(y.z * scale, y.w * scale);
    *reinterpret_cast<uint4*>(dqkv + ((long)s * batch + b) * 3L * heads * D + h * D + c) = u;
  }
}

constexpr int FWD_SMEM = 5 * TILE_BYTES;
constexpr int BWD_SMEM = 6 * TILE_BYTES + 8192 + 4 * 64 * 4;

}  // namespace

cudaError_t flash_attn_fwd(const __nv_bfloat16* qkv, __nv_bfloat16* out, float* lse, int S, int batch, int heads,
                           int head_dim, cudaStream_t stream) {
  if (head_dim != D || S % BR != 0) return cudaErrorInvalidValue;
  static bool configured = false;
  if (!configured) {
    cudaFuncSetAttribute(flash_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, FWD_SMEM);
    configured = true;
  }
  const float scale_log2 = (1.0f / sqrtf((float)D)) * 1.4426950408889634f;
  dim3 grid(S / BR, batch * heads);
  flash_fwd_kernel<<<grid, THREADS, FWD_SMEM, stream>>>(qkv, out, lse, S, batch, heads, scale_log2);
  return cudaGetLastError();
}

cudaError_t flash_attn_bwd_dot(const __nv_bfloat16* dout, const __nv_bfloat16* out, float* dvec, int S, int batch,
                               int heads, cudaStream_t stream) {
  const long rows = (long)batch * heads * S;
  flash_bwd_dot_kernel<<<(rows + 7) / 8, 256, 0, stream>>>(dout, out, dvec, S, batch, heads);
  return cudaGetLastError();
}

cudaError_t flash_attn_bwd(const __nv_bfloat16* dout, const __nv_bfloat16* qkv, const __nv_bfloat16* out,
                           const float* lse, float* dvec, float* dq_acc, __nv_bfloat16* dqkv, int S, int batch,
                           int heads, int head_dim, cudaStream_t stream) {
  if (head_dim != D || S % BR != 0) return cudaErrorInvalidValue;
  static bool configured = false;
  if (!configured) {
    cudaFuncSetAttribute(flash_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, BWD_SMEM);
    configured = true;
  }
  const long rows = (long)batch * heads * S;
  flash_bwd_dot_kernel<<<(rows + 7) / 8, 256, 0, stream>>>(dout, out, dvec, S, batch, heads);
  cudaError_t e = cudaMemsetAsync(dq_acc, 0, rows * D * sizeof(float), stream);
  if (e != cudaSuccess) return e;
  const float scale = 1.0f / sqrtf((float)D);
  dim3 grid(S / BC, batch * heads);
  flash_bwd_kernel<<<grid, THREADS, BWD_SMEM, stream>>>(qkv, dout, lse, dvec, dq_acc, dqkv, S, batch, heads, scale);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const long work = rows * (D / 8);
  const int blocks = (int)((work + 255) / 256 < 148 * 16 ? (work + 255) / 256 : 148 * 16);
  flash_bwd_dq_kernel<<<blocks, 256, 0, stream>>>(dq_acc, dqkv, S, batch, heads, scale);
  return cudaGetLastError();
}

}  // namespace nmb
