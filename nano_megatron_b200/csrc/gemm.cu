// Persistent, warp-specialized bf16 GEMM on 5th-generation tensor cores (sm_100a).
// Reference ops: the torch matmuls of the linear layers and LM head
// (nano_megatron/tp_layers.py:58,82; model.py:192) and their autograd backward.
//
//   C[M,N] (op)= sum_k A(m,k) * B(k,n)      fp32 accumulation in TMEM
//
// Layout of one CTA (one per SM, 192 threads):
//   warp 0      TMA producer: loads 128x64 A and 256x64 B tiles (128-byte
//               swizzle) into a 4-stage shared-memory ring, one elected lane.
//   warp 1      MMA issuer: tcgen05.mma 128x256x16 per k-step into one of two
//               TMEM accumulators (2 x 256 columns), commits free the smem
//               stage and, at the end of a tile, hand the accumulator over.
//   warps 2-5   epilogue: tcgen05.ld the accumulator rows, convert, and stage
//               32-row boxes in 128-byte-swizzled shared memory (two 4 KB
//               buffers per warp), from which TMA stores them -- or, for the
//               fp32 accumulate mode, TMA-reduce-adds them into C, so the
//               read-modify-write happens in L2 instead of through the SMs;
//               overlaps the next tile's MMAs (double-buffered accumulator).
//
// Operand majorness is a template parameter, so one kernel covers the three
// products of a linear layer without transposing anything in memory:
//   forward  Y = X W        A = X [M,K] (K-major), B = W [K,N] (N-major)
//   dgrad    dX = dY W^T    A = dY (K-major),      B = W [N',K'] (K-major)
//   wgrad    dW += X^T dY   A = X  (M-major),      B = dY (N-major)
// Out-of-range rows/columns of a partial tile are zero-filled by TMA and
// masked in the epilogue. Requirements: 16-byte aligned bases and row strides
// (every dim multiple of 8 bf16 elements), N % 8 == 0.
//
// CTA-pair mode (PAIR, for the large products): a cluster of two CTAs works on
// one 256x256 tile with cta_group::2 MMAs. Each CTA stages 128 rows of A and
// 128 columns of B per k-block (32 KB instead of 48 KB, so six stages fit
// instead of four) with TMA loads whose bytes count on CTA 0's full barrier;
// CTA 0's MMA warp issues every MMA and its commits arrive on the barrier of
// both CTAs (free the stage, accumulator ready); each CTA's TMEM holds its 128
// rows of the accumulator and its epilogue writes them, then arrives on CTA
// 0's "accumulator free" barrier. No load uses cluster multicast.
//
// Split-K (accumulate mode only): when the output has too few tiles to fill
// the last wave of CTAs, each tile's K range is cut into `splits` pieces and
// every (piece, tile) pair is its own work unit; the fp32 reduce-add of the
// epilogue sums the pieces in L2. The weight gradients of a tensor-parallel
// rank are such outputs (at tp4 the attention-output gradient is 64 tiles).
//
// SwiGLU mode (OUT == 3, forward of the fused gate|up projection): B is the
// gate|up weight [K][2F]. A tile's four 64-column B boxes come from columns
// n0, n0+64 of the gate half and F+n0, F+n0+64 of the up half, so the 256
// accumulator columns of a row hold gate and up of the same 128 features.
// The epilogue rounds both to bf16 (the values the unfused path stores),
// writes a = bf16(bf16(silu(g)) * u) -- the arithmetic of swiglu_fwd_kernel --
// and, when the backward needs them, g and u through two [M][F] views of gu.
//
// Every mbarrier wait is bounded; a timeout records an error code in `err`
// and the kernel drains and returns instead of spinning forever.

#include <cuda.h>
#include <cuda_bf16.h>
#include <cstdlib>
#include <cuda_runtime.h>

#include "gemm.cuh"
#include "ptx.cuh"

namespace nmb {

namespace {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int A_TILE_BYTES = BM * BK * 2;  // 16 KB
constexpr int B_TILE_BYTES = BN * BK * 2;  // 32 KB
constexpr int STAGE_BYTES = A_TILE_BYTES + B_TILE_BYTES;
constexpr int STG_BUF = 4096;                 // one staged box: 32 rows x 128 B
constexpr int STAGING_BYTES = 4 * 2 * STG_BUF;  // two buffers per epilogue warp
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + STAGING_BYTES + 1024 /*align*/ + 256 /*barriers*/;
constexpr int THREADS = 192;
constexpr int GROUP_M = 16;
// CTA-pair mode: a 256x256 tile per pair; each CTA stages 128 rows of A and
// 128 columns of B (32 KB per k-block), so six stages fit where one CTA fits four.
constexpr int PAIR_STAGES = 6;
constexpr int PAIR_STAGE_BYTES = A_TILE_BYTES + B_TILE_BYTES / 2;
static_assert(PAIR_STAGES * PAIR_STAGE_BYTES == STAGES * STAGE_BYTES, "both modes use the same shared memory");

__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int& tm, int& tn) {
  const int span = GROUP_M * num_n;
  const int g = t / span;
  const int first = g * GROUP_M;
  const int size = min(num_m - first, GROUP_M);
  const int r = t - g * span;
  tm = first + r % size;
  tn = r / size;
}

template <bool A_MN, bool B_MN, int OUT, bool PAIR>
__global__ void __launch_bounds__(THREADS, 1)
gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                 const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmG,
                 const __grid_constant__ CUtensorMap tmU, int M, int N, int K, bool save_gu, int splits,
                 int* err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int ST = PAIR ? PAIR_STAGES : STAGES;            // ring depth
  constexpr int SB = PAIR ? PAIR_STAGE_BYTES : STAGE_BYTES;  // bytes per stage in this CTA
  constexpr int TM = PAIR ? 2 * BM : BM;                     // tile rows (per pair / per CTA)
  constexpr int BN_CTA = PAIR ? BN / 2 : BN;                 // B columns staged by this CTA
  uint8_t* staging = smem + ST * SB;
  uint64_t* full = reinterpret_cast<uint64_t*>(staging + STAGING_BYTES);
  uint64_t* empty = full + ST;
  uint64_t* tfull = empty + ST;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  constexpr bool SWIGLU = OUT == 3;
  const int F = N / 2;  // SwiGLU: features per half
  const int num_m = (M + TM - 1) / TM;
  const int num_n = SWIGLU ? (F + BN / 2 - 1) / (BN / 2) : (N + BN - 1) / BN;
  // the pair: CTA `rank` of cluster `first_unit`; units are scheduled per pair
  const int rank = PAIR ? (int)cluster_ctarank() : 0;
  const bool leader = rank == 0;
  const int first_unit = PAIR ? blockIdx.x / 2 : blockIdx.x;
  const int unit_stride = PAIR ? gridDim.x / 2 : gridDim.x;
  const int num_tiles = num_m * num_n;
  const int num_k = (K + BK - 1) / BK;
  // work unit u: tile u % num_tiles, K piece u / num_tiles (one piece unless split)
  const int num_units = num_tiles * splits;
  auto k_range = [&](int u, int& kb0, int& kb1) {
    const int piece = u / num_tiles;
    kb0 = (int)((long)num_k * piece / splits);
    kb1 = (int)((long)num_k * (piece + 1) / splits);
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      // pair: one arrival per epilogue warp of either CTA (on CTA 0's barrier)
      mbar_init(&tempty[b], PAIR ? 8 : 128);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    if (PAIR) {
      tmem_alloc_pair(tmem_slot, 512);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, 512);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (PAIR) cluster_sync();  // the peer's barriers exist before anything arrives on them
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    int stage = 0;
    uint32_t phase = 0;
    // A load of this CTA: a 64 x 64 box at (x, y), counted on this CTA's
    // full barrier, or on the pair leader's in pair mode
    auto load = [&](uint8_t* dst, const CUtensorMap* map, int s, int x, int y) {
      if (PAIR) tma_load_2d_pair(dst, map, &full[s], x, y);
      else tma_load_2d(dst, map, &full[s], x, y);
    };
    const int a_row0 = rank * BM;      // this CTA's rows within a tile
    const int b_col0 = rank * BN_CTA;  // this CTA's columns within a tile
    for (int u = first_unit; u < num_units && !*abort_flag; u += unit_stride) {
      int tm, tn, kb0, kb1;
      tile_coords(u % num_tiles, num_m, num_n, tm, tn);
      k_range(u, kb0, kb1);
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1, err)) { *abort_flag = 1; break; }
        uint8_t* a_dst = smem + stage * SB;
        uint8_t* b_dst = a_dst + A_TILE_BYTES;
        if (leader) mbar_arrive_expect_tx(&full[stage], PAIR ? 2 * SB : SB);  // both CTAs' halves
        const int k0 = kb * BK;
        const int arow = tm * TM + a_row0;
        if (A_MN) {
          // two 64(m) x 64(k) boxes
          load(a_dst, &tmA, stage, arow, k0);
          load(a_dst + 8192, &tmA, stage, arow + 64, k0);
        } else {
          load(a_dst, &tmA, stage, k0, arow);
        }
        if (SWIGLU) {
          // accumulator columns [0,128) = gate [n0, n0+128), [128,256) = up [F+n0, F+n0+128);
          // in pair mode CTA 0 stages the gate half and CTA 1 the up half
#pragma unroll
          for (int j = 0; j < BN_CTA / 64; ++j) {
            const int half = PAIR ? rank : (j >> 1);
            load(b_dst + j * 8192, &tmB, stage, half * F + tn * (BN / 2) + 64 * (j & 1), k0);
          }
        } else if (B_MN) {
#pragma unroll
          for (int j = 0; j < BN_CTA / 64; ++j) load(b_dst + j * 8192, &tmB, stage, tn * BN + b_col0 + 64 * j, k0);
        } else {
          load(b_dst, &tmB, stage, k0, tn * BN + b_col0);
        }
        if (++stage == ST) { stage = 0; phase ^= 1; }
      }
    }
  } else if (warp == 1 && lane == 0 && leader) {
    // ------------------------------------------------------------- MMA issue
    constexpr uint32_t idesc = idesc_bf16_f32(TM, BN, A_MN, B_MN);
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int u = first_unit; u < num_units && !*abort_flag; u += unit_stride) {
      if (!mbar_wait(&tempty[acc], acc_phase ^ 1, err)) { *abort_flag = 1; break; }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + acc * BN;
      int kb0, kb1;
      k_range(u, kb0, kb1);
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&full[stage], phase, err)) { *abort_flag = 1; break; }
        tc_fence_after();
        const uint32_t a_base = smem_u32(smem + stage * SB);
        const uint32_t b_base = a_base + A_TILE_BYTES;
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          // K-major: advance 32 bytes inside the 128-byte swizzle row.
          // MN-major: advance 16 k-rows of 128 bytes.
          const uint64_t a_desc = A_MN ? smem_desc_sw128(a_base + kk * 2048, 8192, 1024)
                                       : smem_desc_sw128(a_base + kk * 32, 0, 1024);
          const uint64_t b_desc = B_MN ? smem_desc_sw128(b_base + kk * 2048, 8192, 1024)
                                       : smem_desc_sw128(b_base + kk * 32, 0, 1024);
          if (PAIR) mma_bf16_ss_pair(d_tmem, a_desc, b_desc, idesc, (kb > kb0) || kk != 0);
          else mma_bf16_ss(d_tmem, a_desc, b_desc, idesc, (kb > kb0) || kk != 0);
        }
        if (PAIR) mma_commit_pair(&empty[stage]);  // frees the stage in both CTAs
        else mma_commit(&empty[stage]);
        if (++stage == ST) { stage = 0; phase ^= 1; }
      }
      if (PAIR) mma_commit_pair(&tfull[acc]);
      else mma_commit(&tfull[acc]);
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
    }
  } else if (warp >= 2) {
    // ------------------------------------------------------------- epilogue
    const int quarter = warp & 3;  // TMEM lanes [32*quarter, 32*quarter+32)
    uint8_t* stg = staging + quarter * 2 * STG_BUF;
    constexpr int CW = OUT == 0 ? 64 : 32;  // columns per staged box (128 B of a row)
    int nbox = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    // the accumulator of a tile is free again once every epilogue warp read it
    auto release_acc = [&](int b) {
      tc_fence_before();
      if (PAIR) {
        __syncwarp();
        if (lane == 0) mbar_arrive_leader(&tempty[b]);
      } else {
        mbar_arrive(&tempty[b]);
      }
    };
    for (int u = first_unit; u < num_units; u += unit_stride) {
      if (*abort_flag) break;
      int tm, tn;
      tile_coords(u % num_tiles, num_m, num_n, tm, tn);
      if (!mbar_wait(&tfull[acc], acc_phase, err)) { *abort_flag = 1; break; }
      tc_fence_after();
      const int row0 = tm * TM + rank * BM + quarter * 32;
      const uint32_t t_row = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN;
      if (SWIGLU) {
        // One box of a row = 64 bf16 (128 B) in the 128-byte swizzle: stage it
        // and TMA-store it to `map` at (col, row0) unless the box is past F.
        auto store_box = [&](const CUtensorMap* map, const float* v, int col) {
          uint8_t* buf = stg + (nbox & 1) * STG_BUF;
          if (lane == 0) bulk_wait_group_read<1>();
          __syncwarp();
          uint8_t* row = buf + lane * 128;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            uint4 u;
            u.x = pack_bf16x2(v[8 * j + 0], v[8 * j + 1]);
            u.y = pack_bf16x2(v[8 * j + 2], v[8 * j + 3]);
            u.z = pack_bf16x2(v[8 * j + 4], v[8 * j + 5]);
            u.w = pack_bf16x2(v[8 * j + 6], v[8 * j + 7]);
            *reinterpret_cast<uint4*>(row + ((j ^ (lane & 7)) << 4)) = u;
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            if (col < F && row0 < M) tma_store_2d(map, buf, col, row0);
            bulk_commit_group();
          }
          ++nbox;
        };
#pragma unroll 1
        for (int c = 0; c < BN / 2; c += 64) {
          uint32_t gr[64], ur[64];
          tmem_ld_32x32b_x32(t_row + c, *reinterpret_cast<uint32_t(*)[32]>(&gr[0]));
          tmem_ld_32x32b_x32(t_row + c + 32, *reinterpret_cast<uint32_t(*)[32]>(&gr[32]));
          tmem_ld_32x32b_x32(t_row + BN / 2 + c, *reinterpret_cast<uint32_t(*)[32]>(&ur[0]));
          tmem_ld_32x32b_x32(t_row + BN / 2 + c + 32, *reinterpret_cast<uint32_t(*)[32]>(&ur[32]));
          tmem_wait_ld_regs(*reinterpret_cast<uint32_t(*)[32]>(&gr[0]));
          tmem_wait_ld_regs(*reinterpret_cast<uint32_t(*)[32]>(&gr[32]));
          tmem_wait_ld_regs(*reinterpret_cast<uint32_t(*)[32]>(&ur[0]));
          tmem_wait_ld_regs(*reinterpret_cast<uint32_t(*)[32]>(&ur[32]));
          float g[64], u[64];
#pragma unroll
          for (int j = 0; j < 64; ++j) {
            g[j] = __bfloat162float(__float2bfloat16_rn(__uint_as_float(gr[j])));
            u[j] = __bfloat162float(__float2bfloat16_rn(__uint_as_float(ur[j])));
          }
          const int col = tn * (BN / 2) + c;
          if (save_gu) {
            store_box(&tmG, g, col);
            store_box(&tmU, u, col);
          }
#pragma unroll
          for (int j = 0; j < 64; ++j) {
            const float sl = g[j] / (1.f + __expf(-g[j]));
            g[j] = __bfloat162float(__float2bfloat16_rn(sl)) * u[j];
          }
          store_box(&tmC, g, col);
        }
        release_acc(acc);
        if (++acc == 2) { acc = 0; acc_phase ^= 1; }
        continue;
      }
#pragma unroll 1
      for (int c = 0; c < BN; c += CW) {
        uint32_t r[CW];
        tmem_ld_32x32b_x32(t_row + c, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
        if (OUT == 0) tmem_ld_32x32b_x32(t_row + c + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32 % CW]));
        tmem_wait_ld_regs(*reinterpret_cast<uint32_t(*)[32]>(&r[0]));
        if (OUT == 0) tmem_wait_ld_regs(*reinterpret_cast<uint32_t(*)[32]>(&r[32 % CW]));
        uint8_t* buf = stg + (nbox & 1) * STG_BUF;
        // the box stored from this buffer two boxes ago must have been read out
        if (lane == 0) bulk_wait_group_read<1>();
        __syncwarp();
        uint8_t* row = buf + lane * 128;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          uint4 u;
          if (OUT == 0) {
            u.x = pack_bf16x2(__uint_as_float(r[8 * j + 0]), __uint_as_float(r[8 * j + 1]));
            u.y = pack_bf16x2(__uint_as_float(r[8 * j + 2]), __uint_as_float(r[8 * j + 3]));
            u.z = pack_bf16x2(__uint_as_float(r[8 * j + 4]), __uint_as_float(r[8 * j + 5]));
            u.w = pack_bf16x2(__uint_as_float(r[8 * j + 6]), __uint_as_float(r[8 * j + 7]));
          } else {
            u = make_uint4(r[4 * j], r[4 * j + 1], r[4 * j + 2], r[4 * j + 3]);
          }
          *reinterpret_cast<uint4*>(row + ((j ^ (lane & 7)) << 4)) = u;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          const int col = tn * BN + c;
          if (col < N && row0 < M) {  // boxes past the edge are skipped; partial ones are clipped by TMA
            if (OUT == 2) tma_reduce_add_2d(&tmC, buf, col, row0);
            else tma_store_2d(&tmC, buf, col, row0);
          }
          bulk_commit_group();
        }
        ++nbox;
      }
      release_acc(acc);
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
    }
    // every store / reduce must be complete before the CTA (and its smem) goes
    if (lane == 0) bulk_wait_group<0>();
  }

  tc_fence_before();
  __syncthreads();
  if (PAIR) cluster_sync();  // the leader's last MMAs and commits into this CTA are done
  if (warp == 1) {
    tc_fence_after();
    if (PAIR) tmem_dealloc_pair(tmem_base, 512);
    else tmem_dealloc(tmem_base, 512);
  }
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (p == nullptr || q != cudaDriverEntryPointSuccess) return nullptr;
    fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// Pieces per tile for the accumulate mode: the smallest count (up to 8, at
// least 8 k-blocks per piece) whose last wave of work units is at least 90 %
// full, else the count with the fullest last wave.
int split_count(int tiles, int num_k, int sms) {
  int best = 1;
  double best_fill = 0.0;
  for (int s = 1; s <= 8 && (s == 1 || num_k / s >= 8); ++s) {
    const long units = (long)tiles * s;
    const long waves = (units + sms - 1) / sms;
    const double fill = (double)units / (double)(waves * sms);
    if (fill >= 0.9) return s;
    if (fill > best_fill + 1e-9) {
      best_fill = fill;
      best = s;
    }
  }
  return best;
}

template <bool A_MN, bool B_MN, int OUT, bool PAIR>
cudaError_t launch(const GemmArgs& g, cudaStream_t stream) {
  auto kernel = gemm_bf16_kernel<A_MN, B_MN, OUT, PAIR>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  constexpr int TM = PAIR ? 2 * BM : BM;
  constexpr int BN_CTA = PAIR ? BN / 2 : BN;
  CUtensorMap ta, tb;
  // A: K-major stored [M][K] (lda = row stride), or M-major stored [K][M].
  if (!make_tmap_bf16_2d(&ta, g.A, A_MN ? g.M : g.K, A_MN ? g.K : g.M, g.lda, 64, A_MN ? 64 : BM)) return cudaErrorInvalidValue;
  if (!make_tmap_bf16_2d(&tb, g.B, B_MN ? g.N : g.K, B_MN ? g.K : g.N, g.ldb, 64, B_MN ? 64 : BN_CTA))
    return cudaErrorInvalidValue;
  constexpr bool fp32_out = OUT == 1 || OUT == 2;
  const int out_cols = OUT == 3 ? g.N / 2 : g.N;
  const int tiles = ((g.M + TM - 1) / TM) * (OUT == 3 ? (out_cols + BN / 2 - 1) / (BN / 2) : (g.N + BN - 1) / BN);
  const int slots = PAIR ? g.num_sms / 2 : g.num_sms;  // concurrent work units
  const int splits = OUT == 2 ? split_count(tiles, (g.K + BK - 1) / BK, slots) : 1;
  const int units = tiles * splits;
  const int grid = (units < slots ? units : slots) * (PAIR ? 2 : 1);
  CUtensorMap tc, tg, tu;
  if (!make_tmap_out_2d(&tc, g.C, fp32_out, out_cols, g.M, g.ldc * (fp32_out ? 4 : 2), 32))
    return cudaErrorInvalidValue;
  tg = tu = tc;
  const bool save_gu = OUT == 3 && g.gu != nullptr;
  if (save_gu) {
    // gate and up halves of gu as two [M][F] views with row stride ldgu
    const __nv_bfloat16* gu = static_cast<const __nv_bfloat16*>(g.gu);
    if (!make_tmap_out_2d(&tg, gu, false, out_cols, g.M, g.ldgu * 2, 32) ||
        !make_tmap_out_2d(&tu, gu + out_cols, false, out_cols, g.M, g.ldgu * 2, 32))
      return cudaErrorInvalidValue;
  }
  if (!PAIR) {
    kernel<<<grid, THREADS, SMEM_BYTES, stream>>>(ta, tb, tc, tg, tu, g.M, g.N, g.K, save_gu, splits, g.err);
    return cudaGetLastError();
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(THREADS, 1, 1);
  cfg.dynamicSmemBytes = SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, ta, tb, tc, tg, tu, g.M, g.N, g.K, save_gu, splits, g.err);
}

// CTA pairs (one 256x256 tile per pair, six-stage rings) for the large
// products: measured 1513-1583 TFLOP/s against 1399-1451 with one CTA per tile
// at 8192 x {12288, 28672} x 4096 and 8192 x 4096 x 14336, and 7-18 % faster
// weight gradients there; at 8192 x 3072 x 4096 or K = 1024 the pair was
// slower (longer per-tile pipeline fill for the same number of waves).
// NMB_GEMM_PAIR=0 selects one CTA per tile everywhere.
bool use_pair(const GemmArgs& g) {
  static int enabled = -1;
  if (enabled < 0) {
    const char* v = getenv("NMB_GEMM_PAIR");
    enabled = (v != nullptr && v[0] == '0') ? 0 : 1;
  }
  return enabled == 1 && g.M >= 2048 && g.N >= 4096 && g.K >= 2048 && g.num_sms >= 2;
}

template <bool A_MN, bool B_MN, int OUT>
cudaError_t launch_any(const GemmArgs& g, cudaStream_t stream) {
  return use_pair(g) ? launch<A_MN, B_MN, OUT, true>(g, stream) : launch<A_MN, B_MN, OUT, false>(g, stream);
}

}  // namespace

bool make_tmap_bf16_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_elems,
                       uint32_t box_inner, uint32_t box_outer) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_elems * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool make_tmap_out_2d(CUtensorMap* map, const void* base, bool fp32, uint64_t inner, uint64_t outer,
                      uint64_t row_stride_bytes, uint32_t box_outer) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {fp32 ? 32u : 64u, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, fp32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                  const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool make_tmap_bf16_3d(CUtensorMap* map, const void* base, const uint64_t dims[3], const uint64_t strides_bytes[2],
                       const uint32_t box[3]) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  cuuint64_t d[3] = {dims[0], dims[1], dims[2]};
  cuuint64_t st[2] = {strides_bytes[0], strides_bytes[1]};
  cuuint32_t bx[3] = {box[0], box[1], box[2]};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), d, st, bx, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

cudaError_t gemm_bf16(const GemmArgs& g, cudaStream_t stream) {
  if (g.M <= 0 || g.N <= 0 || g.K <= 0) return cudaSuccess;
  if (!g.a_mn && g.b_mn && g.out == OutMode::kBf16) return launch_any<false, true, 0>(g, stream);
  if (!g.a_mn && g.b_mn && g.out == OutMode::kF32) return launch_any<false, true, 1>(g, stream);
  if (!g.a_mn && !g.b_mn && g.out == OutMode::kBf16) return launch_any<false, false, 0>(g, stream);
  if (!g.a_mn && !g.b_mn && g.out == OutMode::kF32) return launch_any<false, false, 1>(g, stream);
  if (g.a_mn && g.b_mn && g.out == OutMode::kF32Accumulate) return launch_any<true, true, 2>(g, stream);
  if (g.a_mn && g.b_mn && g.out == OutMode::kF32) return launch_any<true, true, 1>(g, stream);
  if (!g.a_mn && !g.b_mn && g.out == OutMode::kF32Accumulate) return launch_any<false, false, 2>(g, stream);
  if (!g.a_mn && g.b_mn && g.out == OutMode::kF32Accumulate) return launch_any<false, true, 2>(g, stream);
  if (!g.a_mn && g.b_mn && g.out == OutMode::kSwiGLU) {
    if (g.N % 16 != 0) return cudaErrorInvalidValue;  // F % 8 == 0: 16-byte aligned up half
    return launch_any<false, true, 3>(g, stream);
  }
  return cudaErrorInvalidValue;
}

}  // namespace nmb
