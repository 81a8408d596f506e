// Persistent, warp-specialized bf16 GEMM on 5th-generation tensor cores (sm_100a).
//
//   C[M,N] (op)= sum_k A(m,k) * B(k,n)      fp32 accumulation in TMEM
//
// Layout of one CTA (one per SM, 192 threads):
//   warp 0      TMA producer: loads 128x64 A and 256x64 B tiles (128-byte
//               swizzle) into a 4-stage shared-memory ring, one elected lane.
//   warp 1      MMA issuer: tcgen05.mma 128x256x16 per k-step into one of two
//               TMEM accumulators (2 x 256 columns), commits free the smem
//               stage and, at the end of a tile, hand the accumulator over.
//   warps 2-5   epilogue: tcgen05.ld 32 columns at a time, convert, store;
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
// Every mbarrier wait is bounded; a timeout records an error code in `err`
// and the kernel drains and returns instead of spinning forever.

#include <cuda.h>
#include <cuda_runtime.h>

#include "gemm.cuh"
#include "ptx.cuh"

namespace nmb {

namespace {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int A_TILE_BYTES = BM * BK * 2;  // 16 KB
constexpr int B_TILE_BYTES = BN * BK * 2;  // 32 KB
constexpr int STAGE_BYTES = A_TILE_BYTES + B_TILE_BYTES;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
constexpr int THREADS = 192;
constexpr int GROUP_M = 16;

__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int& tm, int& tn) {
  const int span = GROUP_M * num_n;
  const int g = t / span;
  const int first = g * GROUP_M;
  const int size = min(num_m - first, GROUP_M);
  const int r = t - g * span;
  tm = first + r % size;
  tn = r / size;
}

template <bool A_MN, bool B_MN, int OUT>
__global__ void __launch_bounds__(THREADS, 1)
gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, void* C,
                 long ldc, int M, int N, int K, int* err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int num_m = (M + BM - 1) / BM;
  const int num_n = (N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int num_k = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 128);
    }
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
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    int stage = 0;
    uint32_t phase = 0;
    for (int t = blockIdx.x; t < num_tiles && !*abort_flag; t += gridDim.x) {
      int tm, tn;
      tile_coords(t, num_m, num_n, tm, tn);
      for (int kb = 0; kb < num_k; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1, err)) { *abort_flag = 1; break; }
        uint8_t* a_dst = smem + stage * STAGE_BYTES;
        uint8_t* b_dst = a_dst + A_TILE_BYTES;
        mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
        const int k0 = kb * BK;
        if (A_MN) {
          // two 64(m) x 64(k) boxes
          tma_load_2d(a_dst, &tmA, &full[stage], tm * BM, k0);
          tma_load_2d(a_dst + 8192, &tmA, &full[stage], tm * BM + 64, k0);
        } else {
          tma_load_2d(a_dst, &tmA, &full[stage], k0, tm * BM);
        }
        if (B_MN) {
#pragma unroll
          for (int j = 0; j < 4; ++j) tma_load_2d(b_dst + j * 8192, &tmB, &full[stage], tn * BN + 64 * j, k0);
        } else {
          tma_load_2d(b_dst, &tmB, &full[stage], k0, tn * BN);
        }
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------- MMA issue
    constexpr uint32_t idesc = idesc_bf16_f32(BM, BN, A_MN, B_MN);
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < num_tiles && !*abort_flag; t += gridDim.x) {
      if (!mbar_wait(&tempty[acc], acc_phase ^ 1, err)) { *abort_flag = 1; break; }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + acc * BN;
      for (int kb = 0; kb < num_k; ++kb) {
        if (!mbar_wait(&full[stage], phase, err)) { *abort_flag = 1; break; }
        tc_fence_after();
        const uint32_t a_base = smem_u32(smem + stage * STAGE_BYTES);
        const uint32_t b_base = a_base + A_TILE_BYTES;
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          // K-major: advance 32 bytes inside the 128-byte swizzle row.
          // MN-major: advance 16 k-rows of 128 bytes.
          const uint64_t a_desc = A_MN ? smem_desc_sw128(a_base + kk * 2048, 8192, 1024)
                                       : smem_desc_sw128(a_base + kk * 32, 0, 1024);
          const uint64_t b_desc = B_MN ? smem_desc_sw128(b_base + kk * 2048, 8192, 1024)
                                       : smem_desc_sw128(b_base + kk * 32, 0, 1024);
          mma_bf16_ss(d_tmem, a_desc, b_desc, idesc, (kb | kk) != 0);
        }
        mma_commit(&empty[stage]);
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
      mma_commit(&tfull[acc]);
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
    }
  } else if (warp >= 2) {
    // ------------------------------------------------------------- epilogue
    const int quarter = warp & 3;  // TMEM lanes [32*quarter, 32*quarter+32)
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
      if (*abort_flag) break;
      int tm, tn;
      tile_coords(t, num_m, num_n, tm, tn);
      if (!mbar_wait(&tfull[acc], acc_phase, err)) { *abort_flag = 1; break; }
      tc_fence_after();
      const int row = tm * BM + quarter * 32 + lane;
      const uint32_t t_row = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN;
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(t_row + c, r);
        tmem_wait_ld();
        const int col = tn * BN + c;
        if (row < M && col < N) {
          if (OUT == 0) {
            __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(C) + (long)row * ldc + col;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              if (col + 8 * j < N) {
                uint4 v;
                v.x = pack_bf16x2(__uint_as_float(r[8 * j + 0]), __uint_as_float(r[8 * j + 1]));
                v.y = pack_bf16x2(__uint_as_float(r[8 * j + 2]), __uint_as_float(r[8 * j + 3]));
                v.z = pack_bf16x2(__uint_as_float(r[8 * j + 4]), __uint_as_float(r[8 * j + 5]));
                v.w = pack_bf16x2(__uint_as_float(r[8 * j + 6]), __uint_as_float(r[8 * j + 7]));
                *reinterpret_cast<uint4*>(out + 8 * j) = v;
              }
            }
          } else {
            float* out = reinterpret_cast<float*>(C) + (long)row * ldc + col;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              if (col + 4 * j < N) {
                float4 v = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                       __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
                if (OUT == 2) {
                  const float4 o = *reinterpret_cast<const float4*>(out + 4 * j);
                  v.x += o.x; v.y += o.y; v.z += o.z; v.w += o.w;
                }
                *reinterpret_cast<float4*>(out + 4 * j) = v;
              }
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
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

template <bool A_MN, bool B_MN, int OUT>
cudaError_t launch(const GemmArgs& g, cudaStream_t stream) {
  auto kernel = gemm_bf16_kernel<A_MN, B_MN, OUT>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  CUtensorMap ta, tb;
  // A: K-major stored [M][K] (lda = row stride), or M-major stored [K][M].
  if (!make_tmap_bf16_2d(&ta, g.A, A_MN ? g.M : g.K, A_MN ? g.K : g.M, g.lda, 64, A_MN ? 64 : BM)) return cudaErrorInvalidValue;
  if (!make_tmap_bf16_2d(&tb, g.B, B_MN ? g.N : g.K, B_MN ? g.K : g.N, g.ldb, 64, B_MN ? 64 : BN)) return cudaErrorInvalidValue;
  const int tiles = ((g.M + BM - 1) / BM) * ((g.N + BN - 1) / BN);
  const int grid = tiles < g.num_sms ? tiles : g.num_sms;
  kernel<<<grid, THREADS, SMEM_BYTES, stream>>>(ta, tb, g.C, g.ldc, g.M, g.N, g.K, g.err);
  return cudaGetLastError();
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
  if (!g.a_mn && g.b_mn && g.out == OutMode::kBf16) return launch<false, true, 0>(g, stream);
  if (!g.a_mn && g.b_mn && g.out == OutMode::kF32) return launch<false, true, 1>(g, stream);
  if (!g.a_mn && !g.b_mn && g.out == OutMode::kBf16) return launch<false, false, 0>(g, stream);
  if (!g.a_mn && !g.b_mn && g.out == OutMode::kF32) return launch<false, false, 1>(g, stream);
  if (g.a_mn && g.b_mn && g.out == OutMode::kF32Accumulate) return launch<true, true, 2>(g, stream);
  if (g.a_mn && g.b_mn && g.out == OutMode::kF32) return launch<true, true, 1>(g, stream);
  if (!g.a_mn && !g.b_mn && g.out == OutMode::kF32Accumulate) return launch<false, false, 2>(g, stream);
  if (!g.a_mn && g.b_mn && g.out == OutMode::kF32Accumulate) return launch<false, true, 2>(g, stream);
  return cudaErrorInvalidValue;
}

}  // namespace nmb
