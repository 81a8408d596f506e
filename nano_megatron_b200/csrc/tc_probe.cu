// Cycle probe for tcgen05.mma kind::f16 at M=128 on one SM: the cycles each
// product of a long chain takes, for N = 64, 128 or 256 and the A operand
// from shared memory (SS) or from TMEM (TS), issued in unrolled runs of 8 as
// the kernels issue them (`iters` is rounded down to a multiple of 8). The
// operands are zeros; what is measured is the time per instruction, which the
// attention kernels' tile shapes are chosen from (on B200 an N=64 product
// takes about 48 cycles, where its arithmetic alone would take 32).

#include <cuda_runtime.h>

#include "kernels.cuh"
#include "ptx.cuh"

namespace nmb {

namespace {

template <int N, bool TS>
__global__ void __launch_bounds__(128, 1) mma_cycles_kernel(long long* out, int iters, int* err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t bar;
  __shared__ uint32_t slot;
  const int warp = threadIdx.x / 32;
  for (int i = threadIdx.x; i < 65536 / 4; i += blockDim.x) reinterpret_cast<uint32_t*>(smem)[i] = 0u;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(&slot, 512);
    tmem_relinquish();
  }
  // make the generic-proxy zeros visible to the tensor core's async proxy
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = slot;
  if (threadIdx.x == 0) {
    const uint32_t sb = smem_u32(smem);
    constexpr uint32_t idesc = idesc_bf16_f32(128, N, false, false);
    const uint64_t ad = smem_desc_sw128(sb, 0, 1024), bd = smem_desc_sw128(sb + 32768, 0, 1024);
    // D at columns [0, N), the TS operand A at columns 448..479
    for (int i = 0; i < 8; ++i) mma_bf16_ss(tmem, ad, bd, idesc, i > 0);
    mma_commit(&bar);
    bool ok = mbar_wait(&bar, 0, err);
    tc_fence_after();
    const long long t0 = clock64();
    // runs of 8 unrolled products, as the kernels issue them
    for (int i = 0; i < iters / 8 && ok; ++i) {
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const uint64_t step = (uint64_t)((u & 3) * 2);  // next 16-element k-step of the 128-byte row
        if (TS) mma_bf16_ts(tmem, tmem + 448 + (u & 3) * 8, bd + step, idesc, 1);
        else mma_bf16_ss(tmem, ad + step, bd + step, idesc, 1);
      }
    }
    mma_commit(&bar);
    ok = ok && mbar_wait(&bar, 1, err);
    const long long t1 = clock64();
    out[0] = ok ? t1 - t0 : -1;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int N, bool TS>
cudaError_t launch_probe(long long* out, int iters, int* err, cudaStream_t stream) {
  constexpr int smem = 65536 + 1024;
  cudaError_t e = cudaFuncSetAttribute(mma_cycles_kernel<N, TS>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  mma_cycles_kernel<N, TS><<<1, 128, smem, stream>>>(out, iters, err);
  return cudaGetLastError();
}

}  // namespace

cudaError_t tc_mma_cycles(int n, bool ts, int iters, long long* out, int* err, cudaStream_t stream) {
  switch (n) {
    case 64: return ts ? launch_probe<64, true>(out, iters, err, stream) : launch_probe<64, false>(out, iters, err, stream);
    case 128:
      return ts ? launch_probe<128, true>(out, iters, err, stream) : launch_probe<128, false>(out, iters, err, stream);
    case 256:
      return ts ? launch_probe<256, true>(out, iters, err, stream) : launch_probe<256, false>(out, iters, err, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace nmb
