// Data-parallel gradient averaging over NVLink peer memory: one kernel does a
// two-shot all-reduce of one span ("bucket") of the flat fp32 gradient buffer,
// with the 1/dp scale applied in the same pass.
//
// Every rank of the DP group maps every other rank's gradient buffer and flag
// area (symmetric memory). For a call with epoch e on rank r:
//   1. CTA 0 announces ready[r] = e in every peer's flag area (release,
//      system scope); the buffer span is final because the kernel runs after
//      the backward kernels that wrote it (stream order). Every CTA waits until
//      all peers announced e (acquire).
//   2. Rank r owns slice r of the span. Each CTA sums its part of slice r over
//      all ranks' buffers (peer loads), multiplies by 1/dp, and stores the
//      result into every rank's buffer (peer stores). Ranks write disjoint
//      slices, and each reads only its own slice, so nothing overlaps.
//   3. After a system fence each CTA sets done[r][cta] = e in every peer's
//      flag area. Every CTA then waits for all peers' done flags. After that
//      the whole span of this rank's buffer holds the average.
// A rank writes into a peer's buffer only after that peer announced the same
// epoch, so the peer's gradients for this span are final and none of its
// earlier reads are pending. Every wait is bounded (timeout -> error word and
// early return; results are then garbage and the host raises).

#include <cuda_runtime.h>

#include <cstdint>

#include "dp_reduce.cuh"
#include "ptx.cuh"

namespace nmb {

namespace {

constexpr int kDpThreads = 512;

__device__ __forceinline__ void st_release_sys_i32(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ int ld_acquire_sys_i32(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ bool wait_at_least(const int* flag, int want, int* err, uint64_t timeout_ns) {
  if (ld_acquire_sys_i32(flag) >= want) return true;
  const uint64_t start = globaltimer_ns();
  while (true) {
    for (int i = 0; i < 32; ++i) {
      if (ld_acquire_sys_i32(flag) >= want) return true;
      __nanosleep(128);
    }
    if (globaltimer_ns() - start > timeout_ns) {
      report_error(err, kPeerTimeout);
      return false;
    }
  }
}

__global__ void __launch_bounds__(kDpThreads) dp_allreduce_kernel(const DpReduceArgs a) {
  __shared__ int ok;
  const int e = a.epoch;
  if (threadIdx.x == 0) {
    ok = 1;
    if (blockIdx.x == 0)
      for (int p = 0; p < a.world; ++p)
        if (p != a.rank) st_release_sys_i32(a.flags[p] + kDpReadyOff + a.rank, e);
    const int* mine = a.flags[a.rank];
    for (int p = 0; p < a.world && ok; ++p)
      if (p != a.rank && !wait_at_least(mine + kDpReadyOff + p, e, a.err, a.timeout_ns)) ok = 0;
  }
  __syncthreads();
  if (!ok) return;

  // slice of this rank, in float4 units (span offset and length are multiples of 4)
  const long n4 = a.n / 4;
  const long per = (n4 + a.world - 1) / a.world;
  const long lo = min(n4, (long)a.rank * per), hi = min(n4, lo + per);
  for (long i = lo + blockIdx.x * (long)kDpThreads + threadIdx.x; i < hi; i += (long)gridDim.x * kDpThreads) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int p = 0; p < a.world; ++p) {
      const float4 v = __ldcg(reinterpret_cast<const float4*>(a.buf[p] + a.offset) + i);
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
    acc.x *= a.scale; acc.y *= a.scale; acc.z *= a.scale; acc.w *= a.scale;
    for (int p = 0; p < a.world; ++p) reinterpret_cast<float4*>(a.buf[p] + a.offset)[i] = acc;
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int p = 0; p < a.world; ++p)
      if (p != a.rank) st_release_sys_i32(a.flags[p] + kDpDoneOff + a.rank * kDpMaxCtas + blockIdx.x, e);
    const int* mine = a.flags[a.rank];
    for (int p = 0; p < a.world && ok; ++p) {
      if (p == a.rank) continue;
      for (int c = 0; c < (int)gridDim.x && ok; ++c)
        if (!wait_at_least(mine + kDpDoneOff + p * kDpMaxCtas + c, e, a.err, a.timeout_ns)) ok = 0;
    }
  }
}

}  // namespace

cudaError_t dp_allreduce(const DpReduceArgs& a, cudaStream_t stream) {
  if (a.n <= 0) return cudaSuccess;
  if (a.world < 1 || a.world > kDpMaxRanks || a.rank < 0 || a.rank >= a.world || a.n % 4 != 0 ||
      a.offset % 4 != 0 || a.epoch <= 0)
    return cudaErrorInvalidValue;
  const long per4 = (a.n / 4 + a.world - 1) / a.world;
  long blocks = (per4 + 4L * kDpThreads - 1) / (4L * kDpThreads);  // about 4 float4 per thread
  if (blocks < 1) blocks = 1;
  if (blocks > kDpMaxCtas) blocks = kDpMaxCtas;
  dp_allreduce_kernel<<<(int)blocks, kDpThreads, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace nmb
