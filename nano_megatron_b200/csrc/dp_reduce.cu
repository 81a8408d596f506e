// Data-parallel gradient averaging over NVLink peer memory: one kernel does a
// two-shot all-reduce of one span ("bucket") of the flat fp32 gradient buffer,
// with the 1/dp scale applied in the same pass. Reference op: the flat
// all-reduce and divide of nano_megatron/grads.py:35-54.
//
// Every rank of the DP group maps every other rank's gradient buffer and flag
// area (symmetric memory). For a call with epoch e on rank r:
//   1. Every CTA announces ready[r] = e in every peer's flag area (release,
//      system scope; idempotent, so no peer depends on a particular CTA being
//      scheduled). The span is final because the kernel runs after the
//      backward kernels that wrote it (stream order). Every CTA waits until
//      all peers announced e (acquire).
//   2. Rank r owns slice r of the span. The CTAs sum slice r over all ranks'
//      buffers (peer loads, W x U = 8 independent 16-byte loads in flight per
//      thread, templated on the group size W), scale by 1/dp and store the
//      result into every rank's buffer (peer stores). Ranks write disjoint
//      slices and each reads only its own slice, so nothing overlaps.
//   3. After a system fence each CTA adds 1 to done[r] in every peer's flag
//      area (system-scope atomic) and to its own rank's finished counter. The
//      CTA that finishes last on this rank waits until done[p] reached the
//      grid size for every peer p (every peer's slice has landed here), then
//      resets the counters for the next call. When the kernel ends, the whole
//      span of this rank's buffer holds the average.
// A rank writes into a peer's buffer only after that peer announced the same
// epoch, so the peer's gradients for this span are final and none of its
// earlier reads are pending; for the same reason no increment of the next call
// can reach a counter before this call reset it. Every wait is bounded
// (timeout -> error word and early return; results are then garbage and the
// host raises).

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

__device__ __forceinline__ void add4(float4& a, const float4& b) {
  a.x += b.x; a.y += b.y; a.z += b.z; a.w += b.w;
}

template <int W>
__global__ void __launch_bounds__(kDpThreads) dp_allreduce_kernel(const DpReduceArgs a) {
  constexpr int U = W >= 8 ? 1 : 8 / W;  // float4 per rank per thread per step
  __shared__ int ok;
  const int e = a.epoch;
  int* mine = a.flags[a.rank];
  if ((int)threadIdx.x < W && (int)threadIdx.x != a.rank)
    st_release_sys_i32(a.flags[threadIdx.x] + kDpReadyOff + a.rank, e);
  if (threadIdx.x == 0) {
    ok = 1;
    for (int p = 0; p < W && ok; ++p)
      if (p != a.rank && !wait_at_least(mine + kDpReadyOff + p, e, a.err, a.timeout_ns)) ok = 0;
  }
  __syncthreads();
  if (!ok) return;

  // slice of this rank, in float4 units (span offset and length are multiples of 4)
  const long n4 = a.n / 4;
  const long per = (n4 + W - 1) / W;
  const long lo = min(n4, (long)a.rank * per), hi = min(n4, lo + per);
  const float4* src[W];
  float4* dst[W];
#pragma unroll
  for (int p = 0; p < W; ++p) {
    dst[p] = reinterpret_cast<float4*>(a.buf[p] + a.offset);
    src[p] = dst[p];
  }
  const long stride = (long)gridDim.x * kDpThreads;
  long i = lo + blockIdx.x * (long)kDpThreads + threadIdx.x;
  for (; i + (U - 1) * stride < hi; i += U * stride) {
    float4 v[W][U];
#pragma unroll
    for (int p = 0; p < W; ++p)
#pragma unroll
      for (int u = 0; u < U; ++u) v[p][u] = __ldcg(src[p] + i + u * stride);
#pragma unroll
    for (int u = 0; u < U; ++u) {
      float4 acc = v[0][u];
#pragma unroll
      for (int p = 1; p < W; ++p) add4(acc, v[p][u]);
      acc.x *= a.scale; acc.y *= a.scale; acc.z *= a.scale; acc.w *= a.scale;
#pragma unroll
      for (int p = 0; p < W; ++p) dst[p][i + u * stride] = acc;
    }
  }
  for (; i < hi; i += stride) {
    float4 acc = __ldcg(src[0] + i);
#pragma unroll
    for (int p = 1; p < W; ++p) add4(acc, __ldcg(src[p] + i));
    acc.x *= a.scale; acc.y *= a.scale; acc.z *= a.scale; acc.w *= a.scale;
#pragma unroll
    for (int p = 0; p < W; ++p) dst[p][i] = acc;
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int p = 0; p < W; ++p)
      if (p != a.rank) atomicAdd_system(a.flags[p] + kDpDoneOff + a.rank, 1);
    __threadfence();
    const int finished = atomicAdd(mine + kDpFinishedOff, 1) + 1;
    if (finished == (int)gridDim.x) {
      bool all = true;
      for (int p = 0; p < W && all; ++p)
        if (p != a.rank && !wait_at_least(mine + kDpDoneOff + p, (int)gridDim.x, a.err, a.timeout_ns)) all = false;
      if (all) {
        for (int p = 0; p < W; ++p) mine[kDpDoneOff + p] = 0;
        mine[kDpFinishedOff] = 0;
        __threadfence();
      }
    }
  }
}

}  // namespace

cudaError_t dp_allreduce(const DpReduceArgs& a, int num_sms, cudaStream_t stream) {
  if (a.n <= 0) return cudaSuccess;
  if (a.world < 1 || a.world > kDpMaxRanks || a.rank < 0 || a.rank >= a.world || a.n % 4 != 0 ||
      a.offset % 4 != 0 || a.epoch <= 0 || num_sms < 1)
    return cudaErrorInvalidValue;
  // at most one CTA on every other SM: the averaging runs beside the
  // backward's GEMMs, whose CTAs do not fit next to one of ours on an SM, so
  // half the SMs stay free for them; fewer CTAs for small spans (about 8
  // float4 of the slice per thread). 74 CTAs x 512 threads x 8 loads of 16 B
  // keep about 5 MB in flight, far above what the NVLink latency needs.
  const long per4 = (a.n / 4 + a.world - 1) / a.world;
  long blocks = (per4 + 8L * kDpThreads - 1) / (8L * kDpThreads);
  if (blocks < 1) blocks = 1;
  const int cap = num_sms > 1 ? num_sms / 2 : 1;
  if (blocks > cap) blocks = cap;
  switch (a.world) {
#define NMB_DP(W) \
  case W: dp_allreduce_kernel<W><<<(int)blocks, kDpThreads, 0, stream>>>(a); break;
    NMB_DP(1) NMB_DP(2) NMB_DP(3) NMB_DP(4) NMB_DP(5) NMB_DP(6) NMB_DP(7) NMB_DP(8)
#undef NMB_DP
  }
  return cudaGetLastError();
}

}  // namespace nmb
