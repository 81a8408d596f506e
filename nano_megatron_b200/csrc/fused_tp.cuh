// Host interface of the fused tensor-parallel GEMM + collective kernels (fused_tp.cu).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace nmb {

constexpr int kAllGatherGemm = 0;
constexpr int kReduceScatterGemm = 1;
constexpr int kMaxRanks = 8;
constexpr int kMaxCtas = 160;
constexpr int kMaxTiles = 16384;
// int32 flag offsets inside the workspace's flag area
constexpr int kReadyOff = 0;                                   // [kMaxRanks]
constexpr int kAgDoneOff = kMaxRanks;                          // [kMaxRanks][kMaxCtas]
constexpr int kRsDoneOff = kAgDoneOff + kMaxRanks * kMaxCtas;  // [kMaxTiles][kMaxRanks]
constexpr long kFlagInts = kRsDoneOff + (long)kMaxTiles * kMaxRanks;

struct FusedTpArgs {
  int M, N, K;          // M = rows of the full (gathered) sequence
  int rank, world;      // position in the TP group
  int m_chunk;          // M / world, a multiple of 128
  __nv_bfloat16* out;   // all-gather: [M][ldo]; reduce-scatter: [m_chunk][ldo]
  long ldo;
  uint8_t* ws[kMaxRanks];  // every rank's symmetric workspace, mapped in this process
  long gather_off, recv_off, flags_off;  // byte offsets inside the workspace
  const __nv_bfloat16* a_local;  // all-gather: this rank's shard [m_chunk][K]; reduce-scatter: A [M][K]
  long lda_local;
  uint32_t epoch;       // per-call sequence number, identical on all ranks, > 0
  int copy_own;         // all-gather: also copy the own shard into the own gather slot
  int* err;             // device error word
  uint64_t timeout_ns;  // bound on every cross-GPU wait
};

cudaError_t fused_tp_gemm(int mode, const FusedTpArgs& args, const void* B, long ldb, bool b_mn, int num_sms,
                          cudaStream_t stream);

}  // namespace nmb
