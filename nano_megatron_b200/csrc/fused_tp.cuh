// Host interface of the fused tensor-parallel GEMM + collective kernels (fused_tp.cu).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace nmb {

constexpr int kAllGatherGemm = 0;
constexpr int kReduceScatterGemm = 1;
// all-gather -> LM-head GEMM with the cross-entropy statistics in the epilogue
constexpr int kAllGatherGemmCE = 2;
// all-gather -> gate|up GEMM with the SwiGLU epilogue: B is [K][2F] (gate |
// up halves), out = silu(X W_gate) * (X W_up) [M][F], gu (optional) [M][2F]
constexpr int kAllGatherGemmSwiGLU = 3;
constexpr int kMaxRanks = 8;
constexpr int kMaxCtas = 160;
constexpr int kMaxTiles = 16384;
// int32 flag offsets inside the workspace's flag area
constexpr int kReadyOff = 0;                                   // [kMaxRanks]
constexpr int kAgDoneOff = kMaxRanks;                          // [kMaxRanks][kMaxCtas]
constexpr int kRsDoneOff = kAgDoneOff + kMaxRanks * kMaxCtas;  // [kMaxTiles][kMaxRanks]
constexpr int kMaxCeBlocks = 1024;
constexpr long kCeFlagOff = kRsDoneOff + (long)kMaxTiles * kMaxRanks;  // [kMaxRanks][kMaxCeBlocks]
// work-claim counters of the fused GEMM kernels, [kind][call parity]: tiles,
// all-gather push slices, gathered-input copy slices (local atomics only)
constexpr long kClaimOff = kCeFlagOff + (long)kMaxRanks * kMaxCeBlocks;
constexpr int kClaimTiles = 0, kClaimPush = 2, kClaimSave = 4;
constexpr long kFlagInts = kClaimOff + 8;

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
  // all-gather modes: optional private copy [M][K] of the gathered input,
  // filled by the comm warps while the GEMM runs (null = none)
  __nv_bfloat16* save_out;
  // kAllGatherGemmCE: per-row statistics of the bf16-rounded logits of every
  // 256-column tile tn: ce_part[tn * M + row] = (max, sum exp(v - max)); the
  // tile holding column labels[row] - vocab_start writes ce_target[row].
  const int64_t* labels;
  long vocab_start;
  float2* ce_part;
  float* ce_target;
  // kAllGatherGemmSwiGLU: bf16 pre-activation output [M][ldgu] (null = not written)
  __nv_bfloat16* gu;
  long ldgu;
};

cudaError_t fused_tp_gemm(int mode, const FusedTpArgs& args, const void* B, long ldb, bool b_mn, int num_sms,
                          cudaStream_t stream);

// Cross-entropy merge: per row, combines the num_n tile statistics of
// kAllGatherGemmCE into (max, sum-exp, target logit) of this rank's vocabulary
// shard, exchanges them with the other ranks of the TP group through the
// symmetric workspace (pushed with plain peer stores, one flag per block) and
// writes loss = log(sum) + max - target, the global max and the global sum.
struct CeMergeArgs {
  const float2* part;          // [num_n][T]
  const float* target_logit;   // [T], read where the label is in [vocab_start, vocab_end)
  const int64_t* labels;       // [T]
  long vocab_start, vocab_end;
  int T, num_n, rank, world;
  uint8_t* ws[kMaxRanks];      // every rank's workspace (unused when world == 1)
  long data_off, flags_off;    // data: [2 slots][kMaxRanks][T] float4
  uint32_t epoch;              // per-merge sequence number, identical on all ranks, > 0
  int* err;
  uint64_t timeout_ns;
  float* loss;
  float* gmax;
  float* gsum;
};

cudaError_t ce_merge(const CeMergeArgs& args, cudaStream_t stream);

}  // namespace nmb
