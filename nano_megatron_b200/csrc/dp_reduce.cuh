// Host interface of the data-parallel gradient averaging kernel (dp_reduce.cu).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace nmb {

constexpr int kDpMaxRanks = 8;
constexpr int kDpMaxCtas = 64;
// int32 offsets inside each rank's flag area
constexpr int kDpReadyOff = 0;                                    // [kDpMaxRanks]
constexpr int kDpDoneOff = kDpMaxRanks;                           // [kDpMaxRanks][kDpMaxCtas]
constexpr int kDpFlagInts = kDpDoneOff + kDpMaxRanks * kDpMaxCtas;

struct DpReduceArgs {
  float* buf[kDpMaxRanks];  // every rank's flat gradient buffer, mapped in this process
  int* flags[kDpMaxRanks];  // every rank's flag area (kDpFlagInts ints)
  long offset, n;           // span [offset, offset + n) in elements; both multiples of 4
  int rank, world;
  int epoch;                // per-call sequence number, identical on all ranks, > 0
  float scale;              // 1 / world
  int* err;
  uint64_t timeout_ns;
};

// buf[r][span] = scale * sum over ranks of buf[p][span], on every rank.
cudaError_t dp_allreduce(const DpReduceArgs& args, cudaStream_t stream);

}  // namespace nmb
