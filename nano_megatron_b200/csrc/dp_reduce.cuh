// Host interface of the data-parallel gradient averaging kernel (dp_reduce.cu).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace nmb {

constexpr int kDpMaxRanks = 8;
// int32 offsets inside each rank's flag area
constexpr int kDpReadyOff = 0;                       // [kDpMaxRanks] epoch announced by each peer
constexpr int kDpDoneOff = kDpMaxRanks;              // [kDpMaxRanks] CTAs of each peer that delivered
constexpr int kDpFinishedOff = 2 * kDpMaxRanks;      // CTAs of this rank that finished
constexpr int kDpFlagInts = 2 * kDpMaxRanks + 8;

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
// The grid depends only on (n, world, num_sms), so it is the same on every
// rank of the group (the completion count relies on it).
cudaError_t dp_allreduce(const DpReduceArgs& args, int num_sms, cudaStream_t stream);

}  // namespace nmb
