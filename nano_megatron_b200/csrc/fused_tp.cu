// Tensor-parallel GEMMs fused with their sequence-parallel collectives over
// NVLink peer memory (one kernel does the math and the communication).
// Reference ops: x @ W with the sequence all-gather / reduce-scatter around it
// (nano_megatron/tp_layers.py:54-88, mappings.py:109-134, used at
// model.py:113-128 and 147-153), and the LM head with the vocab-parallel cross
// entropy (model.py:185-192, cross_entropy.py:16-65).
//
//   all-gather -> GEMM   Y[M,N] = AG(x)[M,K] @ B     (QKV, gate|up forward;
//                                                      row-parallel dgrad)
//   GEMM -> reduce-scatter   out[M/t,N] = RS(A[M,K] @ B)   (proj, down forward;
//                                                      column-parallel dgrad)
//
// Both are the persistent tcgen05 GEMM of gemm.cu (TMA producer warp, MMA
// warp, four epilogue warps, double-buffered TMEM accumulator) plus one comm
// warp, working in a symmetric workspace that every rank of the TP group has
// mapped (peer pointers `ws[r]`):
//
//   workspace = gather [M][K] bf16 | recv [t][M/t][N] bf16 | flags (int32)
//
// all-gather -> GEMM (rank r):
//   * comm warp: announces `ready[r] = epoch` on every peer, then pushes this
//     CTA's slice of the local shard x into peer p's gather buffer, rows of
//     chunk r, for p = r-1, r-2, ... (the peer that needs chunk r soonest
//     first), each after p announced ready; then sets ag_done[r][cta] = epoch
//     on p (release, system scope, after a system fence).
//   * tiles run chunk by chunk starting with the own chunk, whose A tiles TMA
//     reads straight from x. Before the first tile of chunk c the producer
//     waits until all of c's CTAs have set ag_done[c][*] (acquire), fences the
//     async proxy, and TMA-loads A from the local gather buffer. Only local
//     memory is ever read by TMA (peer data arrives by plain stores).
// GEMM -> reduce-scatter (rank r):
//   * tiles run chunk r+1, r+2, ... and the own chunk last. The epilogue of a
//     foreign tile converts the fp32 accumulator to bf16 and stores it into
//     the owner's recv[r] slot (peer stores), then sets rs_done[tile][r].
//     The epilogue of an own tile waits for rs_done[tile][*] of every peer and
//     writes acc + sum of the peers' partials (fp32 sum) to the output.
//   * no rank waits before it has pushed everything the others wait on, so
//     the protocol cannot deadlock as long as every rank runs the kernel.
//
// all-gather -> LM-head GEMM -> cross-entropy statistics (kAllGatherGemmCE):
//   * the all-gather -> GEMM above with logits = AG(x) @ W^T; the epilogue
//     rounds each logit to bf16 (the stored value), and per row and 256-column
//     tile keeps the running max and sum of exp(v - max) (one query row per
//     epilogue thread, so no cross-thread reduction) plus the target logit.
//     ce_merge (below) then combines tiles and ranks; fp32 logits are never
//     materialized.
// all-gather -> gate|up GEMM -> SwiGLU (kAllGatherGemmSwiGLU): B is the gate|up
//   weight [K][2F]; a tile's four 64-column B boxes are gate columns n0, n0+64
//   and up columns F+n0, F+n0+64, so an accumulator row holds gate and up of
//   the same 128 features. The epilogue writes a = bf16(bf16(silu(g)) * u)
//   with g, u rounded to bf16 first (the unfused arithmetic) and, if asked,
//   the pre-activation halves through two [M][F] views of gu.
// Optional copy of the gathered input (all-gather modes, `save_out`): after
// its pushes the comm warp of CTA b copies slice b of every chunk (its own
// from x, chunk c once peer c's CTA b flagged it) into save_out, overlapping
// the GEMM; the weight gradient then needs no second all-gather.
//
// Reuse of the workspace across calls: every call carries a new epoch; a rank
// writes into a peer's buffers only after that peer announced the epoch,
// i.e. after the peer's previous kernels (which read the buffers) finished.
// Every wait is bounded (`timeout_ns`): on expiry the kernel records
// kPeerTimeout in the error word, stops waiting and returns (results are then
// garbage and the host raises).

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "fused_tp.cuh"
#include "gemm.cuh"
#include "ptx.cuh"

namespace nmb {

namespace {

constexpr int BM = 128, BN = 256, BK = 64;
constexpr int A_TILE_BYTES = BM * BK * 2;
constexpr int B_TILE_BYTES = BN * BK * 2;
constexpr int STAGE_BYTES = A_TILE_BYTES + B_TILE_BYTES;
// The reduce-scatter variant has a 32 KB staging area in which each epilogue
// warp assembles half rows (128 columns, 256 B) of its 32 output rows; a
// partial tile crosses NVLink as two such halves, each warp instruction
// writing two contiguous 256-byte row pieces instead of 64-byte pieces of 32
// different rows.
constexpr int HALF_ROW = BN / 2 * 2;                   // 256 B
constexpr int STAGING_BYTES = 4 * 32 * HALF_ROW;
template <int MODE>
struct Cfg {
  static constexpr int STAGES = 4;
  // all-gather modes: two 4 KB output boxes (32 rows x 128 B) per epilogue warp
  static constexpr int STAGING = MODE == kReduceScatterGemm ? STAGING_BYTES : 4 * 2 * 4096;
  static constexpr int SMEM = STAGES * STAGE_BYTES + STAGING + 1024 + 512;
};
constexpr int THREADS = 224;  // 7 warps: producer, MMA, 4 epilogue, comm
constexpr float kLog2e = 1.4426950408889634f;

template <int MODE>
constexpr bool is_ag() {
  return MODE != kReduceScatterGemm;
}

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

__device__ __forceinline__ void epilogue_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Wait until *flag >= want. Returns false (and records kPeerTimeout) on expiry.
__device__ bool wait_flag(const int* flag, int want, int* err, uint64_t timeout_ns, volatile int* abort_flag) {
  if (ld_acquire_sys(flag) >= want) return true;
  const uint64_t start = globaltimer_ns();
  while (true) {
    if (*abort_flag) return false;
    for (int i = 0; i < 32; ++i) {
      if (ld_acquire_sys(flag) >= want) return true;
      __nanosleep(64);
    }
    if (globaltimer_ns() - start > timeout_ns) {
      report_error(err, kPeerTimeout);
      *abort_flag = 1;
      return false;
    }
  }
}

// mbarrier wait that gives up at once when another role has aborted.
__device__ bool mbar_wait_abortable(uint64_t* bar, uint32_t parity, int* err, volatile int* abort_flag,
                                    uint64_t timeout_ns = 20000000000ull) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = globaltimer_ns();
  while (true) {
    if (*abort_flag) return false;
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - start > timeout_ns) {
      report_error(err, kBarrierTimeout);
      *abort_flag = 1;
      return false;
    }
  }
}

__device__ __forceinline__ int* flags_of(const FusedTpArgs& a, int rank) {
  return reinterpret_cast<int*>(a.ws[rank] + a.flags_off);
}

// Work claiming. With more than one rank, tiles and all-gather slices are
// claimed from counters in this rank's flag area, in a fixed order, by
// whichever CTAs are running: no rank ever waits for work that is bound to a
// particular CTA of a peer, so the kernel finishes even when other kernels
// (NCCL, the data-parallel reduction) hold some SMs and only part of the grid
// is resident at a time. Each call uses the counters of its epoch's parity
// and zeroes the other parity's, which the previous call (complete, by
// stream order) used. A group of one assigns work statically.
__device__ __forceinline__ int* claim_ctr(const FusedTpArgs& a, int* my_flags, int kind) {
  return a.world > 1 ? my_flags + kClaimOff + kind + (a.epoch & 1u) : nullptr;
}

__device__ __forceinline__ int claim(int* ctr, int it) {
  return ctr != nullptr ? atomicAdd(ctr, 1) : (int)blockIdx.x + it * (int)gridDim.x;
}

constexpr int kQueue = 4;  // tiles handed from the producer to the MMA warp and the epilogue

struct TileInfo {
  int tm, tn, chunk, local;
};

template <int MODE>
__device__ __forceinline__ TileInfo tile_of(int t, const FusedTpArgs& a, int mt_chunk, int num_n) {
  const int per_chunk = mt_chunk * num_n;
  const int slot = t / per_chunk;
  TileInfo ti;
  ti.local = t - slot * per_chunk;
  ti.chunk = is_ag<MODE>() ? (a.rank + slot) % a.world : (a.rank + 1 + slot) % a.world;
  ti.tm = ti.chunk * mt_chunk + ti.local % mt_chunk;
  ti.tn = ti.local / mt_chunk;
  return ti;
}

template <int MODE, bool B_MN>
__global__ void __launch_bounds__(THREADS, 1)
fused_tp_kernel(const __grid_constant__ CUtensorMap tmA_local, const __grid_constant__ CUtensorMap tmA_gather,
                const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmOut,
                const __grid_constant__ CUtensorMap tmG, const __grid_constant__ CUtensorMap tmU,
                const FusedTpArgs a) {
  constexpr bool SWIGLU = MODE == kAllGatherGemmSwiGLU;
  constexpr int STAGES = Cfg<MODE>::STAGES;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* staging = smem + STAGES * STAGE_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(staging + Cfg<MODE>::STAGING);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* mma_done = tempty + 2;
  uint64_t* qfull = mma_done + 1;     // [kQueue] tile index published
  uint64_t* qempty = qfull + kQueue;  // [kQueue] read by the MMA warp and the epilogue leader
  int* tq = reinterpret_cast<int*>(qempty + kQueue);  // [kQueue] claimed tile, -1 = no more
  volatile int* ep_tile = tq + kQueue;                // [2] tile broadcast to the epilogue warps
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(const_cast<int*>(ep_tile) + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int mt_chunk = a.m_chunk / BM;
  const int F = a.N / 2;  // SwiGLU: features per half
  const int num_n = SWIGLU ? (F + BN / 2 - 1) / (BN / 2) : (a.N + BN - 1) / BN;
  const int num_tiles = a.world * mt_chunk * num_n;
  const int num_k = (a.K + BK - 1) / BK;
  const int epoch = (int)a.epoch;
  int* my_flags = flags_of(a, a.rank);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 128);
    }
    mbar_init(mma_done, 1);
    for (int q = 0; q < kQueue; ++q) {
      mbar_init(&qfull[q], 1);
      mbar_init(&qempty[q], 2);
    }
    *abort_flag = 0;
    if (a.world > 1) {  // the previous call's counters, for the next call
      const int other = (int)((a.epoch + 1) & 1u);
      my_flags[kClaimOff + kClaimTiles + other] = 0;
      my_flags[kClaimOff + kClaimPush + other] = 0;
      my_flags[kClaimOff + kClaimSave + other] = 0;
    }
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

  if (warp == 6) {
    // ---------------------------------------------------------------- comm
    // Every CTA announces the epoch (idempotent), so a peer never waits for a
    // particular CTA of this rank to be scheduled.
    if (lane < a.world && lane != a.rank) st_release_sys(flags_of(a, lane) + kReadyOff + a.rank, epoch);
    if (is_ag<MODE>()) {
      // The local shard is cut into S = gridDim.x slices (16-byte units). A
      // job is one slice pushed to one destination; jobs are claimed from a
      // counter by whichever comm warps are running, destination-major (the
      // peer that needs chunk r soonest first, the own gather slot last), so
      // every slice is delivered as long as one CTA of this rank is resident.
      const int S = gridDim.x;
      const long total = (long)a.m_chunk * a.K / 8;
      const long per = (total + S - 1) / S;
      const uint4* src = reinterpret_cast<const uint4*>(a.a_local);
      const long chunk_off = a.gather_off + (long)a.rank * a.m_chunk * a.K * 2;
      const int dests = a.world - 1 + (a.copy_own ? 1 : 0);
      int* push_ctr = claim_ctr(a, my_flags, kClaimPush);
      uint32_t ready_seen = 0;
      for (int it = 0;; ++it) {
        int job = 0;
        if (lane == 0) job = claim(push_ctr, it);
        job = __shfl_sync(0xffffffffu, job, 0);
        if (job >= dests * S || *abort_flag) break;
        const int d = job / S, slice = job - d * S;
        const int p = d < a.world - 1 ? (a.rank - 1 - d + a.world) % a.world : a.rank;
        if (p != a.rank && !((ready_seen >> p) & 1u)) {
          bool ok = true;
          if (lane == 0) ok = wait_flag(my_flags + kReadyOff + p, epoch, a.err, a.timeout_ns, abort_flag);
          ok = __shfl_sync(0xffffffffu, ok, 0);
          if (!ok) break;
          ready_seen |= 1u << p;
        }
        const long beg = per * slice, end = min(total, beg + per);
        uint4* dst = reinterpret_cast<uint4*>(a.ws[p] + chunk_off);
        long i = beg + lane;
        for (; i + 31 * 8 < end; i += 32 * 8) {
          uint4 v[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) v[u] = src[i + 32 * u];
#pragma unroll
          for (int u = 0; u < 8; ++u) dst[i + 32 * u] = v[u];
        }
        for (; i < end; i += 32) dst[i] = src[i];
        if (p != a.rank) {
          __threadfence_system();
          __syncwarp();
          if (lane == 0) st_release_sys(flags_of(a, p) + kAgDoneOff + a.rank * kMaxCtas + slice, epoch);
        }
      }
      if (a.save_out != nullptr) {
        // Private copy of the gathered input: job = (chunk in arrival order, slice).
        const long chunk_units = (long)a.m_chunk * a.K / 8;
        int* save_ctr = claim_ctr(a, my_flags, kClaimSave);
        for (int it = 0;; ++it) {
          int job = 0;
          if (lane == 0) job = claim(save_ctr, it);
          job = __shfl_sync(0xffffffffu, job, 0);
          if (job >= a.world * S || *abort_flag) break;
          const int j = job / S, slice = job - j * S;
          const int c = (a.rank + j) % a.world;  // own chunk first, then in arrival order
          const uint4* from = src;
          if (c != a.rank) {
            bool ok = true;
            if (lane == 0) ok = wait_flag(my_flags + kAgDoneOff + c * kMaxCtas + slice, epoch, a.err,
                                          a.timeout_ns, abort_flag);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            __syncwarp();
            if (!ok) break;
            from = reinterpret_cast<const uint4*>(a.ws[a.rank] + a.gather_off) + c * chunk_units;
          }
          uint4* to = reinterpret_cast<uint4*>(a.save_out) + c * chunk_units;
          const long beg = per * slice, end = min(total, beg + per);
          long i = beg + lane;
          for (; i + 31 * 8 < end; i += 32 * 8) {
            uint4 v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) v[u] = __ldcg(from + i + 32 * u);
#pragma unroll
            for (int u = 0; u < 8; ++u) to[i + 32 * u] = v[u];
          }
          for (; i < end; i += 32) to[i] = __ldcg(from + i);
        }
      }
    }
  } else if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer
    tma_prefetch_desc(&tmA_local);
    tma_prefetch_desc(&tmB);
    uint32_t ready_mask = 1u << a.rank;
    int stage = 0;
    uint32_t phase = 0;
    int issued[STAGES];  // parity of the last load issued into each stage, -1 if none
#pragma unroll
    for (int s = 0; s < STAGES; ++s) issued[s] = -1;
    int* tile_ctr = claim_ctr(a, my_flags, kClaimTiles);
    int next = claim(tile_ctr, 0);  // claimed one tile ahead: the atomic's latency hides behind a tile
    for (int it = 0;; ++it) {
      const int slot = it & (kQueue - 1);
      if (!mbar_wait_abortable(&qempty[slot], ((uint32_t)(it / kQueue) & 1u) ^ 1u, a.err, abort_flag)) break;
      const int t = (*abort_flag || next >= num_tiles) ? -1 : next;
      tq[slot] = t;
      mbar_arrive(&qfull[slot]);
      if (t < 0) break;
      next = claim(tile_ctr, it + 1);
      const TileInfo ti = tile_of<MODE>(t, a, mt_chunk, num_n);
      const bool from_gather = is_ag<MODE>() && ti.chunk != a.rank;
      if (from_gather && !((ready_mask >> ti.chunk) & 1u)) {
        const int* done = my_flags + kAgDoneOff + ti.chunk * kMaxCtas;
        for (int c = 0; c < (int)gridDim.x; ++c)
          if (!wait_flag(done + c, epoch, a.err, a.timeout_ns, abort_flag)) break;
        fence_proxy_async_global();
        ready_mask |= 1u << ti.chunk;
      }
      const CUtensorMap* amap = from_gather ? &tmA_gather : &tmA_local;
      const int arow = (is_ag<MODE>() && !from_gather) ? (ti.tm * BM - a.rank * a.m_chunk) : ti.tm * BM;
      for (int kb = 0; kb < num_k; ++kb) {
        if (!mbar_wait_abortable(&empty[stage], phase ^ 1, a.err, abort_flag)) break;
        uint8_t* a_dst = smem + stage * STAGE_BYTES;
        uint8_t* b_dst = a_dst + A_TILE_BYTES;
        mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
        issued[stage] = (int)phase;
        const int k0 = kb * BK;
        tma_load_2d(a_dst, amap, &full[stage], k0, arow);
        if (SWIGLU) {
#pragma unroll
          for (int j = 0; j < 4; ++j)
            tma_load_2d(b_dst + j * 8192, &tmB, &full[stage], (j >> 1) * F + ti.tn * (BN / 2) + 64 * (j & 1), k0);
        } else if (B_MN) {
#pragma unroll
          for (int j = 0; j < 4; ++j) tma_load_2d(b_dst + j * 8192, &tmB, &full[stage], ti.tn * BN + 64 * j, k0);
        } else {
          tma_load_2d(b_dst, &tmB, &full[stage], k0, ti.tn * BN);
        }
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
    }
    // Never leave a TMA copy in flight at exit (matters only after an abort).
    for (int s = 0; s < STAGES; ++s)
      if (issued[s] >= 0) mbar_wait(&full[s], (uint32_t)issued[s], nullptr, 1000000000ull);
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------- MMA issue
    constexpr uint32_t idesc = idesc_bf16_f32(BM, BN, false, B_MN);
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int it = 0;; ++it) {
      const int slot = it & (kQueue - 1);
      if (!mbar_wait_abortable(&qfull[slot], (uint32_t)(it / kQueue) & 1u, a.err, abort_flag)) break;
      const int t = tq[slot];
      mbar_arrive(&qempty[slot]);
      if (t < 0) break;
      if (!mbar_wait_abortable(&tempty[acc], acc_phase ^ 1, a.err, abort_flag)) break;
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + acc * BN;
      for (int kb = 0; kb < num_k; ++kb) {
        if (!mbar_wait_abortable(&full[stage], phase, a.err, abort_flag)) break;
        tc_fence_after();
        const uint32_t a_base = smem_u32(smem + stage * STAGE_BYTES);
        const uint32_t b_base = a_base + A_TILE_BYTES;
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          const uint64_t a_desc = smem_desc_sw128(a_base + kk * 32, 0, 1024);
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
    // Let the last MMAs finish before TMEM is released (matters only after an abort).
    mma_commit(mma_done);
    mbar_wait(mma_done, 0, nullptr, 1000000000ull);
  } else if (warp >= 2 && warp <= 5) {
    // ------------------------------------------------------------- epilogue
    const int quarter = warp & 3;
    const bool leader = warp == 2 && lane == 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    uint32_t ready_mask = 1u << a.rank;
    // all-gather modes: output rows go through swizzled 64-column boxes that
    // TMA stores (two buffers per warp, one box per two 32-column chunks)
    uint8_t* box_stg = staging + quarter * 2 * 4096;
    int nbox = 0;
    // reduce-scatter: write half h (columns [128h, 128h + 128)) of the warp's
    // 32 staged rows to the owner of a foreign tile; lanes 0-15 take one row,
    // lanes 16-31 the next, so each instruction writes two 256-byte pieces
    auto flush_half = [&](const TileInfo& ft, int h) {
      __syncwarp();
      const int sub = lane >> 4, ch = lane & 15;
      const int col = ft.tn * BN + h * (BN / 2) + ch * 8;
      const int row0 = ft.tm * BM + quarter * 32 - ft.chunk * a.m_chunk;
      __nv_bfloat16* dst0 = reinterpret_cast<__nv_bfloat16*>(a.ws[ft.chunk] + a.recv_off) +
                            ((long)a.rank * a.m_chunk + row0) * a.N + col;
#pragma unroll 4
      for (int r2 = 0; r2 < 16; ++r2) {
        const int rr = 2 * r2 + sub;
        const uint4 u = *reinterpret_cast<const uint4*>(staging + (quarter * 32 + rr) * HALF_ROW +
                                                         ((ch ^ (rr & 7)) << 4));
        if (col < a.N) *reinterpret_cast<uint4*>(dst0 + (long)rr * a.N) = u;
      }
      __syncwarp();
    };
    // Control flow here is uniform over the 128 epilogue threads (named
    // barriers): the leader takes the next tile from the queue and hands it to
    // all four warps; after an abort it hands out -1 and everyone leaves.
    for (int it = 0;; ++it) {
      if (leader) {
        const int slot = it & (kQueue - 1);
        int next = -1;
        if (mbar_wait_abortable(&qfull[slot], (uint32_t)(it / kQueue) & 1u, a.err, abort_flag)) next = tq[slot];
        mbar_arrive(&qempty[slot]);
        ep_tile[it & 1] = next;
      }
      epilogue_bar();
      const int t = ep_tile[it & 1];
      if (t < 0) break;
      const TileInfo ti = tile_of<MODE>(t, a, mt_chunk, num_n);
      mbar_wait_abortable(&tfull[acc], acc_phase, a.err, abort_flag);
      tc_fence_after();
      const int row = ti.tm * BM + quarter * 32 + lane;
      const int row_local = row - ti.chunk * a.m_chunk;
      const uint32_t t_row = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN;
      if (SWIGLU) {
        const int row0 = ti.tm * BM + quarter * 32;
        auto store_box = [&](const CUtensorMap* map, const float* v, int col) {
          uint8_t* buf = box_stg + (nbox & 1) * 4096;
          if (lane == 0) bulk_wait_group_read<1>();
          __syncwarp();
          uint8_t* brow = buf + lane * 128;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            uint4 u;
            u.x = pack_bf16x2(v[8 * j + 0], v[8 * j + 1]);
            u.y = pack_bf16x2(v[8 * j + 2], v[8 * j + 3]);
            u.z = pack_bf16x2(v[8 * j + 4], v[8 * j + 5]);
            u.w = pack_bf16x2(v[8 * j + 6], v[8 * j + 7]);
            *reinterpret_cast<uint4*>(brow + ((j ^ (lane & 7)) << 4)) = u;
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            if (col < F) tma_store_2d(map, buf, col, row0);
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
          tmem_wait_ld();
          float g[64], u[64];
#pragma unroll
          for (int j = 0; j < 64; ++j) {
            g[j] = __bfloat162float(__float2bfloat16_rn(__uint_as_float(gr[j])));
            u[j] = __bfloat162float(__float2bfloat16_rn(__uint_as_float(ur[j])));
          }
          const int col = ti.tn * (BN / 2) + c;
          if (a.gu != nullptr) {
            store_box(&tmG, g, col);
            store_box(&tmU, u, col);
          }
#pragma unroll
          for (int j = 0; j < 64; ++j) {
            const float sl = g[j] / (1.f + __expf(-g[j]));
            g[j] = __bfloat162float(__float2bfloat16_rn(sl)) * u[j];
          }
          store_box(&tmOut, g, col);
        }
        tc_fence_before();
        mbar_arrive(&tempty[acc]);
        if (++acc == 2) { acc = 0; acc_phase ^= 1; }
        continue;
      }
      // cross-entropy statistics of this row over the tile's columns
      float ce_m = -INFINITY, ce_s = 0.f;
      long ce_col = -1;  // target column relative to the tile, if inside
      if (MODE == kAllGatherGemmCE) ce_col = a.labels[row] - a.vocab_start - (long)ti.tn * BN;
      if (MODE == kReduceScatterGemm) {
        // foreign tile: wait once for the owner's ready; own tile: wait for all partials
        if (ti.chunk != a.rank && !((ready_mask >> ti.chunk) & 1u)) {
          if (leader) wait_flag(my_flags + kReadyOff + ti.chunk, epoch, a.err, a.timeout_ns, abort_flag);
          ready_mask |= 1u << ti.chunk;
          epilogue_bar();
        } else if (ti.chunk == a.rank) {
          if (leader) {
            const int* done = my_flags + kRsDoneOff + ti.local * kMaxRanks;
            for (int s = 0; s < a.world; ++s)
              if (s != a.rank && !wait_flag(done + s, epoch, a.err, a.timeout_ns, abort_flag)) break;
          }
          epilogue_bar();
        }
      }
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        if (MODE == kReduceScatterGemm && ti.chunk != a.rank && c == BN / 2) flush_half(ti, 0);
        uint32_t r[32];
        tmem_ld_32x32b_x32(t_row + c, r);
        tmem_wait_ld();
        const int col = ti.tn * BN + c;
        if (!is_ag<MODE>() && col >= a.N) continue;
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
        __nv_bfloat16* dst;
        if (MODE == kAllGatherGemmCE && col < a.N) {
          const int nv = min(32, a.N - col);
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __bfloat162float(__float2bfloat16_rn(v[j]));
          float mx = -INFINITY;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j < nv) mx = fmaxf(mx, v[j]);
          const float nm = fmaxf(ce_m, mx);
          const float nml = nm * kLog2e;
          float s0 = 0.f, s1 = 0.f;
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            if (j < nv) s0 += fast_exp2(fmaf(v[j], kLog2e, -nml));
            if (j + 1 < nv) s1 += fast_exp2(fmaf(v[j + 1], kLog2e, -nml));
          }
          ce_s = ce_s * fast_exp2((ce_m - nm) * kLog2e) + (s0 + s1);
          ce_m = nm;
          const long tc = ce_col - c;
          if (tc >= 0 && tc < nv) {
            float tv = 0.f;
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (j == tc) tv = v[j];
            a.ce_target[row] = tv;
          }
        }
        if (is_ag<MODE>()) {
          const int half = (c >> 5) & 1;
          uint8_t* buf = box_stg + (nbox & 1) * 4096;
          if (half == 0) {
            // the box stored from this buffer two boxes ago must have been read out
            if (lane == 0) bulk_wait_group_read<1>();
            __syncwarp();
          }
          uint8_t* brow = buf + lane * 128;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint4 u;
            u.x = pack_bf16x2(v[8 * j + 0], v[8 * j + 1]);
            u.y = pack_bf16x2(v[8 * j + 2], v[8 * j + 3]);
            u.z = pack_bf16x2(v[8 * j + 4], v[8 * j + 5]);
            u.w = pack_bf16x2(v[8 * j + 6], v[8 * j + 7]);
            *reinterpret_cast<uint4*>(brow + (((4 * half + j) ^ (lane & 7)) << 4)) = u;
          }
          if (half == 1) {
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              const int bcol = col - 32;
              if (bcol < a.N) tma_store_2d(&tmOut, buf, bcol, ti.tm * BM + quarter * 32);
              bulk_commit_group();
            }
            ++nbox;
          }
          continue;
        } else if (ti.chunk != a.rank) {
          // stage this thread's 32 columns (row `lane` of the warp's 32 rows);
          // 16-byte chunk j of a row sits at position j ^ (row % 8)
          uint8_t* srow = staging + (quarter * 32 + lane) * HALF_ROW;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint4 u;
            u.x = pack_bf16x2(v[8 * j + 0], v[8 * j + 1]);
            u.y = pack_bf16x2(v[8 * j + 2], v[8 * j + 3]);
            u.z = pack_bf16x2(v[8 * j + 4], v[8 * j + 5]);
            u.w = pack_bf16x2(v[8 * j + 6], v[8 * j + 7]);
            const int chunk = (c & (BN / 2 - 1)) / 8 + j;  // 16-byte chunk within the half row
            *reinterpret_cast<uint4*>(srow + ((chunk ^ (lane & 7)) << 4)) = u;
          }
          continue;
        } else {
          for (int s = 0; s < a.world; ++s) {
            if (s == a.rank) continue;
            const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(a.ws[a.rank] + a.recv_off) +
                                       ((long)s * a.m_chunk + row_local) * a.N + col;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              if (col + 8 * j < a.N) {
                const uint4 u = *reinterpret_cast<const uint4*>(src + 8 * j);
                float2 f;
                f = unpack_bf16x2(u.x); v[8 * j + 0] += f.x; v[8 * j + 1] += f.y;
                f = unpack_bf16x2(u.y); v[8 * j + 2] += f.x; v[8 * j + 3] += f.y;
                f = unpack_bf16x2(u.z); v[8 * j + 4] += f.x; v[8 * j + 5] += f.y;
                f = unpack_bf16x2(u.w); v[8 * j + 6] += f.x; v[8 * j + 7] += f.y;
              }
            }
          }
          dst = a.out + (long)row_local * a.ldo + col;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (col + 8 * j < a.N) {
            uint4 u;
            u.x = pack_bf16x2(v[8 * j + 0], v[8 * j + 1]);
            u.y = pack_bf16x2(v[8 * j + 2], v[8 * j + 3]);
            u.z = pack_bf16x2(v[8 * j + 4], v[8 * j + 5]);
            u.w = pack_bf16x2(v[8 * j + 6], v[8 * j + 7]);
            *reinterpret_cast<uint4*>(dst + 8 * j) = u;
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      if (MODE == kAllGatherGemmCE) a.ce_part[(long)ti.tn * a.M + row] = make_float2(ce_m, ce_s);
      if (MODE == kReduceScatterGemm && ti.chunk != a.rank) {
        flush_half(ti, 1);
        __threadfence_system();
        epilogue_bar();
        if (leader) st_release_sys(flags_of(a, ti.chunk) + kRsDoneOff + ti.local * kMaxRanks + a.rank, epoch);
      }
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
    }
    // every TMA store of an output box must be complete before the CTA goes
    if (is_ag<MODE>() && lane == 0) bulk_wait_group<0>();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

template <int MODE, bool B_MN>
cudaError_t launch(const FusedTpArgs& a, const void* B, long ldb, int num_sms, cudaStream_t stream) {
  auto kernel = fused_tp_kernel<MODE, B_MN>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<MODE>::SMEM);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  CUtensorMap ta_local, ta_gather, tb;
  if (is_ag<MODE>()) {
    if (!make_tmap_bf16_2d(&ta_local, a.a_local, a.K, a.m_chunk, a.lda_local, 64, BM)) return cudaErrorInvalidValue;
    if (a.world == 1) {
      ta_gather = ta_local;  // nothing to gather: no workspace is needed
    } else if (!make_tmap_bf16_2d(&ta_gather, a.ws[a.rank] + a.gather_off, a.K, a.M, a.K, 64, BM)) {
      return cudaErrorInvalidValue;
    }
  } else {
    if (!make_tmap_bf16_2d(&ta_local, a.a_local, a.K, a.M, a.lda_local, 64, BM)) return cudaErrorInvalidValue;
    ta_gather = ta_local;
  }
  if (!make_tmap_bf16_2d(&tb, B, B_MN ? a.N : a.K, B_MN ? a.K : a.N, ldb, 64, B_MN ? 64 : BN))
    return cudaErrorInvalidValue;
  constexpr bool swiglu = MODE == kAllGatherGemmSwiGLU;
  const int out_cols = swiglu ? a.N / 2 : a.N;
  CUtensorMap tout = tb;  // reduce-scatter writes its rows itself
  if (is_ag<MODE>() && !make_tmap_out_2d(&tout, a.out, false, out_cols, a.M, (uint64_t)a.ldo * 2, 32))
    return cudaErrorInvalidValue;
  CUtensorMap tg = tout, tu = tout;
  if (swiglu && a.gu != nullptr &&
      (!make_tmap_out_2d(&tg, a.gu, false, out_cols, a.M, (uint64_t)a.ldgu * 2, 32) ||
       !make_tmap_out_2d(&tu, a.gu + out_cols, false, out_cols, a.M, (uint64_t)a.ldgu * 2, 32)))
    return cudaErrorInvalidValue;
  const int num_n = swiglu ? (out_cols + BN / 2 - 1) / (BN / 2) : (a.N + BN - 1) / BN;
  const int tiles = a.world * (a.m_chunk / BM) * num_n;
  int grid = tiles < num_sms ? tiles : num_sms;
  if (grid > kMaxCtas) grid = kMaxCtas;
  kernel<<<grid, THREADS, Cfg<MODE>::SMEM, stream>>>(ta_local, ta_gather, tb, tout, tg, tu, a);
  return cudaGetLastError();
}

__device__ __forceinline__ void merge_lse(float& m, float& s, float m2, float s2) {
  const float nm = fmaxf(m, m2);
  if (nm == -INFINITY) return;
  s = s * __expf(m - nm) + s2 * __expf(m2 - nm);
  m = nm;
}

constexpr int CE_THREADS = 256;

__global__ void __launch_bounds__(CE_THREADS) ce_merge_kernel(const CeMergeArgs a) {
  const int row = blockIdx.x * CE_THREADS + threadIdx.x;
  const bool live = row < a.T;
  float m = -INFINITY, s = 0.f, t = 0.f;
  if (live) {
    for (int n = 0; n < a.num_n; ++n) {
      const float2 p = a.part[(long)n * a.T + row];
      merge_lse(m, s, p.x, p.y);
    }
    const long lbl = a.labels[row];
    if (lbl >= a.vocab_start && lbl < a.vocab_end) t = a.target_logit[row];
  }
  if (a.world > 1) {
    __shared__ int ok;
    __shared__ int abort_flag;
    const long slot = (long)(a.epoch & 1u) * kMaxRanks * a.T;
    if (live) {
      const float4 mine = make_float4(m, s, t, 0.f);
      for (int p = 0; p < a.world; ++p) {
        float4* dst = reinterpret_cast<float4*>(a.ws[p] + a.data_off) + slot + (long)a.rank * a.T;
        dst[row] = mine;
      }
      __threadfence_system();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence_system();
      for (int p = 0; p < a.world; ++p)
        if (p != a.rank)
          st_release_sys(reinterpret_cast<int*>(a.ws[p] + a.flags_off) + kCeFlagOff + a.rank * kMaxCeBlocks +
                             blockIdx.x,
                         (int)a.epoch);
      abort_flag = 0;
      ok = 1;
      const int* mine = reinterpret_cast<const int*>(a.ws[a.rank] + a.flags_off) + kCeFlagOff;
      for (int p = 0; p < a.world && ok; ++p)
        if (p != a.rank &&
            !wait_flag(mine + p * kMaxCeBlocks + blockIdx.x, (int)a.epoch, a.err, a.timeout_ns, &abort_flag))
          ok = 0;
    }
    __syncthreads();
    if (!ok || !live) return;
    const float4* src = reinterpret_cast<const float4*>(a.ws[a.rank] + a.data_off) + slot;
    m = -INFINITY;
    s = 0.f;
    t = 0.f;
    for (int p = 0; p < a.world; ++p) {
      const float4 q = __ldcv(src + (long)p * a.T + row);
      merge_lse(m, s, q.x, q.y);
      t += q.z;
    }
  }
  if (!live) return;
  a.loss[row] = logf(s) + m - t;
  a.gmax[row] = m;
  a.gsum[row] = s;
}

}  // namespace

cudaError_t ce_merge(const CeMergeArgs& a, cudaStream_t stream) {
  if (a.T <= 0) return cudaSuccess;
  const int blocks = (a.T + CE_THREADS - 1) / CE_THREADS;
  if (a.world < 1 || a.world > kMaxRanks || blocks > kMaxCeBlocks || a.epoch == 0) return cudaErrorInvalidValue;
  ce_merge_kernel<<<blocks, CE_THREADS, 0, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t fused_tp_gemm(int mode, const FusedTpArgs& a, const void* B, long ldb, bool b_mn, int num_sms,
                          cudaStream_t stream) {
  if (a.world < 1 || a.world > kMaxRanks || a.m_chunk % BM != 0 || a.M != a.m_chunk * a.world || a.N % 8 != 0 ||
      a.K % 8 != 0)
    return cudaErrorInvalidValue;
  if (mode == kReduceScatterGemm && (a.m_chunk / BM) * ((a.N + BN - 1) / BN) > kMaxTiles) return cudaErrorInvalidValue;
  if (mode == kAllGatherGemm) {
    return b_mn ? launch<kAllGatherGemm, true>(a, B, ldb, num_sms, stream)
                : launch<kAllGatherGemm, false>(a, B, ldb, num_sms, stream);
  }
  if (mode == kAllGatherGemmSwiGLU) {
    if (!b_mn || a.N % 16 != 0) return cudaErrorInvalidValue;  // F % 8 == 0: aligned up half
    return launch<kAllGatherGemmSwiGLU, true>(a, B, ldb, num_sms, stream);
  }
  if (mode == kAllGatherGemmCE) {
    if (a.labels == nullptr || a.ce_part == nullptr || a.ce_target == nullptr || b_mn) return cudaErrorInvalidValue;
    return launch<kAllGatherGemmCE, false>(a, B, ldb, num_sms, stream);
  }
  return b_mn ? launch<kReduceScatterGemm, true>(a, B, ldb, num_sms, stream)
              : launch<kReduceScatterGemm, false>(a, B, ldb, num_sms, stream);
}

}  // namespace nmb
