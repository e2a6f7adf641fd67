// Tensor-parallel plumbing shared by the kernels that exchange data between GPUs.
//
// One process per GPU.  Every rank allocates one "symmetric heap" of the same size and layout
// and shares it through CUDA IPC; a buffer is named by its byte offset in the heap, the same on
// every rank.  Offset 0 holds the signal counters: uint32 [kTpMaxPoints][kTpMaxRanks], where
// counter [p][s] in rank q's heap counts the CTAs of rank s that finished their part of signal
// point p for q (see the cross-GPU signal helpers in common.cuh); after them sits the rank's
// step counter ("epoch"), advanced on the device at the start of every step.
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

#include "common.cuh"
#include "splitk.cuh"

namespace mvb {

constexpr int kTpMaxRanks = 8;
constexpr int kTpMaxPoints = 1024;
// Signal counters, then this rank's step counter (int32 at kTpEpochOffset), then this rank's
// per-point CTA arrival counters (uint32 [kTpMaxPoints] at kTpArriveOffset).
constexpr int64_t kTpEpochOffset = static_cast<int64_t>(kTpMaxPoints) * kTpMaxRanks * 4;
constexpr int64_t kTpArriveOffset = kTpEpochOffset + 256;
constexpr int64_t kTpSignalBytes = kTpArriveOffset + static_cast<int64_t>(kTpMaxPoints) * 4;

// Called by one thread of each CTA of a signalling kernel, after a barrier over the CTA's
// stores.  The CTAs meet on a local (GPU-scope, acquire-release) arrival counter; the last of
// the `ctas` re-arms it and releases, at system scope, the stores of all of them to every rank
// (one increment of each rank's counter per launch): one system-scope release fence, cumulative
// over what the last CTA acquired, then a relaxed increment per rank.
__device__ __forceinline__ void signal_ranks_once(uint32_t* arrive, uint32_t ctas, uint32_t* const* signal,
                                                  int nranks) {
  uint32_t old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(arrive) : "memory");
  if (old == ctas - 1) {
    asm volatile("st.relaxed.gpu.global.u32 [%0], 0;" ::"l"(arrive) : "memory");
    fence_acq_rel_sys();
    for (int q = 0; q < nranks; ++q) signal_add_relaxed_sys(signal[q]);
  }
}

// Extra arguments of a tensor-parallel GEMM (nranks == 0: an ordinary call).
struct TpGemm {
  int nranks;
  int rank;
  int rows_per_rank;                    // batch rows each rank owns (push mode)
  float* recv[kTpMaxRanks];             // push mode: each rank's receive area for this call
  __nv_bfloat16* y[kTpMaxRanks];        // all-gather mode: each rank's output, this rank's columns
  uint32_t* signal[kTpMaxRanks];        // each rank's counter [point][this rank], or all null
  uint32_t* arrive;                     // this rank's arrival counter of the signal point
  uint32_t arrive_total;                // CTAs of this launch
  const uint32_t* wait;                 // this rank's counters [point][0..nranks) X waits for, or null
  uint32_t wait_count;                  // CTAs per rank that signal the awaited point each step
  const int32_t* epoch;                 // device: current step number (>= 1)
};

// Receive-area layout of pushed split-K partials: [src rank][tile][contributor][owned row][128].
__host__ __device__ __forceinline__ int64_t sk_push_offset(const SplitKPlan& p, int src, int t, int j, int rpr,
                                                           int bl, int r) {
  return ((((static_cast<int64_t>(src) * p.tiles + t) * p.maxc + j) * rpr + bl) * kSplitBM + r);
}

inline int64_t splitk_push_bytes(const SplitKPlan& p, int nranks, int rpr) {
  return static_cast<int64_t>(nranks) * p.tiles * p.maxc * rpr * kSplitBM * 4;
}

}  // namespace mvb

// Host-side communicator behind the C ABI's opaque mvb_tp_comm.
struct mvb_tp_comm {
  int rank;
  int nranks;
  int device;
  int64_t heap_bytes;
  char* base[mvb::kTpMaxRanks];     // every rank's heap as mapped in this process
  bool opened[mvb::kTpMaxRanks];    // mapped through cudaIpcOpenMemHandle (closed on destroy)
  int32_t* epoch;                   // device step counter (in the local heap) read by every waiting kernel
  uint32_t point_count[mvb::kTpMaxPoints];  // signals per rank per step at each point (set at launch)

  uint32_t* signal_slot(int q, int point) const {
    return reinterpret_cast<uint32_t*>(base[q]) + static_cast<int64_t>(point) * mvb::kTpMaxRanks + rank;
  }
  uint32_t* arrive_slot(int point) const {
    return reinterpret_cast<uint32_t*>(base[rank] + mvb::kTpArriveOffset) + point;
  }
  const uint32_t* wait_row(int point) const {
    return reinterpret_cast<const uint32_t*>(base[rank]) + static_cast<int64_t>(point) * mvb::kTpMaxRanks;
  }
};
