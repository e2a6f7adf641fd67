// Tensor parallelism across the GPUs of one node, one process per GPU.
//
// The reference has only a stub here (distributed/tensor_parallel.py:14-35 raises for
// tp_size > 1); this is the Megatron-style split of the decode step that its design notes
// describe: column-parallel q/k/v and gate/up, row-parallel o_proj and down_proj, vocab-parallel
// lm_head.  The exchanges are done by the kernels themselves over NVLink peer memory:
//
//  * a row-parallel GEMM (mvb_tp_gemm_bf16 with a receive area) pushes its fp32 split-K
//    partials straight into the receive area of the rank that owns each batch row, then
//    signals every rank;
//  * mvb_tp_fused_add_rmsnorm_gemm on the owner sums the pushed partials over ranks, applies
//    residual + RMSNorm and writes the normalised rows into every rank's activation buffer
//    (all-gather), then signals;
//  * the next column-parallel GEMM waits for those signals before its activation loads;
//  * the vocab-parallel lm_head GEMM stores its logits columns into every rank's full logits
//    buffer, and mvb_tp_wait holds the sampler until all columns arrived, so every rank draws
//    the same tokens without a broadcast.
//
// Memory: one symmetric heap per rank (cudaMalloc at setup, shared with CUDA IPC); signal
// counters at offset 0.  No multicast objects and no TMA load ever reads a peer's memory: peer
// traffic is plain stores and the signal reductions.
#include <cstring>

#include "common.cuh"
#include "host.h"
#include "splitk.cuh"
#include "tp.cuh"

namespace mvb {

int gemm_launch(void* y, int64_t ldy, const void* x, int64_t ldx, const void* w, int64_t ldw, int64_t m, int64_t n,
                int64_t k, int epilogue, const void* aux, int64_t ld_aux, void* workspace, int64_t workspace_bytes,
                const TpGemm& tp, int64_t max_ctas, int* grid_out, mvb_stream_t stream);

namespace {

__global__ void tp_wait_kernel(const uint32_t* counters, int n, uint32_t count, const int32_t* epoch, unsigned* err) {
  pdl_launch_dependents();
  pdl_wait();
  if (threadIdx.x == 0) wait_counters(counters, n, static_cast<uint32_t>(*epoch) * count, err);
}

// Advances the step counter once the previous step's kernels are done with it.
__global__ void tp_begin_step_kernel(int32_t* epoch) {
  pdl_launch_dependents();
  pdl_wait();
  if (threadIdx.x == 0) *epoch += 1;
}

}  // namespace
}  // namespace mvb

using namespace mvb;

extern "C" int64_t mvb_tp_signal_bytes(void) { return kTpSignalBytes; }

extern "C" int mvb_tp_heap_alloc(int64_t bytes, void** base, void* ipc_handle) {
  MVB_REQUIRE(base && ipc_handle, "mvb_tp_heap_alloc: null pointer");
  MVB_REQUIRE(bytes >= kTpSignalBytes, "mvb_tp_heap_alloc: %lld bytes < the %lld-byte signal area", (long long)bytes,
              (long long)kTpSignalBytes);
  void* p = nullptr;
  MVB_TRY(cuda_status(cudaMalloc(&p, static_cast<size_t>(bytes)), "mvb_tp_heap_alloc: cudaMalloc"));
  cudaIpcMemHandle_t h;
  int rc = cuda_status(cudaMemset(p, 0, static_cast<size_t>(bytes)), "mvb_tp_heap_alloc: cudaMemset");
  if (rc == MVB_OK) rc = cuda_status(cudaIpcGetMemHandle(&h, p), "mvb_tp_heap_alloc: cudaIpcGetMemHandle");
  if (rc == MVB_OK) rc = cuda_status(cudaDeviceSynchronize(), "mvb_tp_heap_alloc: synchronize");
  if (rc != MVB_OK) {
    cudaFree(p);
    return rc;
  }
  std::memcpy(ipc_handle, &h, sizeof(h));
  *base = p;
  return MVB_OK;
}

extern "C" int mvb_tp_heap_free(void* base) {
  if (!base) return MVB_OK;
  return cuda_status(cudaFree(base), "mvb_tp_heap_free");
}

extern "C" int mvb_tp_comm_init(int rank, int nranks, void* local_base, const void* ipc_handles, int64_t heap_bytes,
                                mvb_tp_comm** out) {
  MVB_REQUIRE(out && local_base && ipc_handles, "mvb_tp_comm_init: null pointer");
  MVB_REQUIRE(nranks >= 1 && nranks <= kTpMaxRanks && rank >= 0 && rank < nranks,
              "mvb_tp_comm_init: rank %d of %d (at most %d ranks)", rank, nranks, kTpMaxRanks);
  MVB_REQUIRE(heap_bytes >= kTpSignalBytes, "mvb_tp_comm_init: heap too small");
  static_assert(sizeof(cudaIpcMemHandle_t) == MVB_TP_IPC_HANDLE_BYTES, "IPC handle size");
  mvb_tp_comm* c = new mvb_tp_comm();
  std::memset(c, 0, sizeof(*c));
  c->rank = rank;
  c->nranks = nranks;
  c->heap_bytes = heap_bytes;
  c->epoch = reinterpret_cast<int32_t*>(static_cast<char*>(local_base) + kTpEpochOffset);
  cudaGetDevice(&c->device);
  const char* hs = static_cast<const char*>(ipc_handles);
  for (int q = 0; q < nranks; ++q) {
    if (q == rank) {
      c->base[q] = static_cast<char*>(local_base);
      continue;
    }
    cudaIpcMemHandle_t h;
    std::memcpy(&h, hs + static_cast<size_t>(q) * MVB_TP_IPC_HANDLE_BYTES, sizeof(h));
    void* p = nullptr;
    const int rc = cuda_status(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess),
                               "mvb_tp_comm_init: cudaIpcOpenMemHandle");
    if (rc != MVB_OK) {
      for (int r = 0; r < q; ++r)
        if (c->opened[r]) cudaIpcCloseMemHandle(c->base[r]);
      delete c;
      return rc;
    }
    c->base[q] = static_cast<char*>(p);
    c->opened[q] = true;
  }
  *out = c;
  return MVB_OK;
}

extern "C" int mvb_tp_comm_destroy(mvb_tp_comm* comm) {
  if (!comm) return MVB_OK;
  int rc = MVB_OK;
  for (int q = 0; q < comm->nranks; ++q)
    if (comm->opened[q]) {
      const int r = cuda_status(cudaIpcCloseMemHandle(comm->base[q]), "mvb_tp_comm_destroy");
      if (rc == MVB_OK) rc = r;
    }
  delete comm;
  return rc;
}

extern "C" int64_t mvb_tp_recv_bytes(int64_t m, int64_t n, int64_t k, int nranks, int device) {
  int sms = mvb_num_sms(device);
  if (sms <= 0) sms = 148;
  if (nranks <= 0 || m % nranks != 0 || k % kSplitBK != 0) return -1;
  return splitk_push_bytes(splitk_plan_push(m, n, k, sms, nranks), nranks, static_cast<int>(m / nranks));
}

extern "C" int mvb_tp_gemm_bf16(mvb_tp_comm* comm, const void* x, int64_t ldx, const void* w, int64_t ldw, int64_t m,
                                int64_t n, int64_t k, int epilogue, void* workspace, int64_t workspace_bytes,
                                int64_t out_offset, int64_t ldy, int wait_point, int signal_point,
                                mvb_stream_t stream) {
  MVB_REQUIRE(comm, "mvb_tp_gemm_bf16: null communicator");
  const int nr = comm->nranks;
  MVB_REQUIRE(wait_point >= -1 && wait_point < kTpMaxPoints && signal_point >= -1 && signal_point < kTpMaxPoints,
              "mvb_tp_gemm_bf16: bad signal points");
  MVB_REQUIRE(wait_point < 0 || comm->point_count[wait_point] > 0, "mvb_tp_gemm_bf16: nothing signals point %d",
              wait_point);
  TpGemm tp{};
  tp.nranks = nr;
  tp.rank = comm->rank;
  tp.epoch = comm->epoch;
  if (wait_point >= 0) {
    tp.wait = comm->wait_row(wait_point);
    tp.wait_count = comm->point_count[wait_point];
  }
  const bool push = epilogue == MVB_EPI_PARTIALS && out_offset >= 0;
  const bool gather = epilogue == MVB_EPI_STORE && out_offset >= 0;
  MVB_REQUIRE(out_offset < 0 || push || gather,
              "mvb_tp_gemm_bf16: an output offset needs MVB_EPI_PARTIALS (push) or MVB_EPI_STORE (all-gather)");
  MVB_REQUIRE((signal_point >= 0) == (push || gather), "mvb_tp_gemm_bf16: push / all-gather calls signal a point");
  MVB_REQUIRE(epilogue != MVB_EPI_STORE || gather, "mvb_tp_gemm_bf16: MVB_EPI_STORE needs an output offset");
  if (push) {
    MVB_REQUIRE(m % nr == 0, "mvb_tp_gemm_bf16: m %lld not a multiple of %d ranks", (long long)m, nr);
    const int sms = current_sm_count();
    MVB_REQUIRE(sms > 0, "mvb_tp_gemm_bf16: no device");
    tp.rows_per_rank = static_cast<int>(m / nr);
    const int64_t need = splitk_push_bytes(splitk_plan_push(m, n, k, sms, nr), nr, tp.rows_per_rank);
    MVB_REQUIRE(out_offset >= kTpSignalBytes && out_offset % 16 == 0 && out_offset + need <= comm->heap_bytes,
                "mvb_tp_gemm_bf16: receive area outside the heap");
    for (int q = 0; q < nr; ++q) tp.recv[q] = reinterpret_cast<float*>(comm->base[q] + out_offset);
  }
  if (gather) {
    MVB_REQUIRE(ldy >= n && out_offset >= kTpSignalBytes && out_offset % 2 == 0 &&
                    out_offset + ((m - 1) * ldy + n) * 2 <= comm->heap_bytes,
                "mvb_tp_gemm_bf16: all-gather output outside the heap");
    for (int q = 0; q < nr; ++q) tp.y[q] = reinterpret_cast<__nv_bfloat16*>(comm->base[q] + out_offset);
  }
  if (signal_point >= 0) {
    for (int q = 0; q < nr; ++q) tp.signal[q] = comm->signal_slot(q, signal_point);
    tp.arrive = comm->arrive_slot(signal_point);
    const int sms = current_sm_count();
    MVB_REQUIRE(sms > 0, "mvb_tp_gemm_bf16: no device");
    const int64_t tiles = epilogue == MVB_EPI_SWIGLU_PARTIALS ? (n / 2 + 63) / 64 : (n + kSplitBM - 1) / kSplitBM;
    const int64_t total = tiles * (k / kSplitBK);
    int64_t ctas = push ? splitk_push_ctas(m, n, k, sms, nr) : splitk_ctas(m, sms);
    if (gather && ctas > tiles * 16) ctas = tiles * 8;  // the merge path's contributor cap (gemm_launch)
    tp.arrive_total = static_cast<uint32_t>(total < ctas ? total : ctas);   // the GEMM's grid
  }
  int grid = 0;
  const int64_t max_ctas = push ? splitk_push_ctas(m, n, k, current_sm_count(), nr) : 0;
  MVB_TRY(gemm_launch(nullptr, gather ? ldy : 0, x, ldx, w, ldw, m, n, k, epilogue, nullptr, 0, workspace,
                      workspace_bytes, tp, max_ctas, &grid, stream));
  if (signal_point >= 0) {
    MVB_REQUIRE(static_cast<uint32_t>(grid) == tp.arrive_total, "mvb_tp_gemm_bf16: grid mismatch");
    comm->point_count[signal_point] = 1;
  }
  return MVB_OK;
}

extern "C" int mvb_tp_wait(mvb_tp_comm* comm, int point, mvb_stream_t stream) {
  MVB_REQUIRE(comm && point >= 0 && point < kTpMaxPoints, "mvb_tp_wait: bad arguments");
  MVB_REQUIRE(comm->point_count[point] > 0, "mvb_tp_wait: nothing signals point %d", point);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  return launch("tp_wait", tp_wait_kernel, dim3(1), dim3(32), 0, st, comm->wait_row(point), comm->nranks,
                comm->point_count[point], comm->epoch, device_status_ptr());
}

extern "C" int mvb_tp_begin_step(mvb_tp_comm* comm, mvb_stream_t stream) {
  MVB_REQUIRE(comm, "mvb_tp_begin_step: null communicator");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  return launch("tp_begin_step", tp_begin_step_kernel, dim3(1), dim3(32), 0, st, comm->epoch);
}
