// Library status, error messages, device status word, tensor-map encoding.
#include <atomic>
#include <mutex>
#include <utility>

#include "common.cuh"
#include "host.h"

// One status word per device that loads the library.  Kernels receive its address
// (mvb::device_status_ptr) and OR MVB_DEV_* bits into it instead of faulting.
__device__ unsigned int g_mvb_device_status;

namespace mvb {

namespace {
thread_local char g_msg[512] = "";
std::atomic<int> g_pdl{0};
constexpr int kMaxDevices = 64;
unsigned* g_status_ptr[kMaxDevices] = {};
int g_sms[kMaxDevices] = {};
std::mutex g_mu;

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;
}  // namespace

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return MVB_OK;
  return fail(MVB_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

static int current_device() {
  int dev = 0;
  cudaGetDevice(&dev);
  return dev;
}

unsigned* device_status_ptr() {
  int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return nullptr;
  if (g_status_ptr[dev] == nullptr) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_status_ptr[dev] == nullptr) {
      void* p = nullptr;
      if (cudaGetSymbolAddress(&p, g_mvb_device_status) != cudaSuccess) return nullptr;
      g_status_ptr[dev] = static_cast<unsigned*>(p);
    }
  }
  return g_status_ptr[dev];
}

int current_sm_count() {
  int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return 0;
  if (g_sms[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    g_sms[dev] = n;
  }
  return g_sms[dev];
}

bool pdl_enabled() { return g_pdl.load(std::memory_order_relaxed) != 0; }

int encode_tiled(CUtensorMap* map, CUtensorMapDataType dtype, uint32_t rank, const void* base, const uint64_t* dims,
                 const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swz) {
  if (g_encode == nullptr) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_encode == nullptr) {
      void* fn = nullptr;
      cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
      cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
      if (e != cudaSuccess || fn == nullptr || q != cudaDriverEntryPointSuccess)
        return fail(MVB_ERR_DRIVER, "cuTensorMapEncodeTiled entry point unavailable");
      g_encode = reinterpret_cast<EncodeTiledFn>(fn);
    }
  }
  cuuint64_t d[5];
  cuuint64_t s[4];
  cuuint32_t b[5];
  cuuint32_t es[5];
  for (uint32_t i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    es[i] = 1;
    if (i + 1 < rank) s[i] = strides_bytes[i];
  }
  CUresult r = g_encode(map, dtype, rank, const_cast<void*>(base), d, s, b, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MVB_ERR_INVALID_ARG, "cuTensorMapEncodeTiled failed (CUresult %d)", int(r));
  return MVB_OK;
}

}  // namespace mvb

extern "C" {

const char* mvb_last_error(void) { return mvb::g_msg; }

int mvb_version(void) { return 1; }

int mvb_num_sms(int device) {
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return 0;
  return n;
}

int mvb_set_pdl(int enable) { return mvb::g_pdl.exchange(enable ? 1 : 0); }

int mvb_device_status(unsigned int* status, int clear, mvb_stream_t stream) {
  MVB_REQUIRE(status != nullptr, "mvb_device_status: status is NULL");
  unsigned* p = mvb::device_status_ptr();
  if (p == nullptr) return mvb::fail(MVB_ERR_CUDA, "device status word unavailable");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  MVB_TRY(mvb::cuda_status(cudaMemcpyAsync(status, p, sizeof(unsigned), cudaMemcpyDeviceToHost, st),
                           "mvb_device_status: read"));
  MVB_TRY(mvb::cuda_status(cudaStreamSynchronize(st), "mvb_device_status: sync"));
  if (clear) {
    MVB_TRY(mvb::cuda_status(cudaMemsetAsync(p, 0, sizeof(unsigned), st), "mvb_device_status: clear"));
    MVB_TRY(mvb::cuda_status(cudaStreamSynchronize(st), "mvb_device_status: sync"));
  }
  return MVB_OK;
}

}  // extern "C"
