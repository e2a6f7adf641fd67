// Host-side helpers shared by the C-ABI entry points.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <utility>

#include "../../include/mvb200.h"

namespace mvb {

// Records `msg` as this thread's last error and returns `code`.
int fail(int code, const char* fmt, ...);

// Returns MVB_ERR_CUDA with the CUDA error string when `e` is an error, else MVB_OK.
int cuda_status(cudaError_t e, const char* what);

// Device address of the status word on the current device (looked up once per device).
unsigned* device_status_ptr();

// SM count of the current device (cached per device).
int current_sm_count();

// Programmatic-dependent-launch switch (mvb_set_pdl).
bool pdl_enabled();

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda needed).
int encode_tiled(CUtensorMap* map, CUtensorMapDataType dtype, uint32_t rank, const void* base,
                 const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swz);

inline size_t dtype_size(int dtype) {
  switch (dtype) {
    case MVB_F32: return 4;
    case MVB_F16: return 2;
    case MVB_BF16: return 2;
    case MVB_I32: return 4;
    case MVB_I64: return 8;
    default: return 0;
  }
}

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Launch `kernel` with the PDL attribute when enabled.
template <typename... KArgs, typename... Args>
int launch(const char* name, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
           Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  cfg.attrs = attr;
  cfg.numAttrs = 0;
  if (pdl_enabled()) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.numAttrs = 1;
  }
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  return cuda_status(e, name);
}

// Launch with a (cluster_x, 1, 1) thread-block cluster, plus the PDL attribute when enabled.
template <typename... KArgs, typename... Args>
int launch_cluster(const char* name, void (*kernel)(KArgs...), dim3 grid, dim3 block, unsigned cluster_x,
                   size_t smem, cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster_x;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (pdl_enabled()) {
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.numAttrs = 2;
  }
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  return cuda_status(e, name);
}

// Opt a kernel into more than 48 KB of dynamic shared memory (idempotent).
template <typename... KArgs>
int set_smem(void (*kernel)(KArgs...), size_t bytes, const char* name) {
  cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(kernel),
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
  return cuda_status(e, name);
}

}  // namespace mvb

#define MVB_REQUIRE(cond, ...)                                      \
  do {                                                              \
    if (!(cond)) return ::mvb::fail(MVB_ERR_INVALID_ARG, __VA_ARGS__); \
  } while (0)

#define MVB_TRY(expr)               \
  do {                              \
    int _mvb_rc = (expr);           \
    if (_mvb_rc != MVB_OK) return _mvb_rc; \
  } while (0)
