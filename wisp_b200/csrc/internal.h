// internal.h -- host-side helpers shared by the wisp_b200 translation units.
#pragma once

#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <utility>

#include "wisp_b200.h"

namespace wb {

// Launches a kernel of the per-layer chain in plain stream order (errors are
// left for cudaGetLastError).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                            cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = nullptr;
  cfg.numAttrs = 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// The same launch as a programmatic dependent of the kernel before it on the
// stream: its CTAs may start while that kernel is still running (once all of
// that kernel's CTAs have started and triggered), and must execute
// griddepcontrol.wait (wb::pdl_wait) before they read anything that kernel,
// or any kernel before it, writes. Used for one edge only, router logits ->
// decode planner in the single-GPU decode chain: measured on B200 (CUDA
// graph, L2 flushed), making the gate/up kernel a dependent of the planner
// cost Mixtral b1 6 us, and the down kernel a dependent of gate/up gained
// nothing.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_k_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// The register path's unit plans of one grouped call, as the decode planner
// (route.cu) writes them in place of the grouped call's own planner
// (grouped.cu): the plan arrays in the call's workspace and the numbers that
// shape them.
struct DecodeUnits {
  int32_t* units_gu;
  int32_t* units_dn;
  uint8_t* xq;   // q16 input rows in the same workspace
  int per_gu, per_dn, cols, sk_rows, ks_dn, nk_dn, target;
};

// Fill a WispErrCtx the way the reference's WISP_ERR_SET does
// (csrc/core/wisp_engine.h:66-72) and return the code.
inline WispError set_err(WispErrCtx* err, WispError code, const char* file, int line,
                         const char* fmt, ...) {
  if (err) {
    err->code = code;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(err->message, sizeof(err->message), fmt, ap);
    va_end(ap);
    err->file = file;
    err->line = line;
  }
  return code;
}

}  // namespace wb

#define WB_FAIL(code, ...) ::wb::set_err(err, code, __FILE__, __LINE__, __VA_ARGS__)

#define WB_CUDA_CHECK(call)                                                          \
  do {                                                                               \
    cudaError_t _e = (call);                                                         \
    if (_e != cudaSuccess)                                                           \
      return WB_FAIL(WISP_ERR_CUDA, "CUDA error: %s", cudaGetErrorString(_e));       \
  } while (0)
