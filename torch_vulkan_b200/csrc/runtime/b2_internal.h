// Internal helpers shared by the runtime and the kernel translation units of libb2rt.so.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../../include/b2rt.h"

namespace b2 {

// Per-thread last error (b2rt_last_error). Returns `code` so callers can `return fail(...)`.
int fail(int code, const std::string& msg);
int fail_cuda(cudaError_t e, const char* what);
inline int check_cuda(cudaError_t e, const char* what) { return e == cudaSuccess ? 0 : fail_cuda(e, what); }

// Device properties cached by b2rt_init (called lazily by every entry point).
struct DeviceInfo {
  int device = -1;
  int sm_count = 0;
  int smem_optin = 0;  // max dynamic shared memory per block (bytes)
  int cc_major = 0, cc_minor = 0;
  bool tcgen05 = false;  // sm_100a kernels usable (compute capability 10.0)
  bool coop_launch = false;  // cooperative launches (every CTA of a grid resident at once) supported
};
const DeviceInfo& device_info();  // initialises on first use; device < 0 when no GPU
int ensure_init();

// Launch bookkeeping: counts launches, and when profiling is on brackets the launch with events.
struct LaunchScope {
  const char* name;
  cudaStream_t stream;
  cudaEvent_t ev0 = nullptr;
  explicit LaunchScope(const char* kernel_name, cudaStream_t s);
  ~LaunchScope();
};
// Checks cudaGetLastError after a launch.
int after_launch(const char* what);

// Programmatic dependent launch: a kernel launched this way may start (prologue: barrier init,
// descriptor prefetch) while the previous kernel on the stream drains; it calls griddepcontrol.wait
// before touching global memory or tensor memory. Eager launches only; off with B2_NO_PDL=1.
bool pdl_enabled();

template <typename... KArgs, typename... Args>
int launch_pdl(const char* name, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
               Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  // Under stream capture the plain edge is kept: replaying a graph whose kernel nodes carry
  // programmatic edges measured slower on B200 than the same graph without them.
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (pdl_enabled() && cudaStreamIsCapturing(st, &cs) != cudaSuccess) {
    (void)cudaGetLastError();
    cs = cudaStreamCaptureStatusActive;
  }
  cfg.numAttrs = (pdl_enabled() && cs == cudaStreamCaptureStatusNone) ? 1 : 0;
  cudaError_t e;
  {
    LaunchScope ls(name, st);
    e = cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
  }
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return fail_cuda(e, name);
  }
  return after_launch(name);
}

// Device error word (bounded waits that expired write a non-zero code here).
int* device_error_ptr();
void stat_add(int id, uint64_t v);

inline size_t dtype_size(int dt) {
  switch (dt) {
    case B2_F32: return 4;
    case B2_BF16: return 2;
    case B2_F16: return 2;
    case B2_F64: return 8;
    case B2_I8: return 1;
    default: return 0;
  }
}

}  // namespace b2
