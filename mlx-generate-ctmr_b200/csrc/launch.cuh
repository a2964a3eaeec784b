// Kernel launches with programmatic dependent launch (PDL).
//
// Every kernel of this library is launched with the stream attribute that lets
// it start while the previous kernel in the stream is still finishing, and
// every kernel calls griddep_wait() before it touches global memory (the
// persistent conv kernels after their shared-memory / TMEM set-up). The wait
// returns once the preceding grid has completed and its writes are visible, so
// the ordering of a plain launch is kept while the launch latency and the
// set-up overlap the predecessor's tail. Each kernel signals
// griddep_launch_dependents() right away: its successor may then be scheduled
// as soon as this grid's last blocks are resident. Inside a CUDA-graph capture
// the attribute becomes a programmatic edge. CTMR_DISABLE_PDL=1 turns it off.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cstdlib>
#include <utility>

namespace ctmr {

__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }

// Streaming multiprocessors of the current device: the unit every grid-size plan of this
// library is measured in (148 on a B200). Queried once per device.
inline int device_sm_count() {
  static std::atomic<int> cached[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return 148;
  if (dev < 64) {
    const int hit = cached[dev].load(std::memory_order_relaxed);
    if (hit > 0) return hit;
  }
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n < 1) return 148;
  if (dev < 64) cached[dev].store(n, std::memory_order_relaxed);
  return n;
}

inline bool pdl_enabled() {
  static const bool on = std::getenv("CTMR_DISABLE_PDL") == nullptr;
  return on;
}

template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                          Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

}  // namespace ctmr
