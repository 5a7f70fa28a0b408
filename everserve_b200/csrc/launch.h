// Kernel launches with the programmatic-dependent-launch attribute (and a cluster shape when asked).
//
// Every kernel of the decode chain is launched through `launch_ex`, so inside a captured CUDA graph
// each kernel's prologue (barrier set-up, TMEM allocation, weight prefetch) overlaps the tail of
// the kernel before it. ES_PDL=0 turns the attribute off (plain stream order).
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <cstdlib>
#include <utility>

namespace es {

inline bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("ES_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

// Kernel attributes (shared-memory size, cluster permissions) are set per device: `done` keeps one
// bit per device index, and `set_up` runs on the current device until it has succeeded there.
// Two threads may both run it for one device; setting an attribute twice is harmless.
template <typename F>
cudaError_t once_per_device(std::atomic<uint64_t>& done, F&& set_up) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = (dev >= 0 && dev < 64) ? (uint64_t(1) << dev) : 0;
  if (bit != 0 && (done.load(std::memory_order_acquire) & bit) != 0) return cudaSuccess;
  e = set_up();
  if (e == cudaSuccess && bit != 0) done.fetch_or(bit, std::memory_order_acq_rel);
  return e;
}

template <typename... KArgs, typename... Args>
cudaError_t launch_ex(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                      int cluster_z, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (cluster_z > 0) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = 1;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = (unsigned)cluster_z;
    n++;
  }
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    n++;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace es
