// Shared device helpers for the everserve_b200 sm_100a kernels.
//
// Everything here is written for one target: sm_100a (B200). Vector widths assume 16-byte
// aligned rows; callers check alignment on the host before launching.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define ES_DEVICE __device__ __forceinline__

namespace es {

// Status words a kernel writes when it gives up a bounded wait. The host reads them after the
// launch; a non-zero word means the result is not valid and the context is still usable.
enum Status : int32_t {
  kOk = 0,
  kTimeout = 1,      // a bounded wait ran out (peer flag, mbarrier)
  kAborted = 2,      // the host raised the abort word
  kBadShape = 3,     // a launch-time check failed on the device side
  kDead = 4,         // a member awaited stopped its heartbeat (its process is gone)
};

ES_DEVICE uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Programmatic dependent launch (PDL). A kernel launched with the programmatic-serialization
// attribute may start while the previous kernel of its stream finishes. `pdl_wait` blocks the
// calling thread until that kernel has completed and its writes are visible: every read of data a
// previous kernel produced, and every global write, comes after it. Only reads of data no kernel
// of the step writes (weights) may come before. `pdl_launch` lets the next kernel start launching;
// kernels call it after their wait, so at most two kernels of a stream overlap. Both are no-ops
// for a launch without the attribute.
ES_DEVICE void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
ES_DEVICE void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

ES_DEVICE float bf2f(__nv_bfloat16 x) { return __bfloat162float(x); }
ES_DEVICE __nv_bfloat16 f2bf(float x) { return __float2bfloat16_rn(x); }

// Unpack eight bf16 held in a uint4 into fp32.
ES_DEVICE void unpack8(const uint4& v, float* f) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; i++) {
    float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

ES_DEVICE uint4 pack8(const float* f) {
  uint4 v;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; i++) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return v;
}

ES_DEVICE float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

ES_DEVICE float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum for blockDim.x <= 1024; `red` holds at least 32 floats.
ES_DEVICE float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  const int nw = (blockDim.x + 31) >> 5;
  float t = (threadIdx.x < nw) ? red[threadIdx.x] : 0.f;
  if (warp == 0) t = warp_sum(t);
  if (threadIdx.x == 0) red[0] = t;
  __syncthreads();
  return red[0];
}

// System-scope acquire/release for flags that other GPUs write or read over NVLink.
ES_DEVICE uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Spin loads: relaxed (no ordering per iteration); the waiter orders what follows with one
// fence_acquire_sys once the value it waits for has arrived.
ES_DEVICE uint32_t ld_relaxed_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
ES_DEVICE void fence_acquire_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
ES_DEVICE void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
ES_DEVICE uint64_t ld_volatile_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
ES_DEVICE int64_t ld_volatile_i64(const int64_t* p) {
  int64_t v;
  asm volatile("ld.volatile.global.s64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

}  // namespace es
