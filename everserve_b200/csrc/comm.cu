// Failure-detecting all-reduce ("fdar"): sum a bf16 vector over the members of a tensor-parallel
// group through peer memory, in member order, with bounded waits (see comm.cuh for the protocol).
//
// One CTA per chunk of kChunk elements: it pushes its chunk into every member's buffer at its own
// sender row with 16-byte stores over NVLink, publishes one flag per member (system-scope release
// after a system fence), waits on its own buffer for every member's flag of the chunk, then sums
// the members' chunks in member order in fp32 (one rounding) into `out`. Decode-size tensors (up
// to 1 Mi elements, the data region of one sender) take this path; larger ones go to NCCL.
#include "api.h"
#include "comm.cuh"

namespace es {
namespace comm {
namespace {

constexpr int kThreads = 256;
constexpr int kChunk = 4096;  // elements per CTA and flag slot

__global__ void __launch_bounds__(kThreads) fdar_kernel(const __nv_bfloat16* __restrict__ inp,
                                                        __nv_bfloat16* __restrict__ out, int n, View v) {
  __shared__ uint32_t s_seq;
  __shared__ int s_order[kMaxRows];
  __shared__ int s_count;
  __shared__ int s_fail;
  if (threadIdx.x == 0) {
    s_seq = v.call[0] + 1;
    const int c = v.order[0];
    s_count = c < 0 ? 0 : (c > kMaxRows ? kMaxRows : c);
    for (int i = 0; i < s_count; i++) s_order[i] = v.order[1 + i];
    s_fail = kOk;
  }
  __syncthreads();
  const uint32_t seq = s_seq, parity = seq & 1u;
  const int count = s_count;
  const int c = blockIdx.x;
  const int e0 = c * kChunk, e1 = min(n, e0 + kChunk);
  const int nvec = (e1 - e0) / 8;  // whole 16-byte vectors; the tail goes element by element
  const uint64_t my_base = v.peers[v.row];
  // push this member's chunk to every member
  const uint4* src = reinterpret_cast<const uint4*>(inp + e0);
  for (int k = 0; k < count; k++) {
    uint4* dst = reinterpret_cast<uint4*>(data_ptr(v.peers[s_order[k]], parity, v.row) + (size_t)e0 * 2);
    for (int i = threadIdx.x; i < nvec; i += kThreads) dst[i] = src[i];
    __nv_bfloat16* dt = reinterpret_cast<__nv_bfloat16*>(dst);
    for (int i = e0 + nvec * 8 + threadIdx.x; i < e1; i += kThreads) dt[i - e0] = inp[i];
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < count) st_release_sys(flag_ptr(v.peers[s_order[threadIdx.x]], parity, v.row, c), seq);
  if (threadIdx.x == 0) s_fail = wait_members(v, my_base, parity, c, seq, s_order, count);
  __syncthreads();
  if (s_fail == kOk) {
    for (int i = threadIdx.x; i < nvec; i += kThreads) {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int k = 0; k < count; k++) {
        const uint4 w = reinterpret_cast<const uint4*>(data_ptr(my_base, parity, s_order[k]) + (size_t)e0 * 2)[i];
        float f[8];
        unpack8(w, f);
#pragma unroll
        for (int j = 0; j < 8; j++) acc[j] += f[j];
      }
      reinterpret_cast<uint4*>(out + e0)[i] = pack8(acc);
    }
    for (int i = e0 + nvec * 8 + threadIdx.x; i < e1; i += kThreads) {
      float acc = 0.f;
      for (int k = 0; k < count; k++)
        acc += bf2f(reinterpret_cast<const __nv_bfloat16*>(data_ptr(my_base, parity, s_order[k]))[i]);
      out[i] = f2bf(acc);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) finish_call(v, seq, s_fail);
}

}  // namespace
}  // namespace comm

int64_t comm_buffer_bytes() { return (int64_t)comm::kBufferBytes; }
int64_t comm_max_elems() { return (int64_t)(comm::kDataBytes / 2); }

cudaError_t launch_fdar(const void* inp, void* out, int64_t n, const CommArgs& c, cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  if (n > comm_max_elems() || reinterpret_cast<uintptr_t>(inp) % 16 != 0 || reinterpret_cast<uintptr_t>(out) % 16 != 0)
    return cudaErrorInvalidValue;
  comm::View v{};
  v.peers = c.peers;
  v.order = c.order;
  v.call = c.call;
  v.ctrl = reinterpret_cast<comm::Ctrl*>(c.ctrl);
  v.row = c.row;
  const int grid = (int)((n + comm::kChunk - 1) / comm::kChunk);
  comm::fdar_kernel<<<grid, comm::kThreads, 0, stream>>>(static_cast<const __nv_bfloat16*>(inp),
                                                         static_cast<__nv_bfloat16*>(out), (int)n, v);
  return cudaGetLastError();
}

}  // namespace es
