// Failure-detecting all-reduce ("fdar"): sum a bf16 vector over the members of a tensor-parallel
// group through peer memory, in member order, with bounded waits (see comm.cuh for the protocol).
//
// One CTA per chunk of kChunk elements: it pushes its chunk into every member's buffer at its own
// sender row with 16-byte stores over NVLink, publishes one flag per member (system-scope release
// after a system fence), waits on its own buffer for every member's flag of the chunk, then sums
// the members' chunks in member order in fp32 (one rounding) into `out`. Decode-size tensors (up
// to 1 Mi elements, the data region of one sender) take this path; larger ones go to NCCL.
#include "api.h"
#include "launch.h"
#include "comm.cuh"

namespace es {
namespace comm {
namespace {

constexpr int kThreads = 256;
constexpr int kChunk = 4096;  // elements per CTA and flag slot

__global__ void __launch_bounds__(kThreads) fdar_kernel(const __nv_bfloat16* __restrict__ inp,
                                                        __nv_bfloat16* __restrict__ out, int n, View v) {
  pdl_wait();
  pdl_launch();
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
  if (v.mc) {
    // NVLS: one multicast store per vector reaches every member (the tail in whole words too)
    uint4* dst = reinterpret_cast<uint4*>(data_ptr(v.mc, parity, v.row) + (size_t)e0 * 2);
    for (int i = threadIdx.x; i < nvec; i += kThreads) mc_st_v4(dst + i, src[i]);
    if (threadIdx.x == 0 && e1 > e0 + nvec * 8) {
      uint4 t = make_uint4(0, 0, 0, 0);
      __nv_bfloat16* tb = reinterpret_cast<__nv_bfloat16*>(&t);
      for (int i = e0 + nvec * 8; i < e1; i++) tb[i - e0 - nvec * 8] = inp[i];
      mc_st_v4(dst + nvec, t);
    }
  } else {
    for (int k = 0; k < count; k++) {
      uint4* dst = reinterpret_cast<uint4*>(data_ptr(v.peers[s_order[k]], parity, v.row) + (size_t)e0 * 2);
      for (int i = threadIdx.x; i < nvec; i += kThreads) dst[i] = src[i];
      __nv_bfloat16* dt = reinterpret_cast<__nv_bfloat16*>(dst);
      for (int i = e0 + nvec * 8 + threadIdx.x; i < e1; i += kThreads) dt[i - e0] = inp[i];
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) __threadfence_system();
  __syncthreads();
  if (v.mc) {
    if (threadIdx.x == 0) mc_st_release_u32(flag_ptr(v.mc, parity, v.row, c), seq);
  } else if (threadIdx.x < count) {
    st_release_sys(flag_ptr(v.peers[s_order[threadIdx.x]], parity, v.row, c), seq);
  }
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

// LL all-reduce for small tensors: each 8-byte word carries two bf16 and the block's call number,
// so a word is its own flag: no fence, no flag round trip, no end-of-call counter. One thread per
// word; every block keeps its own call counter, so its words' region and parity are its own.
constexpr int kLLThreads = 256;

__global__ void __launch_bounds__(kLLThreads) fdar_ll_kernel(const __nv_bfloat16* __restrict__ inp,
                                                             __nv_bfloat16* __restrict__ out, int n, View v) {
  pdl_wait();
  pdl_launch();
  __shared__ uint32_t s_seq;
  __shared__ int s_order[kMaxRows];
  __shared__ int s_count;
  if (threadIdx.x == 0) {
    uint32_t* ctr = v.seqs + kSeqSlots + blockIdx.x;
    s_seq = *ctr + 1;
    *ctr = s_seq;
    const int c = v.order[0];
    s_count = c < 0 ? 0 : (c > kMaxRows ? kMaxRows : c);
    for (int i = 0; i < s_count; i++) s_order[i] = v.order[1 + i];
  }
  __syncthreads();
  const uint32_t seq = s_seq, parity = seq & 1u;
  const int count = s_count;
  const int i = blockIdx.x * kLLThreads + threadIdx.x;  // word index
  const int n2 = (n + 1) / 2;
  if (i >= n2) return;
  const bool pair = 2 * i + 1 < n;
  const uint32_t lo = __bfloat16_as_ushort(inp[2 * i]);
  const uint32_t hi = pair ? __bfloat16_as_ushort(inp[2 * i + 1]) : 0u;
  const uint64_t word = ((uint64_t)seq << 32) | (hi << 16) | lo;
  if (v.mc) {
    mc_st_u64(ll_small_ptr(v.mc, parity, v.row) + i, word);
  } else {
    for (int k = 0; k < count; k++) st_u64_relaxed(ll_small_ptr(v.peers[s_order[k]], parity, v.row) + i, word);
  }
  const uint64_t my_base = v.peers[v.row];
  float a0 = 0.f, a1 = 0.f;
  uint64_t t0 = 0;
  bool named = false;
  uint32_t spins = 0;
  int fail = kOk;
  for (int k = 0; k < count && fail == kOk; k++) {
    const uint32_t bits = ll_wait(v, ll_small_ptr(my_base, parity, s_order[k]) + i, seq, s_order[k], t0, named, spins, fail);
    a0 += __bfloat162float(__ushort_as_bfloat16((unsigned short)(bits & 0xFFFFu)));
    a1 += __bfloat162float(__ushort_as_bfloat16((unsigned short)(bits >> 16)));
  }
  if (fail != kOk) {
    volatile Ctrl* c = v.ctrl;
    c->status = (uint32_t)fail;
    return;
  }
  out[2 * i] = f2bf(a0);
  if (pair) out[2 * i + 1] = f2bf(a1);
}

}  // namespace
}  // namespace comm

int64_t comm_ll_max_elems() { return (int64_t)(comm::kLLSmallBytes / 8 * 2); }

int64_t comm_buffer_bytes() { return (int64_t)comm::kBufferBytes; }
int64_t comm_max_elems() { return (int64_t)(comm::kDataBytes / 2); }

cudaError_t launch_fdar(const void* inp, void* out, int64_t n, const CommArgs& c, cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  if (n > comm_max_elems() || reinterpret_cast<uintptr_t>(inp) % 16 != 0 || reinterpret_cast<uintptr_t>(out) % 16 != 0 ||
      c.seqs == nullptr)
    return cudaErrorInvalidValue;
  comm::View v{};
  v.seqs = c.seqs;
  v.peers = c.peers;
  v.mc = c.mc;
  v.order = c.order;
  v.call = c.call;
  v.ctrl = reinterpret_cast<comm::Ctrl*>(c.ctrl);
  v.row = c.row;
  if (n <= comm_ll_max_elems()) {
    const int words = (int)((n + 1) / 2);
    const int grid = (words + comm::kLLThreads - 1) / comm::kLLThreads;
    return launch_ex(comm::fdar_ll_kernel, dim3(grid), dim3(comm::kLLThreads), 0, stream, 0,
                     static_cast<const __nv_bfloat16*>(inp), static_cast<__nv_bfloat16*>(out), (int)n, v);
  }
  const int grid = (int)((n + comm::kChunk - 1) / comm::kChunk);
  return launch_ex(comm::fdar_kernel, dim3(grid), dim3(comm::kThreads), 0, stream, 0,
                   static_cast<const __nv_bfloat16*>(inp), static_cast<__nv_bfloat16*>(out), (int)n, v);
}

}  // namespace es
