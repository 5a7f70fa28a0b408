// Failure-detecting all-reduce ("fdar"): sum a bf16 vector over the members of a tensor-parallel
// group through peer memory, in member order, with bounded waits (see comm.cuh for the protocol).
//
// Decode-size tensors (up to 512 Ki elements) take the LL kernel: every 8-byte word carries two
// bf16 and the call number, pushed to every member, so one round trip and no flags. Larger ones take
// the two-shot kernel (a reduce-scatter to chunk owners, then the owners' sums to every member),
// up to 1 Mi elements per member per call; the host splits bigger tensors into calls.
#include <algorithm>
#include <cstdlib>

#include "api.h"
#include "launch.h"
#include "comm.cuh"

namespace es {
namespace comm {
namespace {

constexpr int kThreads = 256;
constexpr int kChunk = kChunkElems;

// Two-shot all-reduce (tensors above the LL path): a persistent grid, CTA b taking chunks b,
// b + grid, ... in the same order on every member (chunk c's owner: member c % count).
//   1. the CTA writes this member's part of every one of its chunks into the owner's data row for
//      this member (at the owner's local index c / count), then one release fence and a flag per
//      chunk at its owner;
//   2. for the chunks this member owns: wait for every member's flag, sum the parts in member
//      order in fp32 (one rounding) into `out` and into every other member's gather area; then one
//      fence and the chunks' gather flags at every other member;
//   3. for the chunks others own: wait for the owner's gather flag, copy the sum out.
// A CTA's chunks travel together and it fences twice per call, not per chunk, so the bytes of all
// of them are on the links at once. Each member sends about twice (count - 1) / count of the
// vector and receives as much. Every wait is bounded.
ES_DEVICE void fence_release_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

ES_DEVICE void copy_part(const __nv_bfloat16* __restrict__ src, char* dst, int len) {
  const int nvec = len / 8;  // whole 16-byte vectors; the tail element by element
  for (int i = threadIdx.x; i < nvec; i += kThreads)
    reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(src)[i];
  for (int i = nvec * 8 + threadIdx.x; i < len; i += kThreads) reinterpret_cast<__nv_bfloat16*>(dst)[i] = src[i];
}

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
  const uint64_t my_base = v.peers[v.row];
  const int nchunks = (n + kChunk - 1) / kChunk;
  // an owner's chunks must fit one data row of each sender: at most kDataBytes / chunk per member
  if (nchunks > (int)(kDataBytes / (kChunk * 2)) * count) {
    if (threadIdx.x == 0) finish_call(v, seq, kBadShape);
    return;
  }
  if (count > 0) {
    // 1. this member's parts, to their owners
    for (int c = blockIdx.x; c < nchunks; c += gridDim.x) {
      const int owner = s_order[c % count];
      const int e0 = c * kChunk, e1 = min(n, e0 + kChunk);
      copy_part(inp + e0, data_ptr(v.peers[owner], parity, v.row) + (size_t)(c / count) * kChunk * 2, e1 - e0);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      fence_release_sys();
      for (int c = blockIdx.x; c < nchunks; c += gridDim.x)
        st_release_sys(flag_ptr(v.peers[s_order[c % count]], parity, v.row, c / count), seq);
    }
    // 2. the chunks this member owns: summed in member order, to `out` and every member
    bool owns = false;
    for (int c = blockIdx.x; c < nchunks; c += gridDim.x) {
      if (s_order[c % count] != v.row) continue;
      owns = true;
      const size_t local = (size_t)(c / count) * kChunk * 2;
      const int e0 = c * kChunk, e1 = min(n, e0 + kChunk);
      const int nvec = (e1 - e0) / 8;
      if (threadIdx.x == 0) s_fail = wait_members(v, my_base, parity, c / count, seq, s_order, count);
      __syncthreads();
      if (s_fail != kOk) break;
      for (int i = threadIdx.x; i < nvec; i += kThreads) {
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int k = 0; k < count; k++) {
          const uint4 w = reinterpret_cast<const uint4*>(data_ptr(my_base, parity, s_order[k]) + local)[i];
          float f[8];
          unpack8(w, f);
#pragma unroll
          for (int j = 0; j < 8; j++) acc[j] += f[j];
        }
        const uint4 r = pack8(acc);
        reinterpret_cast<uint4*>(out + e0)[i] = r;
        for (int k = 0; k < count; k++)
          if (s_order[k] != v.row) reinterpret_cast<uint4*>(ag_ptr(v.peers[s_order[k]], parity) + (size_t)e0 * 2)[i] = r;
      }
      for (int i = e0 + nvec * 8 + threadIdx.x; i < e1; i += kThreads) {
        float acc = 0.f;
        for (int k = 0; k < count; k++)
          acc += bf2f(reinterpret_cast<const __nv_bfloat16*>(data_ptr(my_base, parity, s_order[k]) + local)[i - e0]);
        const __nv_bfloat16 r = f2bf(acc);
        out[i] = r;
        for (int k = 0; k < count; k++)
          if (s_order[k] != v.row) reinterpret_cast<__nv_bfloat16*>(ag_ptr(v.peers[s_order[k]], parity))[i] = r;
      }
      __syncthreads();  // s_fail is rewritten by the next chunk's wait
    }
    __syncthreads();
    if (owns && s_fail == kOk && threadIdx.x == 0) {
      fence_release_sys();
      for (int c = blockIdx.x; c < nchunks; c += gridDim.x) {
        if (s_order[c % count] != v.row) continue;
        for (int k = 0; k < count; k++)
          if (s_order[k] != v.row) st_release_sys(ag_flag_ptr(v.peers[s_order[k]], parity, c), seq);
      }
    }
    // 3. the chunks others own: the owner's sum, from this member's gather area
    for (int c = blockIdx.x; s_fail == kOk && c < nchunks; c += gridDim.x) {
      const int owner = s_order[c % count];
      if (owner == v.row) continue;
      const int e0 = c * kChunk, e1 = min(n, e0 + kChunk);
      if (threadIdx.x == 0) s_fail = wait_flag(v, ag_flag_ptr(my_base, parity, c), seq, owner);
      __syncthreads();
      if (s_fail != kOk) break;
      const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(ag_ptr(my_base, parity) + (size_t)e0 * 2);
      copy_part(src, reinterpret_cast<char*>(out + e0), e1 - e0);
      __syncthreads();
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
// elements one all-reduce call takes: each member owns at most a data row's worth of chunks
int64_t comm_max_elems(int64_t members) {
  return std::max<int64_t>(1, std::min<int64_t>(members, comm::kMaxRows)) * (int64_t)(comm::kDataBytes / 2);
}

cudaError_t launch_fdar(const void* inp, void* out, int64_t n, const CommArgs& c, cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  if (reinterpret_cast<uintptr_t>(inp) % 16 != 0 || reinterpret_cast<uintptr_t>(out) % 16 != 0 || c.seqs == nullptr)
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
  // the two-shot path: the member count is a device table (it changes with membership), so the
  // call's size is checked against the largest group; the caller keeps calls within its own count
  if (n > (int64_t)comm::kMaxChunks * comm::kChunk) return cudaErrorInvalidValue;
  static int sms[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (sms[dev] == 0 && cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return cudaErrorInvalidDevice;
  // persistent: every CTA resident at once (they wait on peers' CTAs of the same index)
  const int chunks = (int)((n + comm::kChunk - 1) / comm::kChunk);
  // ES_FDAR_CTAS_PER_SM (tuning): CTAs per SM of the persistent grid (default 2)
  static const int per_sm = [] {
    const char* e = std::getenv("ES_FDAR_CTAS_PER_SM");
    const int v = e ? std::atoi(e) : 2;
    return v >= 1 && v <= 8 ? v : 2;
  }();
  const int grid = std::min(chunks, per_sm * sms[dev]);
  return launch_ex(comm::fdar_kernel, dim3(grid), dim3(comm::kThreads), 0, stream, 0,
                   static_cast<const __nv_bfloat16*>(inp), static_cast<__nv_bfloat16*>(out), (int)n, v);
}

}  // namespace es
