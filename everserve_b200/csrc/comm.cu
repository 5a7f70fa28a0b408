// Failure-detecting all-reduce ("fdar"): sum a bf16 vector over the members of a tensor-parallel
// group through peer memory, in member order, with bounded waits (see comm.cuh for the protocol).
//
// Decode-size tensors (up to 512 Ki elements) take the one-shot LL kernel: every 8-byte word
// carries two bf16 and the call number, pushed to every member, so one round trip and no flags.
// Larger ones take the two-shot kernel on the same LL words (a reduce-scatter to chunk owners,
// then the owners' sums to every member), up to 512 Ki elements per member per call; the host
// splits bigger tensors into calls.
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

// Two-shot all-reduce (tensors above the one-shot LL path), on LL words: every 8-byte word
// carries two bf16 and the call number, so a word is its own arrival flag and the kernel needs no
// fence and no flag round trip (system-scope fences measured several microseconds each here,
// which made a fenced two-shot latency-bound). A persistent grid, CTA b taking chunks b,
// b + grid, ... in the same order on every member; chunk c's owner is member c % count:
//   1. the CTA writes this member's part of each of its chunks, as LL words, into the owner's
//      data row for this member (at the owner's local index c / count);
//   2. for the chunks this member owns: each thread polls its words from every member in member
//      order, sums them in fp32 (one rounding), writes the sum to `out` and, as LL words, into
//      every other member's gather area;
//   3. for the chunks others own: each thread polls its words in this member's gather area.
// Each member sends about twice (count - 1) / count of the vector (in words of twice its bytes)
// and receives as much. Every wait is bounded (abort word, the sender's heartbeat, hard limit).
constexpr int kWordsPerChunk = kChunk / 2;

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
  const int nw = (n + 1) / 2;  // words of the whole vector
  // an owner's chunks must fit one data row of each sender (in words)
  if (nchunks > (int)(kDataBytes / 8 / kWordsPerChunk) * count) {
    if (threadIdx.x == 0) finish_call(v, seq, kBadShape);
    return;
  }
  auto word_of = [&](const __nv_bfloat16* src, int w) -> uint64_t {
    const uint32_t lo = __bfloat16_as_ushort(src[2 * w]);
    const uint32_t hi = 2 * w + 1 < n ? __bfloat16_as_ushort(src[2 * w + 1]) : 0u;
    return ((uint64_t)seq << 32) | (hi << 16) | lo;
  };
  int fail = kOk;
  if (count > 0) {
    // 1. this member's parts, to their owners
    for (int c = blockIdx.x; c < nchunks; c += gridDim.x) {
      const int owner = s_order[c % count];
      uint64_t* dst = reinterpret_cast<uint64_t*>(data_ptr(v.peers[owner], parity, v.row)) +
                      (size_t)(c / count) * kWordsPerChunk;
      const int w0 = c * kWordsPerChunk, w1 = min(nw, w0 + kWordsPerChunk);
      for (int w = w0 + threadIdx.x; w < w1; w += kThreads) st_u64_relaxed(dst + (w - w0), word_of(inp, w));
    }
    uint64_t t0 = 0;
    bool named = false;
    uint32_t spins = 0;
    // 2. the chunks this member owns: every member's words, summed in member order
    for (int c = blockIdx.x; fail == kOk && c < nchunks; c += gridDim.x) {
      if (s_order[c % count] != v.row) continue;
      const size_t local = (size_t)(c / count) * kWordsPerChunk;
      const int w0 = c * kWordsPerChunk, w1 = min(nw, w0 + kWordsPerChunk);
      for (int w = w0 + threadIdx.x; fail == kOk && w < w1; w += kThreads) {
        float a0 = 0.f, a1 = 0.f;
        for (int k = 0; k < count && fail == kOk; k++) {
          const uint64_t* src = reinterpret_cast<const uint64_t*>(data_ptr(my_base, parity, s_order[k])) + local;
          const uint32_t bits = ll_wait(v, src + (w - w0), seq, s_order[k], t0, named, spins, fail);
          a0 += __bfloat162float(__ushort_as_bfloat16((unsigned short)(bits & 0xFFFFu)));
          a1 += __bfloat162float(__ushort_as_bfloat16((unsigned short)(bits >> 16)));
        }
        if (fail != kOk) break;
        const __nv_bfloat16 r0 = f2bf(a0), r1 = f2bf(a1);
        out[2 * w] = r0;
        if (2 * w + 1 < n) out[2 * w + 1] = r1;
        const uint64_t word = ((uint64_t)seq << 32) | ((uint32_t)__bfloat16_as_ushort(r1) << 16) |
                              (uint32_t)__bfloat16_as_ushort(r0);
        for (int k = 0; k < count; k++)
          if (s_order[k] != v.row) st_u64_relaxed(reinterpret_cast<uint64_t*>(ag_ptr(v.peers[s_order[k]], parity)) + w, word);
      }
    }
    // 3. the chunks others own: the owner's sums, from this member's gather area
    const uint64_t* gather = reinterpret_cast<const uint64_t*>(ag_ptr(my_base, parity));
    for (int c = blockIdx.x; fail == kOk && c < nchunks; c += gridDim.x) {
      const int owner = s_order[c % count];
      if (owner == v.row) continue;
      const int w0 = c * kWordsPerChunk, w1 = min(nw, w0 + kWordsPerChunk);
      for (int w = w0 + threadIdx.x; fail == kOk && w < w1; w += kThreads) {
        const uint32_t bits = ll_wait(v, gather + w, seq, owner, t0, named, spins, fail);
        if (fail != kOk) break;
        out[2 * w] = __ushort_as_bfloat16((unsigned short)(bits & 0xFFFFu));
        if (2 * w + 1 < n) out[2 * w + 1] = __ushort_as_bfloat16((unsigned short)(bits >> 16));
      }
    }
  }
  if (fail != kOk) atomicCAS(&s_fail, kOk, fail);
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
  // an owner's chunks fill at most one data row of LL words (two elements per 8-byte word) per sender
  return std::max<int64_t>(1, std::min<int64_t>(members, comm::kMaxRows)) * (int64_t)(comm::kDataBytes / 8 * 2);
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
  if (n > comm_max_elems(comm::kMaxRows)) return cudaErrorInvalidValue;
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
