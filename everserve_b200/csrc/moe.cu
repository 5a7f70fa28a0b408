// Expert-parallel all-to-all over NVLink peer memory: each member's tokens go to the members that
// own their experts (dispatch), the experts run as GEMMs over what they received, and each
// token's expert outputs come back, weighted, to the member that holds the token (combine).
//
// Every member owns one symmetric buffer (a driver VMM allocation the others map), laid out as
//   flags  uint32 [kMaxRows sender position][kMaxLocal expert][kMaxSplits]  dispatch flags
//   ready  uint32 [kMaxRows owner position]                                outputs-ready flags
//   counts uint32 [kMaxLocal expert][kMaxRows sender position]            rows each sender sent
//   recv   bf16   [el][W * cap][H]   local expert el's input: sender p's rows at [p*cap, p*cap + n)
//   y      bf16   [el][W * cap][H]   the expert's output rows, at the same places
// Each sender writes its rows for an expert in (token, slot) order, so a row's place depends only
// on the sender's own routing: no count exchange precedes the data, and every member can compute
// where each of its tokens' rows went. Padded rows past a segment's count are never read: the
// expert GEMMs skip token tiles that hold none of them (the `valid` input of the GEMM), and the
// combine reads only the rows its tokens were given.
//
// One call = dispatch (pushes, then waits for every sender's flags), the expert GEMMs on each
// member, `ready` (raises this member's flag in every member's buffer once its outputs are
// written), combine (waits for every owner's flag, then reads each token's k rows from the owners'
// buffers and sums them in slot order in fp32). Calls are numbered by a per-member counter in
// device memory that the combine's last CTA advances; the number is the flag value. A member can
// be at most one call ahead of another (its next dispatch waits for everyone's), and by then every
// reader of the buffers it writes has finished the previous call, so no half of a buffer is
// double-booked.
//
// Positions, not rows: expert ownership and buffer places follow a member's position in the
// expert-parallel group; the device member table maps a position to the row (buffer) that holds
// it, so a spare that takes a lost member's position inherits its experts without re-laying out.
//
// Emulation: a launch can play `nz` consecutive positions (blockIdx.z), each with its own call
// counter and control words, with every buffer local; one kernel then carries the whole group's
// traffic on one GPU. Waiting CTAs wait only for CTAs that never wait, so the launch finishes
// however the CTAs are scheduled.
//
// Failure detection as in the tensor-parallel collectives: every wait is bounded; past `bound_ns`
// it names the late member's row in the late mask; the abort word or the hard limit ends it, and
// the status word says why. Nothing traps.
#include <algorithm>

#include "api.h"
#include "comm.cuh"
#include "common.cuh"
#include "launch.h"

namespace es {
namespace moe {

constexpr int kMaxLocal = 32;
constexpr int kMaxSplits = 32;
constexpr int kThreads = 256;
constexpr size_t kFlagsOff = 0;
constexpr size_t kReadyOff = kFlagsOff + (size_t)comm::kMaxRows * kMaxLocal * kMaxSplits * 4;
constexpr size_t kCountsOff = kReadyOff + (size_t)comm::kMaxRows * 4;
constexpr size_t kHeaderBytes = 64 * 1024;
static_assert(kCountsOff + (size_t)kMaxLocal * comm::kMaxRows * 4 <= kHeaderBytes, "header fits");
constexpr int kOverflow = 4;  // a sender had more rows for an expert than a segment holds

ES_DEVICE uint32_t* flag_at(uint64_t base, int sender, int el, int split) {
  return reinterpret_cast<uint32_t*>(base + kFlagsOff) + ((size_t)sender * kMaxLocal + el) * kMaxSplits + split;
}
ES_DEVICE uint32_t* ready_at(uint64_t base, int owner) {
  return reinterpret_cast<uint32_t*>(base + kReadyOff) + owner;
}
ES_DEVICE uint32_t* count_at(uint64_t base, int el, int sender) {
  return reinterpret_cast<uint32_t*>(base + kCountsOff) + (size_t)el * comm::kMaxRows + sender;
}

struct Member {
  int pos, row, W;
  uint32_t* call;
  comm::Ctrl* ctrl;
};

// The position comes from the device table (entry 1 + kMaxRows), so captured graphs follow a
// spare's takeover; a process holding no position (a spare before its take) has row -1.
ES_DEVICE Member member_of(const MoeArgs& a) {
  Member m;
  m.pos = a.members[1 + comm::kMaxRows] + (int)blockIdx.z;
  m.W = a.members[0];
  m.row = (m.pos >= 0 && m.pos < m.W && m.W <= comm::kMaxRows) ? a.members[1 + m.pos] : -1;
  m.call = a.call + 2 * blockIdx.z;
  m.ctrl = reinterpret_cast<comm::Ctrl*>(a.ctrl) + blockIdx.z;
  return m;
}

ES_DEVICE void set_status(comm::Ctrl* ctrl, int failure) {
  volatile comm::Ctrl* c = ctrl;
  c->status = (uint32_t)failure;
}

// Wait until *f == seq; past the bound name `late_row`; kOk, kAborted or kTimeout.
ES_DEVICE int wait_flag(const uint32_t* f, uint32_t seq, comm::Ctrl* ctrl, int late_row, uint64_t t0, bool& named) {
  uint32_t spins = 0;
  while (ld_relaxed_sys(f) != seq) {
    if ((++spins & 1023u) == 0) {
      volatile comm::Ctrl* c = ctrl;
      if (c->abort) return kAborted;
      const uint64_t now = global_ns() - t0;
      const uint64_t bound = c->bound_ns;
      if (!named && bound != 0 && now > bound) {
        c->late = c->late | (1u << late_row);
        named = true;
      }
      if (now > comm::kHardLimitNs) return kTimeout;
    }
  }
  fence_acquire_sys();
  return kOk;
}

// grid (E + 1, splits, nz): CTA (e, split) sends its share of expert e's rows; CTA (E, 0) waits for
// every sender's flags in this member's own buffer.
__global__ void __launch_bounds__(kThreads) dispatch_kernel(const __nv_bfloat16* __restrict__ x, int64_t x_member,
                                                            const int32_t* __restrict__ ids,
                                                            int32_t* __restrict__ pos, int T, MoeArgs a) {
  __shared__ int s_warp[kThreads / 32];
  __shared__ int s_n;
  __shared__ int s_t[kThreads], s_i[kThreads];
  __shared__ int s_fail;
  pdl_wait();  // the tokens and their routing come from the kernels before
  pdl_launch();
  const Member m = member_of(a);
  if (m.row < 0) return;  // no position: nothing to send or receive
  const uint32_t seq = *reinterpret_cast<volatile uint32_t*>(m.call) + 1;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t H = a.H;
  const uint64_t own = a.peers[m.row];

  if ((int)blockIdx.x == a.E) {  // the waiter
    if (blockIdx.y != 0) return;
    if (tid == 0) s_fail = kOk;
    __syncthreads();
    const int n = m.W * a.el * a.splits;
    const uint64_t t0 = global_ns();
    for (int i = tid; i < n && own != 0; i += kThreads) {
      const int p = i / (a.el * a.splits), el = (i / a.splits) % a.el, s = i % a.splits;
      bool named = false;
      const int r = wait_flag(flag_at(own, p, el, s), seq, m.ctrl, a.members[1 + p], t0, named);
      if (r != kOk) atomicCAS(&s_fail, kOk, r);
    }
    __syncthreads();
    if (tid == 0) {
      if (own == 0) s_fail = kBadShape;
      if (s_fail != kOk) set_status(m.ctrl, s_fail);
      __threadfence();
    }
    return;
  }

  const int e = blockIdx.x, split = blockIdx.y, S = a.splits;
  const int dpos = e / a.el, el = e % a.el;
  const uint64_t dst = dpos < m.W ? a.peers[a.members[1 + dpos]] : 0;
  if (dst == 0) {  // an owner without a mapped buffer: nothing can be sent (the waiter times out)
    if (tid == 0) set_status(m.ctrl, kBadShape);
    return;
  }
  const int32_t* my_ids = ids + (size_t)blockIdx.z * T * a.k;
  int32_t* my_pos = pos + (size_t)blockIdx.z * T * a.k;
  const __nv_bfloat16* my_x = x + (size_t)blockIdx.z * x_member;
  const int n = T * a.k;
  const int64_t vecs = H / 8;  // 16-byte vectors per row
  __nv_bfloat16* recv = reinterpret_cast<__nv_bfloat16*>(dst + kHeaderBytes) +
                        ((size_t)el * m.W * a.cap + (size_t)m.pos * a.cap) * H;
  int base = 0, overflow = 0;
  for (int c = 0; c < n; c += kThreads) {
    const int idx = c + tid;
    const bool match = idx < n && my_ids[idx] == e;
    const unsigned mask = __ballot_sync(0xffffffffu, match);
    if (lane == 0) s_warp[warp] = __popc(mask);
    if (tid == 0) s_n = 0;
    __syncthreads();
    int before = 0, total = 0;
#pragma unroll
    for (int w = 0; w < kThreads / 32; w++) {
      before += w < warp ? s_warp[w] : 0;
      total += s_warp[w];
    }
    if (match) {
      const int i = base + before + __popc(mask & ((1u << lane) - 1u));
      if (split == 0) my_pos[idx] = i;
      if (i >= a.cap) {
        overflow = 1;
      } else if (i % S == split) {
        const int slot = atomicAdd(&s_n, 1);
        s_t[slot] = idx / a.k;
        s_i[slot] = i;
      }
    }
    __syncthreads();
    // one warp per row: 16-byte loads from this member's tokens, 16-byte stores into the owner's
    for (int r = warp; r < s_n; r += kThreads / 32) {
      const uint4* src = reinterpret_cast<const uint4*>(my_x + (size_t)s_t[r] * H);
      uint4* out = reinterpret_cast<uint4*>(recv + (size_t)s_i[r] * H);
      for (int64_t v = lane; v < vecs; v += 32) out[v] = src[v];
    }
    base += total;
    __syncthreads();  // the shared list is rebuilt by the next chunk
  }
  if (overflow) set_status(m.ctrl, kOverflow);
  if (split == 0 && tid == 0) *count_at(dst, el, m.pos) = (uint32_t)(base < a.cap ? base : a.cap);
  __threadfence_system();  // each thread's peer stores, before the barrier the flag follows
  __syncthreads();
  if (tid == 0) {
    __threadfence_system();  // every thread's stores above, then the flag
    st_release_sys(flag_at(dst, m.pos, el, split), seq);
  }
}

// grid (1, 1, nz), W threads: this member's outputs are written; tell every member.
__global__ void ready_kernel(MoeArgs a) {
  pdl_wait();  // the expert GEMMs that wrote y
  pdl_launch();
  const Member m = member_of(a);
  if (m.row < 0) return;
  const uint32_t seq = *reinterpret_cast<volatile uint32_t*>(m.call) + 1;
  const int p = threadIdx.x;
  if (p >= m.W) return;
  const uint64_t base = a.peers[a.members[1 + p]];
  if (base == 0) return;  // that member's combine times out and names this one's row's absence
  __threadfence_system();
  st_release_sys(ready_at(base, m.pos), seq);
}

// grid (blocks, 1, nz): waits for every owner's ready flag, then for each of this member's tokens
// out[t] = sum over slots j (in order) of w[t, j] * y_owner(e)[e % el][pos * cap + place[t, j]].
__global__ void __launch_bounds__(kThreads) combine_kernel(const int32_t* __restrict__ ids,
                                                           const float* __restrict__ weights,
                                                           const int32_t* __restrict__ place,
                                                           __nv_bfloat16* __restrict__ out, int64_t out_member,
                                                           int T, MoeArgs a) {
  __shared__ int s_fail;
  pdl_wait();
  pdl_launch();
  const Member m = member_of(a);
  if (m.row < 0) return;  // uniform over the CTA: no barrier below is reached by only some threads
  const uint32_t seq = *reinterpret_cast<volatile uint32_t*>(m.call) + 1;
  const uint64_t own = a.peers[m.row];
  const int tid = threadIdx.x;
  if (tid == 0) s_fail = own == 0 ? kBadShape : kOk;
  __syncthreads();
  if (tid < m.W && own != 0) {
    bool named = false;
    const int r = wait_flag(ready_at(own, tid), seq, m.ctrl, a.members[1 + tid], global_ns(), named);
    if (r != kOk) atomicCAS(&s_fail, kOk, r);
  }
  __syncthreads();
  const int fail = s_fail;
  if (fail == kOk) {
    const int64_t H = a.H, vecs = H / 8;
    const size_t seg = (size_t)m.W * a.cap;
    const int32_t* my_ids = ids + (size_t)blockIdx.z * T * a.k;
    const float* my_w = weights + (size_t)blockIdx.z * T * a.k;
    const int32_t* my_place = place + (size_t)blockIdx.z * T * a.k;
    __nv_bfloat16* my_out = out + (size_t)blockIdx.z * out_member;
    for (int t = blockIdx.x; t < T; t += gridDim.x) {
      for (int64_t v = tid; v < vecs; v += kThreads) {
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int j = 0; j < a.k; j++) {
          const int e = my_ids[t * a.k + j];
          const int i = my_place[t * a.k + j];
          if (e < 0 || e >= a.E || i < 0 || i >= a.cap) continue;
          const uint64_t src = a.peers[a.members[1 + e / a.el]];
          if (src == 0) continue;
          const __nv_bfloat16* y = reinterpret_cast<const __nv_bfloat16*>(src + kHeaderBytes) +
                                   (size_t)a.el * seg * H + ((size_t)(e % a.el) * seg + (size_t)m.pos * a.cap + i) * H;
          const uint4 raw = __ldcg(reinterpret_cast<const uint4*>(y) + v);
          float f[8];
          unpack8(raw, f);
          const float w = my_w[t * a.k + j];
#pragma unroll
          for (int q = 0; q < 8; q++) acc[q] += w * f[q];
        }
        reinterpret_cast<uint4*>(my_out + (size_t)t * H)[v] = pack8(acc);
      }
    }
  } else if (tid == 0) {
    set_status(m.ctrl, fail);
  }
  // the last CTA of this member advances its call counter
  if (tid == 0) {
    __threadfence();
    const unsigned per_member = gridDim.x;
    if (atomicAdd(m.call + 1, 1u) == per_member - 1) {
      m.call[1] = 0;
      __threadfence();
      atomicExch(m.call, seq);
    }
  }
}

bool valid_args(const MoeArgs& a, int T) {
  return a.E > 0 && a.el > 0 && a.el <= kMaxLocal && a.E % a.el == 0 && a.k > 0 && a.k <= a.E && a.H > 0 &&
         a.H % 8 == 0 && a.splits > 0 && a.splits <= kMaxSplits && a.nz > 0 && a.cap >= T &&
         a.nz <= comm::kMaxRows && a.E / a.el <= comm::kMaxRows && a.peers && a.members && a.call && a.ctrl;
}

}  // namespace moe

int64_t moe_header_bytes() { return (int64_t)moe::kHeaderBytes; }
int64_t moe_counts_offset() { return (int64_t)moe::kCountsOff; }
int64_t moe_counts_stride() { return comm::kMaxRows; }

int64_t moe_buffer_bytes(int64_t el, int64_t W, int64_t cap, int64_t H) {
  return (int64_t)moe::kHeaderBytes + 2 * el * W * cap * H * 2;
}

cudaError_t launch_moe_dispatch(const void* x, int64_t x_member, const int32_t* ids, int32_t* pos, int T,
                                const MoeArgs& a, cudaStream_t stream) {
  if (!moe::valid_args(a, T)) return cudaErrorInvalidValue;
  if (reinterpret_cast<uintptr_t>(x) % 16 != 0 || x_member % 8 != 0) return cudaErrorInvalidValue;
  return launch_ex(moe::dispatch_kernel, dim3((unsigned)a.E + 1, (unsigned)a.splits, (unsigned)a.nz),
                   dim3(moe::kThreads), 0, stream, 0, static_cast<const __nv_bfloat16*>(x), x_member, ids, pos, T, a);
}

cudaError_t launch_moe_ready(const MoeArgs& a, cudaStream_t stream) {
  if (!moe::valid_args(a, 0)) return cudaErrorInvalidValue;
  return launch_ex(moe::ready_kernel, dim3(1, 1, (unsigned)a.nz), dim3(32), 0, stream, 0, a);
}

cudaError_t launch_moe_combine(const int32_t* ids, const float* weights, const int32_t* pos, void* out,
                               int64_t out_member, int T, int num_sms, const MoeArgs& a, cudaStream_t stream) {
  if (!moe::valid_args(a, T)) return cudaErrorInvalidValue;
  if (reinterpret_cast<uintptr_t>(out) % 16 != 0 || out_member % 8 != 0) return cudaErrorInvalidValue;
  // at least one CTA per member even for no tokens: its last CTA advances the call counter
  const int per = std::max(1, std::min(T, std::max(1, 4 * num_sms / a.nz)));
  return launch_ex(moe::combine_kernel, dim3((unsigned)per, 1, (unsigned)a.nz), dim3(moe::kThreads), 0, stream, 0,
                   ids, weights, pos, static_cast<__nv_bfloat16*>(out), out_member, T, a);
}

}  // namespace es
