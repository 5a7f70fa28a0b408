// Peer-memory collectives of a tensor-parallel group over NVLink (one process per GPU).
//
// Every member owns one symmetric buffer in its device memory: a driver VMM allocation whose
// descriptor is passed to the other members over a Unix socket, each of which maps it for its own
// device (vmm.cpp). Its memory lives until every mapping is released, so a member that dies leaves
// it valid under the survivors' bounded waits. Layout:
//   flags: uint32 [2 parity][kMaxRows sender][kFlagSlots]
//   data : bytes  [2 parity][kMaxRows sender][kDataBytes]
// A call pushes this member's contribution into every member's buffer at its own sender row
// (remote stores over NVLink), raises one flag per slot on every member, then waits only on its own
// buffer (local polls) for every member's flag and sums the members' rows in member order in fp32.
// The member order is a device table, so a captured CUDA graph follows a membership change
// without recapture; a spare in the position of a lost rank sums in that rank's place, which keeps
// the result bit-identical across the change.
//
// Calls are numbered by a per-buffer call counter in device memory (the last CTA of a call
// advances it); the number is the flag value and its low bit the parity, so a member one call
// ahead writes the other half of the buffer.
//
// Failure detection: every wait is bounded. After `bound_ns` (host-written, 0 = off) a waiting CTA
// ORs the rows it still waits for into the host-visible late mask and keeps waiting; the host's
// abort word (polled every 1024 spins) or a hard limit ends the wait, the call returns garbage and
// the status word says why. Nothing here traps or spins without a bound.
//
// Heartbeats: every member's process advances a beat word in its row of the slot region from a
// native thread (about every 0.5 ms, whatever its Python thread is doing). A wait that sees the
// beat of the member it waits for stand still for `beat_limit_us` (host-written, 0 = off) names
// that member late and leaves with kDead: a member whose process died is named in milliseconds,
// by the kernel itself, instead of after the bound and the host's checks.
#pragma once

#include <stdint.h>

#include "common.cuh"

namespace es {
namespace comm {

constexpr int kMaxRows = 8;            // members: up to seven ranks and a spare
constexpr int kFlagSlots = 4096;
constexpr size_t kDataBytes = 1 << 21;  // 2 MiB per sender per parity
constexpr size_t kFlagBytes = (size_t)2 * kMaxRows * kFlagSlots * 4;
// LL regions: 8-byte words (seq << 32 | two bf16). The GEMM epilogue's words, then small fdar's.
constexpr size_t kLLGemmBytes = 1 << 21;  // per sender per parity: tiles * 64 * 128 / 2 words
constexpr size_t kLLSmallBytes = 1 << 21; // per sender per parity: 256 Ki words = 512 Ki elements
constexpr size_t kLLGemmOff = kFlagBytes + (size_t)2 * kMaxRows * kDataBytes;
constexpr size_t kLLSmallOff = kLLGemmOff + (size_t)2 * kMaxRows * kLLGemmBytes;
constexpr size_t kLLResOff = kLLSmallOff + (size_t)2 * kMaxRows * kLLSmallBytes;
// the two-shot fused GEMM's results: [2 parity][kLLGemmBytes], each word written by its tile's owner
// Two-shot all-reduce of large tensors (comm.cu): chunks of kChunkElems, chunk c owned by member
// c % count; senders write their part of an owned chunk into the owner's data rows (at the owner's
// local chunk index), the owner sums and writes the result into every member's gather area, then
// raises the chunk's gather flag there.
constexpr int kChunkElems = 4096;
constexpr int kMaxChunks = kMaxRows * (int)(kDataBytes / (kChunkElems * 2));  // 2048: 8 Mi elements
constexpr size_t kAGFlagOff = kLLResOff + (size_t)2 * kLLGemmBytes;
constexpr size_t kAGFlagBytes = (size_t)2 * kMaxChunks * 4;                     // [2 parity][chunk] u32
constexpr size_t kAGOff = kAGFlagOff + ((kAGFlagBytes + 4095) & ~(size_t)4095);
constexpr size_t kAGBytes = (size_t)kMaxRows * kDataBytes;                      // per parity: a whole call
// All-gather into a GEMM (gemm.cu, kAG): every member's token slice lands, by peer stores of a few
// pusher CTAs, in every member's gather rows [2 parity][kAGGemmBytes] (rows in member order), and
// each pusher raises a flag per (parity, sender, pusher) there; the GEMM reads the rows with TMA.
constexpr int kAGPushers = 16;
constexpr size_t kAGGemmFlagOff = kAGOff + (size_t)2 * kAGBytes;
constexpr size_t kAGGemmFlagBytes = 4096;  // [2][kMaxRows][kAGPushers] u32
constexpr size_t kAGGemmOff = kAGGemmFlagOff + kAGGemmFlagBytes;
constexpr size_t kAGGemmBytes = (size_t)4 << 20;  // per parity: e.g. 64 rows of K = 16384 bf16 x 2
constexpr int kAGSeqSlot = 4095;                  // the gathering GEMM's call counter in `seqs` ...
constexpr int kAGDoneSlot = 4094;                 // ... and its CTAs-done counter
constexpr size_t kBufferBytes = kAGGemmOff + (size_t)2 * kAGGemmBytes;
constexpr int kSeqSlots = 4096;  // per-slot LL call counters (this member's device memory)
constexpr uint64_t kHardLimitNs = 5000000000ull;  // a wait never outlives 5 s

// Host-mapped control words of one member (pinned host memory the device reads and writes); the
// members' rows lie kRowBytes apart in the slot region, so a kernel finds a peer's row from its own.
struct Ctrl {
  uint32_t abort;          // host: non-zero makes waiting kernels leave
  uint32_t late;           // device: mask of rows a wait has been waiting for past bound_ns
  uint64_t bound_ns;       // host: 0 = never name late members
  uint32_t status;         // device: last failure (kTimeout / kAborted / kDead)
  uint32_t beat;           // the member's process: its heartbeat counter
  uint32_t beat_limit_us;  // host: a beat standing still this long means the member is dead (0 = off)
  uint32_t pad;
};
constexpr int kRowBytes = 256;  // slot region row stride (parallel/slot.py ROW_BYTES)

// Device view of a member's place in the group (kernel parameter, by value).
struct View {
  uint32_t* seqs;         // [2 * kSeqSlots] LL call counters: GEMM slots, then small-fdar blocks
  const uint64_t* peers;  // [kMaxRows] base address of each row's buffer (0 = not mapped)
  uint64_t mc;            // multicast (NVLS) address of the group's buffers; 0: push with P2P stores
  const int32_t* order;   // [1 + kMaxRows]: count, rows in member order
  uint32_t* call;         // [2]: call counter, CTAs done in the current call
  Ctrl* ctrl;             // host-mapped control words of this member (device address)
  int row;                // this member's row
};

// ---- NVLS multicast stores: one store reaches the same offset of every member's buffer ------------
ES_DEVICE void mc_st_v4(void* mc_addr, uint4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc_addr), "f"(__uint_as_float(v.x)),
               "f"(__uint_as_float(v.y)), "f"(__uint_as_float(v.z)), "f"(__uint_as_float(v.w))
               : "memory");
}
ES_DEVICE void mc_st_v2(void* mc_addr, uint2 v) {
  asm volatile("multimem.st.relaxed.sys.global.v2.f32 [%0], {%1, %2};" ::"l"(mc_addr), "f"(__uint_as_float(v.x)),
               "f"(__uint_as_float(v.y))
               : "memory");
}
ES_DEVICE void mc_st_release_u32(void* mc_addr, uint32_t v) {
  asm volatile("multimem.st.release.sys.global.u32 [%0], %1;" ::"l"(mc_addr), "r"(v) : "memory");
}
// Order this thread's accesses through the multicast alias against unicast accesses to the buffer.
ES_DEVICE void fence_alias() { asm volatile("fence.proxy.alias;" ::: "memory"); }

ES_DEVICE uint64_t* ll_res_ptr(uint64_t base, uint32_t parity) {
  return reinterpret_cast<uint64_t*>(reinterpret_cast<char*>(base) + kLLResOff + (size_t)parity * kLLGemmBytes);
}
ES_DEVICE uint64_t* ll_gemm_ptr(uint64_t base, uint32_t parity, int sender) {
  return reinterpret_cast<uint64_t*>(reinterpret_cast<char*>(base) + kLLGemmOff +
                                     ((size_t)parity * kMaxRows + sender) * kLLGemmBytes);
}
ES_DEVICE uint64_t* ll_small_ptr(uint64_t base, uint32_t parity, int sender) {
  return reinterpret_cast<uint64_t*>(reinterpret_cast<char*>(base) + kLLSmallOff +
                                     ((size_t)parity * kMaxRows + sender) * kLLSmallBytes);
}
ES_DEVICE void st_u64_relaxed(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
ES_DEVICE uint64_t ld_u64_relaxed(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
ES_DEVICE void mc_st_u64(void* mc_addr, uint64_t v) {
  asm volatile("multimem.st.relaxed.sys.global.v2.f32 [%0], {%1, %2};" ::"l"(mc_addr),
               "f"(__uint_as_float((uint32_t)v)), "f"(__uint_as_float((uint32_t)(v >> 32)))
               : "memory");
}

// The control words of row `row` (a member's row of the slot region, found from this member's).
ES_DEVICE volatile Ctrl* ctrl_of(const View& v, int row) {
  return reinterpret_cast<volatile Ctrl*>(reinterpret_cast<char*>(v.ctrl) + (ptrdiff_t)(row - v.row) * kRowBytes);
}

// Heartbeat watch of one awaited member: true once its beat has stood still past the limit.
struct BeatWatch {
  uint32_t last = 0;
  uint64_t since = 0;
  ES_DEVICE bool stopped(const View& v, int sender, uint64_t now) {
    const uint32_t lim = v.ctrl->beat_limit_us;
    if (lim == 0) return false;
    const uint32_t b = ctrl_of(v, sender)->beat;
    if (since == 0 || b != last) {
      last = b;
      since = now;
      return false;
    }
    return now - since > (uint64_t)lim * 1000ull;
  }
};

// Poll one LL word of `sender` until it carries `seq`; returns its two bf16 (as bits) or reports
// a failure through `fail` (aborted / dead / hard limit). `t0`, `named` and `spins` persist per
// thread.
ES_DEVICE uint32_t ll_wait(const View& v, const uint64_t* w, uint32_t seq, int sender, uint64_t& t0, bool& named,
                           uint32_t& spins, int& fail) {
  uint64_t x = ld_u64_relaxed(w);
  BeatWatch beat;
  while ((uint32_t)(x >> 32) != seq) {
    if ((++spins & 1023u) == 0) {
      volatile Ctrl* c = v.ctrl;
      if (t0 == 0) t0 = global_ns();
      if (c->abort) {
        fail = kAborted;
        return 0;
      }
      if (beat.stopped(v, sender, global_ns())) {
        c->late = c->late | (1u << sender);
        fail = kDead;
        return 0;
      }
      const uint64_t now = global_ns() - t0;
      const uint64_t bound = c->bound_ns;
      if (!named && bound != 0 && now > bound) {
        c->late = c->late | (1u << sender);
        named = true;
      }
      if (now > kHardLimitNs) {
        fail = kTimeout;
        return 0;
      }
    }
    x = ld_u64_relaxed(w);
  }
  return (uint32_t)x;
}

ES_DEVICE uint32_t* ag_flag_ptr(uint64_t base, uint32_t parity, int chunk) {
  return reinterpret_cast<uint32_t*>(reinterpret_cast<char*>(base) + kAGFlagOff) + (size_t)parity * kMaxChunks + chunk;
}
ES_DEVICE char* ag_ptr(uint64_t base, uint32_t parity) {
  return reinterpret_cast<char*>(base) + kAGOff + (size_t)parity * kAGBytes;
}

// Wait until the flag at `f` (in this member's own buffer) equals `seq`, raised by member `sender`:
// bounded like every wait (abort word, the sender's heartbeat, the bound naming it late, the hard
// limit). Called by one thread; returns kOk or the failure.
ES_DEVICE int wait_flag(const View& v, const uint32_t* f, uint32_t seq, int sender) {
  const uint64_t t0 = global_ns();
  uint64_t bound = 0;
  bool named = false;
  uint32_t spins = 0;
  BeatWatch beat;
  while (ld_relaxed_sys(f) != seq) {
    if ((++spins & 1023u) == 0) {
      volatile Ctrl* c = v.ctrl;
      if (c->abort) return kAborted;
      const uint64_t t = global_ns();
      if (beat.stopped(v, sender, t)) {
        c->late = c->late | (1u << sender);
        return kDead;
      }
      if (bound == 0) bound = c->bound_ns;
      if (!named && bound != 0 && t - t0 > bound) {
        c->late = c->late | (1u << sender);
        named = true;
      }
      if (t - t0 > kHardLimitNs) return kTimeout;
    }
  }
  fence_acquire_sys();
  return kOk;
}

ES_DEVICE uint32_t* ag_gemm_flag_ptr(uint64_t base, uint32_t parity, int sender, int pusher) {
  return reinterpret_cast<uint32_t*>(reinterpret_cast<char*>(base) + kAGGemmFlagOff) +
         ((size_t)parity * kMaxRows + sender) * kAGPushers + pusher;
}
ES_DEVICE char* ag_gemm_ptr(uint64_t base, uint32_t parity) {
  return reinterpret_cast<char*>(base) + kAGGemmOff + (size_t)parity * kAGGemmBytes;
}

ES_DEVICE uint32_t* flag_ptr(uint64_t base, uint32_t parity, int sender, int slot) {
  return reinterpret_cast<uint32_t*>(base) + ((size_t)parity * kMaxRows + sender) * kFlagSlots + slot;
}
ES_DEVICE char* data_ptr(uint64_t base, uint32_t parity, int sender) {
  return reinterpret_cast<char*>(base) + kFlagBytes + ((size_t)parity * kMaxRows + sender) * kDataBytes;
}

// Wait until every member's flag for `slot` in this member's buffer equals `seq`. Called by one
// thread; returns kOk, kAborted or kTimeout.
ES_DEVICE int wait_members(const View& v, uint64_t my_base, uint32_t parity, int slot, uint32_t seq,
                           const int* order, int count) {
  const uint64_t t0 = global_ns();
  uint64_t bound = 0;
  bool named = false;
  uint32_t spins = 0;
  for (int i = 0; i < count; i++) {
    const int sender = order[i];
    const uint32_t* f = flag_ptr(my_base, parity, sender, slot);
    BeatWatch beat;
    while (ld_relaxed_sys(f) != seq) {
      if ((++spins & 1023u) == 0) {
        volatile Ctrl* c = v.ctrl;
        if (c->abort) return kAborted;
        if (beat.stopped(v, sender, global_ns())) {
          c->late = c->late | (1u << sender);
          return kDead;
        }
        const uint64_t now = global_ns() - t0;
        if (bound == 0) bound = c->bound_ns;
        if (!named && bound != 0 && now > bound) {
          uint32_t mask = 0;
          for (int k = i; k < count; k++)
            if (ld_acquire_sys(flag_ptr(my_base, parity, order[k], slot)) != seq) mask |= 1u << order[k];
          // host-mapped memory: a plain read-modify-write (device atomics on mapped host memory are
          // not guaranteed); a bit a concurrent CTA drops is named again by that CTA's own wait
          volatile Ctrl* cw = v.ctrl;
          cw->late = cw->late | mask;
          named = true;
        }
        if (now > kHardLimitNs) return kTimeout;
      }
    }
  }
  fence_acquire_sys();
  if (v.mc) fence_alias();
  return kOk;
}

// Called by thread 0 of every CTA at the end of a call: the last CTA advances the call counter.
ES_DEVICE void finish_call(const View& v, uint32_t seq, int failure) {
  if (failure != kOk) {
    volatile Ctrl* cw = v.ctrl;
    cw->status = (uint32_t)failure;
  }
  __threadfence();
  if (atomicAdd(v.call + 1, 1u) == gridDim.x * gridDim.y * gridDim.z - 1) {
    v.call[1] = 0;
    __threadfence();
    atomicExch(v.call, seq);
  }
}

}  // namespace comm
}  // namespace es
