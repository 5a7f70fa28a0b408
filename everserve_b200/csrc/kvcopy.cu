// Committed-KV copies between the paged cache and a staging buffer.
//
// gather: one launch copies one step's rows of every layer and every held kv head into a staging
//         buffer laid out [layers, heads, capacity, 2, d]. The staging buffer is normally pinned
//         host memory mapped into the device (the per-node store's shared-memory file), so the
//         copy runs on a side stream behind the forward and the step thread never reads device
//         memory.
// scatter: the inverse, used by a spare restoring a lost rank's rows: staging -> cache.
// Each cache is addressed through five element strides (block, offset, head, kv, element), so
// any of the supported cache layouts works. A negative slot is a padding row: gather writes
// zeros for it, scatter skips it.
#include <algorithm>

#include "api.h"
#include "common.cuh"

namespace es {
namespace {

struct KvCopyParams {
  const int64_t* layer_ptrs;  // device addresses of each layer's cache
  const int64_t* slots;       // [n]
  const int64_t* heads;       // [H] kv head indices held by this rank
  char* staging;              // [L, H, cap, 2, d] elements of elem bytes
  int64_t n, cap, d, block_size, H;
  int64_t s_block, s_off, s_head, s_kv;  // element strides
  int elem;                               // bytes per element
};

template <bool kGather>
__device__ __forceinline__ void copy_row(const KvCopyParams& p, int64_t t, int l) {
  const int64_t slot = p.slots[t];
  const int vec_per_row = (int)(p.d * p.elem / 16);
  const int per_head = 2 * vec_per_row;
  const int total = (int)p.H * per_head;
  char* cache = reinterpret_cast<char*>(p.layer_ptrs[l]);
  const int64_t blk = slot >= 0 ? slot / p.block_size : 0;
  const int64_t off = slot >= 0 ? slot % p.block_size : 0;
  for (int i = threadIdx.x; i < total; i += blockDim.x) {
    const int hi = i / per_head;
    const int r = i % per_head;
    const int kv = r / vec_per_row;
    const int v = r % vec_per_row;
    const int64_t h = p.heads[hi];
    const int64_t src_el = blk * p.s_block + off * p.s_off + h * p.s_head + kv * p.s_kv;
    uint4* cptr = reinterpret_cast<uint4*>(cache + src_el * p.elem) + v;
    const int64_t dst_el = (((int64_t)l * p.H + hi) * p.cap + t) * 2 * p.d + kv * p.d;
    uint4* sptr = reinterpret_cast<uint4*>(p.staging + dst_el * p.elem) + v;
    if (kGather) {
      *sptr = slot >= 0 ? *cptr : make_uint4(0, 0, 0, 0);
    } else if (slot >= 0) {
      *cptr = *sptr;
    }
  }
}

// CTAs walk the (row, layer) pairs; threads cover (head, kv, 16-byte vector). d * elem must be a
// multiple of 16.
template <bool kGather>
__global__ void kv_copy_kernel(KvCopyParams p, int64_t L) {
  for (int64_t item = blockIdx.x; item < p.n * L; item += gridDim.x) {
    const int64_t t = item % p.n;
    const int l = (int)(item / p.n);
    copy_row<kGather>(p, t, l);
  }
}

}  // namespace

cudaError_t launch_kv_copy(const KvCopyArgs& a, bool gather, cudaStream_t stream) {
  if (a.strides[4] != 1 || (a.d * a.elem) % 16 != 0 || reinterpret_cast<uintptr_t>(a.staging) % 16 != 0 ||
      a.n > a.cap)
    return cudaErrorInvalidValue;
  if (a.n == 0 || a.L == 0) return cudaSuccess;
  KvCopyParams p{};
  p.layer_ptrs = a.layer_ptrs;
  p.slots = a.slots;
  p.heads = a.heads;
  p.staging = static_cast<char*>(a.staging);
  p.n = a.n;
  p.cap = a.cap;
  p.d = a.d;
  p.block_size = a.block_size;
  p.H = a.H;
  p.s_block = a.strides[0];
  p.s_off = a.strides[1];
  p.s_head = a.strides[2];
  p.s_kv = a.strides[3];
  p.elem = a.elem;
  // the per-step gather writes a few MB into host-mapped staging over PCIe, on a side stream next
  // to the step's kernels: a few CTAs keep up with the link and leave the SMs to the step; the
  // scatter of a restore takes the whole device
  const int64_t items = a.n * a.L;
  const int64_t cap = gather ? std::max<int64_t>(32, items / 64) : ((int64_t)1 << 20);
  const unsigned grid = (unsigned)std::min<int64_t>(items, cap);
  if (gather)
    kv_copy_kernel<true><<<grid, 128, 0, stream>>>(p, a.L);
  else
    kv_copy_kernel<false><<<grid, 128, 0, stream>>>(p, a.L);
  return cudaGetLastError();
}

}  // namespace es
