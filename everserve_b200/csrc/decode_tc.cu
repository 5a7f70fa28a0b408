// Paged decode attention on the fifth-generation tensor cores (tcgen05, TMEM, TMA), persistent.
//
// One query token per sequence; its G = Hq / Hkv query heads share a kv head (GQA). The work is
// split into items (sequence, kv head, split of 256 positions). A CTA per SM walks the items
// b + k * grid, and per item:
//   * warp 8 lane 0 (producer): TMA of the item's G query rows (two 64-column halves, rows padded
//     to 16 with zeros), then its keys and values in 128-position chunks: per cache block one box
//     per 64-column half, into 32 KB stages: a key ring of two (the item's two chunks, free again
//     once the score MMAs have read them) and a value ring of four (two items: values wait for
//     the softmax), so the next item's keys load while this item's values are still held;
//   * warp 9 lane 0 (MMA issuer): S^T = K . Q^T for each chunk (M = 128 positions on the TMEM
//     lanes, N = 16 head columns), then, once P is written, O^T = V^T . P^T over the item's 256
//     positions (M = 128 head dims, V read straight from the cache tile as an MN-major operand);
//     the scores of item n + 1 are computed while the softmax warps finish item n;
//   * warps 0-7 (softmax, two groups of four taking alternate items, each with its own TMEM
//     columns, P buffer and barriers, so one group's reductions, ticket and merge overlap the
//     other's item): thread t of a group owns TMEM lane t: position t of each chunk for the
//     scores, head dim t for the output. Per head the maximum and the sum over the 256 positions are block
//     reductions; P goes to shared memory as bf16 in the MMA's swizzled layout. The item's
//     normalized output, maximum and sum go to the split scratch, and the last split of a
//     (sequence, kv head) to finish (one atomic ticket per pair) merges the splits in split order
//     and writes the bf16 output, as the mma.sync kernel does, so both produce the same partials'
//     format and merge.
// Decode attention is bound by the K/V bytes; the tensor core takes the arithmetic off the warps,
// which keep only the reductions, and the producer keeps up to six stages loaded per SM. Every
// wait is bounded; a wait that runs out sets the status word and the roles leave.
#include <cuda.h>

#include <algorithm>
#include <atomic>
#include <cstdlib>

#include "api.h"
#include "common.cuh"
#include "launch.h"
#include "ptx.cuh"
#include "tmap.h"

namespace es {
namespace dtc {

constexpr int D = 128;                 // head dim (two 64-column halves)
constexpr int kChunk = 128;            // positions per chunk (MMA M of S, K of a PV half)
constexpr int kPart = 256;             // positions per item (two chunks)
constexpr int kN = 16;                 // head columns of the MMAs (G <= 16, zero rows above G)
constexpr int kKStages = 2;               // the key ring: one item's two chunks (freed by the S MMAs)
constexpr int kVStages = 4;               // the value ring: two items (freed by the PV MMAs, later)
constexpr int kStages = kKStages + kVStages;
constexpr int kStageBytes = 2 * kChunk * 128;  // [half][128 rows][128 B]
constexpr int kHalfBytes = kChunk * 128;
constexpr int kQBytes = 2 * kN * 128;          // [half][16 rows][128 B]
constexpr int kPBytes = (kPart / 64) * kN * 128;  // [64-position chunk][16 rows][128 B]
constexpr int kGroup = 128;               // softmax threads of one group (one per TMEM lane)
constexpr int kGroups = 2;                 // items alternate between the groups
constexpr int kThreads = kGroups * kGroup + 64;  // + producer warp + MMA warp
constexpr int kProducerWarp = kGroups * 4, kMmaWarp = kProducerWarp + 1;
constexpr int kTmemCols = 128;  // group g: S at [32 g, 32 g + 32), O at [64 + 16 g, 64 + 16 g + 16)
constexpr int kOCol = 64;
constexpr int kSmem = 1024 + kStages * kStageBytes + 2 * kQBytes + kGroups * kPBytes + 512;
static_assert(kSmem <= 227 * 1024, "shared memory");

struct Params {
  const int* block_tables;
  int bt_stride;
  const int* ctx_lens;
  float* part_o;   // [B, Hq, max_splits, D]
  float* part_ml;  // [B, Hq, max_splits, 2]
  int* tickets;    // [B, Hkv]
  __nv_bfloat16* out;
  int64_t out_stride;
  int B, hq, hkv, max_splits, n_items;
  float scale_log2;
  int* status;
};

struct Item {
  int b, kvh, split, s0, s1, ctx;
};

ES_DEVICE Item item_of(const Params& p, int it) {
  Item x;
  x.split = it % p.max_splits;
  const int rest = it / p.max_splits;
  x.kvh = rest % p.hkv;
  x.b = rest / p.hkv;
  x.ctx = p.ctx_lens[x.b];
  x.s0 = x.split * kPart;
  x.s1 = min(x.ctx, x.s0 + kPart);
  return x;
}

// byte offset of P^T[head h][position k] in the MMA's swizzled K-major layout
ES_DEVICE uint32_t p_off(int h, int k) {
  const int kc = k >> 6, col = k & 63;
  return (uint32_t)(kc * kN * 128 + h * 128 + ((((col * 2) >> 4) ^ (h & 7)) << 4) + ((col * 2) & 15));
}

template <int BS>
__global__ void __launch_bounds__(kThreads, 1)
    decode_tc_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap cmap, Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;
  uint8_t* q_s = ring + kStages * kStageBytes;  // [2 buffers]
  uint8_t* p_s = q_s + 2 * kQBytes;           // [group]
  uint64_t* bar = reinterpret_cast<uint64_t*>(p_s + kGroups * kPBytes);
  uint64_t* kv_full = bar;                 // [kStages]: keys [0, kKStages), values after
  uint64_t* kv_empty = bar + kStages;      // [kStages]
  uint64_t* q_full = bar + 2 * kStages;    // [2]
  uint64_t* q_empty = q_full + 2;          // [2]
  uint64_t* s_full = q_empty + 2;          // [group]
  uint64_t* s_free = s_full + kGroups;     // [group]
  uint64_t* p_full = s_free + kGroups;     // [group]
  uint64_t* o_full = p_full + kGroups;     // [group]
  uint64_t* mma_done = o_full + kGroups;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  __shared__ float red_m[kGroups][4][kN], red_l[kGroups][4][kN];
  __shared__ int s_fail, s_last[kGroups];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.hq / p.hkv;

  if (threadIdx.x == 0) {
    s_fail = 0;
    ptx::prefetch_tmap(&qmap);
    ptx::prefetch_tmap(&cmap);
    for (int s = 0; s < kStages; s++) {
      ptx::mbar_init(&kv_full[s], 1);
      ptx::mbar_init(&kv_empty[s], 1);
    }
    for (int s = 0; s < 2; s++) {
      ptx::mbar_init(&q_full[s], 1);
      ptx::mbar_init(&q_empty[s], 1);
    }
    for (int g = 0; g < kGroups; g++) {
      ptx::mbar_init(&s_full[g], 1);
      ptx::mbar_init(&s_free[g], kGroup);
      ptx::mbar_init(&p_full[g], kGroup);
      ptx::mbar_init(&o_full[g], 1);
    }
    ptx::mbar_init(mma_done, 1);
    ptx::fence_mbar_init();
  }
  // stale shared memory must be finite (a masked position's P is 0, and 0 * NaN is not), and the
  // query rows above G must stay zero: clear the ring, Q and P once
  for (int i = threadIdx.x; i < (kStages * kStageBytes + 2 * kQBytes + kGroups * kPBytes) / 16; i += kThreads)
    reinterpret_cast<uint4*>(smem)[i] = make_uint4(0u, 0u, 0u, 0u);
  ptx::fence_proxy_async();
  if (warp == kMmaWarp) ptx::tmem_alloc(tmem_slot, kTmemCols);
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();  // q, the cache rows and the context lengths come from the kernels before
  pdl_launch();

  if (warp == kProducerWarp) {
    // ---- producer: the whole warp; lane 0 waits and arms the barriers, the lanes issue the
    // copies (one block-table entry per lane, loaded together once per item) --------------------
    int n = 0;  // non-empty items so far
    bool ok = true;
    for (int it = blockIdx.x; ok && it < p.n_items; it += gridDim.x) {
      const Item x = item_of(p, it);
      if (x.s0 >= x.ctx) continue;
      const int qb = n & 1;
      const int nblk_item = (x.s1 - x.s0 + BS - 1) / BS;  // blocks of the item (<= kPart / BS <= 32)
      const int* bt = p.block_tables + (size_t)x.b * p.bt_stride;
      const int my_blk = lane < nblk_item ? bt[x.s0 / BS + lane] : 0;
      if (lane == 0) {
        ok = n < 2 || ptx::mbar_wait(&q_empty[qb], ((n >> 1) - 1) & 1);
        if (ok) {
          ptx::mbar_arrive_expect_tx(&q_full[qb], 2 * G * 128);
          const int qrow = x.b * p.hq + x.kvh * G;
          ptx::tma_load_2d(q_s + qb * kQBytes, &qmap, 0, qrow, &q_full[qb]);
          ptx::tma_load_2d(q_s + qb * kQBytes + kN * 128, &qmap, 64, qrow, &q_full[qb]);
        }
      }
      ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
      for (int part = 0; ok && part < 4; part++) {
        const int kv = part >> 1, c = part & 1;
        // the item's c-th chunk of keys (values): the ring's (2 n + c)-th use
        const uint32_t u = 2u * n + c;
        const int nst = kv ? kVStages : kKStages;
        const int st = (kv ? kKStages : 0) + (int)(u % nst);
        const int first = x.s0 + c * kChunk;
        const int nblk = first >= x.s1 ? 0 : min(kChunk / BS, (x.s1 - first + BS - 1) / BS);
        if (lane == 0) {
          ok = u < (uint32_t)nst || ptx::mbar_wait(&kv_empty[st], ((u / nst) - 1) & 1);
          if (ok) ptx::mbar_arrive_expect_tx(&kv_full[st], (uint32_t)nblk * BS * 256);
        }
        ok = __shfl_sync(0xFFFFFFFFu, ok, 0);  // the stage is armed before any copy to it
        // lane 2 j + h copies block j's half h (at most 2 * kChunk / BS <= 16 copies per chunk)
        const int j = lane >> 1, half = lane & 1;
        const int blk = __shfl_sync(0xFFFFFFFFu, my_blk, (c * (kChunk / BS) + j) & 31);
        if (ok && j < nblk) {
          const int row = ((blk * 2 + kv) * p.hkv + x.kvh) * BS;
          ptx::tma_load_2d(ring + st * kStageBytes + half * kHalfBytes + j * BS * 128, &cmap, half * 64, row,
                           &kv_full[st]);
        }
      }
      if (ok) n++;
    }
    if (lane == 0) {
      if (!ok) s_fail = 1;
      // no copy of this CTA may land after it leaves: wait for the last uses of every stage
      const uint32_t uses = 2u * n;
      for (uint32_t u = uses > (uint32_t)kKStages ? uses - kKStages : 0; u < uses; u++)
        ptx::mbar_wait(&kv_full[u % kKStages], (u / kKStages) & 1);
      for (uint32_t u = uses > (uint32_t)kVStages ? uses - kVStages : 0; u < uses; u++)
        ptx::mbar_wait(&kv_full[kKStages + u % kVStages], (u / kVStages) & 1);
      for (int r = max(0, n - 2); r < n; r++) ptx::mbar_wait(&q_full[r & 1], (r >> 1) & 1);
    }
  } else if (warp == kMmaWarp) {
    // ---- MMA issuer ---------------------------------------------------------------------------
    if (lane == 0) {
      constexpr uint32_t idesc_s = ptx::idesc_bf16_f32(kChunk, kN);
      constexpr uint32_t idesc_o = ptx::idesc_bf16_f32(D, kN) | (1u << 15);  // A (V^T) MN-major
      bool ok = true;
      int n = 0;
      // item m goes to softmax group m & 1: its S and O columns, its P buffer, its barriers
      auto issue_s = [&](int m) -> bool {
        const int qb = m & 1, sb = m & 1;
        if (!ptx::mbar_wait(&q_full[qb], (m >> 1) & 1)) return false;
        if (m >= kGroups && !ptx::mbar_wait(&s_free[sb], ((m >> 1) - 1) & 1)) return false;
        for (int c = 0; c < 2; c++) {
          const uint32_t u = 2u * m + c;
          const int st = (int)(u % kKStages);
          if (!ptx::mbar_wait(&kv_full[st], (u / kKStages) & 1)) return false;
          ptx::tc_fence_after();
          const uint8_t* kt = ring + st * kStageBytes;
#pragma unroll
          for (int ks = 0; ks < D / 16; ks++) {
            const int h = ks >> 2, w = ks & 3;
            const uint64_t ad = ptx::sw128_kmajor_desc(ptx::smem_u32(kt + h * kHalfBytes)) + 2 * w;
            const uint64_t bd = ptx::sw128_kmajor_desc(ptx::smem_u32(q_s + qb * kQBytes + h * kN * 128)) + 2 * w;
            ptx::mma_f16_ss(tmem + sb * 32 + c * kN, ad, bd, idesc_s, ks > 0 ? 1u : 0u);
          }
          ptx::mma_commit(&kv_empty[st]);
        }
        ptx::mma_commit(&s_full[sb]);
        ptx::mma_commit(&q_empty[qb]);
        return true;
      };
      auto issue_pv = [&](int m) -> bool {
        const int g = m & 1;
        if (!ptx::mbar_wait(&p_full[g], (m >> 1) & 1)) return false;
        for (int c = 0; c < 2; c++) {
          const uint32_t u = 2u * m + c;
          const int st = kKStages + (int)(u % kVStages);
          if (!ptx::mbar_wait(&kv_full[st], (u / kVStages) & 1)) return false;
          ptx::tc_fence_after();
          const uint8_t* vt = ring + st * kStageBytes;
#pragma unroll
          for (int ks = 0; ks < kChunk / 16; ks++) {
            const uint64_t ad = ptx::sw128_mnmajor_desc(ptx::smem_u32(vt + ks * 16 * 128), kHalfBytes);
            const int k = c * kChunk + ks * 16;
            const uint64_t bd =
                ptx::sw128_kmajor_desc(ptx::smem_u32(p_s + g * kPBytes + (k >> 6) * kN * 128)) + 2 * ((k >> 4) & 3);
            ptx::mma_f16_ss(tmem + kOCol + g * kN, ad, bd, idesc_o, (c > 0 || ks > 0) ? 1u : 0u);
          }
          ptx::mma_commit(&kv_empty[st]);
        }
        ptx::mma_commit(&o_full[g]);
        return true;
      };
      for (int it = blockIdx.x; ok && it < p.n_items; it += gridDim.x) {
        const Item x = item_of(p, it);
        if (x.s0 >= x.ctx) continue;
        ok = issue_s(n);
        if (ok && n >= 1) ok = issue_pv(n - 1);
        n++;
      }
      if (ok && n >= 1) ok = issue_pv(n - 1);
      if (!ok) s_fail = 1;
      ptx::mma_commit(mma_done);  // every MMA issued above has completed once this arrives
      ptx::mbar_wait(mma_done, 0);
    }
  } else {
    // ---- softmax groups: group g takes the CTA's non-empty items n with n % 2 == g -------------
    const int g = warp >> 2, wq = warp & 3;
    const int t = (warp & 3) * 32 + lane;  // TMEM lane: a position of each chunk, then a head dim
    const uint32_t lane_addr = tmem + ((uint32_t)(wq * 32) << 16);
    const int bar_id = 1 + g;
    uint8_t* pg = p_s + g * kPBytes;
    const float c = p.scale_log2;
    bool ok = true;
    int n = 0;
    for (int it = blockIdx.x; it < p.n_items; it += gridDim.x) {
      const Item x = item_of(p, it);
      if (x.s0 >= x.ctx) {
        if (x.split == 0 && g == 0)  // an empty history: the output is zero
          for (int i = t; i < G * D; i += kGroup)
            p.out[(size_t)x.b * p.out_stride + (size_t)x.kvh * G * D + i] = f2bf(0.f);
        continue;
      }
      const int mine = n & 1, jj = n >> 1;
      n++;
      if (mine != g) continue;
      ok = ptx::mbar_wait(&s_full[g], jj & 1) && ok;
      ptx::tc_fence_after();
      float s0[kN], s1[kN];
      ptx::tmem_ld16(lane_addr + g * 32, s0);
      ptx::tmem_ld16(lane_addr + g * 32 + kN, s1);
      ptx::tc_fence_before();
      ptx::mbar_arrive(&s_free[g]);
      const bool v0 = x.s0 + t < x.s1, v1 = x.s0 + kChunk + t < x.s1;
      // per head: the maximum over the item's positions
#pragma unroll
      for (int h = 0; h < kN; h++) {
        s0[h] = v0 ? s0[h] * c : -INFINITY;
        s1[h] = v1 ? s1[h] * c : -INFINITY;
        if (h < G) {
          float m = fmaxf(s0[h], s1[h]);
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
          if (lane == 0) red_m[g][wq][h] = m;
        }
      }
      if (ptx::named_bar_or(bar_id, kGroup, !ok)) break;  // the group's four warps leave together
      float mh[kN], lh[kN];
#pragma unroll
      for (int h = 0; h < kN; h++) {
        if (h < G) {
          mh[h] = fmaxf(fmaxf(red_m[g][0][h], red_m[g][1][h]), fmaxf(red_m[g][2][h], red_m[g][3][h]));
          const float p0 = exp2f(s0[h] - mh[h]), p1 = exp2f(s1[h] - mh[h]);
          *reinterpret_cast<__nv_bfloat16*>(pg + p_off(h, t)) = __float2bfloat16(p0);
          *reinterpret_cast<__nv_bfloat16*>(pg + p_off(h, kChunk + t)) = __float2bfloat16(p1);
          float l = p0 + p1;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xFFFFFFFFu, l, o);
          if (lane == 0) red_l[g][wq][h] = l;
        }
      }
      ptx::fence_proxy_async();  // the tensor core reads P through the async proxy
      ptx::tc_fence_before();
      ptx::mbar_arrive(&p_full[g]);
      ptx::named_bar(bar_id, kGroup);
#pragma unroll
      for (int h = 0; h < kN; h++)
        if (h < G) lh[h] = (red_l[g][0][h] + red_l[g][1][h]) + (red_l[g][2][h] + red_l[g][3][h]);
      ok = ptx::mbar_wait(&o_full[g], jj & 1) && ok;
      ptx::tc_fence_after();
      float o[kN];
      ptx::tmem_ld16(lane_addr + kOCol + g * kN, o);
      ptx::tc_fence_before();
      // this split's normalized output, maximum and sum (the merge's input format)
#pragma unroll
      for (int h = 0; h < kN; h++) {
        if (h < G) {
          const size_t row = ((size_t)x.b * p.hq + x.kvh * G + h) * p.max_splits + x.split;
          p.part_o[row * D + t] = o[h] / lh[h];
          if (t == 0) {
            p.part_ml[row * 2] = mh[h];
            p.part_ml[row * 2 + 1] = lh[h];
          }
        }
      }
      // the last split of the pair merges every split's (o, m, l) in split order; the group's
      // writes are ordered before its ticket by the barrier and one fence
      ptx::named_bar(bar_id, kGroup);
      const int ns = min(p.max_splits, (x.ctx + kPart - 1) / kPart);
      if (t == 0) {
        __threadfence();
        int* tk = p.tickets + (size_t)x.b * p.hkv + x.kvh;
        const bool last = atomicAdd(tk, 1) == ns - 1;
        if (last) *tk = 0;  // every split of this launch has counted: the next launch starts at zero
        s_last[g] = last;
      }
      ptx::named_bar(bar_id, kGroup);
      if (s_last[g]) {
        __threadfence();
        for (int hh = 0; hh < G; hh++) {
          const size_t row0 = ((size_t)x.b * p.hq + x.kvh * G + hh) * p.max_splits;
          const float* ml = p.part_ml + row0 * 2;
          const float* po = p.part_o + row0 * D + t;
          // the splits' values in batches of eight independent loads, combined in split order
          float m = -INFINITY;
          for (int b0 = 0; b0 < ns; b0 += 8) {
            float v[8];
#pragma unroll
            for (int u = 0; u < 8; u++) v[u] = b0 + u < ns ? __ldcg(ml + (b0 + u) * 2) : -INFINITY;
#pragma unroll
            for (int u = 0; u < 8; u++) m = fmaxf(m, v[u]);
          }
          float num = 0.f, den = 0.f;
          for (int b0 = 0; b0 < ns; b0 += 8) {
            float mm[8], ll[8], oo[8];
#pragma unroll
            for (int u = 0; u < 8; u++) {
              const bool in = b0 + u < ns;
              mm[u] = in ? __ldcg(ml + (b0 + u) * 2) : 0.f;
              ll[u] = in ? __ldcg(ml + (b0 + u) * 2 + 1) : 0.f;
              oo[u] = in ? __ldcg(po + (size_t)(b0 + u) * D) : 0.f;
            }
#pragma unroll
            for (int u = 0; u < 8; u++) {
              if (b0 + u < ns) {
                const float w = ll[u] * exp2f(mm[u] - m);
                num += w * oo[u];
                den += w;
              }
            }
          }
          p.out[(size_t)x.b * p.out_stride + (size_t)(x.kvh * G + hh) * D + t] = f2bf(num / den);
        }
      }
    }
    if (!ok && t == 0) s_fail = 1;
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) ptx::tmem_dealloc(tmem, kTmemCols);
  if (threadIdx.x == 0 && s_fail && p.status) atomicExch(p.status, (int)kTimeout);
}

template <int BS>
cudaError_t launch(const CUtensorMap& qm, const CUtensorMap& cm, const Params& p, int grid, cudaStream_t stream) {
  static std::atomic<uint64_t> configured{0};
  cudaError_t e = once_per_device(configured, [] {
    return cudaFuncSetAttribute(decode_tc_kernel<BS>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
  });
  if (e != cudaSuccess) return e;
  return launch_ex(decode_tc_kernel<BS>, dim3(grid), dim3(kThreads), kSmem, stream, 0, qm, cm, p);
}

}  // namespace dtc

bool decode_tc_supported(const DecodeArgs& a) {
  const int G = a.hkv > 0 ? a.hq / a.hkv : 0;
  return a.d == 128 && (a.block_size == 16 || a.block_size == 32) && G >= 1 && G <= dtc::kN &&
         a.hq % a.hkv == 0 && a.part_tokens == dtc::kPart && a.q_stride == (int64_t)a.hq * a.d &&
         a.tickets != nullptr;
}

cudaError_t launch_decode_tc_maps(const DecodeArgs& a, const CUtensorMap& qm, const CUtensorMap& cm,
                                  cudaStream_t stream) {
  if (!decode_tc_supported(a)) return cudaErrorInvalidValue;
  if (a.B == 0) return cudaSuccess;
  dtc::Params p{};
  p.block_tables = a.block_tables;
  p.bt_stride = (int)a.bt_stride;
  p.ctx_lens = a.ctx_lens;
  p.part_o = a.part_o;
  p.part_ml = a.part_ml;
  p.tickets = a.tickets;
  p.out = static_cast<__nv_bfloat16*>(a.out);
  p.out_stride = a.out_stride;
  p.B = a.B;
  p.hq = a.hq;
  p.hkv = a.hkv;
  p.max_splits = a.max_splits;
  p.n_items = a.B * a.hkv * a.max_splits;
  p.scale_log2 = a.scale * 1.4426950408889634f;
  p.status = a.status;
  static int sms[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (sms[dev] == 0 && cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return cudaErrorInvalidDevice;
  const int grid = std::min(p.n_items, sms[dev]);  // persistent: one CTA per SM
  return a.block_size == 16 ? dtc::launch<16>(qm, cm, p, grid, stream) : dtc::launch<32>(qm, cm, p, grid, stream);
}

cudaError_t launch_decode_tc(const DecodeArgs& a, cudaStream_t stream) {
  if (!decode_tc_supported(a)) return cudaErrorInvalidValue;
  if (a.B == 0) return cudaSuccess;
  CUtensorMap qm, cm;
  // q as [B * Hq rows, D]: one box = the G query rows of a kv head, one 64-column half
  cudaError_t e = tmap::bf16_2d(&qm, const_cast<void*>(a.q), (int64_t)a.B * a.hq, a.d, a.d, a.hq / a.hkv, 64);
  if (e != cudaSuccess) return e;
  // the cache as [num_blocks * 2 * Hkv * BS rows, D]: one box = a block's rows, one 64-column half
  e = tmap::bf16_2d(&cm, const_cast<void*>(a.cache), a.num_blocks * 2 * a.hkv * a.block_size, a.d, a.d, a.block_size,
                    64);
  if (e != cudaSuccess) return e;
  return launch_decode_tc_maps(a, qm, cm, stream);
}

}  // namespace es
