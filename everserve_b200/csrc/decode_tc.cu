// Paged decode attention on the fifth-generation tensor cores (tcgen05, TMEM, TMA), persistent.
//
// One query token per sequence; its G = Hq / Hkv query heads share a kv head (GQA). The work is
// split into items (sequence, kv head, split of 256 positions). A CTA per SM walks the items
// b + k * grid, and per item:
//   * warp 4 lane 0 (producer): TMA of the item's G query rows (two 64-column halves, rows padded
//     to 16 with zeros), then its keys and values in 128-position chunks: per cache block one box
//     per 64-column half, into a ring of 32 KB stages (K0, K1, V0, V1 per item), running up to the
//     ring's depth ahead of the consumers, across items;
//   * warp 5 lane 0 (MMA issuer): S^T = K . Q^T for each chunk (M = 128 positions on the TMEM
//     lanes, N = 16 head columns), then, once P is written, O^T = V^T . P^T over the item's 256
//     positions (M = 128 head dims, V read straight from the cache tile as an MN-major operand);
//     the scores of item n + 1 are computed while the softmax warps finish item n;
//   * warps 0-3 (softmax): thread t owns TMEM lane t: position t of each chunk for the scores,
//     head dim t for the output. Per head the maximum and the sum over the 256 positions are block
//     reductions; P goes to shared memory as bf16 in the MMA's swizzled layout. The item's
//     normalized output, maximum and sum go to the split scratch, and the last split of a
//     (sequence, kv head) to finish (one atomic ticket per pair) merges the splits in split order
//     and writes the bf16 output, as the mma.sync kernel does, so both produce the same partials'
//     format and merge.
// Decode attention is bound by the K/V bytes; the tensor core takes the arithmetic off the warps,
// which keep only the reductions, and the producer keeps up to six stages in flight per SM. Every
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
constexpr int kStages = 6;
constexpr int kStageBytes = 2 * kChunk * 128;  // [half][128 rows][128 B]
constexpr int kHalfBytes = kChunk * 128;
constexpr int kQBytes = 2 * kN * 128;          // [half][16 rows][128 B]
constexpr int kPBytes = (kPart / 64) * kN * 128;  // [64-position chunk][16 rows][128 B]
constexpr int kSoftmax = 128;
constexpr int kThreads = kSoftmax + 64;
constexpr int kTmemCols = 128;  // S0 [0, 32), S1 [32, 64), O [64, 80)
constexpr int kOCol = 64;
constexpr int kSmem = 1024 + kStages * kStageBytes + 2 * kQBytes + kPBytes + 512;
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
  uint8_t* p_s = q_s + 2 * kQBytes;
  uint64_t* bar = reinterpret_cast<uint64_t*>(p_s + kPBytes);
  uint64_t* kv_full = bar;                 // [kStages]
  uint64_t* kv_empty = bar + kStages;      // [kStages]
  uint64_t* q_full = bar + 2 * kStages;    // [2]
  uint64_t* q_empty = q_full + 2;          // [2]
  uint64_t* s_full = q_empty + 2;          // [2]
  uint64_t* s_free = s_full + 2;           // [2]
  uint64_t* p_full = s_free + 2;
  uint64_t* o_full = p_full + 1;
  uint64_t* mma_done = o_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  __shared__ float red_m[4][kN], red_l[4][kN];
  __shared__ int s_fail, s_last;

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
      ptx::mbar_init(&s_full[s], 1);
      ptx::mbar_init(&s_free[s], kSoftmax);
    }
    ptx::mbar_init(p_full, kSoftmax);
    ptx::mbar_init(o_full, 1);
    ptx::mbar_init(mma_done, 1);
    ptx::fence_mbar_init();
  }
  // stale shared memory must be finite (a masked position's P is 0, and 0 * NaN is not), and the
  // query rows above G must stay zero: clear the ring, Q and P once
  for (int i = threadIdx.x; i < (kStages * kStageBytes + 2 * kQBytes + kPBytes) / 16; i += kThreads)
    reinterpret_cast<uint4*>(smem)[i] = make_uint4(0u, 0u, 0u, 0u);
  ptx::fence_proxy_async();
  if (warp == 5) ptx::tmem_alloc(tmem_slot, kTmemCols);
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();  // q, the cache rows and the context lengths come from the kernels before
  pdl_launch();

  if (warp == 4) {
    // ---- producer -----------------------------------------------------------------------------
    if (lane == 0) {
      int n = 0;  // non-empty items so far
      uint32_t q = 0;  // stages issued so far
      bool ok = true;
      for (int it = blockIdx.x; ok && it < p.n_items; it += gridDim.x) {
        const Item x = item_of(p, it);
        if (x.s0 >= x.ctx) continue;
        const int qb = n & 1;
        if (n >= 2 && !ptx::mbar_wait(&q_empty[qb], ((n >> 1) - 1) & 1)) {
          ok = false;
          break;
        }
        ptx::mbar_arrive_expect_tx(&q_full[qb], 2 * G * 128);
        const int qrow = x.b * p.hq + x.kvh * G;
        ptx::tma_load_2d(q_s + qb * kQBytes, &qmap, 0, qrow, &q_full[qb]);
        ptx::tma_load_2d(q_s + qb * kQBytes + kN * 128, &qmap, 64, qrow, &q_full[qb]);
        const int* bt = p.block_tables + (size_t)x.b * p.bt_stride;
        for (int part = 0; part < 4; part++, q++) {
          const int st = (int)(q % kStages);
          if (q >= (uint32_t)kStages && !ptx::mbar_wait(&kv_empty[st], ((q / kStages) - 1) & 1)) {
            ok = false;
            break;
          }
          const int kv = part >> 1, c = part & 1;
          const int first = x.s0 + c * kChunk;
          const int nblk = first >= x.s1 ? 0 : min(kChunk / BS, (x.s1 - first + BS - 1) / BS);
          ptx::mbar_arrive_expect_tx(&kv_full[st], (uint32_t)nblk * BS * 256);
          uint8_t* dst = ring + st * kStageBytes;
          for (int j = 0; j < nblk; j++) {
            const int blk = bt[first / BS + j];
            const int row = ((blk * 2 + kv) * p.hkv + x.kvh) * BS;
            ptx::tma_load_2d(dst + j * BS * 128, &cmap, 0, row, &kv_full[st]);
            ptx::tma_load_2d(dst + kHalfBytes + j * BS * 128, &cmap, 64, row, &kv_full[st]);
          }
        }
        n++;
      }
      if (!ok) s_fail = 1;
      // no copy of this CTA may land after it leaves: wait for the stages still in flight
      for (uint32_t r = q > (uint32_t)kStages ? q - kStages : 0; r < q; r++)
        ptx::mbar_wait(&kv_full[r % kStages], (r / kStages) & 1);
      for (int r = max(0, n - 2); r < n; r++) ptx::mbar_wait(&q_full[r & 1], (r >> 1) & 1);
    }
  } else if (warp == 5) {
    // ---- MMA issuer ---------------------------------------------------------------------------
    if (lane == 0) {
      constexpr uint32_t idesc_s = ptx::idesc_bf16_f32(kChunk, kN);
      constexpr uint32_t idesc_o = ptx::idesc_bf16_f32(D, kN) | (1u << 15);  // A (V^T) MN-major
      bool ok = true;
      int n = 0;
      auto issue_s = [&](int m) -> bool {
        const int qb = m & 1, sb = m & 1;
        if (!ptx::mbar_wait(&q_full[qb], (m >> 1) & 1)) return false;
        if (m >= 2 && !ptx::mbar_wait(&s_free[sb], ((m >> 1) - 1) & 1)) return false;
        for (int c = 0; c < 2; c++) {
          const uint32_t qi = 4u * m + c;
          const int st = (int)(qi % kStages);
          if (!ptx::mbar_wait(&kv_full[st], (qi / kStages) & 1)) return false;
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
        if (!ptx::mbar_wait(p_full, m & 1)) return false;
        for (int c = 0; c < 2; c++) {
          const uint32_t qi = 4u * m + 2 + c;
          const int st = (int)(qi % kStages);
          if (!ptx::mbar_wait(&kv_full[st], (qi / kStages) & 1)) return false;
          ptx::tc_fence_after();
          const uint8_t* vt = ring + st * kStageBytes;
#pragma unroll
          for (int ks = 0; ks < kChunk / 16; ks++) {
            const uint64_t ad = ptx::sw128_mnmajor_desc(ptx::smem_u32(vt + ks * 16 * 128), kHalfBytes);
            const int k = c * kChunk + ks * 16;
            const uint64_t bd = ptx::sw128_kmajor_desc(ptx::smem_u32(p_s + (k >> 6) * kN * 128)) + 2 * ((k >> 4) & 3);
            ptx::mma_f16_ss(tmem + kOCol, ad, bd, idesc_o, (c > 0 || ks > 0) ? 1u : 0u);
          }
          ptx::mma_commit(&kv_empty[st]);
        }
        ptx::mma_commit(o_full);
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
    // ---- softmax warps ------------------------------------------------------------------------
    const int t = threadIdx.x;  // TMEM lane: a position of each chunk, then a head dim
    const uint32_t lane_addr = tmem + ((uint32_t)(warp * 32) << 16);
    const float c = p.scale_log2;
    bool ok = true;
    int n = 0;
    for (int it = blockIdx.x; it < p.n_items; it += gridDim.x) {
      const Item x = item_of(p, it);
      if (x.s0 >= x.ctx) {
        if (x.split == 0)  // an empty history: the output is zero
          for (int i = t; i < G * D; i += kSoftmax)
            p.out[(size_t)x.b * p.out_stride + (size_t)x.kvh * G * D + i] = f2bf(0.f);
        continue;
      }
      const int sb = n & 1;
      ok = ptx::mbar_wait(&s_full[sb], (n >> 1) & 1) && ok;
      ptx::tc_fence_after();
      float s0[kN], s1[kN];
      ptx::tmem_ld16(lane_addr + sb * 32, s0);
      ptx::tmem_ld16(lane_addr + sb * 32 + kN, s1);
      ptx::tc_fence_before();
      ptx::mbar_arrive(&s_free[sb]);
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
          if (lane == 0) red_m[warp][h] = m;
        }
      }
      if (ptx::named_bar_or(1, kSoftmax, !ok)) break;  // the four warps leave together
      float mh[kN], lh[kN];
#pragma unroll
      for (int h = 0; h < kN; h++) {
        if (h < G) {
          mh[h] = fmaxf(fmaxf(red_m[0][h], red_m[1][h]), fmaxf(red_m[2][h], red_m[3][h]));
          const float p0 = exp2f(s0[h] - mh[h]), p1 = exp2f(s1[h] - mh[h]);
          *reinterpret_cast<__nv_bfloat16*>(p_s + p_off(h, t)) = __float2bfloat16(p0);
          *reinterpret_cast<__nv_bfloat16*>(p_s + p_off(h, kChunk + t)) = __float2bfloat16(p1);
          float l = p0 + p1;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xFFFFFFFFu, l, o);
          if (lane == 0) red_l[warp][h] = l;
        }
      }
      ptx::fence_proxy_async();  // the tensor core reads P through the async proxy
      ptx::tc_fence_before();
      ptx::mbar_arrive(p_full);
      ptx::named_bar(1, kSoftmax);
#pragma unroll
      for (int h = 0; h < kN; h++)
        if (h < G) lh[h] = (red_l[0][h] + red_l[1][h]) + (red_l[2][h] + red_l[3][h]);
      ok = ptx::mbar_wait(o_full, n & 1) && ok;
      ptx::tc_fence_after();
      float o[kN];
      ptx::tmem_ld16(lane_addr + kOCol, o);
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
      n++;
      // the last split of the pair merges every split's (o, m, l) in split order
      __threadfence();
      ptx::named_bar(1, kSoftmax);
      const int ns = min(p.max_splits, (x.ctx + kPart - 1) / kPart);
      if (t == 0) {
        int* tk = p.tickets + (size_t)x.b * p.hkv + x.kvh;
        s_last = atomicAdd(tk, 1) == ns - 1;
        if (s_last) *tk = 0;  // every split of this launch has counted: the next launch starts at zero
      }
      ptx::named_bar(1, kSoftmax);
      if (s_last) {
        __threadfence();
        for (int g = 0; g < G; g++) {
          const size_t row0 = ((size_t)x.b * p.hq + x.kvh * G + g) * p.max_splits;
          float m = -INFINITY;
          for (int sp = 0; sp < ns; sp++) m = fmaxf(m, __ldcg(p.part_ml + (row0 + sp) * 2));
          float num = 0.f, den = 0.f;
          for (int sp = 0; sp < ns; sp++) {
            const float w = __ldcg(p.part_ml + (row0 + sp) * 2 + 1) * exp2f(__ldcg(p.part_ml + (row0 + sp) * 2) - m);
            num += w * __ldcg(p.part_o + (row0 + sp) * D + t);
            den += w;
          }
          p.out[(size_t)x.b * p.out_stride + (size_t)(x.kvh * G + g) * D + t] = f2bf(num / den);
        }
      }
    }
    if (!ok && t == 0) s_fail = 1;
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 5) ptx::tmem_dealloc(tmem, kTmemCols);
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
