// Paged causal attention for prefill on the fifth-generation tensor cores (tcgen05, TMEM, TMA).
//
// Query rows are the step's new tokens of each sequence ([T, Hq, D], positions consecutive within a
// sequence); keys and values come from the paged cache ([num_blocks, 2, Hkv, BS, D]) through the
// sequence's block table, so a chunk of a long prompt sees everything written before it.
//
// One CTA = one tile of up to 128 query rows of one sequence x one query head. The host lists the
// tiles ([seq, first row, rows, first position]) longest-history first, so the causal tail does not
// end the grid on one long tile. Per CTA:
//   * warp 8 lane 0 (producer): TMA of the Q tile once, then per KV tile of 128 keys one TMA box per
//     (cache block, 64-column chunk) of K and of V into a two-stage ring (128-byte swizzle);
//   * warp 9 lane 0 (MMA issuer): S_j = Q.K_j^T into one of two TMEM S buffers, then, once the
//     softmax warps have written P_{j-1}, PV = P_{j-1}.V_{j-1} into the TMEM PV buffer (V is the B
//     operand in MN-major layout straight from the cache, no transpose);
//   * warps 0-7 (softmax): a thread owns one row and half of the tile's columns (warps w and w + 4
//     read the same TMEM lanes). It masks the causal diagonal, exchanges its half-row maximum with
//     its partner, writes P as bf16 into the swizzled shared tile the next MMA reads, and keeps the
//     running output of its half row in registers: O = O * alpha + PV after each PV.
// The tensor core computes S_{j+1} and PV_j while the softmax warps work on tile j, so the MMAs and
// the exponentials overlap. Every wait is bounded; a wait that runs out sets the status word and
// the warps leave their loops together (named-barrier OR), free TMEM and return.
#include <cuda.h>

#include <atomic>

#include "api.h"
#include "common.cuh"
#include "launch.h"
#include "ptx.cuh"
#include "tmap.h"

namespace es {
namespace prefill {

constexpr int kBM = 128;  // query rows per tile (MMA M)
constexpr int kBN = 128;  // keys per KV tile (MMA N of S, K of P.V)
constexpr int kSoftmaxThreads = 256;
constexpr int kThreads = kSoftmaxThreads + 64;  // + producer warp + MMA warp
constexpr int kTmemCols = 512;                  // S0 [0, 128), S1 [128, 256), PV [256, 256 + D)
constexpr float kLog2e = 1.4426950408889634f;

template <int D>
struct Cfg {
  static constexpr int kChunks = D / 64;              // 128-byte column chunks of a Q/K/V row
  static constexpr int kQBytes = kBM * D * 2;
  static constexpr int kKVBytes = kBN * D * 2;        // one K (or V) tile
  static constexpr int kChunkBytes = kBN * 128;       // one 64-column chunk of a 128-row tile
  static constexpr int kPBytes = kBM * kBN * 2;
  static constexpr int kStages = 2;
  static constexpr int kHalf = D / 2;                 // output columns per softmax thread
  static constexpr int kBarBytes = 256;
  static constexpr int kSmem = 1024 + kQBytes + kStages * 2 * kKVBytes + kPBytes + kBarBytes;
  static_assert(kSmem <= 227 * 1024, "shared memory");
};

struct Params {
  const int4* tiles;  // [n]: sequence, first row, rows, first position
  const int* block_tables;
  int bt_stride;
  __nv_bfloat16* out;  // [T, Hq * D]
  int64_t out_stride;
  int hq, hkv;
  float scale_log2;
  int* status;
};

template <int D, int BS>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap cmap, Params p) {
  using C = Cfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* q_s = smem;
  uint8_t* kv_s = q_s + C::kQBytes;  // [stage][K tile, V tile]
  uint8_t* p_s = kv_s + C::kStages * 2 * C::kKVBytes;
  uint64_t* bar = reinterpret_cast<uint64_t*>(p_s + C::kPBytes);
  uint64_t* q_full = bar;
  uint64_t* kv_full = bar + 1;   // [2]
  uint64_t* kv_empty = bar + 3;  // [2]
  uint64_t* s_full = bar + 5;    // [2]
  uint64_t* s_free = bar + 7;    // [2]
  uint64_t* p_full = bar + 9;
  uint64_t* pv_full = bar + 10;
  uint64_t* mma_done = bar + 11;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 12);
  __shared__ float red[2][2][kBM];  // [iteration parity][half][row]: half-row maxima, then sums
  __shared__ int s_fail;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.x;
  const int4 tile = p.tiles[blockIdx.y];
  const int seq = tile.x, row0 = tile.y, nrows = tile.z, pos0 = tile.w;
  const int kvh = h / (p.hq / p.hkv);
  const int last_pos = pos0 + nrows - 1;
  const int J = last_pos / kBN + 1;  // KV tiles this query tile sees
  const int* bt = p.block_tables + (size_t)seq * p.bt_stride;

  if (threadIdx.x == 0) {
    s_fail = 0;
    ptx::prefetch_tmap(&qmap);
    ptx::prefetch_tmap(&cmap);
    ptx::mbar_init(q_full, 1);
    for (int s = 0; s < 2; s++) {
      ptx::mbar_init(&kv_full[s], 1);
      ptx::mbar_init(&kv_empty[s], 1);
      ptx::mbar_init(&s_full[s], 1);
      ptx::mbar_init(&s_free[s], kSoftmaxThreads);
    }
    ptx::mbar_init(p_full, kSoftmaxThreads);
    ptx::mbar_init(pv_full, 1);
    ptx::mbar_init(mma_done, 1);
    ptx::fence_mbar_init();
  }
  if (warp == 9) ptx::tmem_alloc(tmem_slot, kTmemCols);
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();  // q and the cache rows come from the kernels before
  pdl_launch();

  if (warp == 8) {
    // ---- producer -------------------------------------------------------------------------------
    if (lane == 0) {
      ptx::mbar_arrive_expect_tx(q_full, C::kQBytes);
      for (int c = 0; c < C::kChunks; c++) ptx::tma_load_2d(q_s + c * kBM * 128, &qmap, h * D + c * 64, row0, q_full);
      int issued = 0;
      for (int j = 0; j < J; j++) {
        const int s = j & 1;
        if (j >= 2 && !ptx::mbar_wait(&kv_empty[s], ((j >> 1) - 1) & 1)) {
          s_fail = 1;
          break;
        }
        ptx::mbar_arrive_expect_tx(&kv_full[s], 2 * C::kKVBytes);
        uint8_t* kdst = kv_s + s * 2 * C::kKVBytes;
        uint8_t* vdst = kdst + C::kKVBytes;
#pragma unroll 1
        for (int i = 0; i < kBN / BS; i++) {
          const int key0 = j * kBN + i * BS;
          // keys past the last row's position are masked; their box reads the sequence's first block
          const int blk = bt[key0 <= last_pos ? key0 / BS : 0];
          const int row_k = ((blk * 2 + 0) * p.hkv + kvh) * BS;
          const int row_v = ((blk * 2 + 1) * p.hkv + kvh) * BS;
#pragma unroll
          for (int c = 0; c < C::kChunks; c++) {
            ptx::tma_load_2d(kdst + c * C::kChunkBytes + i * BS * 128, &cmap, c * 64, row_k, &kv_full[s]);
            ptx::tma_load_2d(vdst + c * C::kChunkBytes + i * BS * 128, &cmap, c * 64, row_v, &kv_full[s]);
          }
        }
        issued = j + 1;
      }
      // no copy of this CTA may land after it leaves: wait for the last stages issued
      for (int j = max(0, issued - 2); j < issued; j++) ptx::mbar_wait(&kv_full[j & 1], (j >> 1) & 1);
      ptx::mbar_wait(q_full, 0);
    }
  } else if (warp == 9) {
    // ---- MMA issuer -----------------------------------------------------------------------------
    if (lane == 0) {
      constexpr uint32_t idesc_s = ptx::idesc_bf16_f32(kBM, kBN);
      constexpr uint32_t idesc_o = ptx::idesc_bf16_f32_bmn(kBM, D);
      bool ok = ptx::mbar_wait(q_full, 0);
      for (int j = 0; ok && j <= J; j++) {
        if (j < J) {
          const int s = j & 1;
          if (!ptx::mbar_wait(&kv_full[s], (j >> 1) & 1) || (j >= 2 && !ptx::mbar_wait(&s_free[s], ((j >> 1) - 1) & 1))) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          const uint8_t* kt = kv_s + s * 2 * C::kKVBytes;
#pragma unroll
          for (int kk = 0; kk < D / 16; kk++) {
            const int c = kk >> 2, w = kk & 3;
            const uint64_t ad = ptx::sw128_kmajor_desc(ptx::smem_u32(q_s + c * kBM * 128)) + 2 * w;
            const uint64_t bd = ptx::sw128_kmajor_desc(ptx::smem_u32(kt + c * C::kChunkBytes)) + 2 * w;
            ptx::mma_f16_ss(tmem + s * kBN, ad, bd, idesc_s, kk > 0 ? 1u : 0u);
          }
          ptx::mma_commit(&s_full[s]);
        }
        if (j >= 1) {
          const int jj = j - 1, s = jj & 1;
          if (!ptx::mbar_wait(p_full, jj & 1)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          const uint8_t* vt = kv_s + s * 2 * C::kKVBytes + C::kKVBytes;
#pragma unroll
          for (int kk = 0; kk < kBN / 16; kk++) {
            const int c = kk >> 2, w = kk & 3;
            const uint64_t ad = ptx::sw128_kmajor_desc(ptx::smem_u32(p_s + c * kBM * 128)) + 2 * w;
            const uint64_t bd = ptx::sw128_mnmajor_desc(ptx::smem_u32(vt + kk * 16 * 128), C::kChunkBytes);
            ptx::mma_f16_ss(tmem + 2 * kBN, ad, bd, idesc_o, kk > 0 ? 1u : 0u);
          }
          ptx::mma_commit(pv_full);
          ptx::mma_commit(&kv_empty[s]);
        }
      }
      if (!ok) s_fail = 1;
      ptx::mma_commit(mma_done);  // every MMA issued above has completed once this arrives
      ptx::mbar_wait(mma_done, 0);
    }
  } else {
    // ---- softmax warps --------------------------------------------------------------------------
    const int quad = warp & 3, half = warp >> 2;
    const int r = quad * 32 + lane;  // row of the tile (TMEM lane)
    const int pos = pos0 + r;
    const uint32_t lane_addr = tmem + ((uint32_t)(quad * 32) << 16);
    const float c = p.scale_log2;
    float o[C::kHalf];
#pragma unroll
    for (int i = 0; i < C::kHalf; i++) o[i] = 0.f;
    float m = -INFINITY, l = 0.f, alpha_prev = 0.f;
    bool ok = true;
    int j = 0;
    for (; j < J; j++) {
      const int s = j & 1;
      ok = ptx::mbar_wait(&s_full[s], (j >> 1) & 1) && ok;
      ptx::tc_fence_after();
      float sv[64];
#pragma unroll
      for (int q = 0; q < 4; q++) ptx::tmem_ld16(lane_addr + s * kBN + half * 64 + q * 16, sv + q * 16);
      ptx::tc_fence_before();
      ptx::mbar_arrive(&s_free[s]);
      const int key0 = j * kBN + half * 64;
      float mx = -INFINITY;
#pragma unroll
      for (int i = 0; i < 64; i++) {
        if (key0 + i > pos) sv[i] = -INFINITY;
        mx = fmaxf(mx, sv[i]);
      }
      red[j & 1][half][r] = mx;
      if (ptx::named_bar_or(1, kSoftmaxThreads, !ok)) break;  // all 256 threads leave together
      mx = fmaxf(mx, red[j & 1][half ^ 1][r]);
      const float m_new = fmaxf(m, mx);
      const bool none = m_new == -INFINITY;  // a padding row past the sequence sees no key
      const float alpha = (m == -INFINITY) ? 0.f : exp2f((m - m_new) * c);
      const float mc = none ? 0.f : m_new * c;
      uint32_t pk[32];
      float psum = 0.f;
#pragma unroll
      for (int i = 0; i < 32; i++) {
        const float p0 = exp2f(fmaf(sv[2 * i], c, -mc));
        const float p1 = exp2f(fmaf(sv[2 * i + 1], c, -mc));
        psum += p0 + p1;
        pk[i] = ptx::pack_bf16x2(p0, p1);
      }
      l = l * alpha + psum;
      m = m_new;
      if (j >= 1) {
        // PV of the previous tile: its MMA has also finished reading the P buffer
        ok = ptx::mbar_wait(pv_full, (j - 1) & 1) && ok;
        ptx::tc_fence_after();
#pragma unroll
        for (int q = 0; q < C::kHalf / 16; q++) {
          float pv[16];
          ptx::tmem_ld16(lane_addr + 2 * kBN + half * C::kHalf + q * 16, pv);
#pragma unroll
          for (int i = 0; i < 16; i++) o[q * 16 + i] = fmaf(o[q * 16 + i], alpha_prev, pv[i]);
        }
      }
      // P_j, keys half*64 .. +63 = the tile's 64-column chunk `half`, as the MMA's swizzled layout
      uint8_t* prow = p_s + half * kBM * 128 + r * 128;
#pragma unroll
      for (int u = 0; u < 8; u++)
        *reinterpret_cast<uint4*>(prow + ((u ^ (r & 7)) << 4)) = make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
      ptx::fence_proxy_async();  // the tensor core reads P through the async proxy
      ptx::tc_fence_before();
      ptx::mbar_arrive(p_full);
      alpha_prev = alpha;
    }
    if (j == J && J > 0) {
      ok = ptx::mbar_wait(pv_full, (J - 1) & 1) && ok;
      ptx::tc_fence_after();
#pragma unroll
      for (int q = 0; q < C::kHalf / 16; q++) {
        float pv[16];
        ptx::tmem_ld16(lane_addr + 2 * kBN + half * C::kHalf + q * 16, pv);
#pragma unroll
        for (int i = 0; i < 16; i++) o[q * 16 + i] = fmaf(o[q * 16 + i], alpha_prev, pv[i]);
      }
    }
    // the row's sum is the two halves' partial sums (both taken against the same maxima)
    red[J & 1][half][r] = l;
    const bool any_fail = ptx::named_bar_or(1, kSoftmaxThreads, !ok || j != J);
    if (!any_fail && r < nrows) {
      const float inv = 1.f / (l + red[J & 1][half ^ 1][r]);
      __nv_bfloat16* dst = p.out + (size_t)(row0 + r) * p.out_stride + (size_t)h * D + half * C::kHalf;
#pragma unroll
      for (int u = 0; u < C::kHalf / 8; u++) {
        float f[8];
#pragma unroll
        for (int i = 0; i < 8; i++) f[i] = o[u * 8 + i] * inv;
        reinterpret_cast<uint4*>(dst)[u] = pack8(f);
      }
    }
    if (any_fail && threadIdx.x == 0) s_fail = 1;
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 9) ptx::tmem_dealloc(tmem, kTmemCols);
  if (threadIdx.x == 0 && s_fail && p.status) atomicExch(p.status, (int)kTimeout);
}

template <int D, int BS>
cudaError_t launch(const CUtensorMap& qm, const CUtensorMap& cm, const Params& p, int n_tiles, cudaStream_t stream) {
  using C = Cfg<D>;
  static std::atomic<uint64_t> configured{0};
  cudaError_t e = once_per_device(configured, [] {
    return cudaFuncSetAttribute(prefill_kernel<D, BS>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
  });
  if (e != cudaSuccess) return e;
  return launch_ex(prefill_kernel<D, BS>, dim3(p.hq, n_tiles), dim3(kThreads), C::kSmem, stream, 0, qm, cm, p);
}

}  // namespace prefill

cudaError_t launch_paged_prefill(const PrefillArgs& a, cudaStream_t stream) {
  if (a.n_tiles == 0 || a.T == 0) return cudaSuccess;
  if (a.hkv <= 0 || a.hq % a.hkv != 0 || a.n_tiles > 65535 || a.hq > 65535) return cudaErrorInvalidValue;
  if (!((a.d == 128 || a.d == 64) && (a.block_size == 16 || a.block_size == 32))) return cudaErrorInvalidValue;
  if (a.q_stride != (int64_t)a.hq * a.d || a.out_stride % 8 != 0) return cudaErrorInvalidValue;
  if (reinterpret_cast<uintptr_t>(a.out) % 16 != 0) return cudaErrorInvalidValue;
  prefill::Params p{};
  p.tiles = reinterpret_cast<const int4*>(a.tiles);
  p.block_tables = a.block_tables;
  p.bt_stride = (int)a.bt_stride;
  p.out = static_cast<__nv_bfloat16*>(a.out);
  p.out_stride = a.out_stride;
  p.hq = a.hq;
  p.hkv = a.hkv;
  p.scale_log2 = a.scale * prefill::kLog2e;
  p.status = a.status;
  CUtensorMap qm, cm;
  cudaError_t e = tmap::bf16_2d(&qm, const_cast<void*>(a.q), a.T, (int64_t)a.hq * a.d, a.q_stride, prefill::kBM, 64);
  if (e != cudaSuccess) return e;
  e = tmap::bf16_2d(&cm, const_cast<void*>(a.cache), a.num_blocks * 2 * a.hkv * a.block_size, a.d, a.d, a.block_size,
                    64);
  if (e != cudaSuccess) return e;
  if (a.d == 128) {
    return a.block_size == 16 ? prefill::launch<128, 16>(qm, cm, p, a.n_tiles, stream)
                              : prefill::launch<128, 32>(qm, cm, p, a.n_tiles, stream);
  }
  return a.block_size == 16 ? prefill::launch<64, 16>(qm, cm, p, a.n_tiles, stream)
                            : prefill::launch<64, 32>(qm, cm, p, a.n_tiles, stream);
}

}  // namespace es
