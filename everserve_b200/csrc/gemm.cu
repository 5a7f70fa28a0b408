// tcgen05 GEMM for the decoder's linear layers: out[M, N] = x[M, K] . w[N, K]^T (+ residual), bf16
// in, fp32 accumulate in TMEM, bf16 out.
//
// Design (sm_100a):
//   * swap-AB: the MMA's M side (128 TMEM lanes) runs over the weight rows and its N side over
//     tokens, so a decode batch of 1..256 tokens fills one MMA without padding the weights;
//   * one CTA = one 128-row weight slice x one token tile x one K split. Warp 0 lane 0 issues TMA
//     loads into a STAGES-deep ring of 128-byte-swizzled shared tiles, warp 1 lane 0 issues
//     tcgen05.mma (128 x BN x 16) into TMEM, all four warps drain TMEM with tcgen05.ld;
//   * split-K for the decode shapes, whose weight streaming needs every SM: each split writes its
//     fp32 partial into a workspace and the last CTA of a tile (a device counter) sums the
//     partials in split order, so the result does not depend on which split finishes last;
//   * the number of splits depends on (N, K) only, never on the token count: a row of the output is
//     the same function of its inputs whatever else is in the batch.
// Every mbarrier wait is bounded by the global timer; a wait that runs out writes a status word.
#include <cuda.h>

#include "api.h"
#include "common.cuh"
#include "ptx.cuh"
#include "tmap.h"

namespace es {
namespace gemm {

constexpr int BM = 128;  // weight rows per tile (MMA M)
constexpr int BK = 64;   // bf16 per k-block: one 128-byte swizzle row
constexpr int kThreads = 128;

template <int BN>
struct Cfg {
  static constexpr int kStages = BN <= 64 ? 8 : (BN == 128 ? 6 : 4);
  static constexpr int kABytes = BM * BK * 2;
  static constexpr int kBBytes = BN * BK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTmemCols = BN < 32 ? 32 : BN;
  // tiles + barriers + tmem slot, plus 1 KB so the tile base can be aligned to 1024
  static constexpr int kSmem = kStages * kStageBytes + 1024 + 256;
};

struct Params {
  __nv_bfloat16* out;
  const __nv_bfloat16* residual;  // optional, same shape as out
  float* ws;                      // [splits, M, N] fp32 when splits > 1
  int* counters;                  // one per (n tile, m tile) when splits > 1
  int* status;
  int M, N, K;
  int ldo, ldr;
  int kb_total, kb_per_split, splits;
};

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x, Params p) {
  using C = Cfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* a_tiles = smem;
  uint8_t* b_tiles = smem + C::kStages * C::kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kStages * C::kStageBytes);
  uint64_t* empty = full + C::kStages;
  uint64_t* done = empty + C::kStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  __shared__ int s_last;
  __shared__ int s_fail;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * BM;
  const int m0 = blockIdx.y * BN;
  const int split = blockIdx.z;
  const int kb0 = split * p.kb_per_split;
  const int kb1 = min(p.kb_total, kb0 + p.kb_per_split);
  const int nkb = kb1 - kb0;

  if (threadIdx.x == 0) {
    s_fail = 0;
    ptx::prefetch_tmap(&tmap_w);
    ptx::prefetch_tmap(&tmap_x);
    for (int s = 0; s < C::kStages; s++) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], 1);
    }
    ptx::mbar_init(done, 1);
    ptx::fence_mbar_init();
  }
  if (warp == 2) ptx::tmem_alloc(tmem_slot, C::kTmemCols);
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // producer: TMA ring
    for (int i = 0; i < nkb; i++) {
      const int s = i % C::kStages;
      if (i >= C::kStages) {
        if (!ptx::mbar_wait(&empty[s], ((i / C::kStages) - 1) & 1)) {
          s_fail = 1;
          break;
        }
      }
      ptx::mbar_arrive_expect_tx(&full[s], C::kStageBytes);
      const int kx = (kb0 + i) * BK;
      ptx::tma_load_2d(a_tiles + s * C::kABytes, &tmap_w, kx, n0, &full[s]);
      ptx::tma_load_2d(b_tiles + s * C::kBBytes, &tmap_x, kx, m0, &full[s]);
    }
  } else if (warp == 1 && lane == 0) {
    // MMA issuer
    constexpr uint32_t idesc = ptx::idesc_bf16_f32(BM, BN);
    for (int i = 0; i < nkb; i++) {
      const int s = i % C::kStages;
      if (!ptx::mbar_wait(&full[s], (i / C::kStages) & 1)) {
        s_fail = 1;
        break;
      }
      ptx::tc_fence_after();
      const uint64_t ad = ptx::sw128_kmajor_desc(ptx::smem_u32(a_tiles + s * C::kABytes));
      const uint64_t bd = ptx::sw128_kmajor_desc(ptx::smem_u32(b_tiles + s * C::kBBytes));
#pragma unroll
      for (int k = 0; k < BK / 16; k++) {
        // advancing 16 bf16 (32 bytes) along K inside the swizzle atom adds 2 to the address field
        ptx::mma_f16_ss(tmem, ad + 2 * k, bd + 2 * k, idesc, (i > 0 || k > 0) ? 1u : 0u);
      }
      ptx::mma_commit(&empty[s]);
    }
    ptx::mma_commit(done);
  }
  __syncwarp();

  // epilogue: warp w owns TMEM lanes [32w, 32w + 32) = weight rows n0 + 32w + lane
  const bool ok = ptx::mbar_wait(done, 0);
  ptx::tc_fence_after();
  if (!ok) s_fail = 1;
  const int n = n0 + warp * 32 + lane;
  const bool nvalid = n < p.N;
  const int mrem = p.M - m0;
  if (p.splits == 1) {
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 16) {
      float v[16];
      ptx::tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + c0, v);
      if (nvalid) {
#pragma unroll
        for (int j = 0; j < 16; j++) {
          if (c0 + j < mrem) {
            const int m = m0 + c0 + j;
            float r = v[j];
            if (p.residual) r += bf2f(p.residual[(size_t)m * p.ldr + n]);
            p.out[(size_t)m * p.ldo + n] = f2bf(r);
          }
        }
      }
    }
  } else {
    float* ws = p.ws + (size_t)split * p.M * p.N;
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 16) {
      float v[16];
      ptx::tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + c0, v);
      if (nvalid) {
#pragma unroll
        for (int j = 0; j < 16; j++) {
          if (c0 + j < mrem) __stcg(ws + (size_t)(m0 + c0 + j) * p.N + n, v[j]);
        }
      }
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
      int* ctr = p.counters + blockIdx.y * gridDim.x + blockIdx.x;
      const int prev = atomicAdd(ctr, 1);
      s_last = (prev == p.splits - 1);
      if (s_last) *ctr = 0;  // ready for the next call (and the next graph replay)
    }
    __syncthreads();
    if (s_last) {
      __threadfence();
      // sum the partials in split order: thread = weight row, loop over tokens
      const int mcount = min(BN, mrem);
      for (int c = 0; c < mcount; c++) {
        if (nvalid) {
          const size_t off = (size_t)(m0 + c) * p.N + n;
          float acc = 0.f;
          for (int s = 0; s < p.splits; s++) acc += __ldcg(p.ws + (size_t)s * p.M * p.N + off);
          if (p.residual) acc += bf2f(p.residual[(size_t)(m0 + c) * p.ldr + n]);
          p.out[(size_t)(m0 + c) * p.ldo + n] = f2bf(acc);
        }
      }
    }
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 2) ptx::tmem_dealloc(tmem, C::kTmemCols);
  if (threadIdx.x == 0 && s_fail && p.status) atomicExch(p.status, (int)kTimeout);
}

template <int BN>
cudaError_t launch(const CUtensorMap& mw, const CUtensorMap& mx, const Params& p, int tiles_n, int tiles_m,
                   cudaStream_t stream) {
  using C = Cfg<BN>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(gemm_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  dim3 grid(tiles_n, tiles_m, p.splits);
  gemm_kernel<BN><<<grid, kThreads, C::kSmem, stream>>>(mw, mx, p);
  return cudaGetLastError();
}

}  // namespace gemm

int64_t gemm_pick_bn(int64_t M) {
  if (M <= 16) return 16;
  if (M <= 32) return 32;
  if (M <= 64) return 64;
  if (M <= 128) return 128;
  return 256;
}

int64_t gemm_tiles(int64_t M, int64_t N) {
  const int64_t bn = gemm_pick_bn(M);
  return ((N + gemm::BM - 1) / gemm::BM) * ((M + bn - 1) / bn);
}

// Split count for a weight of N rows and K columns: enough CTAs to give every SM a slice of the
// weight, never below 4 k-blocks per split. A function of (N, K) only.
int64_t gemm_pick_splits(int64_t N, int64_t K, int64_t num_sms) {
  const int64_t tiles = (N + gemm::BM - 1) / gemm::BM;
  const int64_t kb = (K + gemm::BK - 1) / gemm::BK;
  if (tiles >= num_sms) return 1;
  int64_t best = 1;
  double best_score = 0.0;
  for (int64_t s = 1; s <= 16; s++) {
    if (kb / s < 4) break;
    const int64_t kps = (kb + s - 1) / s;
    const int64_t real = (kb + kps - 1) / kps;  // splits that actually hold k-blocks
    if (real != s) continue;
    const int64_t ctas = tiles * s;
    const int64_t waves = (ctas + num_sms - 1) / num_sms;
    const double util = (double)ctas / (double)(waves * num_sms);
    const double score = util - 0.01 * (double)s;  // prefer fewer splits at equal utilisation
    if (score > best_score + 1e-9) {
      best_score = score;
      best = s;
    }
  }
  return best;
}

cudaError_t launch_gemm_bf16(const GemmArgs& a, cudaStream_t stream) {
  if (a.M == 0 || a.N == 0) return cudaSuccess;
  if (a.K % 8 != 0 || (a.ldx * 2) % 16 != 0 || (a.ldw * 2) % 16 != 0) return cudaErrorInvalidValue;
  if (reinterpret_cast<uintptr_t>(a.x) % 16 != 0 || reinterpret_cast<uintptr_t>(a.w) % 16 != 0)
    return cudaErrorInvalidValue;
  const int BN = (int)gemm_pick_bn(a.M);
  const int tiles_n = (int)((a.N + gemm::BM - 1) / gemm::BM);
  const int tiles_m = (int)((a.M + BN - 1) / BN);
  const int kb_total = (int)((a.K + gemm::BK - 1) / gemm::BK);
  if (a.splits < 1 || a.splits > kb_total) return cudaErrorInvalidValue;
  const int kps = (kb_total + a.splits - 1) / a.splits;
  if ((kb_total + kps - 1) / kps != a.splits) return cudaErrorInvalidValue;
  if (a.splits > 1 && (a.ws == nullptr || a.counters == nullptr)) return cudaErrorInvalidValue;
  if (tiles_m > 65535) return cudaErrorInvalidValue;
  gemm::Params p{};
  p.out = static_cast<__nv_bfloat16*>(a.out);
  p.residual = static_cast<const __nv_bfloat16*>(a.residual);
  p.ws = a.ws;
  p.counters = a.counters;
  p.status = a.status;
  p.M = (int)a.M;
  p.N = (int)a.N;
  p.K = (int)a.K;
  p.ldo = (int)a.ldo;
  p.ldr = (int)a.ldr;
  p.kb_total = kb_total;
  p.kb_per_split = kps;
  p.splits = a.splits;
  CUtensorMap mw, mx;
  cudaError_t e = tmap::bf16_2d(&mw, const_cast<void*>(a.w), a.N, a.K, a.ldw, gemm::BM, gemm::BK);
  if (e != cudaSuccess) return e;
  e = tmap::bf16_2d(&mx, const_cast<void*>(a.x), a.M, a.K, a.ldx, BN, gemm::BK);
  if (e != cudaSuccess) return e;
  switch (BN) {
    case 16: return gemm::launch<16>(mw, mx, p, tiles_n, tiles_m, stream);
    case 32: return gemm::launch<32>(mw, mx, p, tiles_n, tiles_m, stream);
    case 64: return gemm::launch<64>(mw, mx, p, tiles_n, tiles_m, stream);
    case 128: return gemm::launch<128>(mw, mx, p, tiles_n, tiles_m, stream);
    default: return gemm::launch<256>(mw, mx, p, tiles_n, tiles_m, stream);
  }
}

}  // namespace es
