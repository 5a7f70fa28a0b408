// Stream-K decode GEMM: out[M, N] = x[M, K] . w[N, K]^T for decode batches (M <= 64 tokens).
//
// A decode step streams every weight once, so a GEMM's time is its weight bytes over the share of
// HBM bandwidth its SMs pull; any SM that runs out of work early leaves bandwidth unused. Tiled
// grids leave such tails whenever the tile count is not a multiple of the CTA slots (224 tiles of
// gate_up on 296 slots: half the SMs stream two tiles, half one). Here the work is cut evenly
// instead: the N/128 weight tiles x K/64 k-blocks form one sequence of units, and each of the
// grid's G = 2 x #SMs persistent CTAs takes a contiguous run of U/G units, crossing tile
// boundaries where its run does.
//
// Per CTA (192 threads, two per SM): warp 0 lane 0 streams its units' weight and activation tiles
// by TMA (128-byte swizzle) into a 4-stage ring, warp 1 lane 0 issues tcgen05.mma (swap-AB: weight
// rows on M = 128, tokens on N = 64) into TMEM, one accumulator per segment of the run (the part of
// a tile it covers; the first segment keeps its own, the others take two in turn), and warps 2-5
// drain finished segments while the next ones accumulate:
//   * a segment covering a whole tile writes its output directly;
//   * a segment that ends before its tile's last k-block (a CTA's last segment) stores its fp32
//     partial in the workspace slot of its CTA and raises its flag (the launch's epoch number);
//   * the segment holding a tile's last k-block (a CTA's first segment, drained after all the
//     others so no partial ever waits behind a finish) waits for the flags of the CTAs before it
//     that hold the tile's earlier k-blocks, adds their partials to its own in CTA order (a fixed
//     order for the shape), and writes the output.
// The cut depends only on (N, K, G), never on M, so a token's result does not depend on the batch
// around it. Every wait is bounded (a wait that runs out sets the status word).
//
// With `silu` the weight rows come interleaved by 64 (tile t = gate rows 64t..64t+63, then the
// matching up rows) and the epilogue writes silu(gate) * up of the bf16-rounded products, the
// arithmetic of the separate SiLU-mul kernel, for 64 output columns per tile.
#include <cuda.h>

#include <atomic>

#include "api.h"
#include "common.cuh"
#include "launch.h"
#include "ptx.cuh"
#include "tmap.h"

namespace es {
namespace gemm_sk {

constexpr int BM = 128;  // weight rows per tile (MMA M)
constexpr int BN = 64;   // token columns (MMA N): every decode batch
constexpr int BK = 64;   // one 128-byte swizzle row of bf16
constexpr int kStages = 4;
constexpr int kThreads = 192;
constexpr int kCtasPerSm = 2;
constexpr int kABytes = BM * BK * 2;
constexpr int kBBytes = BN * BK * 2;
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kXchgBytes = BN * 64 * 2;  // the up half of a tile as bf16, for the SiLU epilogue
constexpr int kSmem = 1024 + kStages * kStageBytes + kXchgBytes + 256;
constexpr int kTmemCols = 4 * BN;  // the first segment's accumulator, two in turn for the rest (power of 2)
constexpr int kEpi = 128;          // epilogue threads

struct Params {
  __nv_bfloat16* out;
  const __nv_bfloat16* residual;
  int* status;
  int M, N, ldo, ldr;
  int kb, tiles;
  long long units;  // tiles * kb
  int G;            // CTAs of the grid
  float* ws;        // [G][BN][BM] fp32 partials
  uint32_t* sync;   // [0] epoch, [1] CTAs done, [2 + c] flag of CTA c's partial
  const float* scale;
  const __nv_bfloat16* pre;
  int ldp;
  int silu;
};

ES_DEVICE long long unit_begin(const Params& p, int c) { return (long long)c * p.units / p.G; }

ES_DEVICE float pre_terms(const Params& p, float acc, size_t m, int n) {
  if (p.scale) acc *= p.scale[m];
  if (p.pre) acc += bf2f(p.pre[m * p.ldp + n]);
  return acc;
}

__global__ void __launch_bounds__(kThreads, kCtasPerSm)
    sk_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x, Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* a_tiles = smem;
  uint8_t* b_tiles = smem + kStages * kABytes;
  __nv_bfloat16* xchg = reinterpret_cast<__nv_bfloat16*>(smem + kStages * kStageBytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes + kXchgBytes);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;  // [3]: the two turns, then the first segment's
  uint64_t* acc_empty = acc_full + 3;    // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  __shared__ int s_fail;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.x;
  const long long u0 = unit_begin(p, c), u1 = unit_begin(p, c + 1);
  const int n_units = (int)(u1 - u0);

  if (threadIdx.x == 0) {
    s_fail = 0;
    ptx::prefetch_tmap(&tmap_w);
    ptx::prefetch_tmap(&tmap_x);
    for (int s = 0; s < kStages; s++) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 3; b++) ptx::mbar_init(&acc_full[b], 1);
    for (int b = 0; b < 2; b++) ptx::mbar_init(&acc_empty[b], kEpi);
    ptx::fence_mbar_init();
  }
  if (warp == 1) ptx::tmem_alloc(tmem_slot, kTmemCols);
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---- producer: the run's units in order (weights of the first stages before the wait) ----
    if (lane == 0) {
      const uint64_t pol = ptx::policy_evict_first();  // the weights are read once per step
      const int pre = min(n_units, kStages);
      for (int i = 0; i < pre; i++) {
        const long long u = u0 + i;
        const int t = (int)(u / p.kb), k = (int)(u % p.kb);
        ptx::mbar_arrive_expect_tx(&full[i], kStageBytes);
        ptx::tma_load_2d_hint(a_tiles + i * kABytes, &tmap_w, k * BK, t * BM, &full[i], pol);
      }
      pdl_wait();
      pdl_launch();
      for (int i = 0; i < pre; i++) {
        const int k = (int)((u0 + i) % p.kb);
        ptx::tma_load_2d(b_tiles + i * kBBytes, &tmap_x, k * BK, 0, &full[i]);
      }
      for (int i = pre; i < n_units; i++) {
        const int s = i % kStages;
        if (!ptx::mbar_wait(&empty[s], ((i / kStages) - 1) & 1)) {
          s_fail = 1;
          break;
        }
        const long long u = u0 + i;
        const int t = (int)(u / p.kb), k = (int)(u % p.kb);
        ptx::mbar_arrive_expect_tx(&full[s], kStageBytes);
        ptx::tma_load_2d_hint(a_tiles + s * kABytes, &tmap_w, k * BK, t * BM, &full[s], pol);
        ptx::tma_load_2d(b_tiles + s * kBBytes, &tmap_x, k * BK, 0, &full[s]);
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer: one accumulator per segment (a tile's part of the run), two in turn ----
    if (lane == 0) {
      pdl_wait();
      constexpr uint32_t idesc = ptx::idesc_bf16_f32(BM, BN);
      int seg = 0;
      bool ok = true;
      for (int i = 0; i < n_units && ok; seg++) {
        // the first segment (the one that may finish a tile begun by the CTAs before) keeps its own
        // accumulator until the end; the others take two accumulators in turn
        const int b = seg == 0 ? 2 : (seg - 1) & 1;
        const int turn = seg == 0 ? 0 : (seg - 1) >> 1;
        const long long u = u0 + i;
        const int k0 = (int)(u % p.kb);
        const int len = (int)min((long long)(p.kb - k0), u1 - u);
        if (seg >= 3 && !ptx::mbar_wait(&acc_empty[b], (turn - 1) & 1)) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        for (int q = 0; q < len; q++, i++) {
          const int s = i % kStages;
          if (!ptx::mbar_wait(&full[s], (i / kStages) & 1)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          const uint64_t ad = ptx::sw128_kmajor_desc(ptx::smem_u32(a_tiles + s * kABytes));
          const uint64_t bd = ptx::sw128_kmajor_desc(ptx::smem_u32(b_tiles + s * kBBytes));
#pragma unroll
          for (int kk = 0; kk < BK / 16; kk++)
            ptx::mma_f16_ss(tmem + b * BN, ad + 2 * kk, bd + 2 * kk, idesc, (q > 0 || kk > 0) ? 1u : 0u);
          ptx::mma_commit(&empty[s]);
        }
        ptx::mma_commit(&acc_full[b]);  // arrives even after a failure, so the epilogue never waits for nothing
      }
      if (!ok) s_fail = 1;
    }
  } else {
    // ---- epilogue: warps 2-5, thread = weight row r of the tile (TMEM lane) ----
    pdl_wait();
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const int et = threadIdx.x - 64;  // 0..127
    const uint32_t epoch = ptx::ld_acquire_gpu(p.sync) + 1;
    const int mcount = min(p.M, BN);
    uint32_t* flags = p.sync + 2;
    bool ok = true;
    // one segment: its accumulator drained, then parked (a tile's first k-blocks), finished (the
    // tile's last k-blocks: the earlier CTAs' partials added) or written whole
    auto segment = [&](int seg, long long u, int len) {
      const int b = seg == 0 ? 2 : (seg - 1) & 1;
      const int turn = seg == 0 ? 0 : (seg - 1) >> 1;
      const int t = (int)(u / p.kb);
      const int k0 = (int)(u % p.kb);
      const int k1 = k0 + len;
      ok = ptx::mbar_wait(&acc_full[b], turn & 1) && ok;
      ptx::tc_fence_after();
      float v[BN];
      const uint32_t taddr = tmem + ((uint32_t)(quad * 32) << 16) + b * BN;
#pragma unroll
      for (int c0 = 0; c0 < BN; c0 += 16) ptx::tmem_ld16(taddr + c0, v + c0);
      ptx::tc_fence_before();
      if (b < 2) ptx::mbar_arrive(&acc_empty[b]);
      if (k1 < p.kb) {
        // a partial of the tile's first k-blocks: park it for the CTA that finishes the tile
        float* slot = p.ws + (size_t)c * BN * BM;
#pragma unroll
        for (int col = 0; col < BN; col++)
          if (col < mcount) slot[col * BM + r] = v[col];
        __threadfence();
        ptx::named_bar(1, kEpi);
        if (et == 0) ptx::st_release_gpu(flags + c, epoch);
        return;
      }
      if (k0 > 0) {
        // finish the tile: this CTA's k-blocks (the tile's last), then the partials of the CTAs
        // before it in CTA order (a fixed order for the shape)
        int first = c - 1;
        const long long tile_u0 = (long long)t * p.kb;
        while (first > 0 && unit_begin(p, first) > tile_u0) first--;
        for (int cc = first; cc < c; cc++) {
          if (et == 0) {
            const uint64_t t0 = global_ns();
            uint32_t spins = 0;
            while (ptx::ld_acquire_gpu(flags + cc) != epoch) {
              if ((++spins & 255u) == 0 && global_ns() - t0 > 2000000000ull) {
                s_fail = 1;
                break;
              }
            }
          }
          ptx::named_bar(1, kEpi);
          const float* slot = p.ws + (size_t)cc * BN * BM;
#pragma unroll
          for (int col = 0; col < BN; col++)
            if (col < mcount) v[col] += __ldcg(slot + col * BM + r);  // past L1
        }
      }
      const int n = t * BM + r;
      if (!p.silu) {
        if (n < p.N) {
#pragma unroll
          for (int col = 0; col < BN; col++) {
            if (col < mcount) {
              float o = pre_terms(p, v[col], (size_t)col, n);
              if (p.residual) o += bf2f(p.residual[(size_t)col * p.ldr + n]);
              p.out[(size_t)col * p.ldo + n] = f2bf(o);
            }
          }
        }
      } else {
        // rows 64..127 of the tile are the up projections of rows 0..63's gates
        ptx::named_bar(1, kEpi);  // the previous tile's readers are done with the exchange buffer
        if (r >= 64) {
#pragma unroll
          for (int col = 0; col < BN; col++)
            if (col < mcount) xchg[col * 64 + (r - 64)] = f2bf(v[col]);
        }
        ptx::named_bar(1, kEpi);
        if (r < 64 && t * 64 + r < p.N / 2) {
#pragma unroll
          for (int col = 0; col < BN; col++) {
            if (col < mcount) {
              const float g = bf2f(f2bf(v[col]));
              const float up = bf2f(xchg[col * 64 + r]);
              p.out[(size_t)col * p.ldo + t * 64 + r] = f2bf(g / (1.f + __expf(-g)) * up);
            }
          }
        }
      }
    };
    // The first segment is drained last: its finish waits for other CTAs' partials, and nothing
    // this CTA parks may wait behind that (or every CTA would wait for the one before it).
    const int len0 = (int)min((long long)(p.kb - (int)(u0 % p.kb)), u1 - u0);
    int seg = 1;
    for (int i = len0; i < n_units; seg++) {
      const long long u = u0 + i;
      const int len = (int)min((long long)(p.kb - (int)(u % p.kb)), u1 - u);
      segment(seg, u, len);
      i += len;
    }
    segment(0, u0, len0);
    if (!ok) s_fail = 1;
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) ptx::tmem_dealloc(tmem, kTmemCols);
  if (threadIdx.x == 0) {
    if (s_fail && p.status) atomicExch(p.status, (int)kTimeout);
    // the last CTA to finish publishes the epoch: the next launch's flags must exceed it
    __threadfence();
    if (atomicAdd(p.sync + 1, 1u) == (uint32_t)p.G - 1) {
      p.sync[1] = 0;
      __threadfence();
      ptx::st_release_gpu(p.sync, ptx::ld_acquire_gpu(p.sync) + 1);
    }
  }
}

}  // namespace gemm_sk

int64_t gemm_sk_ws_floats(int64_t num_sms) { return num_sms * gemm_sk::kCtasPerSm * gemm_sk::BN * gemm_sk::BM; }
int64_t gemm_sk_sync_words(int64_t num_sms) { return 2 + num_sms * gemm_sk::kCtasPerSm; }

cudaError_t launch_gemm_stream(const GemmArgs& a, bool silu, cudaStream_t stream) {
  using namespace gemm_sk;
  if (a.M == 0 || a.N == 0) return cudaSuccess;
  if (a.M > BN || a.K % 8 != 0 || (a.ldx * 2) % 16 != 0 || (a.ldw * 2) % 16 != 0) return cudaErrorInvalidValue;
  if (reinterpret_cast<uintptr_t>(a.x) % 16 != 0 || reinterpret_cast<uintptr_t>(a.w) % 16 != 0)
    return cudaErrorInvalidValue;
  if (a.ws == nullptr || a.sync == nullptr || a.num_sms <= 0) return cudaErrorInvalidValue;
  if (silu && (a.N % BM != 0 || a.residual != nullptr || a.scale != nullptr || a.pre != nullptr))
    return cudaErrorInvalidValue;
  Params p{};
  p.out = static_cast<__nv_bfloat16*>(a.out);
  p.residual = static_cast<const __nv_bfloat16*>(a.residual);
  p.status = a.status;
  p.M = (int)a.M;
  p.N = (int)a.N;
  p.ldo = (int)a.ldo;
  p.ldr = (int)a.ldr;
  p.kb = (int)((a.K + BK - 1) / BK);
  p.tiles = (int)((a.N + BM - 1) / BM);
  p.units = (long long)p.tiles * p.kb;
  p.G = (int)std::min<long long>((long long)a.num_sms * kCtasPerSm, p.units);
  p.ws = a.ws;
  p.sync = a.sync;
  p.scale = a.scale;
  p.pre = static_cast<const __nv_bfloat16*>(a.pre);
  p.ldp = (int)a.ldp;
  p.silu = silu ? 1 : 0;
  CUtensorMap mw, mx;
  cudaError_t e = tmap::bf16_2d(&mw, const_cast<void*>(a.w), a.N, a.K, a.ldw, BM, BK);
  if (e != cudaSuccess) return e;
  e = tmap::bf16_2d(&mx, const_cast<void*>(a.x), a.M, a.K, a.ldx, BN, BK);
  if (e != cudaSuccess) return e;
  static std::atomic<uint64_t> configured{0};
  e = once_per_device(configured, [] {
    return cudaFuncSetAttribute(sk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
  });
  if (e != cudaSuccess) return e;
  return launch_ex(sk_kernel, dim3(p.G), dim3(kThreads), kSmem, stream, 0, mw, mx, p);
}

}  // namespace es
