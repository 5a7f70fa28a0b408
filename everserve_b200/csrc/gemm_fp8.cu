// Block-scaled fp8 GEMM: out[M, N] = sum over 128-wide K blocks kb of
//     (x8[M, kb] . w8[N, kb]^T) * x_scale[m, kb] * w_scale[n / 128, kb]
// with e4m3 operands (x: one scale per token and 128 K; w: one scale per 128 x 128 block), fp32
// accumulation, bf16 out. This is the weight format of the fp8 serving configuration: a decode step
// reads half the bytes of bf16 weights.
//
// Design (sm_100a), the bf16 decode GEMM's shape (gemm.cu) with the scales applied per K block:
//   * swap-AB: weight rows on the MMA's M = 128 (TMEM lanes), tokens on N = 64; token tiles of 64
//     over M in the grid;
//   * a 128-wide fp8 K block is one 128-byte swizzle row, so A/B tiles are the bf16 kernel's;
//     tcgen05.mma kind::f8f6f4 takes K = 32 per instruction, four per block;
//   * every K block accumulates into one of two TMEM accumulators in turn (accumulate off at the
//     block's first MMA). The epilogue warps drain a block's accumulator while the next block's MMAs
//     run, and add it into fp32 registers scaled by x_scale[m, kb] * w_scale[tile, kb];
//   * split-K over a thread-block cluster for decode shapes (the bf16 kernel's plan): each CTA's
//     scaled fp32 partial goes to its shared memory and the cluster sums them in rank order through
//     distributed shared memory. The split depends on (N, K, #SMs), never on M.
// With `silu` the weight rows come gate/up interleaved by 64 and the epilogue writes silu(gate) * up
// of the bf16-rounded sums (the layout and arithmetic of the bf16 kernel's SiLU epilogue).
// Every wait is bounded; a wait that runs out sets the status word.
#include <cuda.h>
#include <cuda_fp8.h>

#include <algorithm>
#include <atomic>

#include "api.h"
#include "common.cuh"
#include "launch.h"
#include "ptx.cuh"
#include "tmap.h"

namespace es {
namespace gemm8 {

constexpr int BM = 128;  // weight rows per tile (MMA M)
constexpr int BN = 64;   // tokens per tile (MMA N)
constexpr int BK = 128;  // fp8 per K block: one 128-byte swizzle row, one scale
constexpr int kThreads = 192;
constexpr int kStages = 4;
constexpr int kABytes = BM * BK;
constexpr int kBBytes = BN * BK;
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kSmem = 1024 + kStages * kStageBytes + 256;
constexpr int kTmemCols = 2 * BN;
static_assert(BN * BM * 4 <= kStages * kStageBytes, "the partial tile fits the drained ring");

struct Params {
  __nv_bfloat16* out;
  const __nv_bfloat16* residual;
  const float* x_scale;  // [M, kb] (row stride xs_ld)
  const float* w_scale;  // [ceil(N / 128), kb] (row stride ws_ld)
  int* status;
  int M, N, ldo, ldr, xs_ld, ws_ld;
  int kb, splits, silu;
};

// instruction descriptor of tcgen05.mma kind::f8f6f4: e4m3 A and B (format 0), both K-major, fp32 D
__host__ __device__ constexpr uint32_t idesc_e4m3_f32(int m, int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

ES_DEVICE void mma_f8_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__global__ void __launch_bounds__(kThreads, 1)
    fp8_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x, Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* a_tiles = smem;
  uint8_t* b_tiles = smem + kStages * kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;  // [2]
  uint64_t* acc_empty = acc_full + 2;    // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  float* partial = reinterpret_cast<float*>(smem);  // [BN][BM] once the ring is drained
  __shared__ int s_fail;
  __shared__ float s_scale[2][BN];  // per K block: w_scale x x_scale of each token (two in turn)

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x;
  const int n0 = tile * BM;
  const int m0 = blockIdx.y * BN;
  const int S = p.splits;
  const int kps = (p.kb + S - 1) / S;
  const int kb0 = blockIdx.z * kps;
  const int nkb = max(0, min(p.kb, kb0 + kps) - kb0);

  if (threadIdx.x == 0) {
    s_fail = 0;
    ptx::prefetch_tmap(&tmap_w);
    ptx::prefetch_tmap(&tmap_x);
    for (int s = 0; s < kStages; s++) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      ptx::mbar_init(&acc_full[b], 1);
      ptx::mbar_init(&acc_empty[b], 128);
    }
    ptx::fence_mbar_init();
  }
  if (warp == 1) ptx::tmem_alloc(tmem_slot, kTmemCols);
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  float acc[BN];
#pragma unroll
  for (int c = 0; c < BN; c++) acc[c] = 0.f;
  const int mcount = min(BN, p.M - m0);

  if (warp == 0) {
    if (lane == 0) {
      // weights of the first stages before the wait (no kernel of the step writes them)
      const int pre = min(nkb, kStages);
      for (int i = 0; i < pre; i++) {
        ptx::mbar_arrive_expect_tx(&full[i], kStageBytes);
        ptx::tma_load_2d(a_tiles + i * kABytes, &tmap_w, (kb0 + i) * BK, n0, &full[i]);
      }
      pdl_wait();
      pdl_launch();
      for (int i = 0; i < pre; i++) ptx::tma_load_2d(b_tiles + i * kBBytes, &tmap_x, (kb0 + i) * BK, m0, &full[i]);
      for (int i = pre; i < nkb; i++) {
        const int s = i % kStages;
        if (!ptx::mbar_wait(&empty[s], ((i / kStages) - 1) & 1)) {
          s_fail = 1;
          break;
        }
        ptx::mbar_arrive_expect_tx(&full[s], kStageBytes);
        ptx::tma_load_2d(a_tiles + s * kABytes, &tmap_w, (kb0 + i) * BK, n0, &full[s]);
        ptx::tma_load_2d(b_tiles + s * kBBytes, &tmap_x, (kb0 + i) * BK, m0, &full[s]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      pdl_wait();
      constexpr uint32_t idesc = idesc_e4m3_f32(BM, BN);
      for (int i = 0; i < nkb; i++) {
        const int s = i % kStages, b = i & 1;
        if ((i >= 2 && !ptx::mbar_wait(&acc_empty[b], ((i >> 1) - 1) & 1)) ||
            !ptx::mbar_wait(&full[s], (i / kStages) & 1)) {
          s_fail = 1;
          break;
        }
        ptx::tc_fence_after();
        const uint64_t ad = ptx::sw128_kmajor_desc(ptx::smem_u32(a_tiles + s * kABytes));
        const uint64_t bd = ptx::sw128_kmajor_desc(ptx::smem_u32(b_tiles + s * kBBytes));
#pragma unroll
        for (int kk = 0; kk < BK / 32; kk++) mma_f8_ss(tmem + b * BN, ad + 2 * kk, bd + 2 * kk, idesc, kk > 0 ? 1u : 0u);
        ptx::mma_commit(&empty[s]);
        ptx::mma_commit(&acc_full[b]);
      }
    }
  } else {
    // epilogue warps 2-5: thread = weight row r; every K block's product, scaled, into registers
    pdl_wait();
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const uint32_t lane_addr = tmem + ((uint32_t)(q * 32) << 16);
    bool ok = true;
    for (int i = 0; i < nkb; i++) {
      const int b = i & 1, kb = kb0 + i;
      // the block's combined scale per token, staged once in shared memory for the 128 threads
      const int et = threadIdx.x - 64;
      if (et < BN) s_scale[i & 1][et] = et < mcount ? p.w_scale[(size_t)tile * p.ws_ld + kb] *
                                                          p.x_scale[(size_t)(m0 + et) * p.xs_ld + kb]
                                                    : 0.f;
      ptx::named_bar(1, 128);
      ok = ptx::mbar_wait(&acc_full[b], (i >> 1) & 1) && ok;
      ptx::tc_fence_after();
#pragma unroll
      for (int c0 = 0; c0 < BN; c0 += 16) {
        float v[16];
        ptx::tmem_ld16(lane_addr + b * BN + c0, v);
#pragma unroll
        for (int c = 0; c < 16; c++) acc[c0 + c] = fmaf(v[c], s_scale[i & 1][c0 + c], acc[c0 + c]);
      }
      ptx::tc_fence_before();
      ptx::mbar_arrive(&acc_empty[b]);
    }
    if (!ok) s_fail = 1;
  }
  __syncwarp();

  // this CTA's scaled partial into its (drained) ring, then the cluster's sum by row slices
  if (warp >= 2) {
    const int r = (warp & 3) * 32 + lane;
#pragma unroll
    for (int c = 0; c < BN; c++) partial[c * BM + r] = acc[c];
  }
  ptx::cluster_sync();
  const uint32_t rank = ptx::cluster_rank();
  const uint32_t local = ptx::smem_u32(partial);
  if (!p.silu) {
    const int rows = ((BM / S) + 3) & ~3;
    const int r0 = min(BM, (int)rank * rows);
    const int r1 = (int)rank + 1 == S ? BM : min(BM, r0 + rows);
    const int span4 = (r1 - r0) >> 2;
    for (int e = threadIdx.x; e < span4 * mcount; e += kThreads) {
      const int col = e / span4, row = r0 + (e % span4) * 4;
      const uint32_t off = (uint32_t)((col * BM + row) * 4);
      float4 sum = ptx::ld_cluster_v4(ptx::map_cluster(local + off, 0));
      for (int k = 1; k < S; k++) {
        const float4 t = ptx::ld_cluster_v4(ptx::map_cluster(local + off, (uint32_t)k));
        sum.x += t.x;
        sum.y += t.y;
        sum.z += t.z;
        sum.w += t.w;
      }
      const float o[4] = {sum.x, sum.y, sum.z, sum.w};
      const size_t m = (size_t)(m0 + col);
#pragma unroll
      for (int z = 0; z < 4; z++) {
        const int n = n0 + row + z;
        if (n < p.N) {
          float val = o[z];
          if (p.residual) val += bf2f(p.residual[m * p.ldr + n]);
          p.out[m * p.ldo + n] = f2bf(val);
        }
      }
    }
  } else {
    const int rows64 = ((64 / S) + 3) & ~3;
    const int g0 = min(64, (int)rank * rows64);
    const int g1 = (int)rank + 1 == S ? 64 : min(64, g0 + rows64);
    const int gspan4 = (g1 - g0) >> 2;
    for (int e = threadIdx.x; e < gspan4 * mcount; e += kThreads) {
      const int col = e / gspan4, row = g0 + (e % gspan4) * 4;
      const uint32_t offg = (uint32_t)((col * BM + row) * 4), offu = offg + 64 * 4;
      float4 g = ptx::ld_cluster_v4(ptx::map_cluster(local + offg, 0));
      float4 u = ptx::ld_cluster_v4(ptx::map_cluster(local + offu, 0));
      for (int k = 1; k < S; k++) {
        const float4 a = ptx::ld_cluster_v4(ptx::map_cluster(local + offg, (uint32_t)k));
        const float4 c = ptx::ld_cluster_v4(ptx::map_cluster(local + offu, (uint32_t)k));
        g.x += a.x;
        g.y += a.y;
        g.z += a.z;
        g.w += a.w;
        u.x += c.x;
        u.y += c.y;
        u.z += c.z;
        u.w += c.w;
      }
      const float gv[4] = {g.x, g.y, g.z, g.w}, uv[4] = {u.x, u.y, u.z, u.w};
      const size_t m = (size_t)(m0 + col);
#pragma unroll
      for (int z = 0; z < 4; z++) {
        const int n = n0 / 2 + row + z;
        if (n < p.N / 2) {
          const float gq = bf2f(f2bf(gv[z])), uq = bf2f(f2bf(uv[z]));
          p.out[m * p.ldo + n] = f2bf(gq / (1.f + __expf(-gq)) * uq);
        }
      }
    }
  }
  ptx::cluster_sync();  // no CTA leaves while another still reads its shared memory
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) ptx::tmem_dealloc(tmem, kTmemCols);
  if (threadIdx.x == 0 && s_fail && p.status) atomicExch(p.status, (int)kTimeout);
}

// x [M, K] bf16 -> x8 [M, K] e4m3 and x_scale [M, K / 128]: per token and 128-wide block, the scale
// maps the block's largest magnitude to the e4m3 maximum (scale = amax * (1/448), values multiplied
// by 1/scale). One warp per (token, block).
__global__ void quant_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, uint8_t* __restrict__ x8,
                             int64_t ld8, float* __restrict__ scale, int64_t lds, int M, int K) {
  pdl_wait();
  pdl_launch();
  const int lane = threadIdx.x & 31;
  const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int kbs = K / 128;
  if (w >= (int64_t)M * kbs) return;
  const int m = (int)(w / kbs), kb = (int)(w % kbs);
  const __nv_bfloat16* src = x + (size_t)m * ldx + kb * 128 + lane * 4;
  float f[4];
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 4; i++) {
    f[i] = bf2f(src[i]);
    amax = fmaxf(amax, fabsf(f[i]));
  }
  amax = warp_max(amax);
  const float s = amax > 0.f ? amax * (1.f / 448.f) : 1.f;
  const float inv = 1.f / s;
  uint32_t packed = 0;
#pragma unroll
  for (int i = 0; i < 4; i++)
    packed |= (uint32_t)__nv_cvt_float_to_fp8(f[i] * inv, __NV_SATFINITE, __NV_E4M3) << (8 * i);
  *reinterpret_cast<uint32_t*>(x8 + (size_t)m * ld8 + kb * 128 + lane * 4) = packed;
  if (lane == 0) scale[(size_t)m * lds + kb] = s;
}

}  // namespace gemm8

cudaError_t launch_quant_fp8(const void* x, int64_t ldx, void* x8, int64_t ld8, float* scale, int64_t lds, int64_t M,
                             int64_t K, cudaStream_t stream) {
  if (M == 0) return cudaSuccess;
  if (K % 128 != 0 || ldx % 4 != 0 || ld8 % 4 != 0) return cudaErrorInvalidValue;
  const int64_t warps = M * (K / 128);
  const int threads = 256;
  const int64_t blocks = (warps * 32 + threads - 1) / threads;
  if (blocks > 0x7fffffff) return cudaErrorInvalidValue;
  return launch_ex(gemm8::quant_kernel, dim3((unsigned)blocks), dim3(threads), 0, stream, 0,
                   static_cast<const __nv_bfloat16*>(x), ldx, static_cast<uint8_t*>(x8), ld8, scale, lds, (int)M,
                   (int)K);
}

cudaError_t launch_gemm_fp8(const Fp8GemmArgs& a, cudaStream_t stream) {
  using namespace gemm8;
  if (a.M == 0 || a.N == 0) return cudaSuccess;
  if (a.K % BK != 0 || a.ldx % 16 != 0 || a.ldw % 16 != 0) return cudaErrorInvalidValue;
  if (reinterpret_cast<uintptr_t>(a.x) % 16 != 0 || reinterpret_cast<uintptr_t>(a.w) % 16 != 0)
    return cudaErrorInvalidValue;
  if (a.silu && (a.N % BM != 0 || a.residual != nullptr)) return cudaErrorInvalidValue;
  Params p{};
  p.out = static_cast<__nv_bfloat16*>(a.out);
  p.residual = static_cast<const __nv_bfloat16*>(a.residual);
  p.x_scale = a.x_scale;
  p.w_scale = a.w_scale;
  p.status = a.status;
  p.M = (int)a.M;
  p.N = (int)a.N;
  p.ldo = (int)a.ldo;
  p.ldr = (int)a.ldr;
  p.xs_ld = (int)a.xs_ld;
  p.ws_ld = (int)a.ws_ld;
  p.kb = (int)(a.K / BK);
  p.silu = a.silu;
  int splits = 1, cps = 1;
  gemm_plan(std::min<int64_t>(a.M, 64), a.N, a.K / 2, a.num_sms, &splits, &cps);  // K/2: the bf16 plan's k-blocks
  p.splits = std::max(1, std::min(splits, p.kb));
  const unsigned tiles_n = (unsigned)((a.N + BM - 1) / BM);
  const unsigned tiles_m = (unsigned)((a.M + BN - 1) / BN);
  if (tiles_m > 65535) return cudaErrorInvalidValue;
  CUtensorMap mw, mx;
  cudaError_t e = tmap::u8_2d(&mw, const_cast<void*>(a.w), a.N, a.K, a.ldw, BM, BK);
  if (e != cudaSuccess) return e;
  e = tmap::u8_2d(&mx, const_cast<void*>(a.x), a.M, a.K, a.ldx, BN, BK);
  if (e != cudaSuccess) return e;
  static std::atomic<uint64_t> configured{0};
  e = once_per_device(configured, [] {
    cudaError_t r = cudaFuncSetAttribute(fp8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (r != cudaSuccess) return r;
    return cudaFuncSetAttribute(fp8_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  });
  if (e != cudaSuccess) return e;
  return launch_ex(fp8_kernel, dim3(tiles_n, tiles_m, (unsigned)p.splits), dim3(kThreads), kSmem, stream, p.splits,
                   mw, mx, p);
}

}  // namespace es
