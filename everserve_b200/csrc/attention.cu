// Paged attention for decode: one query token per sequence against its paged K/V history.
//
// Cache layout (one layer): [num_blocks, 2 (k, v), kv_heads, block_size, head_dim] bf16, so the
// K (or V) rows of one (block, kv head) are one contiguous tile of block_size * head_dim * 2 bytes.
// A CTA owns one (sequence, kv head, split of at most part_tokens positions) and serves the G <= 8 query
// heads that share the kv head (GQA). Thread 0 streams whole K and V tiles into a 3-stage shared
// ring with TMA (128-byte swizzle, so the tensor-core fragment loads below are bank-conflict free);
// each of the 4 warps takes one block of every stage and computes S = q.K^T and O += P.V with
// mma.sync m16n8k16 (the G query heads padded to 16 rows: decode attention is memory-bound, the
// tensor cores only remove the SIMT arithmetic from the critical path), keeping its own online
// softmax state. The warps merge at the end and each split writes (o / l, m, l); a small kernel
// then merges the splits in split order (or, with ES_ATTN_MERGE=fused, the last split of a
// (sequence, kv head) to finish merges them, one atomic ticket per pair, and there is no second
// launch). The split length is fixed per engine, so a sequence's result never depends on the
// batch around it.
#include <cuda.h>

#include <cstdlib>
#include <cstring>

#include "api.h"
#include "launch.h"
#include "common.cuh"
#include "ptx.cuh"
#include "tmap.h"

namespace es {
namespace attn {

constexpr int kThreads = 128;
constexpr int kWarps = 4;
constexpr float kLog2e = 1.4426950408889634f;

struct DecodeParams {
  const __nv_bfloat16* q;  // [B, Hq, D] rows of q_stride elements
  int64_t q_stride;
  const int* block_tables;
  int bt_stride;
  const int* ctx_lens;
  float* part_o;   // [B, Hq, max_splits, D]
  float* part_ml;  // [B, Hq, max_splits, 2]
  int* tickets;    // [B, Hkv] zero between launches: splits of the pair done so far (nullable)
  const uint8_t* pf;  // memory the next kernel reads, fetched into L2 meanwhile (nullable)
  int64_t pf_bytes;
  int cluster;  // the splits of a (sequence, kv head) form one cluster and merge through DSMEM
  int early;    // issue the K/V chunks that need no output of the kernel before ahead of the wait
  __nv_bfloat16* out;  // [B, Hq * D] rows of out_stride
  int64_t out_stride;
  int hq, hkv, max_splits, part_tokens;
  float scale_log2;  // softmax scale * log2(e)
  int* status;
};

template <int D, int BS, int kStages>
struct DecodeCfg {
  static constexpr int kTileBytes = BS * D * 2;             // one (block, kv head) of K or V
  static constexpr int kStageBytes = kWarps * 2 * kTileBytes;
  static constexpr int kRowsPerTok = D / 64;                 // 128-byte TMA rows per position
  static constexpr int kSmem = kStages * kStageBytes + 1024 + 128;
  static_assert(kWarps * 8 * D * 4 + kWarps * 8 * 2 * 4 + 8 * D * 4 + 8 * 2 * 4 <= kStages * kStageBytes,
                "the warp and cluster merge buffers fit the ring");
};

// byte offset of element (t, d) of a K/V tile written by TMA with 128-byte swizzle
template <int D>
ES_DEVICE uint32_t swz(int t, int d) {
  const int hr = t * (D / 64) + (d >> 6);
  const int chunk = (d & 63) >> 3;
  return (uint32_t)(hr * 128 + ((chunk ^ (hr & 7)) << 4) + (d & 7) * 2);
}

template <int D, int BS, int kStages>
__global__ void __launch_bounds__(kThreads) decode_kernel(const __grid_constant__ CUtensorMap cmap, DecodeParams p) {
  // Before the wait for the kernel before (the qkv projection, which writes q and each sequence's
  // newest K/V row) only what earlier kernels and earlier steps wrote is read: the context lengths,
  // the block tables (read past L1) and, with `early`, the K/V rows of blocks before a sequence's
  // last one, so the first stage of the history can stream while the projection finishes.
  using C = DecodeCfg<D, BS, kStages>;
  constexpr int NT = D / 8;  // n-tiles of the output
  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + kStages * C::kStageBytes);

  // grid (splits, sequences, kv heads): the splits of a pair are neighbours, so the CTAs of splits
  // a short history does not reach leave among the busy ones, not as a wave at the end; a cluster
  // launch keeps (sequences, kv heads, splits) with the splits along z, its cluster dimension
  const int split = p.cluster ? blockIdx.z : blockIdx.x;
  const int b = p.cluster ? blockIdx.x : blockIdx.y;
  const int kvh = p.cluster ? blockIdx.y : blockIdx.z;
  const int ctx = __ldcg(p.ctx_lens + b);
  // a sequence's splits are equal to a block (at most part_tokens each), not part_tokens and a
  // short rest: the CTAs of a step are closer in length; the count is ceil(ctx / part_tokens) as
  // the merges assume, and no split is empty (ns - 1 splits of at most part_tokens are below ctx)
  const int ns_b = max(1, min(p.max_splits, (ctx + p.part_tokens - 1) / p.part_tokens));
  const int plen = ((ctx + ns_b - 1) / ns_b + BS - 1) / BS * BS;
  const int s0 = split * plen;
  const int G = p.hq / p.hkv;
  const bool empty = s0 >= ctx;
  if (empty && !p.cluster) {
    pdl_wait();
    pdl_launch();
    if (split == 0)  // an empty history: the output is zero
      for (int i = threadIdx.x; i < G * D; i += kThreads)
        p.out[(size_t)b * p.out_stride + (size_t)kvh * G * D + i] = f2bf(0.f);
    return;
  }
  // (an empty split of a cluster stays for the cluster's barriers and contributes nothing)
  const int s1 = empty ? s0 : min(ctx, s0 + plen);
  const int blk0 = s0 / BS, blk1 = (s1 + BS - 1) / BS;
  const int nchunks = empty ? 0 : (blk1 - blk0 + kWarps - 1) / kWarps;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gid = lane >> 2, tig = lane & 3;
  const int* bt = p.block_tables + (size_t)b * p.bt_stride;

  if (tid == 0) {
    ptx::prefetch_tmap(&cmap);
    for (int s = 0; s < kStages; s++) ptx::mbar_init(&full[s], 1);
    ptx::fence_mbar_init();
  }
  __syncthreads();

  // the history is read once per step: its lines go first, ahead of what later kernels keep
  const uint64_t pol = ptx::policy_evict_first();
  auto issue = [&](int c) {
    const int st = c % kStages;
    const int first = blk0 + c * kWarps;
    const int n = min(kWarps, blk1 - first);
    ptx::mbar_arrive_expect_tx(&full[st], (uint32_t)(2 * C::kTileBytes * n));
    for (int i = 0; i < n; i++) {
      const int64_t phys = __ldcg(bt + first + i);
      const int row_k = (int)(((phys * 2 + 0) * p.hkv + kvh) * BS * C::kRowsPerTok);
      const int row_v = (int)(((phys * 2 + 1) * p.hkv + kvh) * BS * C::kRowsPerTok);
      uint8_t* dst = ring + st * C::kStageBytes + i * 2 * C::kTileBytes;
      ptx::tma_load_2d_hint(dst, &cmap, 0, row_k, &full[st], pol);
      ptx::tma_load_2d_hint(dst + C::kTileBytes, &cmap, 0, row_v, &full[st], pol);
    }
  };
  // chunks holding none of the sequence's last block go before the wait; the rest after it
  const int last_blk = (ctx - 1) / BS;
  int early = 0;
  if (tid == 0 && p.early)
    for (; early < kStages - 1 && early < nchunks && blk0 + (early + 1) * kWarps - 1 < last_blk; early++) issue(early);
  pdl_wait();
  pdl_launch();
  if (tid == 0) {
    for (int c = early; c < kStages - 1 && c < nchunks; c++) issue(c);
    ptx::l2_prefetch_share(p.pf, p.pf_bytes, (int)(blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z)),
                           (int)(gridDim.x * gridDim.y * gridDim.z));
  }

  // q fragments (rows = the G heads, zero above G; rows 8..15 are always zero)
  uint32_t qa[D / 16][2];
  {
    const __nv_bfloat16* qrow = p.q + (size_t)b * p.q_stride + (size_t)(kvh * G + gid) * D;
#pragma unroll
    for (int ks = 0; ks < D / 16; ks++) {
      if (gid < G) {
        qa[ks][0] = *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + tig * 2);
        qa[ks][1] = *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 8 + tig * 2);
      } else {
        qa[ks][0] = qa[ks][1] = 0u;
      }
    }
  }
  float o[NT][4];
#pragma unroll
  for (int i = 0; i < NT; i++) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_run = -INFINITY, l_run = 0.f;  // row gid; l is this thread's partial sum

  bool failed = false;
  for (int c = 0; c < nchunks; c++) {
    if (tid == 0 && c + kStages - 1 < nchunks) issue(c + kStages - 1);
    const int st = c % kStages;
    const bool ok = ptx::mbar_wait(&full[st], (c / kStages) & 1);
    if (__syncthreads_or(!ok)) {
      failed = true;
      break;
    }
    const int blk = blk0 + c * kWarps + warp;
    if (blk < blk1) {
      const uint32_t kbase = ptx::smem_u32(ring + st * C::kStageBytes + warp * 2 * C::kTileBytes);
      const uint32_t vbase = kbase + C::kTileBytes;
#pragma unroll
      for (int tb = 0; tb < BS / 16; tb++) {
        const int tok0 = blk * BS + tb * 16;  // global position of the step's first row
        // S = q . K^T for 16 positions (two n-tiles of 8)
        // the even and odd k-steps accumulate apart (four independent chains), then add
        float s[2][4], s_odd[2][4];
#pragma unroll
        for (int j = 0; j < 2; j++)
#pragma unroll
          for (int e = 0; e < 4; e++) s[j][e] = s_odd[j][e] = 0.f;
#pragma unroll
        for (int kp = 0; kp < D / 32; kp++) {
#pragma unroll
          for (int j = 0; j < 2; j++) {
            uint32_t b0, b1, b2, b3;
            const int t = tb * 16 + j * 8 + (lane & 7);
            const int d = kp * 32 + (lane >> 3) * 8;
            ptx::ldmatrix_x4(kbase + swz<D>(t, d), b0, b1, b2, b3);
            const uint32_t a0[4] = {qa[2 * kp][0], 0u, qa[2 * kp][1], 0u};
            const uint32_t a1[4] = {qa[2 * kp + 1][0], 0u, qa[2 * kp + 1][1], 0u};
            ptx::mma_bf16_16816(s[j], a0, b0, b1);
            ptx::mma_bf16_16816(s_odd[j], a1, b2, b3);
          }
        }
#pragma unroll
        for (int j = 0; j < 2; j++)
#pragma unroll
          for (int e = 0; e < 4; e++) s[j][e] += s_odd[j][e];
        // online softmax on row gid (this thread: positions tig*2+{0,1} of each n-tile)
        float v[4];
        float mx = -INFINITY;
#pragma unroll
        for (int j = 0; j < 2; j++) {
#pragma unroll
          for (int e = 0; e < 2; e++) {
            const int pos = tok0 + j * 8 + tig * 2 + e;
            const float x = pos < s1 ? s[j][e] * p.scale_log2 : -INFINITY;
            v[j * 2 + e] = x;
            mx = fmaxf(mx, x);
          }
        }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float m_new = fmaxf(m_run, mx);
        const bool none = m_new == -INFINITY;  // no valid position seen yet
        const float alpha = m_run == -INFINITY ? 0.f : exp2f(m_run - m_new);
        float pr[4];
#pragma unroll
        for (int i = 0; i < 4; i++) pr[i] = none ? 0.f : exp2f(v[i] - m_new);
        l_run = l_run * alpha + (pr[0] + pr[1] + pr[2] + pr[3]);
        m_run = m_new;
#pragma unroll
        for (int i = 0; i < NT; i++) {
          o[i][0] *= alpha;
          o[i][1] *= alpha;
        }
        const uint32_t pa[4] = {ptx::pack_bf16x2(pr[0], pr[1]), 0u, ptx::pack_bf16x2(pr[2], pr[3]), 0u};
        // O += P . V
#pragma unroll
        for (int np = 0; np < D / 16; np++) {
          uint32_t b0, b1, b2, b3;
          const int mi = lane >> 3;
          const int t = tb * 16 + (mi & 1) * 8 + (lane & 7);
          const int d = np * 16 + (mi >> 1) * 8;
          ptx::ldmatrix_x4_trans(vbase + swz<D>(t, d), b0, b1, b2, b3);
          ptx::mma_bf16_16816(o[2 * np], pa, b0, b1);
          ptx::mma_bf16_16816(o[2 * np + 1], pa, b2, b3);
        }
      }
    }
    __syncthreads();  // the stage is free for the next issue
  }
  if (failed && tid == 0 && p.status) atomicExch(p.status, (int)kTimeout);
  // merge the warps: row gid's (m, l, o) of each warp, then combine in warp order (a failed split
  // writes nothing but still takes its ticket, so the pair's count stays whole)
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
  float* red_o = reinterpret_cast<float*>(ring);  // [warp][8][D]
  float* red_ml = red_o + kWarps * 8 * D;         // [warp][8][2]
  if (!failed && gid < G) {
#pragma unroll
    for (int i = 0; i < NT; i++) {
      red_o[(warp * 8 + gid) * D + i * 8 + tig * 2] = o[i][0];
      red_o[(warp * 8 + gid) * D + i * 8 + tig * 2 + 1] = o[i][1];
    }
    if (tig == 0) {
      red_ml[(warp * 8 + gid) * 2] = m_run;
      red_ml[(warp * 8 + gid) * 2 + 1] = l_run;
    }
  }
  __syncthreads();
  float* cl_o = red_ml + kWarps * 8 * 2;  // cluster mode: this split's [G][D] output, then [G][2]
  float* cl_ml = cl_o + G * D;
  for (int i = tid; !failed && i < G * D; i += kThreads) {
    const int g = i / D, e = i % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; w++) M = fmaxf(M, red_ml[(w * 8 + g) * 2]);
    float num = 0.f, den = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; w++) {
      const float mw = red_ml[(w * 8 + g) * 2];
      const float f = mw == -INFINITY ? 0.f : exp2f(mw - M);
      num += red_o[(w * 8 + g) * D + e] * f;
      den += red_ml[(w * 8 + g) * 2 + 1] * f;
    }
    if (p.cluster) {
      cl_o[g * D + e] = num / den;
      if (e == 0) {
        cl_ml[g * 2] = M;
        cl_ml[g * 2 + 1] = den;
      }
      continue;
    }
    const size_t row = ((size_t)b * p.hq + kvh * G + g) * p.max_splits + split;
    p.part_o[row * D + e] = num / den;
    if (e == 0) {
      p.part_ml[row * 2] = M;
      p.part_ml[row * 2 + 1] = den;
    }
  }
  if (p.cluster) {
    // the pair's splits are this cluster (rank = split): each CTA merges a share of the G x D
    // outputs over the splits' partials in their shared memory, in split order (the merge
    // kernel's arithmetic), then waits until every CTA has read its partials
    ptx::cluster_sync();
    const int ns = min(p.max_splits, (ctx + p.part_tokens - 1) / p.part_tokens);
    const uint32_t o_local = ptx::smem_u32(cl_o), ml_local = ptx::smem_u32(cl_ml);
    for (int i = split * kThreads + tid; i < G * D; i += (int)gridDim.z * kThreads) {
      const int g = i / D, e = i % D;
      float m = -INFINITY;
      for (int sp = 0; sp < ns; sp++)
        m = fmaxf(m, ptx::ld_cluster_f32(ptx::map_cluster(ml_local + g * 8, (uint32_t)sp)));
      float num = 0.f, den = 0.f;
      for (int sp = 0; sp < ns; sp++) {
        const float ms = ptx::ld_cluster_f32(ptx::map_cluster(ml_local + g * 8, (uint32_t)sp));
        const float ls = ptx::ld_cluster_f32(ptx::map_cluster(ml_local + g * 8 + 4, (uint32_t)sp));
        const float w = ls * exp2f(ms - m);
        num += w * ptx::ld_cluster_f32(ptx::map_cluster(o_local + (g * D + e) * 4, (uint32_t)sp));
        den += w;
      }
      p.out[(size_t)b * p.out_stride + (size_t)(kvh * G + g) * D + e] = f2bf(ns > 0 ? num / den : 0.f);
    }
    ptx::cluster_sync();
    return;
  }
  // without tickets the merge kernel merges the splits; with them the last split of the pair
  // merges every split's (o, m, l) in split order
  if (p.tickets == nullptr) return;
  __shared__ int s_last;
  __syncthreads();  // every thread's partials are written before the one fence and the ticket
  const int ns = min(p.max_splits, (ctx + p.part_tokens - 1) / p.part_tokens);
  if (tid == 0) {
    __threadfence();
    int* tk = p.tickets + (size_t)b * p.hkv + kvh;
    s_last = atomicAdd(tk, 1) == ns - 1;
    if (s_last) *tk = 0;  // every split of this launch has counted: the next launch starts at zero
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int i = tid; i < G * D; i += kThreads) {
    const int g = i / D, e = i % D;
    const size_t row0 = ((size_t)b * p.hq + kvh * G + g) * p.max_splits;
    const float* ml = p.part_ml + row0 * 2;
    const float* po = p.part_o + row0 * D + e;
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
    p.out[(size_t)b * p.out_stride + (size_t)(kvh * G + g) * D + e] = f2bf(num / den);
  }
}

// Merge the splits of every (sequence, head) in split order; out rows of out_stride elements. The
// same arithmetic, in the same order, as the in-kernel merge of the last split. One warp per
// (sequence, head), eight to a CTA (a CTA per pair would be thousands of tiny CTAs); each lane
// merges four consecutive elements of the row with 16-byte loads.
constexpr int kMergeWarps = 8;
__global__ void __launch_bounds__(kMergeWarps * 32)
    decode_merge_kernel(const float* __restrict__ part_o, const float* __restrict__ part_ml,
                        const int* __restrict__ ctx_lens, __nv_bfloat16* __restrict__ out, int64_t out_stride,
                        int B, int hq, int max_splits, int part_tokens, int d) {
  pdl_wait();
  pdl_launch();
  const int pair = blockIdx.x * kMergeWarps + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (pair >= B * hq) return;
  const int b = pair / hq, h = pair % hq;
  const int ctx = ctx_lens[b];
  const int ns = min(max_splits, (ctx + part_tokens - 1) / part_tokens);
  const size_t row0 = ((size_t)b * hq + h) * max_splits;
  float m = -INFINITY;
  for (int s = 0; s < ns; s++) m = fmaxf(m, part_ml[(row0 + s) * 2]);
  for (int e4 = lane; e4 < d / 4; e4 += 32) {
    float num[4] = {0.f, 0.f, 0.f, 0.f}, den = 0.f;
    for (int s = 0; s < ns; s++) {
      const float w = part_ml[(row0 + s) * 2 + 1] * exp2f(part_ml[(row0 + s) * 2] - m);
      const float4 o = *reinterpret_cast<const float4*>(part_o + (row0 + s) * d + e4 * 4);
      num[0] += w * o.x;
      num[1] += w * o.y;
      num[2] += w * o.z;
      num[3] += w * o.w;
      den += w;
    }
    __nv_bfloat16* dst = out + (size_t)b * out_stride + (size_t)h * d + e4 * 4;
#pragma unroll
    for (int j = 0; j < 4; j++) dst[j] = f2bf(ns > 0 ? num[j] / den : 0.f);
  }
}
inline dim3 merge_grid(int B, int hq) { return dim3((unsigned)((B * hq + kMergeWarps - 1) / kMergeWarps)); }

template <int D, int BS, int S>
cudaError_t launch_decode(const CUtensorMap& map, const DecodeParams& p, int B, cudaStream_t stream) {
  using C = DecodeCfg<D, BS, S>;
  static std::atomic<uint64_t> configured{0};
  cudaError_t e = once_per_device(configured, [] {
    return cudaFuncSetAttribute(decode_kernel<D, BS, S>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
  });
  if (e != cudaSuccess) return e;
  const dim3 grid = p.cluster ? dim3(B, p.hkv, p.max_splits) : dim3(p.max_splits, B, p.hkv);
  return launch_ex(decode_kernel<D, BS, S>, grid, dim3(kThreads), C::kSmem, stream, p.cluster ? p.max_splits : 0,
                   map, p);
}

template <int D, int BS>
cudaError_t launch_stages(int stages, const CUtensorMap& map, const DecodeParams& p, int B, cudaStream_t stream) {
  switch (stages) {
    case 2: return launch_decode<D, BS, 2>(map, p, B, stream);
    case 4: return launch_decode<D, BS, 4>(map, p, B, stream);
    default: return launch_decode<D, BS, 3>(map, p, B, stream);
  }
}

// Kernel choices read once per process: ES_ATTN_TC=1 takes the tcgen05 kernel where it applies;
// otherwise the persistent kernel (decode_persist.cu) where it applies, unless ES_ATTN_PERSIST=0;
// otherwise this file's kernel, whose splits the merge kernel merges, or with ES_ATTN_MERGE=fused
// the last split (tickets), or with ES_ATTN_MERGE=cluster the cluster through distributed shared
// memory. Both entry points (the binding and the allocation-free one) follow the same choices.
bool use_tc() {
  static const bool on = [] {
    const char* v = std::getenv("ES_ATTN_TC");
    return v && v[0] == '1';
  }();
  return on;
}
// ES_ATTN_EARLY=1: the K/V copies that need no output of the kernel before go ahead of the wait
// for it (measured level with issuing them after it, so off by default)
bool early_loads() {
  static const bool on = [] {
    const char* v = std::getenv("ES_ATTN_EARLY");
    return v && v[0] == '1';
  }();
  return on;
}
bool fused_merge() {
  static const bool on = [] {
    const char* v = std::getenv("ES_ATTN_MERGE");
    return v && std::strcmp(v, "fused") == 0;
  }();
  return on;
}
// ES_ATTN_MERGE=cluster: the splits of a pair form a thread-block cluster (up to 8) and merge
// through distributed shared memory; no partials in global memory, no second launch
bool cluster_merge(int max_splits) {
  static const bool on = [] {
    const char* v = std::getenv("ES_ATTN_MERGE");
    return v && std::strcmp(v, "cluster") == 0;
  }();
  return on && max_splits >= 1 && max_splits <= 8;
}

}  // namespace attn

cudaError_t launch_paged_decode(const DecodeArgs& a, cudaStream_t stream) {
  if (a.B == 0) return cudaSuccess;
  if (attn::use_tc() && decode_tc_supported(a)) return launch_decode_tc(a, stream);
  if (!attn::fused_merge() && !attn::cluster_merge(a.max_splits) && decode_persist_supported(a))
    return launch_decode_persist(a, stream);
  if (a.hkv <= 0 || a.hq % a.hkv != 0 || a.hq / a.hkv > 8 || a.part_tokens % 64 != 0 || a.max_splits <= 0 ||
      a.B > 65535)
    return cudaErrorInvalidValue;
  if (a.s_kv != (int64_t)a.hkv * a.block_size * a.d || a.s_block != 2 * a.s_kv) return cudaErrorInvalidValue;
  attn::DecodeParams p{};
  p.q = static_cast<const __nv_bfloat16*>(a.q);
  p.q_stride = a.q_stride;
  p.block_tables = a.block_tables;
  p.bt_stride = (int)a.bt_stride;
  p.ctx_lens = a.ctx_lens;
  p.part_o = a.part_o;
  p.part_ml = a.part_ml;
  p.hq = a.hq;
  p.hkv = a.hkv;
  p.max_splits = a.max_splits;
  p.part_tokens = a.part_tokens;
  p.scale_log2 = a.scale * attn::kLog2e;
  p.status = a.status;
  p.tickets = attn::fused_merge() ? a.tickets : nullptr;
  p.cluster = attn::cluster_merge(a.max_splits) ? 1 : 0;
  if (p.cluster) p.tickets = nullptr;
  p.early = attn::early_loads() ? 1 : 0;
  p.pf = static_cast<const uint8_t*>(a.prefetch);
  p.pf_bytes = a.prefetch_bytes;
  p.out = static_cast<__nv_bfloat16*>(a.out);
  p.out_stride = a.out_stride;
  if (attn::fused_merge() && p.tickets == nullptr) return cudaErrorInvalidValue;
  // the layer's cache as rows of 64 elements (128 bytes); one box = one (block, kv head) tile
  const int64_t rows = a.num_blocks * 2 * a.hkv * a.block_size * (a.d / 64);
  const int box_rows = a.block_size * (a.d / 64);
  CUtensorMap map;
  cudaError_t e = tmap::bf16_2d(&map, const_cast<void*>(a.cache), rows, 64, 64, box_rows, 64);
  if (e != cudaSuccess) return e;
  if (a.d == 128 && a.block_size == 16) e = attn::launch_stages<128, 16>(a.stages, map, p, a.B, stream);
  else if (a.d == 64 && a.block_size == 16) e = attn::launch_stages<64, 16>(a.stages, map, p, a.B, stream);
  else if (a.d == 128 && a.block_size == 32) e = attn::launch_stages<128, 32>(a.stages, map, p, a.B, stream);
  else if (a.d == 64 && a.block_size == 32) e = attn::launch_stages<64, 32>(a.stages, map, p, a.B, stream);
  else return cudaErrorInvalidValue;
  if (e != cudaSuccess || p.tickets != nullptr || p.cluster) return e;
  return launch_ex(attn::decode_merge_kernel, attn::merge_grid(a.B, a.hq), dim3(attn::kMergeWarps * 32), 0, stream,
                   0, (const float*)a.part_o, (const float*)a.part_ml, a.ctx_lens, static_cast<__nv_bfloat16*>(a.out),
                   a.out_stride, a.B, a.hq, a.max_splits, a.part_tokens, a.d);
}

}  // namespace es

// ---------------------------------------------------------------------------------------------
// Allocation-free entry point (declared and documented in es_noalloc.h; no counterpart in the
// reference). Its split-KV scratch is this file-scope device array, not caller memory.
#include <mutex>

#include "es_noalloc.h"

namespace {

// + the status word (and padding), then the split tickets of every (sequence, kv head) pair
constexpr size_t kNoAllocFloats = (size_t)ES_NOALLOC_PART_FLOATS + ES_NOALLOC_ML_FLOATS + 64 + ES_NOALLOC_TICKETS;
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocFloats];

constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
float* g_noalloc_ptr[kNoAllocMaxDevices] = {};
thread_local const char* g_noalloc_err = "";

// The array's device address on the current device, looked up once per device.
cudaError_t noalloc_scratch(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kNoAllocMaxDevices) {
    g_noalloc_err = "device index above the supported maximum";
    return cudaErrorInvalidDevice;
  }
  std::lock_guard<std::mutex> g(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) {
      g_noalloc_err = "cudaGetSymbolAddress of the scratch array failed";
      return e;
    }
    g_noalloc_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return cudaSuccess;
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int es_noalloc_setup(void) {
  float* p = nullptr;
  return (int)noalloc_scratch(&p);
}

extern "C" __attribute__((visibility("default"))) const char* es_noalloc_last_error(void) { return g_noalloc_err; }

extern "C" __attribute__((visibility("default"))) int es_noalloc_status(void* stream, int* status) {
  float* base = nullptr;
  cudaError_t e = noalloc_scratch(&base);
  if (e != cudaSuccess) return (int)e;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int* st = reinterpret_cast<int*>(base + ES_NOALLOC_PART_FLOATS + ES_NOALLOC_ML_FLOATS);
  e = cudaMemcpyAsync(status, st, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (e != cudaSuccess) return (int)e;
  return (int)cudaStreamSynchronize(s);
}

extern "C" __attribute__((visibility("default"))) int es_paged_decode_noalloc(
    const void* q, int64_t q_stride, const void* cache, int64_t num_blocks, int kv_heads, int block_size,
    int head_dim, const int* block_tables, int64_t bt_stride, const int* ctx_lens, void* out, int64_t out_stride,
    int batch, int q_heads, int max_model_len, float scale, void* stream) {
  using namespace es;
  g_noalloc_err = "";
  if (batch == 0) return (int)cudaSuccess;
  constexpr int kPart = 256;  // positions per split (the regular entry point takes its split length as given)
  if (batch < 0 || kv_heads <= 0 || q_heads % kv_heads != 0 || q_heads / kv_heads > 8 || max_model_len <= 0) {
    g_noalloc_err = "bad shape: q_heads must be 1..8 times kv_heads and max_model_len positive";
    return (int)cudaErrorInvalidValue;
  }
  if (!((head_dim == 128 || head_dim == 64) && (block_size == 16 || block_size == 32))) {
    g_noalloc_err = "head_dim must be 64 or 128 and block_size 16 or 32";
    return (int)cudaErrorInvalidValue;
  }
  const int64_t splits = (max_model_len + kPart - 1) / kPart;
  if ((int64_t)batch * q_heads * splits * head_dim > ES_NOALLOC_PART_FLOATS ||
      (int64_t)batch * q_heads * splits * 2 > ES_NOALLOC_ML_FLOATS) {
    g_noalloc_err = "batch * q_heads * ceil(max_model_len / 256) * head_dim exceeds the fixed scratch (2^21 floats)";
    return (int)cudaErrorInvalidValue;
  }
  if ((int64_t)batch * kv_heads > ES_NOALLOC_TICKETS) {
    g_noalloc_err = "batch * kv_heads exceeds the fixed split tickets (4096)";
    return (int)cudaErrorInvalidValue;
  }
  float* base = nullptr;
  cudaError_t e = noalloc_scratch(&base);
  if (e != cudaSuccess) return (int)e;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int* status = reinterpret_cast<int*>(base + ES_NOALLOC_PART_FLOATS + ES_NOALLOC_ML_FLOATS);
  e = cudaMemsetAsync(status, 0, sizeof(int), s);  // the status word starts each call at zero
  if (e != cudaSuccess) return (int)e;
  attn::DecodeParams p{};
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.q_stride = q_stride;
  p.block_tables = block_tables;
  p.bt_stride = (int)bt_stride;
  p.ctx_lens = ctx_lens;
  p.part_o = base;
  p.part_ml = base + ES_NOALLOC_PART_FLOATS;
  p.hq = q_heads;
  p.hkv = kv_heads;
  p.max_splits = (int)splits;
  p.part_tokens = kPart;
  p.scale_log2 = scale * attn::kLog2e;
  p.status = status;
  // zero when the library loads; each launch leaves them at zero again
  int* tickets = reinterpret_cast<int*>(base + ES_NOALLOC_PART_FLOATS + ES_NOALLOC_ML_FLOATS + 64);
  p.tickets = attn::fused_merge() ? tickets : nullptr;
  p.cluster = attn::cluster_merge((int)splits) ? 1 : 0;
  if (p.cluster) p.tickets = nullptr;
  p.early = attn::early_loads() ? 1 : 0;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.out_stride = out_stride;
  // tensor map encoded on the stack (no cache: nothing is allocated, not even on the host heap)
  tmap::EncodeFn enc = tmap::encoder();
  if (enc == nullptr) {
    g_noalloc_err = "cuTensorMapEncodeTiled is not available";
    return (int)cudaErrorNotSupported;
  }
  const int64_t rows = num_blocks * 2 * kv_heads * block_size * (head_dim / 64);
  CUtensorMap map;
  std::memset(&map, 0, sizeof(map));
  const cuuint64_t dims[2] = {64, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {128};
  const cuuint32_t box[2] = {64, (cuuint32_t)(block_size * (head_dim / 64))};
  const cuuint32_t estr[2] = {1, 1};
  if (reinterpret_cast<uintptr_t>(cache) % 16 != 0 ||
      enc(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(cache), dims, strides, box, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
    g_noalloc_err = "the cache cannot be described by a TMA map (alignment or size)";
    return (int)cudaErrorInvalidValue;
  }
  // the tcgen05 kernel where it applies, as the regular entry point (the same result bit for bit);
  // its maps too are encoded here, on the stack
  DecodeArgs da{};
  da.q = q;
  da.q_stride = q_stride;
  da.cache = cache;
  da.block_tables = block_tables;
  da.bt_stride = bt_stride;
  da.ctx_lens = ctx_lens;
  da.out = out;
  da.out_stride = out_stride;
  da.part_o = p.part_o;
  da.part_ml = p.part_ml;
  da.tickets = tickets;
  da.status = status;
  da.B = batch;
  da.hq = q_heads;
  da.hkv = kv_heads;
  da.d = head_dim;
  da.block_size = block_size;
  da.max_splits = (int)splits;
  da.part_tokens = kPart;
  da.num_blocks = num_blocks;
  da.s_kv = (int64_t)kv_heads * block_size * head_dim;
  da.s_block = 2 * da.s_kv;
  da.scale = scale;
  if (attn::use_tc() && decode_tc_supported(da)) {
    CUtensorMap qm;
    std::memset(&qm, 0, sizeof(qm));
    const cuuint64_t qdims[2] = {(cuuint64_t)head_dim, (cuuint64_t)batch * q_heads};
    const cuuint64_t qstrides[1] = {(cuuint64_t)head_dim * 2};
    const cuuint32_t qbox[2] = {64, (cuuint32_t)(q_heads / kv_heads)};
    const cuuint64_t cdims[2] = {(cuuint64_t)head_dim, (cuuint64_t)(num_blocks * 2 * kv_heads * block_size)};
    const cuuint64_t cstrides[1] = {(cuuint64_t)head_dim * 2};
    const cuuint32_t cbox[2] = {64, (cuuint32_t)block_size};
    CUtensorMap cm;
    std::memset(&cm, 0, sizeof(cm));
    if (reinterpret_cast<uintptr_t>(q) % 16 != 0 ||
        enc(&qm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(q), qdims, qstrides, qbox, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS ||
        enc(&cm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(cache), cdims, cstrides, cbox, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
      g_noalloc_err = "q or the cache cannot be described by a TMA map (alignment or size)";
      return (int)cudaErrorInvalidValue;
    }
    return (int)launch_decode_tc_maps(da, qm, cm, s);
  }
  if (!attn::fused_merge() && !p.cluster && decode_persist_supported(da)) {
    // the persistent kernel, as the regular entry point takes it; its map has 16 positions a box
    CUtensorMap pm;
    std::memset(&pm, 0, sizeof(pm));
    const cuuint32_t pbox[2] = {64, (cuuint32_t)(16 * (head_dim / 64))};
    if (enc(&pm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(cache), dims, strides, pbox, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
      g_noalloc_err = "the cache cannot be described by a TMA map (alignment or size)";
      return (int)cudaErrorInvalidValue;
    }
    return (int)launch_decode_persist_map(da, pm, s);
  }
  if (head_dim == 128 && block_size == 16) e = attn::launch_stages<128, 16>(2, map, p, batch, s);
  else if (head_dim == 64 && block_size == 16) e = attn::launch_stages<64, 16>(2, map, p, batch, s);
  else if (head_dim == 128 && block_size == 32) e = attn::launch_stages<128, 32>(2, map, p, batch, s);
  else e = attn::launch_stages<64, 32>(2, map, p, batch, s);
  if (e == cudaSuccess && p.tickets == nullptr && !p.cluster) {
    attn::decode_merge_kernel<<<attn::merge_grid(batch, q_heads), attn::kMergeWarps * 32, 0, s>>>(
        p.part_o, p.part_ml, ctx_lens, static_cast<__nv_bfloat16*>(out), out_stride, batch, q_heads, (int)splits, kPart,
        head_dim);
    e = cudaGetLastError();
  }
  return (int)e;
}
