// Paged attention for decode: one query token per sequence against its paged K/V history.
//
// Cache layout (one layer): [num_blocks, 2 (k, v), kv_heads, block_size, head_dim] bf16, so the
// K (or V) rows of one (block, kv head) are one contiguous run of block_size * head_dim * 2 bytes.
// A CTA owns one (sequence, kv head, split of part_tokens positions) and serves the G query heads
// that share the kv head (GQA). One thread issues one-dimensional bulk async copies of whole
// blocks into a 3-stage shared-memory ring (mbarrier completion), so a CTA keeps ~64 KB of K/V in
// flight with a handful of instructions; 128 threads compute q.k, an online softmax and p.v out of
// shared memory. Each split writes (o / l, m, l) and a second kernel merges the splits in split
// order. The split length is fixed, so a sequence's result never depends on the batch around it.
#include "api.h"
#include "common.cuh"
#include "ptx.cuh"

namespace es {
namespace attn {

constexpr int kThreads = 128;
constexpr int kChunk = 64;   // positions per pipeline stage
constexpr int kStages = 3;
constexpr float kLog2e = 1.4426950408889634f;

struct DecodeParams {
  const __nv_bfloat16* q;  // [B, Hq, D] rows of q_stride elements
  int64_t q_stride;
  const __nv_bfloat16* cache;
  int64_t s_block, s_kv;  // element strides of the cache layout
  const int* block_tables;
  int bt_stride;
  const int* ctx_lens;
  float* part_o;   // [B, Hq, max_splits, D]
  float* part_ml;  // [B, Hq, max_splits, 2]
  int hq, hkv, max_splits, part_tokens;
  float scale_log2;  // softmax scale * log2(e)
  int* status;
};

template <int G, int D, int BS>
struct DecodeCfg {
  static constexpr int DPT = (D == 128 && G <= 4) ? 16 : 8;  // dims per thread in q.k
  static constexpr int TPT = D / DPT;                         // threads per position in q.k
  static constexpr int TOK = kThreads / TPT;                  // positions per q.k pass
  static constexpr int VPT = DPT / 8;                         // uint4 per thread per position
  static constexpr int DT = D / 8;                            // threads per row in p.v
  static constexpr int TL = kThreads / DT;                    // position lanes in p.v
  static constexpr int CB = kChunk / BS;                      // blocks per stage
  static constexpr int kTileElems = kChunk * D;
  static constexpr size_t kSmem = 2ull * kStages * kTileElems * 2       // K and V rings
                                  + (size_t)G * D * 4                    // q (fp32, prescaled)
                                  + (size_t)G * kChunk * 4               // logits / probabilities
                                  + 3ull * 8 * 4                         // running m, l, rescale
                                  + kStages * 8 + 16;                    // mbarriers
  static_assert((size_t)TL * G * D * 4 <= 2ull * kStages * kTileElems * 2, "reduction buffer fits the rings");
  static_assert(kChunk % BS == 0 && kChunk % TOK == 0, "chunk shape");
};

template <int G, int D, int BS>
__global__ void __launch_bounds__(kThreads) decode_kernel(DecodeParams p) {
  using C = DecodeCfg<G, D, BS>;
  extern __shared__ __align__(128) uint8_t smem[];
  __nv_bfloat16* kbuf = reinterpret_cast<__nv_bfloat16*>(smem);
  __nv_bfloat16* vbuf = kbuf + kStages * C::kTileElems;
  float* qs = reinterpret_cast<float*>(vbuf + kStages * C::kTileElems);
  float* lg = qs + G * D;
  float* mrun = lg + G * kChunk;
  float* lrun = mrun + 8;
  float* scl = lrun + 8;
  uint64_t* full = reinterpret_cast<uint64_t*>(scl + 8);
  float* red = reinterpret_cast<float*>(smem);  // aliases the rings once they are drained

  const int b = blockIdx.x, kvh = blockIdx.y, split = blockIdx.z;
  const int ctx = p.ctx_lens[b];
  const int s0 = split * p.part_tokens;
  if (s0 >= ctx) return;
  const int s1 = min(ctx, s0 + p.part_tokens);
  const int nchunks = (s1 - s0 + kChunk - 1) / kChunk;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int* bt = p.block_tables + (size_t)b * p.bt_stride;
  const size_t head_off = (size_t)kvh * BS * D;

  if (tid == 0) {
    for (int s = 0; s < kStages; s++) ptx::mbar_init(&full[s], 1);
    ptx::fence_mbar_init();
  }
  // q of the G heads, fp32, prescaled so the softmax runs in base 2
  for (int i = tid; i < G * D; i += kThreads) {
    const int g = i / D, e = i % D;
    qs[i] = bf2f(p.q[(size_t)b * p.q_stride + (size_t)(kvh * G + g) * D + e]) * p.scale_log2;
  }
  if (tid < G) {
    mrun[tid] = -INFINITY;
    lrun[tid] = 0.f;
  }
  __syncthreads();

  auto issue = [&](int c) {
    const int t0 = s0 + c * kChunk;
    const int t1 = min(s1, t0 + kChunk);
    const int blk0 = t0 / BS;
    const int nblk = (t1 + BS - 1) / BS - blk0;
    const int st = c % kStages;
    constexpr uint32_t kBlockBytes = BS * D * 2;
    ptx::mbar_arrive_expect_tx(&full[st], 2u * kBlockBytes * nblk);
    for (int i = 0; i < nblk; i++) {
      const int64_t phys = bt[blk0 + i];
      const __nv_bfloat16* src = p.cache + phys * p.s_block + head_off;
      ptx::bulk_g2s(kbuf + st * C::kTileElems + i * BS * D, src, kBlockBytes, &full[st]);
      ptx::bulk_g2s(vbuf + st * C::kTileElems + i * BS * D, src + p.s_kv, kBlockBytes, &full[st]);
    }
  };

  if (tid == 0) {
    for (int c = 0; c < kStages - 1 && c < nchunks; c++) issue(c);
  }

  // q.k mapping: position group grp, sub-lane sub; the thread's v-th uint4 is row index sub + v*TPT
  const int grp = tid / C::TPT, sub = tid % C::TPT;
  float qr[G][C::DPT];
#pragma unroll
  for (int g = 0; g < G; g++)
#pragma unroll
    for (int v = 0; v < C::VPT; v++)
#pragma unroll
      for (int e = 0; e < 8; e++) qr[g][v * 8 + e] = qs[g * D + (sub + v * C::TPT) * 8 + e];

  // p.v mapping: position lane tl, 8-dim column dc
  const int tl = tid / C::DT, dc = tid % C::DT;
  float acc[G][8];
#pragma unroll
  for (int g = 0; g < G; g++)
#pragma unroll
    for (int e = 0; e < 8; e++) acc[g][e] = 0.f;

  bool failed = false;
  for (int c = 0; c < nchunks; c++) {
    if (tid == 0 && c + kStages - 1 < nchunks) issue(c + kStages - 1);
    const int st = c % kStages;
    const bool ok = ptx::mbar_wait(&full[st], (c / kStages) & 1);
    if (__syncthreads_or(!ok)) {  // every thread leaves together, so no barrier is left half-met
      failed = true;
      break;
    }
    const int t0 = s0 + c * kChunk;
    const int nvalid = min(kChunk, s1 - t0);
    const __nv_bfloat16* kt = kbuf + st * C::kTileElems;
    const __nv_bfloat16* vt = vbuf + st * C::kTileElems;
    // q.k
#pragma unroll
    for (int pass = 0; pass < kChunk / C::TOK; pass++) {
      const int j = pass * C::TOK + grp;
      float s[G];
#pragma unroll
      for (int g = 0; g < G; g++) s[g] = 0.f;
      if (j < nvalid) {
        const uint4* row = reinterpret_cast<const uint4*>(kt + j * D);
#pragma unroll
        for (int v = 0; v < C::VPT; v++) {
          float kf[8];
          unpack8(row[sub + v * C::TPT], kf);
#pragma unroll
          for (int g = 0; g < G; g++)
#pragma unroll
            for (int e = 0; e < 8; e++) s[g] += qr[g][v * 8 + e] * kf[e];
        }
      }
#pragma unroll
      for (int g = 0; g < G; g++) {
#pragma unroll
        for (int o = C::TPT / 2; o > 0; o >>= 1) s[g] += __shfl_xor_sync(0xffffffffu, s[g], o);
      }
      if (sub == 0) {
#pragma unroll
        for (int g = 0; g < G; g++) lg[g * kChunk + j] = j < nvalid ? s[g] : -INFINITY;
      }
    }
    __syncthreads();
    // online softmax, one warp per head
    for (int g = warp; g < G; g += kThreads / 32) {
      const float a = lg[g * kChunk + lane], bb = lg[g * kChunk + lane + 32];
      const float mx = warp_max(fmaxf(a, bb));
      const float mold = mrun[g];
      const float mnew = fmaxf(mold, mx);
      const float pa = exp2f(a - mnew), pb = exp2f(bb - mnew);
      lg[g * kChunk + lane] = pa;
      lg[g * kChunk + lane + 32] = pb;
      const float sum = warp_sum(pa + pb);
      if (lane == 0) {
        const float f = exp2f(mold - mnew);
        scl[g] = f;
        lrun[g] = lrun[g] * f + sum;
        mrun[g] = mnew;
      }
    }
    __syncthreads();
    // p.v
#pragma unroll
    for (int g = 0; g < G; g++) {
      const float f = scl[g];
#pragma unroll
      for (int e = 0; e < 8; e++) acc[g][e] *= f;
    }
    for (int j = tl; j < nvalid; j += C::TL) {
      float vf[8];
      unpack8(reinterpret_cast<const uint4*>(vt + j * D)[dc], vf);
#pragma unroll
      for (int g = 0; g < G; g++) {
        const float pj = lg[g * kChunk + j];
#pragma unroll
        for (int e = 0; e < 8; e++) acc[g][e] += pj * vf[e];
      }
    }
    __syncthreads();
  }
  if (failed) {
    if (tid == 0 && p.status) atomicExch(p.status, (int)kTimeout);
    return;
  }
  // merge the position lanes in lane order
#pragma unroll
  for (int g = 0; g < G; g++)
#pragma unroll
    for (int e = 0; e < 8; e++) red[(tl * G + g) * D + dc * 8 + e] = acc[g][e];
  __syncthreads();
  for (int i = tid; i < G * D; i += kThreads) {
    const int g = i / D, e = i % D;
    float o = 0.f;
    for (int l = 0; l < C::TL; l++) o += red[(l * G + g) * D + e];
    const size_t row = ((size_t)b * p.hq + kvh * G + g) * p.max_splits + split;
    p.part_o[row * D + e] = o / lrun[g];
    if (e == 0) {
      p.part_ml[row * 2] = mrun[g];
      p.part_ml[row * 2 + 1] = lrun[g];
    }
  }
}

// Merge the splits of every (sequence, head) in split order; out rows of out_stride elements.
__global__ void decode_merge_kernel(const float* __restrict__ part_o, const float* __restrict__ part_ml,
                                    const int* __restrict__ ctx_lens, __nv_bfloat16* __restrict__ out,
                                    int64_t out_stride, int hq, int max_splits, int part_tokens, int d) {
  const int b = blockIdx.x, h = blockIdx.y;
  const int ctx = ctx_lens[b];
  const int ns = min(max_splits, (ctx + part_tokens - 1) / part_tokens);
  const size_t row0 = ((size_t)b * hq + h) * max_splits;
  float m = -INFINITY;
  for (int s = 0; s < ns; s++) m = fmaxf(m, part_ml[(row0 + s) * 2]);
  for (int e = threadIdx.x; e < d; e += blockDim.x) {
    float num = 0.f, den = 0.f;
    for (int s = 0; s < ns; s++) {
      const float w = part_ml[(row0 + s) * 2 + 1] * exp2f(part_ml[(row0 + s) * 2] - m);
      num += w * part_o[(row0 + s) * d + e];
      den += w;
    }
    out[(size_t)b * out_stride + (size_t)h * d + e] = f2bf(ns > 0 ? num / den : 0.f);
  }
}

template <int G, int D, int BS>
cudaError_t launch_decode(const DecodeParams& p, int B, cudaStream_t stream) {
  using C = DecodeCfg<G, D, BS>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e =
        cudaFuncSetAttribute(decode_kernel<G, D, BS>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::kSmem);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  dim3 grid(B, p.hkv, p.max_splits);
  decode_kernel<G, D, BS><<<grid, kThreads, C::kSmem, stream>>>(p);
  return cudaGetLastError();
}

template <int D, int BS>
cudaError_t dispatch_g(int G, const DecodeParams& p, int B, cudaStream_t s) {
  switch (G) {
    case 1: return launch_decode<1, D, BS>(p, B, s);
    case 2: return launch_decode<2, D, BS>(p, B, s);
    case 3: return launch_decode<3, D, BS>(p, B, s);
    case 4: return launch_decode<4, D, BS>(p, B, s);
    case 5: return launch_decode<5, D, BS>(p, B, s);
    case 6: return launch_decode<6, D, BS>(p, B, s);
    case 7: return launch_decode<7, D, BS>(p, B, s);
    case 8: return launch_decode<8, D, BS>(p, B, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace attn

cudaError_t launch_paged_decode(const DecodeArgs& a, cudaStream_t stream) {
  if (a.B == 0) return cudaSuccess;
  if (a.hkv <= 0 || a.hq % a.hkv != 0 || a.part_tokens % attn::kChunk != 0 || a.max_splits <= 0)
    return cudaErrorInvalidValue;
  attn::DecodeParams p{};
  p.q = static_cast<const __nv_bfloat16*>(a.q);
  p.q_stride = a.q_stride;
  p.cache = static_cast<const __nv_bfloat16*>(a.cache);
  p.s_block = a.s_block;
  p.s_kv = a.s_kv;
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
  const int G = a.hq / a.hkv;
  cudaError_t e;
  if (a.d == 128 && a.block_size == 16) e = attn::dispatch_g<128, 16>(G, p, a.B, stream);
  else if (a.d == 64 && a.block_size == 16) e = attn::dispatch_g<64, 16>(G, p, a.B, stream);
  else if (a.d == 128 && a.block_size == 32) e = attn::dispatch_g<128, 32>(G, p, a.B, stream);
  else if (a.d == 64 && a.block_size == 32) e = attn::dispatch_g<64, 32>(G, p, a.B, stream);
  else return cudaErrorInvalidValue;
  if (e != cudaSuccess) return e;
  dim3 mgrid(a.B, a.hq);
  attn::decode_merge_kernel<<<mgrid, a.d, 0, stream>>>(a.part_o, a.part_ml, a.ctx_lens,
                                                       static_cast<__nv_bfloat16*>(a.out), a.out_stride, a.hq,
                                                       a.max_splits, a.part_tokens, a.d);
  return cudaGetLastError();
}

}  // namespace es
