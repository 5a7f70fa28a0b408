// Token-wise kernels of the decoder: RMSNorm (plain and fused with the residual add), RoPE fused
// with the paged-KV write, SiLU-mul, embedding gather and greedy argmax.
//
// All of them are memory-bound; each reads its inputs once with 16-byte vector loads and writes
// its outputs once. Results do not depend on how many tokens are in the batch (one CTA per
// token, fixed reduction trees), so a replayed step computes bit-identical rows.
#include <algorithm>
#include <cstdlib>

#include "api.h"
#include "common.cuh"
#include "launch.h"

namespace es {
namespace {

// ---------------------------------------------------------------------------------------------
// RMSNorm: y = x * rsqrt(mean(x^2) + eps) * w, fp32 inside, one bf16 rounding on the way out.
// With `residual`, first r = bf16(x + r) is stored back into `residual` and normalised.
// One CTA per token; each thread keeps VPT vectors of 8 elements in registers.
template <int VPT, bool kResidual>
__global__ void rmsnorm_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ residual,
                               const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ y,
                               int hidden, int x_stride, int y_stride, float eps, int early) {
  const int nvec = hidden >> 3;
  // the weight is no kernel's output: its loads can be in flight before the wait for the kernel
  // before (ES_NORM_EARLY=0: after it)
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  uint4 wv[VPT];
  if (early) {
#pragma unroll
    for (int j = 0; j < VPT; j++) {
      const int i = threadIdx.x + j * blockDim.x;
      if (i < nvec) wv[j] = wr[i];
    }
  }
  pdl_wait();
  pdl_launch();
  if (!early) {
#pragma unroll
    for (int j = 0; j < VPT; j++) {
      const int i = threadIdx.x + j * blockDim.x;
      if (i < nvec) wv[j] = wr[i];
    }
  }
  __shared__ float red[32];
  const int t = blockIdx.x;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)t * x_stride);
  uint4* rr = kResidual ? reinterpret_cast<uint4*>(residual + (size_t)t * hidden) : nullptr;
  float v[VPT][8];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < VPT; j++) {
    const int i = threadIdx.x + j * blockDim.x;
    if (i < nvec) {
      uint4 a = xr[i];
      unpack8(a, v[j]);
      if (kResidual) {
        float r[8];
        unpack8(rr[i], r);
#pragma unroll
        for (int e = 0; e < 8; e++) v[j][e] += r[e];
        uint4 s = pack8(v[j]);
        rr[i] = s;
        unpack8(s, v[j]);  // normalise the stored (rounded) residual
      }
#pragma unroll
      for (int e = 0; e < 8; e++) ss += v[j][e] * v[j][e];
    }
  }
  ss = block_sum(ss, red);
  const float inv = rsqrtf(ss / (float)hidden + eps);
  uint4* yr = reinterpret_cast<uint4*>(y + (size_t)t * y_stride);
#pragma unroll
  for (int j = 0; j < VPT; j++) {
    const int i = threadIdx.x + j * blockDim.x;
    if (i < nvec) {
      float wf[8], o[8];
      unpack8(wv[j], wf);
#pragma unroll
      for (int e = 0; e < 8; e++) o[e] = v[j][e] * inv * wf[e];
      yr[i] = pack8(o);
    }
  }
}

// ---------------------------------------------------------------------------------------------
// RoPE (rotate-half convention) on q and k, then the paged-KV write of k and v.
// qkv: [T, (Hq + 2 Hkv) * D]; cos_sin: [max_pos, D] fp32 (cos in [0, D/2), sin in [D/2, D));
// cache: one layer, laid out by the five element strides (block, offset, head, kv, elem).
__global__ void rope_kv_kernel(const __nv_bfloat16* __restrict__ qkv, const __nv_bfloat16* __restrict__ bias,
                               const int64_t* __restrict__ positions, const float* __restrict__ cos_sin,
                               const int64_t* __restrict__ slots, __nv_bfloat16* __restrict__ q_out,
                               __nv_bfloat16* __restrict__ cache, int hq, int hkv, int d, int block_size,
                               int64_t s_block, int64_t s_off, int64_t s_head, int64_t s_kv) {
  pdl_wait();
  pdl_launch();
  const int t = blockIdx.x;
  const int half = d >> 1;
  const int row = (hq + 2 * hkv) * d;
  const __nv_bfloat16* src = qkv + (size_t)t * row;
  const int64_t pos = positions[t];
  const float* cs = cos_sin + pos * d;
  const int64_t slot = slots[t];
  const int64_t blk = slot >= 0 ? slot / block_size : 0;
  const int64_t off = slot >= 0 ? slot % block_size : 0;
  __nv_bfloat16* cbase = cache + blk * s_block + off * s_off;
  // rotated pairs of q and k
  const int pairs = (hq + hkv) * half;
  for (int p = threadIdx.x; p < pairs; p += blockDim.x) {
    const int h = p / half, i = p % half;
    const int base = h * d;
    float a = bf2f(src[base + i]), b = bf2f(src[base + i + half]);
    if (bias) {
      a += bf2f(bias[base + i]);
      b += bf2f(bias[base + i + half]);
    }
    const float c = cs[i], s = cs[half + i];
    const float ra = a * c - b * s, rb = b * c + a * s;
    if (h < hq) {
      __nv_bfloat16* q = q_out + (size_t)t * hq * d + base;
      q[i] = f2bf(ra);
      q[i + half] = f2bf(rb);
    } else if (slot >= 0) {
      __nv_bfloat16* k = cbase + (h - hq) * s_head;
      k[i] = f2bf(ra);
      k[i + half] = f2bf(rb);
    }
  }
  if (slot < 0) return;
  const int vn = hkv * d;
  for (int e = threadIdx.x; e < vn; e += blockDim.x) {
    const int h = e / d, i = e % d;
    const int col = (hq + hkv) * d + e;
    float v = bf2f(src[col]);
    if (bias) v += bf2f(bias[col]);
    cbase[s_kv + h * s_head + i] = f2bf(v);
  }
}

// ---------------------------------------------------------------------------------------------
// out[t, i] = silu(g[t, i]) * u[t, i], g and u the two halves of gate_up's row, or (interleaved)
// alternating runs of 64: g[i] at (i / 64) * 128 + i % 64 and u 64 further.
__global__ void silu_mul_kernel(const __nv_bfloat16* __restrict__ gu, __nv_bfloat16* __restrict__ out, int inter,
                                int64_t rows, int interleaved) {
  pdl_wait();
  pdl_launch();
  const int nvec = inter >> 3;
  const int64_t total = rows * nvec;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = idx / nvec;
    const int i = (int)(idx % nvec);
    const uint4* row = reinterpret_cast<const uint4*>(gu + t * 2 * inter);
    float g[8], u[8], o[8];
    const int gi = interleaved ? (i >> 3) * 16 + (i & 7) : i;  // 8 vectors = 64 elements per run
    unpack8(row[gi], g);
    unpack8(row[interleaved ? gi + 8 : nvec + i], u);
#pragma unroll
    for (int e = 0; e < 8; e++) o[e] = g[e] / (1.f + __expf(-g[e])) * u[e];
    reinterpret_cast<uint4*>(out + t * inter)[i] = pack8(o);
  }
}

// ---------------------------------------------------------------------------------------------
// Multi-step decode: turn a step's sampled ids into the next step's inputs on the device.
// st: [4, B] int64 rows (ids, positions, slots, context lengths); rows with context 0 are padding.
__global__ void decode_advance_kernel(int64_t* __restrict__ st, const int64_t* __restrict__ sampled,
                                      const int* __restrict__ bt, int bt_stride, int b, int B, int bs) {
  pdl_wait();
  pdl_launch();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= b) return;
  if (st[3 * B + i] <= 0) return;
  const int64_t pos = st[B + i] + 1;
  st[i] = sampled[i];
  st[B + i] = pos;
  st[3 * B + i] = pos + 1;
  st[2 * B + i] = (int64_t)bt[(size_t)i * bt_stride + pos / bs] * bs + pos % bs;
}

// ---------------------------------------------------------------------------------------------
__global__ void embed_kernel(const int64_t* __restrict__ ids, const __nv_bfloat16* __restrict__ table,
                             __nv_bfloat16* __restrict__ out, int hidden, int64_t vocab) {
  pdl_wait();
  pdl_launch();
  const int t = blockIdx.x;
  int64_t id = ids[t];
  if (id < 0 || id >= vocab) id = 0;
  const uint4* src = reinterpret_cast<const uint4*>(table + id * hidden);
  uint4* dst = reinterpret_cast<uint4*>(out + (size_t)t * hidden);
  for (int i = threadIdx.x; i < (hidden >> 3); i += blockDim.x) dst[i] = src[i];
}

// ---------------------------------------------------------------------------------------------
// Greedy argmax over a bf16 row; ties go to the lowest index (torch.argmax's rule).
__global__ void argmax_kernel(const __nv_bfloat16* __restrict__ logits, int64_t* __restrict__ out, int vocab,
                              int64_t stride) {
  pdl_wait();
  pdl_launch();
  const __nv_bfloat16* row = logits + blockIdx.x * stride;
  float best = -INFINITY;
  int idx = 0x7fffffff;
  const bool vec = ((vocab & 7) == 0) && ((stride & 7) == 0);
  if (vec) {
    const uint4* r = reinterpret_cast<const uint4*>(row);
    for (int i = threadIdx.x; i < (vocab >> 3); i += blockDim.x) {
      float f[8];
      unpack8(r[i], f);
#pragma unroll
      for (int e = 0; e < 8; e++) {
        if (f[e] > best) {
          best = f[e];
          idx = i * 8 + e;
        }
      }
    }
  } else {
    for (int i = threadIdx.x; i < vocab; i += blockDim.x) {
      const float f = bf2f(row[i]);
      if (f > best) {
        best = f;
        idx = i;
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ob > best || (ob == best && oi < idx)) {
      best = ob;
      idx = oi;
    }
  }
  __shared__ float sb[32];
  __shared__ int si[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) {
    sb[warp] = best;
    si[warp] = idx;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    best = lane < nw ? sb[lane] : -INFINITY;
    idx = lane < nw ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
      if (ob > best || (ob == best && oi < idx)) {
        best = ob;
        idx = oi;
      }
    }
    if (lane == 0) out[blockIdx.x] = idx == 0x7fffffff ? 0 : idx;
  }
}

// ---------------------------------------------------------------------------------------------
// Mixture routing: softmax over E expert logits, the top k (ties to the lowest index), their
// probabilities renormalised, and for this rank's experts [e0, e0 + el) the weight of each token
// (0 where the expert is not among the token's top k). One warp per token, E <= 64.
__global__ void moe_route_kernel(const __nv_bfloat16* __restrict__ logits, int64_t stride, int T, int E, int k,
                                 int e0, int el, float* __restrict__ scale, int32_t* __restrict__ ids,
                                 float* __restrict__ weights) {
  pdl_wait();
  pdl_launch();
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  const __nv_bfloat16* row = logits + (size_t)t * stride;
  float x0 = lane < E ? bf2f(row[lane]) : -INFINITY;
  float x1 = lane + 32 < E ? bf2f(row[lane + 32]) : -INFINITY;
  float m = fmaxf(x0, x1);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float p0 = lane < E ? expf(x0 - m) : 0.f, p1 = lane + 32 < E ? expf(x1 - m) : 0.f;
  float sum = p0 + p1;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  p0 /= sum;
  p1 /= sum;
  // top k by repeated arg-max (ties to the lowest index)
  bool s0 = false, s1 = false;
  float chosen = 0.f;
  for (int r = 0; r < k; r++) {
    float bv = -1.f;
    int bi = 0x7fffffff;
    if (!s0 && lane < E) bv = p0, bi = lane;
    if (!s1 && lane + 32 < E && (p1 > bv)) bv = p1, bi = lane + 32;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) bv = ov, bi = oi;
    }
    if (bi == lane) s0 = true;
    if (bi == lane + 32) s1 = true;
    chosen += bv;
    if (lane == 0 && ids) {
      ids[(size_t)t * k + r] = bi;
      weights[(size_t)t * k + r] = bv;
    }
  }
  if (lane == 0 && ids)
    for (int r = 0; r < k; r++) weights[(size_t)t * k + r] /= chosen;
  for (int e = 0; e < el; e++) {  // the same trip count on every lane: the shuffles take the warp
    const int g = e0 + e;
    const float v0 = __shfl_sync(0xffffffffu, s0 ? p0 : 0.f, g & 31);
    const float v1 = __shfl_sync(0xffffffffu, s1 ? p1 : 0.f, g & 31);
    if (lane == 0) scale[(size_t)e * T + t] = (g < 32 ? v0 : v1) / chosen;
  }
}

}  // namespace

cudaError_t launch_moe_route(const void* logits, int64_t stride, int T, int E, int k, int e0, int el, float* scale,
                             int32_t* ids, float* weights, cudaStream_t stream) {
  if (T == 0) return cudaSuccess;
  if (E > 64 || k < 1 || k > E || el > 32 || e0 < 0 || e0 + el > E) return cudaErrorInvalidValue;
  if ((el > 0 && !scale) || (!ids != !weights)) return cudaErrorInvalidValue;
  constexpr int kWarps = 4;
  return launch_ex(moe_route_kernel, dim3((unsigned)((T + kWarps - 1) / kWarps)), dim3(32 * kWarps), 0, stream, 0,
                   static_cast<const __nv_bfloat16*>(logits), stride, T, E, k, e0, el, scale, ids, weights);
}

cudaError_t launch_decode_advance(int64_t* st, const int64_t* sampled, const int* bt, int64_t bt_stride, int b, int B,
                                  int bs, cudaStream_t stream) {
  if (b == 0) return cudaSuccess;
  return launch_ex(decode_advance_kernel, dim3((b + 127) / 128), dim3(128), 0, stream, 0, st, sampled, bt,
                   (int)bt_stride, b, B, bs);
}

cudaError_t launch_rmsnorm(const void* x, void* residual, const void* w, void* y, int64_t rows, int hidden,
                           int64_t x_stride, int64_t y_stride, float eps, cudaStream_t stream) {
  if (hidden % 8 != 0) return cudaErrorInvalidValue;
  if (rows == 0) return cudaSuccess;
  const int nvec = hidden / 8;
  const int threads = std::min(1024, ((nvec + 31) / 32) * 32);
  const int vpt = (nvec + threads - 1) / threads;
  if (vpt > 4) return cudaErrorInvalidValue;
  auto xp = static_cast<const __nv_bfloat16*>(x);
  auto rp = static_cast<__nv_bfloat16*>(residual);
  auto wp = static_cast<const __nv_bfloat16*>(w);
  auto yp = static_cast<__nv_bfloat16*>(y);
  const int xs = (int)x_stride, ys = (int)y_stride;
  static const int early = [] {
    const char* v = std::getenv("ES_NORM_EARLY");
    return v && v[0] == '0' ? 0 : 1;
  }();
#define ES_LAUNCH_RMS(V)                                                                                      \
  return rp ? launch_ex(rmsnorm_kernel<V, true>, dim3((unsigned)rows), dim3(threads), 0, stream, 0, xp, rp, wp, yp, \
                        hidden, xs, ys, eps, early)                                                               \
            : launch_ex(rmsnorm_kernel<V, false>, dim3((unsigned)rows), dim3(threads), 0, stream, 0, xp, rp, wp, yp, \
                        hidden, xs, ys, eps, early);
  if (vpt == 1) {
    ES_LAUNCH_RMS(1)
  } else if (vpt == 2) {
    ES_LAUNCH_RMS(2)
  } else {
    ES_LAUNCH_RMS(4)
  }
#undef ES_LAUNCH_RMS
}

cudaError_t launch_rope_kv(const void* qkv, const void* bias, const int64_t* positions, const float* cos_sin,
                           const int64_t* slots, void* q_out, void* cache, int64_t T, int hq, int hkv, int d,
                           int block_size, const int64_t* st, cudaStream_t stream) {
  if (T == 0) return cudaSuccess;
  if (d % 2 != 0 || st[4] != 1) return cudaErrorInvalidValue;
  return launch_ex(rope_kv_kernel, dim3((unsigned)T), dim3(256), 0, stream, 0, static_cast<const __nv_bfloat16*>(qkv),
                   static_cast<const __nv_bfloat16*>(bias), positions, cos_sin, slots,
                   static_cast<__nv_bfloat16*>(q_out), static_cast<__nv_bfloat16*>(cache), hq, hkv, d, block_size,
                   st[0], st[1], st[2], st[3]);
}

cudaError_t launch_silu_mul(const void* gu, void* out, int64_t rows, int inter, bool interleaved,
                            cudaStream_t stream) {
  if (inter % 8 != 0 || (interleaved && inter % 64 != 0)) return cudaErrorInvalidValue;
  if (rows == 0) return cudaSuccess;
  const int64_t total = rows * (inter / 8);
  const int threads = 256;
  const int64_t blocks = std::min<int64_t>((total + threads - 1) / threads, 148 * 16);
  return launch_ex(silu_mul_kernel, dim3((unsigned)blocks), dim3(threads), 0, stream, 0,
                   static_cast<const __nv_bfloat16*>(gu), static_cast<__nv_bfloat16*>(out), inter, rows,
                   interleaved ? 1 : 0);
}

cudaError_t launch_embed(const int64_t* ids, const void* table, void* out, int64_t T, int hidden, int64_t vocab,
                         cudaStream_t stream) {
  if (hidden % 8 != 0) return cudaErrorInvalidValue;
  if (T == 0) return cudaSuccess;
  return launch_ex(embed_kernel, dim3((unsigned)T), dim3(128), 0, stream, 0, ids,
                   static_cast<const __nv_bfloat16*>(table), static_cast<__nv_bfloat16*>(out), hidden, vocab);
}

cudaError_t launch_argmax(const void* logits, int64_t* out, int64_t rows, int vocab, int64_t stride,
                          cudaStream_t stream) {
  if (rows == 0) return cudaSuccess;
  return launch_ex(argmax_kernel, dim3((unsigned)rows), dim3(1024), 0, stream, 0,
                   static_cast<const __nv_bfloat16*>(logits), out, vocab, stride);
}

}  // namespace es
