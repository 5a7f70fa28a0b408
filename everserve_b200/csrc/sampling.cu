// Seeded temperature / top-k / top-p sampling, one CTA per row, deterministic.
//
// A row's token is the Gumbel-max draw argmax(z + g) over the tokens that top-k and top-p keep,
// where z = logit / temperature and g = -log(-log(u)) with u a counter-based uniform of (seed,
// position, token index): SplitMix64 (Steele, Lea, Flood, OOPSLA 2014) of a Weyl sequence, the
// same draw the host sampler makes, so a replayed step samples the same token on any member.
//
// The kept set is a prefix of the order "z descending, then index ascending" (a stable sort):
// top-k keeps its first k tokens, top-p the tokens whose mass ranked above them is below p. Both
// cut-offs are found without a sort by a three-level radix select on the order-preserving 32-bit
// key of z (11 + 11 + 10 bits), with shared-memory histograms of counts (top-k) and of masses
// (top-p). Masses are fixed point, round(exp(z - max) * 2^32) as integers, so every sum is exact
// and the same in any order: the draw does not depend on how the row's threads were scheduled.
// Warps combine the lanes that hit one bin (match + reduce) before one shared atomic per bin.
// Ties at a cut-off value are resolved by index with one prefix count over the row.
//
// Greedy rows (temperature <= 0) take the plain argmax, lowest index on ties.
//
// Reference parity: the sampler parameters of the vLLM engine the reference serves (temperature,
// top_k, top_p, seed); the counter-based draw is this framework's (exact replay needs it).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "api.h"
#include "common.cuh"
#include "launch.h"

namespace es {
namespace smp {

constexpr int kThreads = 1024;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxBins = 2048;
constexpr uint64_t kGolden = 0x9E3779B97F4A7C15ull;
constexpr uint64_t kM1 = 0xBF58476D1CE4E5B9ull;
constexpr uint64_t kM2 = 0x94D049BB133111EBull;
constexpr uint64_t kPos = 0xD1B54A32D192ED03ull;
constexpr uint32_t kNoBin = 0xFFFFFFFFu;

__device__ __forceinline__ uint64_t mix(uint64_t x) {
  x = (x ^ (x >> 30)) * kM1;
  x = (x ^ (x >> 27)) * kM2;
  return x ^ (x >> 31);
}

// Larger key = larger value; -0 and +0 share the key of +0 (a sort treats them as equal).
__device__ __forceinline__ uint32_t key_of(float z) {
  uint32_t b = __float_as_uint(z);
  if ((b << 1) == 0) b = 0;
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ float value_of(uint32_t key) {
  return __uint_as_float((key & 0x80000000u) ? (key & 0x7FFFFFFFu) : ~key);
}

__device__ __forceinline__ uint64_t mass_of(float z, float zmax) {
  return (uint64_t)__float2ull_rn(expf(z - zmax) * 4294967296.0f);
}

template <typename T>
__device__ __forceinline__ float load(const T* row, int i);
template <>
__device__ __forceinline__ float load<__nv_bfloat16>(const __nv_bfloat16* row, int i) {
  return __bfloat162float(row[i]);
}
template <>
__device__ __forceinline__ float load<float>(const float* row, int i) {
  return row[i];
}

struct Shared {
  uint32_t cnt_k[kMaxBins];
  uint32_t cnt_p[kMaxBins];
  unsigned long long mass[kMaxBins];
  uint32_t w_cnt_k[kWarps], w_cnt_p[kWarps];
  unsigned long long w_mass[kWarps];
  float w_f[kWarps];
  int w_i[kWarps];
  double w_d[kWarps];
  uint32_t sel_k, sel_p;
  uint32_t need_k, ties_k, ties_p;
  unsigned long long above_p, total;
  int tie_index;
};

// Adds a lane's contribution to bin `bin` (kNoBin: none) of the histograms, one atomic per bin and
// warp. Every lane of the warp calls it.
__device__ __forceinline__ void hist_add(Shared& s, uint32_t bin, uint32_t add_k, uint32_t add_p, uint64_t m,
                                         int lane) {
  const unsigned grp = __match_any_sync(0xFFFFFFFFu, bin);
  if (bin == kNoBin) return;
  const uint32_t ck = __reduce_add_sync(grp, add_k);
  const uint32_t cp = __reduce_add_sync(grp, add_p);
  // a mass is at most 2^32: two 24-bit halves keep the 32-lane sums within 32 bits
  const uint32_t lo = __reduce_add_sync(grp, (uint32_t)(m & 0xFFFFFFu));
  const uint32_t hi = __reduce_add_sync(grp, (uint32_t)(m >> 24));
  if (lane == __ffs(grp) - 1) {
    if (ck) atomicAdd(&s.cnt_k[bin], ck);
    if (cp) {
      atomicAdd(&s.cnt_p[bin], cp);
      atomicAdd(&s.mass[bin], ((unsigned long long)hi << 24) + lo);
    }
  }
}

template <typename V>
__device__ __forceinline__ V warp_incl_scan(V v, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const V t = __shfl_up_sync(0xFFFFFFFFu, v, o);
    if (lane >= o) v += t;
  }
  return v;
}

// Walks the `nb` bins from the top (thread t holds the bins at descending positions 2t, 2t+1):
// picks the top-k bin holding the need-th token and the top-p bin holding the last token whose
// mass above stays below P.
__device__ void select_bins(Shared& s, int nb, bool k_on, bool p_on, double P, int lane, int warp) {
  const int t = threadIdx.x;
  // what the level before left (written before its last barrier; rewritten after this one's)
  const uint32_t need = s.need_k;
  const unsigned long long base = s.above_p;
  uint32_t bins[2];
  uint32_t ck[2] = {0, 0}, cp[2] = {0, 0};
  unsigned long long m[2] = {0, 0};
#pragma unroll
  for (int j = 0; j < 2; j++) {
    const int pos = 2 * t + j;
    bins[j] = pos < nb ? (uint32_t)(nb - 1 - pos) : kNoBin;
    if (bins[j] != kNoBin) {
      ck[j] = s.cnt_k[bins[j]];
      cp[j] = s.cnt_p[bins[j]];
      m[j] = s.mass[bins[j]];
    }
  }
  const uint32_t tk = ck[0] + ck[1];
  const unsigned long long tm = m[0] + m[1];
  const uint32_t ik = warp_incl_scan(tk, lane);
  const unsigned long long im = warp_incl_scan(tm, lane);
  if (lane == 31) {
    s.w_cnt_k[warp] = ik;
    s.w_mass[warp] = im;
  }
  __syncthreads();
  if (warp == 0) {
    const uint32_t a = s.w_cnt_k[lane];
    const unsigned long long b = s.w_mass[lane];
    const uint32_t sa = warp_incl_scan(a, lane);
    const unsigned long long sb = warp_incl_scan(b, lane);
    s.w_cnt_k[lane] = sa - a;  // exclusive
    s.w_mass[lane] = sb - b;
    if (lane == 31) s.total = sb;
  }
  __syncthreads();
  uint32_t above_k = s.w_cnt_k[warp] + ik - tk;
  unsigned long long above_m = s.w_mass[warp] + im - tm;
#pragma unroll
  for (int j = 0; j < 2; j++) {
    if (bins[j] == kNoBin) break;
    if (k_on && above_k < need && need <= above_k + ck[j]) {
      s.sel_k = bins[j];
      s.need_k = need - above_k;
      s.ties_k = ck[j];
    }
    if (p_on && cp[j] > 0 && (double)(base + above_m) < P) atomicMin(&s.sel_p, bins[j]);
    above_k += ck[j];
    above_m += m[j];
  }
  __syncthreads();
  // the owner of the chosen top-p bin passes down the mass above it
  if (p_on) {
#pragma unroll
    for (int j = 0; j < 2; j++) {
      if (bins[j] != kNoBin && bins[j] == s.sel_p) {
        unsigned long long am = s.w_mass[warp] + im - tm + (j == 1 ? m[0] : 0ull);
        s.above_p = base + am;
        s.ties_p = cp[j];
      }
    }
  }
  __syncthreads();
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    sample_kernel(const T* __restrict__ logits, int64_t stride, int vocab, const int64_t* __restrict__ positions,
                  const float* __restrict__ temperature, const int64_t* __restrict__ top_k,
                  const float* __restrict__ top_p, const int64_t* __restrict__ seeds, int64_t* __restrict__ out) {
  __shared__ Shared s;
  pdl_wait();
  pdl_launch();
  const int row_i = blockIdx.x;
  const T* row = logits + (size_t)row_i * stride;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float temp_in = temperature[row_i];

  // block argmax of (score, index) with the lowest index on ties; `f` or `d` carries the score
  auto argmax_f = [&](float best, int idx) -> int {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xFFFFFFFFu, best, o);
      const int oi = __shfl_xor_sync(0xFFFFFFFFu, idx, o);
      if (ob > best || (ob == best && oi < idx)) {
        best = ob;
        idx = oi;
      }
    }
    if (lane == 0) {
      s.w_f[warp] = best;
      s.w_i[warp] = idx;
    }
    __syncthreads();
    if (warp == 0) {
      best = s.w_f[lane];
      idx = s.w_i[lane];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ob = __shfl_xor_sync(0xFFFFFFFFu, best, o);
        const int oi = __shfl_xor_sync(0xFFFFFFFFu, idx, o);
        if (ob > best || (ob == best && oi < idx)) {
          best = ob;
          idx = oi;
        }
      }
      if (lane == 0) s.w_i[0] = idx;
    }
    __syncthreads();
    const int r = s.w_i[0];
    __syncthreads();
    return r;
  };

  if (!(temp_in > 0.f)) {
    float best = -INFINITY;
    int idx = 0x7FFFFFFF;
    for (int i = threadIdx.x; i < vocab; i += kThreads) {
      const float f = load(row, i);
      if (f > best) {
        best = f;
        idx = i;
      }
    }
    const int r = argmax_f(best, idx);
    if (threadIdx.x == 0) out[row_i] = r == 0x7FFFFFFF ? 0 : r;
    return;
  }

  const float temp = fmaxf(temp_in, 1e-6f);
  int64_t k_req = top_k[row_i];
  const float p_req = top_p[row_i];
  if (p_req <= 0.f) k_req = 1;  // top-p of nothing keeps the top token: top-k of one
  const bool k_on = k_req > 0 && k_req < vocab;
  const bool p_on = p_req < 1.f && p_req > 0.f;

  // the row's maximum z
  float zmax = -INFINITY;
  for (int i = threadIdx.x; i < vocab; i += kThreads) zmax = fmaxf(zmax, __fdiv_rn(load(row, i), temp));
  {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) zmax = fmaxf(zmax, __shfl_xor_sync(0xFFFFFFFFu, zmax, o));
    if (lane == 0) s.w_f[warp] = zmax;
    __syncthreads();
    if (warp == 0) {
      float v = s.w_f[lane];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
      if (lane == 0) s.w_f[0] = v;
    }
    __syncthreads();
    zmax = s.w_f[0];
    __syncthreads();
  }

  // the cut-off: the last kept token is the tie_rank-th token (by index) of key `cut`
  uint32_t cut = 0;
  uint32_t cut_rank = 0, cut_ties = 0;
  bool any_cut = false;
  if (k_on || p_on) {
    if (threadIdx.x == 0) {
      s.need_k = (uint32_t)k_req;
      s.above_p = 0;
    }
    uint32_t pre_k = 0, pre_p = 0;
    double P = 0.0;
    for (int lvl = 0; lvl < 3; lvl++) {
      const int nbits = lvl == 2 ? 10 : 11;  // key bits 31..21, 20..10, 9..0
      const int sh = lvl == 0 ? 21 : (lvl == 1 ? 10 : 0);
      const int nb = 1 << nbits;
      for (int b = threadIdx.x; b < nb; b += kThreads) {
        s.cnt_k[b] = 0;
        s.cnt_p[b] = 0;
        s.mass[b] = 0;
      }
      if (threadIdx.x == 0) s.sel_p = kNoBin;
      __syncthreads();
      const int hs = sh + nbits;
      const uint32_t dmask = (uint32_t)nb - 1;
      const int span = (vocab + kThreads - 1) / kThreads * kThreads;  // every lane runs every round
      for (int i = threadIdx.x; i < span; i += kThreads) {
        uint32_t bin = kNoBin, ak = 0, ap = 0;
        uint64_t m = 0;
        if (i < vocab) {
          const float z = __fdiv_rn(load(row, i), temp);
          const uint32_t key = key_of(z);
          const uint32_t hi = lvl == 0 ? 0u : (key >> hs);
          if (k_on && hi == pre_k) ak = 1;
          if (p_on && hi == pre_p) {
            m = mass_of(z, zmax);
            ap = m > 0 ? 1 : 0;  // a massless token is ranked after every kept one
          }
          if (ak | ap) bin = (key >> sh) & dmask;
        }
        hist_add(s, bin, ak, ap, ap ? m : 0, lane);
      }
      __syncthreads();
      if (lvl == 0 && p_on) {
        // the total mass: every token with mass lands in the first level
        unsigned long long tm = 0;
        for (int b = threadIdx.x; b < nb; b += kThreads) tm += s.mass[b];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) tm += __shfl_xor_sync(0xFFFFFFFFu, tm, o);
        if (lane == 0) s.w_mass[warp] = tm;
        __syncthreads();
        unsigned long long E = 0;
        for (int w = 0; w < kWarps; w++) E += s.w_mass[w];
        P = (double)p_req * (double)E;
        __syncthreads();
      }
      select_bins(s, nb, k_on, p_on, P, lane, warp);
      if (k_on) pre_k = (lvl == 0 ? 0u : pre_k << nbits) | s.sel_k;
      if (p_on) pre_p = (lvl == 0 ? 0u : pre_p << nbits) | s.sel_p;
    }
    // top-k: pre_k is the k-th token's key and need_k its rank among that key's ties
    // top-p: pre_p is the last kept token's key; its ties keep while the mass above stays below P
    uint32_t key_c = 0, rank_c = 0, ties_c = 0;
    if (k_on) {
      key_c = pre_k;
      rank_c = s.need_k;
      ties_c = s.ties_k;
    }
    if (p_on) {
      const uint32_t np = s.ties_p;
      const double e = (double)mass_of(value_of(pre_p), zmax);
      const double room = P - (double)s.above_p;  // > 0 by the choice of the bin
      double q = e > 0.0 ? ceil(room / e) : (double)np;
      if (q < 1.0) q = 1.0;
      const uint32_t rp = q >= (double)np ? np : (uint32_t)q;
      // the earlier of the two cut-offs in the order (a larger key, or fewer ties of one key)
      if (!k_on || pre_p > key_c || (pre_p == key_c && rp < rank_c)) {
        key_c = pre_p;
        rank_c = rp;
        ties_c = np;
      }
    }
    cut = key_c;
    cut_rank = rank_c;
    cut_ties = ties_c;
    any_cut = true;
  }

  // the index of the cut-off tie, unless every tie of the cut-off key is kept
  int cut_index = 0x7FFFFFFF;
  if (any_cut && cut_rank < cut_ties) {
    const int chunk = (vocab + kThreads - 1) / kThreads;
    const int a = threadIdx.x * chunk, b = min(vocab, a + chunk);
    uint32_t c = 0;
    for (int i = a; i < b; i++) c += key_of(__fdiv_rn(load(row, i), temp)) == cut;
    const uint32_t inc = warp_incl_scan(c, lane);
    if (lane == 31) s.w_cnt_k[warp] = inc;
    if (threadIdx.x == 0) s.tie_index = 0x7FFFFFFF;
    __syncthreads();
    if (warp == 0) {
      const uint32_t v = s.w_cnt_k[lane];
      s.w_cnt_p[lane] = warp_incl_scan(v, lane) - v;
    }
    __syncthreads();
    uint32_t before = s.w_cnt_p[warp] + inc - c;
    if (before < cut_rank && cut_rank <= before + c) {
      for (int i = a; i < b; i++) {
        if (key_of(__fdiv_rn(load(row, i), temp)) == cut && ++before == cut_rank) {
          s.tie_index = i;
          break;
        }
      }
    }
    __syncthreads();
    cut_index = s.tie_index;
  }

  // Gumbel-max over the kept tokens
  const uint64_t base = mix((uint64_t)seeds[row_i] * kGolden + (uint64_t)positions[row_i] * kPos);
  double best = -INFINITY;
  int idx = 0x7FFFFFFF;
  for (int i = threadIdx.x; i < vocab; i += kThreads) {
    const float z = __fdiv_rn(load(row, i), temp);
    if (any_cut) {
      const uint32_t key = key_of(z);
      if (key < cut || (key == cut && i > cut_index)) continue;
    }
    const uint64_t x = mix(base + (uint64_t)(i + 1) * kGolden);
    const double u = ((double)(x >> 11) + 0.5) * (1.0 / 9007199254740992.0);
    const double sc = (double)z - log(-log(u));
    if (sc > best) {
      best = sc;
      idx = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const double ob = __shfl_xor_sync(0xFFFFFFFFu, best, o);
    const int oi = __shfl_xor_sync(0xFFFFFFFFu, idx, o);
    if (ob > best || (ob == best && oi < idx)) {
      best = ob;
      idx = oi;
    }
  }
  if (lane == 0) {
    s.w_d[warp] = best;
    s.w_i[warp] = idx;
  }
  __syncthreads();
  if (warp == 0) {
    best = s.w_d[lane];
    idx = s.w_i[lane];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const double ob = __shfl_xor_sync(0xFFFFFFFFu, best, o);
      const int oi = __shfl_xor_sync(0xFFFFFFFFu, idx, o);
      if (ob > best || (ob == best && oi < idx)) {
        best = ob;
        idx = oi;
      }
    }
    if (lane == 0) out[row_i] = idx == 0x7FFFFFFF ? 0 : idx;
  }
}

}  // namespace smp

cudaError_t launch_sample(const SampleArgs& a, cudaStream_t stream) {
  if (a.rows == 0) return cudaSuccess;
  if (a.vocab <= 0 || a.vocab >= (1 << 30)) return cudaErrorInvalidValue;
  if (a.fp32)
    return launch_ex(smp::sample_kernel<float>, dim3((unsigned)a.rows), dim3(smp::kThreads), 0, stream, 0,
                     static_cast<const float*>(a.logits), a.stride, a.vocab, a.positions, a.temperature, a.top_k,
                     a.top_p, a.seeds, a.out);
  return launch_ex(smp::sample_kernel<__nv_bfloat16>, dim3((unsigned)a.rows), dim3(smp::kThreads), 0, stream, 0,
                   static_cast<const __nv_bfloat16*>(a.logits), a.stride, a.vocab, a.positions, a.temperature,
                   a.top_k, a.top_p, a.seeds, a.out);
}

}  // namespace es
