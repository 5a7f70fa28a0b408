// Seeded temperature / top-k / top-p sampling, one CTA per row, deterministic.
//
// A row's token is the Gumbel-max draw argmax(z + g) over the tokens that top-k and top-p keep,
// where z = logit / temperature and g = -log(-log(u)) with u a counter-based uniform of (seed,
// position, token index): SplitMix64 (Steele, Lea, Flood, OOPSLA 2014) of a Weyl sequence, the
// same draw the host sampler makes, so a replayed step samples the same token on any member.
//
// The kept set is a prefix of the order "z descending, then index ascending" (a stable sort):
// top-k keeps its first k tokens, top-p the tokens whose mass ranked above them is below p. Both
// cut-offs are found without a sort. For bf16 logits z orders the tokens as the logits do (a
// positive temperature keeps distinct bf16 values distinct in fp32), so one pass builds a
// histogram over the 65,536 bf16 values in shared memory (16-bit counts, two to a word) and the
// cut-offs are scans over its bins: counts for top-k, counts times each value's mass for top-p.
// fp32 logits (and a bf16 row with more than 65,535 copies of one value) take a three-level radix
// select on the order-preserving 32-bit key of z (11 + 11 + 10 bits) instead, warps combining the
// lanes that hit one bin (match + reduce) before one shared atomic per bin. Masses are fixed point,
// round(exp(z - max) * 2^32) as integers, so every sum is exact and the same in any order: the draw
// does not depend on how the row's threads were scheduled. Ties at a cut-off value are resolved by
// index with one prefix count over the row.
//
// The Gumbel term is computed exactly (float64, as the host sampler does) only for tokens that can
// still win: a float32 upper bound of g, with a margin well above its rounding, rules out the rest.
//
// Greedy rows (temperature <= 0) take the plain argmax, lowest index on ties.
//
// Reference parity: the sampler parameters of the vLLM engine the reference serves (temperature,
// top_k, top_p, seed); the counter-based draw is this framework's (exact replay needs it).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <atomic>
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
  uint32_t w_cnt_k[kWarps], w_cnt_p[kWarps];
  unsigned long long w_mass[kWarps];
  float w_f[kWarps];
  int w_i[kWarps];
  double w_d[kWarps];
  uint32_t sel_k, sel_p;
  uint32_t need_k, ties_k, ties_p;
  unsigned long long above_p, total;
  int tie_index;
  int overflow;
  uint32_t key_k, key_p, kmax;
};

// Radix-select histograms (aliasing the 16-bit value histogram, which is not in use then).
struct Radix {
  uint32_t* cnt_k;
  uint32_t* cnt_p;
  unsigned long long* mass;
};

constexpr int kHistWords = 32768;  // 65,536 16-bit counts, two per word
constexpr int kBinsPerThread = 65536 / kThreads;
constexpr size_t kDynSmem = (size_t)kHistWords * 4;
static_assert(kMaxBins * (4 + 4 + 8) <= kDynSmem, "the radix histograms fit the value histogram's space");

// Order-preserving key of a bf16 value (as its bits); -0 and +0 share the key of +0.
__device__ __forceinline__ uint32_t key16_of(uint32_t bits) {
  if ((bits & 0x7FFFu) == 0) bits = 0;
  return (bits & 0x8000u) ? (~bits & 0xFFFFu) : (bits | 0x8000u);
}
__device__ __forceinline__ float value16_of(uint32_t key) {
  const uint32_t bits = (key & 0x8000u) ? (key & 0x7FFFu) : (~key & 0xFFFFu);
  return __bfloat162float(__ushort_as_bfloat16((unsigned short)bits));
}
template <typename T>
__device__ __forceinline__ uint32_t bits16(const T* row, int i);
template <>
__device__ __forceinline__ uint32_t bits16<__nv_bfloat16>(const __nv_bfloat16* row, int i) {
  return __bfloat16_as_ushort(row[i]);
}
template <>
__device__ __forceinline__ uint32_t bits16<float>(const float*, int) {
  return 0;
}

// Adds a lane's contribution to bin `bin` (kNoBin: none) of the histograms, one atomic per bin and
// warp. Every lane of the warp calls it.
__device__ __forceinline__ void hist_add(const Radix& r, uint32_t bin, uint32_t add_k, uint32_t add_p, uint64_t m,
                                         int lane) {
  const unsigned grp = __match_any_sync(0xFFFFFFFFu, bin);
  if (bin == kNoBin) return;
  const uint32_t ck = __reduce_add_sync(grp, add_k);
  const uint32_t cp = __reduce_add_sync(grp, add_p);
  // a mass is at most 2^32: two 24-bit halves keep the 32-lane sums within 32 bits
  const uint32_t lo = __reduce_add_sync(grp, (uint32_t)(m & 0xFFFFFFu));
  const uint32_t hi = __reduce_add_sync(grp, (uint32_t)(m >> 24));
  if (lane == __ffs(grp) - 1) {
    if (ck) atomicAdd(&r.cnt_k[bin], ck);
    if (cp) {
      atomicAdd(&r.cnt_p[bin], cp);
      atomicAdd(&r.mass[bin], ((unsigned long long)hi << 24) + lo);
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
__device__ void select_bins(Shared& s, const Radix& r, int nb, bool k_on, bool p_on, double P, int lane, int warp) {
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
      ck[j] = r.cnt_k[bins[j]];
      cp[j] = r.cnt_p[bins[j]];
      m[j] = r.mass[bins[j]];
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

// Block-wide helpers (every thread of the CTA calls them).
__device__ float block_max_f(Shared& s, float v, int lane, int warp) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
  if (lane == 0) s.w_f[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float x = s.w_f[lane];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xFFFFFFFFu, x, o));
    if (lane == 0) s.w_f[0] = x;
  }
  __syncthreads();
  const float r = s.w_f[0];
  __syncthreads();
  return r;
}

// Exclusive prefix (in thread order) of a per-thread count and of a per-thread mass; totals out.
__device__ void block_scan(Shared& s, uint32_t c, unsigned long long m, uint32_t* c_excl, unsigned long long* m_excl,
                           unsigned long long* m_total, int lane, int warp) {
  const uint32_t ic = warp_incl_scan(c, lane);
  const unsigned long long im = warp_incl_scan(m, lane);
  if (lane == 31) {
    s.w_cnt_k[warp] = ic;
    s.w_mass[warp] = im;
  }
  __syncthreads();
  if (warp == 0) {
    const uint32_t a = s.w_cnt_k[lane];
    const unsigned long long b = s.w_mass[lane];
    const uint32_t sa = warp_incl_scan(a, lane);
    const unsigned long long sb = warp_incl_scan(b, lane);
    s.w_cnt_k[lane] = sa - a;
    s.w_mass[lane] = sb - b;
    if (lane == 31) s.total = sb;
  }
  __syncthreads();
  *c_excl = s.w_cnt_k[warp] + ic - c;
  *m_excl = s.w_mass[warp] + im - m;
  *m_total = s.total;
  __syncthreads();
}

// Row argmax (lowest index on ties) of a double score; thread 0 gets the index.
__device__ int block_argmax_d(Shared& s, double best, int idx, int lane, int warp) {
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
  }
  return idx;
}

// The rank (1-based, by index) among the ties of the cut-off tie from the two cut-offs: the earlier
// of the two in the order (a larger key, or fewer ties of one key).
struct Cut {
  uint32_t key = 0, rank = 0, ties = 0;
};
__device__ Cut combine(bool k_on, uint32_t key_k, uint32_t rank_k, uint32_t ties_k, bool p_on, uint32_t key_p,
                       double room, double e, uint32_t ties_p) {
  Cut c;
  if (k_on) {
    c.key = key_k;
    c.rank = rank_k;
    c.ties = ties_k;
  }
  if (p_on) {
    // the j-th tie (0-based) has mass above + j * e ranked above it; it stays while that is below P
    double q = e > 0.0 ? ceil(room / e) : (double)ties_p;
    if (q < 1.0) q = 1.0;
    const uint32_t rp = q >= (double)ties_p ? ties_p : (uint32_t)q;
    if (!k_on || key_p > c.key || (key_p == c.key && rp < c.rank)) {
      c.key = key_p;
      c.rank = rp;
      c.ties = ties_p;
    }
  }
  return c;
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    sample_kernel(const T* __restrict__ logits, int64_t stride, int vocab, const int64_t* __restrict__ positions,
                  const float* __restrict__ temperature, const int64_t* __restrict__ top_k,
                  const float* __restrict__ top_p, const int64_t* __restrict__ seeds, int64_t* __restrict__ out) {
  __shared__ Shared s;
  extern __shared__ __align__(16) uint32_t dyn[];
  pdl_wait();
  pdl_launch();
  const int row_i = blockIdx.x;
  const T* row = logits + (size_t)row_i * stride;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float temp_in = temperature[row_i];
  constexpr bool kBf16 = sizeof(T) == 2;

  if (!(temp_in > 0.f)) {
    // greedy: the plain argmax of the logits
    float best = -INFINITY;
    int idx = 0x7FFFFFFF;
    for (int i = tid; i < vocab; i += kThreads) {
      const float f = load(row, i);
      if (f > best) {
        best = f;
        idx = i;
      }
    }
    const int r = block_argmax_d(s, (double)best, idx, lane, warp);
    if (tid == 0) out[row_i] = r == 0x7FFFFFFF ? 0 : r;
    return;
  }

  const float temp = fmaxf(temp_in, 1e-6f);
  int64_t k_req = top_k[row_i];
  const float p_req = top_p[row_i];
  if (p_req <= 0.f) k_req = 1;  // top-p of nothing keeps the top token: top-k of one
  const bool k_on = k_req > 0 && k_req < vocab;
  const bool p_on = p_req < 1.f && p_req > 0.f;
  const bool any_cut = k_on || p_on;

  // ---- bf16: one histogram over the 65,536 values ------------------------------------------
  bool use16 = false;
  float zmax = -INFINITY;
  Cut cut;
  if (kBf16) {
    for (int w = tid; w < kHistWords; w += kThreads) dyn[w] = 0u;
    if (tid == 0) s.overflow = 0;
    __syncthreads();
    for (int i = tid; i < vocab; i += kThreads) {
      const uint32_t key = key16_of(bits16(row, i));
      const uint32_t sh = (key & 1u) << 4;
      const uint32_t old = atomicAdd(&dyn[key >> 1], 1u << sh);
      if (((old >> sh) & 0xFFFFu) == 0xFFFFu) s.overflow = 1;  // a 16-bit count wrapped
    }
    __syncthreads();
    use16 = s.overflow == 0;
  }
  if (use16) {
    // thread t holds the bins at descending positions [t * 64, t * 64 + 64): keys 65535 - position
    const uint32_t top = 65535u - (uint32_t)tid * kBinsPerThread;
    auto count_of = [&](uint32_t key) -> uint32_t { return (dyn[key >> 1] >> ((key & 1u) << 4)) & 0xFFFFu; };
    uint32_t mine_max = 0, ctot = 0;
    for (int j = 0; j < kBinsPerThread; j++) {
      const uint32_t c = count_of(top - j);
      if (c && !mine_max) mine_max = top - j + 1;  // + 1: zero means none
      ctot += c;
    }
    // the largest key present (a block max over integers, through the float helper's slots)
    if (lane == 0) s.w_i[warp] = 0;
    __syncthreads();
    atomicMax(&s.w_i[warp], (int)mine_max);
    __syncthreads();
    if (tid == 0) {
      int m = 0;
      for (int w = 0; w < kWarps; w++) m = max(m, s.w_i[w]);
      s.kmax = (uint32_t)(m - 1);
      s.key_p = 0xFFFFFFFFu;
    }
    __syncthreads();
    const uint32_t kmax = s.kmax;
    zmax = __fdiv_rn(value16_of(kmax), temp);
    if (any_cut) {
      // masses of this thread's bins (each value's mass times its count)
      unsigned long long mtot = 0;
      if (p_on)
        for (int j = 0; j < kBinsPerThread; j++) {
          const uint32_t c = count_of(top - j);
          if (c) mtot += (unsigned long long)c * mass_of(__fdiv_rn(value16_of(top - j), temp), zmax);
        }
      uint32_t c_ex;
      unsigned long long m_ex, E;
      block_scan(s, ctot, mtot, &c_ex, &m_ex, &E, lane, warp);
      const double P = (double)p_req * (double)E;
      const uint32_t need = (uint32_t)k_req;
      uint32_t run_c = c_ex;
      unsigned long long run_m = m_ex;
      uint32_t cand_p = 0xFFFFFFFFu;
      for (int j = 0; j < kBinsPerThread; j++) {
        const uint32_t key = top - j;
        const uint32_t c = count_of(key);
        if (c == 0) continue;
        if (k_on && run_c < need && need <= run_c + c) {
          s.key_k = key;
          s.need_k = need - run_c;
          s.ties_k = c;
        }
        unsigned long long e = 0;
        if (p_on) {
          e = mass_of(__fdiv_rn(value16_of(key), temp), zmax);
          if ((double)run_m < P) cand_p = key;  // the last such bin in the order: its smallest key
        }
        run_c += c;
        run_m += (unsigned long long)c * e;
      }
      if (p_on && cand_p != 0xFFFFFFFFu) atomicMin(&s.key_p, cand_p);
      __syncthreads();
      if (p_on) {
        // the owner of the chosen bin passes down the mass above it
        const uint32_t kp = s.key_p;
        if (kp <= top && kp + kBinsPerThread > top) {
          unsigned long long above = m_ex;
          for (uint32_t key = top; key > kp; key--) {
            const uint32_t c = count_of(key);
            if (c) above += (unsigned long long)c * mass_of(__fdiv_rn(value16_of(key), temp), zmax);
          }
          s.above_p = above;
          s.ties_p = count_of(kp);
        }
      }
      __syncthreads();
      double room = 0.0, e = 0.0;
      if (p_on) {
        room = P - (double)s.above_p;
        e = (double)mass_of(__fdiv_rn(value16_of(s.key_p), temp), zmax);
      }
      cut = combine(k_on, s.key_k, s.need_k, s.ties_k, p_on, s.key_p, room, e, s.ties_p);
    }
  } else {
    // ---- fp32 logits, or a bf16 row with a value held more than 65,535 times: radix select --
    float zm = -INFINITY;
    for (int i = tid; i < vocab; i += kThreads) zm = fmaxf(zm, __fdiv_rn(load(row, i), temp));
    zmax = block_max_f(s, zm, lane, warp);
    if (any_cut) {
      Radix r{dyn, dyn + kMaxBins, reinterpret_cast<unsigned long long*>(dyn + 2 * kMaxBins)};
      if (tid == 0) {
        s.need_k = (uint32_t)k_req;
        s.above_p = 0;
      }
      uint32_t pre_k = 0, pre_p = 0;
      double P = 0.0;
      for (int lvl = 0; lvl < 3; lvl++) {
        const int nbits = lvl == 2 ? 10 : 11;  // key bits 31..21, 20..10, 9..0
        const int sh = lvl == 0 ? 21 : (lvl == 1 ? 10 : 0);
        const int nb = 1 << nbits;
        for (int b = tid; b < nb; b += kThreads) {
          r.cnt_k[b] = 0;
          r.cnt_p[b] = 0;
          r.mass[b] = 0;
        }
        if (tid == 0) s.sel_p = kNoBin;
        __syncthreads();
        const int hs = sh + nbits;
        const uint32_t dmask = (uint32_t)nb - 1;
        const int span = (vocab + kThreads - 1) / kThreads * kThreads;  // every lane runs every round
        for (int i = tid; i < span; i += kThreads) {
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
          hist_add(r, bin, ak, ap, ap ? m : 0, lane);
        }
        __syncthreads();
        if (lvl == 0 && p_on) {
          // the total mass: every token with mass lands in the first level
          unsigned long long tm = 0;
          for (int b = tid; b < nb; b += kThreads) tm += r.mass[b];
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) tm += __shfl_xor_sync(0xFFFFFFFFu, tm, o);
          if (lane == 0) s.w_mass[warp] = tm;
          __syncthreads();
          unsigned long long E = 0;
          for (int w = 0; w < kWarps; w++) E += s.w_mass[w];
          P = (double)p_req * (double)E;
          __syncthreads();
        }
        select_bins(s, r, nb, k_on, p_on, P, lane, warp);
        if (k_on) pre_k = (lvl == 0 ? 0u : pre_k << nbits) | s.sel_k;
        if (p_on) pre_p = (lvl == 0 ? 0u : pre_p << nbits) | s.sel_p;
      }
      const double room = p_on ? P - (double)s.above_p : 0.0;
      const double e = p_on ? (double)mass_of(value_of(pre_p), zmax) : 0.0;
      cut = combine(k_on, pre_k, s.need_k, s.ties_k, p_on, pre_p, room, e, s.ties_p);
    }
  }
  // a token's key in the order: its bf16 value's (histogram path) or its z's (radix path)
  auto key_at = [&](int i) -> uint32_t {
    return use16 ? key16_of(bits16(row, i)) : key_of(__fdiv_rn(load(row, i), temp));
  };

  // the index of the cut-off tie, unless every tie of the cut-off key is kept
  int cut_index = 0x7FFFFFFF;
  if (any_cut && cut.rank < cut.ties) {
    const int chunk = (vocab + kThreads - 1) / kThreads;
    const int a = tid * chunk, b = min(vocab, a + chunk);
    uint32_t c = 0;
    for (int i = a; i < b; i++) c += key_at(i) == cut.key;
    const uint32_t inc = warp_incl_scan(c, lane);
    if (lane == 31) s.w_cnt_k[warp] = inc;
    if (tid == 0) s.tie_index = 0x7FFFFFFF;
    __syncthreads();
    if (warp == 0) {
      const uint32_t v = s.w_cnt_k[lane];
      s.w_cnt_p[lane] = warp_incl_scan(v, lane) - v;
    }
    __syncthreads();
    uint32_t before = s.w_cnt_p[warp] + inc - c;
    if (before < cut.rank && cut.rank <= before + c) {
      for (int i = a; i < b; i++) {
        if (key_at(i) == cut.key && ++before == cut.rank) {
          s.tie_index = i;
          break;
        }
      }
    }
    __syncthreads();
    cut_index = s.tie_index;
  }

  // Gumbel-max over the kept tokens. g = -log(-log u) in float64 decides; a float32 upper bound of
  // it rules out the tokens that cannot beat this thread's best so far (a later index never wins
  // a tie within the thread).
  const uint64_t base = mix((uint64_t)seeds[row_i] * kGolden + (uint64_t)positions[row_i] * kPos);
  double best = -INFINITY;
  int idx = 0x7FFFFFFF;
  for (int i = tid; i < vocab; i += kThreads) {
    if (any_cut) {
      const uint32_t key = key_at(i);
      if (key < cut.key || (key == cut.key && i > cut_index)) continue;
    }
    const float z = __fdiv_rn(load(row, i), temp);
    const uint64_t k53 = mix(base + (uint64_t)(i + 1) * kGolden) >> 11;
    // L = -log(u) from the side that keeps its precision: u itself below 1/2, 1 - u (exact) above
    float L;
    if (k53 < (1ull << 52)) {
      L = -logf((float)(((double)k53 + 0.5) * (1.0 / 9007199254740992.0)));
    } else {
      const double one_minus_u = ((double)((1ull << 53) - k53) - 0.5) * (1.0 / 9007199254740992.0);
      L = -log1pf(-(float)one_minus_u);
    }
    const float gf = -logf(L);
    const float g_hi = gf + 1e-5f * (1.f + fabsf(gf));  // above g by far more than the roundings
    if ((double)z + (double)g_hi <= best) continue;
    const double u = ((double)k53 + 0.5) * (1.0 / 9007199254740992.0);
    const double sc = (double)z - log(-log(u));
    if (sc > best) {
      best = sc;
      idx = i;
    }
  }
  const int r = block_argmax_d(s, best, idx, lane, warp);
  if (tid == 0) out[row_i] = r == 0x7FFFFFFF ? 0 : r;
}

}  // namespace smp

cudaError_t launch_sample(const SampleArgs& a, cudaStream_t stream) {
  if (a.rows == 0) return cudaSuccess;
  if (a.vocab <= 0 || a.vocab >= (1 << 30)) return cudaErrorInvalidValue;
  static std::atomic<uint64_t> configured{0};
  cudaError_t e = once_per_device(configured, [] {
    cudaError_t r = cudaFuncSetAttribute(smp::sample_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smp::kDynSmem);
    if (r != cudaSuccess) return r;
    return cudaFuncSetAttribute(smp::sample_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)smp::kDynSmem);
  });
  if (e != cudaSuccess) return e;
  if (a.fp32)
    return launch_ex(smp::sample_kernel<float>, dim3((unsigned)a.rows), dim3(smp::kThreads), smp::kDynSmem, stream, 0,
                     static_cast<const float*>(a.logits), a.stride, a.vocab, a.positions, a.temperature, a.top_k,
                     a.top_p, a.seeds, a.out);
  return launch_ex(smp::sample_kernel<__nv_bfloat16>, dim3((unsigned)a.rows), dim3(smp::kThreads), smp::kDynSmem,
                   stream, 0, static_cast<const __nv_bfloat16*>(a.logits), a.stride, a.vocab, a.positions,
                   a.temperature, a.top_k, a.top_p, a.seeds, a.out);
}

}  // namespace es
