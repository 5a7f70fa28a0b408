// Persistent paged decode attention: one CTA per SM streams its share of every sequence's history.
//
// The work of a decode step is the list of items (sequence b, kv head, split of part_tokens
// positions), pair-major: the splits of one (sequence, kv head) pair are consecutive. Every CTA
// takes one contiguous range of that list (the same number of items each, so the SMs finish
// together whatever the lengths), and within a CTA:
//
//   * a producer warp walks the range and streams it: per item the G query rows (one bulk copy
//     into a small ring of q slots), then the K and V rows 16 positions at a time (TMA, 128-byte
//     swizzle, evict-first) into a ring per consumer warp; unit j of an item goes to warp
//     (j + kv head + split) % 7, a function of the item alone (a warp's share of the split, and so
//     the rounding of the split's result, never depends on the batch), rotated so the warps that
//     take an item's extra units change from item to item; the producer runs ahead across item
//     boundaries (no ramp per item, no tail per CTA);
//   * seven consumer warps each compute S = q.K^T and O += P.V with mma.sync m16n8k16 on their
//     units with their own online softmax, then the seven merge through shared memory into the
//     split's (o, m, l);
//   * the splits of a pair that lies wholly inside the range are merged right there, in split
//     order, into the bf16 output (no partials in global memory, no second launch); a pair cut by
//     a range boundary writes its splits' partials, and the last CTA to finish its share (an
//     atomic ticket per pair, at most two such pairs per CTA) merges them in split order.
//
// Both merges run the same sequential update (`merge_step`, rounded operations only), so a
// sequence's output does not depend on where the range boundaries fell, i.e. on the batch.
// The reference's decode attention is a paged kernel per (sequence, head) block
// (core/csrc/attention/paged_attention.cu); this kernel is this framework's own design.
#include <cuda.h>

#include <algorithm>
#include <atomic>

#include "api.h"
#include "launch.h"
#include "common.cuh"
#include "ptx.cuh"
#include "tmap.h"

namespace es {
namespace persist {

constexpr int kConsumers = 7;  // consumer warps (with the producer, 8 warps: no register-file rounding)
constexpr int kThreads = (kConsumers + 1) * 32;  // + the producer warp
constexpr int kCombine = kConsumers * 32;      // threads of the consumer warps
constexpr int kQSlots = 4;
constexpr int kMaxPer = (8 * 128 + kConsumers * 32 - 1) / (kConsumers * 32);  // outputs per consumer thread (G * D <= 8 * 128)
constexpr int kBarCombine = 1;
constexpr float kLog2e = 1.4426950408889634f;
constexpr int kAlignSlack = 1024 + 64;  // the ring's 1024-byte alignment, and the static words

struct Params {
  const __nv_bfloat16* q;  // [B, Hq, D] rows of q_stride elements
  int64_t q_stride;
  const int* block_tables;
  int64_t bt_stride;
  const int* ctx_lens;
  float* part_o;   // [B, Hq, max_splits, D] (pairs cut by a range boundary only)
  float* part_ml;  // [B, Hq, max_splits, 2]
  int* tickets;    // [B, Hkv] zero between launches
  __nv_bfloat16* out;  // [B, Hq * D] rows of out_stride
  int64_t out_stride;
  const uint8_t* pf;  // memory the next kernel reads, fetched into L2 meanwhile (nullable)
  int64_t pf_bytes;
  int B, hq, hkv, block_size, max_splits, part_tokens, ws;
  float scale_log2;
  int* status;
};

// Shared-memory layout, from the launch's shapes (the host computes the same to size the launch).
struct Layout {
  int bars, pre, q, red_o, red_ml, ring, total;
  __host__ __device__ static Layout make(int B, int G, int D, int ws) {
    Layout L;
    int off = 0;
    L.bars = off;  // full[8][ws], empty[8][ws], qfull[4], qempty[4]
    off += (2 * kConsumers * ws + 2 * kQSlots) * 8;
    L.pre = off;  // B + 1 ints: items before each sequence, then B context lengths
    off += ((2 * B + 1) * 4 + 15) / 16 * 16;
    L.q = off;
    off += kQSlots * G * D * 2;
    L.red_o = off;  // two buffers: items alternate, so one barrier per item suffices
    off += 2 * kConsumers * G * D * 4;
    L.red_ml = off;
    off += 2 * kConsumers * G * 2 * 4;
    L.ring = (off + 1023) / 1024 * 1024;
    L.total = L.ring + kConsumers * ws * 2 * 16 * D * 2;
    return L;
  }
};

ES_DEVICE int splits_of(int ctx, const Params& p) {
  return ctx <= 0 ? 1 : min(p.max_splits, (ctx + p.part_tokens - 1) / p.part_tokens);
}

// One split's (o, m, l) folded into the running state of one output, in split order. Rounded
// operations only, so the update is the same wherever it is compiled.
ES_DEVICE void merge_step(float& m, float& den, float& acc, float ms, float ls, float os) {
  if (ms == -INFINITY) return;  // an empty split
  const float mn = fmaxf(m, ms);
  const float a = m == -INFINITY ? 0.f : exp2f(__fsub_rn(m, mn));
  const float w = __fmul_rn(ls, exp2f(__fsub_rn(ms, mn)));
  acc = __fadd_rn(__fmul_rn(acc, a), __fmul_rn(w, os));
  den = __fadd_rn(__fmul_rn(den, a), w);
  m = mn;
}
ES_DEVICE float merge_final(float den, float acc) { return den > 0.f ? __fdiv_rn(acc, den) : 0.f; }

// byte offset of element (t, d) of a 16-position K/V tile written by TMA with 128-byte swizzle
template <int D>
ES_DEVICE uint32_t swz(int t, int d) {
  const int hr = t * (D / 64) + (d >> 6);
  const int chunk = (d & 63) >> 3;
  return (uint32_t)(hr * 128 + ((chunk ^ (hr & 7)) << 4) + (d & 7) * 2);
}

// Walks the items of a range in order: (sequence, kv head, split), with the pair's bounds.
struct Cursor {
  int b, kvh, split, ns, ctx;
  int64_t item, pair0;  // this item's index and its pair's first item
};

// the first unit of an item that consumer warp w takes (then every kConsumers-th)
ES_DEVICE int first_unit(int w, const Cursor& c) { return (w - (c.kvh + c.split) % kConsumers + kConsumers) % kConsumers; }

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    decode_persist_kernel(const __grid_constant__ CUtensorMap cmap, Params p) {
  constexpr int NT = D / 8;
  constexpr int kTile = 16 * D * 2;  // 16 positions of K (or of V)
  constexpr int kRowsPerTok = D / 64;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int G = p.hq / p.hkv;
  const Layout L = Layout::make(p.B, G, D, p.ws);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);  // [warp][ws]
  uint64_t* empty = full + kConsumers * p.ws;
  uint64_t* qfull = empty + kConsumers * p.ws;
  uint64_t* qempty = qfull + kQSlots;
  int* pre = reinterpret_cast<int*>(smem + L.pre);
  int* ctxs = pre + p.B + 1;
  __nv_bfloat16* qsl = reinterpret_cast<__nv_bfloat16*>(smem + L.q);
  float* red_o2 = reinterpret_cast<float*>(smem + L.red_o);    // [2][warp][G][D]
  float* red_ml2 = reinterpret_cast<float*>(smem + L.red_ml);  // [2][warp][G][2]
  uint8_t* ring = smem + L.ring;                              // [warp][ws][K, V]
  __shared__ int s_fail;
  __shared__ int s_last;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // a bounded wait that ran out: every role stops waiting, the host reads the status word
  auto give_up = [&]() {
    *(volatile int*)&s_fail = 1;
    if (p.status) atomicExch(p.status, (int)kTimeout);
  };
  if (tid == 0) {
    s_fail = 0;
    ptx::prefetch_tmap(&cmap);
    for (int i = 0; i < kConsumers * p.ws; i++) {
      ptx::mbar_init(&full[i], 1);
      ptx::mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < kQSlots; i++) {
      ptx::mbar_init(&qfull[i], 1);
      ptx::mbar_init(&qempty[i], kConsumers);
    }
    ptx::fence_mbar_init();
  }
  pdl_wait();  // q, the cache rows of this step and the context lengths come from earlier kernels
  pdl_launch();
  // items before each sequence: counts, then one warp's running scan
  for (int b = tid; b < p.B; b += kThreads) {
    const int ctx = p.ctx_lens[b];
    ctxs[b] = ctx;
    pre[b + 1] = splits_of(ctx, p) * p.hkv;
  }
  __syncthreads();
  if (warp == 0) {
    int carry = 0;
    for (int b0 = 0; b0 < p.B; b0 += 32) {
      const int b = b0 + lane;
      int v = b < p.B ? pre[b + 1] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += u;
      }
      if (b < p.B) pre[b + 1] = carry + v;
      carry += __shfl_sync(0xffffffffu, v, 31);
    }
    if (lane == 0) pre[0] = 0;
  }
  __syncthreads();
  const int64_t n_items = pre[p.B];
  const int64_t i0 = n_items * blockIdx.x / gridDim.x, i1 = n_items * (blockIdx.x + 1) / gridDim.x;
  if (i0 >= i1) return;
  // the sequence of the first item: the last b with pre[b] <= i0
  Cursor c0;
  {
    int lo = 0, hi = p.B - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (pre[mid] <= i0) lo = mid;
      else hi = mid - 1;
    }
    c0.b = lo;
    c0.ctx = ctxs[lo];
    c0.ns = splits_of(c0.ctx, p);
    const int64_t r = i0 - pre[lo];
    c0.kvh = (int)(r / c0.ns);
    c0.split = (int)(r % c0.ns);
    c0.item = i0;
    c0.pair0 = i0 - c0.split;
  }
  auto advance = [&](Cursor& c) {
    c.item++;
    if (++c.split < c.ns) return;
    c.split = 0;
    c.pair0 = c.item;
    if (++c.kvh < p.hkv) return;
    c.kvh = 0;
    if (++c.b < p.B) {
      c.ctx = ctxs[c.b];
      c.ns = splits_of(c.ctx, p);
    }
  };
  const int qbytes = G * D * 2;

  if (warp == kConsumers) {
    // ---------------- producer ----------------
    // Lane w < kConsumers feeds consumer warp w. The lanes poll their next slot without blocking
    // (mbarrier.test_wait) in one converged loop, so every lane whose slot is free issues in the
    // same pass and no lane's wait holds up the others; the item's block-table entries are fetched
    // one item ahead (lane u holds units u and u + 32). Lane 0 also streams the q rows.
    if (lane == 0) ptx::l2_prefetch_share(p.pf, p.pf_bytes, (int)blockIdx.x, (int)gridDim.x);
    const uint64_t pol = ptx::policy_evict_first();
    int cnt = 0;  // lane w < kConsumers: units issued to consumer warp w
    int qi = 0;
    bool ok = true;
    // physical block of unit u of item x (-1 past the item's units)
    auto fetch = [&](const Cursor& x, int u) -> int {
      const int s0 = x.split * p.part_tokens;
      const int s1 = min(x.ctx, s0 + p.part_tokens);
      if (s0 + u * 16 >= s1) return -1;
      return p.block_tables[(size_t)x.b * p.bt_stride + (s0 + u * 16) / p.block_size];
    };
    Cursor c = c0;
    int ph0 = fetch(c, lane), ph1 = fetch(c, lane + 32);
    uint64_t t_idle = 0;  // global time when the lanes last made no progress (0: they did)
    for (int64_t it = i0; it < i1 && ok; it++, advance(c)) {
      const int s0 = c.split * p.part_tokens;
      const int s1 = min(c.ctx, s0 + p.part_tokens);
      const int nu = s1 > s0 ? (s1 - s0 + 15) / 16 : 0;
      int n0 = -1, n1 = -1;
      if (it + 1 < i1) {
        Cursor n = c;
        advance(n);
        n0 = fetch(n, lane);
        n1 = fetch(n, lane + 32);
      }
      if (lane == 0) {
        const int qs = qi % kQSlots;
        if (qi >= kQSlots && !ptx::mbar_wait(&qempty[qs], ((qi / kQSlots) - 1) & 1)) ok = false;
        if (ok) {
          ptx::mbar_arrive_expect_tx(&qfull[qs], (uint32_t)qbytes);
          ptx::bulk_g2s(qsl + (size_t)qs * G * D, p.q + (size_t)c.b * p.q_stride + (size_t)c.kvh * G * D,
                        (uint32_t)qbytes, &qfull[qs]);
        }
      }
      qi++;
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0 && *(volatile int*)&s_fail == 0;
      int j = lane < kConsumers ? first_unit(lane, c) : nu;  // this lane's next unit of the item
      while (ok) {
        const bool pending = j < nu;
        if (!__any_sync(0xffffffffu, pending)) break;
        // unit j's block: from lane j % 32 (units below 64), else straight from the table
        const int a = __shfl_sync(0xffffffffu, ph0, j & 31), b1 = __shfl_sync(0xffffffffu, ph1, j & 31);
        bool issued = false;
        if (pending) {
          const int slot = cnt % p.ws;
          if (cnt < p.ws || ptx::mbar_test(&empty[lane * p.ws + slot], ((cnt / p.ws) - 1) & 1)) {
            const int64_t phys = j < 32 ? a : (j < 64 ? b1 : fetch(c, j));
            const int tok = s0 + j * 16;
            const int64_t row = ((phys * 2 * p.hkv + c.kvh) * p.block_size + tok % p.block_size) * kRowsPerTok;
            const int64_t vrow = row + (int64_t)p.hkv * p.block_size * kRowsPerTok;
            uint64_t* fb = &full[lane * p.ws + slot];
            uint8_t* dst = ring + (size_t)(lane * p.ws + slot) * 2 * kTile;
            ptx::mbar_arrive_expect_tx(fb, 2 * kTile);
            ptx::tma_load_2d_hint(dst, &cmap, 0, (int32_t)row, fb, pol);
            ptx::tma_load_2d_hint(dst + kTile, &cmap, 0, (int32_t)vrow, fb, pol);
            cnt++;
            j += kConsumers;
            issued = true;
          }
        }
        // every ring was full: back off briefly, and give up after the wait bound
        if (!__any_sync(0xffffffffu, issued)) {
          const uint64_t now = global_ns();
          if (t_idle == 0) t_idle = now;
          else if (now - t_idle > 2000000000ull) ok = false;
          __nanosleep(64);
        } else {
          t_idle = 0;
        }
        ok = __all_sync(0xffffffffu, ok) && *(volatile int*)&s_fail == 0;
      }
      ph0 = n0;
      ph1 = n1;
    }
    if (!ok) {
      if (lane == 0) give_up();
      // the consumers stop waiting; let this warp's copies in flight land before the CTA leaves
      if (lane < kConsumers)
        for (int k = max(0, cnt - p.ws); k < cnt; k++)
          ptx::mbar_wait(&full[lane * p.ws + k % p.ws], (k / p.ws) & 1, 100000000ull);
    }
    return;
  }

  // ---------------- consumers ----------------
  const int gid = lane >> 2, tig = lane & 3;
  const int GD = G * D;
  float acc[kMaxPer], rm[kMaxPer], rd[kMaxPer];  // running merge of this thread's outputs
  int cnt = 0, qi = 0;
  Cursor c = c0;
  for (int64_t it = i0; it < i1; it++, advance(c)) {
    const int s0 = c.split * p.part_tokens;
    const int s1 = min(c.ctx, s0 + p.part_tokens);
    const int nu = s1 > s0 ? (s1 - s0 + 15) / 16 : 0;
    bool failed = *(volatile int*)&s_fail != 0;
    // q fragments (rows = the G heads, zero above G; rows 8..15 are always zero)
    uint32_t qa[D / 16][2];
    {
      const int qs = qi % kQSlots;
      if (!failed && !ptx::mbar_wait(&qfull[qs], (qi / kQSlots) & 1)) {
        failed = true;
        give_up();
      }
      const __nv_bfloat16* qrow = qsl + (size_t)qs * GD + (size_t)gid * D;
#pragma unroll
      for (int ks = 0; ks < D / 16; ks++) {
        if (gid < G && !failed) {
          qa[ks][0] = *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + tig * 2);
          qa[ks][1] = *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 8 + tig * 2);
        } else {
          qa[ks][0] = qa[ks][1] = 0u;
        }
      }
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&qempty[qs]);
      qi++;
    }
    float o[NT][4];
#pragma unroll
    for (int i = 0; i < NT; i++) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float m_run = -INFINITY, l_run = 0.f;
    for (int j = first_unit(warp, c); j < nu; j += kConsumers) {
      const int slot = cnt % p.ws;
      if (!failed && !ptx::mbar_wait(&full[warp * p.ws + slot], (cnt / p.ws) & 1)) {
        failed = true;
        give_up();
      }
      failed = __any_sync(0xffffffffu, failed) || *(volatile int*)&s_fail != 0;
      cnt++;
      if (failed) continue;
      const uint32_t kbase = ptx::smem_u32(ring + (size_t)(warp * p.ws + slot) * 2 * kTile);
      const uint32_t vbase = kbase + kTile;
      const int tok0 = s0 + j * 16;
      // S = q . K^T over the 16 positions: the even and odd k-steps accumulate apart (four
      // independent chains of D / 32 instead of two of D / 16), then add
      float s[2][4], s_odd[2][4];
#pragma unroll
      for (int jn = 0; jn < 2; jn++)
#pragma unroll
        for (int e = 0; e < 4; e++) s[jn][e] = s_odd[jn][e] = 0.f;
#pragma unroll
      for (int kp = 0; kp < D / 32; kp++) {
#pragma unroll
        for (int jn = 0; jn < 2; jn++) {
          uint32_t b0, b1, b2, b3;
          const int t = jn * 8 + (lane & 7);
          const int d = kp * 32 + (lane >> 3) * 8;
          ptx::ldmatrix_x4(kbase + swz<D>(t, d), b0, b1, b2, b3);
          const uint32_t a0[4] = {qa[2 * kp][0], 0u, qa[2 * kp][1], 0u};
          const uint32_t a1[4] = {qa[2 * kp + 1][0], 0u, qa[2 * kp + 1][1], 0u};
          ptx::mma_bf16_16816(s[jn], a0, b0, b1);
          ptx::mma_bf16_16816(s_odd[jn], a1, b2, b3);
        }
      }
#pragma unroll
      for (int jn = 0; jn < 2; jn++)
#pragma unroll
        for (int e = 0; e < 4; e++) s[jn][e] += s_odd[jn][e];
      float v[4];
      float mx = -INFINITY;
#pragma unroll
      for (int jn = 0; jn < 2; jn++) {
#pragma unroll
        for (int e = 0; e < 2; e++) {
          const int pos = tok0 + jn * 8 + tig * 2 + e;
          const float x = pos < s1 ? s[jn][e] * p.scale_log2 : -INFINITY;
          v[jn * 2 + e] = x;
          mx = fmaxf(mx, x);
        }
      }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float m_new = fmaxf(m_run, mx);
      const bool none = m_new == -INFINITY;
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
#pragma unroll
      for (int np = 0; np < D / 16; np++) {
        uint32_t b0, b1, b2, b3;
        const int mi = lane >> 3;
        const int t = (mi & 1) * 8 + (lane & 7);
        const int d = np * 16 + (mi >> 1) * 8;
        ptx::ldmatrix_x4_trans(vbase + swz<D>(t, d), b0, b1, b2, b3);
        ptx::mma_bf16_16816(o[2 * np], pa, b0, b1);
        ptx::mma_bf16_16816(o[2 * np + 1], pa, b2, b3);
      }
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&empty[warp * p.ws + slot]);
    }
    // merge the eight warps' (o, m, l) into the split's
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
    // this item's buffers were last read by the combine two items back, which every thread finished
    // before the barrier of the item between
    float* red_o = red_o2 + (size_t)((it - i0) & 1) * kConsumers * GD;
    float* red_ml = red_ml2 + (size_t)((it - i0) & 1) * kConsumers * G * 2;
    if (gid < G) {
#pragma unroll
      for (int i = 0; i < NT; i++) {
        red_o[(warp * G + gid) * D + i * 8 + tig * 2] = failed ? 0.f : o[i][0];
        red_o[(warp * G + gid) * D + i * 8 + tig * 2 + 1] = failed ? 0.f : o[i][1];
      }
      if (tig == 0) {
        red_ml[(warp * G + gid) * 2] = failed ? -INFINITY : m_run;
        red_ml[(warp * G + gid) * 2 + 1] = failed ? 0.f : l_run;
      }
    }
    ptx::named_bar(kBarCombine, kCombine);
    const int64_t pair1 = c.pair0 + c.ns;
    const bool cut = c.pair0 < i0 || pair1 > i1;  // the pair's splits are not all in this range
#pragma unroll
    for (int k = 0; k < kMaxPer; k++) {
      const int e = tid + k * kCombine;
      if (e >= GD) continue;
      const int g = e / D, d = e % D;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kConsumers; w++) M = fmaxf(M, red_ml[(w * G + g) * 2]);
      float num = 0.f, den = 0.f;
#pragma unroll
      for (int w = 0; w < kConsumers; w++) {
        const float mw = red_ml[(w * G + g) * 2];
        const float f = mw == -INFINITY ? 0.f : exp2f(mw - M);
        num += red_o[(w * G + g) * D + d] * f;
        den += red_ml[(w * G + g) * 2 + 1] * f;
      }
      const float os = den > 0.f ? __fdiv_rn(num, den) : 0.f;
      const float ms = den > 0.f ? M : -INFINITY;
      if (cut) {
        const size_t row = ((size_t)c.b * p.hq + c.kvh * G + g) * p.max_splits + c.split;
        p.part_o[row * D + d] = os;
        if (d == 0) {
          p.part_ml[row * 2] = ms;
          p.part_ml[row * 2 + 1] = den;
        }
      } else {
        if (c.split == 0) {
          rm[k] = -INFINITY;
          rd[k] = 0.f;
          acc[k] = 0.f;
        }
        merge_step(rm[k], rd[k], acc[k], ms, den, os);
        if (c.split == c.ns - 1)
          p.out[(size_t)c.b * p.out_stride + (size_t)(c.kvh * G + g) * D + d] = f2bf(merge_final(rd[k], acc[k]));
      }
    }
    // a cut pair: after this range's last split of it, count the splits in; the last range merges
    if (cut && (c.item == pair1 - 1 || it == i1 - 1)) {
      __threadfence();
      ptx::named_bar(kBarCombine, kCombine);
      if (tid == 0) {
        const int mine = (int)(min(pair1, i1) - max(c.pair0, i0));
        int* tk = p.tickets + (size_t)c.b * p.hkv + c.kvh;
        const int before = atomicAdd(tk, mine);
        s_last = before + mine == c.ns;
        if (s_last) *tk = 0;  // every range has counted: the next launch starts at zero
      }
      ptx::named_bar(kBarCombine, kCombine);
      if (s_last) {
        __threadfence();
        for (int e = tid; e < GD; e += kCombine) {
          const int g = e / D, d = e % D;
          const size_t row0 = ((size_t)c.b * p.hq + c.kvh * G + g) * p.max_splits;
          float m = -INFINITY, dn = 0.f, ac = 0.f;
          for (int sp = 0; sp < c.ns; sp++)
            merge_step(m, dn, ac, __ldcg(p.part_ml + (row0 + sp) * 2), __ldcg(p.part_ml + (row0 + sp) * 2 + 1),
                       __ldcg(p.part_o + (row0 + sp) * D + d));
          p.out[(size_t)c.b * p.out_stride + (size_t)(c.kvh * G + g) * D + d] = f2bf(merge_final(dn, ac));
        }
      }
    }
  }
}

// the opt-in shared memory of the current device, and its SM count
struct DeviceInfo {
  int smem = 0, sms = 0;
};
DeviceInfo device_info() {
  static DeviceInfo info[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return DeviceInfo{};
  if (info[dev].sms == 0) {
    DeviceInfo d;
    cudaDeviceGetAttribute(&d.smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
    info[dev] = d;
  }
  return info[dev];
}

// K/V ring depth per consumer warp that fits the device (0 when fewer than two units fit)
int ring_depth(int B, int G, int D) {
  const DeviceInfo di = device_info();
  for (int ws = 4; ws >= 2; ws--)
    if (Layout::make(B, G, D, ws).total + kAlignSlack <= di.smem) return ws;
  return 0;
}

// ES_ATTN_PERSIST=1 turns the kernel on for the process (default off: at 64 sequences of 1K
// positions it measured level with the split kernel at splits of 512 and slower at 384 and 256);
// set_decode_persist changes it at run time (tests)
std::atomic<int>& mode() {
  static std::atomic<int> m{[] {
    const char* v = std::getenv("ES_ATTN_PERSIST");
    return v && v[0] == '1' ? 1 : 0;
  }()};
  return m;
}
bool enabled() { return mode().load(std::memory_order_relaxed) != 0; }

template <int D>
cudaError_t launch(const CUtensorMap& map, const Params& p, int smem, int grid, cudaStream_t stream) {
  static std::atomic<uint64_t> configured{0};
  cudaError_t e = once_per_device(configured, [] {
    // the opt-in maximum less the kernel's static words (the launches stay below it: ring_depth)
    return cudaFuncSetAttribute(decode_persist_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                device_info().smem - 64);
  });
  if (e != cudaSuccess) return e;
  return launch_ex(decode_persist_kernel<D>, dim3(grid), dim3(kThreads), (size_t)smem, stream, 0, map, p);
}

}  // namespace persist

int set_decode_persist(int on) { return persist::mode().exchange(on ? 1 : 0); }

bool decode_persist_supported(const DecodeArgs& a) {
  if (!persist::enabled()) return false;
  if (a.hkv <= 0 || a.hq % a.hkv != 0 || a.hq / a.hkv > 8 || a.part_tokens % 64 != 0 || a.max_splits <= 0)
    return false;
  if (a.d != 64 && a.d != 128) return false;
  if (a.block_size % 16 != 0 || a.tickets == nullptr) return false;
  if (a.s_kv != (int64_t)a.hkv * a.block_size * a.d || a.s_block != 2 * a.s_kv) return false;
  // the q rows go by bulk copy: 16-byte aligned rows and starts
  if (reinterpret_cast<uintptr_t>(a.q) % 16 != 0 || a.q_stride % 8 != 0) return false;
  if (a.B > 4096) return false;
  return persist::ring_depth(a.B, a.hq / a.hkv, a.d) >= 2;
}

cudaError_t launch_decode_persist_map(const DecodeArgs& a, const CUtensorMap& map, cudaStream_t stream) {
  if (!decode_persist_supported(a)) return cudaErrorInvalidValue;
  const int G = a.hq / a.hkv;
  persist::Params p{};
  p.q = static_cast<const __nv_bfloat16*>(a.q);
  p.q_stride = a.q_stride;
  p.block_tables = a.block_tables;
  p.bt_stride = a.bt_stride;
  p.ctx_lens = a.ctx_lens;
  p.part_o = a.part_o;
  p.part_ml = a.part_ml;
  p.tickets = a.tickets;
  p.out = static_cast<__nv_bfloat16*>(a.out);
  p.out_stride = a.out_stride;
  p.pf = static_cast<const uint8_t*>(a.prefetch);
  p.pf_bytes = a.prefetch_bytes;
  p.B = a.B;
  p.hq = a.hq;
  p.hkv = a.hkv;
  p.block_size = a.block_size;
  p.max_splits = a.max_splits;
  p.part_tokens = a.part_tokens;
  p.ws = persist::ring_depth(a.B, G, a.d);
  p.scale_log2 = a.scale * persist::kLog2e;
  p.status = a.status;
  const int smem = persist::Layout::make(a.B, G, a.d, p.ws).total + 1024;
  const int grid = std::max(1, persist::device_info().sms);
  if (a.d == 128) return persist::launch<128>(map, p, smem, grid, stream);
  return persist::launch<64>(map, p, smem, grid, stream);
}

cudaError_t launch_decode_persist(const DecodeArgs& a, cudaStream_t stream) {
  if (!decode_persist_supported(a)) return cudaErrorInvalidValue;
  // the layer's cache as rows of 64 elements (128 bytes); one box = 16 positions of one kv head
  const int64_t rows = a.num_blocks * 2 * a.hkv * a.block_size * (a.d / 64);
  CUtensorMap map;
  cudaError_t e = tmap::bf16_2d(&map, const_cast<void*>(a.cache), rows, 64, 64, 16 * (a.d / 64), 64);
  if (e != cudaSuccess) return e;
  return launch_decode_persist_map(a, map, stream);
}

}  // namespace es
