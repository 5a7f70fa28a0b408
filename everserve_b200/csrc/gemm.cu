// tcgen05 GEMM for the decoder's linear layers: out[M, N] = x[M, K] . w[N, K]^T (+ residual), bf16
// in, fp32 accumulate in TMEM, bf16 out.
//
// Design (sm_100a):
//   * swap-AB: the MMA's M side (128 TMEM lanes) runs over weight rows, its N side over tokens,
//     so a decode batch of 1..256 tokens is one MMA tile without padding the weights;
//   * one CTA = one 128-row weight slice x one token tile x one K split. Warp 0 lane 0 issues TMA
//     loads into a STAGES-deep ring of 128-byte-swizzled tiles, warp 1 lane 0 issues
//     tcgen05.mma into TMEM, warps 2-5 drain TMEM (tcgen05.ld) in the epilogue;
//   * split-K for the decode shapes, whose weight streaming needs every SM: the S CTAs that
//     share a tile form one thread-block cluster. Each writes its fp32 partial into its own
//     shared memory, a cluster barrier publishes them, and CTA j sums rows [j*128/S, ...) of the
//     tile over the S partials in rank order through distributed shared memory. No partial
//     touches global memory and no CTA polls;
//   * S depends on (N, K, #SMs) only, never on the token count, so a row's result is the same
//     whatever else is in the batch.
// Every mbarrier wait is bounded by the global timer; a wait that runs out writes a status word.
#include <cuda.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <unordered_map>

#include <unistd.h>  // environ

#include "api.h"
#include "comm.cuh"
#include "common.cuh"
#include "launch.h"
#include "ptx.cuh"
#include "tmap.h"

namespace es {
namespace gemm {

constexpr int BM = 128;  // weight rows per tile (MMA M)
constexpr int BK = 64;   // bf16 per k-block: one 128-byte swizzle row
constexpr int kThreads = 192;

// decode tiles (BN <= 64) run two CTAs per SM so one CTA's start-up and reduction overlap the
// other's streaming; larger tiles run one CTA per SM with a deeper ring
template <int BN, int CPS = (BN <= 64 ? 2 : 1)>
struct Cfg {
  static constexpr int kCps = CPS;
  static constexpr int kStages = CPS == 2 ? 4 : (BN <= 64 ? 8 : (BN == 128 ? 6 : 4));
  static constexpr int kABytes = BM * BK * 2;
  static constexpr int kBBytes = BN * BK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTmemCols = BN < 32 ? 32 : BN;
  static constexpr int kSmem = kStages * kStageBytes + 1024 + 256;
  static_assert(BN * BM * 4 <= kStages * kStageBytes, "the partial tile fits the drained ring");
};

struct Params {
  __nv_bfloat16* out;
  const __nv_bfloat16* residual;
  int* status;
  int M, N, ldo, ldr;
  int kb, splits;
  const float* scale;          // per row of x (token): multiplies the product (nullable)
  const __nv_bfloat16* pre;    // added to the (scaled) product before any reduction (nullable)
  int ldp;
  int two_shot;                // fused all-reduce as reduce-scatter to tile owners + all-gather
  const uint32_t* valid;       // grouped rows: valid[s] rows of segment s (rows [s*cap, (s+1)*cap)) are live
  int valid_cap, valid_segs;
  int silu;                    // rows gate/up interleaved by 64: out[m, N/2] = silu(gate) * up
  int rs_per;                  // fused reduce-scatter: member at position j keeps tokens [j*rs_per, (j+1)*rs_per)
  // fused all-gather: this member's ag_per token rows (ag_x, row stride ag_ldx) go to every member's
  // gather rows at its position; the GEMM's activations are those rows (K = ag_k)
  const __nv_bfloat16* ag_x;
  int ag_per, ag_ldx, ag_k;
  // weights pre-packed per (tile, k-block) as 16 KB blocks already in the swizzled shared-memory
  // layout (pack_weight): one bulk copy per stage reads them sequentially (nullable)
  const uint8_t* w_packed;
  // bytes the next kernel will read (its weights), fetched into L2 while this one runs (nullable)
  const uint8_t* pf;
  int64_t pf_bytes;
  RopeOut rope;  // the qkv projection's RoPE + paged-KV write epilogue when rope.q_out is set
  int ahead;     // weight k-blocks fetched into L2 beyond the ring (decode GEMMs), 0: none
};

// The fused all-gather's wait: every member's pushers have raised their flags for this call in this
// member's buffer. One thread; `pushers` flags per member, read together (independent loads). Bounded
// like every peer wait (abort word, the sender's heartbeat, the hard limit).
ES_DEVICE int wait_gather(const comm::View& cv, uint32_t parity, uint32_t seq, const int* order, int count,
                          int pushers) {
  const uint64_t base = cv.peers[cv.row];
  const uint64_t t0 = global_ns();
  for (int k = 0; k < count; k++) {
    const uint32_t* f = comm::ag_gemm_flag_ptr(base, parity, order[k], 0);
    comm::BeatWatch beat;
    uint32_t spins = 0;
    while (true) {
      uint32_t v[comm::kAGPushers];
#pragma unroll
      for (int i = 0; i < comm::kAGPushers; i++) v[i] = i < pushers ? ptx::ld_acquire_gpu(f + i) : seq;
      bool all = true;
#pragma unroll
      for (int i = 0; i < comm::kAGPushers; i++) all = all && v[i] == seq;
      if (all) break;
      if ((++spins & 63u) == 0) {
        volatile comm::Ctrl* c = cv.ctrl;
        if (c->abort) return kAborted;
        const uint64_t now = global_ns();
        if (beat.stopped(cv, order[k], now)) {
          c->late = c->late | (1u << order[k]);
          return kDead;
        }
        if (now - t0 > comm::kHardLimitNs) return kTimeout;
      }
    }
  }
  return kOk;
}

// A token tile [m0, m0 + BN) of a grouped GEMM holds a live row: some segment it overlaps has a
// count reaching into it. Tiles without one are skipped whole (their output rows are padding).
ES_DEVICE bool tile_live(const Params& p, int m0, int BN) {
  const int last = min(p.M, m0 + BN) - 1;
  for (int seg = m0 / p.valid_cap; seg <= last / p.valid_cap && seg < p.valid_segs; seg++) {
    const int lo = max(m0, seg * p.valid_cap) - seg * p.valid_cap;
    if (lo < (int)p.valid[seg]) return true;
  }
  return false;
}

// the product's epilogue terms before a reduction over members: acc * scale[m] + pre[m, n]
ES_DEVICE float pre_terms(const Params& p, float acc, size_t m, int n) {
  if (p.scale) acc *= p.scale[m];
  if (p.pre) acc += bf2f(p.pre[m * p.ldp + n]);
  return acc;
}

// The partials of a cluster at byte offset `off` of each CTA's partial tile, loaded, and their sum
// in rank order. Loads are issued for one element while the previous element is summed (software
// pipelined): a distributed-shared-memory load has a long latency, and with in-order issue an add
// right after each load would make every load wait for the one before it.
struct ClusterRow {
  float4 v[8];
};
ES_DEVICE void cluster_load(ClusterRow& r, uint32_t local, uint32_t off, int S) {
#pragma unroll
  for (int k = 0; k < 8; k++)
    if (k < S) r.v[k] = ptx::ld_cluster_v4(ptx::map_cluster(local + off, (uint32_t)k));
}
ES_DEVICE float4 cluster_total(const ClusterRow& r, int S) {
  float4 acc = r.v[0];
#pragma unroll
  for (int k = 1; k < 8; k++) {
    if (k < S) {
      acc.x += r.v[k].x;
      acc.y += r.v[k].y;
      acc.z += r.v[k].z;
      acc.w += r.v[k].w;
    }
  }
  return acc;
}
ES_DEVICE float4 cluster_sum(uint32_t local, uint32_t off, int S) {
  ClusterRow r;
  cluster_load(r, local, off, S);
  return cluster_total(r, S);
}

// kAR: the row-parallel variant whose epilogue sums the tile over the group's members (comm.cuh)
template <int BN, int CPS, bool kAR>
__global__ void __launch_bounds__(kThreads, CPS)
    gemm_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                const __grid_constant__ CUtensorMap tmap_x1, Params p, comm::View cv) {
  using C = Cfg<BN, CPS>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* a_tiles = smem;
  uint8_t* b_tiles = smem + C::kStages * C::kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kStages * C::kStageBytes);
  uint64_t* empty = full + C::kStages;
  uint64_t* done = empty + C::kStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  float* partial = reinterpret_cast<float*>(smem);  // [BN][BM] once the ring is drained
  __shared__ int s_fail;
  __shared__ uint32_t s_seq;
  __shared__ int s_order[comm::kMaxRows];
  __shared__ int s_count;
  __shared__ int s_pos;  // this member's position in the member order (reduce-scatter, all-gather)
  __shared__ uint32_t s_agseq;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * BM;
  const int m0 = blockIdx.y * BN;
  const int S = p.splits;
  const int split = blockIdx.z;
  const int kps = (p.kb + S - 1) / S;
  const int kb0 = split * kps;
  const int nkb = max(0, min(p.kb, kb0 + kps) - kb0);

  if (!kAR && p.valid != nullptr) {
    // the counts come from the kernel before; every CTA of a cluster shares the token tile, so a
    // skipped tile's cluster leaves together, before any barrier, TMEM allocation or copy
    pdl_wait();
    if (!tile_live(p, m0, BN)) return;
  }
  if (threadIdx.x == 0) {
    s_fail = 0;
    if (p.w_packed == nullptr) ptx::prefetch_tmap(&tmap_w);
    ptx::prefetch_tmap(&tmap_x);
    for (int s = 0; s < C::kStages; s++) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], 1);
    }
    ptx::mbar_init(done, 1);
    ptx::fence_mbar_init();
  }
  if (warp == 1) ptx::tmem_alloc(tmem_slot, C::kTmemCols);
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const bool producer = warp == 0 && lane == 0;
  if (!producer) {
    pdl_wait();  // everything below reads what the previous kernel wrote, or writes global memory
    pdl_launch();
  }
  if ((kAR || p.ag_per) && threadIdx.x == 64) {
    const int cnt = cv.order[0];
    s_count = cnt < 0 ? 0 : (cnt > comm::kMaxRows ? comm::kMaxRows : cnt);
    s_pos = -1;
    for (int i = 0; i < s_count; i++) {
      s_order[i] = cv.order[1 + i];
      if (s_order[i] == cv.row) s_pos = i;
    }
    if (p.ag_per) s_agseq = cv.seqs[comm::kAGSeqSlot] + 1;
  }
  const int n_ctas = (int)(gridDim.x * gridDim.y * gridDim.z);
  const int pushers = min(comm::kAGPushers, n_ctas);
  if (p.ag_per) {
    __syncthreads();  // the order, position and call number above
    // the first CTAs push this member's rows to every member (its rows at its position), then
    // raise their flag there; every CTA's producer waits for all of them before its activations
    const int lin = (int)(blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z));
    if (lin < pushers && threadIdx.x >= 64 && s_pos >= 0) {
      const uint32_t parity = s_agseq & 1u;
      const int vrow = p.ag_k / 8;  // 16-byte vectors per row
      const int total_v = p.ag_per * vrow;
      const int v0 = (int)((long long)total_v * lin / pushers), v1 = (int)((long long)total_v * (lin + 1) / pushers);
      for (int k = 0; k < s_count; k++) {
        char* dst = comm::ag_gemm_ptr(cv.peers[s_order[k]], parity) + (size_t)s_pos * p.ag_per * p.ag_k * 2;
        for (int i = v0 + (int)threadIdx.x - 64; i < v1; i += kThreads - 64) {
          const int r = i / vrow, c = i % vrow;
          reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(p.ag_x + (size_t)r * p.ag_ldx)[c];
        }
      }
      __threadfence_system();
      ptx::named_bar(2, kThreads - 64);
      if (threadIdx.x == 64)
        for (int k = 0; k < s_count; k++)
          st_release_sys(comm::ag_gemm_flag_ptr(cv.peers[s_order[k]], parity, cv.row, lin), s_agseq);
    }
  }

  if (producer) {
    // Every CTA reads the same small activation matrix: walking the k-blocks from the same start,
    // the CTAs of all weight tiles would ask the same L2 lines for the same block at once. Each
    // tile starts its walk at its own offset instead (a fixed order per tile, so a row's sum does
    // not depend on the batch).
    const int rot = nkb > 0 ? (int)(blockIdx.x % (unsigned)nkb) : 0;
    auto kblk = [&](int i) { return kb0 + (i + rot) % nkb; };
    // the weight tiles of the first stages depend on no kernel of the step: stream them while the
    // previous kernel finishes, then the activation tiles once it has
    const int pre = min(nkb, C::kStages);
    // a decode GEMM (one token tile) reads each weight byte once: mark its lines first to go, so
    // streaming them does not evict what is kept in L2 for later kernels
    const bool once = gridDim.y == 1;
    const uint64_t pol = ptx::policy_evict_first();
    auto load_w = [&](int stage, int kb) {
      uint8_t* dst = a_tiles + stage * C::kABytes;
      if (p.w_packed) {
        const uint8_t* src = p.w_packed + ((size_t)blockIdx.x * p.kb + kb) * C::kABytes;
        if (once) ptx::bulk_g2s_hint(dst, src, C::kABytes, &full[stage], pol);
        else ptx::bulk_g2s(dst, src, C::kABytes, &full[stage]);
      } else if (once) {
        ptx::tma_load_2d_hint(dst, &tmap_w, kb * BK, n0, &full[stage], pol);
      } else {
        ptx::tma_load_2d(dst, &tmap_w, kb * BK, n0, &full[stage]);
      }
    };
    // beyond the ring, the next `ahead` weight k-blocks are fetched into L2, so more of the
    // stream is in flight from DRAM than the ring's shared memory holds
    auto ahead_w = [&](int i) {
      if (!once || i >= nkb) return;
      const int kb = kblk(i);
      if (p.w_packed) ptx::l2_prefetch(p.w_packed + ((size_t)blockIdx.x * p.kb + kb) * C::kABytes, C::kABytes);
      else ptx::tma_prefetch_2d(&tmap_w, kb * BK, n0);
    };
    for (int i = 0; i < pre; i++) {
      ptx::mbar_arrive_expect_tx(&full[i], C::kStageBytes);
      load_w(i, kblk(i));
    }
    for (int i = pre; i < pre + p.ahead; i++) ahead_w(i);
    ptx::l2_prefetch_share(p.pf, p.pf_bytes, (int)(blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z)),
                           (int)(gridDim.x * gridDim.y * gridDim.z));
    pdl_wait();
    pdl_launch();
    const CUtensorMap* xmap = &tmap_x;
    if (p.ag_per) {
      // the gathered rows of this call's parity, once every member's pushers have landed them
      const int r = wait_gather(cv, s_agseq & 1u, s_agseq, s_order, s_count, pushers);
      if (r != kOk) {
        s_fail = r;
        volatile comm::Ctrl* cw = cv.ctrl;
        cw->status = (uint32_t)r;
      }
      if (s_agseq & 1u) xmap = &tmap_x1;
    }
    for (int i = 0; i < pre; i++) ptx::tma_load_2d(b_tiles + i * C::kBBytes, xmap, kblk(i) * BK, m0, &full[i]);
    for (int i = pre; i < nkb; i++) {
      const int s = i % C::kStages;
      if (i >= C::kStages && !ptx::mbar_wait(&empty[s], ((i / C::kStages) - 1) & 1)) {
        s_fail = 1;
        break;
      }
      ptx::mbar_arrive_expect_tx(&full[s], C::kStageBytes);
      const int kx = kblk(i) * BK;
      load_w(s, kblk(i));
      ahead_w(i + p.ahead);
      ptx::tma_load_2d(b_tiles + s * C::kBBytes, xmap, kx, m0, &full[s]);
    }
  } else if (warp == 1 && lane == 0) {
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
      for (int kk = 0; kk < BK / 16; kk++)
        ptx::mma_f16_ss(tmem, ad + 2 * kk, bd + 2 * kk, idesc, (i > 0 || kk > 0) ? 1u : 0u);
      ptx::mma_commit(&empty[s]);
    }
    ptx::mma_commit(done);  // always arrives, so the epilogue never waits for nothing
  }
  __syncwarp();

  const int mrem = p.M - m0;
  if (warp >= 2) {
    const int q = warp & 3;  // TMEM lane quadrant of this warp
    const int r = q * 32 + lane;
    const int n = n0 + r;
    if (!ptx::mbar_wait(done, 0)) s_fail = 1;
    ptx::tc_fence_after();
    const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16);
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 16) {
      float v[16];
      ptx::tmem_ld16(taddr + c0, v);
      if (nkb == 0) {
#pragma unroll
        for (int j = 0; j < 16; j++) v[j] = 0.f;
      }
      if (S > 1 || kAR || p.silu || p.rope.q_out) {
        // the ring is drained (all MMAs completed before `done`), so its smem holds the partial
#pragma unroll
        for (int j = 0; j < 16; j++) partial[(c0 + j) * BM + r] = v[j];
      } else if (n < p.N) {
#pragma unroll
        for (int j = 0; j < 16; j++) {
          if (c0 + j < mrem) {
            const size_t m = (size_t)(m0 + c0 + j);
            float o = pre_terms(p, v[j], m, n);
            if (p.residual) o += bf2f(p.residual[m * p.ldr + n]);
            p.out[m * p.ldo + n] = f2bf(o);
          }
        }
      }
    }
  }
  if (S > 1 || kAR || p.silu || p.rope.q_out) {
    // publish the partials to the cluster, then reduce this CTA's row slice over all of them
    ptx::cluster_sync();
    const uint32_t rank = ptx::cluster_rank();
    const int rows = ((BM / S) + 3) & ~3;
    const int r0 = min(BM, (int)rank * rows);
    const int r1 = (int)rank + 1 == S ? BM : min(BM, r0 + rows);
    const int span4 = (r1 - r0) >> 2;
    const int mcount = min(BN, mrem);
    const int total = span4 * mcount;
    const uint32_t local = ptx::smem_u32(partial);
    if (kAR) {
      // One call number per output tile, shared by the cluster's CTAs: every word of the tile in
      // this call carries it, and consecutive calls of any fused GEMM over the tile alternate its
      // parity half. (A number per cluster rank would not: two GEMMs with different splits give a
      // word to different ranks, and a member one kernel ahead could overwrite words a slower
      // member still polls.) Rank 0 advances it after the last cluster barrier, once every CTA of
      // the cluster has read it; every member makes the same calls, so the numbers agree.
      if (threadIdx.x == 0) s_seq = cv.seqs[blockIdx.x] + 1;
      __syncthreads();
    }
    const uint32_t seq = kAR ? s_seq : 0u, parity = seq & 1u;
    if (!kAR && p.silu) {
      // SiLU-mul epilogue: this rank sums gate rows [g0, g1) of the tile and their up rows 64
      // further over the partials (rank order, as the plain reduction), rounds both to bf16 as the
      // plain GEMM's output would be, and applies the SiLU-mul kernel's arithmetic
      const int rows64 = ((64 / S) + 3) & ~3;
      const int g0 = min(64, (int)rank * rows64);
      const int g1 = (int)rank + 1 == S ? 64 : min(64, g0 + rows64);
      const int gspan4 = (g1 - g0) >> 2;
      for (int e = threadIdx.x; e < gspan4 * mcount; e += kThreads) {
        const int col = e / gspan4, row = g0 + (e % gspan4) * 4;
        const uint32_t offg = (uint32_t)((col * BM + row) * 4), offu = offg + 64 * 4;
        const float4 g = cluster_sum(local, offg, S);
        const float4 u = cluster_sum(local, offu, S);
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
    if (!kAR && p.rope.q_out) {
      // RoPE + KV-write epilogue: tile = one head of 128 dims (q heads, then k, then v). This rank
      // sums dims [g0, g1) of the first half and their partners 64 further (rank order), rounds
      // them to bf16 as the qkv output would be, rotates q and k by the token's position and
      // writes q to q_out and k, v to the token's cache slot (the rope_kv_write arithmetic)
      const RopeOut& R = p.rope;
      const int head = blockIdx.x;
      const int rows64 = ((64 / S) + 3) & ~3;
      const int g0 = min(64, (int)rank * rows64);
      const int g1 = (int)rank + 1 == S ? 64 : min(64, g0 + rows64);
      const int gspan4 = (g1 - g0) >> 2;
      for (int e = threadIdx.x; e < gspan4 * mcount; e += kThreads) {
        const int col = e / gspan4, i = g0 + (e % gspan4) * 4;
        const uint32_t off_a = (uint32_t)((col * BM + i) * 4), off_b = off_a + 64 * 4;
        const float4 fa = cluster_sum(local, off_a, S);
        const float4 fb = cluster_sum(local, off_b, S);
        const float av[4] = {fa.x, fa.y, fa.z, fa.w}, bv[4] = {fb.x, fb.y, fb.z, fb.w};
        const size_t m = (size_t)(m0 + col);
        float ra[4], rb[4];
        if (head < R.hq + R.hkv) {
          const float* cs = R.cos_sin + R.positions[m] * 128;
#pragma unroll
          for (int z = 0; z < 4; z++) {
            const float a = bf2f(f2bf(av[z])), b = bf2f(f2bf(bv[z]));
            const float c = cs[i + z], sn = cs[64 + i + z];
            ra[z] = a * c - b * sn;
            rb[z] = b * c + a * sn;
          }
        } else {
#pragma unroll
          for (int z = 0; z < 4; z++) {
            ra[z] = av[z];
            rb[z] = bv[z];
          }
        }
        const uint2 wa = make_uint2(ptx::pack_bf16x2(ra[0], ra[1]), ptx::pack_bf16x2(ra[2], ra[3]));
        const uint2 wb = make_uint2(ptx::pack_bf16x2(rb[0], rb[1]), ptx::pack_bf16x2(rb[2], rb[3]));
        __nv_bfloat16* dst;
        if (head < R.hq) {
          dst = static_cast<__nv_bfloat16*>(R.q_out) + m * (size_t)R.hq * 128 + (size_t)head * 128;
        } else {
          const int64_t slot = R.slots[m];
          if (slot < 0) continue;
          const int64_t blk = slot / R.block_size, off = slot % R.block_size;
          dst = static_cast<__nv_bfloat16*>(R.cache) + blk * R.s_block + off * R.s_off +
                (head < R.hq + R.hkv ? (int64_t)(head - R.hq) * R.s_head
                                     : R.s_kv + (int64_t)(head - R.hq - R.hkv) * R.s_head);
        }
        *reinterpret_cast<uint2*>(dst + i) = wa;
        *reinterpret_cast<uint2*>(dst + i + 64) = wb;
      }
    }
    const int ptotal = (p.silu || p.rope.q_out) ? 0 : total;
    ClusterRow cur, nxt;
    if ((int)threadIdx.x < ptotal) {
      const int e = threadIdx.x;
      cluster_load(cur, local, (uint32_t)(((e / span4) * BM + r0 + (e % span4) * 4) * 4), S);
    }
    for (int e = threadIdx.x; e < ptotal; e += kThreads) {
      const int col = e / span4, row = r0 + (e % span4) * 4;
      const int en = e + kThreads;
      if (en < ptotal) cluster_load(nxt, local, (uint32_t)(((en / span4) * BM + r0 + (en % span4) * 4) * 4), S);
      float4 acc = cluster_total(cur, S);
      cur = nxt;
      if (p.scale || p.pre) {
        const size_t mm = (size_t)(m0 + col);
        const int nn = n0 + row;
        acc.x = pre_terms(p, acc.x, mm, min(nn, p.N - 1));
        acc.y = pre_terms(p, acc.y, mm, min(nn + 1, p.N - 1));
        acc.z = pre_terms(p, acc.z, mm, min(nn + 2, p.N - 1));
        acc.w = pre_terms(p, acc.w, mm, min(nn + 3, p.N - 1));
      }
      if (kAR) {
        // this member's bf16 partial (what an unfused GEMM would output) as two LL words, to every
        // member: each word carries the call number, so it is its own arrival flag
        const size_t widx = ((size_t)(blockIdx.x * BN + col) * BM + row) / 2;
        const uint64_t w0 = ((uint64_t)seq << 32) | ptx::pack_bf16x2(acc.x, acc.y);
        const uint64_t w1 = ((uint64_t)seq << 32) | ptx::pack_bf16x2(acc.z, acc.w);
        if (p.rs_per) {
          // reduce-scatter by tokens: the words of token `col` go to the member keeping it only
          const int op = col / p.rs_per;
          if (op < s_count) {
            uint64_t* d = comm::ll_gemm_ptr(cv.peers[s_order[op]], parity, cv.row) + widx;
            comm::st_u64_relaxed(d, w0);
            comm::st_u64_relaxed(d + 1, w1);
          }
        } else if (p.two_shot) {
          // reduce-scatter: only the tile's owner takes the partials (1/count of the words a
          // one-shot push sends)
          uint64_t* d = comm::ll_gemm_ptr(cv.peers[s_order[blockIdx.x % s_count]], parity, cv.row) + widx;
          comm::st_u64_relaxed(d, w0);
          comm::st_u64_relaxed(d + 1, w1);
        } else if (cv.mc) {
          uint64_t* d = comm::ll_gemm_ptr(cv.mc, parity, cv.row) + widx;
          comm::mc_st_u64(d, w0);
          comm::mc_st_u64(d + 1, w1);
        } else {
          for (int k = 0; k < s_count; k++) {
            uint64_t* d = comm::ll_gemm_ptr(cv.peers[s_order[k]], parity, cv.row) + widx;
            comm::st_u64_relaxed(d, w0);
            comm::st_u64_relaxed(d + 1, w1);
          }
        }
        continue;
      }
      const size_t m = (size_t)(m0 + col);
      float o[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
      for (int z = 0; z < 4; z++) {
        const int n = n0 + row + z;
        if (n < p.N) {
          if (p.residual) o[z] += bf2f(p.residual[m * p.ldr + n]);
          p.out[m * p.ldo + n] = f2bf(o[z]);
        }
      }
    }
    if (kAR) {
      // sum every member's words in member order (polling the words themselves). Two-shot: only
      // the tile's owner sums, then pushes the sums to the others, who poll for them instead.
      const uint64_t my_base = cv.peers[cv.row];
      const int owner_row = s_count > 0 ? s_order[blockIdx.x % s_count] : cv.row;
      const bool owner = p.rs_per || !p.two_shot || owner_row == cv.row;
      uint64_t t0 = 0;
      bool named = false;
      uint32_t spins = 0;
      int fail = kOk;
      for (int e = threadIdx.x; e < total && fail == kOk; e += kThreads) {
        const int col = e / span4, row = r0 + (e % span4) * 4;
        if (p.rs_per && col / p.rs_per != s_pos) continue;  // another member keeps this token
        const size_t widx = ((size_t)(blockIdx.x * BN + col) * BM + row) / 2;
        float o[4] = {0.f, 0.f, 0.f, 0.f};
        if (!owner) {
          const uint64_t* src = comm::ll_res_ptr(my_base, parity) + widx;
          const uint32_t a = comm::ll_wait(cv, src, seq, owner_row, t0, named, spins, fail);
          const uint32_t b = comm::ll_wait(cv, src + 1, seq, owner_row, t0, named, spins, fail);
          if (fail != kOk) break;
          const float2 lo = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&a));
          const float2 hi = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&b));
          o[0] = lo.x;
          o[1] = lo.y;
          o[2] = hi.x;
          o[3] = hi.y;
        }
        for (int k = 0; owner && k < s_count && fail == kOk; k++) {
          const uint64_t* src = comm::ll_gemm_ptr(my_base, parity, s_order[k]) + widx;
          const uint32_t a = comm::ll_wait(cv, src, seq, s_order[k], t0, named, spins, fail);
          const uint32_t b = comm::ll_wait(cv, src + 1, seq, s_order[k], t0, named, spins, fail);
          const float2 lo = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&a));
          const float2 hi = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&b));
          o[0] += lo.x;
          o[1] += lo.y;
          o[2] += hi.x;
          o[3] += hi.y;
        }
        if (fail != kOk) break;
        if (p.two_shot && !p.rs_per && owner) {
          // all-gather: the reduced words (rounded to bf16 once, as every member will use them)
          const uint64_t r0w = ((uint64_t)seq << 32) | ptx::pack_bf16x2(o[0], o[1]);
          const uint64_t r1w = ((uint64_t)seq << 32) | ptx::pack_bf16x2(o[2], o[3]);
          for (int k = 0; k < s_count; k++) {
            if (s_order[k] == cv.row) continue;
            uint64_t* d = comm::ll_res_ptr(cv.peers[s_order[k]], parity) + widx;
            comm::st_u64_relaxed(d, r0w);
            comm::st_u64_relaxed(d + 1, r1w);
          }
          const float2 lo = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&r0w));
          const float2 hi = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&r1w));
          o[0] = lo.x;  // the owner uses the same rounded sums as everyone else
          o[1] = lo.y;
          o[2] = hi.x;
          o[3] = hi.y;
        }
        // reduce-scatter: this member's slice starts at its first token (out and residual rows)
        const size_t m = (size_t)(m0 + col - (p.rs_per ? s_pos * p.rs_per : 0));
#pragma unroll
        for (int z = 0; z < 4; z++) {
          const int n = n0 + row + z;
          if (n < p.N) {
            if (p.residual) o[z] += bf2f(p.residual[m * p.ldr + n]);
            p.out[m * p.ldo + n] = f2bf(o[z]);
          }
        }
      }
      if (fail != kOk) {
        s_fail = fail;
        volatile comm::Ctrl* cw = cv.ctrl;
        cw->status = (uint32_t)fail;
      }
    }
    ptx::cluster_sync();  // no CTA leaves while another still reads its shared memory
    if (kAR && rank == 0 && threadIdx.x == 0) cv.seqs[blockIdx.x] = s_seq;
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) ptx::tmem_dealloc(tmem, C::kTmemCols);
  if (threadIdx.x == 0) {
    if (s_fail && p.status)
      atomicExch(p.status, (s_fail == kAborted || s_fail == kDead) ? s_fail : (int)kTimeout);
    if (p.ag_per) {
      // the last CTA of the call advances the gathering GEMM's call number (every CTA has read it)
      __threadfence();
      if (atomicAdd(cv.seqs + comm::kAGDoneSlot, 1u) == (uint32_t)n_ctas - 1) {
        cv.seqs[comm::kAGDoneSlot] = 0;
        __threadfence();
        ptx::st_release_gpu(cv.seqs + comm::kAGSeqSlot, s_agseq);
      }
    }
  }
}

template <int BN, int CPS = (BN <= 64 ? 2 : 1), bool kAR = false>
cudaError_t launch(const CUtensorMap& mw, const CUtensorMap& mx, const Params& p, dim3 grid, cudaStream_t stream,
                   const comm::View& cv = comm::View{}, const CUtensorMap* mx_odd = nullptr) {
  const CUtensorMap& mx1 = mx_odd ? *mx_odd : mx;  // the gathered rows of odd calls (all-gather GEMM)
  using C = Cfg<BN, CPS>;
  static std::atomic<uint64_t> configured{0};
  cudaError_t e = once_per_device(configured, [] {
    cudaError_t r =
        cudaFuncSetAttribute(gemm_kernel<BN, CPS, kAR>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
    if (r != cudaSuccess) return r;
    return cudaFuncSetAttribute(gemm_kernel<BN, CPS, kAR>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  });
  if (e != cudaSuccess) return e;
  return launch_ex(gemm_kernel<BN, CPS, kAR>, grid, dim3(kThreads), C::kSmem, stream, p.splits, mw, mx, mx1, p, cv);
}

// The largest split whose clusters all fit on the device at once (the fused all-reduce waits on
// peers, so every CTA of the grid must be resident together).
template <int BN, int CPS>
int resident_split(int tiles, int want) {
  using C = Cfg<BN, CPS>;
  cudaError_t e =
      cudaFuncSetAttribute(gemm_kernel<BN, CPS, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
  if (e != cudaSuccess) return 0;
  e = cudaFuncSetAttribute(gemm_kernel<BN, CPS, true>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (e != cudaSuccess) return 0;
  for (int s = want; s >= 1; s--) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(tiles, 1, s);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = C::kSmem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, gemm_kernel<BN, CPS, true>, &cfg) != cudaSuccess) {
      cudaGetLastError();
      continue;
    }
    if (clusters >= tiles) return s;
  }
  return 0;
}

}  // namespace gemm

int64_t gemm_pick_bn(int64_t M) {
  if (M <= 16) return 16;
  if (M <= 32) return 32;
  if (M <= 64) return 64;
  if (M <= 128) return 128;
  return 256;
}

// Cluster split for an N x K weight at decode sizes: as many CTAs per tile as the SM slots allow,
// at most 8 (the portable cluster size), each with at least 16 k-blocks (each CTA pays a fixed
// start-up and reduction cost, so fewer longer CTAs stream faster: measured on B200, the 6144 x
// 4096 projection takes 18 us at 4 splits against 25 us at 6), relaxed to 8 and then 4 k-blocks
// when that would leave fewer CTAs than half the SMs. A function of (N, K, #SMs) only.
static int64_t split_for(int64_t tiles, int64_t kb, int64_t slots, int64_t num_sms) {
  int64_t s = 1;
  for (int64_t min_kb : {16, 8, 4}) {
    s = std::max<int64_t>(1, slots / tiles);
    s = std::min<int64_t>(s, 8);  // portable cluster size: a cluster of 16 needs 16 free SMs in one GPC
    s = std::min<int64_t>(s, std::max<int64_t>(1, kb / min_kb));
    if (tiles * s >= num_sms / 2) break;
  }
  while (s > 1 && (kb + s - 1) / s * (s - 1) >= kb) s--;  // every split holds k-blocks
  return s;
}

void gemm_plan(int64_t M, int64_t N, int64_t K, int64_t num_sms, int* splits, int* cps) {
  // tuning overrides for measurements, decode sizes: ES_GEMM_PLAN_<N>x<K>="<splits>,<ctas per SM>"
  // for one weight shape, ES_GEMM_PLAN for every shape
  static const bool any_forced = [] {  // read the environment per launch only when it has any
    for (char** e = environ; e != nullptr && *e != nullptr; e++)
      if (std::strncmp(*e, "ES_GEMM_PLAN", 12) == 0) return true;
    return false;
  }();
  if (any_forced && M <= 64) {
    char name[64];
    snprintf(name, sizeof(name), "ES_GEMM_PLAN_%lldx%lld", (long long)N, (long long)K);
    const char* forced = std::getenv(name);
    if (forced == nullptr) forced = std::getenv("ES_GEMM_PLAN");
    int s = 0, c = 0;
    if (forced != nullptr && sscanf(forced, "%d,%d", &s, &c) == 2 && s >= 1 && s <= 8 && (c == 1 || c == 2)) {
      *splits = s;
      *cps = c;
      return;
    }
  }
  if (M > 64) {
    *splits = 1;
    *cps = 1;
    return;
  }
  const int64_t tiles = (N + gemm::BM - 1) / gemm::BM;
  const int64_t kb = (K + gemm::BK - 1) / gemm::BK;
  const int64_t s1 = split_for(tiles, kb, num_sms, num_sms), s2 = split_for(tiles, kb, 2 * num_sms, num_sms);
  if (s1 >= 4 || (s1 == s2 && tiles <= num_sms)) {
    *splits = (int)s1;
    *cps = 1;
  } else {
    *splits = (int)s2;
    *cps = 2;
  }
}

int64_t gemm_pick_splits(int64_t M, int64_t N, int64_t K, int64_t num_sms) {
  int s, c;
  gemm_plan(M, N, K, num_sms, &s, &c);
  return s;
}

int64_t gemm_ws_floats(int64_t num_sms) { return gemm_sk_ws_floats(num_sms); }
int64_t gemm_sync_words(int64_t num_sms) { return gemm_sk_sync_words(num_sms); }

// Decode-size plain GEMMs with several waves of weight tiles (the vocabulary projection: 1002 tiles
// on 296 CTA slots, a last wave 40 % full) take the stream-K kernel (gemm_stream.cu), about 5 %
// faster there; the others stay on the cluster split-K kernel below, which is as fast or faster on
// the shapes measured. ES_GEMM_STREAM=1 sends every decode-size plain GEMM to stream-K.
static bool stream_k_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("ES_GEMM_STREAM");
    return v && v[0] == '1';
  }();
  return on;
}

// Weight k-blocks a decode GEMM fetches into L2 ahead of its ring (ES_GEMM_L2AHEAD; default 0:
// two, four and eight blocks ahead measured no faster in the decode step)
static int l2_ahead() {
  static const int v = [] {
    const char* e = std::getenv("ES_GEMM_L2AHEAD");
    const int x = e ? std::atoi(e) : 0;
    return x < 0 ? 0 : (x > 16 ? 16 : x);
  }();
  return v;
}

// The weight's operand: a tensor map of the row-major weight, or (pre-packed weight) nothing, the
// kernel reading the packed blocks by bulk copies. Checks the alignment either needs.
static cudaError_t weight_map(const GemmArgs& a, CUtensorMap* mw) {
  if (a.w_packed != nullptr) {
    if (reinterpret_cast<uintptr_t>(a.w_packed) % 16 != 0) return cudaErrorInvalidValue;
    std::memset(mw, 0, sizeof(*mw));
    return cudaSuccess;
  }
  if ((a.ldw * 2) % 16 != 0 || reinterpret_cast<uintptr_t>(a.w) % 16 != 0) return cudaErrorInvalidValue;
  return tmap::bf16_2d(mw, const_cast<void*>(a.w), a.N, a.K, a.ldw, gemm::BM, gemm::BK);
}

cudaError_t launch_gemm_bf16(const GemmArgs& a, cudaStream_t stream) {
  if (a.M == 0 || a.N == 0) return cudaSuccess;
  const int64_t n_tiles = (a.N + gemm::BM - 1) / gemm::BM;
  if (a.M <= 64 && a.valid == nullptr && a.ws != nullptr && a.sync != nullptr && a.w_packed == nullptr &&
      a.rope == nullptr && (stream_k_enabled() || n_tiles > 4 * (int64_t)a.num_sms))
    return launch_gemm_stream(a, a.silu != 0, stream);
  if (a.silu && (a.N % gemm::BM != 0 || a.residual != nullptr || a.scale != nullptr || a.pre != nullptr ||
                 a.valid != nullptr))
    return cudaErrorInvalidValue;
  if (a.K % 8 != 0 || (a.ldx * 2) % 16 != 0) return cudaErrorInvalidValue;
  if (reinterpret_cast<uintptr_t>(a.x) % 16 != 0) return cudaErrorInvalidValue;
  const int BN = (int)gemm_pick_bn(a.M);
  gemm::Params p{};
  p.out = static_cast<__nv_bfloat16*>(a.out);
  p.residual = static_cast<const __nv_bfloat16*>(a.residual);
  p.status = a.status;
  p.M = (int)a.M;
  p.N = (int)a.N;
  p.ldo = (int)a.ldo;
  p.ldr = (int)a.ldr;
  p.kb = (int)((a.K + gemm::BK - 1) / gemm::BK);
  p.scale = a.scale;
  p.pre = static_cast<const __nv_bfloat16*>(a.pre);
  p.ldp = (int)a.ldp;
  p.silu = a.silu;
  p.w_packed = static_cast<const uint8_t*>(a.w_packed);
  p.pf = static_cast<const uint8_t*>(a.prefetch);
  p.pf_bytes = a.prefetch_bytes;
  p.ahead = l2_ahead();
  if (a.rope != nullptr) {
    const RopeOut& R = *a.rope;
    if (a.N != (int64_t)(R.hq + 2 * R.hkv) * 128 || a.silu || a.residual != nullptr || a.scale != nullptr ||
        a.pre != nullptr || a.valid != nullptr || R.q_out == nullptr || R.cache == nullptr || R.block_size <= 0 ||
        reinterpret_cast<uintptr_t>(R.q_out) % 8 != 0 || reinterpret_cast<uintptr_t>(R.cache) % 8 != 0 ||
        R.s_off % 4 != 0 || R.s_head % 4 != 0 || R.s_kv % 4 != 0 || R.s_block % 4 != 0)
      return cudaErrorInvalidValue;
    p.rope = R;
  }
  if (a.valid != nullptr) {
    if (a.valid_cap <= 0 || a.valid_segs <= 0 || a.valid_cap * a.valid_segs < a.M) return cudaErrorInvalidValue;
    p.valid = a.valid;
    p.valid_cap = (int)a.valid_cap;
    p.valid_segs = a.valid_segs;
  }
  int cps = 1;
  gemm_plan(a.M, a.N, a.K, a.num_sms, &p.splits, &cps);
  const unsigned tiles_n = (unsigned)((a.N + gemm::BM - 1) / gemm::BM);
  const unsigned tiles_m = (unsigned)((a.M + BN - 1) / BN);
  if (tiles_m > 65535) return cudaErrorInvalidValue;
  dim3 grid(tiles_n, tiles_m, (unsigned)p.splits);
  CUtensorMap mw, mx;
  cudaError_t e = weight_map(a, &mw);
  if (e != cudaSuccess) return e;
  e = tmap::bf16_2d(&mx, const_cast<void*>(a.x), a.M, a.K, a.ldx, BN, gemm::BK);
  if (e != cudaSuccess) return e;
  switch (BN) {
    case 16: return cps == 1 ? gemm::launch<16, 1>(mw, mx, p, grid, stream) : gemm::launch<16, 2>(mw, mx, p, grid, stream);
    case 32: return cps == 1 ? gemm::launch<32, 1>(mw, mx, p, grid, stream) : gemm::launch<32, 2>(mw, mx, p, grid, stream);
    case 64: return cps == 1 ? gemm::launch<64, 1>(mw, mx, p, grid, stream) : gemm::launch<64, 2>(mw, mx, p, grid, stream);
    case 128: return gemm::launch<128>(mw, mx, p, grid, stream);
    default: return gemm::launch<256>(mw, mx, p, grid, stream);
  }
}

}  // namespace es

namespace es {

cudaError_t launch_gemm_allreduce(const GemmArgs& a, const CommArgs& c, cudaStream_t stream) {
  if (a.M == 0 || a.N == 0) return cudaSuccess;
  if (a.M > 64 || a.K % 8 != 0 || (a.ldx * 2) % 16 != 0) return cudaErrorInvalidValue;
  if (reinterpret_cast<uintptr_t>(a.x) % 16 != 0) return cudaErrorInvalidValue;
  constexpr int BN = 64;  // one token tile for every decode batch: the plan never depends on M
  const int tiles = (int)((a.N + gemm::BM - 1) / gemm::BM);
  if ((size_t)tiles * BN * gemm::BM * 4 > comm::kLLGemmBytes || c.seqs == nullptr) return cudaErrorInvalidValue;
  gemm::Params p{};
  p.out = static_cast<__nv_bfloat16*>(a.out);
  p.residual = static_cast<const __nv_bfloat16*>(a.residual);
  p.status = a.status;
  p.M = (int)a.M;
  p.N = (int)a.N;
  p.ldo = (int)a.ldo;
  p.ldr = (int)a.ldr;
  p.kb = (int)((a.K + gemm::BK - 1) / gemm::BK);
  p.scale = a.scale;
  p.w_packed = static_cast<const uint8_t*>(a.w_packed);
  p.pf = static_cast<const uint8_t*>(a.prefetch);
  p.pf_bytes = a.prefetch_bytes;
  p.ahead = l2_ahead();
  p.pre = static_cast<const __nv_bfloat16*>(a.pre);
  p.ldp = (int)a.ldp;
  p.two_shot = c.mc ? 0 : a.two_shot;  // the multicast variant pushes once already
  p.rs_per = (int)a.rs_per;
  if (a.rs_per < 0 || (a.rs_per > 0 && c.mc)) return cudaErrorInvalidValue;  // reduce-scatter pushes to one member
  int cps = 1;
  gemm_plan(BN, a.N, a.K, a.num_sms, &p.splits, &cps);
  // every CTA waits on peers: the whole grid must be resident at once
  static std::mutex mu;
  static std::unordered_map<long long, int> fit;
  const long long key = ((long long)tiles << 20) | ((long long)p.splits << 4) | cps;
  int s_fit;
  {
    std::lock_guard<std::mutex> g(mu);
    auto it = fit.find(key);
    if (it == fit.end()) {
      s_fit = cps == 1 ? gemm::resident_split<BN, 1>(tiles, p.splits) : gemm::resident_split<BN, 2>(tiles, p.splits);
      fit.emplace(key, s_fit);
    } else {
      s_fit = it->second;
    }
  }
  if (s_fit <= 0) return cudaErrorInvalidConfiguration;
  p.splits = s_fit;
  if (tiles > comm::kAGDoneSlot) return cudaErrorInvalidValue;  // per-tile call numbers below the gather's
  comm::View v{};
  v.seqs = c.seqs;
  v.peers = c.peers;
  v.mc = c.mc;
  v.order = c.order;
  v.call = c.call;
  v.ctrl = reinterpret_cast<comm::Ctrl*>(c.ctrl);
  v.row = c.row;
  CUtensorMap mw, mx;
  cudaError_t e = weight_map(a, &mw);
  if (e != cudaSuccess) return e;
  e = tmap::bf16_2d(&mx, const_cast<void*>(a.x), a.M, a.K, a.ldx, BN, gemm::BK);
  if (e != cudaSuccess) return e;
  dim3 grid((unsigned)tiles, 1, (unsigned)p.splits);
  return cps == 1 ? gemm::launch<BN, 1, true>(mw, mx, p, grid, stream, v)
                  : gemm::launch<BN, 2, true>(mw, mx, p, grid, stream, v);
}

}  // namespace es

namespace es {

cudaError_t launch_gemm_allgather(const GemmArgs& a, const CommArgs& c, int64_t ag_per, int64_t members,
                                  uint64_t own_base, cudaStream_t stream) {
  constexpr int BN = 64;
  const int64_t M = ag_per * members;  // the gathered rows, in member order
  if (ag_per <= 0 || members <= 0 || members > comm::kMaxRows || M > BN || a.N == 0) return cudaErrorInvalidValue;
  if (a.K % 8 != 0 || (a.ldx * 2) % 16 != 0 || a.silu || a.valid != nullptr) return cudaErrorInvalidValue;
  if (reinterpret_cast<uintptr_t>(a.x) % 16 != 0 || own_base % 16 != 0 || c.seqs == nullptr)
    return cudaErrorInvalidValue;
  if ((size_t)M * a.K * 2 > comm::kAGGemmBytes) return cudaErrorInvalidValue;
  const int tiles = (int)((a.N + gemm::BM - 1) / gemm::BM);
  gemm::Params p{};
  p.out = static_cast<__nv_bfloat16*>(a.out);
  p.residual = static_cast<const __nv_bfloat16*>(a.residual);
  p.status = a.status;
  p.M = (int)M;
  p.N = (int)a.N;
  p.ldo = (int)a.ldo;
  p.ldr = (int)a.ldr;
  p.kb = (int)((a.K + gemm::BK - 1) / gemm::BK);
  p.scale = a.scale;
  p.pre = static_cast<const __nv_bfloat16*>(a.pre);
  p.ldp = (int)a.ldp;
  p.ag_x = static_cast<const __nv_bfloat16*>(a.x);
  p.ag_per = (int)ag_per;
  p.ag_ldx = (int)a.ldx;
  p.ag_k = (int)a.K;
  p.w_packed = static_cast<const uint8_t*>(a.w_packed);
  p.pf = static_cast<const uint8_t*>(a.prefetch);
  p.pf_bytes = a.prefetch_bytes;
  p.ahead = l2_ahead();
  int cps = 1;
  gemm_plan(BN, a.N, a.K, a.num_sms, &p.splits, &cps);
  // every CTA waits for the pushers of every member: the whole grid must be resident at once
  const int s_fit = cps == 1 ? gemm::resident_split<BN, 1>(tiles, p.splits) : gemm::resident_split<BN, 2>(tiles, p.splits);
  if (s_fit <= 0) return cudaErrorInvalidConfiguration;
  p.splits = s_fit;
  comm::View v{};
  v.seqs = c.seqs;
  v.peers = c.peers;
  v.order = c.order;
  v.call = c.call;
  v.ctrl = reinterpret_cast<comm::Ctrl*>(c.ctrl);
  v.row = c.row;
  // the gathered rows live in this member's own buffer, one region per call parity
  CUtensorMap mw, mx0, mx1;
  cudaError_t e = weight_map(a, &mw);
  if (e != cudaSuccess) return e;
  char* rows = reinterpret_cast<char*>(own_base) + comm::kAGGemmOff;
  e = tmap::bf16_2d(&mx0, rows, M, a.K, a.K, BN, gemm::BK);
  if (e != cudaSuccess) return e;
  e = tmap::bf16_2d(&mx1, rows + comm::kAGGemmBytes, M, a.K, a.K, BN, gemm::BK);
  if (e != cudaSuccess) return e;
  dim3 grid((unsigned)tiles, 1, (unsigned)p.splits);
  return cps == 1 ? gemm::launch<BN, 1, false>(mw, mx0, p, grid, stream, v, &mx1)
                  : gemm::launch<BN, 2, false>(mw, mx0, p, grid, stream, v, &mx1);
}

}  // namespace es
