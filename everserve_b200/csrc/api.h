// Launch interface of the everserve_b200 sm_100a kernels.
//
// The kernels (.cu) see only CUDA headers; the torch bindings (ops.cpp) check tensors and call
// these launchers with raw pointers on the caller's stream. Every launcher returns a cudaError_t
// (cudaErrorInvalidValue for a shape it refuses), so the .cu files stay free of torch headers.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace es {

// ---- elementwise.cu ---------------------------------------------------------------------------
cudaError_t launch_rmsnorm(const void* x, void* residual, const void* w, void* y, int64_t rows, int hidden,
                           int64_t x_stride, int64_t y_stride, float eps, cudaStream_t s);
cudaError_t launch_rope_kv(const void* qkv, const void* bias, const int64_t* positions, const float* cos_sin,
                           const int64_t* slots, void* q_out, void* cache, int64_t T, int hq, int hkv, int d,
                           int block_size, const int64_t* strides5, cudaStream_t s);
cudaError_t launch_silu_mul(const void* gu, void* out, int64_t rows, int inter, bool interleaved, cudaStream_t s);
cudaError_t launch_embed(const int64_t* ids, const void* table, void* out, int64_t T, int hidden, int64_t vocab,
                         cudaStream_t s);
cudaError_t launch_decode_advance(int64_t* st, const int64_t* sampled, const int* bt, int64_t bt_stride, int b, int B,
                                  int bs, cudaStream_t s);
// Seeded temperature / top-k / top-p sampling of each row (sampling.cu).
struct SampleArgs {
  const void* logits = nullptr;  // [rows, >= vocab] bf16 (or fp32 when fp32), rows `stride` apart
  bool fp32 = false;
  int64_t stride = 0;
  int vocab = 0;
  int64_t rows = 0;
  const int64_t* positions = nullptr;
  const float* temperature = nullptr;  // <= 0: greedy
  const int64_t* top_k = nullptr;      // <= 0: off
  const float* top_p = nullptr;        // >= 1: off
  const int64_t* seeds = nullptr;
  int64_t* out = nullptr;
};
cudaError_t launch_sample(const SampleArgs& a, cudaStream_t stream);

cudaError_t launch_argmax(const void* logits, int64_t* out, int64_t rows, int vocab, int64_t stride, cudaStream_t s);

// ---- comm.cu (peer-memory collectives; layout in comm.cuh) ----------------------------------
struct CommArgs {
  uint32_t* seqs;         // device [2 * 4096]: LL call counters of this member
  const uint64_t* peers;  // device [8]: each row's symmetric buffer (0 = unmapped)
  uint64_t mc;            // NVLS multicast address of the buffers (0: P2P stores)
  const int32_t* order;   // device [9]: member count, rows in member order
  uint32_t* call;         // device [2]: call counter, CTAs finished in the current call
  void* ctrl;             // device address of this member's host-mapped control words
  int row;                // this member's row
};
int64_t comm_buffer_bytes();
int64_t comm_max_elems(int64_t members);
int64_t comm_ll_max_elems();
cudaError_t launch_fdar(const void* inp, void* out, int64_t n, const CommArgs& c, cudaStream_t s);

// ---- gemm.cu -------------------------------------------------------------------------------------
struct GemmArgs {
  const void* x;  // [M, K] bf16, row stride ldx
  const void* w;  // [N, K] bf16, row stride ldw
  void* out;      // [M, N] bf16, row stride ldo
  const void* residual;  // optional [M, N] bf16, row stride ldr
  float* ws;             // unused (split-K partials live in cluster shared memory)
  uint32_t* sync;        // unused
  int* status;           // set non-zero if a bounded wait ran out
  int64_t M, N, K, ldx, ldw, ldo, ldr;
  int num_sms;           // SMs of the device (sizes the split-K clusters)
  // optional epilogue terms, in this order: out = x.w^T * scale[m] + pre[m, n] (then the
  // all-reduce of the fused variant), + residual[m, n]. `scale` (fp32, one per row of x) weights a
  // mixture expert's rows by their routing weight; `pre` (bf16, row stride ldp) carries the rank's
  // sum over the experts before it, so the experts of a rank combine in a fixed order.
  const float* scale = nullptr;
  const void* pre = nullptr;
  int64_t ldp = 0;
  int two_shot = 0;  // fused all-reduce: 1 = reduce-scatter to tile owners, then all-gather
  // grouped rows (an expert over what each sender dispatched to it): rows [s*valid_cap, s*valid_cap
  // + valid[s]) of each of the valid_segs segments are live; token tiles holding no live row are
  // skipped and their output rows left unwritten (plain GEMM only)
  const uint32_t* valid = nullptr;
  int64_t valid_cap = 0;
  int valid_segs = 0;
  // gate/up rows interleaved by 64 (tile t: gate rows 64t.., then their up rows): out[M, N/2] =
  // silu(gate) * up of the bf16-rounded products (no residual, scale, pre or valid)
  int silu = 0;
  // fused reduce-scatter (gemm_allreduce only): the member at position j of the order keeps tokens
  // [j * rs_per, (j + 1) * rs_per) of the sum, in out/residual rows from 0
  int64_t rs_per = 0;
  // the weight pre-packed by (128-row tile, 64-wide k-block) into swizzled 16 KB blocks (nullable)
  const void* w_packed = nullptr;
  // memory the next kernel reads, fetched into L2 while this GEMM runs (nullable; 16-byte aligned)
  const void* prefetch = nullptr;
  int64_t prefetch_bytes = 0;
  // RoPE + paged-KV write epilogue of the qkv projection (nullable): the weight's 128-row tiles are
  // the q heads, then the k heads, then the v heads (head dim 128); the bf16-rounded product is
  // rotated (q, k) and written to q_out [M, hq * 128] and to the cache rows of slots[m] (k, v), the
  // rope_kv_write kernel's arithmetic; `out` is not written
  const struct RopeOut* rope = nullptr;
};
struct RopeOut {
  const int64_t* positions;  // [M]
  const float* cos_sin;      // [max_position, 128]: cos of dims 0..63, then sin
  const int64_t* slots;      // [M] cache slot (block * block_size + offset), < 0: not written
  void* q_out;               // [M, hq * 128] bf16
  void* cache;               // the layer's paged cache, bf16
  int64_t s_block, s_off, s_head, s_kv;  // element strides: block, offset in block, kv head, k -> v
  int hq, hkv, block_size;
};
int64_t gemm_pick_bn(int64_t M);
// the decode split plan (cluster split-K and CTAs per SM) for an N x K bf16 weight at M tokens
void gemm_plan(int64_t M, int64_t N, int64_t K, int64_t num_sms, int* splits, int* cps);
int64_t gemm_pick_splits(int64_t M, int64_t N, int64_t K, int64_t num_sms);
int64_t gemm_ws_floats(int64_t num_sms);
int64_t gemm_sync_words(int64_t num_sms);
cudaError_t launch_gemm_bf16(const GemmArgs& a, cudaStream_t s);
// gemm_stream.cu: the stream-K decode GEMM (M <= 64; `ws`/`sync` sized by gemm_sk_*). With `silu`
// the weight rows are gate/up interleaved by 64 and out[M, N/2] = silu(gate) * up.
int64_t gemm_sk_ws_floats(int64_t num_sms);
int64_t gemm_sk_sync_words(int64_t num_sms);
cudaError_t launch_gemm_stream(const GemmArgs& a, bool silu, cudaStream_t s);
// Mixture routing: per token softmax over E logits (bf16 rows of `stride`), top k (ties to the
// lowest index), renormalised; scale[e, t] for this rank's experts e0 .. e0 + el - 1 (0 when not
// chosen). E <= 64, el <= 32.
// `ids`/`weights` (nullable, [T, k]): each token's chosen experts in rank order and their
// renormalised probabilities; `scale` (nullable when el = 0).
cudaError_t launch_moe_route(const void* logits, int64_t stride, int T, int E, int k, int e0, int el, float* scale,
                             int32_t* ids, float* weights, cudaStream_t s);
// out = sum over the group's members (member order) of x_r . w_r^T (+ residual): the row-parallel
// GEMM with its all-reduce fused into the epilogue (decode sizes, M <= 64).
cudaError_t launch_gemm_allreduce(const GemmArgs& a, const CommArgs& c, cudaStream_t s);
// out[M, N] = X . w^T with X the member-order concatenation of every member's [ag_per, K] rows
// (a.x: this member's), gathered into each member's own buffer (own_base) by the kernel itself:
// the column-parallel GEMM with its all-gather fused (M = ag_per * members <= 64).
cudaError_t launch_gemm_allgather(const GemmArgs& a, const CommArgs& c, int64_t ag_per, int64_t members,
                                  uint64_t own_base, cudaStream_t s);

// ---- moe.cu (expert-parallel all-to-all over peer memory; layout in moe.cu) -----------------------
struct MoeArgs {
  const uint64_t* peers;   // device [8]: each row's MoE buffer (0 = unmapped)
  const int32_t* members;  // device [1 + 8 + 1]: member count W, the row holding each position, then
                           // the first position this process plays (-1: none, a spare before its take)
  uint32_t* call;          // device [2 * nz]: call counter and CTAs done, per emulated member
  void* ctrl;              // control words (comm Ctrl) of the first member; nz of them in a row
  int pos;                 // the host's view of the first position played (the kernels read the table's)
  int nz;                  // members this launch plays (1 with a GPU each)
  int E, el, k, H;         // experts, experts per member, experts per token, hidden size
  int64_t cap;             // rows of one (expert, sender) segment: at least a sender's token count
  int splits;              // dispatch CTAs per expert
};
int64_t moe_header_bytes();
int64_t moe_counts_offset();
int64_t moe_counts_stride();
int64_t moe_buffer_bytes(int64_t el, int64_t W, int64_t cap, int64_t H);
// x [nz][T, H] (member stride x_member elements), ids [nz][T, k]; writes place [nz][T, k]
cudaError_t launch_moe_dispatch(const void* x, int64_t x_member, const int32_t* ids, int32_t* place, int T,
                                const MoeArgs& a, cudaStream_t s);
cudaError_t launch_moe_ready(const MoeArgs& a, cudaStream_t s);
cudaError_t launch_moe_combine(const int32_t* ids, const float* weights, const int32_t* place, void* out,
                               int64_t out_member, int T, int num_sms, const MoeArgs& a, cudaStream_t s);

// ---- attention.cu --------------------------------------------------------------------------------
struct DecodeArgs {
  const void* q;  // [B, Hq, D]
  int64_t q_stride;
  const void* cache;  // [nb, 2, Hkv, bs, D]
  int64_t s_block, s_kv;
  const int* block_tables;
  int64_t bt_stride;
  const int* ctx_lens;
  void* out;  // [B, Hq * D] rows of out_stride
  int64_t out_stride;
  float* part_o;
  float* part_ml;
  int* tickets;  // [B, Hkv] int32, zero before the first launch (each launch leaves it zero)
  int* status;
  int B, hq, hkv, d, block_size, max_splits, part_tokens;
  int64_t num_blocks;
  int stages;  // K/V ring depth (2..4)
  float scale;
  // memory the next kernel reads, fetched into L2 while this one runs (nullable; 16-byte aligned)
  const void* prefetch = nullptr;
  int64_t prefetch_bytes = 0;
};
cudaError_t launch_paged_decode(const DecodeArgs& a, cudaStream_t s);
// the persistent variant (decode_persist.cu; opt-in: ES_ATTN_PERSIST=1, or set_decode_persist, which
// returns the previous setting): one CTA per SM over an equal share of the (sequence, kv head,
// split) items, head dim 64 or 128, G <= 8, block size a multiple of 16, q rows 16-byte aligned;
// tickets required
int set_decode_persist(int on);
bool decode_persist_supported(const DecodeArgs& a);
cudaError_t launch_decode_persist(const DecodeArgs& a, cudaStream_t s);
// the same with the cache's map given: [num_blocks * 2 * Hkv * BS * D / 64, 64] with a box of
// (16 * D / 64 rows, 64 columns), 128-byte swizzled
cudaError_t launch_decode_persist_map(const DecodeArgs& a, const CUtensorMap& cache_map, cudaStream_t s);
// the tcgen05 persistent variant (decode_tc.cu): head dim 128, G <= 16, splits of 256 positions
bool decode_tc_supported(const DecodeArgs& a);
cudaError_t launch_decode_tc(const DecodeArgs& a, cudaStream_t s);
// the same with the tensor maps given: q as [B * Hq, D] with a box of (G rows, 64 columns), the
// cache as [num_blocks * 2 * Hkv * BS, D] with a box of (BS rows, 64 columns), both 128-byte swizzled
cudaError_t launch_decode_tc_maps(const DecodeArgs& a, const CUtensorMap& qm, const CUtensorMap& cm, cudaStream_t s);

// ---- gemm_fp8.cu: block-scaled fp8 (e4m3) GEMM ------------------------------------------------------
struct Fp8GemmArgs {
  const void* x;        // [M, K] e4m3, row stride ldx bytes
  const void* w;        // [N, K] e4m3, row stride ldw bytes
  const float* x_scale; // [M, K / 128], row stride xs_ld
  const float* w_scale; // [ceil(N / 128), K / 128], row stride ws_ld
  void* out;            // [M, N] bf16 (or [M, N / 2] with silu), row stride ldo
  const void* residual; // optional [M, N] bf16, row stride ldr
  int* status;
  int64_t M, N, K, ldx, ldw, ldo, ldr, xs_ld, ws_ld;
  int num_sms;
  int silu = 0;         // gate/up rows interleaved by 64: out = silu(gate) * up
};
cudaError_t launch_gemm_fp8(const Fp8GemmArgs& a, cudaStream_t s);
// per token and 128-wide block: x8 = e4m3(x / scale), scale = amax / 448
cudaError_t launch_quant_fp8(const void* x, int64_t ldx, void* x8, int64_t ld8, float* scale, int64_t lds, int64_t M,
                             int64_t K, cudaStream_t s);

// ---- prefill.cu ----------------------------------------------------------------------------------
struct PrefillArgs {
  const void* q;        // [T, Hq, D] rows of q_stride (= Hq * D) elements
  int64_t q_stride;
  const void* cache;    // [nb, 2, Hkv, bs, D] contiguous
  int64_t num_blocks;
  const int* block_tables;
  int64_t bt_stride;
  const int* tiles;     // [n_tiles, 4] int32: sequence, first row, rows (<= 128), first position
  int n_tiles;
  void* out;            // [T, Hq * D] rows of out_stride
  int64_t out_stride;
  int* status;
  int64_t T;
  int hq, hkv, d, block_size;
  float scale;
};
cudaError_t launch_paged_prefill(const PrefillArgs& a, cudaStream_t s);

// ---- kvcopy.cu -----------------------------------------------------------------------------------
struct KvCopyArgs {
  const int64_t* layer_ptrs;  // device array of per-layer cache addresses
  const int64_t* slots;       // [n]
  const int64_t* heads;       // [H]
  void* staging;              // [L, H, cap, 2, d]
  int64_t n, L, H, cap, d, block_size;
  int64_t strides[5];
  int elem;
};
cudaError_t launch_kv_copy(const KvCopyArgs& a, bool gather, cudaStream_t s);

}  // namespace es
