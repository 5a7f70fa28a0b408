// Torch bindings of the everserve_b200 sm_100a kernels (module everserve_b200._C).
//
// Each binding checks dtypes, shapes and alignment, then calls the kernel's launcher on the
// current CUDA stream. A refused launch raises; nothing falls back to another implementation.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

#include <atomic>
#include <chrono>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "api.h"
#include "vmm.h"

namespace {

#define ES_CHECK_CUDA(expr)                                                              \
  do {                                                                                   \
    cudaError_t _e = (expr);                                                             \
    TORCH_CHECK(_e == cudaSuccess, #expr " failed: ", cudaGetErrorString(_e));            \
  } while (0)

void check_bf16(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.scalar_type() == at::kBFloat16, name, " must be bf16");
}

cudaStream_t cur() { return at::cuda::getCurrentCUDAStream(); }

// Memory the next kernel reads, which this kernel fetches into L2 while it runs (nullable).
template <typename A>
void set_prefetch(A& a, const c10::optional<torch::Tensor>& t) {
  if (!t.has_value() || !t->defined()) return;
  TORCH_CHECK(t->is_cuda() && t->is_contiguous() && reinterpret_cast<uintptr_t>(t->data_ptr()) % 16 == 0,
              "prefetch: a contiguous, 16-byte aligned device tensor");
  a.prefetch = t->data_ptr();
  a.prefetch_bytes = t->numel() * t->element_size();
}

// A weight pre-packed by ops.pack_weight: 16 KB blocks per (128-row tile, 64-wide k-block). `w`
// then only carries the shape [N, K] (a stride-0 view); the kernels read the blocks.
bool packed_weight(es::GemmArgs& a, const c10::optional<torch::Tensor>& w_packed, int64_t N, int64_t K) {
  if (!w_packed.has_value() || !w_packed->defined()) return false;
  const int64_t blocks = ((N + 127) / 128) * ((K + 63) / 64);
  TORCH_CHECK(w_packed->is_cuda() && w_packed->is_contiguous() &&
                  w_packed->numel() * w_packed->element_size() == blocks * 16384,
              "w_packed: the weight packed into (tile, k-block) blocks of 16 KB");
  a.w_packed = w_packed->data_ptr();
  return true;
}

void rmsnorm(torch::Tensor x, c10::optional<torch::Tensor> residual, torch::Tensor w, torch::Tensor y, double eps) {
  check_bf16(x, "x");
  check_bf16(w, "w");
  check_bf16(y, "y");
  const int hidden = (int)x.size(-1);
  TORCH_CHECK(x.stride(-1) == 1 && y.stride(-1) == 1, "rows must be contiguous");
  TORCH_CHECK(w.numel() == hidden, "weight size");
  const int64_t rows = x.numel() / hidden;
  const int64_t xs = x.dim() >= 2 ? x.stride(-2) : hidden;
  const int64_t ys = y.dim() >= 2 ? y.stride(-2) : hidden;
  void* rp = nullptr;
  if (residual.has_value()) {
    check_bf16(*residual, "residual");
    TORCH_CHECK(residual->is_contiguous() && residual->numel() == rows * hidden, "residual must be contiguous");
    rp = residual->data_ptr();
  }
  const c10::cuda::CUDAGuard g(x.device());
  ES_CHECK_CUDA(es::launch_rmsnorm(x.data_ptr(), rp, w.data_ptr(), y.data_ptr(), rows, hidden, xs, ys, (float)eps, cur()));
}

void rope_kv_write(torch::Tensor qkv, c10::optional<torch::Tensor> bias, torch::Tensor positions,
                   torch::Tensor cos_sin, torch::Tensor slots, torch::Tensor q_out, torch::Tensor cache, int64_t hq,
                   int64_t hkv, int64_t block_size, std::vector<int64_t> strides) {
  check_bf16(qkv, "qkv");
  check_bf16(q_out, "q_out");
  check_bf16(cache, "cache");
  TORCH_CHECK(qkv.is_contiguous() && q_out.is_contiguous(), "qkv and q_out must be contiguous");
  TORCH_CHECK(positions.scalar_type() == at::kLong && slots.scalar_type() == at::kLong, "int64 positions/slots");
  TORCH_CHECK(cos_sin.scalar_type() == at::kFloat && cos_sin.is_contiguous() && cos_sin.is_cuda(), "fp32 cos_sin");
  TORCH_CHECK(strides.size() == 5, "five cache strides");
  const int64_t T = qkv.size(0);
  const int d = (int)cos_sin.size(1);
  TORCH_CHECK(qkv.size(1) == (hq + 2 * hkv) * d, "qkv width");
  TORCH_CHECK(positions.numel() >= T && slots.numel() >= T, "positions/slots length");
  const void* bp = nullptr;
  if (bias.has_value()) {
    check_bf16(*bias, "bias");
    bp = bias->data_ptr();
  }
  const c10::cuda::CUDAGuard g(qkv.device());
  ES_CHECK_CUDA(es::launch_rope_kv(qkv.data_ptr(), bp, positions.data_ptr<int64_t>(), cos_sin.data_ptr<float>(),
                                   slots.data_ptr<int64_t>(), q_out.data_ptr(), cache.data_ptr(), T, (int)hq,
                                   (int)hkv, d, (int)block_size, strides.data(), cur()));
}

void silu_mul(torch::Tensor gu, torch::Tensor out, bool interleaved) {
  check_bf16(gu, "gate_up");
  check_bf16(out, "out");
  TORCH_CHECK(gu.is_contiguous() && out.is_contiguous(), "contiguous");
  const int inter = (int)out.size(-1);
  TORCH_CHECK(gu.size(-1) == 2 * inter, "gate_up width");
  TORCH_CHECK(!interleaved || inter % 64 == 0, "interleaved gate_up needs runs of 64");
  const c10::cuda::CUDAGuard g(gu.device());
  ES_CHECK_CUDA(es::launch_silu_mul(gu.data_ptr(), out.data_ptr(), out.numel() / inter, inter, interleaved, cur()));
}

void embed(torch::Tensor ids, torch::Tensor table, torch::Tensor out) {
  check_bf16(table, "table");
  check_bf16(out, "out");
  TORCH_CHECK(ids.scalar_type() == at::kLong && ids.is_cuda(), "ids must be int64 on the device");
  TORCH_CHECK(table.is_contiguous() && out.is_contiguous(), "contiguous");
  const c10::cuda::CUDAGuard g(table.device());
  ES_CHECK_CUDA(es::launch_embed(ids.data_ptr<int64_t>(), table.data_ptr(), out.data_ptr(), ids.numel(),
                                 (int)table.size(1), table.size(0), cur()));
}

void argmax(torch::Tensor logits, torch::Tensor out) {
  check_bf16(logits, "logits");
  TORCH_CHECK(out.scalar_type() == at::kLong && out.is_cuda(), "out must be int64 on the device");
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1, "[rows, vocab] with contiguous rows");
  const c10::cuda::CUDAGuard g(logits.device());
  ES_CHECK_CUDA(es::launch_argmax(logits.data_ptr(), out.data_ptr<int64_t>(), logits.size(0), (int)logits.size(1),
                                  logits.stride(0), cur()));
}

void sample(torch::Tensor logits, torch::Tensor positions, torch::Tensor temperature, torch::Tensor top_k,
            torch::Tensor top_p, torch::Tensor seeds, torch::Tensor out) {
  TORCH_CHECK(logits.is_cuda() && logits.dim() == 2 && logits.stride(1) == 1, "logits [rows, vocab] on the device");
  TORCH_CHECK(logits.scalar_type() == at::kBFloat16 || logits.scalar_type() == at::kFloat, "logits bf16 or fp32");
  const int64_t B = logits.size(0);
  auto vec = [&](const torch::Tensor& t, at::ScalarType st, const char* n) {
    TORCH_CHECK(t.is_cuda() && t.scalar_type() == st && t.is_contiguous() && t.numel() == B, n,
                ": one contiguous value per row on the device");
  };
  vec(positions, at::kLong, "positions");
  vec(temperature, at::kFloat, "temperature");
  vec(top_k, at::kLong, "top_k");
  vec(top_p, at::kFloat, "top_p");
  vec(seeds, at::kLong, "seeds");
  vec(out, at::kLong, "out");
  es::SampleArgs a;
  a.logits = logits.data_ptr();
  a.fp32 = logits.scalar_type() == at::kFloat;
  a.stride = logits.stride(0);
  a.vocab = (int)logits.size(1);
  a.rows = B;
  a.positions = positions.data_ptr<int64_t>();
  a.temperature = temperature.data_ptr<float>();
  a.top_k = top_k.data_ptr<int64_t>();
  a.top_p = top_p.data_ptr<float>();
  a.seeds = seeds.data_ptr<int64_t>();
  a.out = out.data_ptr<int64_t>();
  const c10::cuda::CUDAGuard g(logits.device());
  ES_CHECK_CUDA(es::launch_sample(a, cur()));
}

void decode_advance(torch::Tensor st, torch::Tensor sampled, torch::Tensor bt, int64_t b, int64_t bs) {
  TORCH_CHECK(st.scalar_type() == at::kLong && st.dim() == 2 && st.size(0) == 4 && st.is_contiguous(), "state [4, B]");
  TORCH_CHECK(sampled.scalar_type() == at::kLong && bt.scalar_type() == at::kInt && bt.stride(1) == 1, "dtypes");
  TORCH_CHECK(sampled.numel() >= b && bt.size(0) >= b && b <= st.size(1), "sizes");
  const c10::cuda::CUDAGuard g(st.device());
  ES_CHECK_CUDA(es::launch_decode_advance(st.data_ptr<int64_t>(), sampled.data_ptr<int64_t>(), bt.data_ptr<int>(),
                                          bt.stride(0), (int)b, (int)st.size(1), (int)bs, cur()));
}

// The optional mixture terms of a GEMM epilogue: a per-row fp32 scale and a bf16 accumulator.
void mixture_terms(es::GemmArgs& a, const c10::optional<torch::Tensor>& scale, const c10::optional<torch::Tensor>& pre) {
  if (scale.has_value() && scale->defined()) {
    TORCH_CHECK(scale->scalar_type() == at::kFloat && scale->is_cuda() && scale->is_contiguous() &&
                    scale->numel() >= a.M, "scale: fp32[M] on the device");
    a.scale = scale->data_ptr<float>();
  }
  if (pre.has_value() && pre->defined()) {
    check_bf16(*pre, "pre");
    TORCH_CHECK(pre->size(0) == a.M && pre->size(1) == a.N && pre->stride(1) == 1, "pre shape");
    a.pre = pre->data_ptr();
    a.ldp = pre->stride(0);
  }
}

void gemm_bf16(torch::Tensor x, torch::Tensor w, torch::Tensor out, c10::optional<torch::Tensor> residual,
               torch::Tensor ws, torch::Tensor sync, torch::Tensor status, int64_t num_sms,
               c10::optional<torch::Tensor> scale, c10::optional<torch::Tensor> pre,
               c10::optional<torch::Tensor> valid, int64_t valid_cap, c10::optional<torch::Tensor> w_packed,
               c10::optional<torch::Tensor> prefetch) {
  check_bf16(x, "x");
  check_bf16(w, "w");
  check_bf16(out, "out");
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && out.dim() == 2, "2-D operands");
  es::GemmArgs a{};
  const bool packed = packed_weight(a, w_packed, w.size(0), w.size(1));
  TORCH_CHECK(x.stride(1) == 1 && (packed || w.stride(1) == 1) && out.stride(1) == 1, "K-contiguous operands");
  const int64_t M = x.size(0), K = x.size(1), N = w.size(0);
  TORCH_CHECK(w.size(1) == K, "K mismatch: x has ", K, ", w has ", w.size(1));
  TORCH_CHECK(out.size(0) == M && out.size(1) == N, "out shape");
  TORCH_CHECK(status.scalar_type() == at::kInt && status.is_cuda(), "status must be int32 on the device");
  TORCH_CHECK(ws.scalar_type() == at::kFloat && ws.numel() >= es::gemm_ws_floats(num_sms), "stream-K workspace too small");
  TORCH_CHECK(sync.scalar_type() == at::kInt && sync.numel() >= es::gemm_sync_words(num_sms), "sync words too small");
  a.x = x.data_ptr();
  a.w = w.data_ptr();
  a.out = out.data_ptr();
  a.M = M;
  a.N = N;
  a.K = K;
  a.ldx = x.stride(0);
  a.ldw = w.stride(0);
  a.ldo = out.stride(0);
  a.status = status.data_ptr<int>();
  a.ws = ws.data_ptr<float>();
  a.sync = reinterpret_cast<uint32_t*>(sync.data_ptr<int>());
  a.num_sms = (int)num_sms;
  if (residual.has_value()) {
    check_bf16(*residual, "residual");
    TORCH_CHECK(residual->size(0) == M && residual->size(1) == N && residual->stride(1) == 1, "residual shape");
    a.residual = residual->data_ptr();
    a.ldr = residual->stride(0);
  }
  mixture_terms(a, scale, pre);
  if (valid.has_value() && valid->defined()) {
    TORCH_CHECK(valid->is_cuda() && valid->scalar_type() == at::kInt && valid->is_contiguous(),
                "valid: int32 counts on the device");
    TORCH_CHECK(valid_cap > 0 && valid_cap * valid->numel() >= M, "valid: segments of valid_cap rows cover M");
    a.valid = reinterpret_cast<const uint32_t*>(valid->data_ptr<int32_t>());
    a.valid_cap = valid_cap;
    a.valid_segs = (int)valid->numel();
  }
  set_prefetch(a, prefetch);
  const c10::cuda::CUDAGuard g(x.device());
  ES_CHECK_CUDA(es::launch_gemm_bf16(a, cur()));
}

// out[M, N/2] = silu(gate) * up of x . w^T, w's rows gate/up interleaved by 64 (decode sizes)
void gemm_silu(torch::Tensor x, torch::Tensor w, torch::Tensor out, torch::Tensor ws, torch::Tensor sync,
               torch::Tensor status, int64_t num_sms, c10::optional<torch::Tensor> w_packed,
               c10::optional<torch::Tensor> prefetch) {
  check_bf16(x, "x");
  check_bf16(w, "w");
  check_bf16(out, "out");
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && out.dim() == 2, "2-D operands");
  es::GemmArgs a{};
  const bool packed = packed_weight(a, w_packed, w.size(0), w.size(1));
  TORCH_CHECK(x.stride(1) == 1 && (packed || w.stride(1) == 1) && out.stride(1) == 1, "K-contiguous operands");
  const int64_t M = x.size(0), K = x.size(1), N = w.size(0);
  TORCH_CHECK(w.size(1) == K && N % 128 == 0, "w: [N, K] with N a multiple of 128");
  TORCH_CHECK(out.size(0) == M && out.size(1) == N / 2, "out: [M, N / 2]");
  TORCH_CHECK(ws.scalar_type() == at::kFloat && ws.numel() >= es::gemm_ws_floats(num_sms), "stream-K workspace too small");
  TORCH_CHECK(sync.scalar_type() == at::kInt && sync.numel() >= es::gemm_sync_words(num_sms), "sync words too small");
  a.x = x.data_ptr();
  a.w = w.data_ptr();
  a.out = out.data_ptr();
  a.M = M;
  a.N = N;
  a.K = K;
  a.ldx = x.stride(0);
  a.ldw = w.stride(0);
  a.ldo = out.stride(0);
  a.status = status.data_ptr<int>();
  a.ws = ws.data_ptr<float>();
  a.sync = reinterpret_cast<uint32_t*>(sync.data_ptr<int>());
  a.num_sms = (int)num_sms;
  a.silu = 1;
  set_prefetch(a, prefetch);
  const c10::cuda::CUDAGuard g(x.device());
  ES_CHECK_CUDA(es::launch_gemm_bf16(a, cur()));
}

// q_out[M, hq * 128] and the cache rows of the step's tokens from x . w^T (the qkv projection),
// RoPE and the paged-KV write in the GEMM's epilogue
void gemm_rope(torch::Tensor x, torch::Tensor w, torch::Tensor positions, torch::Tensor cos_sin, torch::Tensor slots,
               torch::Tensor q_out, torch::Tensor cache, int64_t hq, int64_t hkv, int64_t block_size,
               std::vector<int64_t> strides, torch::Tensor ws, torch::Tensor sync, torch::Tensor status,
               int64_t num_sms, c10::optional<torch::Tensor> w_packed, c10::optional<torch::Tensor> prefetch) {
  check_bf16(x, "x");
  check_bf16(w, "w");
  check_bf16(q_out, "q_out");
  check_bf16(cache, "cache");
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && x.stride(1) == 1, "2-D operands, x K-contiguous");
  es::GemmArgs a{};
  const bool packed = packed_weight(a, w_packed, w.size(0), w.size(1));
  TORCH_CHECK(packed || w.stride(1) == 1, "w K-contiguous");
  const int64_t M = x.size(0), K = x.size(1), N = w.size(0);
  TORCH_CHECK(w.size(1) == K && N == (hq + 2 * hkv) * 128, "w: [(hq + 2 hkv) * 128, K]");
  TORCH_CHECK(cos_sin.scalar_type() == at::kFloat && cos_sin.is_contiguous() && cos_sin.size(1) == 128,
              "cos_sin: fp32 [positions, 128]");
  TORCH_CHECK(positions.scalar_type() == at::kLong && slots.scalar_type() == at::kLong &&
                  positions.numel() >= M && slots.numel() >= M && positions.is_cuda() && slots.is_cuda(),
              "int64 positions and slots on the device, one per row");
  TORCH_CHECK(q_out.is_contiguous() && q_out.numel() == M * hq * 128, "q_out: [M, hq, 128] contiguous");
  TORCH_CHECK(strides.size() == 5 && strides[4] == 1, "five cache strides, head dim contiguous");
  TORCH_CHECK(ws.scalar_type() == at::kFloat && ws.numel() >= es::gemm_ws_floats(num_sms), "stream-K workspace too small");
  TORCH_CHECK(sync.scalar_type() == at::kInt && sync.numel() >= es::gemm_sync_words(num_sms), "sync words too small");
  es::RopeOut r{};
  r.positions = positions.data_ptr<int64_t>();
  r.cos_sin = cos_sin.data_ptr<float>();
  r.slots = slots.data_ptr<int64_t>();
  r.q_out = q_out.data_ptr();
  r.cache = cache.data_ptr();
  r.s_block = strides[0];
  r.s_off = strides[1];
  r.s_head = strides[2];
  r.s_kv = strides[3];
  r.hq = (int)hq;
  r.hkv = (int)hkv;
  r.block_size = (int)block_size;
  a.x = x.data_ptr();
  a.w = w.data_ptr();
  a.out = q_out.data_ptr();  // not written: the epilogue writes q_out and the cache
  a.M = M;
  a.N = N;
  a.K = K;
  a.ldx = x.stride(0);
  a.ldw = w.stride(0);
  a.ldo = N;
  a.status = status.data_ptr<int>();
  a.ws = ws.data_ptr<float>();
  a.sync = reinterpret_cast<uint32_t*>(sync.data_ptr<int>());
  a.num_sms = (int)num_sms;
  a.rope = &r;
  set_prefetch(a, prefetch);
  const c10::cuda::CUDAGuard g(x.device());
  ES_CHECK_CUDA(es::launch_gemm_bf16(a, cur()));
}

// ---- block-scaled fp8 ---------------------------------------------------------------------------
void quant_fp8(torch::Tensor x, torch::Tensor x8, torch::Tensor scale) {
  check_bf16(x, "x");
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && x8.dim() == 2 && x8.stride(1) == 1, "2-D row-major operands");
  TORCH_CHECK(x8.element_size() == 1 && x8.sizes() == x.sizes(), "x8: one byte per element, x's shape");
  TORCH_CHECK(scale.scalar_type() == at::kFloat && scale.dim() == 2 && scale.size(0) == x.size(0) &&
                  scale.size(1) == x.size(1) / 128 && scale.stride(1) == 1,
              "scale: fp32 [M, K / 128]");
  const c10::cuda::CUDAGuard g(x.device());
  ES_CHECK_CUDA(es::launch_quant_fp8(x.data_ptr(), x.stride(0), x8.data_ptr(), x8.stride(0), scale.data_ptr<float>(),
                                     scale.stride(0), x.size(0), x.size(1), cur()));
}

void gemm_fp8(torch::Tensor x8, torch::Tensor x_scale, torch::Tensor w8, torch::Tensor w_scale, torch::Tensor out,
              c10::optional<torch::Tensor> residual, torch::Tensor status, int64_t num_sms, bool silu) {
  TORCH_CHECK(x8.element_size() == 1 && w8.element_size() == 1, "fp8 operands (one byte per element)");
  TORCH_CHECK(x8.dim() == 2 && w8.dim() == 2 && x8.stride(1) == 1 && w8.stride(1) == 1, "2-D K-contiguous operands");
  check_bf16(out, "out");
  const int64_t M = x8.size(0), K = x8.size(1), N = w8.size(0);
  TORCH_CHECK(w8.size(1) == K && K % 128 == 0, "K mismatch or not a multiple of 128");
  TORCH_CHECK(x_scale.scalar_type() == at::kFloat && x_scale.size(0) == M && x_scale.size(1) == K / 128 &&
                  x_scale.stride(1) == 1,
              "x_scale: fp32 [M, K / 128]");
  TORCH_CHECK(w_scale.scalar_type() == at::kFloat && w_scale.size(0) == (N + 127) / 128 && w_scale.size(1) == K / 128 &&
                  w_scale.stride(1) == 1,
              "w_scale: fp32 [ceil(N / 128), K / 128]");
  TORCH_CHECK(out.size(0) == M && out.size(1) == (silu ? N / 2 : N) && out.stride(1) == 1, "out shape");
  es::Fp8GemmArgs a{};
  a.x = x8.data_ptr();
  a.w = w8.data_ptr();
  a.x_scale = x_scale.data_ptr<float>();
  a.w_scale = w_scale.data_ptr<float>();
  a.out = out.data_ptr();
  a.status = status.data_ptr<int>();
  a.M = M;
  a.N = N;
  a.K = K;
  a.ldx = x8.stride(0);
  a.ldw = w8.stride(0);
  a.ldo = out.stride(0);
  a.xs_ld = x_scale.stride(0);
  a.ws_ld = w_scale.stride(0);
  a.num_sms = (int)num_sms;
  a.silu = silu ? 1 : 0;
  if (residual.has_value() && residual->defined()) {
    check_bf16(*residual, "residual");
    TORCH_CHECK(residual->size(0) == M && residual->size(1) == N && residual->stride(1) == 1, "residual shape");
    a.residual = residual->data_ptr();
    a.ldr = residual->stride(0);
  }
  const c10::cuda::CUDAGuard g(x8.device());
  ES_CHECK_CUDA(es::launch_gemm_fp8(a, cur()));
}

torch::Tensor moe_route(torch::Tensor logits, int64_t k, int64_t e0, int64_t el) {
  check_bf16(logits, "logits");
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1, "logits: [T, E] rows");
  const int64_t T = logits.size(0), E = logits.size(1);
  auto scale = torch::empty({el, T}, logits.options().dtype(at::kFloat));
  const c10::cuda::CUDAGuard g(logits.device());
  ES_CHECK_CUDA(es::launch_moe_route(logits.data_ptr(), logits.stride(0), (int)T, (int)E, (int)k, (int)e0, (int)el,
                                     scale.data_ptr<float>(), nullptr, nullptr, cur()));
  return scale;
}

// Each token's top k experts (rank order) and their renormalised probabilities: (ids [T, k] int32,
// weights [T, k] fp32).
std::vector<torch::Tensor> moe_topk(torch::Tensor logits, int64_t k) {
  check_bf16(logits, "logits");
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1, "logits: [T, E] rows");
  const int64_t T = logits.size(0), E = logits.size(1);
  auto ids = torch::empty({T, k}, logits.options().dtype(at::kInt));
  auto w = torch::empty({T, k}, logits.options().dtype(at::kFloat));
  const c10::cuda::CUDAGuard g(logits.device());
  ES_CHECK_CUDA(es::launch_moe_route(logits.data_ptr(), logits.stride(0), (int)T, (int)E, (int)k, 0, 0, nullptr,
                                     ids.data_ptr<int32_t>(), w.data_ptr<float>(), cur()));
  return {ids, w};
}

// A uint8 tensor over `nbytes` of device memory at `ptr` that the caller keeps alive (a mapped
// symmetric buffer): lets the GEMMs read and write regions of it.
torch::Tensor device_view(int64_t ptr, int64_t nbytes, int64_t device) {
  TORCH_CHECK(ptr != 0 && nbytes > 0, "an address and a size");
  return torch::from_blob(reinterpret_cast<void*>(ptr), {nbytes},
                          torch::TensorOptions().dtype(at::kByte).device(at::kCUDA, (c10::DeviceIndex)device));
}

// The expert-parallel all-to-all's tables: peers int64[8] (buffer of each row), members int32[10]
// (count, row of each position, this process's first position), call int32[2 * nz], ctrl (device
// address of nz control words).
es::MoeArgs moe_args(torch::Tensor peers, torch::Tensor members, torch::Tensor call, int64_t ctrl, int64_t pos,
                     int64_t nz, int64_t E, int64_t el, int64_t k, int64_t H, int64_t cap, int64_t splits) {
  TORCH_CHECK(peers.is_cuda() && peers.scalar_type() == at::kLong && peers.numel() >= 8, "peers: int64[8] on the device");
  TORCH_CHECK(members.is_cuda() && members.scalar_type() == at::kInt && members.numel() >= 10,
              "members: int32[10] on the device (count, rows of the positions, this process's position)");
  TORCH_CHECK(call.is_cuda() && call.scalar_type() == at::kInt && call.numel() >= 2 * nz,
              "call: int32[2 * nz] on the device");
  TORCH_CHECK(ctrl != 0 && nz >= 1 && nz <= 8 && pos + nz <= 8, "control words and members played");
  es::MoeArgs a{};
  a.peers = reinterpret_cast<const uint64_t*>(peers.data_ptr<int64_t>());
  a.members = members.data_ptr<int32_t>();
  a.call = reinterpret_cast<uint32_t*>(call.data_ptr<int32_t>());
  a.ctrl = reinterpret_cast<void*>(ctrl);
  a.pos = (int)pos;
  a.nz = (int)nz;
  a.E = (int)E;
  a.el = (int)el;
  a.k = (int)k;
  a.H = (int)H;
  a.cap = cap;
  a.splits = (int)splits;
  return a;
}

void moe_dispatch(torch::Tensor x, torch::Tensor ids, torch::Tensor place, torch::Tensor peers, torch::Tensor members,
                  torch::Tensor call, int64_t ctrl, int64_t pos, int64_t E, int64_t el, int64_t cap, int64_t splits) {
  check_bf16(x, "x");
  TORCH_CHECK(x.dim() == 3 && x.is_contiguous(), "x: [members played, T, H] contiguous");
  TORCH_CHECK(ids.is_cuda() && ids.scalar_type() == at::kInt && ids.is_contiguous() && ids.dim() == 3 &&
                  ids.size(0) == x.size(0) && ids.size(1) == x.size(1), "ids: int32 [members played, T, k]");
  TORCH_CHECK(place.is_cuda() && place.scalar_type() == at::kInt && place.is_contiguous() &&
                  place.sizes() == ids.sizes(), "place: int32 like ids");
  const auto a = moe_args(peers, members, call, ctrl, pos, x.size(0), E, el, ids.size(2), x.size(2), cap, splits);
  const c10::cuda::CUDAGuard g(x.device());
  ES_CHECK_CUDA(es::launch_moe_dispatch(x.data_ptr(), x.size(1) * x.size(2), ids.data_ptr<int32_t>(),
                                        place.data_ptr<int32_t>(), (int)x.size(1), a, cur()));
}

void moe_ready(torch::Tensor peers, torch::Tensor members, torch::Tensor call, int64_t ctrl, int64_t pos, int64_t nz,
               int64_t E, int64_t el, int64_t k, int64_t H, int64_t cap) {
  const auto a = moe_args(peers, members, call, ctrl, pos, nz, E, el, k, H, cap, 1);
  const c10::cuda::CUDAGuard g(peers.device());
  ES_CHECK_CUDA(es::launch_moe_ready(a, cur()));
}

void moe_combine(torch::Tensor ids, torch::Tensor weights, torch::Tensor place, torch::Tensor out, torch::Tensor peers,
                 torch::Tensor members, torch::Tensor call, int64_t ctrl, int64_t pos, int64_t E, int64_t el,
                 int64_t cap, int64_t num_sms) {
  check_bf16(out, "out");
  TORCH_CHECK(out.dim() == 3 && out.is_contiguous(), "out: [members played, T, H] contiguous");
  TORCH_CHECK(ids.is_cuda() && ids.scalar_type() == at::kInt && ids.is_contiguous() && ids.dim() == 3 &&
                  ids.size(0) == out.size(0) && ids.size(1) == out.size(1), "ids: int32 [members played, T, k]");
  TORCH_CHECK(weights.is_cuda() && weights.scalar_type() == at::kFloat && weights.is_contiguous() &&
                  weights.sizes() == ids.sizes(), "weights: fp32 like ids");
  TORCH_CHECK(place.is_cuda() && place.scalar_type() == at::kInt && place.is_contiguous() &&
                  place.sizes() == ids.sizes(), "place: int32 like ids");
  const auto a = moe_args(peers, members, call, ctrl, pos, out.size(0), E, el, ids.size(2), out.size(2), cap, 1);
  const c10::cuda::CUDAGuard g(out.device());
  ES_CHECK_CUDA(es::launch_moe_combine(ids.data_ptr<int32_t>(), weights.data_ptr<float>(), place.data_ptr<int32_t>(),
                                       out.data_ptr(), out.size(1) * out.size(2), (int)out.size(1), (int)num_sms, a,
                                       cur()));
}

es::CommArgs comm_args(torch::Tensor peers, torch::Tensor order, torch::Tensor call, int64_t ctrl, int64_t row,
                       int64_t mc, torch::Tensor seqs) {
  TORCH_CHECK(seqs.is_cuda() && seqs.scalar_type() == at::kInt && seqs.numel() >= 8192, "seqs: int32[8192] on the device");
  TORCH_CHECK(peers.is_cuda() && peers.scalar_type() == at::kLong && peers.numel() >= 8, "peers: int64[8] on the device");
  TORCH_CHECK(order.is_cuda() && order.scalar_type() == at::kInt && order.numel() >= 9, "order: int32[9] on the device");
  TORCH_CHECK(call.is_cuda() && call.scalar_type() == at::kInt && call.numel() >= 2, "call: int32[2] on the device");
  TORCH_CHECK(ctrl != 0 && row >= 0 && row < 8, "control words and row");
  es::CommArgs c{};
  c.peers = reinterpret_cast<const uint64_t*>(peers.data_ptr<int64_t>());
  c.order = order.data_ptr<int32_t>();
  c.call = reinterpret_cast<uint32_t*>(call.data_ptr<int32_t>());
  c.ctrl = reinterpret_cast<void*>(ctrl);
  c.row = (int)row;
  c.mc = (uint64_t)mc;
  c.seqs = reinterpret_cast<uint32_t*>(seqs.data_ptr<int32_t>());
  return c;
}

void fdar(torch::Tensor inp, torch::Tensor out, torch::Tensor peers, torch::Tensor order, torch::Tensor call,
          int64_t ctrl, int64_t row, int64_t mc, torch::Tensor seqs) {
  check_bf16(inp, "inp");
  check_bf16(out, "out");
  TORCH_CHECK(inp.is_contiguous() && out.is_contiguous() && inp.numel() == out.numel(), "contiguous, same size");
  const c10::cuda::CUDAGuard g(inp.device());
  ES_CHECK_CUDA(es::launch_fdar(inp.data_ptr(), out.data_ptr(), inp.numel(), comm_args(peers, order, call, ctrl, row, mc, seqs),
                                cur()));
}

void gemm_allreduce(torch::Tensor x, torch::Tensor w, torch::Tensor out, c10::optional<torch::Tensor> residual,
                    torch::Tensor status, int64_t num_sms, torch::Tensor peers, torch::Tensor order, torch::Tensor call,
                    int64_t ctrl, int64_t row, int64_t mc, torch::Tensor seqs, c10::optional<torch::Tensor> scale,
                    c10::optional<torch::Tensor> pre, int64_t two_shot, int64_t rs_per,
                    c10::optional<torch::Tensor> w_packed, c10::optional<torch::Tensor> prefetch) {
  check_bf16(x, "x");
  check_bf16(w, "w");
  check_bf16(out, "out");
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && out.dim() == 2, "2-D operands");
  es::GemmArgs a{};
  const bool packed = packed_weight(a, w_packed, w.size(0), w.size(1));
  TORCH_CHECK(x.stride(1) == 1 && (packed || w.stride(1) == 1) && out.stride(1) == 1, "K-contiguous operands");
  const int64_t M = x.size(0), K = x.size(1), N = w.size(0);
  TORCH_CHECK(w.size(1) == K && out.size(1) == N && out.size(0) == (rs_per > 0 ? rs_per : M), "shapes");
  TORCH_CHECK(M <= 64, "the fused all-reduce GEMM takes decode batches (M <= 64)");
  a.x = x.data_ptr();
  a.w = w.data_ptr();
  a.out = out.data_ptr();
  a.M = M;
  a.N = N;
  a.K = K;
  a.ldx = x.stride(0);
  a.ldw = w.stride(0);
  a.ldo = out.stride(0);
  a.status = status.data_ptr<int>();
  a.num_sms = (int)num_sms;
  if (residual.has_value()) {
    check_bf16(*residual, "residual");
    TORCH_CHECK(residual->size(0) == out.size(0) && residual->size(1) == N && residual->stride(1) == 1,
                "residual shape (out's rows)");
    a.residual = residual->data_ptr();
    a.ldr = residual->stride(0);
  }
  mixture_terms(a, scale, pre);
  a.two_shot = (int)two_shot;
  a.rs_per = rs_per;
  set_prefetch(a, prefetch);
  const c10::cuda::CUDAGuard g(x.device());
  ES_CHECK_CUDA(es::launch_gemm_allreduce(a, comm_args(peers, order, call, ctrl, row, mc, seqs), cur()));
}

void gemm_allgather(torch::Tensor x, torch::Tensor w, torch::Tensor out, c10::optional<torch::Tensor> residual,
                    torch::Tensor status, int64_t num_sms, torch::Tensor peers, torch::Tensor order, torch::Tensor call,
                    int64_t ctrl, int64_t row, int64_t mc, torch::Tensor seqs, int64_t members, int64_t own_base,
                    c10::optional<torch::Tensor> w_packed) {
  check_bf16(x, "x");
  check_bf16(w, "w");
  check_bf16(out, "out");
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && out.dim() == 2, "2-D operands");
  es::GemmArgs a{};
  const bool packed = packed_weight(a, w_packed, w.size(0), w.size(1));
  TORCH_CHECK(x.stride(1) == 1 && (packed || w.stride(1) == 1) && out.stride(1) == 1, "K-contiguous operands");
  const int64_t per = x.size(0), K = x.size(1), N = w.size(0);
  TORCH_CHECK(w.size(1) == K && out.size(0) == per * members && out.size(1) == N, "shapes: out is [per * members, N]");
  a.x = x.data_ptr();
  a.w = w.data_ptr();
  a.out = out.data_ptr();
  a.M = per * members;
  a.N = N;
  a.K = K;
  a.ldx = x.stride(0);
  a.ldw = w.stride(0);
  a.ldo = out.stride(0);
  a.status = status.data_ptr<int>();
  a.num_sms = (int)num_sms;
  if (residual.has_value() && residual->defined()) {
    check_bf16(*residual, "residual");
    TORCH_CHECK(residual->size(0) == a.M && residual->size(1) == N && residual->stride(1) == 1, "residual shape");
    a.residual = residual->data_ptr();
    a.ldr = residual->stride(0);
  }
  const c10::cuda::CUDAGuard g(x.device());
  ES_CHECK_CUDA(es::launch_gemm_allgather(a, comm_args(peers, order, call, ctrl, row, mc, seqs), per, members,
                                          (uint64_t)own_base, cur()));
}


void paged_decode(torch::Tensor q, torch::Tensor cache, torch::Tensor block_tables, torch::Tensor ctx_lens,
                  torch::Tensor out, torch::Tensor part_o, torch::Tensor part_ml, torch::Tensor tickets,
                  torch::Tensor status, int64_t max_splits, int64_t part_tokens, double scale, int64_t stages,
                  c10::optional<torch::Tensor> prefetch) {
  check_bf16(q, "q");
  check_bf16(cache, "cache");
  check_bf16(out, "out");
  TORCH_CHECK(cache.dim() == 5 && cache.is_contiguous(), "cache must be contiguous [nb, 2, Hkv, bs, D]");
  TORCH_CHECK(block_tables.scalar_type() == at::kInt && ctx_lens.scalar_type() == at::kInt, "int32 tables");
  TORCH_CHECK(part_o.scalar_type() == at::kFloat && part_ml.scalar_type() == at::kFloat, "fp32 scratch");
  const int B = (int)q.size(0);
  const int hkv = (int)cache.size(2), bs = (int)cache.size(3), d = (int)cache.size(4);
  TORCH_CHECK(q.dim() == 3 && q.size(2) == d && q.stride(2) == 1 && q.stride(1) == d, "q must be [B, Hq, D]");
  const int hq = (int)q.size(1);
  TORCH_CHECK(part_o.numel() >= (int64_t)B * hq * max_splits * d &&
                  part_ml.numel() >= (int64_t)B * hq * max_splits * 2,
              "split scratch too small");
  TORCH_CHECK(out.stride(-1) == 1 && out.size(0) == B, "out rows");
  TORCH_CHECK(block_tables.dim() == 2 && block_tables.size(0) >= B && ctx_lens.numel() >= B, "tables");
  es::DecodeArgs a{};
  a.q = q.data_ptr();
  a.q_stride = q.stride(0);
  a.cache = cache.data_ptr();
  a.s_block = cache.stride(0);
  a.s_kv = cache.stride(1);
  a.block_tables = block_tables.data_ptr<int>();
  a.bt_stride = block_tables.stride(0);
  a.ctx_lens = ctx_lens.data_ptr<int>();
  a.out = out.data_ptr();
  a.out_stride = out.stride(0);
  a.part_o = part_o.data_ptr<float>();
  a.part_ml = part_ml.data_ptr<float>();
  TORCH_CHECK(tickets.is_cuda() && tickets.scalar_type() == at::kInt && tickets.is_contiguous() &&
                  tickets.numel() >= (int64_t)B * hkv,
              "tickets: int32 [B * kv_heads] on the device, zero before the first call");
  a.tickets = tickets.data_ptr<int>();
  a.status = status.data_ptr<int>();
  a.B = B;
  a.hq = hq;
  a.hkv = hkv;
  a.d = d;
  a.block_size = bs;
  a.num_blocks = cache.size(0);
  a.stages = (int)stages;
  a.max_splits = (int)max_splits;
  a.part_tokens = (int)part_tokens;
  a.scale = (float)scale;
  set_prefetch(a, prefetch);
  const c10::cuda::CUDAGuard g(q.device());
  ES_CHECK_CUDA(es::launch_paged_decode(a, cur()));
}

void paged_prefill(torch::Tensor q, torch::Tensor cache, torch::Tensor block_tables, torch::Tensor tiles,
                   torch::Tensor out, torch::Tensor status, double scale) {
  check_bf16(q, "q");
  check_bf16(cache, "cache");
  check_bf16(out, "out");
  TORCH_CHECK(cache.dim() == 5 && cache.is_contiguous(), "cache must be contiguous [nb, 2, Hkv, bs, D]");
  TORCH_CHECK(q.dim() == 3 && q.is_contiguous() && q.size(2) == cache.size(4), "q must be contiguous [T, Hq, D]");
  TORCH_CHECK(out.sizes() == q.sizes() && out.is_contiguous(), "out must be [T, Hq, D] like q");
  TORCH_CHECK(block_tables.scalar_type() == at::kInt && block_tables.dim() == 2, "int32 block tables");
  TORCH_CHECK(tiles.scalar_type() == at::kInt && tiles.dim() == 2 && tiles.size(1) == 4 && tiles.is_contiguous() &&
                  reinterpret_cast<uintptr_t>(tiles.data_ptr()) % 16 == 0,
              "tiles must be a contiguous, 16-byte aligned int32 [n, 4]");
  TORCH_CHECK(status.scalar_type() == at::kInt, "int32 status word");
  es::PrefillArgs a{};
  a.q = q.data_ptr();
  a.q_stride = q.stride(0);
  a.cache = cache.data_ptr();
  a.num_blocks = cache.size(0);
  a.block_tables = block_tables.data_ptr<int>();
  a.bt_stride = block_tables.stride(0);
  a.tiles = tiles.data_ptr<int>();
  a.n_tiles = (int)tiles.size(0);
  a.out = out.data_ptr();
  a.out_stride = out.stride(0);
  a.status = status.data_ptr<int>();
  a.T = q.size(0);
  a.hq = (int)q.size(1);
  a.hkv = (int)cache.size(2);
  a.d = (int)cache.size(4);
  a.block_size = (int)cache.size(3);
  a.scale = (float)scale;
  const c10::cuda::CUDAGuard g(q.device());
  ES_CHECK_CUDA(es::launch_paged_prefill(a, cur()));
}

void kv_copy(bool gather, torch::Tensor layer_ptrs, torch::Tensor slots, torch::Tensor heads, int64_t staging_ptr,
             int64_t cap, int64_t d, int64_t block_size, std::vector<int64_t> strides, int64_t elem) {
  TORCH_CHECK(layer_ptrs.is_cuda() && slots.is_cuda() && heads.is_cuda(), "device index tensors");
  TORCH_CHECK(layer_ptrs.scalar_type() == at::kLong && slots.scalar_type() == at::kLong &&
                  heads.scalar_type() == at::kLong,
              "int64 index tensors");
  TORCH_CHECK(strides.size() == 5, "five strides");
  es::KvCopyArgs a{};
  a.layer_ptrs = layer_ptrs.data_ptr<int64_t>();
  a.slots = slots.data_ptr<int64_t>();
  a.heads = heads.data_ptr<int64_t>();
  a.staging = reinterpret_cast<void*>(staging_ptr);
  a.n = slots.numel();
  a.L = layer_ptrs.numel();
  a.H = heads.numel();
  a.cap = cap;
  a.d = d;
  a.block_size = block_size;
  for (int i = 0; i < 5; i++) a.strides[i] = strides[i];
  a.elem = (int)elem;
  const c10::cuda::CUDAGuard g(slots.device());
  ES_CHECK_CUDA(es::launch_kv_copy(a, gather, cur()));
}

// ---- host helpers ---------------------------------------------------------------------------------

// ---- heartbeats ------------------------------------------------------------------------------
// A native thread that advances a 32-bit counter (a member's beat word in the slot region's shared,
// device-mapped pages) every `period_us`, independent of the Python interpreter: the beat stops only
// when the process does. The kernels' peer waits read it (comm.cuh).
namespace {
struct Beater {
  std::atomic<bool> stop{false};
  std::thread t;
};
std::mutex g_beat_mu;
std::map<int64_t, std::unique_ptr<Beater>> g_beaters;
int64_t g_beat_next = 1;
}  // namespace

int64_t heartbeat_start(int64_t addr, int64_t period_us) {
  TORCH_CHECK(addr != 0 && addr % 4 == 0 && period_us > 0, "heartbeat: a 4-byte aligned word and a period");
  auto b = std::make_unique<Beater>();
  Beater* raw = b.get();
  uint32_t* word = reinterpret_cast<uint32_t*>(addr);
  raw->t = std::thread([raw, word, period_us] {
    while (!raw->stop.load(std::memory_order_relaxed)) {
      __atomic_fetch_add(word, 1u, __ATOMIC_RELEASE);
      std::this_thread::sleep_for(std::chrono::microseconds(period_us));
    }
  });
  std::lock_guard<std::mutex> g(g_beat_mu);
  const int64_t id = g_beat_next++;
  g_beaters.emplace(id, std::move(b));
  return id;
}

void heartbeat_stop(int64_t id) {
  std::unique_ptr<Beater> b;
  {
    std::lock_guard<std::mutex> g(g_beat_mu);
    auto it = g_beaters.find(id);
    if (it == g_beaters.end()) return;
    b = std::move(it->second);
    g_beaters.erase(it);
  }
  b->stop.store(true);
  if (b->t.joinable()) b->t.join();
}

int64_t host_register_mapped(int64_t ptr, int64_t bytes) {
  const cudaError_t e = cudaHostRegister(reinterpret_cast<void*>(ptr), (size_t)bytes,
                                         cudaHostRegisterMapped | cudaHostRegisterPortable);
  if (e != cudaSuccess) {
    // pages the host cannot pin (a file on a disk-backed filesystem): the caller falls back to a
    // pinned copy; the error is cleared first, or the next CUDA call of the process would report it
    cudaGetLastError();
    TORCH_CHECK(false, "cudaHostRegister of ", bytes, " bytes failed: ", cudaGetErrorString(e));
  }
  void* dev = nullptr;
  ES_CHECK_CUDA(cudaHostGetDevicePointer(&dev, reinterpret_cast<void*>(ptr), 0));
  return reinterpret_cast<int64_t>(dev);
}

// The device address of pinned host memory the CUDA runtime allocated (torch's pinned tensors).
int64_t host_device_pointer(int64_t ptr) {
  void* dev = nullptr;
  ES_CHECK_CUDA(cudaHostGetDevicePointer(&dev, reinterpret_cast<void*>(ptr), 0));
  return reinterpret_cast<int64_t>(dev);
}

void host_unregister(int64_t ptr) { ES_CHECK_CUDA(cudaHostUnregister(reinterpret_cast<void*>(ptr))); }

int64_t device_alloc(int64_t bytes) {
  void* p = nullptr;
  ES_CHECK_CUDA(cudaMalloc(&p, (size_t)bytes));
  ES_CHECK_CUDA(cudaMemset(p, 0, (size_t)bytes));
  return reinterpret_cast<int64_t>(p);
}

void device_free(int64_t ptr) { ES_CHECK_CUDA(cudaFree(reinterpret_cast<void*>(ptr))); }

void memset_async(int64_t ptr, int64_t bytes) {
  ES_CHECK_CUDA(cudaMemsetAsync(reinterpret_cast<void*>(ptr), 0, (size_t)bytes, cur()));
}

pybind11::bytes ipc_handle(int64_t ptr) {
  cudaIpcMemHandle_t h;
  ES_CHECK_CUDA(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(ptr)));
  return pybind11::bytes(reinterpret_cast<const char*>(&h), sizeof(h));
}

int64_t ipc_open(const std::string& handle) {
  TORCH_CHECK(handle.size() == sizeof(cudaIpcMemHandle_t), "bad IPC handle size");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle.data(), sizeof(h));
  void* p = nullptr;
  ES_CHECK_CUDA(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(p);
}

void ipc_close(int64_t ptr) { ES_CHECK_CUDA(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr))); }

int cur_device() {
  int d = 0;
  ES_CHECK_CUDA(cudaGetDevice(&d));
  return d;
}

// (ptr, size, handle, fd) of a new exportable buffer on the current device, zeroed.
std::tuple<int64_t, int64_t, int64_t, int64_t> vmm_create(int64_t bytes) {
  es::vmm::Buffer b;
  const char* err = "";
  TORCH_CHECK(es::vmm::create(cur_device(), (uint64_t)bytes, b, &err), "VMM allocation: ", err);
  ES_CHECK_CUDA(cudaMemset(reinterpret_cast<void*>(b.ptr), 0, b.size));
  return {(int64_t)b.ptr, (int64_t)b.size, (int64_t)b.handle, (int64_t)b.fd};
}

// (ptr, size, handle) of another process's buffer, mapped for the current device.
std::tuple<int64_t, int64_t, int64_t> vmm_import(int64_t fd, int64_t bytes) {
  es::vmm::Buffer b;
  const char* err = "";
  TORCH_CHECK(es::vmm::import(cur_device(), (int)fd, (uint64_t)bytes, b, &err), "VMM import: ", err);
  return {(int64_t)b.ptr, (int64_t)b.size, (int64_t)b.handle};
}

void vmm_release(int64_t ptr, int64_t size, int64_t handle, int64_t fd) {
  es::vmm::Buffer b;
  b.ptr = (uint64_t)ptr;
  b.size = (uint64_t)size;
  b.handle = (uint64_t)handle;
  b.fd = (int)fd;
  es::vmm::release(b);
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "everserve_b200 sm_100a kernels";
  m.def("rmsnorm", &rmsnorm, "RMSNorm, optionally fused with the residual add");
  m.def("rope_kv_write", &rope_kv_write, "RoPE on q/k and the paged-KV write of k/v");
  m.def("silu_mul", &silu_mul, "silu(gate) * up (halves, or runs of 64 interleaved)", pybind11::arg("gu"),
        pybind11::arg("out"), pybind11::arg("interleaved") = false);
  m.def("embed", &embed, "embedding gather");
  m.def("argmax", &argmax, "greedy argmax per row");
  m.def("sample", &sample, "seeded temperature / top-k / top-p sampling per row (Gumbel-max)");
  m.def("decode_advance", &decode_advance, "next decode step's inputs from the sampled ids");
  m.def("gemm_bf16", &gemm_bf16, "tcgen05 GEMM out = x . w^T * scale + pre (+ residual)", pybind11::arg("x"),
        pybind11::arg("w"), pybind11::arg("out"), pybind11::arg("residual"), pybind11::arg("ws"), pybind11::arg("sync"),
        pybind11::arg("status"), pybind11::arg("num_sms"), pybind11::arg("scale") = pybind11::none(),
        pybind11::arg("pre") = pybind11::none(), pybind11::arg("valid") = pybind11::none(),
        pybind11::arg("valid_cap") = 0, pybind11::arg("w_packed") = pybind11::none(),
        pybind11::arg("prefetch") = pybind11::none());
  m.def("gemm_pick_bn", &es::gemm_pick_bn);
  m.def("gemm_pick_splits", &es::gemm_pick_splits);
  m.def("gemm_ws_floats", &es::gemm_ws_floats);
  m.def("gemm_sync_words", &es::gemm_sync_words);
  m.def("set_decode_persist", [](int64_t on) { return (int64_t)es::set_decode_persist((int)on); },
        "decode attention on the persistent kernel (1) or the split kernel (0); returns the previous setting",
        pybind11::arg("on"));
  m.def("paged_decode", &paged_decode, "paged decode attention (split-KV, merged)", pybind11::arg("q"),
        pybind11::arg("cache"), pybind11::arg("block_tables"), pybind11::arg("ctx_lens"), pybind11::arg("out"),
        pybind11::arg("part_o"), pybind11::arg("part_ml"), pybind11::arg("tickets"), pybind11::arg("status"),
        pybind11::arg("max_splits"), pybind11::arg("part_tokens"), pybind11::arg("scale"), pybind11::arg("stages"),
        pybind11::arg("prefetch") = pybind11::none());
  m.def("gemm_silu", &gemm_silu, "GEMM with SiLU-mul fused into its epilogue (gate/up rows interleaved by 64)",
        pybind11::arg("x"), pybind11::arg("w"), pybind11::arg("out"), pybind11::arg("ws"), pybind11::arg("sync"),
        pybind11::arg("status"), pybind11::arg("num_sms"), pybind11::arg("w_packed") = pybind11::none(),
        pybind11::arg("prefetch") = pybind11::none());
  m.def("gemm_rope", &gemm_rope, "qkv GEMM with RoPE and the paged-KV write in its epilogue", pybind11::arg("x"),
        pybind11::arg("w"), pybind11::arg("positions"), pybind11::arg("cos_sin"), pybind11::arg("slots"),
        pybind11::arg("q_out"), pybind11::arg("cache"), pybind11::arg("hq"), pybind11::arg("hkv"),
        pybind11::arg("block_size"), pybind11::arg("strides"), pybind11::arg("ws"), pybind11::arg("sync"),
        pybind11::arg("status"), pybind11::arg("num_sms"), pybind11::arg("w_packed") = pybind11::none(),
        pybind11::arg("prefetch") = pybind11::none());
  m.def("quant_fp8", &quant_fp8, "x -> e4m3 with a scale per token and 128-wide block");
  m.def("gemm_fp8", &gemm_fp8, "block-scaled fp8 GEMM (tcgen05 kind::f8f6f4, scales per 128-wide K block)");
  m.def("paged_prefill", &paged_prefill, "paged causal prefill attention (tcgen05: S and P.V in TMEM, TMA K/V tiles)");
  m.def("moe_route", &moe_route, "mixture routing: per-token weights of this rank's experts [el, T]");
  m.def("moe_topk", &moe_topk, "mixture routing: each token's top k experts and their weights");
  m.def("moe_dispatch", &moe_dispatch, "expert-parallel dispatch of tokens to their experts' owners (peer stores)");
  m.def("moe_ready", &moe_ready, "expert-parallel: this member's expert outputs are written");
  m.def("moe_combine", &moe_combine, "expert-parallel combine: each token's weighted expert outputs (peer loads)");
  m.def("moe_buffer_bytes", &es::moe_buffer_bytes);
  m.def("device_view", &device_view, "uint8 tensor over caller-owned device memory");
  m.def("moe_header_bytes", &es::moe_header_bytes);
  m.def("moe_counts_offset", &es::moe_counts_offset);
  m.def("moe_counts_stride", &es::moe_counts_stride);
  m.def("fdar", &fdar, "failure-detecting all-reduce over peer memory (member order)");
  m.def("gemm_allreduce", &gemm_allreduce, "row-parallel GEMM with the all-reduce fused into its epilogue",
        pybind11::arg("x"), pybind11::arg("w"), pybind11::arg("out"), pybind11::arg("residual"), pybind11::arg("status"),
        pybind11::arg("num_sms"), pybind11::arg("peers"), pybind11::arg("order"), pybind11::arg("call"),
        pybind11::arg("ctrl"), pybind11::arg("row"), pybind11::arg("mc"), pybind11::arg("seqs"),
        pybind11::arg("scale") = pybind11::none(), pybind11::arg("pre") = pybind11::none(),
        pybind11::arg("two_shot") = 0, pybind11::arg("rs_per") = 0, pybind11::arg("w_packed") = pybind11::none(),
        pybind11::arg("prefetch") = pybind11::none());
  m.def("gemm_allgather", &gemm_allgather,
        "column-parallel GEMM with the all-gather of its token rows fused (peer stores into each member's buffer)",
        pybind11::arg("x"), pybind11::arg("w"), pybind11::arg("out"), pybind11::arg("residual"), pybind11::arg("status"),
        pybind11::arg("num_sms"), pybind11::arg("peers"), pybind11::arg("order"), pybind11::arg("call"),
        pybind11::arg("ctrl"), pybind11::arg("row"), pybind11::arg("mc"), pybind11::arg("seqs"),
        pybind11::arg("members"), pybind11::arg("own_base"), pybind11::arg("w_packed") = pybind11::none());
  m.def("comm_buffer_bytes", &es::comm_buffer_bytes);
  m.def("comm_max_elems", &es::comm_max_elems, "elements one all-reduce call takes for a group of `members`",
        pybind11::arg("members") = 1);
  m.def("comm_ll_max_elems", &es::comm_ll_max_elems);
  m.def("kv_gather", [](torch::Tensor lp, torch::Tensor s, torch::Tensor h, int64_t st, int64_t cap, int64_t d,
                        int64_t bs, std::vector<int64_t> str, int64_t el) { kv_copy(true, lp, s, h, st, cap, d, bs, str, el); },
        "paged cache -> staging rows, all layers in one launch");
  m.def("kv_scatter", [](torch::Tensor lp, torch::Tensor s, torch::Tensor h, int64_t st, int64_t cap, int64_t d,
                         int64_t bs, std::vector<int64_t> str, int64_t el) { kv_copy(false, lp, s, h, st, cap, d, bs, str, el); },
        "staging rows -> paged cache");
  m.def("host_register_mapped", &host_register_mapped);
  m.def("heartbeat_start", &heartbeat_start, "advance a beat word every period_us from a native thread; returns its id");
  m.def("heartbeat_stop", &heartbeat_stop, "stop a heartbeat thread");
  m.def("host_unregister", &host_unregister);
  m.def("host_device_pointer", &host_device_pointer, "device address of runtime-allocated pinned host memory");
  m.def("device_alloc", &device_alloc);
  m.def("device_free", &device_free);
  m.def("memset_async", &memset_async);
  m.def("ipc_handle", &ipc_handle);
  m.def("ipc_open", &ipc_open);
  m.def("ipc_close", &ipc_close);
  m.def("vmm_create", &vmm_create, "exportable device buffer (driver VMM): (ptr, size, handle, fd)");
  m.def("vmm_import", &vmm_import, "map another process's exported buffer: (ptr, size, handle)");
  m.def("vmm_release", &vmm_release);
}
