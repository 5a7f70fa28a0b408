"""Decoder ops: the sm_100a kernels for CUDA tensors, the PyTorch reference for CPU tensors.

``ops_for(device)`` returns the op set a model runs with. :class:`KernelOps` calls only the
compiled kernels (it raises if the extension is missing) and owns their scratch memory: the
split-K workspace and tile counters of the GEMM, the split-KV partials of decode attention and a
status word that bounded waits set. :class:`RefOps` is the CPU engine's arithmetic.
"""

from __future__ import annotations

import math
import os
import threading

import torch

from . import ref
from .. import _ext

__all__ = ["KernelOps", "RefOps", "deinterleave_gate_up", "dequantize_fp8", "interleave_gate_up", "ops_for",
           "prefill_tiles", "quantize_act_fp8", "quantize_weight_fp8", "ref"]


class RefOps:
    """PyTorch reference ops (CPU engine, fp32)."""

    kind = "ref"

    def __init__(self, device: torch.device | str = "cpu"):
        self.device = torch.device(device)

    def embed(self, ids, table):
        return table[ids]

    def rmsnorm(self, x, w, eps, residual=None):
        return ref.rmsnorm(x, w, eps, residual)

    def linear(self, x, w, bias=None, residual=None, out=None, scale=None, pre=None, valid=None, valid_cap=0,
               prefetch=None):
        # rows a grouped GEMM would skip are padding nobody reads: computing them changes nothing
        y = ref.linear(x, dense(w), bias, residual, scale, pre)
        if out is not None:
            out.copy_(y)
            return out
        return y

    def moe_route(self, logits, k, e0, el):
        return ref.moe_route(logits, k, e0, el)

    def moe_topk(self, logits, k):
        return ref.moe_topk(logits, k)

    def rope_kv_write(self, qkv, bias, positions, cos_sin, slots, cache, hq, hkv, block_size):
        return ref.rope_kv_write(qkv, bias, positions, cos_sin, slots, cache, hq, hkv, block_size)

    def linear_rope_kv(self, x, w, positions, cos_sin, slots, cache, hq, hkv, block_size, prefetch=None):
        return self.rope_kv_write(self.linear(x, w), None, positions, cos_sin, slots, cache, hq, hkv, block_size)

    def decode_attention(self, q, cache, block_tables, ctx_lens, scale, max_model_len=None, prefetch=None):
        B = q.shape[0]
        seq = torch.arange(B, device=q.device)
        return ref.paged_attention(q, cache, block_tables, ctx_lens, seq, ctx_lens.long() - 1, scale)

    def prefill_attention(self, q, cache, block_tables, ctx_lens, q_seq, q_pos, scale, tiles=None):
        return ref.paged_attention(q, cache, block_tables, ctx_lens, q_seq, q_pos, scale)

    def silu_mul(self, gu, interleaved: bool = False):
        if interleaved:
            gu = deinterleave_gate_up(gu.t()).t()
        return ref.silu_mul(gu)

    def linear_silu(self, x, w, prefetch=None):
        return self.silu_mul(self.linear(x, w), interleaved=True)

    def linear_fp8(self, x, w8, w_scale, residual=None, silu: bool = False):
        """The fp8 GEMM's arithmetic in fp32: activations quantized by the kernel's rule, both
        operands dequantized, one product (its rounding differs from the kernel's per-block sums)."""
        q, sc = quantize_act_fp8(x)
        y = dequantize_fp8(q, sc, 1) @ dequantize_fp8(w8, w_scale, 128).t()
        if residual is not None:
            y = y + residual.float()
        y = y.to(x.dtype)
        return self.silu_mul(y, interleaved=True) if silu else y

    def argmax(self, logits):
        return ref.argmax(logits)

    def sample(self, logits, positions, sb):
        """Seeded temperature / top-k / top-p draw of each row (engine.sampling.sample)."""
        from ..engine.sampling import sample

        return sample(logits, positions, sb)

    def check_status(self):
        return 0


class KernelOps:
    """The sm_100a kernels on one CUDA device, with their scratch memory."""

    kind = "kernel"
    # positions per decode-attention split (fixed per process: batch-invariant results); a multiple
    # of 64, ES_ATTN_PART overrides. 384 measured faster than 256 and 320 at 1K contexts (fewer,
    # longer CTAs and a smaller merge)
    PART_TOKENS = int(os.environ.get("ES_ATTN_PART", "384"))
    # K/V ring depth of decode attention: two stages leave room for three CTAs per SM, which
    # measured faster in the decode step than a deeper ring with two
    ATTN_STAGES = int(os.environ.get("ES_ATTN_STAGES", "2"))

    def __init__(self, device: torch.device | str):
        self.device = torch.device(device)
        assert self.device.type == "cuda", "KernelOps runs on CUDA devices"
        self.C = _ext.load()
        props = torch.cuda.get_device_properties(self.device)
        self.num_sms = props.multi_processor_count
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._ws = torch.empty(0, dtype=torch.float32, device=self.device)
        self._ctr = torch.zeros(0, dtype=torch.int32, device=self.device)
        self._part_o = torch.empty(0, dtype=torch.float32, device=self.device)
        self._part_ml = torch.empty(0, dtype=torch.float32, device=self.device)
        self._tickets = torch.zeros(0, dtype=torch.int32, device=self.device)
        self._lock = threading.Lock()

    # ---- scratch ------------------------------------------------------------------------------
    def _ensure(self, name: str, numel: int, dtype, zero: bool = False) -> torch.Tensor:
        buf = getattr(self, name)
        if buf.numel() >= numel:
            return buf
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError(f"{name} scratch must be reserved before CUDA graph capture ({numel} elements)")
        new = (torch.zeros if zero else torch.empty)(max(numel, 1), dtype=dtype, device=self.device)
        setattr(self, name, new)
        return new

    def reserve_linear(self, max_m: int = 0, shapes=None):
        """The GEMM's stream-K scratch: one fp32 partial tile per SM and the sync words."""
        self._ensure("_ws", int(self.C.gemm_ws_floats(self.num_sms)), torch.float32)
        self._ensure("_ctr", int(self.C.gemm_sync_words(self.num_sms)), torch.int32, zero=True)

    def max_splits(self, max_model_len: int) -> int:
        return max(1, (max_model_len + self.PART_TOKENS - 1) // self.PART_TOKENS)

    def reserve_attention(self, max_batch: int, hq: int, d: int, max_model_len: int):
        ms = self.max_splits(max_model_len)
        self._ensure("_part_o", max_batch * hq * ms * d, torch.float32)
        self._ensure("_part_ml", max_batch * hq * ms * 2, torch.float32)
        # one split ticket per (sequence, kv head); every launch leaves them at zero
        self._ensure("_tickets", max_batch * hq, torch.int32, zero=True)

    # ---- ops ----------------------------------------------------------------------------------
    def embed(self, ids, table):
        out = torch.empty(ids.shape[0], table.shape[1], dtype=table.dtype, device=table.device)
        self.C.embed(ids, table, out)
        return out

    def rmsnorm(self, x, w, eps, residual=None):
        y = torch.empty_like(x)
        self.C.rmsnorm(x, residual, w, y, eps)
        return y

    def linear(self, x, w, bias=None, residual=None, out=None, scale=None, pre=None, valid=None, valid_cap=0,
               w_packed=None, prefetch=None):
        """`valid` (int32 counts of segments of `valid_cap` rows) makes it a grouped GEMM whose
        token tiles holding no counted row are skipped and left unwritten. `w_packed`
        (``pack_weight(w)``) streams the weight as contiguous swizzled blocks instead of tiles."""
        M, K = x.shape
        N = w.shape[0]
        if out is None:
            out = torch.empty(M, N, dtype=x.dtype, device=x.device)
        self.reserve_linear()
        if bias is not None:
            # bias folds into the residual input of the epilogue
            b = bias.expand(M, N) if residual is None else residual + bias
            residual = b.contiguous()
        if isinstance(w, PackedWeight):
            w, w_packed = w.carrier, w.packed
        self.C.gemm_bf16(x, w, out, residual, self._ws, self._ctr, self.status, self.num_sms, scale, pre, valid,
                         valid_cap, w_packed, prefetch_target(prefetch))
        return out

    def quant_fp8(self, x):
        """x [M, K] bf16 -> (e4m3 [M, K], fp32 scales [M, K/128]) on the device."""
        M, K = x.shape
        q = torch.empty(M, K, dtype=torch.float8_e4m3fn, device=x.device)
        sc = torch.empty(M, K // 128, dtype=torch.float32, device=x.device)
        self.C.quant_fp8(x.contiguous(), q, sc)
        return q, sc

    def linear_fp8(self, x, w8, w_scale, residual=None, silu: bool = False):
        """x . w^T for block-scaled e4m3 weights (``quantize_weight_fp8``): the activations quantized
        per token and 128-wide block, then the tcgen05 fp8 GEMM; `silu` for gate/up interleaved
        weights (out [M, N/2])."""
        q, sc = self.quant_fp8(x)
        N = w8.shape[0]
        out = torch.empty(x.shape[0], N // 2 if silu else N, dtype=torch.bfloat16, device=x.device)
        self.C.gemm_fp8(q, sc, w8, w_scale, out, residual, self.status, self.num_sms, silu)
        return out

    def moe_route(self, logits, k, e0, el):
        return self.C.moe_route(logits.contiguous(), k, e0, el)

    def moe_topk(self, logits, k):
        ids, w = self.C.moe_topk(logits.contiguous(), k)
        return ids, w

    def rope_kv_write(self, qkv, bias, positions, cos_sin, slots, cache, hq, hkv, block_size):
        T = qkv.shape[0]
        d = cos_sin.shape[1]
        q = torch.empty(T, hq, d, dtype=qkv.dtype, device=qkv.device)
        self.C.rope_kv_write(qkv, bias, positions, cos_sin, slots, q, cache, hq, hkv, block_size,
                             list(cache.stride()[i] for i in (0, 3, 2, 1, 4)))
        return q

    def linear_rope_kv(self, x, w, positions, cos_sin, slots, cache, hq, hkv, block_size, prefetch=None):
        """The qkv projection with RoPE and the paged-KV write in the GEMM's epilogue: q [T, hq, 128]
        and the cache rows of `slots`, as ``rope_kv_write(linear(x, w), ...)`` computes them (the
        product rounded to bf16 before the rotation). Head dim 128, no qkv bias."""
        T = x.shape[0]
        q = torch.empty(T, hq, 128, dtype=x.dtype, device=x.device)
        self.reserve_linear()
        wt, wp = weight_args(w)
        self.C.gemm_rope(x, wt, positions, cos_sin, slots, q, cache, hq, hkv, block_size,
                         list(cache.stride()[i] for i in (0, 3, 2, 1, 4)), self._ws, self._ctr, self.status,
                         self.num_sms, wp, prefetch_target(prefetch))
        return q

    def decode_attention(self, q, cache, block_tables, ctx_lens, scale, max_model_len=None, prefetch=None):
        """`prefetch` (a tensor or packed weight the next kernel reads) is fetched into L2 while the
        attention streams the history, which it marks first to be evicted."""
        B, hq, d = q.shape
        bs = cache.shape[3]
        if max_model_len is None:
            max_model_len = block_tables.shape[1] * bs
        ms = self.max_splits(max_model_len)
        self.reserve_attention(B, hq, d, max_model_len)
        out = torch.empty(B, hq, d, dtype=q.dtype, device=q.device)
        self.C.paged_decode(q, cache, block_tables, ctx_lens, out, self._part_o, self._part_ml, self._tickets,
                            self.status, ms, self.PART_TOKENS, scale, self.ATTN_STAGES, prefetch_target(prefetch))
        return out

    def prefill_attention(self, q, cache, block_tables, ctx_lens, q_seq, q_pos, scale, tiles=None):
        """Causal attention of the step's new rows over their sequences' paged history (the tcgen05
        prefill kernel). `tiles` ([n, 4] int32 on the device: sequence, first row, rows, first
        position) comes with the step's inputs; without it the tiles are derived here, which reads
        q_seq and q_pos back to the host."""
        if tiles is None:
            tiles = prefill_tiles(q_seq.tolist(), q_pos.tolist(), device=q.device)
        qc = q.contiguous()
        out = torch.empty_like(qc)
        self.C.paged_prefill(qc, cache, block_tables, tiles, out, self.status, scale)
        return out

    def silu_mul(self, gu, interleaved: bool = False):
        out = torch.empty(*gu.shape[:-1], gu.shape[-1] // 2, dtype=gu.dtype, device=gu.device)
        self.C.silu_mul(gu, out, interleaved)
        return out

    def linear_silu(self, x, w, prefetch=None):
        """silu(gate) * up of x . w^T for a gate/up weight interleaved by 64 rows
        (``interleave_gate_up``): one GEMM with the SiLU-mul in its epilogue (each 128-row tile
        holds 64 gates and their up rows)."""
        M = x.shape[0]
        self.reserve_linear()
        out = torch.empty(M, w.shape[0] // 2, dtype=x.dtype, device=x.device)
        wt, wp = weight_args(w)
        self.C.gemm_silu(x, wt, out, self._ws, self._ctr, self.status, self.num_sms, wp, prefetch_target(prefetch))
        return out

    def argmax(self, logits):
        out = torch.empty(logits.shape[0], dtype=torch.int64, device=logits.device)
        self.C.argmax(logits, out)
        return out

    def sample(self, logits, positions, sb):
        """The sampling kernel: the same Gumbel-max draw over the same kept tokens as
        engine.sampling.sample, with the top-p mass summed exactly in fixed point (the host
        sampler's float running sum can differ at the cut-off by a rounding)."""
        out = torch.empty(logits.shape[0], dtype=torch.int64, device=logits.device)
        if logits.dtype not in (torch.bfloat16, torch.float32):
            logits = logits.float()
        if logits.stride(1) != 1:
            logits = logits.contiguous()
        self.C.sample(logits, positions.to(torch.int64).contiguous(), sb.temperature.float().contiguous(),
                      sb.top_k.to(torch.int64).contiguous(), sb.top_p.float().contiguous(),
                      sb.seed.to(torch.int64).contiguous(), out)
        return out

    def check_status(self) -> int:
        """Read (and clear) the status word that bounded waits set; non-zero means a timeout."""
        v = int(self.status.item())
        if v:
            self.status.zero_()
        return v


FP8_MAX = 448.0  # largest finite e4m3


def pack_weight(w: torch.Tensor) -> torch.Tensor:
    """A [N, K] bf16 weight laid out as the GEMM's shared-memory stages: per 128-row tile and 64-wide
    k-block (tile-major), one 16 KB block of 128 rows of 128 bytes whose 16-byte chunk c of row r sits
    at chunk c ^ (r % 8) (the 128-byte swizzle the MMA descriptors name). Rows past N and columns past
    K are zero. One bulk copy per stage then reads the weight front to back."""
    N, K = w.shape
    T, KB = (N + 127) // 128, (K + 63) // 64
    pad = torch.zeros(T * 128, KB * 64, dtype=w.dtype, device=w.device)
    pad[:N, :K] = w
    blocks = pad.view(T, 128, KB, 8, 8).permute(0, 2, 1, 3, 4)  # [T, KB, row, chunk, 8]
    r = torch.arange(128, device=w.device).view(128, 1)
    src = torch.arange(8, device=w.device).view(1, 8) ^ (r % 8)  # stored chunk c' holds logical c' ^ (r % 8)
    out = blocks[:, :, torch.arange(128, device=w.device).view(128, 1), src]
    return out.contiguous().view(torch.uint8).view(-1)


def unpack_weight(packed: torch.Tensor, n: int, k: int) -> torch.Tensor:
    """The [n, k] bf16 weight of ``pack_weight`` (the chunk swizzle is its own inverse)."""
    T, KB = (n + 127) // 128, (k + 63) // 64
    blocks = packed.view(torch.bfloat16).view(T, KB, 128, 8, 8)
    r = torch.arange(128, device=packed.device).view(128, 1)
    src = torch.arange(8, device=packed.device).view(1, 8) ^ (r % 8)
    rows = blocks[:, :, r, src].permute(0, 2, 1, 3, 4).reshape(T * 128, KB * 64)
    return rows[:n, :k].contiguous()


class PackedWeight:
    """A bf16 [N, K] weight kept only as ``pack_weight(w)``, which the GEMM streams by one bulk copy
    per stage. ``carrier`` is a stride-0 [N, K] view of one element: it carries the shape through
    the bindings, whose kernels then read ``packed`` alone."""

    __slots__ = ("packed", "n", "k", "carrier")

    def __init__(self, w: torch.Tensor):
        self.n, self.k = (int(v) for v in w.shape)
        self.packed = pack_weight(w)
        self.carrier = torch.zeros(1, dtype=w.dtype, device=w.device).expand(self.n, self.k)

    @property
    def shape(self) -> torch.Size:
        return torch.Size((self.n, self.k))

    @property
    def dtype(self):
        return self.carrier.dtype

    @property
    def device(self):
        return self.carrier.device

    def dim(self) -> int:
        return 2

    def numel(self) -> int:
        return self.n * self.k

    def element_size(self) -> int:
        return self.carrier.element_size()

    def unpack(self) -> torch.Tensor:
        return unpack_weight(self.packed, self.n, self.k)


def weight_args(w):
    """(the tensor a binding takes as `w`, the packed blocks or None)."""
    return (w.carrier, w.packed) if isinstance(w, PackedWeight) else (w, None)


# off by default: with the weights' and the history's lines marked evict-first, fetching the next
# kernel's weights into L2 during the kernel before measured slower in the decode step
L2_PREFETCH = os.environ.get("ES_L2_PREFETCH", "0") == "1"


def prefetch_target(t):
    """The tensor whose bytes a kernel fetches into L2 for the next kernel (None: nothing), from a
    tensor or a packed weight; ES_L2_PREFETCH=1 turns the prefetches on."""
    if t is None or not L2_PREFETCH:
        return None
    return t.packed if isinstance(t, PackedWeight) else t


def dense(w) -> torch.Tensor:
    """The [N, K] tensor of a weight, packed or not."""
    return w.unpack() if isinstance(w, PackedWeight) else w


def quantize_weight_fp8(w: torch.Tensor, block: int = 128) -> tuple[torch.Tensor, torch.Tensor]:
    """[N, K] weight -> (e4m3 [N, K], fp32 scales [ceil(N/128), K/128]): each 128 x 128 block's
    scale maps its largest magnitude to the e4m3 maximum."""
    N, K = w.shape
    assert K % block == 0, "K must be a multiple of 128"
    nb = (N + block - 1) // block
    wf = w.float()
    if N % block:
        wf = torch.cat([wf, torch.zeros(nb * block - N, K, dtype=wf.dtype, device=wf.device)])
    blocks = wf.view(nb, block, K // block, block)
    amax = blocks.abs().amax(dim=(1, 3))
    scale = torch.where(amax > 0, amax / FP8_MAX, torch.ones_like(amax))
    q = (blocks / scale[:, None, :, None]).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)
    return q.view(nb * block, K)[:N].contiguous(), scale.contiguous()


def dequantize_fp8(q: torch.Tensor, scale: torch.Tensor, rows_per_scale: int, block: int = 128) -> torch.Tensor:
    """The fp32 values of e4m3 data [R, K] with one scale per (rows_per_scale rows, 128 columns)."""
    R, K = q.shape
    s = scale.repeat_interleave(rows_per_scale, dim=0)[:R].repeat_interleave(block, dim=1)
    return q.float() * s


def quantize_act_fp8(x: torch.Tensor, block: int = 128) -> tuple[torch.Tensor, torch.Tensor]:
    """Per token and 128-wide block (the kernel's rule, restated): (e4m3 [M, K], fp32 [M, K/128])."""
    M, K = x.shape
    xb = x.float().view(M, K // block, block)
    amax = xb.abs().amax(dim=2)
    scale = torch.where(amax > 0, amax * (1.0 / FP8_MAX), torch.ones_like(amax))
    q = (xb * (1.0 / scale)[:, :, None]).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)
    return q.view(M, K), scale


def interleave_gate_up(gu: torch.Tensor, run: int = 64) -> torch.Tensor:
    """[2I, H] gate rows then up rows -> runs of `run` gate rows each followed by the matching up
    rows: the layout whose 128-row GEMM tiles hold a gate and its up projection together."""
    inter = gu.shape[0] // 2
    g, u = gu[:inter], gu[inter:]
    return torch.stack([g.reshape(inter // run, run, -1), u.reshape(inter // run, run, -1)], 1).reshape(gu.shape)


def deinterleave_gate_up(w: torch.Tensor, run: int = 64) -> torch.Tensor:
    """The inverse of ``interleave_gate_up``."""
    inter = w.shape[0] // 2
    v = w.reshape(inter // run, 2, run, -1)
    return torch.cat([v[:, 0].reshape(inter, -1), v[:, 1].reshape(inter, -1)], 0)


PREFILL_ROWS = 128  # query rows per tile of the prefill kernel


def prefill_tiles(q_seq, q_pos, device=None, rows: int = PREFILL_ROWS) -> torch.Tensor:
    """The prefill kernel's work list from each row's sequence index and position (rows of one
    sequence consecutive, positions increasing by one): tiles of at most `rows` rows, as int32
    [n, 4] (sequence, first row, rows, first position), the longest history first so the causal
    tail of long sequences starts early."""
    tiles = []
    t, T = 0, len(q_seq)
    while t < T:
        s = q_seq[t]
        e = t
        while e < T and q_seq[e] == s:
            e += 1
        for r0 in range(t, e, rows):
            n = min(rows, e - r0)
            tiles.append((int(s), r0, n, int(q_pos[r0])))
        t = e
    tiles.sort(key=lambda x: -(x[3] + x[2]))
    out = torch.tensor(tiles or [(0, 0, 0, 0)], dtype=torch.int32)[: len(tiles)]
    return out.to(device, non_blocking=True) if device is not None else out


_CACHE: dict[str, object] = {}


def ops_for(device: torch.device | str):
    dev = torch.device(device)
    key = str(dev)
    if key not in _CACHE:
        _CACHE[key] = KernelOps(dev) if dev.type == "cuda" else RefOps(dev)
    return _CACHE[key]


def softmax_scale(head_dim: int) -> float:
    return 1.0 / math.sqrt(head_dim)
