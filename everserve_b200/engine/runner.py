"""Model runner: one rank's forward over its KV cache, with CUDA graphs for decode.

Inputs reach the device in one pass per step: the host packs ids, positions, slots and context
lengths into one pinned int64 buffer and the block tables into one pinned int32 buffer, and two
asynchronous copies land them in the static device buffers the captured graphs read. Decode runs
as a graph replay per batch bucket (padded rows have slot -1 and context length 0, which every
kernel skips). Prefill runs eagerly.

``decode_loop(k)`` runs k decode steps with no host round trip: after each replay a small kernel
turns the sampled ids into the next step's inputs (position + 1, the slot from the block table).
The engine uses it for multi-step decoding when no request can finish inside the window.

A batch with a sampled (temperature > 0) row stages its rows' sampling parameters into static
buffers too and runs its own graph per bucket; greedy batches keep the greedy graphs.
"""

from __future__ import annotations

import torch

from ..models.llama import DecoderLM, StepInput
from ..ops import prefill_tiles
from .sampling import SamplingBatch
from .scheduler import StepPlan

_BUCKETS = (1, 2, 4, 8, 16, 24, 32, 48, 64, 96, 128, 192, 256)


class ModelRunner:
    def __init__(self, model: DecoderLM, num_blocks: int, block_size: int = 16, max_batch: int = 64,
                 max_model_len: int = 4096, use_graphs: bool = True):
        self.model = model
        self.device = model.device
        self.block_size = block_size
        self.num_blocks = num_blocks
        self.max_batch = max_batch
        self.max_model_len = max_model_len
        self.max_blocks = (max_model_len + block_size - 1) // block_size
        self.use_graphs = use_graphs and self.device.type == "cuda"
        shape = model.kv_cache_shape(num_blocks, block_size)
        self.caches = [torch.zeros(shape, dtype=model.dtype, device=self.device) for _ in range(model.l1 - model.l0)]
        self.buckets = [b for b in _BUCKETS if b < max_batch] + [max_batch]
        B = max_batch
        pin = self.device.type == "cuda"
        # host staging: rows = ids, positions, slots, ctx_lens
        self.h_i64 = torch.zeros(4, B, dtype=torch.int64, pin_memory=pin)
        self.h_bt = torch.zeros(B, self.max_blocks, dtype=torch.int32, pin_memory=pin)
        self.h_i64_np = self.h_i64.numpy()
        self.h_bt_np = self.h_bt.numpy()
        self._bt_rows = [(None, 0)] * B  # per staging row: ((request, table version), entries written)
        self.h2d_bytes = 0
        self.d_i64 = torch.zeros(4, B, dtype=torch.int64, device=self.device)
        self.d_bt = torch.zeros(B, self.max_blocks, dtype=torch.int32, device=self.device)
        self.d_ctx32 = torch.zeros(B, dtype=torch.int32, device=self.device)
        self.d_seq = torch.arange(B, dtype=torch.int64, device=self.device)
        # sampling parameters: rows temperature, top_p (float32) and top_k, seed (int64)
        self.h_sf = torch.zeros(2, B, dtype=torch.float32, pin_memory=pin)
        self.h_si = torch.zeros(2, B, dtype=torch.int64, pin_memory=pin)
        self.d_sf = torch.zeros(2, B, dtype=torch.float32, device=self.device)
        self.d_si = torch.zeros(2, B, dtype=torch.int64, device=self.device)
        self.graphs: dict[tuple[int, bool], torch.cuda.CUDAGraph] = {}  # (bucket, sampled)
        self.graph_out: dict[tuple[int, bool], torch.Tensor] = {}
        self.h_out = torch.zeros(B, dtype=torch.int64, pin_memory=pin)
        # pipelined steps: two pinned result buffers (a step's ids are read while the next runs), and
        # the event after the last staged host -> device copies (the pinned staging buffers are
        # rewritten only once those copies have run)
        self.h_ids = [torch.zeros(B, dtype=torch.int64, pin_memory=pin) for _ in range(2)]
        self._ids_slot = 0
        self._staged = None
        self._pool = None
        self.last_logprobs = None  # (chosen [B], top ids [B, k], top values [B, k]) of the last step
        if self.device.type == "cuda" and model.ops.kind == "kernel":
            model.ops.reserve_linear(max(max_batch, 1), model.linear_shapes())
            model.ops.reserve_attention(max_batch, model.hq, model.d, max_model_len)

    # ---- inputs ----------------------------------------------------------------------------------
    def _bucket(self, n: int) -> int:
        for b in self.buckets:
            if b >= n:
                return b
        raise ValueError(f"batch {n} above max_batch {self.max_batch}")

    @staticmethod
    def sampled(plan: StepPlan) -> bool:
        return any(r.sampling is not None for r in plan.reqs)

    @staticmethod
    def logprobs_k(plan: StepPlan) -> int | None:
        ks = [r.logprobs for r in plan.reqs if r.logprobs is not None]
        return max(ks) if ks else None

    def logprob_rows(self, n: int) -> list | None:
        """The last step's log-probability records of its first n rows, on the host:
        [(log-probability, [(token, log-probability), ...]), ...]; None when it made none."""
        if self.last_logprobs is None:
            return None
        chosen, idx, val = (t[:n].cpu() for t in self.last_logprobs)
        return [(float(chosen[i]), list(zip(idx[i].tolist(), val[i].tolist()))) for i in range(len(chosen))]

    def _stage_sampling(self, plan: StepPlan, b: int) -> None:
        hf, hi = self.h_sf.numpy(), self.h_si.numpy()
        hf[0, :b], hf[1, :b], hi[0, :b], hi[1, :b] = 0.0, 1.0, 0, 0
        for i, r in enumerate(plan.reqs):
            if r.sampling is not None:
                hf[0, i], hi[0, i], hf[1, i], hi[1, i] = r.sampling
        self.d_sf[:, :b].copy_(self.h_sf[:, :b], non_blocking=True)
        self.d_si[:, :b].copy_(self.h_si[:, :b], non_blocking=True)
        self.h2d_bytes += 2 * b * 4 + 2 * b * 8

    def _sampling_batch(self, b: int) -> SamplingBatch:
        return SamplingBatch(temperature=self.d_sf[0, :b], top_k=self.d_si[0, :b], top_p=self.d_sf[1, :b],
                             seed=self.d_si[1, :b])

    def stage_decode(self, plan: StepPlan) -> int:
        """Copy a decode plan's inputs into the static device buffers; returns the bucket size."""
        if self._staged is not None:
            self._staged.synchronize()  # the previous step's copies have read the staging buffers
            self._staged = None
        n = len(plan.reqs)
        b = self._bucket(n)
        h = self.h_i64_np
        bs = self.block_size
        hbt = self.h_bt_np
        ids, pos, slots = [], [], []
        rows = self._bt_rows
        for i, r in enumerate(plan.reqs):
            p = r.start_pos
            bt = r.block_table
            ids.append(r.token_ids[0])
            pos.append(p)
            slots.append(bt[p // bs] * bs + p % bs)
            # a row's block table is written only where it changed (a request keeps its row while
            # it runs; its table grows by appending)
            key = (r.req_id, r.bt_version)
            done = rows[i][1] if rows[i][0] == key else 0
            if len(bt) > done:
                hbt[i, done : len(bt)] = bt[done:]
            rows[i] = (key, len(bt))
        for i in range(n, b):
            rows[i] = (None, 0)
        h[:, n:b] = 0
        h[2, n:b] = -1
        if n:
            h[0, :n] = ids
            h[1, :n] = pos
            h[2, :n] = slots
            h[3, :n] = h[1, :n] + 1
        self.d_i64[:, :b].copy_(self.h_i64[:, :b], non_blocking=True)
        self.d_bt[:b].copy_(self.h_bt[:b], non_blocking=True)
        self.h2d_bytes = 4 * b * 8 + b * self.max_blocks * 4
        if self.sampled(plan):
            self._stage_sampling(plan, b)
        if self.device.type == "cuda":
            self._staged = torch.cuda.Event()
            self._staged.record(torch.cuda.current_stream(self.device))
        return b

    def _decode_input(self, b: int, sampled: bool = False) -> StepInput:
        self.d_ctx32[:b].copy_(self.d_i64[3, :b])
        return StepInput(ids=self.d_i64[0, :b], positions=self.d_i64[1, :b], slots=self.d_i64[2, :b],
                         block_tables=self.d_bt[:b], ctx_lens=self.d_ctx32[:b], q_seq=self.d_seq[:b],
                         logits_idx=self.d_seq[:b], is_decode=True, max_model_len=self.max_model_len,
                         sampling=self._sampling_batch(b) if sampled else None)

    def prefill_input(self, plan: StepPlan) -> StepInput:
        ids, pos, slots, seq, last, ctx = [], [], [], [], [], []
        bs = self.block_size
        bt = torch.zeros(len(plan.reqs), self.max_blocks, dtype=torch.int32)
        for i, r in enumerate(plan.reqs):
            n = len(r.token_ids)
            ids += r.token_ids
            ps = list(range(r.start_pos, r.start_pos + n))
            pos += ps
            slots += [r.block_table[p // bs] * bs + p % bs for p in ps]
            seq += [i] * n
            last.append(len(ids) - 1)
            ctx.append(r.start_pos + n)
            bt[i, : len(r.block_table)] = torch.tensor(r.block_table, dtype=torch.int32)
        dev = self.device
        t = lambda v, dt=torch.int64: torch.tensor(v, dtype=dt).to(dev, non_blocking=True)  # noqa: E731
        sb = None
        if self.sampled(plan):
            ps = [r.sampling or (0.0, 0, 1.0, 0) for r in plan.reqs]
            sb = SamplingBatch(temperature=t([p[0] for p in ps], torch.float32), top_k=t([p[1] for p in ps]),
                               top_p=t([p[2] for p in ps], torch.float32), seed=t([p[3] for p in ps]))
        tiles = prefill_tiles(seq, pos, device=dev) if self.model.ops.kind == "kernel" else None
        return StepInput(ids=t(ids), positions=t(pos), slots=t(slots), block_tables=bt.to(dev),
                         ctx_lens=t(ctx, torch.int32), q_seq=t(seq), logits_idx=t(last), is_decode=False,
                         max_model_len=self.max_model_len, sampling=sb, prefill_tiles=tiles)

    # ---- forward ---------------------------------------------------------------------------------
    def forward(self, inp: StepInput, hidden=None, residual=None):
        return self.model.forward(inp, self.caches, hidden, residual)

    def execute(self, plan: StepPlan, hidden=None, residual=None):
        """Run one step. Last stage: sampled ids (device int64 [n]); other stages: (hidden, residual).

        A step asked for log-probabilities runs eagerly and leaves them in ``last_logprobs``."""
        k = self.logprobs_k(plan)
        self.last_logprobs = None
        self.model.step_logprobs = None
        if plan.is_prefill:
            inp = self.prefill_input(plan)
            inp.logprobs_k = k
            out = self.forward(inp, hidden, residual)
            self.last_logprobs = self.model.step_logprobs if k is not None else None
            return out
        n = len(plan.reqs)
        b = self.stage_decode(plan)
        key = (b, self.sampled(plan))
        if k is not None:
            inp = self._decode_input(*key)
            inp.logprobs_k = k
            out = self.forward(inp, hidden, residual)
            self.last_logprobs = self.model.step_logprobs
            if isinstance(out, tuple):
                return out[0][:n], out[1][:n]
            return out[:n]
        if self.use_graphs and self.model.last and self.model.first:
            g = self.graphs.get(key)
            if g is None:
                self._capture(*key)
                g = self.graphs[key]
            g.replay()
            return self.graph_out[key][:n]
        out = self.forward(self._decode_input(*key), hidden, residual)
        if isinstance(out, tuple):
            return out[0][:n], out[1][:n]
        return out[:n]

    def _capture(self, b: int, sampled: bool = False) -> None:
        # warm up on a side stream (allocator and lazily configured kernels), then capture
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        saved = self.d_i64[:, :b].clone(), self.d_bt[:b].clone()
        with torch.cuda.stream(s):
            for _ in range(2):
                self.forward(self._decode_input(b, sampled))
        torch.cuda.current_stream(self.device).wait_stream(s)
        self.d_i64[:, :b].copy_(saved[0])
        self.d_bt[:b].copy_(saved[1])
        g = torch.cuda.CUDAGraph()
        if self._pool is None:
            self._pool = torch.cuda.graph_pool_handle()
        with torch.cuda.graph(g, pool=self._pool):
            out = self.forward(self._decode_input(b, sampled))
        self.graphs[(b, sampled)] = g
        self.graph_out[(b, sampled)] = out

    def release_graphs(self) -> None:
        """Drop every captured graph (a graph holding NCCL calls must go before the process group)."""
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        self.graphs.clear()
        self.graph_out.clear()
        self._pool = None

    def capture_all(self) -> None:
        if not self.use_graphs:
            return
        for b in self.buckets:
            if (b, False) not in self.graphs:
                self._capture(b)

    # ---- multi-step decode -----------------------------------------------------------------------
    def decode_loop(self, plan: StepPlan, k: int, after_step=None) -> torch.Tensor:
        """k decode steps from `plan` without host round trips; returns device ids [k, n].

        Every request's block table must already cover positions start_pos .. start_pos + k - 1.
        ``after_step(i)`` is called on the host once step i's kernels are enqueued (the KV
        connector enqueues that step's commit behind them).
        """
        n = len(plan.reqs)
        b = self.stage_decode(plan)
        key = (b, self.sampled(plan))
        out = torch.empty(k, n, dtype=torch.int64, device=self.device)
        if self.use_graphs and key not in self.graphs:
            self._capture(*key)
        bs = self.block_size
        for i in range(k):
            if self.use_graphs:
                self.graphs[key].replay()
                ids = self.graph_out[key]
            else:
                ids = self.forward(self._decode_input(*key))
            out[i] = ids[:n]
            if after_step is not None:
                after_step(i)
            if i + 1 < k:
                self._advance(b, ids, bs)
        return out

    def _advance(self, b: int, ids: torch.Tensor, bs: int) -> None:
        ops = self.model.ops
        if ops.kind == "kernel":
            ops.C.decode_advance(self.d_i64, ids, self.d_bt, b, bs)
            return
        d = self.d_i64
        live = d[3, :b] > 0
        d[0, :b] = torch.where(live, ids[:b], d[0, :b])
        d[1, :b] += live.long()
        d[3, :b] += live.long()
        pos = d[1, :b]
        blk = self.d_bt[:b].gather(1, (pos // bs).clamp(max=self.max_blocks - 1)[:, None].to(torch.int64))[:, 0]
        d[2, :b] = torch.where(live, blk.long() * bs + pos % bs, torch.full_like(pos, -1))

    # ---- pipelined decode -------------------------------------------------------------------------
    def launch_next(self, plan: StepPlan, prev_ids: torch.Tensor) -> torch.Tensor:
        """Enqueue the decode step `plan` whose fed token of row i is the previous step's sampled id
        `prev_ids[i]`, still on the device; returns its sampled ids (device [n]). Positions, slots,
        context lengths, block tables and sampling parameters go from the host as in `execute`; only
        the ids row is taken on the device, so the step can be enqueued before the previous step's
        ids reach the host."""
        n = len(plan.reqs)
        b = self.stage_decode(plan)
        self.d_i64[0, :n].copy_(prev_ids[:n])
        key = (b, self.sampled(plan))
        if self.use_graphs and self.model.last and self.model.first:
            if key not in self.graphs:
                self._capture(*key)
            self.graphs[key].replay()
            return self.graph_out[key][:n]
        return self.forward(self._decode_input(*key))[:n]

    def start_fetch(self, ids: torch.Tensor):
        """Start the device -> pinned host copy of a step's sampled ids (behind the work enqueued so
        far); `collect` waits for that copy alone. Two buffers alternate, so a step's ids can be in
        flight while the previous step's are read."""
        n = ids.numel()
        self._ids_slot ^= 1
        buf = self.h_ids[self._ids_slot]
        if n > buf.numel():
            buf = self.h_ids[self._ids_slot] = torch.zeros(n, dtype=torch.int64, pin_memory=self.device.type == "cuda")
        buf[:n].copy_(ids.reshape(-1), non_blocking=True)
        ev = None
        if self.device.type == "cuda":
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream(self.device))
        return buf, n, ev

    @staticmethod
    def collect(handle) -> list[int]:
        buf, n, ev = handle
        if ev is not None:
            ev.synchronize()
        return buf[:n].tolist()

    def fetch(self, ids: torch.Tensor) -> list[int]:
        """Device -> pinned host copy of sampled ids, synchronised on the copy's stream."""
        n = ids.numel()
        if n > self.h_out.numel():
            self.h_out = torch.zeros(n, dtype=torch.int64, pin_memory=self.device.type == "cuda")
        self.h_out[:n].copy_(ids.reshape(-1), non_blocking=True)
        if self.device.type == "cuda":
            torch.cuda.current_stream(self.device).synchronize()
        return self.h_out[:n].tolist()
