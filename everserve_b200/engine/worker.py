"""A worker: one rank's model shard, KV cache and runner.

Rank r of a TP x PP layout sits at pipeline stage r // tp and tensor column r % tp (the
reference's layout rule, core/everserve/comm/layout.py:24-77). The worker builds its shard of the
model, sizes and allocates its paged KV cache, and executes step plans. Between pipeline stages the
hidden state and residual travel through the stage transport (``parallel.exchange.Exchange``).
"""

from __future__ import annotations

import torch

from ..models.llama import DecoderLM, TPGroup
from .config import EngineConfig
from .runner import ModelRunner
from .scheduler import StepPlan


def stage_layers(num_layers: int, pp: int, stage: int) -> tuple[int, int]:
    """Even split of layers over stages; the first stages take the remainder."""
    base, extra = divmod(num_layers, pp)
    start = stage * base + min(stage, extra)
    return start, start + base + (1 if stage < extra else 0)


class Worker:
    def __init__(self, cfg: EngineConfig, rank: int = 0, collective=None, pipe=None, device=None, weights=None):
        self.cfg = cfg
        self.rank = rank
        tp, pp = cfg.tensor_parallel, cfg.pipeline_parallel
        self.stage, self.column = rank // tp, rank % tp
        self.pipe = pipe  # stage transport (send/recv of hidden + residual), None for pp == 1
        self.device = torch.device(device or cfg.device)
        if self.device.type == "cuda":
            if self.device.index is None:
                self.device = torch.device("cuda", torch.cuda.current_device())
            torch.cuda.set_device(self.device)
        self.tp = TPGroup(self.column, tp, collective)
        layers = stage_layers(cfg.model.layers, pp, self.stage)
        init = "none" if (cfg.checkpoint or weights is not None) else "random"
        self.model = DecoderLM(cfg.model, self.device, cfg.dtype, cfg.seed, self.tp, layers, init=init,
                               quant=getattr(cfg, "quant", None),
                               sequence_parallel=getattr(cfg, "sequence_parallel", False))
        if weights is not None:  # a resident copy (pinned host memory): copied in, no init
            for k, t in weights.items():
                self.model._put(k, t)
        elif cfg.checkpoint:
            from ..models.weights import load_hf_checkpoint

            load_hf_checkpoint(self.model, cfg.checkpoint)
        if cfg.moe_routed:
            self.model.enable_routed_experts(max(cfg.max_prefill_tokens, cfg.max_batch))
        self.num_blocks = cfg.num_blocks or self._auto_blocks()
        self.runner = ModelRunner(self.model, self.num_blocks, cfg.block_size, cfg.max_batch, cfg.max_model_len,
                                  cfg.use_cuda_graphs and pp == 1)

    def _auto_blocks(self) -> int:
        per_block = self.model.bytes_per_block(self.cfg.block_size)
        if self.device.type != "cuda":
            return max(64, (self.cfg.max_batch * self.cfg.max_model_len) // self.cfg.block_size + 1)
        free, _ = torch.cuda.mem_get_info(self.device)
        reserve = 4 << 30  # activations, graphs, scratch
        n = int((free * self.cfg.kv_memory_fraction - reserve) // per_block)
        need = (self.cfg.max_batch * self.cfg.max_model_len) // self.cfg.block_size + self.cfg.max_batch
        return max(16, min(n, need))

    @property
    def is_last_stage(self) -> bool:
        return self.model.last

    def execute(self, plan: StepPlan):
        """Run one step of the plan on this rank; the last stage returns the sampled ids (device)."""
        hidden = residual = None
        if not self.model.first:
            hidden, residual = self.pipe.recv_hidden(plan.num_tokens if plan.is_prefill else len(plan.reqs))
        out = self.runner.execute(plan, hidden, residual)
        if not self.model.last:
            self.pipe.send_hidden(*out)
            return None
        return out
