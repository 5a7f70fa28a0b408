"""The serving engine: scheduler + executor, with the plugin surface of the fault-tolerance layer.

Public API::

    eng = Engine(EngineConfig("llama-3-8b"))
    rid = eng.add_request(prompt_ids, SamplingParams(max_tokens=64))
    while eng.has_work():
        for req_id, token, finished in eng.step():
            ...
    eng.generate([[1, 2, 3]], max_tokens=8)  # -> [[...8 ids...]]

Plugin surface (what the reference's vLLM adapter hooks, adapters/vllm/README.md:5-27):
  * ``step_fn``: the step function the serving loop calls; ``wrap_step`` installs a wrapper (the
    reference's A47 step-loop hook, serving.py:44-86);
  * ``executor``: runs plans on the workers; a fault-tolerant executor replaces it;
  * ``connector``: the KV connector called around each step (begin / end / finished / commit);
  * the collective the model's row-parallel linears go through (``parallel.collective``).
"""

from __future__ import annotations

from typing import Callable

import torch

from .block_manager import BlockManager
from .config import EngineConfig
from .request import Request, SamplingParams
from .scheduler import Scheduler, StepPlan


class LocalExecutor:
    """Runs the plan on this process's worker (tp = pp = 1, or one SPMD rank of a TP group)."""

    def __init__(self, cfg: EngineConfig, rank: int = 0, collective=None):
        from .worker import Worker

        self.worker = Worker(cfg, rank=rank, collective=collective)
        self.num_blocks = self.worker.num_blocks

    def execute(self, plan: StepPlan):
        return self.worker.execute(plan)

    def fetch(self, ids) -> list[int]:
        return self.worker.runner.fetch(ids)

    def logprobs(self, n: int) -> list | None:
        return self.worker.runner.logprob_rows(n)

    def decode_loop(self, plan: StepPlan, k: int, after_step=None):
        return self.worker.runner.decode_loop(plan, k, after_step)

    def shutdown(self):
        """Release the graphs, then the collective's peer mappings and buffers."""
        import gc

        self.worker.runner.release_graphs()
        gc.collect()
        coll = self.worker.tp.collective
        if coll is not None and hasattr(coll, "close"):
            coll.close()


class Engine:
    def __init__(self, cfg: EngineConfig, executor=None, connector=None):
        self.cfg = cfg
        self.executor = executor if executor is not None else LocalExecutor(cfg)
        self.blocks = BlockManager(self.executor.num_blocks, cfg.block_size)
        self.scheduler = Scheduler(self.blocks, cfg.max_batch, cfg.max_prefill_tokens, cfg.max_model_len)
        self.connector = connector
        self.step_fn: Callable[[], list] = self._step
        self.last_plan: StepPlan | None = None

    # ---- requests --------------------------------------------------------------------------------
    def add_request(self, prompt: list[int], params: SamplingParams | None = None, req_id: str | None = None) -> str:
        req = Request(list(prompt), params or SamplingParams())
        if req_id is not None:
            req.req_id = req_id
        self.scheduler.add(req)
        return req.req_id

    def has_work(self) -> bool:
        return self.scheduler.has_work()

    def request(self, req_id: str) -> Request:
        return self.scheduler.requests[req_id]

    # ---- stepping --------------------------------------------------------------------------------
    def wrap_step(self, wrapper: Callable[[Callable[[], list]], Callable[[], list]]) -> None:
        """Install a wrapper around the step function (the serving loop's hook point)."""
        self.step_fn = wrapper(self.step_fn)

    def step(self) -> list[tuple[str, int | None, bool]]:
        return self.step_fn()

    def _step(self) -> list[tuple[str, int | None, bool]]:
        plan = self.scheduler.schedule()
        if plan is None:
            return []
        self.last_plan = plan
        if self.connector is not None:
            self.connector.begin_step(plan, self.scheduler)
        ids = self.executor.execute(plan)
        tokens = self.executor.fetch(ids)
        lp = None
        if any(sr.logprobs is not None for sr in plan.reqs) and hasattr(self.executor, "logprobs"):
            lp = self.executor.logprobs(len(plan.reqs))
        if self.connector is not None:
            self.connector.end_step(plan, self.scheduler)
        out = self.scheduler.update(plan, tokens, lp)
        tell = getattr(self.executor, "finished", None)
        for req_id, _, fin in out:
            if fin:
                if self.connector is not None:
                    self.connector.finished(req_id)
                if tell is not None:
                    tell(req_id)
        return out

    def decode_steps(self, k: int) -> list[list[int]]:
        """k decode steps on the device with one host round trip (multi-step decoding).

        Valid when every running request is at its last token and none can finish within k steps;
        returns the k new ids of each running request.
        """
        sch = self.scheduler
        assert not sch.waiting and not sch.one_token_replay, "multi-step decode needs a settled batch"
        plan = sch.schedule()
        assert plan is not None and not plan.is_prefill
        for sr in plan.reqs:
            req = sch.requests[sr.req_id]
            assert sr.sample and len(req.outputs) + k <= req.params.max_tokens
            self.blocks.grow(req.blocks, req.num_computed + k)
            sr.block_table = list(req.blocks)
        hook = None
        if self.connector is not None and hasattr(self.connector, "decode_hook"):
            hook = self.connector.decode_hook(plan, k)  # every device step's rows are committed
        ids = self.executor.decode_loop(plan, k, hook) if hook is not None else self.executor.decode_loop(plan, k)
        rows = self.executor.fetch(ids)
        n = len(plan.reqs)
        toks = [rows[i * n : (i + 1) * n] for i in range(k)]
        for i in range(k):
            if i > 0:
                for sr in plan.reqs:
                    sr.start_pos += 1
                    r = sch.requests[sr.req_id]
                    sr.token_ids = [r.token_at(r.num_tokens - 1)]
            sch.update(plan, toks[i])
        sch.step_id += k - 1
        return [[toks[i][j] for i in range(k)] for j in range(n)]

    def generate(self, prompts: list[list[int]], max_tokens: int = 16, **sampling) -> list[list[int]]:
        """Every prompt to completion; `sampling`: temperature, top_k, top_p, seed (greedy by default)."""
        ids = [self.add_request(p, SamplingParams(max_tokens=max_tokens, **sampling)) for p in prompts]
        while self.has_work():
            self.step()
        return [self.scheduler.requests[i].outputs for i in ids]

    def shutdown(self):
        self.executor.shutdown()


def default_device() -> str:
    return "cuda" if torch.cuda.is_available() else "cpu"
