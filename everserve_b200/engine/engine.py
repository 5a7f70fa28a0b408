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

from dataclasses import dataclass
from typing import Callable

import torch

from .block_manager import BlockManager
from .config import EngineConfig
from .request import Request, SamplingParams, Status
from .scheduler import ScheduledReq, Scheduler, StepPlan


@dataclass
class _InFlight:
    """A decode step enqueued before the previous step's ids were read: its plan, its sampled ids on
    the device, and the pending copy of them to the host."""

    plan: StepPlan
    ids: object
    handle: object


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

    # pipelined decode (Engine.step keeps one step in flight): see ModelRunner.launch_next
    def launch_next(self, plan: StepPlan, prev_ids):
        return self.worker.runner.launch_next(plan, prev_ids)

    def start_fetch(self, ids):
        return self.worker.runner.start_fetch(ids)

    def collect(self, handle) -> list[int]:
        return self.worker.runner.collect(handle)

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
        self._ahead: _InFlight | None = None
        self.async_decode = bool(getattr(cfg, "async_decode", False)) and hasattr(self.executor, "launch_next")

    # ---- requests --------------------------------------------------------------------------------
    def add_request(self, prompt: list[int], params: SamplingParams | None = None, req_id: str | None = None) -> str:
        req = Request(list(prompt), params or SamplingParams())
        if req_id is not None:
            req.req_id = req_id
        self.scheduler.add(req)
        return req.req_id

    def has_work(self) -> bool:
        return self.scheduler.has_work() or self._ahead is not None

    def request(self, req_id: str) -> Request:
        return self.scheduler.requests[req_id]

    # ---- stepping --------------------------------------------------------------------------------
    def wrap_step(self, wrapper: Callable[[Callable[[], list]], Callable[[], list]]) -> None:
        """Install a wrapper around the step function (the serving loop's hook point)."""
        self.step_fn = wrapper(self.step_fn)

    def step(self) -> list[tuple[str, int | None, bool]]:
        return self.step_fn()

    def _step(self) -> list[tuple[str, int | None, bool]]:
        if self._ahead is not None:
            return self._step_in_flight()
        plan = self.scheduler.schedule()
        if plan is None:
            return []
        self.last_plan = plan
        if self.connector is not None:
            self.connector.begin_step(plan, self.scheduler)
        ids = self.executor.execute(plan)
        if self._can_run_ahead(plan):
            # read this step's ids while the next step runs
            handle = self.executor.start_fetch(ids)
            if self.connector is not None:
                self.connector.end_step(plan, self.scheduler)
            self._ahead = self._enqueue_next(plan, ids)
            return self._apply(plan, self.executor.collect(handle))
        tokens = self.executor.fetch(ids)
        lp = None
        if any(sr.logprobs is not None for sr in plan.reqs) and hasattr(self.executor, "logprobs"):
            lp = self.executor.logprobs(len(plan.reqs))
        if self.connector is not None:
            self.connector.end_step(plan, self.scheduler)
        return self._apply(plan, tokens, lp)

    def _apply(self, plan: StepPlan, tokens: list[int], lp=None) -> list[tuple[str, int | None, bool]]:
        out = self.scheduler.update(plan, tokens, lp)
        tell = getattr(self.executor, "finished", None)
        for req_id, _, fin in out:
            if fin:
                if self.connector is not None:
                    self.connector.finished(req_id)
                if tell is not None:
                    tell(req_id)
        return out

    # ---- one decode step in flight ---------------------------------------------------------------
    def _can_run_ahead(self, plan: StepPlan) -> bool:
        """Whether the decode step after `plan` (whose ids are not yet applied) may be enqueued now:
        a settled batch (no request waiting, none replaying), every row sampled and without
        log-probabilities, every request still running with room for two more tokens (the pending
        one and the next) within max_tokens and the model length, and the next block available.
        An end-of-sequence token in the pending step is seen only after the next step ran; that
        step's row is then dropped."""
        if not self.async_decode or plan.is_prefill:
            return False
        sch = self.scheduler
        if sch.waiting or sch.one_token_replay or not plan.reqs:
            return False
        need = 0
        bs = self.blocks.block_size
        for sr in plan.reqs:
            req = sch.requests[sr.req_id]
            if not sr.sample or sr.logprobs is not None or req.status is not Status.RUNNING:
                return False
            if len(req.outputs) + 2 > req.params.max_tokens or sr.start_pos + 2 > self.cfg.max_model_len:
                return False
            if sr.start_pos + 1 >= len(req.blocks) * bs:
                need += 1
        return need <= self.blocks.free_blocks

    def _enqueue_next(self, plan: StepPlan, ids) -> _InFlight:
        """Enqueue the step after `plan`: every row one position on, its token the device's sample."""
        sch = self.scheduler
        nxt = StepPlan(step=sch.step_id, is_prefill=False)
        sch.step_id += 1
        for sr in plan.reqs:
            req = sch.requests[sr.req_id]
            p = sr.start_pos + 1
            self.blocks.grow(req.blocks, p + 1)
            # token_ids holds a stand-in until the previous step's ids are read (the device feeds it)
            nxt.reqs.append(ScheduledReq(sr.req_id, [-1], p, req.blocks, sample=True, bt_version=req.blocks_version,
                                         sampling=sr.sampling))
        if self.connector is not None:
            self.connector.begin_step(nxt, sch)
        nids = self.executor.launch_next(nxt, ids)
        handle = self.executor.start_fetch(nids)
        if self.connector is not None:
            self.connector.end_step(nxt, sch)
        return _InFlight(nxt, nids, handle)

    def _step_in_flight(self) -> list[tuple[str, int | None, bool]]:
        """Take the results of the step in flight, first enqueueing the one after it when the batch
        is still settled (no request finished by the last applied step)."""
        cur, self._ahead = self._ahead, None
        self.last_plan = cur.plan
        sch = self.scheduler
        live = [sr for sr in cur.plan.reqs if sch.requests[sr.req_id].status is Status.RUNNING]
        if len(live) == len(cur.plan.reqs) and self._can_run_ahead(cur.plan):
            self._ahead = self._enqueue_next(cur.plan, cur.ids)
        tokens = self.executor.collect(cur.handle)
        keep = StepPlan(step=cur.plan.step, is_prefill=False)
        kept = []
        for sr, tok in zip(cur.plan.reqs, tokens):
            req = sch.requests[sr.req_id]
            if req.status is not Status.RUNNING:
                continue  # finished by the step before: this row was computed past its end
            sr.token_ids = [req.token_at(sr.start_pos)]
            keep.reqs.append(sr)
            kept.append(tok)
        return self._apply(keep, kept)

    def flush(self) -> list[tuple[str, int | None, bool]]:
        """Apply the decode step in flight, if any (before multi-step decoding or a shutdown)."""
        if self._ahead is None:
            return []
        saved, self.async_decode = self.async_decode, False
        try:
            return self._step_in_flight()
        finally:
            self.async_decode = saved

    def decode_steps(self, k: int) -> list[list[int]]:
        """k decode steps on the device with one host round trip (multi-step decoding).

        Valid when every running request is at its last token and none can finish within k steps;
        returns the k new ids of each running request.
        """
        self.flush()
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
        self.flush()
        self.executor.shutdown()


def default_device() -> str:
    return "cuda" if torch.cuda.is_available() else "cpu"
