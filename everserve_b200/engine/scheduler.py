"""Continuous-batching scheduler.

Each step is either a prefill step (new requests' uncomputed tokens, as many requests as the token
and block budgets allow) or a decode-shaped step (every running request feeds exactly one token).
Requests join and leave the running batch between steps. When a decode step cannot get a KV block,
the most recently admitted request is preempted: its blocks are freed and it is recomputed later
by a prefill over its prompt and outputs.

The plan a step produces (:class:`StepPlan`) is all a worker needs to run the forward: token ids,
start positions and block tables. The executor ships it to every worker; the KV connector sees it
to know which slots the step writes.
"""

from __future__ import annotations

from collections import deque
from dataclasses import dataclass, field

from .block_manager import BlockManager
from .request import Request, Status


@dataclass
class ScheduledReq:
    req_id: str
    token_ids: list[int]
    start_pos: int
    block_table: list[int]
    sample: bool  # the last fed position is the request's last token: its sample is a new output
    expect: int | None = None  # replayed position: the output already recorded there
    sampling: tuple | None = None  # (temperature, top_k, top_p, seed); None: greedy
    bt_version: int = 0  # the request's blocks_version: a staged table is valid while it holds
    logprobs: int | None = None  # how many alternatives' log-probabilities to report (None: none)


@dataclass
class StepPlan:
    step: int
    is_prefill: bool
    reqs: list[ScheduledReq] = field(default_factory=list)

    @property
    def num_tokens(self) -> int:
        return sum(len(r.token_ids) for r in self.reqs)

    def slots(self, block_size: int) -> list[list[int]]:
        out = []
        for r in self.reqs:
            out.append([r.block_table[p // block_size] * block_size + p % block_size
                        for p in range(r.start_pos, r.start_pos + len(r.token_ids))])
        return out


class Scheduler:
    def __init__(self, blocks: BlockManager, max_batch: int = 64, max_prefill_tokens: int = 8192,
                 max_model_len: int = 4096):
        self.bm = blocks
        self.max_batch = max_batch
        self.max_prefill_tokens = max_prefill_tokens
        self.max_model_len = max_model_len
        self.waiting: deque[Request] = deque()
        self.running: list[Request] = []
        self.requests: dict[str, Request] = {}
        self.step_id = 0
        self._arrivals = 0
        self.preemptions: list[str] = []
        self.one_token_replay = False  # after a resume: decode shape until every request caught up

    def add(self, req: Request) -> None:
        if len(req.prompt) == 0:
            raise ValueError("empty prompt")
        if len(req.prompt) + req.params.max_tokens > self.max_model_len:
            raise ValueError(f"request needs {len(req.prompt) + req.params.max_tokens} positions, "
                             f"max_model_len is {self.max_model_len}")
        req.arrival = self._arrivals
        self._arrivals += 1
        self.requests[req.req_id] = req
        self.waiting.append(req)

    def has_work(self) -> bool:
        return bool(self.waiting or self.running)

    # ---- planning --------------------------------------------------------------------------------
    def schedule(self) -> StepPlan | None:
        self.preemptions = []
        plan = None if self.one_token_replay else self._schedule_prefill()
        if plan is None:
            plan = self._schedule_decode()
        if plan is not None:
            plan.step = self.step_id
            self.step_id += 1
        return plan

    def _schedule_prefill(self) -> StepPlan | None:
        if not self.waiting:
            return None
        plan = StepPlan(step=0, is_prefill=True)
        budget = self.max_prefill_tokens
        while self.waiting and len(self.running) < self.max_batch:
            req = self.waiting[0]
            n = req.num_tokens - req.num_computed
            if plan.reqs and n > budget:
                break
            if not self.bm.can_grow(req.blocks, req.num_tokens):
                break
            self.waiting.popleft()
            self.bm.grow(req.blocks, req.num_tokens)
            req.status = Status.RUNNING
            self.running.append(req)
            plan.reqs.append(ScheduledReq(req.req_id, req.tokens[req.num_computed:], req.num_computed,
                                          list(req.blocks), sample=True,
                                          sampling=req.params.sampling_key(req.req_id),
                                          logprobs=req.params.logprobs))
            budget -= n
        return plan if plan.reqs else None

    def _schedule_decode(self) -> StepPlan | None:
        if not self.running:
            return None
        # every running request feeds position num_computed; make sure its block exists
        self.running.sort(key=lambda r: r.arrival)
        i = 0
        bs = self.bm.block_size
        while i < len(self.running):
            req = self.running[i]
            if req.num_computed < len(req.blocks) * bs:  # its next position is in a block it holds
                i += 1
                continue
            if self.bm.can_grow(req.blocks, req.num_computed + 1):
                self.bm.grow(req.blocks, req.num_computed + 1)
                i += 1
                continue
            victim = self.running.pop()  # youngest
            self._preempt(victim)
            if victim is req:
                continue
        if not self.running:
            return None
        plan = StepPlan(step=0, is_prefill=False)
        for req in self.running[: self.max_batch]:
            p = req.num_computed
            last = p == req.num_tokens - 1
            # the block list is handed over, not copied: a plan is staged before the next schedule
            # grows it, and growth only appends
            plan.reqs.append(ScheduledReq(req.req_id, [req.token_at(p)], p, req.blocks, sample=last,
                                          bt_version=req.blocks_version,
                                          expect=None if last else req.token_at(p + 1),
                                          sampling=req.params.sampling_key(req.req_id),
                                          logprobs=req.params.logprobs if last else None))
        return plan

    def _preempt(self, req: Request) -> None:
        self.bm.free(req.blocks)
        req.blocks_version += 1
        req.num_computed = 0
        req.committed = 0
        req.status = Status.WAITING
        self.waiting.appendleft(req)
        self.preemptions.append(req.req_id)

    # ---- results ---------------------------------------------------------------------------------
    def update(self, plan: StepPlan, sampled: list[int], logprobs: list | None = None) -> list[tuple[str, int | None, bool]]:
        """Apply one step's sampled ids (and each row's log-probability record when the step made
        them); returns (req_id, new token or None, finished) per request."""
        out = []
        for i, (sr, tok) in enumerate(zip(plan.reqs, sampled)):
            req = self.requests[sr.req_id]
            req.num_computed = sr.start_pos + len(sr.token_ids)
            new = None
            if sr.sample:
                req.outputs.append(int(tok))
                new = int(tok)
                if sr.logprobs is not None and logprobs is not None:
                    lp, top = logprobs[i]
                    req.logprobs.append((lp, top[: sr.logprobs]))
            elif sr.expect is not None and int(tok) != sr.expect:
                req.replay_mismatches += 1
            fin = sr.sample and req.done_generating()
            if fin:
                req.status = Status.FINISHED
                self.running.remove(req)
                self.bm.free(req.blocks)
                req.blocks_version += 1
            out.append((sr.req_id, new, fin))
        if self.one_token_replay and all(r.num_computed >= r.num_tokens - 1 for r in self.running):
            self.one_token_replay = False
        return out

    # ---- resume ----------------------------------------------------------------------------------
    def resume_from_committed(self) -> None:
        """After a membership change: restart every running request at its committed point.

        A request with nothing committed goes back to the waiting queue (its prompt is prefilled
        again, in prefill shape as the first time); the others restart at ``min(committed, n - 1)``
        and replay their uncommitted positions one per step in decode shape.
        """
        for req in sorted([r for r in self.running if r.committed == 0], key=lambda r: -r.arrival):
            self.running.remove(req)
            self.bm.free(req.blocks)
            req.blocks_version += 1
            req.num_computed = 0
            req.status = Status.WAITING
            self.waiting.appendleft(req)
        for req in self.running:
            req.num_computed = req.resume_point()
        self.one_token_replay = any(r.num_computed < r.num_tokens - 1 for r in self.running)
