"""The engine on CPU (fp32 reference ops): scheduling, paging, preemption, replay."""

import torch

from everserve_b200.engine import Engine, EngineConfig, SamplingParams
from everserve_b200.engine.block_manager import BlockManager
from everserve_b200.engine.request import Request
from everserve_b200.engine.scheduler import Scheduler
from everserve_b200.engine.worker import stage_layers
from everserve_b200.models.config import TINY_LLAMA, TINY_MIXTRAL, TINY_QWEN


def _engine(model=TINY_LLAMA, **kw):
    args = dict(device="cpu", dtype=torch.float32, max_batch=4, max_model_len=256, num_blocks=64)
    args.update(kw)
    return Engine(EngineConfig(model, **args))


def test_block_manager_lowest_first():
    bm = BlockManager(8, 16)
    a, b = [], []
    bm.grow(a, 20)
    bm.grow(b, 1)
    assert a == [0, 1] and b == [2]
    bm.free(a)
    c = []
    bm.grow(c, 40)
    assert c == [0, 1, 3]
    assert bm.slot(c, 33) == 3 * 16 + 1


def test_generate_matches_recompute():
    for model in (TINY_LLAMA, TINY_QWEN, TINY_MIXTRAL):
        eng = _engine(model)
        out = eng.generate([[1, 2, 3, 4, 5], [7, 8, 9]], max_tokens=6)
        assert all(len(o) == 6 for o in out)
        # a fresh engine prefilling prompt + outputs[:-1] predicts the same last token
        eng2 = _engine(model)
        assert eng2.generate([[1, 2, 3, 4, 5] + out[0][:-1]], max_tokens=1)[0] == [out[0][-1]]


def test_batching_does_not_change_tokens():
    prompts = [[i, i + 3, i + 5] for i in range(6)]
    together = _engine(max_batch=6).generate(prompts, max_tokens=5)
    alone = [_engine(max_batch=1).generate([p], max_tokens=5)[0] for p in prompts]
    assert together == alone


def test_preemption_recomputes():
    eng = _engine(num_blocks=6, max_batch=4)
    prompts = [[1] * 30, [2] * 30, [3] * 30]
    out = eng.generate(prompts, max_tokens=20)
    ref = [_engine(num_blocks=64).generate([p], max_tokens=20)[0] for p in prompts]
    assert out == ref


def test_resume_replays_exactly():
    eng = _engine()
    ids = [eng.add_request([5, 6, 7, 8], SamplingParams(max_tokens=12)) for _ in range(2)]
    for _ in range(7):
        eng.step()
    for i in ids:
        eng.request(i).committed = 6  # the store holds 6 positions
    before = [list(eng.request(i).outputs) for i in ids]
    eng.scheduler.resume_from_committed()
    while eng.has_work():
        eng.step()
    for i, b in zip(ids, before):
        r = eng.request(i)
        assert r.outputs[: len(b)] == b
        assert r.replay_mismatches == 0
    ref = _engine().generate([[5, 6, 7, 8]], max_tokens=12)[0]
    assert eng.request(ids[0]).outputs == ref


def test_stage_layers():
    assert stage_layers(24, 2, 0) == (0, 12) and stage_layers(24, 2, 1) == (12, 24)
    assert stage_layers(5, 2, 0) == (0, 3) and stage_layers(5, 2, 1) == (3, 5)


def test_scheduler_rejects_long():
    s = Scheduler(BlockManager(4, 16), max_model_len=32)
    try:
        s.add(Request([1] * 30, SamplingParams(max_tokens=10)))
    except ValueError:
        return
    raise AssertionError("expected ValueError")


def test_async_decode_matches_sync():
    """Engine.step with one decode step in flight (the next step enqueued before the last step's
    ids are read) gives the same tokens as the synchronous loop: greedy and seeded sampling,
    requests ending on their length at different steps and on an end-of-sequence token, requests
    joining mid-run, and the KV connector sees the same commits."""

    class Log:
        def __init__(self):
            self.commits, self.done = [], []

        def begin_step(self, plan, scheduler):
            pass

        def end_step(self, plan, scheduler):
            self.commits.append(sorted((r.req_id, r.start_pos + len(r.token_ids)) for r in plan.reqs))

        def finished(self, req_id):
            self.done.append(req_id)

    def run(async_decode, eos=None):
        eng = _engine(max_batch=4, async_decode=async_decode)
        log = Log()
        eng.connector = log
        sp = [SamplingParams(max_tokens=9), SamplingParams(max_tokens=4, temperature=0.8, seed=3),
              SamplingParams(max_tokens=12, temperature=1.1, top_k=5, seed=7)]
        if eos is not None:
            sp[0] = SamplingParams(max_tokens=30, eos_id=eos, ignore_eos=False)
        ids = [eng.add_request([3 + i, 9, 4 + 2 * i], p) for i, p in enumerate(sp)]
        steps = 0
        while eng.has_work():
            eng.step()
            steps += 1
            if steps == 5:  # a request joins while the others decode
                ids.append(eng.add_request([11, 12], SamplingParams(max_tokens=6)))
        outs = [eng.request(r).outputs for r in ids]
        # requests by their index (ids differ between engines); commits per request, in order
        index = {r: i for i, r in enumerate(ids)}
        per = {}
        for c in log.commits:
            for rid, n in c:
                per.setdefault(index[rid], []).append(n)
        return outs, per, sorted(index[r] for r in log.done), eng

    sync_out, sync_commits, sync_done, _ = run(False)
    async_out, async_commits, async_done, eng = run(True)
    assert async_out == sync_out
    assert async_done == sync_done
    for rid, ns in sync_commits.items():
        # the asynchronous loop may commit one row past a request's end (computed, then dropped)
        got = async_commits[rid]
        assert got[: len(ns)] == ns and len(got) <= len(ns) + 1
    assert eng.async_decode
    # an end-of-sequence token: the step already in flight for that request is dropped
    eos = sync_out[0][2]
    s_out, _, _, _ = run(False, eos=eos)
    a_out, _, _, _ = run(True, eos=eos)
    assert a_out == s_out and s_out[0][-1] == eos and len(s_out[0]) <= 3


def _run_all(eng, prompts, params):
    ids = [eng.add_request(p, sp) for p, sp in zip(prompts, params)]
    while eng.has_work():
        eng.step()
    return [eng.request(r) for r in ids]


def test_async_decode_under_block_pressure():
    """With few KV blocks the asynchronous loop must not take the block the scheduler would have
    used (it enqueues a step ahead only when the blocks it needs are free): preemptions recompute,
    and the tokens equal the synchronous loop's and a roomy engine's."""
    prompts = [[1] * 30, [2] * 30, [3] * 30]
    params = [SamplingParams(max_tokens=20) for _ in prompts]
    outs = {}
    for async_decode in (False, True):
        eng = _engine(num_blocks=6, max_batch=4, async_decode=async_decode)
        outs[async_decode] = [r.outputs for r in _run_all(eng, prompts, params)]
        assert eng.blocks.free_blocks == 6  # every block given back
    roomy = [r.outputs for r in _run_all(_engine(num_blocks=64), prompts, params)]
    assert outs[True] == outs[False] == roomy


def test_async_decode_with_logprobs_and_multistep():
    """A request asking for log-probabilities keeps its batch synchronous (the records come from the
    step's logits); multi-step decoding after asynchronous steps first applies the step in flight.
    Both give the synchronous loop's tokens and records."""
    def run(async_decode):
        eng = _engine(async_decode=async_decode)
        a = eng.add_request([4, 5, 6], SamplingParams(max_tokens=6, logprobs=2))
        b = eng.add_request([7, 8], SamplingParams(max_tokens=6))
        while eng.has_work():
            eng.step()
        ra, rb = eng.request(a), eng.request(b)
        # a settled greedy batch: asynchronous steps, then a multi-step window, then more steps
        c = eng.add_request([1, 2, 3], SamplingParams(max_tokens=14))
        d = eng.add_request([3, 2, 1], SamplingParams(max_tokens=14))
        for _ in range(4):
            eng.step()
        window = eng.decode_steps(3)  # after the flush: the in-flight step's token comes first
        rc, rd = eng.request(c), eng.request(d)
        for r, w in zip((rc, rd), window):
            assert r.outputs[-3:] == w
        while eng.has_work():
            eng.step()
        return (ra.outputs, [(round(lp, 5), [t for t, _ in top]) for lp, top in ra.logprobs], rb.outputs,
                rc.outputs, rd.outputs)

    sync, asyn = run(False), run(True)
    assert asyn == sync
    assert len(sync[3]) == 14 and len(sync[4]) == 14
