"""Seeded sampling: deterministic per (seed, position), filters honoured, distribution right, and
exact replay through the engine (a resumed request samples the tokens it sampled before)."""

import torch

from everserve_b200.engine.config import EngineConfig
from everserve_b200.engine.engine import Engine
from everserve_b200.engine.request import SamplingParams
from everserve_b200.engine.sampling import SamplingBatch, sample, uniforms


def _sb(B, t=1.0, k=0, p=1.0, seed=7):
    return SamplingBatch(torch.full((B,), t), torch.full((B,), k, dtype=torch.int64), torch.full((B,), p),
                         torch.full((B,), seed, dtype=torch.int64))


def test_uniforms_are_a_function_of_seed_and_position():
    a = uniforms(torch.tensor([1, 1, 2]), torch.tensor([5, 6, 5]), 1000)
    b = uniforms(torch.tensor([1, 1, 2]), torch.tensor([5, 6, 5]), 1000)
    assert torch.equal(a, b)
    assert not torch.equal(a[0], a[1]) and not torch.equal(a[0], a[2])
    assert float(a.min()) > 0 and float(a.max()) < 1
    assert abs(float(a.mean()) - 0.5) < 0.02  # 3000 draws


def test_greedy_rows_and_filters():
    g = torch.Generator().manual_seed(0)
    logits = torch.randn(6, 50, generator=g)
    # temperature 0: the argmax
    assert torch.equal(sample(logits, torch.arange(6), _sb(6, t=0.0)), logits.argmax(1))
    # top_k 1 (or a tiny top_p) at any temperature: the argmax too
    assert torch.equal(sample(logits, torch.arange(6), _sb(6, t=5.0, k=1)), logits.argmax(1))
    assert torch.equal(sample(logits, torch.arange(6), _sb(6, t=5.0, p=1e-6)), logits.argmax(1))
    # top_k 3: always one of the three largest
    top3 = logits.topk(3, dim=1).indices
    for pos in range(50):
        ids = sample(logits, torch.full((6,), pos), _sb(6, t=3.0, k=3))
        assert bool((top3 == ids[:, None]).any(1).all())


def test_distribution_follows_the_softmax():
    logits = torch.tensor([[2.0, 1.0, 0.0, -1.0]])
    counts = torch.zeros(4)
    for pos in range(4000):
        counts[sample(logits, torch.tensor([pos]), _sb(1, t=1.0, seed=11))] += 1
    want = torch.softmax(logits[0], 0)
    assert torch.allclose(counts / 4000, want, atol=0.03), (counts / 4000, want)


def test_engine_sampling_is_reproducible_and_replays_exactly():
    cfg = EngineConfig(model="tiny-qwen", device="cpu", dtype=torch.float32, num_blocks=64, max_batch=4,
                       max_model_len=128, use_cuda_graphs=False)
    prompts = [[1, 2, 3, 4], [5, 6, 7, 8, 9]]
    sp = SamplingParams(max_tokens=12, temperature=0.9, top_p=0.9, top_k=20, seed=123)

    def run():
        eng = Engine(cfg)
        ids = [eng.add_request(p, sp) for p in prompts]
        while eng.has_work():
            eng.step()
        return eng, [eng.request(i).outputs for i in ids]

    eng, a = run()
    _, b = run()
    assert a == b
    greedy = Engine(cfg).generate(prompts, max_tokens=12)
    assert a != greedy  # sampling actually sampled
    # a resumed request (as after a failover: committed state lost) replays to the same tokens
    eng2 = Engine(cfg)
    ids = [eng2.add_request(p, sp) for p in prompts]
    for _ in range(6):
        eng2.step()
    for i in ids:  # only part of what ran is committed: the rest is replayed one position per step
        r = eng2.request(i)
        r.committed = len(r.prompt) + 2
    eng2.scheduler.resume_from_committed()
    while eng2.has_work():
        eng2.step()
    assert [eng2.request(i).outputs for i in ids] == a
    assert all(eng2.request(i).replay_mismatches == 0 for i in ids)


def test_logprobs_match_the_models_distribution():
    cfg = EngineConfig(model="tiny-qwen", device="cpu", dtype=torch.float32, num_blocks=64, max_batch=4,
                       max_model_len=128, use_cuda_graphs=False)
    eng = Engine(cfg)
    prompt = [3, 1, 4, 1, 5]
    a = eng.add_request(prompt, SamplingParams(max_tokens=5, logprobs=3))
    b = eng.add_request([9, 9, 9], SamplingParams(max_tokens=5))  # no logprobs asked: none recorded
    while eng.has_work():
        eng.step()
    ra, rb = eng.request(a), eng.request(b)
    assert len(ra.logprobs) == 5 and rb.logprobs == []
    for tok, (lp, top) in zip(ra.outputs, ra.logprobs):
        assert len(top) == 3 and top[0][0] == tok  # greedy: the chosen token is the most likely
        assert abs(lp - top[0][1]) < 1e-6 and top[0][1] >= top[1][1] >= top[2][1]
    # the first output's log-probability against the model's own logits
    worker = Engine(cfg).executor.worker
    from everserve_b200.engine.scheduler import ScheduledReq, StepPlan

    plan = StepPlan(0, True, [ScheduledReq("x", prompt, 0, list(range(1)), True)])
    inp = worker.runner.prefill_input(plan)
    lg = worker.model.logits(inp, worker.runner.caches)
    want = torch.log_softmax(lg.float(), -1)[0, ra.outputs[0]]
    assert abs(float(want) - ra.logprobs[0][0]) < 1e-4
