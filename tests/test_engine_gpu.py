"""The engine on a B200: kernel forward vs the reference forward, graphs vs eager, multi-step decode."""

import pytest
import torch

from everserve_b200.engine import Engine, EngineConfig, SamplingParams
from everserve_b200.models.config import TINY_LLAMA, TINY_MIXTRAL, TINY_QWEN
from everserve_b200.ops import RefOps

pytestmark = pytest.mark.gpu


def _cfg(model, graphs=True):
    return EngineConfig(model, device="cuda", max_batch=8, max_model_len=512, num_blocks=256,
                        use_cuda_graphs=graphs)


@pytest.mark.parametrize("model", [TINY_LLAMA, TINY_QWEN, TINY_MIXTRAL])
def test_kernel_forward_matches_reference(cuda, model):
    eng = Engine(_cfg(model, graphs=False))
    worker = eng.executor.worker
    prompts = [[3, 1, 4, 1, 5, 9, 2, 6], list(range(40, 77))]
    for p in prompts:
        eng.add_request(p, SamplingParams(max_tokens=4))
    plan = eng.scheduler.schedule()
    runner = worker.runner
    inp = runner.prefill_input(plan)
    model_obj = worker.model
    logits_k = model_obj.logits(inp, runner.caches)
    kops = model_obj.ops
    model_obj.ops = RefOps("cuda")
    try:
        caches_ref = [torch.zeros_like(c) for c in runner.caches]
        logits_r = model_obj.logits(inp, caches_ref)
    finally:
        model_obj.ops = kops
    torch.testing.assert_close(logits_k.float(), logits_r.float(), rtol=5e-2, atol=5e-2)


def test_graphs_match_eager_and_multistep(cuda):
    prompts = [[i, i + 1, i + 2, 7] for i in range(1, 6)]
    outs = []
    for graphs in (False, True):
        eng = Engine(_cfg(TINY_LLAMA, graphs))
        outs.append(eng.generate(prompts, max_tokens=12))
    assert outs[0] == outs[1]
    eng = Engine(_cfg(TINY_LLAMA, True))
    ids = [eng.add_request(p, SamplingParams(max_tokens=12)) for p in prompts]
    eng.step()  # prefill
    eng.step()  # first decode step
    eng.decode_steps(8)
    while eng.has_work():
        eng.step()
    assert [eng.request(i).outputs for i in ids] == outs[1]


def test_sampled_graphs_match_eager_and_replay(cuda):
    """Seeded sampling in captured decode graphs draws what eager decode draws, run after run."""
    prompts = [[3, 1, 4, 1, 5, 9, 2, 6], list(range(40, 77)), [7] * 20]
    kw = dict(max_tokens=24, temperature=0.7, top_p=0.9, top_k=50, seed=2024)
    eager = Engine(_cfg(TINY_QWEN, graphs=False)).generate(prompts, **kw)
    graphs = Engine(_cfg(TINY_QWEN, graphs=True)).generate(prompts, **kw)
    again = Engine(_cfg(TINY_QWEN, graphs=True)).generate(prompts, **kw)
    greedy = Engine(_cfg(TINY_QWEN, graphs=True)).generate(prompts, max_tokens=24)
    assert graphs == again and graphs == eager
    assert graphs != greedy


def test_logprobs_on_the_device(cuda):
    """A request asking for log-probabilities runs its steps eagerly; the greedy token is the most
    likely one and its log-probability matches the top entry."""
    eng = Engine(_cfg(TINY_QWEN, graphs=True))
    rid = eng.add_request([3, 1, 4, 1, 5, 9], SamplingParams(max_tokens=6, logprobs=4))
    other = eng.add_request([2, 7, 1, 8], SamplingParams(max_tokens=6))
    while eng.has_work():
        eng.step()
    r = eng.request(rid)
    assert len(r.logprobs) == 6 and eng.request(other).logprobs == []
    for tok, (lp, top) in zip(r.outputs, r.logprobs):
        assert top[0][0] == tok and abs(lp - top[0][1]) < 1e-5 and len(top) == 4


def test_fp8_forward_matches_reference_and_graphs(cuda):
    """The fp8 configuration on the kernels: block-scaled fp8 GEMMs (SiLU fused) against the same
    model through the reference ops, and decode graphs against eager steps."""
    cfg = EngineConfig(TINY_LLAMA, device="cuda", max_batch=8, max_model_len=512, num_blocks=256, quant="fp8",
                       use_cuda_graphs=False)
    eng = Engine(cfg)
    worker = eng.executor.worker
    eng.add_request([3, 1, 4, 1, 5, 9, 2, 6], SamplingParams(max_tokens=4))
    plan = eng.scheduler.schedule()
    runner = worker.runner
    inp = runner.prefill_input(plan)
    m = worker.model
    logits_k = m.logits(inp, runner.caches)
    kops = m.ops
    m.ops = RefOps("cuda")
    try:
        logits_r = m.logits(inp, [torch.zeros_like(c) for c in runner.caches])
    finally:
        m.ops = kops
    torch.testing.assert_close(logits_k.float(), logits_r.float(), rtol=5e-2, atol=5e-2)
    outs = []
    for graphs in (False, True):
        e = Engine(EngineConfig(TINY_LLAMA, device="cuda", max_batch=8, max_model_len=512, num_blocks=256,
                                quant="fp8", use_cuda_graphs=graphs))
        outs.append(e.generate([[1, 2, 3], [7, 7, 7, 7]], max_tokens=6))
    assert outs[0] == outs[1]


def test_async_decode_matches_sync_on_graphs(cuda):
    """One decode step in flight (the next step's token fed from the last sample on the device, its
    graph replayed before the last ids are read) gives the synchronous loop's tokens: greedy and
    seeded sampling, requests of different lengths, one joining mid-run."""
    prompts = [[i, i + 1, i + 2, 7] for i in range(1, 6)]
    params = [SamplingParams(max_tokens=12), SamplingParams(max_tokens=5, temperature=0.9, seed=4),
              SamplingParams(max_tokens=16, temperature=1.2, top_k=7, top_p=0.9, seed=5),
              SamplingParams(max_tokens=9), SamplingParams(max_tokens=3)]
    outs = []
    for async_decode in (False, True):
        cfg = _cfg(TINY_LLAMA, True)
        cfg.async_decode = async_decode
        eng = Engine(cfg)
        assert eng.async_decode == async_decode
        ids = [eng.add_request(p, sp) for p, sp in zip(prompts, params)]
        n = 0
        while eng.has_work():
            eng.step()
            n += 1
            if n == 4:
                ids.append(eng.add_request([9, 8, 7], SamplingParams(max_tokens=7)))
        outs.append([eng.request(r).outputs for r in ids])
    assert outs[0] == outs[1]
