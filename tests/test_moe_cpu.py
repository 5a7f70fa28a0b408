"""The mixture layer: routing and the expert-ordered combine against a token-by-token oracle."""

import torch

from everserve_b200.models.config import TINY_MIXTRAL
from everserve_b200.models.llama import DecoderLM
from everserve_b200.ops import ref


def _naive_moe(model, h, p):
    c, W = model.cfg, model.weights
    out = torch.zeros(h.shape[0], c.hidden)
    for t in range(h.shape[0]):
        probs = torch.softmax(h[t].float() @ W[p + "router"].float().t(), -1)
        order = sorted(range(c.num_experts), key=lambda e: (-probs[e].item(), e))[: c.top_k]
        norm = sum(probs[e] for e in order)
        for e in order:
            gu = h[t].float() @ W[p + f"e{e}.gate_up"].float().t()
            g, u = gu[: c.intermediate], gu[c.intermediate :]
            y = (torch.nn.functional.silu(g) * u) @ W[p + f"e{e}.down"].float().t()
            out[t] += probs[e] / norm * y
    return out


def test_moe_layer_matches_token_oracle():
    m = DecoderLM(TINY_MIXTRAL, "cpu", torch.float32, seed=3)
    h = torch.randn(9, TINY_MIXTRAL.hidden, generator=torch.Generator().manual_seed(1))
    got = m._moe(h, "l0.")
    torch.testing.assert_close(got, _naive_moe(m, h, "l0."), rtol=1e-4, atol=1e-5)


def test_route_ties_go_to_the_lowest_expert():
    logits = torch.tensor([[1.0, 3.0, 3.0, 0.0], [2.0, 2.0, 2.0, 2.0]])
    w = ref.moe_route(logits, 2, 0, 4)  # [experts, tokens]
    assert torch.equal((w[:, 0] > 0), torch.tensor([False, True, True, False]))
    assert torch.equal((w[:, 1] > 0), torch.tensor([True, True, False, False]))
    torch.testing.assert_close(w.sum(0), torch.ones(2))
    assert torch.equal(ref.moe_route(logits, 2, 1, 2), w[1:3])
