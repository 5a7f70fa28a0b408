"""The expert-parallel all-to-all's layout, restated in torch on the CPU.

The kernels place each (token, slot) row at its rank among the sender's rows for the same expert
(``ref.expert_places``), in segment ``sender * cap`` of the owner's expert buffer; the experts run
over whole segments (padding included); the combine reads each token's rows back at those places
and sums them in slot order. This restatement of the layout must equal the dense oracle, which is
what the GPU test then holds the kernels to.
"""

import torch

from everserve_b200.ops import RefOps, ref
from everserve_b200.parallel.moe_a2a import default_cap


def _expert_weights(E, H, I, seed=0):
    g = torch.Generator().manual_seed(seed)
    return ([torch.randn(2 * I, H, generator=g) * 0.05 for _ in range(E)],
            [torch.randn(H, I, generator=g) * 0.05 for _ in range(E)])


def _expert_fn(gu, dn):
    def f(e, rows):
        a = rows.float() @ gu[e].t()
        i = a.shape[1] // 2
        return (torch.nn.functional.silu(a[:, :i]) * a[:, i:]) @ dn[e].t()
    return f


def _layout(xs, ids, ws, expert, E, W, cap):
    """Dispatch into [owner][el][W * cap] segments, run every expert over its whole buffer, combine."""
    el, H = E // W, xs[0].shape[1]
    recv = torch.full((W, el, W * cap, H), float("nan"))  # padding that must never be read
    places = []
    for p, (x, i) in enumerate(zip(xs, ids)):
        place = ref.expert_places(i, E)
        places.append(place)
        for t in range(i.shape[0]):
            for j in range(i.shape[1]):
                e = int(i[t, j])
                recv[e // el, e % el, p * cap + int(place[t, j])] = x[t].float()
    y = torch.stack([torch.stack([expert(d * el + l, recv[d, l]) for l in range(el)]) for d in range(W)])
    outs = []
    for p, (i, w) in enumerate(zip(ids, ws)):
        acc = torch.zeros(i.shape[0], H)
        for j in range(i.shape[1]):
            e = i[:, j].long()
            acc += w[:, j, None] * y[e // el, e % el, p * cap + places[p][:, j].long()]
        outs.append(acc)
    return outs, places


def test_expert_places_rank_rows_per_expert_in_token_slot_order():
    ids = torch.tensor([[3, 1], [1, 0], [3, 2], [0, 1]], dtype=torch.int32)
    assert ref.expert_places(ids, 4).tolist() == [[0, 0], [1, 0], [1, 0], [1, 2]]


def test_topk_agrees_with_the_per_expert_route():
    g = torch.Generator().manual_seed(1)
    logits = torch.randn(19, 8, generator=g).bfloat16()
    ids, w = ref.moe_topk(logits, 2)
    assert ids.dtype == torch.int32 and torch.allclose(w.sum(-1), torch.ones(19))
    dense = torch.zeros(19, 8).scatter_(1, ids.long(), w)
    assert torch.allclose(dense.t(), ref.moe_route(logits, 2, 0, 8), atol=1e-6)


def test_layout_restatement_equals_the_dense_oracle():
    W, E, k, H, I, T = 4, 8, 2, 32, 16, 23
    gu, dn = _expert_weights(E, H, I)
    expert = _expert_fn(gu, dn)
    g = torch.Generator().manual_seed(2)
    xs = [torch.randn(T, H, generator=g) for _ in range(W)]
    routed = [ref.moe_topk(torch.randn(T, E, generator=g), k) for _ in range(W)]
    ids, ws = [r[0] for r in routed], [r[1] for r in routed]
    cap = default_cap(T)
    got, places = _layout(xs, ids, ws, expert, E, W, cap)
    want = ref.moe_a2a([x.float() for x in xs], ids, ws, expert)
    for a, b in zip(got, want):
        assert torch.isfinite(a).all()  # no padding (NaN) row was read
        assert torch.allclose(a, b, atol=1e-5)
    assert all(int(p.max()) < cap for p in places)


def test_capacity_and_grouped_linear_on_the_reference_ops():
    assert default_cap(1) == 64 and default_cap(64) == 64 and default_cap(65) == 128
    ops = RefOps()
    x, w = torch.randn(8, 16), torch.randn(4, 16)
    out = torch.empty(8, 4)
    y = ops.linear(x, w, out=out, valid=torch.tensor([1, 0], dtype=torch.int32), valid_cap=4)
    assert y is out and torch.allclose(out, x @ w.t(), atol=1e-5)


def test_routed_experts_need_the_kernels_and_a_peer_group(monkeypatch):
    from everserve_b200.engine.config import EngineConfig
    from everserve_b200.models.config import TINY_MIXTRAL
    from everserve_b200.models.llama import DecoderLM

    m = DecoderLM(TINY_MIXTRAL, "cpu", torch.float32)
    assert m.enable_routed_experts(64) is False and m.a2a is None  # reference ops, TP 1: unchanged
    monkeypatch.setenv("ES_MOE_ROUTED", "1")
    assert EngineConfig(TINY_MIXTRAL, device="cpu").moe_routed
    monkeypatch.setenv("ES_MOE_ROUTED", "0")
    assert not EngineConfig(TINY_MIXTRAL, device="cpu").moe_routed


class _OracleA2A:
    """Stands in for the all-to-all on the CPU: the dense oracle over every expert's weights."""

    def __init__(self, weights):
        self.W = weights

    def __call__(self, ops, x, ids, weights, gate_up, down):
        def expert(e, rows):
            return ops.linear(ops.silu_mul(ops.linear(rows, self.W[f"l0.e{e}.gate_up"])), self.W[f"l0.e{e}.down"])
        return torch.stack(ref.moe_a2a(list(x), list(ids), list(weights), expert))


class _Identity:
    def all_reduce(self, t):
        return t


def test_routed_layer_slices_tokens_and_gathers_them_back():
    """The model's routed path (token slices per rank, top-k, the all-to-all, the slices'
    all-gather) equals its every-expert path, at TP 1 and at TP 2 played rank by rank."""
    from everserve_b200.models.config import TINY_MIXTRAL
    from everserve_b200.models.llama import DecoderLM, TPGroup

    full = DecoderLM(TINY_MIXTRAL, "cpu", torch.float32)
    g = torch.Generator().manual_seed(5)
    for T in (1, 2, 7):
        h = torch.randn(T, TINY_MIXTRAL.hidden, generator=g)
        dense = full._moe(h, "l0.")
        full.a2a = _OracleA2A(full.weights)
        assert torch.allclose(full._moe(h, "l0."), dense, atol=1e-4)
        full.a2a = None
        # TP 2: each rank contributes its slice's rows; the all-gather is a sum of disjoint rows
        parts = []
        for r in range(2):
            m = DecoderLM(TINY_MIXTRAL, "cpu", torch.float32, tp=TPGroup(r, 2, _Identity()))
            m.a2a = _OracleA2A(full.weights)
            parts.append(m._moe(h, "l0."))
        assert torch.allclose(parts[0] + parts[1], dense, atol=1e-4)
