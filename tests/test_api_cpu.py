"""The completions server over a CPU engine: plain and streamed completions equal Engine.generate."""

import json

import torch
from fastapi.testclient import TestClient

from everserve_b200.engine.config import EngineConfig
from everserve_b200.engine.engine import Engine
from everserve_b200.serving.api import EngineLoop, build_app


def _cfg():
    return EngineConfig("tiny-llama", device="cpu", dtype=torch.float32, num_blocks=64, max_batch=8, max_model_len=128)


def test_completions_match_generate():
    want = Engine(_cfg()).generate([[5, 6, 7], [1, 2]], max_tokens=5)
    loop = EngineLoop(Engine(_cfg()))
    try:
        c = TestClient(build_app(loop, "tiny-llama", 512))
        assert c.get("/ready").json()["ready"]
        r = c.post("/v1/completions", json={"prompt": [5, 6, 7], "max_tokens": 5}).json()
        assert r["choices"][0]["token_ids"] == want[0]
        assert r["usage"]["completion_tokens"] == 5
        with c.stream("POST", "/v1/completions", json={"prompt": [1, 2], "max_tokens": 5, "stream": True}) as s:
            lines = [ln for ln in s.iter_lines() if ln.startswith("data: ")]
        assert lines[-1] == "data: [DONE]"
        chunks = [json.loads(ln[6:])["choices"][0] for ln in lines[:-1]]
        assert [ch["token_ids"][0] for ch in chunks if ch["token_ids"]] == want[1]
        assert chunks[-1]["finish_reason"] == "length"
        assert c.get("/v1/models").json()["data"][0]["id"] == "tiny-llama"
        r = c.post("/v1/completions", json={"prompt": "hi", "max_tokens": 2}).json()
        assert len(r["choices"][0]["token_ids"]) == 2
    finally:
        loop.close()


def test_completions_sampling_and_logprobs():
    loop = EngineLoop(Engine(_cfg()))
    try:
        c = TestClient(build_app(loop, "tiny-llama", 512))
        body = {"prompt": [5, 6, 7], "max_tokens": 6, "temperature": 0.8, "top_p": 0.9, "seed": 7, "logprobs": 2}
        a = c.post("/v1/completions", json=body).json()["choices"][0]
        b = c.post("/v1/completions", json=body).json()["choices"][0]
        assert a["token_ids"] == b["token_ids"]  # the same seed draws the same tokens
        lp = a["logprobs"]
        assert len(lp["token_logprobs"]) == 6 and all(v <= 0 for v in lp["token_logprobs"])
        assert all(len(t) <= 2 for t in lp["top_logprobs"])
        with c.stream("POST", "/v1/completions", json=dict(body, stream=True)) as s:
            chunks = [json.loads(ln[6:]) for ln in s.iter_lines() if ln.startswith("data: {")]
        chunks = [ch for ch in chunks if ch["choices"][0]["token_ids"]]
        assert [ch["choices"][0]["token_ids"][0] for ch in chunks] == a["token_ids"]
        assert [ch["choices"][0]["logprobs"]["token_logprobs"][0] for ch in chunks] == lp["token_logprobs"]
        g = c.post("/v1/completions", json={"prompt": [5, 6, 7], "max_tokens": 6}).json()["choices"][0]
        assert g["logprobs"] is None
    finally:
        loop.close()


def test_stop_tokens_end_a_completion():
    want = Engine(_cfg()).generate([[5, 6, 7]], max_tokens=8)[0]
    stop = want[3]
    cut = want[: want.index(stop) + 1]
    loop = EngineLoop(Engine(_cfg()))
    try:
        c = TestClient(build_app(loop, "tiny-llama", 512))
        r = c.post("/v1/completions", json={"prompt": [5, 6, 7], "max_tokens": 8, "stop_token_ids": [stop]}).json()
        assert r["choices"][0]["token_ids"] == cut and r["choices"][0]["finish_reason"] == "stop"
        r = c.post("/v1/completions", json={"prompt": [5, 6, 7], "max_tokens": 3}).json()
        assert r["choices"][0]["finish_reason"] == "length"
        with c.stream("POST", "/v1/completions", json={"prompt": [5, 6, 7], "max_tokens": 8, "stream": True,
                                                       "stop_token_ids": [stop]}) as s:
            chunks = [json.loads(ln[6:]) for ln in s.iter_lines() if ln.startswith("data: {")]
        assert chunks[-1]["choices"][0]["finish_reason"] == "stop"
        assert [ch["choices"][0]["token_ids"][0] for ch in chunks[:-1]] == cut
    finally:
        loop.close()
