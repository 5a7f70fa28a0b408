"""An OpenAI-style completions server over an Engine (single process or a multi-process head).

    python -m everserve_b200.serving.api --model llama-3-8b --port 8000 [--checkpoint DIR] [--tp 8 ...]

``POST /v1/completions`` with ``{"prompt": [token ids] | "text", "max_tokens": n, "stream": bool,
"temperature": t, "top_k": k, "top_p": p, "seed": s, "logprobs": n}`` (temperature 0, the default, is greedy;
``logprobs`` n returns each token's log-probability and the n most likely, at most 20;
``stop_token_ids`` end a completion, as the tokenizer's end-of-sequence id does unless ``ignore_eos``)
returns ``choices[0].token_ids`` (and ``text`` when a tokenizer is configured); with
``"stream": true`` it sends one server-sent event per new token. ``GET /v1/models``, ``GET /live``
and ``GET /ready`` report the model and health (``/ready`` is 503 while a membership change is
in flight).

One thread runs the engine's step loop; requests are queued to it and their tokens fanned back out
per request. With a fault-tolerant executor the loop runs through the failover step wrapper, so a
rank loss pauses the streams and they continue with the same tokens.

Without a tokenizer (``--tokenizer DIR`` takes a Hugging Face tokenizer directory), text prompts
are encoded as UTF-8 bytes modulo the vocabulary, which is enough to drive the engine end to end.
"""

from __future__ import annotations

import argparse
import asyncio
import json
import queue
import threading
import time
import uuid
from dataclasses import dataclass, field

from ..engine.engine import Engine
from ..engine.request import SamplingParams


@dataclass
class _Pending:
    prompt: list[int]
    params: SamplingParams
    req_id: str
    out: queue.Queue = field(default_factory=queue.Queue)


class EngineLoop:
    """Runs `engine.step()` on one thread; other threads submit requests and read their tokens."""

    def __init__(self, engine: Engine):
        self.engine = engine
        self._inbox: queue.Queue[_Pending] = queue.Queue()
        self._live: dict[str, _Pending] = {}
        self._stop = threading.Event()
        self.changing = threading.Event()
        self.error: str | None = None
        self._t = threading.Thread(target=self._run, name="engine-loop", daemon=True)
        self._t.start()

    def submit(self, prompt: list[int], params: SamplingParams) -> _Pending:
        p = _Pending(list(prompt), params, f"cmpl-{uuid.uuid4().hex[:12]}")
        self._inbox.put(p)
        return p

    def _run(self) -> None:
        eng = self.engine
        while not self._stop.is_set():
            try:
                while True:
                    p = self._inbox.get_nowait()
                    eng.add_request(p.prompt, p.params, req_id=p.req_id)
                    self._live[p.req_id] = p
            except queue.Empty:
                pass
            if not eng.has_work():
                time.sleep(0.001)
                continue
            try:
                for req_id, tok, fin in eng.step():
                    p = self._live.get(req_id)
                    if p is None:
                        continue
                    if tok is not None:
                        p.out.put(tok)
                    if fin:
                        p.out.put(None)
                        del self._live[req_id]
            except Exception as e:  # noqa: BLE001 - every open request learns of it
                self.error = f"{type(e).__name__}: {e}"
                for p in self._live.values():
                    p.out.put(e)
                self._live.clear()
                return

    def close(self) -> None:
        self._stop.set()
        self._t.join(timeout=5)


def build_app(loop: EngineLoop, model_name: str, vocab: int, tokenizer=None):
    from fastapi import FastAPI, HTTPException
    from fastapi.responses import JSONResponse, StreamingResponse

    app = FastAPI(title="everserve-b200")

    def encode(prompt) -> list[int]:
        if isinstance(prompt, list) and all(isinstance(t, int) for t in prompt):
            return prompt
        if isinstance(prompt, str):
            if tokenizer is not None:
                return tokenizer.encode(prompt)
            return [b % vocab for b in prompt.encode()]
        raise HTTPException(400, "prompt must be a string or a list of token ids")

    def decode(ids: list[int]) -> str | None:
        return tokenizer.decode(ids) if tokenizer is not None else None

    eos_id = getattr(tokenizer, "eos_token_id", None) if tokenizer is not None else None

    @app.get("/live")
    def live():
        return {"live": True}

    @app.get("/ready")
    def ready():
        if loop.error:
            return JSONResponse({"ready": False, "reason": loop.error}, status_code=503)
        ex = loop.engine.executor
        if getattr(ex, "change_pending", lambda: False)():
            return JSONResponse({"ready": False, "reason": "a membership change is in flight"}, status_code=503)
        return {"ready": True}

    @app.get("/v1/models")
    def models():
        return {"object": "list", "data": [{"id": model_name, "object": "model", "owned_by": "everserve-b200"}]}

    @app.post("/v1/completions")
    async def completions(body: dict):
        prompt = encode(body.get("prompt", ""))
        if not prompt:
            raise HTTPException(400, "empty prompt")
        seed = body.get("seed")
        nlp = body.get("logprobs")
        params = SamplingParams(max_tokens=int(body.get("max_tokens", 16)),
                                temperature=float(body.get("temperature", 0.0) or 0.0),
                                top_k=int(body.get("top_k", 0) or 0), top_p=float(body.get("top_p", 1.0) or 1.0),
                                seed=int(seed) if seed is not None else None,
                                logprobs=min(20, int(nlp)) if nlp is not None else None,
                                stop_ids=tuple(int(t) for t in body.get("stop_token_ids") or ()),
                                eos_id=eos_id, ignore_eos=bool(body.get("ignore_eos", eos_id is None)))
        p = loop.submit(prompt, params)
        created = int(time.time())

        def logprobs_of(ids: list[int], first: int = 0):
            """The completions API's logprobs object for outputs first .. first + len(ids)."""
            if params.logprobs is None:
                return None
            recs = loop.engine.request(p.req_id).logprobs[first : first + len(ids)]
            name = lambda t: decode([t]) if decode([t]) is not None else str(t)  # noqa: E731 - ids without a tokenizer
            names = [name(t) for t in ids]
            offsets = [sum(len(x) for x in names[:i]) for i in range(len(names))]
            return {"tokens": names, "token_logprobs": [r[0] for r in recs],
                    "top_logprobs": [{name(t): v for t, v in r[1]} for r in recs], "text_offset": offsets}

        async def tokens():
            while True:
                item = await asyncio.get_running_loop().run_in_executor(None, p.out.get)
                if item is None:
                    return
                if isinstance(item, Exception):
                    raise HTTPException(500, str(item))
                yield item

        if body.get("stream"):
            async def events():
                i = 0
                async for t in tokens():
                    chunk = {"id": p.req_id, "object": "text_completion", "created": created, "model": model_name,
                             "choices": [{"index": 0, "token_ids": [t], "text": decode([t]), "finish_reason": None,
                                          "logprobs": logprobs_of([t], i)}]}
                    i += 1
                    yield f"data: {json.dumps(chunk)}\n\n"
                final = {"id": p.req_id, "object": "text_completion", "created": created, "model": model_name,
                         "choices": [{"index": 0, "token_ids": [], "text": "",
                                      "finish_reason": loop.engine.request(p.req_id).finish_reason() or "length"}]}
                yield f"data: {json.dumps(final)}\n\n"
                yield "data: [DONE]\n\n"

            return StreamingResponse(events(), media_type="text/event-stream")
        ids = [t async for t in tokens()]
        finish = loop.engine.request(p.req_id).finish_reason() or "length"
        return {"id": p.req_id, "object": "text_completion", "created": created, "model": model_name,
                "choices": [{"index": 0, "token_ids": ids, "text": decode(ids), "finish_reason": finish,
                             "logprobs": logprobs_of(ids)}],
                "usage": {"prompt_tokens": len(prompt), "completion_tokens": len(ids),
                          "total_tokens": len(prompt) + len(ids)}}

    return app


def main(argv=None) -> int:
    import torch
    import uvicorn

    from ..engine.config import EngineConfig

    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--model", default="llama-3-8b")
    ap.add_argument("--checkpoint", default=None)
    ap.add_argument("--tokenizer", default=None)
    ap.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--max-batch", type=int, default=64)
    ap.add_argument("--max-model-len", type=int, default=4096)
    a = ap.parse_args(argv)
    dtype = torch.bfloat16 if a.device.startswith("cuda") else torch.float32
    cfg = EngineConfig(a.model, device=a.device, dtype=dtype, max_batch=a.max_batch, max_model_len=a.max_model_len,
                       checkpoint=a.checkpoint)
    tok = None
    if a.tokenizer:
        from transformers import AutoTokenizer

        tok = AutoTokenizer.from_pretrained(a.tokenizer)
    loop = EngineLoop(Engine(cfg))
    uvicorn.run(build_app(loop, cfg.model.name, cfg.model.vocab, tok), host=a.host, port=a.port, log_level="warning")
    loop.close()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
