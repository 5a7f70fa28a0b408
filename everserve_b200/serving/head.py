"""The head of a fault-tolerant multi-process engine, serving completions over HTTP.

    EVERSERVE_SOCKET=unix:/run/everserve/node.sock EVERSERVE_MIRROR_SOCKET=unix:/run/everserve/store.sock \
    EVERSERVE_NODE=n0 python -m everserve_b200.serving.head --engine e0 --model llama-3-8b --tp 8 \
        [--pp 1] [--local-ranks 0,1,...] [--spares 7] [--device cuda] [--port 8000]

The head registers with its node's daemon (``ROLE_HEAD``), starts the ranks of its own node (the
others come from node agents), runs the engine's step loop with the failover wrapper, and serves
the completions API (``everserve_b200.serving.api``) on top of it.
"""

from __future__ import annotations

import argparse
import os


def main(argv=None) -> int:
    import torch
    import uvicorn

    from ..engine.config import EngineConfig
    from ..engine.engine import Engine
    from .api import EngineLoop, build_app
    from ..plugin import register
    from .executor import MultiprocExecutor

    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--engine", required=True)
    ap.add_argument("--model", required=True)
    ap.add_argument("--checkpoint", default=None)
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--pp", type=int, default=1)
    ap.add_argument("--local-ranks", default="", help="ranks this head starts (default: all)")
    ap.add_argument("--spares", default="", help="ranks to start a local spare for")
    ap.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    ap.add_argument("--max-batch", type=int, default=64)
    ap.add_argument("--max-model-len", type=int, default=4096)
    ap.add_argument("--num-blocks", type=int, default=None)
    ap.add_argument("--host", default="0.0.0.0")
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--daemon", default=os.environ.get("EVERSERVE_SOCKET", ""))
    ap.add_argument("--store", default=os.environ.get("EVERSERVE_MIRROR_SOCKET", ""))
    ap.add_argument("--node", default=os.environ.get("EVERSERVE_NODE", ""))
    a = ap.parse_args(argv)
    gpu = a.device.startswith("cuda")
    cfg = EngineConfig(a.model, device=a.device, dtype=torch.bfloat16 if gpu else torch.float32,
                       max_batch=a.max_batch, max_model_len=a.max_model_len, num_blocks=a.num_blocks,
                       tensor_parallel=a.tp, pipeline_parallel=a.pp, use_cuda_graphs=False, checkpoint=a.checkpoint)
    local = [int(r) for r in a.local_ranks.split(",") if r] or None
    spares = tuple(int(r) for r in a.spares.split(",") if r)
    ex = MultiprocExecutor(cfg, engine=a.engine, daemon=a.daemon, store=a.store, spares=spares, node=a.node,
                           device="cuda" if gpu else "cpu", dtype="bfloat16" if gpu else "float32", local_ranks=local)
    eng = Engine(cfg, executor=ex)
    register(eng)  # the failover step hook for the multi-process executor
    loop = EngineLoop(eng)
    try:
        uvicorn.run(build_app(loop, cfg.model.name, cfg.model.vocab), host=a.host, port=a.port, log_level="warning")
    finally:
        loop.close()
        ex.shutdown()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
