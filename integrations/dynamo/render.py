"""Render an everserve-b200 engine as a Dynamo graph deployment (Kubernetes resources).

    python integrations/dynamo/render.py --engine e0 --model llama-3-8b --tp 4 --pp 2 --nodes 2 \
        --spares 1 --image everserve-b200:latest > e0.yaml

Resources: a ``DynamoGraphDeployment`` with a Frontend (the completions server), the Head (the
engine's head: scheduler, executor, ranks of its node), one Node service per further node (node
agents that start their ranks), and spare pods; a headless Service so ranks on other nodes reach
the head's carrier and rendezvous; and the engine's entry for the coordinator's policy (a
ConfigMap fragment). Every pod gets the node contract: the daemon's socket directory, the shared
memory directory, the node group.

Reference parity: integrations/dynamo/everserve_dynamo/render.py:1-451 (the same resources:
graph deployment, headless service, policy entry), for this framework's processes.
"""

from __future__ import annotations

import argparse
import json
import sys

sys.path.insert(0, __import__("os").path.join(__import__("os").path.dirname(__file__), "..", ".."))

from everserve_b200 import podcontract  # noqa: E402


def _pod(name: str, image: str, command: list[str], gpus: int, env: list[dict] | None = None) -> dict:
    return {
        "componentType": name,
        "replicas": 1,
        "extraPodSpec": {
            "securityContext": podcontract.security_context(),
            "volumes": podcontract.volumes(),
            "mainContainer": {
                "image": image,
                "command": command,
                "env": podcontract.env() + (env or []),
                "volumeMounts": podcontract.mounts(),
                "resources": {"limits": {"nvidia.com/gpu": str(gpus)}} if gpus else {},
            },
        },
    }


def render(engine: str, model: str, tp: int, pp: int, nodes: int, spares: int, image: str,
           gpus_per_node: int = 8, port: int = 8000) -> list[dict]:
    world = tp * pp
    if world % nodes:
        raise ValueError(f"{world} ranks do not split over {nodes} nodes")
    per_node = world // nodes
    if per_node > gpus_per_node:
        raise ValueError(f"{per_node} ranks per node exceed {gpus_per_node} GPUs")
    head_svc = f"{engine}-head"
    services = {
        "Frontend": _pod("frontend", image, ["python", "-m", "everserve_b200.serving.api", "--model", model,
                                             "--port", str(port)], 0),
        "Head": _pod("head", image, ["python", "-m", "everserve_b200.serving.head", "--engine", engine, "--model",
                                     model, "--tp", str(tp), "--pp", str(pp), "--local-ranks",
                                     ",".join(map(str, range(per_node)))], per_node,
                     [{"name": "EVERSERVE_HEAD_SERVICE", "value": head_svc}]),
    }
    for n in range(1, nodes):
        ranks = ",".join(str(r) for r in range(n * per_node, (n + 1) * per_node))
        services[f"Node{n}"] = _pod("worker", image, ["python", "-m", "everserve_b200.serving.node", "--engine", engine,
                                                      "--ranks", ranks], per_node)
    for s in range(spares):
        rank = world - 1 - (s % world)
        services[f"Spare{s}"] = _pod("worker", image, ["python", "-m", "everserve_b200.serving.spare"], 1,
                                     [{"name": "EVERSERVE_ENGINE", "value": engine},
                                      {"name": "EVERSERVE_SPARE_RANK", "value": str(rank)}])
    graph = {"apiVersion": "nvidia.com/v1alpha1", "kind": "DynamoGraphDeployment",
             "metadata": {"name": engine, "labels": {"everserve.ai/engine": engine}},
             "spec": {"services": services}}
    headless = {"apiVersion": "v1", "kind": "Service", "metadata": {"name": head_svc},
                "spec": {"clusterIP": "None", "selector": {"everserve.ai/engine": engine, "component": "head"},
                         "ports": [{"name": "carrier", "port": 7700}, {"name": "rendezvous", "port": 7701}]}}
    policy = {"name": engine, "tensorParallel": tp, "pipelineParallel": pp,
              "spares": [{"node": "", "device": 0, "rank": world - 1 - (s % world)} for s in range(spares)]}
    entry = {"apiVersion": "v1", "kind": "ConfigMap", "metadata": {"name": f"{engine}-policy-entry"},
             "data": {"engine.json": json.dumps(policy)}}
    return [graph, headless, entry]


def main() -> int:
    import yaml

    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--engine", required=True)
    ap.add_argument("--model", required=True)
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--pp", type=int, default=1)
    ap.add_argument("--nodes", type=int, default=1)
    ap.add_argument("--spares", type=int, default=0)
    ap.add_argument("--image", default="everserve-b200:latest")
    a = ap.parse_args()
    yaml.safe_dump_all(render(a.engine, a.model, a.tp, a.pp, a.nodes, a.spares, a.image), sys.stdout, sort_keys=False)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
