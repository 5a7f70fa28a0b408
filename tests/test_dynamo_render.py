"""The Dynamo renderer: services for the frontend, head, node agents and spares, with the node
contract on every pod, and a command that names a module this package has."""

import importlib
import os
import sys

import pytest

sys.path.insert(0, os.path.join(os.path.dirname(__file__), "..", "integrations", "dynamo"))

import render  # noqa: E402


def test_render_two_nodes_with_spare():
    graph, headless, entry = render.render("e0", "llama-3-8b", tp=4, pp=2, nodes=2, spares=1, image="img")
    svcs = graph["spec"]["services"]
    assert set(svcs) == {"Frontend", "Head", "Node1", "Spare0"}
    assert "--ranks" in svcs["Node1"]["extraPodSpec"]["mainContainer"]["command"]
    node_cmd = svcs["Node1"]["extraPodSpec"]["mainContainer"]["command"]
    assert node_cmd[node_cmd.index("--ranks") + 1] == "4,5,6,7"
    for s in svcs.values():
        c = s["extraPodSpec"]["mainContainer"]
        assert any(m["mountPath"] == "/run/everserve" for m in c["volumeMounts"])
        mod = c["command"][c["command"].index("-m") + 1]
        importlib.import_module(mod)  # every command runs a module of the package
    assert headless["spec"]["clusterIP"] == "None"
    assert '"pipelineParallel": 2' in entry["data"]["engine.json"]


def test_render_refuses_uneven_split():
    with pytest.raises(ValueError):
        render.render("e0", "m", tp=3, pp=1, nodes=2, spares=0, image="img")
