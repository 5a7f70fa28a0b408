"""Deployment artefacts: alert and dashboard metric names exist in the binaries; the bare-metal
smoke script (coordinator, two daemons and stores, drain, node loss) passes."""

import json
import os
import re
import subprocess

import yaml

from cpp_bins import ROOT, binary

DEPLOY = os.path.join(ROOT, "deploy")


def _exported() -> set:
    names = set()
    for d, _, files in os.walk(os.path.join(ROOT, "cpp")):
        for f in files:
            if f.endswith(".cpp"):
                names |= set(re.findall(r'"(everserve_[a-z_]+)"', open(os.path.join(d, f)).read()))
    return names


def _metrics_in(expr: str) -> set:
    out = set()
    for m in re.findall(r"everserve_[a-z_]+", expr):
        for suffix in ("_bucket", "_sum", "_count"):
            if m.endswith(suffix):
                m = m[: -len(suffix)]
        out.add(m)
    return out


def test_alert_and_dashboard_metrics_exist():
    exported = _exported()
    rules = yaml.safe_load(open(os.path.join(DEPLOY, "grafana", "alerts.yml")))
    used = set()
    for g in rules["groups"]:
        for r in g["rules"]:
            used |= _metrics_in(r["expr"])
    dash = json.load(open(os.path.join(DEPLOY, "grafana", "everserve.json")))
    for p in dash["panels"]:
        for t in p["targets"]:
            used |= _metrics_in(t["expr"])
    missing = sorted(used - exported)
    assert not missing, f"metrics named by alerts/dashboard but not exported: {missing}"


def test_baremetal_smoke():
    for b in ("everserve-coord", "everserve-node", "everserve-store", "everserve-ctl"):
        binary(b)
    r = subprocess.run(["bash", os.path.join(DEPLOY, "baremetal", "smoke.sh")], capture_output=True, text=True,
                       timeout=60)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "smoke: ok" in r.stdout


def test_helm_chart_kubernetes_state_backend():
    """The chart runs the coordinator on a Lease and EverserveState objects by default, ships the
    CRD, and grants the coordinator exactly those resources."""
    chart = os.path.join(DEPLOY, "kubernetes", "everserve")
    crd = yaml.safe_load(open(os.path.join(chart, "crds", "everservestate.yaml")))
    assert crd["spec"]["group"] == "everserve.ai" and crd["spec"]["names"]["plural"] == "everservestates"
    values = yaml.safe_load(open(os.path.join(chart, "values.yaml")))
    assert values["coordinator"]["stateBackend"] == "kubernetes"
    tpl = open(os.path.join(chart, "templates", "coordinator.yaml")).read()
    assert '"--spec-store", "k8s:{{ .Release.Namespace }}"' in tpl
    assert '"--lease", "k8s:{{ .Release.Namespace }}/everserve-coord"' in tpl
    assert "resources: [leases]" in tpl and "resources: [everservestates]" in tpl


def test_helm_chart_node_daemonset_rbac_and_network_policies():
    chart = os.path.join(DEPLOY, "kubernetes", "everserve")
    node = open(os.path.join(chart, "templates", "node.yaml")).read()
    coord = open(os.path.join(chart, "templates", "coordinator.yaml")).read()
    assert "kind: NetworkPolicy" in node and "resources: [nodes], verbs: [get]" in node
    assert "audience: everserve" in node and "--enroll https://everserve-coord" in node
    assert "--compile-cache-dir" in node and "EVERSERVE_COMPILE_CACHE" in node
    assert "resources: [tokenreviews], verbs: [create]" in coord and "--enroll-addr" in coord
    values = yaml.safe_load(open(os.path.join(chart, "values.yaml")))
    assert values["coordinator"]["enrollPort"] == 7682 and values["store"]["replicaPort"] == 7683


def test_every_alert_has_a_runbook_entry():
    rules = yaml.safe_load(open(os.path.join(DEPLOY, "grafana", "alerts.yml")))
    runbook = open(os.path.join(ROOT, "docs", "RUNBOOK.md")).read()
    missing = [r["alert"] for g in rules["groups"] for r in g["rules"] if f"`{r['alert']}`" not in runbook]
    assert not missing, missing
