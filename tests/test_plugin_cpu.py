"""The plugin surface: named patches installed once, the step hook wraps the step function."""

import pytest

from everserve_b200.plugin import PATCHES, register


class FakeEngine:
    def __init__(self):
        self.executor = object()
        self.connector = None
        self.calls = []
        self.step_fn = lambda: self.calls.append("step") or []

    def wrap_step(self, wrapper):
        self.step_fn = wrapper(self.step_fn)


def test_register_installs_named_patches_once():
    eng = FakeEngine()
    conn, ex = object(), object()

    def hook(inner):
        def wrapped():
            eng.calls.append("hook")
            return inner()
        return wrapped

    names = register(eng, executor=ex, connector=conn, step_hook=hook, prepare=False)
    assert names == ["executor", "connector", "step-hook"]
    assert eng.executor is ex and eng.connector is conn and eng.plugin_patches == names
    eng.step_fn()
    assert eng.calls == ["hook", "step"]
    with pytest.raises(RuntimeError, match="already installed"):
        register(eng, step_hook=hook, prepare=False)
    assert {p.name for p in PATCHES} == {"executor", "connector", "step-hook"}


def test_local_executor_gets_no_step_hook():
    eng = FakeEngine()
    assert register(eng, prepare=False) == []
