"""The kernel loader imports the in-tree build, or a build named by ES_EXTENSION_PATH.

Runs in fresh interpreters (the loader caches its result), without a GPU: importing the extension
needs only torch's libraries, which the loader loads first.
"""

import glob
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PROBE = ("from everserve_b200 import _ext; C = _ext.load(); "
         "print(all(hasattr(C, n) for n in ('gemm_bf16', 'fdar', 'moe_dispatch', 'moe_combine', 'moe_topk')), "
         "C.__file__)")


def _built():
    so = sorted(glob.glob(os.path.join(ROOT, "everserve_b200", "_C*.so")))
    if not so:
        pytest.skip("the extension is not built here")
    return so[0]


def _probe(extra):
    env = {k: v for k, v in os.environ.items() if k != "ES_EXTENSION_PATH"}
    env.update(extra)
    r = subprocess.run([sys.executable, "-c", PROBE], cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    return r.stdout.split()


def test_loader_imports_the_in_tree_build():
    so = _built()
    ok, path = _probe({})
    assert ok == "True" and os.path.samefile(path, so)


def test_loader_takes_a_fetched_build(tmp_path):
    so = _built()
    fetched = tmp_path / os.path.basename(so)
    fetched.write_bytes(open(so, "rb").read())
    ok, path = _probe({"ES_EXTENSION_PATH": str(fetched)})
    assert ok == "True" and os.path.samefile(path, fetched)
