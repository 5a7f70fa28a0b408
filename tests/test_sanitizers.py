"""The control plane under sanitizers: the store (with its commit worker threads), the generated
codec and the coordinator's pure functions, built with AddressSanitizer + UndefinedBehaviorSanitizer
and with ThreadSanitizer (`make -C cpp asan tsan`), run through the same tests as the plain build.
A sanitizer report ends the binary with an error, which fails the tests it serves."""

import os
import shutil
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

pytestmark = pytest.mark.slow


@pytest.mark.parametrize("kind", ["asan", "tsan"])
def test_control_plane_under_sanitizer(kind):
    subprocess.run(["make", "-C", os.path.join(ROOT, "cpp"), f"-j{os.cpu_count() or 4}", kind], check=True,
                   stdout=subprocess.DEVNULL, timeout=1200)
    bindir = os.path.join(ROOT, "cpp", f"bin-{kind}")
    unit = subprocess.run([os.path.join(bindir, "everserve-coord-tests")], capture_output=True, text=True, timeout=300)
    assert unit.returncode == 0, unit.stderr[-2000:]
    env = dict(os.environ, EVERSERVE_CPP_BIN=bindir, ASAN_OPTIONS="detect_leaks=0:abort_on_error=0",
               TSAN_OPTIONS="halt_on_error=1:exitcode=66", UBSAN_OPTIONS="halt_on_error=1")
    try:
        r = subprocess.run([sys.executable, "-m", "pytest", "-x", "-q", "-p", "no:cacheprovider",
                            "tests/test_wire_golden.py", "tests/test_store.py", "tests/test_compile_cache.py"],
                           cwd=ROOT, env=env, capture_output=True, text=True, timeout=1200)
    finally:
        # the sanitizer builds are large; the plain build is the one the tree keeps
        for d in (bindir, os.path.join(ROOT, "cpp", f"build-{kind}")):
            shutil.rmtree(d, ignore_errors=True)
    assert r.returncode == 0, (r.stdout[-3000:], r.stderr[-3000:])
