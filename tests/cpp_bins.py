"""Helpers for tests that run the C++ control-plane binaries (built by `make -C cpp`)."""

import os
import socket
import subprocess
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
# EVERSERVE_CPP_BIN points the tests at another build of the binaries (the sanitizer builds)
BIN = os.environ.get("EVERSERVE_CPP_BIN") or os.path.join(ROOT, "cpp", "bin")


def build() -> None:
    subprocess.run(["make", "-C", os.path.join(ROOT, "cpp"), f"-j{os.cpu_count() or 4}"], check=True,
                   stdout=subprocess.DEVNULL)


def binary(name: str) -> str:
    path = os.path.join(BIN, name)
    if not os.path.exists(path):
        build()
    return path


def free_port() -> int:
    from everserve_b200.serving.cluster import free_port as fp

    return fp()


def wait_socket(path: str, timeout: float = 10.0) -> None:
    t0 = time.monotonic()
    while time.monotonic() - t0 < timeout:
        if path.startswith("unix:"):
            if os.path.exists(path[5:]):
                return
        else:
            host, _, port = path.rpartition(":")
            try:
                socket.create_connection((host, int(port)), timeout=0.2).close()
                return
            except OSError:
                pass
        time.sleep(0.02)
    raise TimeoutError(f"{path} did not come up")


class Proc:
    def __init__(self, args, env=None):
        e = dict(os.environ)
        if env:
            e.update(env)
        self.p = subprocess.Popen(args, env=e, stdout=subprocess.DEVNULL, stderr=subprocess.PIPE)

    def stop(self) -> str:
        if self.p.poll() is None:
            self.p.terminate()
            try:
                self.p.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.p.kill()
                self.p.wait()
        return self.p.stderr.read().decode(errors="replace") if self.p.stderr else ""
