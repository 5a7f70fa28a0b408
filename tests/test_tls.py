"""Mutual TLS on the control plane's TCP links: certificates from the CLI, a daemon linked to the
coordinator over TLS, the operator API over HTTPS, and refusals of unauthenticated or misnamed
peers."""

import os
import socket
import ssl
import subprocess
import time

from cpp_bins import Proc, binary, free_port, wait_socket


def _ctl(*args, env=None):
    return subprocess.run([binary("everserve-ctl"), *args], capture_output=True, text=True, timeout=30, env=env)


def test_mtls_control_plane(tmp_path):
    certs = str(tmp_path / "certs")
    assert _ctl("certs", "init", certs).returncode == 0
    for name in ("coord", "n0", "n1", "operator"):
        assert _ctl("certs", "issue", certs, name).returncode == 0
    listen, api = f"127.0.0.1:{free_port()}", f"127.0.0.1:{free_port()}"
    tls = lambda name: dict(os.environ, EVERSERVE_TLS_DIR=certs, EVERSERVE_TLS_NAME=name)  # noqa: E731
    coord = Proc([binary("everserve-coord"), "--listen", listen, "--api-addr", api, "--spec-store",
                  str(tmp_path / "spec")], env=tls("coord"))
    nodes = []
    try:
        wait_socket(listen)
        # n0 links with its own certificate; "n1" presents n0's certificate and is refused
        nodes.append(Proc([binary("everserve-node"), "--node", "n0", "--socket", f"unix:{tmp_path}/n0.sock",
                           "--coordinator", listen], env=tls("n0")))
        nodes.append(Proc([binary("everserve-node"), "--node", "n1", "--socket", f"unix:{tmp_path}/n1.sock",
                           "--coordinator", listen], env=tls("n0")))
        time.sleep(1.5)
        r = _ctl("--api", api, "get", "nodes", env=tls("operator"))
        assert r.returncode == 0, r.stderr
        assert '"name":"n0"' in r.stdout and '"linked":true' in r.stdout
        assert '"name":"n1"' not in r.stdout  # misnamed certificate: refused
        # without a client certificate the API does not answer
        assert _ctl("--api", api, "get", "nodes").returncode != 0
        # a TLS client without a certificate fails the handshake
        ctx = ssl.create_default_context(cafile=os.path.join(certs, "ca.crt"))
        ctx.check_hostname = False
        host, port = api.rsplit(":", 1)
        raw = socket.create_connection((host, int(port)), timeout=5)
        try:
            with ctx.wrap_socket(raw) as s:
                s.sendall(b"GET /v1/nodes HTTP/1.1\r\nHost: x\r\n\r\n")
                got = s.recv(100)
            assert not got
        except (ssl.SSLError, ConnectionResetError, OSError):
            pass
    finally:
        for n in nodes:
            n.stop()
        coord.stop()


def test_renewed_certificate_is_taken_without_a_restart(tmp_path):
    certs = str(tmp_path / "certs")
    assert _ctl("certs", "init", certs).returncode == 0
    assert _ctl("certs", "issue", certs, "coord").returncode == 0
    listen, api = f"127.0.0.1:{free_port()}", f"127.0.0.1:{free_port()}"
    env = dict(os.environ, EVERSERVE_TLS_DIR=certs, EVERSERVE_TLS_NAME="coord", EVERSERVE_TLS_RELOAD_MS="200")
    coord = Proc([binary("everserve-coord"), "--listen", listen, "--api-addr", api, "--spec-store",
                  str(tmp_path / "spec")], env=env)

    def serial():
        ctx = ssl.create_default_context(cafile=os.path.join(certs, "ca.crt"))
        ctx.check_hostname = False
        ctx.load_cert_chain(os.path.join(certs, "coord.crt"), os.path.join(certs, "coord.key"))
        host, port = api.rsplit(":", 1)
        with socket.create_connection((host, int(port)), timeout=5) as raw, ctx.wrap_socket(raw) as s:
            return s.getpeercert()["serialNumber"]

    try:
        wait_socket(api)
        before = serial()
        time.sleep(1.1)  # a new serial (it is taken from the clock)
        assert _ctl("certs", "issue", certs, "coord").returncode == 0
        deadline = time.monotonic() + 10
        after = before
        while time.monotonic() < deadline and after == before:
            time.sleep(0.2)
            after = serial()
        assert after != before
    finally:
        coord.stop()
