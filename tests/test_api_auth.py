"""The operator API gated by Kubernetes tokens instead of client certificates (--api-auth kube):
a (fake) API server's TokenReview says who the bearer is and its SubjectAccessReview whether
that user may do the request's verb on the resource; answers are cached; no client certificate
is asked."""

import json
import os
import socket
import ssl
import subprocess
import threading
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer

from cpp_bins import Proc, binary, free_port, wait_socket

USERS = {"hdr.alice.sig": "alice", "hdr.admin.sig": "admin"}


class FakeAuth:
    def __init__(self):
        self.access = []
        self.tokens = []
        fake = self

        class H(BaseHTTPRequestHandler):
            def do_POST(self):  # noqa: N802
                req = json.loads(self.rfile.read(int(self.headers.get("Content-Length", "0"))))
                if self.path.endswith("/tokenreviews"):
                    tok = req["spec"]["token"]
                    fake.tokens.append(tok)
                    status = {"authenticated": tok in USERS}
                    if tok in USERS:
                        status["user"] = {"username": USERS[tok], "groups": ["system:authenticated"]}
                else:
                    ra = req["spec"]["resourceAttributes"]
                    fake.access.append((req["spec"]["user"], ra["verb"], ra["resource"], ra["group"], ra["namespace"]))
                    allowed = req["spec"]["user"] == "admin" or ra["verb"] in ("get", "list", "watch")
                    status = {"allowed": allowed}
                body = json.dumps({"status": status}).encode()
                self.send_response(201)
                self.send_header("Content-Length", str(len(body)))
                self.end_headers()
                self.wfile.write(body)

            def log_message(self, *a):
                pass

        self.server = ThreadingHTTPServer(("127.0.0.1", 0), H)
        self.url = f"http://127.0.0.1:{self.server.server_address[1]}"
        threading.Thread(target=self.server.serve_forever, daemon=True).start()

    def close(self):
        self.server.shutdown()


def _req(api, ca, method, path, token=None):
    ctx = ssl.create_default_context(cafile=ca)
    host, port = api.rsplit(":", 1)
    head = f"{method} {path} HTTP/1.1\r\nHost: x\r\nContent-Length: 0\r\n"
    if token:
        head += f"Authorization: Bearer {token}\r\n"
    with socket.create_connection((host, int(port)), timeout=5) as raw, ctx.wrap_socket(raw, server_hostname=host) as s:
        s.sendall((head + "\r\n").encode())
        data = b""
        while chunk := s.recv(65536):
            data += chunk
    return int(data.split(b" ", 2)[1])


def test_operator_api_by_token_and_access_review(tmp_path):
    certs = str(tmp_path / "certs")
    ctl = lambda *a: subprocess.run([binary("everserve-ctl"), *a], capture_output=True, timeout=30)  # noqa: E731
    assert ctl("certs", "init", certs).returncode == 0 and ctl("certs", "issue", certs, "coord").returncode == 0
    fake = FakeAuth()
    listen, api = f"127.0.0.1:{free_port()}", f"127.0.0.1:{free_port()}"
    coord = Proc([binary("everserve-coord"), "--listen", listen, "--api-addr", api, "--spec-store",
                  str(tmp_path / "spec"), "--api-auth", "kube", "--api-namespace", "ops"],
                 env=dict(os.environ, EVERSERVE_TLS_DIR=certs, EVERSERVE_TLS_NAME="coord", EVERSERVE_KUBE_API=fake.url))
    try:
        wait_socket(api)
        ca = os.path.join(certs, "ca.crt")
        assert _req(api, ca, "GET", "/v1/nodes") == 401  # no token
        assert _req(api, ca, "GET", "/v1/nodes", "garbage") == 401  # not shaped as a token: never reviewed
        assert "garbage" not in fake.tokens
        assert _req(api, ca, "GET", "/v1/nodes", "hdr.mallory.sig") == 401  # not authenticated
        assert _req(api, ca, "GET", "/v1/nodes", "hdr.alice.sig") == 200
        assert _req(api, ca, "PUT", "/v1/nodes/n0/cordon", "hdr.alice.sig") == 403  # read-only user
        assert _req(api, ca, "PUT", "/v1/nodes/n0/cordon", "hdr.admin.sig") == 200
        assert ("alice", "list", "nodes", "everserve.ai", "ops") in fake.access
        assert ("admin", "update", "nodes", "everserve.ai", "ops") in fake.access
        n = len(fake.tokens)
        assert _req(api, ca, "GET", "/v1/nodes", "hdr.alice.sig") == 200  # answered from the cache
        assert len(fake.tokens) == n
        assert _req(api, ca, "GET", "/healthz") == 200  # liveness needs no token
    finally:
        coord.stop()
        fake.close()
