"""Node enrollment through the real binaries: a daemon with no certificate sends its public key
and its pod's token to the coordinator's enrollment endpoint; the coordinator asks a (fake)
API server's TokenReview which node the token's pod runs on and issues that node's certificate;
the daemon then links over mutual TLS. A token for another node yields that node's name (and the
link is refused for a daemon claiming a different one); an unauthenticated or malformed token
gets nothing."""

import json
import os
import shutil
import socket
import ssl
import stat
import subprocess
import threading
import time
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer

from cpp_bins import Proc, binary, free_port, wait_socket

TOKENS = {"hdr.pod-on-n0.sig": "n0", "hdr.pod-nowhere.sig": None}


class FakeReviews:
    def __init__(self):
        self.reviews = []
        fake = self

        class H(BaseHTTPRequestHandler):
            def do_POST(self):  # noqa: N802
                n = int(self.headers.get("Content-Length", "0"))
                req = json.loads(self.rfile.read(n))
                fake.reviews.append(req)
                tok = req["spec"]["token"]
                node = TOKENS.get(tok)
                status = {"authenticated": tok in TOKENS, "audiences": req["spec"].get("audiences", [])}
                if tok in TOKENS:
                    extra = {"authentication.kubernetes.io/pod-name": ["p"]}
                    if node:
                        extra["authentication.kubernetes.io/node-name"] = [node]
                    status["user"] = {"username": "system:serviceaccount:ns:everserve-node", "extra": extra}
                body = json.dumps({"kind": "TokenReview", "status": status}).encode()
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


def _ctl(*args, env=None):
    return subprocess.run([binary("everserve-ctl"), *args], capture_output=True, text=True, timeout=30, env=env)


def _post(addr, ca, token, body):
    ctx = ssl.create_default_context(cafile=ca)
    host, port = addr.rsplit(":", 1)
    with socket.create_connection((host, int(port)), timeout=5) as raw, ctx.wrap_socket(raw, server_hostname=host) as s:
        s.sendall(f"POST /v1/certificates/node HTTP/1.1\r\nHost: x\r\nAuthorization: Bearer {token}\r\n"
                  f"Content-Length: {len(body)}\r\n\r\n".encode() + body)
        data = b""
        while chunk := s.recv(65536):
            data += chunk
    return int(data.split(b" ", 2)[1])


def test_node_enrolls_by_token_review_then_links_over_mtls(tmp_path):
    certs = str(tmp_path / "certs")
    assert _ctl("certs", "init", certs).returncode == 0
    for name in ("coord", "operator"):
        assert _ctl("certs", "issue", certs, name).returncode == 0
    fake = FakeReviews()
    listen, api, enroll = (f"127.0.0.1:{free_port()}" for _ in range(3))
    tls = lambda name: dict(os.environ, EVERSERVE_TLS_DIR=certs, EVERSERVE_TLS_NAME=name)  # noqa: E731
    coord = Proc([binary("everserve-coord"), "--listen", listen, "--api-addr", api, "--spec-store",
                  str(tmp_path / "spec"), "--enroll-addr", enroll],
                 env=dict(tls("coord"), EVERSERVE_KUBE_API=fake.url))
    nodes = []
    try:
        wait_socket(listen)
        wait_socket(enroll)
        ca = os.path.join(certs, "ca.crt")
        # the endpoint bounds what an unauthenticated caller can do
        assert _post(enroll, ca, "not-a-jwt", b'{"publicKey":"x"}') == 401
        assert _post(enroll, ca, "hdr.pod-on-n0.sig", b"{" + b" " * 5000 + b"}") == 400
        assert _post(enroll, ca, "hdr.pod-nowhere.sig", b'{"publicKey":"x"}') == 401
        assert all(r["spec"]["token"] != "not-a-jwt" for r in fake.reviews)  # refused unread: never reviewed

        def node(name, token, attempts="5"):
            d = tmp_path / f"tls-{name}"
            d.mkdir()
            shutil.copy(ca, d / "ca.crt")  # the bootstrap CA only
            tok = tmp_path / f"token-{name}"
            tok.write_text(token + "\n")
            env = dict(os.environ, EVERSERVE_ENROLL_TOKEN_FILE=str(tok), EVERSERVE_ENROLL_ATTEMPTS=attempts)
            p = Proc([binary("everserve-node"), "--node", name, "--socket", f"unix:{tmp_path}/{name}.sock",
                      "--coordinator", listen, "--enroll", f"https://{enroll}", "--tls-dir", str(d)], env=env)
            nodes.append(p)
            return p, d

        n0, d0 = node("n0", "hdr.pod-on-n0.sig")
        deadline = time.monotonic() + 20
        while time.monotonic() < deadline:
            r = _ctl("--api", api, "get", "nodes", env=tls("operator"))
            if '"name":"n0"' in r.stdout and '"linked":true' in r.stdout:
                break
            time.sleep(0.2)
        assert '"name":"n0"' in r.stdout and '"linked":true' in r.stdout, r.stdout
        issued = json.loads((d0 / "issued.json").read_text())
        assert issued["node"] == "n0" and issued["notAfterMs"] > time.time() * 1000 + 3600_000
        assert stat.S_IMODE(os.stat(d0 / "node.key").st_mode) == 0o600
        # a daemon that claims n1 with a token of a pod on n0 is issued n0's name: its link is refused
        node("n1", "hdr.pod-on-n0.sig")
        time.sleep(2.0)
        r = _ctl("--api", api, "get", "nodes", env=tls("operator"))
        assert '"name":"n1"' not in r.stdout
        # a token the API server does not place on a node: no certificate, the daemon stops
        p2, _ = node("n2", "hdr.pod-nowhere.sig", attempts="1")
        assert p2.p.wait(timeout=20) == 2
    finally:
        for n in nodes:
            n.stop()
        coord.stop()
        fake.close()
