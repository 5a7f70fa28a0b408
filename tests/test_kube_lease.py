"""The coordinator's Kubernetes lease against a fake API server (Lease objects with
resourceVersion conflicts, bearer tokens): the first coordinator holds term 1 and renews it; a
standby takes term 2 once the holder is killed and its renewTime runs out; a holder whose lease
another process took exits rather than write epochs beside it."""

import json
import os
import signal
import subprocess
import threading
import time
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer

from everserve_b200.serving.cluster import binary, free_port, wait_listening


class FakeKube:
    def __init__(self, token="tok-1"):
        self.token = token
        self.leases = {}  # (ns, name) -> object
        self.rv = 0
        self.lock = threading.Lock()
        self.requests = []
        fake = self

        class H(BaseHTTPRequestHandler):
            def _send(self, code, obj=None):
                body = json.dumps(obj).encode() if obj is not None else b""
                self.send_response(code)
                self.send_header("Content-Type", "application/json")
                self.send_header("Content-Length", str(len(body)))
                self.end_headers()
                self.wfile.write(body)

            def _auth(self):
                if self.headers.get("Authorization") != f"Bearer {fake.token}":
                    self._send(401, {"kind": "Status", "code": 401})
                    return False
                return True

            def _key(self):
                parts = self.path.split("/")  # /apis/coordination.k8s.io/v1/namespaces/NS/leases[/NAME]
                return parts[5], (parts[7] if len(parts) > 7 else None)

            def _body(self):
                n = int(self.headers.get("Content-Length", "0"))
                return json.loads(self.rfile.read(n)) if n else {}

            def do_GET(self):  # noqa: N802
                fake.requests.append(("GET", self.path))
                if not self._auth():
                    return
                ns, name = self._key()
                with fake.lock:
                    obj = fake.leases.get((ns, name))
                self._send(200, obj) if obj else self._send(404, {"kind": "Status", "code": 404})

            def do_POST(self):  # noqa: N802
                fake.requests.append(("POST", self.path))
                if not self._auth():
                    return
                ns, _ = self._key()
                obj = self._body()
                name = obj["metadata"]["name"]
                with fake.lock:
                    if (ns, name) in fake.leases:
                        return self._send(409, {"kind": "Status", "code": 409})
                    fake.rv += 1
                    obj["metadata"]["resourceVersion"] = str(fake.rv)
                    fake.leases[(ns, name)] = obj
                self._send(201, obj)

            def do_PUT(self):  # noqa: N802
                fake.requests.append(("PUT", self.path))
                if not self._auth():
                    return
                ns, name = self._key()
                obj = self._body()
                with fake.lock:
                    cur = fake.leases.get((ns, name))
                    if cur is None:
                        return self._send(404, {"kind": "Status", "code": 404})
                    if obj["metadata"].get("resourceVersion") != cur["metadata"]["resourceVersion"]:
                        return self._send(409, {"kind": "Status", "code": 409})
                    fake.rv += 1
                    obj["metadata"]["resourceVersion"] = str(fake.rv)
                    fake.leases[(ns, name)] = obj
                self._send(200, obj)

            def log_message(self, *a):
                pass

        self.server = ThreadingHTTPServer(("127.0.0.1", 0), H)
        self.url = f"http://127.0.0.1:{self.server.server_address[1]}"
        threading.Thread(target=self.server.serve_forever, daemon=True).start()

    def lease(self, ns="ns1", name="coord"):
        with self.lock:
            return json.loads(json.dumps(self.leases.get((ns, name))))

    def take_over(self, holder, ns="ns1", name="coord"):
        """Another process writes the lease (as if it had won it)."""
        with self.lock:
            obj = self.leases[(ns, name)]
            obj["spec"]["holderIdentity"] = holder
            obj["spec"]["leaseTransitions"] += 1
            self.rv += 1
            obj["metadata"]["resourceVersion"] = str(self.rv)

    def close(self):
        self.server.shutdown()


def _coord(tmp_path, name, fake, token_file):
    env = dict(os.environ, EVERSERVE_KUBE_API=fake.url, EVERSERVE_KUBE_TOKEN_FILE=str(token_file))
    api = f"127.0.0.1:{free_port()}"
    log = open(tmp_path / f"{name}.log", "w")  # noqa: SIM115
    p = subprocess.Popen([binary("everserve-coord"), "--listen", f"unix:{tmp_path}/{name}.sock", "--spec-store",
                          str(tmp_path / "spec"), "--lease", "k8s:ns1/coord", "--lease-duration-s", "2",
                          "--lease-holder", name, "--api-addr", api], stdout=log, stderr=subprocess.STDOUT, env=env)
    return p, api


def test_kubernetes_lease_term_standby_and_loss(tmp_path):
    fake = FakeKube()
    token = tmp_path / "token"
    token.write_text("tok-1\n")
    a = b = None
    try:
        a, api_a = _coord(tmp_path, "coord-a", fake, token)
        wait_listening(api_a)
        spec = fake.lease()["spec"]
        assert spec["holderIdentity"] == "coord-a" and spec["leaseTransitions"] == 1
        b, api_b = _coord(tmp_path, "coord-b", fake, token)
        time.sleep(1.5)  # a renews (every 0.5 s); b waits
        assert fake.lease()["spec"]["holderIdentity"] == "coord-a"
        assert any(m == "PUT" for m, _ in fake.requests)
        assert b.poll() is None
        a.send_signal(signal.SIGKILL)
        a.wait()
        wait_listening(api_b, timeout_s=15)  # b takes the lease once a's renewTime is 2 s old
        spec = fake.lease()["spec"]
        assert spec["holderIdentity"] == "coord-b" and spec["leaseTransitions"] == 2
        assert "term 2" in open(tmp_path / "coord-b.log").read()
        # another process writes the lease: b cannot renew it and exits
        fake.take_over("intruder")
        assert b.wait(timeout=10) == 3
        assert "lost" in open(tmp_path / "coord-b.log").read()
    finally:
        for p in (a, b):
            if p is not None and p.poll() is None:
                p.kill()
                p.wait()
        fake.close()
