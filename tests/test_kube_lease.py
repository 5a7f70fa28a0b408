"""The coordinator's Kubernetes lease against a fake API server (Lease objects with
resourceVersion conflicts, bearer tokens): the first coordinator holds term 1 and renews it; a
standby takes term 2 once the holder is killed and its renewTime runs out; a holder whose lease
another process took exits rather than write epochs beside it."""

import base64
import json
import os
import signal
import subprocess
import threading
import time
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer

from everserve_b200.serving.cluster import binary, free_port, wait_listening


class FakeKube:
    """Namespaced objects of any collection (/apis/G/V/namespaces/NS/PLURAL[/NAME]) with
    resourceVersion conflicts, behind a bearer token."""

    def __init__(self, token="tok-1"):
        self.token = token
        self.objects = {}  # (collection path, name) -> object
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
                fake.requests.append((self.command, self.path))
                if self.headers.get("Authorization") != f"Bearer {fake.token}":
                    self._send(401, {"kind": "Status", "code": 401})
                    return False
                return True

            def _key(self):
                parts = self.path.split("?")[0].split("/")  # ['', apis, G, V, namespaces, NS, PLURAL, NAME?]
                return "/".join(parts[:7]), (parts[7] if len(parts) > 7 else None)

            def _body(self):
                n = int(self.headers.get("Content-Length", "0"))
                return json.loads(self.rfile.read(n)) if n else {}

            def do_GET(self):  # noqa: N802
                if not self._auth():
                    return
                coll, name = self._key()
                with fake.lock:
                    if name is None:
                        items = [o for (c, _), o in sorted(fake.objects.items()) if c == coll]
                        return self._send(200, {"kind": "List", "items": items})
                    obj = fake.objects.get((coll, name))
                self._send(200, obj) if obj else self._send(404, {"kind": "Status", "code": 404})

            def do_POST(self):  # noqa: N802
                if not self._auth():
                    return
                coll, _ = self._key()
                obj = self._body()
                name = obj["metadata"]["name"]
                with fake.lock:
                    if (coll, name) in fake.objects:
                        return self._send(409, {"kind": "Status", "code": 409})
                    fake.rv += 1
                    obj["metadata"]["resourceVersion"] = str(fake.rv)
                    fake.objects[(coll, name)] = obj
                self._send(201, obj)

            def do_PUT(self):  # noqa: N802
                if not self._auth():
                    return
                coll, name = self._key()
                obj = self._body()
                with fake.lock:
                    cur = fake.objects.get((coll, name))
                    if cur is None:
                        return self._send(404, {"kind": "Status", "code": 404})
                    if obj["metadata"].get("resourceVersion") != cur["metadata"]["resourceVersion"]:
                        return self._send(409, {"kind": "Status", "code": 409})
                    fake.rv += 1
                    obj["metadata"]["resourceVersion"] = str(fake.rv)
                    fake.objects[(coll, name)] = obj
                self._send(200, obj)

            def do_DELETE(self):  # noqa: N802
                if not self._auth():
                    return
                coll, name = self._key()
                with fake.lock:
                    obj = fake.objects.pop((coll, name), None)
                self._send(200, obj) if obj else self._send(404, {"kind": "Status", "code": 404})

            def log_message(self, *a):
                pass

        self.server = ThreadingHTTPServer(("127.0.0.1", 0), H)
        self.url = f"http://127.0.0.1:{self.server.server_address[1]}"
        threading.Thread(target=self.server.serve_forever, daemon=True).start()

    LEASES = "/apis/coordination.k8s.io/v1/namespaces/ns1/leases"
    STATES = "/apis/everserve.ai/v1/namespaces/ns1/everservestates"

    def lease(self, name="coord"):
        with self.lock:
            return json.loads(json.dumps(self.objects.get((self.LEASES, name))))

    def states(self):
        with self.lock:
            return {o["spec"]["key"]: o for (c, _), o in self.objects.items() if c == self.STATES}

    def take_over(self, holder, name="coord"):
        """Another process writes the lease (as if it had won it)."""
        with self.lock:
            obj = self.objects[(self.LEASES, name)]
            obj["spec"]["holderIdentity"] = holder
            obj["spec"]["leaseTransitions"] += 1
            self.rv += 1
            obj["metadata"]["resourceVersion"] = str(self.rv)

    def close(self):
        self.server.shutdown()


def _coord(tmp_path, name, fake, token_file, spec=None):
    env = dict(os.environ, EVERSERVE_KUBE_API=fake.url, EVERSERVE_KUBE_TOKEN_FILE=str(token_file))
    api = f"127.0.0.1:{free_port()}"
    log = open(tmp_path / f"{name}.log", "w")  # noqa: SIM115
    p = subprocess.Popen([binary("everserve-coord"), "--listen", f"unix:{tmp_path}/{name}.sock", "--spec-store",
                          spec or str(tmp_path / "spec"), "--lease", "k8s:ns1/coord", "--lease-duration-s", "2",
                          "--lease-holder", name, "--api-addr", api], stdout=log, stderr=subprocess.STDOUT, env=env)
    return p, api


def _call(api, method, path, body=None):
    import http.client

    host, port = api.rsplit(":", 1)
    c = http.client.HTTPConnection(host, int(port), timeout=5)
    c.request(method, path, body=json.dumps(body) if body is not None else None)
    r = c.getresponse()
    data = r.read()
    c.close()
    return r.status, json.loads(data) if data else {}


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


def test_spec_in_custom_resources_survives_the_coordinator(tmp_path):
    """Pools and node specs written by one coordinator into EverserveState objects are read back
    by its successor (the lease's next holder)."""
    fake = FakeKube()
    token = tmp_path / "token"
    token.write_text("tok-1")
    policy = tmp_path / "policy.json"
    policy.write_text(json.dumps({"engines": [{"name": "e0", "tensorParallel": 2}]}))
    a = b = None
    try:
        a, api_a = _coord(tmp_path, "coord-a", fake, token, spec="k8s:ns1")
        wait_listening(api_a)
        code, _ = _call(api_a, "PUT", "/v1/nodes/n3/cordon")
        assert code == 200
        code, _ = _call(api_a, "PUT", "/v1/pools/p0", {"engines": [], "wants": 2, "reason": "warm capacity"})
        assert code == 200
        st = fake.states()
        assert "nodes/n3.json" in st and "pools/p0.json" in st
        assert all(o["metadata"]["name"].startswith("es-") for o in st.values())
        a.send_signal(signal.SIGKILL)
        a.wait()
        b, api_b = _coord(tmp_path, "coord-b", fake, token, spec="k8s:ns1")
        wait_listening(api_b, timeout_s=15)
        nodes = {n["metadata"]["name"]: n for n in _call(api_b, "GET", "/v1/nodes")[1]["items"]}
        assert nodes["n3"]["spec"]["unschedulable"] is True
        pool = _call(api_b, "GET", "/v1/pools/p0")[1]
        assert pool["spec"]["wants"] == 2 and pool["spec"]["reason"] == "warm capacity"
        assert pool["metadata"]["generation"] == 1
        code, _ = _call(api_b, "DELETE", "/v1/pools/p0")
        assert code == 200 and "pools/p0.json" not in fake.states()
    finally:
        for p in (a, b):
            if p is not None and p.poll() is None:
                p.kill()
                p.wait()
        fake.close()


def test_file_spec_store_keeps_cordons_across_a_restart(tmp_path):
    from everserve_b200.serving.cluster import ControlPlane

    with ControlPlane(str(tmp_path / "cp"), engines=[{"name": "e0"}]) as cp:
        assert cp.request("PUT", "/v1/nodes/n0/cordon")[0] == 200
        coord = cp.procs["coord"]
        args = list(coord.args)
        coord.kill()
        coord.wait()
        cp._run("coord", args)  # the same flags: the same spec store
        wait_listening(cp.api)
        nodes = {n["metadata"]["name"]: n for n in cp.get("/v1/nodes")["items"]}
        assert nodes["n0"]["spec"]["unschedulable"] is True


class FakeEtcd:
    """etcd v3's JSON gateway, as much as a lease holder uses: lease grant and keepalive, a
    create-if-absent transaction, keys dropped when their lease expires, a revision counter."""

    def __init__(self):
        self.lock = threading.Lock()
        self.rev = 100
        self.leases = {}  # id -> (ttl, expires_at)
        self.kv = {}  # key -> (value, create_revision, lease id)
        self.next_id = 7000
        fake = self

        class H(BaseHTTPRequestHandler):
            def _send(self, obj):
                body = json.dumps(obj).encode()
                self.send_response(200)
                self.send_header("Content-Length", str(len(body)))
                self.end_headers()
                self.wfile.write(body)

            def do_POST(self):  # noqa: N802
                req = json.loads(self.rfile.read(int(self.headers.get("Content-Length", "0"))) or b"{}")
                now = time.monotonic()
                with fake.lock:
                    for lid, (ttl, exp) in list(fake.leases.items()):
                        if exp < now:  # expired: its keys go
                            del fake.leases[lid]
                            for k in [k for k, v in fake.kv.items() if v[2] == lid]:
                                del fake.kv[k]
                                fake.rev += 1
                    if self.path == "/v3/lease/grant":
                        fake.next_id += 1
                        fake.leases[str(fake.next_id)] = (int(req["TTL"]), now + int(req["TTL"]))
                        return self._send({"ID": str(fake.next_id), "TTL": str(req["TTL"])})
                    if self.path == "/v3/lease/keepalive":
                        lid = str(req["ID"])
                        if lid not in fake.leases:
                            return self._send({"result": {"ID": lid}})  # TTL absent: gone
                        ttl = fake.leases[lid][0]
                        fake.leases[lid] = (ttl, now + ttl)
                        return self._send({"result": {"ID": lid, "TTL": str(ttl)}})
                    if self.path == "/v3/kv/txn":
                        key = base64.b64decode(req["compare"][0]["key"]).decode()
                        if key not in fake.kv:
                            put = req["success"][0]["request_put"]
                            fake.rev += 1
                            fake.kv[key] = (base64.b64decode(put["value"]).decode(), fake.rev, str(put["lease"]))
                            return self._send({"header": {"revision": str(fake.rev)}, "succeeded": True})
                        return self._send({"header": {"revision": str(fake.rev)}, "succeeded": False})
                self.send_response(404)
                self.end_headers()

            def log_message(self, *a):
                pass

        self.server = ThreadingHTTPServer(("127.0.0.1", 0), H)
        self.url = f"http://127.0.0.1:{self.server.server_address[1]}"
        threading.Thread(target=self.server.serve_forever, daemon=True).start()

    def holder(self, key="/everserve/coord"):
        with self.lock:
            v = self.kv.get(key)
            return (v[0], v[1]) if v else None

    def revoke_all(self):
        with self.lock:
            self.leases.clear()
            self.kv.clear()

    def close(self):
        self.server.shutdown()


def test_etcd_lease_term_standby_and_loss(tmp_path):
    etcd = FakeEtcd()
    procs = []

    def coord(name):
        api = f"127.0.0.1:{free_port()}"
        log = open(tmp_path / f"{name}.log", "w")  # noqa: SIM115
        p = subprocess.Popen([binary("everserve-coord"), "--listen", f"unix:{tmp_path}/{name}.sock", "--spec-store",
                              str(tmp_path / "spec"), "--lease", f"etcd:{etcd.url}/everserve/coord",
                              "--lease-duration-s", "2", "--lease-holder", name, "--api-addr", api],
                             stdout=log, stderr=subprocess.STDOUT)
        procs.append(p)
        return p, api

    try:
        a, api_a = coord("coord-a")
        wait_listening(api_a)
        held = etcd.holder()
        assert held[0] == "coord-a"
        b, api_b = coord("coord-b")
        time.sleep(1.5)
        assert b.poll() is None and etcd.holder()[0] == "coord-a"  # a keeps its lease alive
        a.send_signal(signal.SIGKILL)
        a.wait()
        wait_listening(api_b, timeout_s=15)  # a's etcd lease expires, its key goes, b creates it
        held_b = etcd.holder()
        assert held_b[0] == "coord-b" and held_b[1] > held[1]  # the term (create revision) grew
        assert f"term {held_b[1]}" in open(tmp_path / "coord-b.log").read()
        etcd.revoke_all()  # b's lease is gone: it stops
        assert b.wait(timeout=10) == 3
    finally:
        for p in procs:
            if p.poll() is None:
                p.kill()
                p.wait()
        etcd.close()
