"""Node notices: the daemon polls a (fake) cloud or cluster endpoint and the coordinator drains the
node when a departure is announced."""

import json
import threading
import time
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer

import pytest

from everserve_b200.serving.cluster import ControlPlane


class Fake:
    """One fake metadata endpoint; `notice` switches the announced departure on."""

    def __init__(self, source: str):
        self.source = source
        self.notice = False
        self.seen_headers = []
        fake = self

        class H(BaseHTTPRequestHandler):
            def _send(self, code, body=b""):
                self.send_response(code)
                self.send_header("Content-Length", str(len(body)))
                self.end_headers()
                self.wfile.write(body)

            def do_PUT(self):  # noqa: N802
                fake.seen_headers.append(dict(self.headers))
                if self.path == "/latest/api/token":
                    return self._send(200, b"tok123")
                self._send(404)

            def do_GET(self):  # noqa: N802
                fake.seen_headers.append(dict(self.headers))
                s, p = fake.source, self.path
                if s == "aws" and p == "/latest/meta-data/spot/instance-action":
                    if self.headers.get("X-aws-ec2-metadata-token") != "tok123":
                        return self._send(401)
                    if fake.notice:
                        return self._send(200, json.dumps({"action": "terminate",
                                                           "time": "2030-01-01T00:00:00Z"}).encode())
                    return self._send(404)
                if s == "gcp" and p.startswith("/computeMetadata/v1/instance/"):
                    if self.headers.get("Metadata-Flavor") != "Google":
                        return self._send(403)
                    if p.endswith("preempted"):
                        return self._send(200, b"TRUE" if fake.notice else b"FALSE")
                    return self._send(200, b"NONE")
                if s == "azure" and p.startswith("/metadata/scheduledevents"):
                    ev = [{"EventType": "Preempt", "NotBefore": "Tue, 01 Jan 2030 00:00:00 GMT",
                           "Resources": ["vm0"]}] if fake.notice else []
                    return self._send(200, json.dumps({"DocumentIncarnation": 1, "Events": ev}).encode())
                if s == "k8s" and p == "/api/v1/nodes/n0":
                    spec = {"taints": [{"key": "ToBeDeletedByClusterAutoscaler", "effect": "NoSchedule"}]} \
                        if fake.notice else {}
                    return self._send(200, json.dumps({"metadata": {"name": "n0"}, "spec": spec}).encode())
                self._send(404)

            def log_message(self, *a):
                pass

        self.server = ThreadingHTTPServer(("127.0.0.1", 0), H)
        self.addr = f"127.0.0.1:{self.server.server_address[1]}"
        threading.Thread(target=self.server.serve_forever, daemon=True).start()

    def close(self):
        self.server.shutdown()


@pytest.mark.parametrize("source", ["aws", "gcp", "azure", "k8s"])
def test_cloud_notice_drains_the_node(tmp_path, source):
    fake = Fake(source)
    try:
        args = ["--notice-source", source, "--notice-endpoint", fake.addr, "--notice-interval-ms", "100"]
        with ControlPlane(str(tmp_path), node_args=args) as cp:
            time.sleep(0.5)
            assert not any("draining" in e["text"] for e in cp.get("/v1/watch")["events"])
            fake.notice = True
            deadline = time.monotonic() + 10
            while time.monotonic() < deadline:
                if any(f"node notice: {source}" in e["text"] for e in cp.get("/v1/watch")["events"]):
                    break
                time.sleep(0.05)
            events = [e["text"] for e in cp.get("/v1/watch")["events"]]
            assert any(f"n0 draining (node notice: {source}" in t for t in events), events
            node = cp.get("/v1/nodes")["items"][0]
            if source in ("aws", "azure"):
                assert node["spec"]["drainByMs"] == 1893456000000  # the announced deadline (2030-01-01)
    finally:
        fake.close()
