"""Liveness and readiness of a head: ``GET /live`` and ``GET /ready`` on a small HTTP server.

``/live`` answers 200 while the process serves. ``/ready`` answers 200 once the engine has
formed its first epoch and no membership change is in flight, else 503 with the reason (a load
balancer takes the engine out while a change completes).

Reference parity: adapters/vllm/everserve_vllm/health.py (the same two endpoints).
"""

from __future__ import annotations

import json
import threading
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer
from typing import Callable


class Health:
    def __init__(self, ready: Callable[[], tuple[bool, str]], host: str = "127.0.0.1", port: int = 0):
        outer = self

        class H(BaseHTTPRequestHandler):
            def do_GET(self):  # noqa: N802 - http.server's name
                if self.path == "/live":
                    code, body = 200, {"live": True}
                elif self.path == "/ready":
                    ok, why = outer.ready()
                    code, body = (200 if ok else 503), {"ready": ok, "reason": why}
                else:
                    code, body = 404, {"error": "not found"}
                data = json.dumps(body).encode()
                self.send_response(code)
                self.send_header("Content-Type", "application/json")
                self.send_header("Content-Length", str(len(data)))
                self.end_headers()
                self.wfile.write(data)

            def log_message(self, *a):
                pass

        self.ready = ready
        self.server = ThreadingHTTPServer((host, port), H)
        self.address = f"{host}:{self.server.server_address[1]}"
        self._t = threading.Thread(target=self.server.serve_forever, name="health", daemon=True)
        self._t.start()

    def close(self) -> None:
        self.server.shutdown()
        self.server.server_close()
