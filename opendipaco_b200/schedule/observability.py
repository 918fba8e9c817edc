"""Live metrics: Prometheus text over HTTP and periodic JSON snapshots
(reference ``schedule/observability.py``). Routes: ``/metrics``, ``/healthz``, ``/``."""

from __future__ import annotations

import json
import logging
import threading
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer

logger = logging.getLogger("opendipaco_b200.metrics")


class MetricsExporter:
    def __init__(self, metrics, *, host: str = "0.0.0.0", port: int = 0,
                 namespace: str = "opendipaco_transport"):
        self.metrics, self.namespace = metrics, namespace
        exporter = self

        class Handler(BaseHTTPRequestHandler):
            def log_message(self, *args):
                pass

            def do_GET(self):  # noqa: N802
                if self.path.startswith("/metrics"):
                    body = exporter.metrics.prometheus(exporter.namespace).encode()
                    ctype = "text/plain; version=0.0.4; charset=utf-8"
                elif self.path.startswith("/healthz"):
                    body, ctype = b"ok\n", "text/plain; charset=utf-8"
                else:
                    body, ctype = (exporter.metrics.report() + "\n").encode(), "text/plain; charset=utf-8"
                self.send_response(200)
                self.send_header("Content-Type", ctype)
                self.send_header("Content-Length", str(len(body)))
                self.end_headers()
                self.wfile.write(body)

        self._httpd = ThreadingHTTPServer((host, port), Handler)
        self.port = self._httpd.server_address[1]
        self._thread = threading.Thread(target=self._httpd.serve_forever, daemon=True)

    def start(self) -> "MetricsExporter":
        self._thread.start()
        return self

    def stop(self) -> None:
        for fn in (self._httpd.shutdown, self._httpd.server_close):
            try:
                fn()
            except Exception:
                pass


class MetricsLogger:
    def __init__(self, metrics, *, interval: float = 10.0, sink=None):
        self.metrics, self.interval = metrics, interval
        self.sink = sink or (lambda d: logger.info("transport_metrics %s", json.dumps(d)))
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._loop, daemon=True)

    def _loop(self) -> None:
        while not self._stop.wait(self.interval):
            try:
                self.sink(self.metrics.summary())
            except Exception:
                logger.exception("metrics sink failed")

    def start(self) -> "MetricsLogger":
        self._thread.start()
        return self

    def stop(self) -> None:
        self._stop.set()
