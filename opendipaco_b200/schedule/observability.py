"""Live views of a server's :class:`~opendipaco_b200.schedule.reactor.TransportMetrics`
while a run is in flight.

* :class:`MetricsExporter` serves three routes over HTTP on a port of its own:
  ``/metrics`` (Prometheus text exposition), ``/healthz`` and ``/`` (the human report).
* :class:`MetricsLogger` hands a JSON-able snapshot to a sink (by default one log line)
  every ``interval`` seconds.

Both only read the metrics object (its accessors take its lock), so they never touch the
transport. Servers start them with ``start_metrics_server()`` /
``start_metrics_logging()`` and stop them in ``shutdown()``. Routes and defaults follow
the reference's ``src/opendipaco/schedule/observability.py``; the implementation (a WSGI
route table, a generic periodic runner) is this module's own.
"""

from __future__ import annotations

import json
import logging
import threading
from socketserver import ThreadingMixIn
from wsgiref.simple_server import WSGIRequestHandler, WSGIServer, make_server

log = logging.getLogger("opendipaco_b200.metrics")

_TEXT = "text/plain; charset=utf-8"


class _QuietHandler(WSGIRequestHandler):
    def log_message(self, *args):  # no per-request access log on stderr
        pass


class _ThreadedWSGIServer(ThreadingMixIn, WSGIServer):
    daemon_threads = True


class MetricsExporter:
    """HTTP endpoint for one metrics object (separate from the transport port)."""

    def __init__(self, metrics, *, host: str = "0.0.0.0", port: int = 0, namespace: str = "opendipaco_transport"):
        self.metrics, self.namespace = metrics, namespace
        self.routes = {
            "/metrics": ("text/plain; version=0.0.4; charset=utf-8", lambda: metrics.prometheus(namespace)),
            "/healthz": (_TEXT, lambda: "ok\n"),
        }
        self._httpd = make_server(host, port, self._app, server_class=_ThreadedWSGIServer,
                                  handler_class=_QuietHandler)
        self.port = self._httpd.server_address[1]
        self._thread = threading.Thread(target=self._httpd.serve_forever, name="odp-metrics-http", daemon=True)

    def _app(self, environ, start_response):
        path = environ.get("PATH_INFO", "/")
        ctype, render = next(((c, r) for prefix, (c, r) in self.routes.items() if path.startswith(prefix)),
                             (_TEXT, lambda: self.metrics.report() + "\n"))
        body = render().encode()
        start_response("200 OK", [("Content-Type", ctype), ("Content-Length", str(len(body)))])
        return [body]

    def start(self) -> "MetricsExporter":
        self._thread.start()
        return self

    def stop(self) -> None:
        for step in (self._httpd.shutdown, self._httpd.server_close):
            try:
                step()
            except Exception:  # best effort: the server may never have started
                pass


class _Periodic:
    """Calls ``fn`` every ``interval`` seconds on a daemon thread until stopped; an
    exception in ``fn`` is logged and does not end the loop."""

    def __init__(self, fn, interval: float, name: str):
        self.fn, self.interval = fn, interval
        self._halt = threading.Event()
        self._thread = threading.Thread(target=self._run, name=name, daemon=True)

    def _run(self) -> None:
        while not self._halt.wait(self.interval):
            try:
                self.fn()
            except Exception:
                log.exception("periodic metrics sink failed")

    def start(self) -> None:
        self._thread.start()

    def stop(self) -> None:
        self._halt.set()


class MetricsLogger:
    """Emit ``metrics.summary()`` every ``interval`` seconds to ``sink`` (default: one
    ``transport_metrics {json}`` log line)."""

    def __init__(self, metrics, *, interval: float = 10.0, sink=None):
        self.metrics, self.interval = metrics, interval
        self.sink = sink if sink is not None else (lambda snap: log.info("transport_metrics %s", json.dumps(snap)))
        self._runner = _Periodic(lambda: self.sink(self.metrics.summary()), interval, "odp-metrics-log")

    def start(self) -> "MetricsLogger":
        self._runner.start()
        return self

    def stop(self) -> None:
        self._runner.stop()
