"""Prometheus metrics of the serving process (rendered by the HTTP server's /metrics).

Parity: SGLang's /metrics that the reference exposes (its `--enable-metrics`), with the scheduler counters
this build keeps (steps, tokens, prefix-cache hits, retractions) and TTFT / end-to-end latency histograms.
"""
from __future__ import annotations

try:
    from prometheus_client import CollectorRegistry, Counter, Gauge, Histogram, generate_latest
except ImportError:  # pragma: no cover
    CollectorRegistry = None

_BUCKETS = (0.005, 0.01, 0.02, 0.05, 0.1, 0.2, 0.5, 1.0, 2.0, 5.0, 10.0, 30.0, 60.0)


class Metrics:
    def __init__(self):
        self.registry = CollectorRegistry() if CollectorRegistry is not None else None
        r = self.registry
        self.requests_total = Counter("snb_requests_total", "requests received", registry=r)
        self.tokens_total = Counter("snb_generated_tokens_total", "tokens generated", registry=r)
        self.ttft = Histogram("snb_time_to_first_token_seconds", "TTFT", buckets=_BUCKETS, registry=r)
        self.e2e = Histogram("snb_e2e_request_latency_seconds", "request latency", buckets=_BUCKETS, registry=r)
        self.running = Gauge("snb_num_running_reqs", "running requests", registry=r)
        self.waiting = Gauge("snb_num_queue_reqs", "queued requests", registry=r)
        self.free_pages = Gauge("snb_kv_free_pages", "free KV pages", registry=r)
        self.cache_hit = Gauge("snb_cache_hit_rate", "prefix-cache hit rate (tokens)", registry=r)
        self.steps = Gauge("snb_scheduler_steps", "scheduler steps", registry=r)
        self.step_ms = Gauge("snb_step_device_ms_p50", "median device time of recent steps (ms)", ["kind"],
                             registry=r)

    def update_from(self, engine) -> None:
        s = engine.scheduler
        self.running.set(len(s.running))
        self.waiting.set(len(s.waiting))
        self.free_pages.set(s.alloc.available())
        pt = s.stats.get("prompt_tokens", 0)
        self.cache_hit.set(s.stats.get("cache_hit_tokens", 0) / pt if pt else 0.0)
        self.steps.set(s.stats.get("steps", 0))
        for kind, name in ((0, "decode"), (1, "prefill_or_mixed")):
            v = sorted(ms for k, ms in list(getattr(s, "device_ms", [])) if k == kind)
            self.step_ms.labels(kind=name).set(v[len(v) // 2] if v else 0.0)

    def render(self) -> str:
        return generate_latest(self.registry).decode()
