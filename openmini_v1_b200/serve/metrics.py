"""Prometheus metrics with the reference's metric names
(openmini-server/src/monitoring/metrics.rs:33-220,
openmini-server/src/monitoring/business_metrics.rs) so existing dashboards keep
working, plus TTFT / TPOT histograms. One registry per server instance.
"""
from __future__ import annotations

import time

from prometheus_client import CollectorRegistry, Counter, Gauge, Histogram, generate_latest

_LAT_MS = (1, 2, 5, 10, 20, 50, 100, 200, 500, 1000, 2000, 5000, 10000, 30000, 60000)


class Metrics:
    def __init__(self, registry: CollectorRegistry | None = None):
        r = self.registry = registry or CollectorRegistry()
        self.requests_total = Counter("openmini_inference_requests_total", "Inference requests", ["endpoint", "status"],
                                      registry=r)
        self.latency_ms = Histogram("openmini_inference_latency_ms", "End-to-end request latency (ms)", ["endpoint"],
                                    buckets=_LAT_MS, registry=r)
        self.request_duration = Histogram("openmini_request_duration_seconds", "Request duration (s)", ["endpoint"],
                                          registry=r)
        self.ttft_ms = Histogram("openmini_time_to_first_token_ms", "Time to first token (ms)", buckets=_LAT_MS,
                                 registry=r)
        self.tpot_ms = Histogram("openmini_time_per_output_token_ms", "Time per output token (ms)",
                                 buckets=(1, 2, 5, 10, 20, 50, 100, 200, 500), registry=r)
        self.tokens_total = Counter("openmini_inference_tokens_total", "Tokens processed", ["kind"], registry=r)
        self.token_throughput = Gauge("openmini_token_throughput", "Generated tokens per second (recent)",
                                      registry=r)
        self.active_requests = Gauge("openmini_active_requests", "Requests in flight", registry=r)
        self.active_connections = Gauge("openmini_active_connections", "Open connections", registry=r)
        self.batch_size = Gauge("openmini_batch_size", "Sequences in the last engine step", registry=r)
        self.queue_length = Gauge("openmini_scheduler_queue_length", "Waiting requests", registry=r)
        self.worker_queue_length = Gauge("openmini_worker_queue_length", "Tasks queued for workers", registry=r)
        self.preemptions_total = Counter("openmini_preemptions_total", "Requests preempted", registry=r)
        self.avg_wait_ms = Gauge("openmini_avg_wait_time_ms", "Average queue wait (ms)", registry=r)
        self.kv_cache_size = Gauge("openmini_kv_cache_size_bytes", "KV cache capacity (bytes)", registry=r)
        self.kv_cache_usage = Gauge("openmini_kv_cache_usage_bytes", "KV cache in use (bytes)", registry=r)
        self.gpu_memory_used = Gauge("openmini_gpu_memory_used_bytes", "Device memory allocated", registry=r)
        self.gpu_util = Gauge("openmini_gpu_utilization_percent", "Device busy fraction (%)", registry=r)
        self.memory_used = Gauge("openmini_memory_used_bytes", "Host RSS", registry=r)
        self.cpu_usage = Gauge("openmini_cpu_usage_percent", "Host CPU usage", registry=r)
        self.model_loaded = Gauge("openmini_model_loaded", "1 when a model is loaded", registry=r)
        self.dsa_topk_latency_us = Histogram("openmini_dsa_top_k_latency_us", "DSA top-k selection latency (us)",
                                             registry=r)
        self.dequantize_ops = Counter("openmini_dequantize_ops_total", "Quantised GEMM calls", registry=r)
        self.dequantize_throughput = Gauge("openmini_dequantize_throughput", "Dequantised weights per second",
                                           registry=r)
        self._tok_window = []

    def observe_request(self, endpoint: str, status: str, seconds: float):
        self.requests_total.labels(endpoint, status).inc()
        self.latency_ms.labels(endpoint).observe(seconds * 1e3)
        self.request_duration.labels(endpoint).observe(seconds)

    def observe_tokens(self, n: int, kind: str = "completion"):
        self.tokens_total.labels(kind).inc(n)
        now = time.time()
        self._tok_window.append((now, n))
        self._tok_window = [(t, k) for t, k in self._tok_window if now - t < 10.0]
        span = max(1e-3, now - self._tok_window[0][0]) if self._tok_window else 1.0
        self.token_throughput.set(sum(k for _, k in self._tok_window) / span)

    def update_engine(self, engine):
        try:
            self.queue_length.set(len(engine.sched.waiting))
            self.batch_size.set(len(engine.sched.running))
            bm = engine.bm
            per = engine.model.kv_bytes_per_block()
            self.kv_cache_size.set(bm.num_blocks * per)
            self.kv_cache_usage.set((bm.num_blocks - bm.num_free()) * per)
            if engine.is_cuda:
                import torch
                self.gpu_memory_used.set(torch.cuda.memory_allocated(engine.device))
        except Exception:
            pass
        try:
            import psutil
            p = psutil.Process()
            self.memory_used.set(p.memory_info().rss)
            self.cpu_usage.set(psutil.cpu_percent(interval=None))
        except Exception:
            pass

    def render(self) -> bytes:
        return generate_latest(self.registry)
