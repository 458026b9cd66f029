"""Logging: JSON-line or plain formatter, level from $OPENMINI_LOG / $RUST_LOG,
and a sampler that rate-limits repetitive messages (the reference's
tracing-subscriber JSON logger and log sampler,
openmini-server/src/logging/mod.rs:27-32, json_logger.rs, log_sampler.rs)."""
from __future__ import annotations

import json
import logging
import os
import sys
import threading
import time


class JsonFormatter(logging.Formatter):
    def format(self, record):
        d = {"ts": round(record.created, 6), "level": record.levelname.lower(), "target": record.name,
             "msg": record.getMessage()}
        for k, v in getattr(record, "fields", {}).items():
            d[k] = v
        if record.exc_info:
            d["exc"] = self.formatException(record.exc_info)
        return json.dumps(d, default=str)


class SamplingFilter(logging.Filter):
    """Let at most ``burst`` records with the same (logger, message template) through per ``window_s``."""

    def __init__(self, burst: int = 10, window_s: float = 1.0):
        super().__init__()
        self.burst, self.window = burst, window_s
        self.counts = {}
        self.lock = threading.Lock()

    def filter(self, record):
        key = (record.name, record.msg)
        now = time.monotonic()
        with self.lock:
            t0, n = self.counts.get(key, (now, 0))
            if now - t0 > self.window:
                t0, n = now, 0
            n += 1
            self.counts[key] = (t0, n)
        return n <= self.burst


def init_logging(level: str | None = None, json_format: bool | None = None, sample_burst: int = 0):
    level = (level or os.environ.get("OPENMINI_LOG") or os.environ.get("RUST_LOG") or "info").upper()
    if json_format is None:
        json_format = os.environ.get("OPENMINI_LOG_JSON", "0") == "1"
    h = logging.StreamHandler(sys.stderr)
    h.setFormatter(JsonFormatter() if json_format else logging.Formatter("%(asctime)s %(levelname)s %(name)s: %(message)s"))
    if sample_burst:
        h.addFilter(SamplingFilter(sample_burst))
    root = logging.getLogger("openmini")
    root.handlers[:] = [h]
    root.setLevel(getattr(logging, level, logging.INFO))
    root.propagate = False
    return root


def log_fields(logger, level, msg, **fields):
    logger.log(level, msg, extra={"fields": fields})
