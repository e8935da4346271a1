"""Prometheus text-format metrics (counters, gauges, cumulative histograms).

Reference: PrometheusExporter (include/monitoring/production_monitoring.hpp:
30-69), whose "histogram" printed one +Inf bucket line per sample, and
LatencyTracker p50/p95/p99 (:72-101).  Here a histogram has fixed cumulative
buckets, `_sum` and `_count`, and quantiles are computed from a bounded window
of raw samples.
"""
from __future__ import annotations

import bisect
import threading
from collections import deque
from typing import Dict, Iterable, List, Optional, Sequence, Tuple

DEFAULT_BUCKETS = (0.001, 0.0025, 0.005, 0.01, 0.025, 0.05, 0.1, 0.25, 0.5, 1.0, 2.5, 5.0, 10.0, 30.0, 60.0)


class _Metric:
    def __init__(self, name: str, help: str):
        self.name, self.help = name, help
        self.lock = threading.Lock()


class Counter(_Metric):
    kind = "counter"

    def __init__(self, name, help=""):
        super().__init__(name, help)
        self.v = 0.0

    def inc(self, n: float = 1.0):
        with self.lock:
            self.v += n

    def lines(self):
        return [f"{self.name} {self.v}"]


class Gauge(_Metric):
    kind = "gauge"

    def __init__(self, name, help=""):
        super().__init__(name, help)
        self.v = 0.0

    def set(self, v: float):
        self.v = float(v)

    def lines(self):
        return [f"{self.name} {self.v}"]


class Histogram(_Metric):
    kind = "histogram"

    def __init__(self, name, help="", buckets: Sequence[float] = DEFAULT_BUCKETS, window: int = 10000):
        super().__init__(name, help)
        self.bounds = sorted(buckets)
        self.counts = [0] * (len(self.bounds) + 1)
        self.sum = 0.0
        self.n = 0
        self.samples: deque = deque(maxlen=window)

    def observe(self, v: float):
        with self.lock:
            self.counts[bisect.bisect_left(self.bounds, v)] += 1
            self.sum += v
            self.n += 1
            self.samples.append(v)

    def quantile(self, q: float) -> float:
        with self.lock:
            s = sorted(self.samples)
        if not s:
            return float("nan")
        k = min(len(s) - 1, max(0, int(round(q * (len(s) - 1)))))
        return s[k]

    def lines(self):
        out, cum = [], 0
        for b, c in zip(self.bounds, self.counts):
            cum += c
            out.append(f'{self.name}_bucket{{le="{b}"}} {cum}')
        out.append(f'{self.name}_bucket{{le="+Inf"}} {self.n}')
        out.append(f"{self.name}_sum {self.sum}")
        out.append(f"{self.name}_count {self.n}")
        return out


class Registry:
    def __init__(self, prefix: str = "lora_kernel_"):
        self.prefix = prefix
        self.metrics: Dict[str, _Metric] = {}

    def _get(self, cls, name, help, **kw):
        full = self.prefix + name
        m = self.metrics.get(full)
        if m is None:
            m = cls(full, help, **kw)
            self.metrics[full] = m
        return m

    def counter(self, name, help="") -> Counter:
        return self._get(Counter, name, help)

    def gauge(self, name, help="") -> Gauge:
        return self._get(Gauge, name, help)

    def histogram(self, name, help="", **kw) -> Histogram:
        return self._get(Histogram, name, help, **kw)

    def exposition(self) -> str:
        lines = []
        for m in self.metrics.values():
            lines.append(f"# HELP {m.name} {m.help}")
            lines.append(f"# TYPE {m.name} {m.kind}")
            lines.extend(m.lines())
        return "\n".join(lines) + "\n"


REGISTRY = Registry()


# ------------------------------------------------------------------ training
B200_BF16_DENSE_TFLOPS = 2250.0  # nominal dense bf16 tensor peak per GPU (no sparsity)


def train_flops_per_token(cfg, seq_len: int) -> float:
    """Model FLOPs of one trained token: TransformerConfig.flops_per_token
    (6 x GEMM parameters + causal attention, forward and backward)."""
    return cfg.flops_per_token(seq_len)


def mfu(tokens_per_s: float, flops_per_token: float, n_gpus: int,
        peak_tflops: float = B200_BF16_DENSE_TFLOPS) -> float:
    """Model FLOPs utilisation: achieved model FLOP/s over n_gpus x peak."""
    return tokens_per_s * flops_per_token / (n_gpus * peak_tflops * 1e12)


class TrainMetrics:
    """Training step records -> Prometheus gauges in REGISTRY and, when a path
    is given, one JSON line per record appended to that file."""

    FIELDS = ("loss", "grad_norm", "loss_scale", "skipped", "lr", "tokens_per_s", "mfu")

    def __init__(self, path: str = "", registry: Optional["Registry"] = None):
        reg = registry or REGISTRY
        self.path = path
        self.g = {k: reg.gauge(f"train_{k}", f"training {k.replace('_', ' ')}") for k in self.FIELDS}
        self.g_step = reg.gauge("train_step", "optimizer steps taken")
        self.f = open(path, "a", buffering=1) if path else None

    def record(self, rec: dict) -> None:
        import json
        for k, g in self.g.items():
            if k in rec and rec[k] is not None:
                g.set(rec[k])
        if "step" in rec:
            self.g_step.set(rec["step"])
        if self.f is not None:
            self.f.write(json.dumps(rec) + "\n")

    def close(self) -> None:
        if self.f is not None:
            self.f.close()
            self.f = None

