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

    def __init__(self, name, help="", labels: Optional[Dict[str, str]] = None):
        super().__init__(name, help)
        self.v = 0.0
        self.labels = dict(labels or {})

    def set(self, v: float):
        self.v = float(v)

    def lines(self):
        if self.labels:
            lab = ",".join(f'{k}="{v}"' for k, v in sorted(self.labels.items()))
            return [f"{self.name}{{{lab}}} {self.v}"]
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

    def gauge(self, name, help="", labels: Optional[Dict[str, str]] = None) -> Gauge:
        if not labels:
            return self._get(Gauge, name, help)
        key = self.prefix + name + "{" + ",".join(f"{k}={v}" for k, v in sorted(labels.items())) + "}"
        m = self.metrics.get(key)
        if m is None:
            m = self.metrics[key] = Gauge(self.prefix + name, help, labels)
        return m

    def histogram(self, name, help="", **kw) -> Histogram:
        return self._get(Histogram, name, help, **kw)

    def exposition(self) -> str:
        """Prometheus text format; series of one name (labelled gauges) share
        one HELP / TYPE header."""
        lines, seen = [], set()
        order: Dict[str, List[_Metric]] = {}
        for m in self.metrics.values():
            order.setdefault(m.name, []).append(m)
        for name, ms in order.items():
            if name not in seen:
                seen.add(name)
                lines.append(f"# HELP {name} {ms[0].help}")
                lines.append(f"# TYPE {name} {ms[0].kind}")
            for m in ms:
                lines.extend(m.lines())
        return "\n".join(lines) + "\n"


class DeviceMetrics:
    """Per-GPU gauges labelled gpu="<index>", refreshed by update(): device
    memory of this process from the CUDA caching allocator (allocated,
    reserved, peak allocated) and, through NVML (read-only queries), GPU
    utilisation, memory in use by all processes, SM clock, power and
    temperature.  Missing sources (no CUDA, no NVML) leave their gauges at 0.

    Reference: GPUUtilizationTracker (a constant 75 %), MemoryProfiler and
    PCIeMonitor (a constant) in include/monitoring/production_monitoring.hpp:122-159."""

    FIELDS = {
        "gpu_memory_allocated_bytes": "device memory held by live tensors of this process",
        "gpu_memory_reserved_bytes": "device memory reserved by this process's caching allocator",
        "gpu_memory_peak_bytes": "peak device memory held by tensors of this process",
        "gpu_utilization_percent": "percent of time a kernel ran in the last sample period (NVML)",
        "gpu_memory_used_bytes": "device memory used by all processes (NVML)",
        "gpu_sm_clock_mhz": "SM clock (NVML)",
        "gpu_power_watts": "board power draw (NVML)",
        "gpu_temperature_celsius": "GPU temperature (NVML)",
    }

    def __init__(self, device_index: int = 0, registry: Optional["Registry"] = None, nvml=None):
        self.idx = int(device_index)
        reg = registry or REGISTRY
        self.g = {k: reg.gauge(k, h, labels={"gpu": str(self.idx)}) for k, h in self.FIELDS.items()}
        self._nvml, self._h = nvml, None

    def _handle(self):
        if self._h is None:
            try:
                if self._nvml is None:
                    import pynvml
                    self._nvml = pynvml
                self._nvml.nvmlInit()
                self._h = self._nvml.nvmlDeviceGetHandleByIndex(self.idx)
            except Exception:
                self._h = False
        return self._h or None

    def update(self) -> Dict[str, float]:
        import torch
        out: Dict[str, float] = {}
        if torch.cuda.is_available() and self.idx < torch.cuda.device_count():
            st = torch.cuda.memory_stats(self.idx)
            out["gpu_memory_allocated_bytes"] = st.get("allocated_bytes.all.current", 0)
            out["gpu_memory_reserved_bytes"] = st.get("reserved_bytes.all.current", 0)
            out["gpu_memory_peak_bytes"] = st.get("allocated_bytes.all.peak", 0)
        h = self._handle()
        if h is not None:
            n = self._nvml
            try:
                out["gpu_utilization_percent"] = n.nvmlDeviceGetUtilizationRates(h).gpu
                out["gpu_memory_used_bytes"] = n.nvmlDeviceGetMemoryInfo(h).used
                out["gpu_sm_clock_mhz"] = n.nvmlDeviceGetClockInfo(h, n.NVML_CLOCK_SM)
                out["gpu_power_watts"] = n.nvmlDeviceGetPowerUsage(h) / 1000.0
                out["gpu_temperature_celsius"] = n.nvmlDeviceGetTemperature(h, n.NVML_TEMPERATURE_GPU)
            except Exception:
                pass
        for k, v in out.items():
            self.g[k].set(v)
        return out


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


# ------------------------------------------------------------------ alerting
class AlertRule:
    """Fires while `metric` (a gauge or counter name without the registry
    prefix, a histogram's quantile with `quantile`) compares `op` to
    `threshold` (op: ">", ">=", "<", "<=") for at least `for_s` seconds."""

    OPS = {">": lambda a, b: a > b, ">=": lambda a, b: a >= b, "<": lambda a, b: a < b, "<=": lambda a, b: a <= b}

    def __init__(self, name: str, metric: str, op: str, threshold: float, for_s: float = 0.0,
                 quantile: Optional[float] = None, labels: Optional[Dict[str, str]] = None):
        if op not in self.OPS:
            raise ValueError(f"alert op must be one of {sorted(self.OPS)}")
        self.name, self.metric, self.op, self.threshold = name, metric, op, float(threshold)
        self.for_s, self.quantile, self.labels = float(for_s), quantile, dict(labels or {})
        self.since: Optional[float] = None


class AlertManager:
    """Evaluates alert rules over a Registry; `check(now)` returns the firing
    alerts (name, metric, value, threshold) and logs each newly firing one.

    Reference: AlertManager (include/monitoring/production_monitoring.hpp:185-196),
    whose check_all returns nothing."""

    def __init__(self, rules: Iterable[AlertRule], registry: Optional["Registry"] = None, log=None):
        import copy
        self.rules = [copy.copy(r) for r in rules]  # a rule's "since" state is per manager
        self.reg = registry or REGISTRY
        self.log = log
        self.firing: Dict[str, dict] = {}

    def _value(self, r: AlertRule) -> Optional[float]:
        for m in self.reg.metrics.values():
            if m.name != self.reg.prefix + r.metric:
                continue
            if isinstance(m, Histogram):
                return m.quantile(r.quantile if r.quantile is not None else 0.5) if m.n else None
            if getattr(m, "labels", {}) == r.labels or not r.labels:
                return m.v
        return None

    def check(self, now: Optional[float] = None) -> List[dict]:
        import time
        now = time.monotonic() if now is None else now
        out = []
        for r in self.rules:
            v = self._value(r)
            if v is None or v != v or not AlertRule.OPS[r.op](v, r.threshold):
                r.since = None
                self.firing.pop(r.name, None)
                continue
            r.since = now if r.since is None else r.since
            if now - r.since >= r.for_s:
                alert = {"name": r.name, "metric": r.metric, "value": v, "op": r.op, "threshold": r.threshold}
                if r.name not in self.firing and self.log is not None:
                    self.log.warning("alert %s: %s %s %s (value %s)", r.name, r.metric, r.op, r.threshold, v)
                self.firing[r.name] = alert
                out.append(alert)
        return out

