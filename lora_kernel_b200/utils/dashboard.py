"""Terminal dashboard for a running server: polls its /metrics and /alerts
and prints one refreshed summary (requests, tokens/s, TTFT and inter-token
latency quantiles, queue, KV-cache use, prefix-cache hit rate, per-GPU
utilisation / memory / power, firing alerts).

    python -m lora_kernel_b200.utils.dashboard --url http://127.0.0.1:8080 [--interval 2] [--once]

Reference: Dashboard (include/monitoring/production_monitoring.hpp:199-215),
which prints fixed text.
"""
from __future__ import annotations

import argparse
import json
import re
import time
import urllib.request
from typing import Dict, List, Optional, Tuple

_LINE = re.compile(r'^([a-zA-Z_:][a-zA-Z0-9_:]*)(\{([^}]*)\})?\s+(\S+)$')


def parse_prometheus(text: str) -> Dict[Tuple[str, Tuple[Tuple[str, str], ...]], float]:
    """{(name, sorted label pairs): value} of a Prometheus text exposition."""
    out = {}
    for line in text.splitlines():
        if not line or line.startswith("#"):
            continue
        m = _LINE.match(line.strip())
        if not m:
            continue
        labels = tuple(sorted(tuple(kv.split("=", 1)) for kv in re.findall(r'[a-zA-Z_]+="[^"]*"', m.group(3) or "")))
        labels = tuple((k, v.strip('"')) for k, v in labels)
        try:
            out[(m.group(1), labels)] = float(m.group(4))
        except ValueError:
            continue
    return out


def histogram_quantile(metrics, name: str, q: float) -> Optional[float]:
    """Upper bound of the bucket holding quantile q of a cumulative histogram."""
    buckets = sorted((float("inf") if dict(l)["le"] == "+Inf" else float(dict(l)["le"]), v)
                     for (n, l), v in metrics.items() if n == name + "_bucket")
    if not buckets or buckets[-1][1] == 0:
        return None
    total = buckets[-1][1]
    for le, c in buckets:
        if c >= q * total:
            return le
    return buckets[-1][0]


def render(metrics, alerts: List[dict], prefix: str = "lora_kernel_", prev=None, dt: float = 0.0) -> str:
    def g(name, labels=()):
        return metrics.get((prefix + name, labels))
    lines = []
    out_tok = g("generation_tokens_total") or 0.0
    rate = ""
    if prev is not None and dt > 0:
        rate = f"  ({(out_tok - (prev.get((prefix + 'generation_tokens_total', ())) or 0.0)) / dt:.0f} out tok/s)"
    lines.append(f"requests {g('requests_total') or 0:.0f}   prompt tokens {g('prompt_tokens_total') or 0:.0f}   "
                 f"generated {out_tok:.0f}{rate}")
    lines.append(f"running {g('num_requests_running') or 0:.0f}   waiting {g('num_requests_waiting') or 0:.0f}   "
                 f"KV cache {100 * (g('kv_cache_usage') or 0):.1f}%   prefix hits "
                 f"{100 * (g('prefix_cache_hit_rate') or 0):.1f}%   preemptions {g('preemptions_total') or 0:.0f}")
    for name, title in (("time_to_first_token_seconds", "TTFT"), ("inter_token_latency_seconds", "ITL"),
                        ("request_queue_time_seconds", "queue")):
        qs = [histogram_quantile(metrics, prefix + name, q) for q in (0.5, 0.9, 0.99)]
        if qs[0] is not None:
            lines.append(f"{title:6s} p50 <= {qs[0]:g}s  p90 <= {qs[1]:g}s  p99 <= {qs[2]:g}s")
    gpus = sorted({dict(l).get("gpu") for (n, l), _ in metrics.items() if n.startswith(prefix + "gpu_") and l})
    for gpu in gpus:
        lab = (("gpu", gpu),)
        lines.append(f"GPU {gpu}: util {g('gpu_utilization_percent', lab) or 0:.0f}%   "
                     f"mem {((g('gpu_memory_used_bytes', lab) or 0) / 2 ** 30):.1f} GiB   "
                     f"SM {g('gpu_sm_clock_mhz', lab) or 0:.0f} MHz   power {g('gpu_power_watts', lab) or 0:.0f} W")
    for a in alerts:
        lines.append(f"ALERT {a['name']}: {a['metric']} {a['op']} {a['threshold']} (now {a['value']:g})")
    return "\n".join(lines)


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description="terminal dashboard of a lora_kernel_b200 server")
    ap.add_argument("--url", default="http://127.0.0.1:8080")
    ap.add_argument("--interval", type=float, default=2.0)
    ap.add_argument("--once", action="store_true")
    a = ap.parse_args(argv)
    prev, t_prev = None, None
    while True:
        with urllib.request.urlopen(a.url + "/metrics", timeout=10) as r:
            metrics = parse_prometheus(r.read().decode())
        try:
            with urllib.request.urlopen(a.url + "/alerts", timeout=10) as r:
                alerts = json.loads(r.read().decode()).get("firing", [])
        except OSError:
            alerts = []
        now = time.monotonic()
        text = render(metrics, alerts, prev=prev, dt=(now - t_prev) if t_prev else 0.0)
        print(text if a.once else "\x1b[2J\x1b[H" + text, flush=True)
        if a.once:
            return
        prev, t_prev = metrics, now
        time.sleep(a.interval)


if __name__ == "__main__":
    main()
