"""Performance regression check for benchmark JSON lines.

    python bench.py > new.json
    python -m lora_kernel_b200.utils.perf_check new.json profiles/bench_llama1b_1gpu.json --tolerance 0.05

Compares the `value` of the newest JSON line of each file (lines that are not
JSON objects are skipped, so a whole log can be passed) and exits 1 when the
new value is worse than the reference by more than the tolerance (direction
from `higher_is_better`).  A run whose clock record shows a thermal or
hardware slowdown is reported as not comparable (exit 2) instead of as a
regression.  The metric, unit, GPU count and model must match.

Reference: PerformanceRegressionTest (in-header testing suite of
include/monitoring/production_monitoring.hpp, which prints passed).
"""
from __future__ import annotations

import argparse
import json
import sys
from typing import Optional

BAD_REASONS = {"hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown"}


def last_json(path: str) -> dict:
    rec: Optional[dict] = None
    with open(path) as f:
        for line in f:
            line = line.strip()
            if line.startswith("{"):
                try:
                    d = json.loads(line)
                except json.JSONDecodeError:
                    continue
                if isinstance(d, dict) and "value" in d:
                    rec = d
    if rec is None:
        raise ValueError(f"{path}: no benchmark JSON line")
    return rec


def compare(new: dict, ref: dict, tolerance: float = 0.05) -> dict:
    """{"status": "ok" | "regression" | "not_comparable", "ratio", "reason"}."""
    for k in ("metric", "unit", "n_gpus"):
        if new.get(k) != ref.get(k):
            return {"status": "not_comparable", "ratio": None, "reason": f"{k} differs: {new.get(k)!r} vs {ref.get(k)!r}"}
    if (new.get("config") or {}).get("model") != (ref.get("config") or {}).get("model"):
        return {"status": "not_comparable", "ratio": None, "reason": "model differs"}
    bad = BAD_REASONS & set((new.get("clocks") or {}).get("reasons", []))
    if bad:
        return {"status": "not_comparable", "ratio": None, "reason": f"clock slowdown during the run: {sorted(bad)}"}
    higher = ref.get("higher_is_better", True)
    ratio = new["value"] / ref["value"] if higher else ref["value"] / new["value"]
    status = "ok" if ratio >= 1.0 - tolerance else "regression"
    return {"status": status, "ratio": round(ratio, 4), "reason": ""}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="benchmark regression check")
    ap.add_argument("new")
    ap.add_argument("reference")
    ap.add_argument("--tolerance", type=float, default=0.05)
    a = ap.parse_args(argv)
    res = compare(last_json(a.new), last_json(a.reference), a.tolerance)
    print(json.dumps(res))
    return {"ok": 0, "regression": 1}.get(res["status"], 2)


if __name__ == "__main__":
    sys.exit(main())
