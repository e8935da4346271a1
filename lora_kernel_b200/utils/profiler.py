"""Tracing and device-timed profiling.

  nvtx_range(name)      NVTX range (visible in Nsight / ncu range filters)
  PhaseTimer            CUDA-event timing per named phase, summed over steps,
                        reported as a table; `max_over_ranks()` reduces each
                        phase with MAX across the process group
  chrome_trace(fn, path) torch.profiler capture exported as a Chrome trace
  ph(name) / collecting(timer)
                        per-phase device timing of the training step: the
                        engine, optimizer and collectives wrap their launches
                        in ph(...), which costs one no-op context unless a
                        PhaseTimer is collecting

Reference: Profiler / ScopedTimer (include/core/profiler.hpp:25-137: host
steady_clock spans, Chrome traceEvents flush, top-10 report).
"""
from __future__ import annotations

import contextlib
import json
from collections import defaultdict
from typing import Callable, Dict, List

import torch


@contextlib.contextmanager
def nvtx_range(name: str):
    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()


class PhaseTimer:
    def __init__(self):
        self.events: Dict[str, List] = defaultdict(list)

    @contextlib.contextmanager
    def phase(self, name: str):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        with nvtx_range(name):
            yield
        e.record()
        self.events[name].append((s, e))

    def totals_ms(self) -> Dict[str, float]:
        torch.cuda.synchronize()
        return {k: sum(s.elapsed_time(e) for s, e in v) for k, v in self.events.items()}

    def max_over_ranks(self) -> Dict[str, float]:
        tot = self.totals_ms()
        if torch.distributed.is_initialized():
            names = [None] * torch.distributed.get_world_size()
            torch.distributed.all_gather_object(names, sorted(tot))
            keys = sorted(set().union(*names))  # a phase some rank never ran counts 0 there
            t = torch.tensor([tot.get(k, 0.0) for k in keys], device="cuda", dtype=torch.float64)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            tot = dict(zip(keys, t.tolist()))
        return tot

    def per_step_ms(self, steps: int) -> Dict[str, float]:
        """Max-over-ranks device time of each phase per step (every rank must
        call this: it is a collective when a process group is up)."""
        return {k: round(v / max(steps, 1), 3) for k, v in sorted(self.max_over_ranks().items())}

    def report(self, top: int = 20) -> str:
        tot = self.max_over_ranks()
        all_ms = sum(tot.values()) or 1.0
        rows = sorted(tot.items(), key=lambda kv: -kv[1])[:top]
        return "\n".join(f"{k:<32} {v:10.3f} ms {100 * v / all_ms:5.1f}%" for k, v in rows)


_ACTIVE: "PhaseTimer | None" = None
_NULL = contextlib.nullcontext()


def ph(name: str):
    """Time the enclosed launches as phase `name` (on the current stream) when
    a PhaseTimer is collecting; otherwise a no-op."""
    t = _ACTIVE
    return _NULL if t is None else t.phase(name)


@contextlib.contextmanager
def collecting(timer: "PhaseTimer"):
    """Make `timer` receive every ph(...) phase inside the block."""
    global _ACTIVE
    prev, _ACTIVE = _ACTIVE, timer
    try:
        yield timer
    finally:
        _ACTIVE = prev


def chrome_trace(fn: Callable[[], None], path: str, steps: int = 1) -> None:
    acts = [torch.profiler.ProfilerActivity.CPU]
    if torch.cuda.is_available():
        acts.append(torch.profiler.ProfilerActivity.CUDA)
    with torch.profiler.profile(activities=acts) as prof:
        for _ in range(steps):
            fn()
        if torch.cuda.is_available():
            torch.cuda.synchronize()
    prof.export_chrome_trace(path)
