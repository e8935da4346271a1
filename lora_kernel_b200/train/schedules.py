"""Learning-rate schedules: the reference's five (LINEAR_WARMUP, COSINE,
COSINE_WITH_RESTARTS, POLYNOMIAL, CONSTANT; include/nn/training_enhancements.hpp:42-91)
plus a linear warm-up prefix on every schedule.  Pure functions of the step, so
they can be evaluated on the host and written into the device state vector.
"""
from __future__ import annotations

import math


def lr_at(step: int, base_lr: float, schedule: str = "constant", warmup_steps: int = 0,
          total_steps: int = 1, min_lr_ratio: float = 0.0, power: float = 1.0,
          num_cycles: int = 1) -> float:
    """Learning rate for optimizer step `step` (0-based)."""
    if warmup_steps > 0 and step < warmup_steps:
        return base_lr * (step + 1) / warmup_steps
    if schedule in ("constant", "none"):
        return base_lr
    t = step - warmup_steps
    span = max(1, total_steps - warmup_steps)
    frac = min(1.0, max(0.0, t / span))
    lo = base_lr * min_lr_ratio
    if schedule == "linear_warmup" or schedule == "linear":
        return lo + (base_lr - lo) * (1.0 - frac)
    if schedule == "cosine":
        return lo + (base_lr - lo) * 0.5 * (1.0 + math.cos(math.pi * frac))
    if schedule == "cosine_restarts" or schedule == "cosine_with_restarts":
        if frac >= 1.0:
            return lo
        cyc = (frac * num_cycles) % 1.0
        return lo + (base_lr - lo) * 0.5 * (1.0 + math.cos(math.pi * cyc))
    if schedule == "polynomial":
        return lo + (base_lr - lo) * (1.0 - frac) ** power
    raise ValueError(f"unknown schedule {schedule!r}")


class LRScheduler:
    """Stateful wrapper mirroring the reference's LRScheduler::get_lr(step)."""

    def __init__(self, base_lr: float, schedule: str = "constant", warmup_steps: int = 0,
                 total_steps: int = 1, min_lr_ratio: float = 0.0, power: float = 1.0,
                 num_cycles: int = 1):
        self.kw = dict(base_lr=base_lr, schedule=schedule, warmup_steps=warmup_steps,
                       total_steps=total_steps, min_lr_ratio=min_lr_ratio, power=power,
                       num_cycles=num_cycles)

    def get_lr(self, step: int) -> float:
        return lr_at(step, **self.kw)

    def set_base_lr(self, lr: float) -> None:
        self.kw["base_lr"] = lr
