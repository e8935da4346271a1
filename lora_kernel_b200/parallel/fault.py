"""Failure detection and host-side fault injection.

HeartbeatMonitor: every rank writes a monotonically increasing beat (step and
wall time) into the process group's key-value store from a daemon thread;
`check()` raises RankFailure naming the ranks whose beat is older than
`timeout_s` (a rank that died, hung on the host or never joined).  Ranks call
check() between steps, before launching the next collective, so no rank ever
leaves a collective or kernel half-done.

FaultInjector: env-driven host faults for tests and drills, parsed from
LORAK_FAULT (comma-separated):
    kill_rank:R@step:S        rank R exits (os._exit(17)) at the start of step S
    delay_rank:R@step:S:SEC   rank R sleeps SEC seconds at step S
    nan_grad@step:S           every rank turns its gradients to NaN at step S
                              (exercises the overflow-skip path)
    raise_rank:R@step:S       rank R raises RuntimeError at step S
Nothing here faults, traps or hangs a GPU: device-side waits are bounded in the
kernels themselves and report through the status word.

Reference: FaultTolerantTrainer (include/distributed/distributed_training.hpp:
292-317, heartbeat always true), BarrierWithTimeout (:204-235, times nothing),
SignalRecoveryHandler (include/core/signal_handler.hpp:12-53, flag never polled).
"""
from __future__ import annotations

import os
import threading
import time
from dataclasses import dataclass
from typing import Tuple, Dict, List, Optional


class RankFailure(RuntimeError):
    def __init__(self, ranks: List[int], msg: str = ""):
        super().__init__(msg or f"ranks {ranks} stopped sending heartbeats")
        self.ranks = ranks


class HeartbeatMonitor:
    def __init__(self, store, rank: int, world: int, interval_s: float = 1.0, timeout_s: float = 10.0,
                 prefix: str = "lorak_hb"):
        self.store, self.rank, self.world = store, rank, world
        self.interval, self.timeout, self.prefix = interval_s, timeout_s, prefix
        self.step = 0
        self._stop = threading.Event()
        self._beat()
        self.thread = threading.Thread(target=self._loop, daemon=True)
        self.thread.start()

    def _beat(self):
        self.store.set(f"{self.prefix}/{self.rank}", f"{self.step}:{time.time():.3f}")

    def _loop(self):
        while not self._stop.wait(self.interval):
            try:
                self._beat()
            except Exception:
                return

    def set_step(self, step: int) -> None:
        self.step = step

    def stale_ranks(self) -> List[int]:
        now = time.time()
        bad = []
        for r in range(self.world):
            try:
                v = self.store.get(f"{self.prefix}/{r}").decode()
                t = float(v.split(":")[1])
            except Exception:
                bad.append(r)
                continue
            if now - t > self.timeout:
                bad.append(r)
        return bad

    def check(self) -> None:
        bad = self.stale_ranks()
        if bad:
            raise RankFailure(bad)

    def stop(self) -> None:
        self._stop.set()


@dataclass
class Fault:
    kind: str
    rank: int
    step: int
    arg: float = 0.0


def parse_faults(spec: Optional[str] = None) -> List[Fault]:
    spec = os.environ.get("LORAK_FAULT", "") if spec is None else spec
    out = []
    for item in filter(None, (s.strip() for s in spec.split(","))):
        head, _, tail = item.partition("@step:")
        parts = tail.split(":")
        step = int(parts[0])
        arg = float(parts[1]) if len(parts) > 1 else 0.0
        kind, _, r = head.partition(":")
        out.append(Fault(kind, int(r) if r else -1, step, arg))
    return out


def kill_is_safe() -> Tuple[bool, str]:
    """Whether ending a rank's process abruptly is allowed here.

    A rank whose device memory is bound to an NVLink multicast (NVLS) object
    must not die in the middle of a job: when that happened the other ranks'
    GPUs raised NVLink faults.  Killing is therefore allowed only for CPU /
    gloo jobs, or for NCCL jobs that run with multicast off in this library
    (LK_NVLS=0) and in NCCL (NCCL_NVLS_ENABLE=0)."""
    import torch.distributed as dist
    backend = dist.get_backend() if dist.is_available() and dist.is_initialized() else None
    if backend in (None, "gloo"):
        return True, ""
    if os.environ.get("LK_NVLS") == "0" and os.environ.get("NCCL_NVLS_ENABLE") == "0":
        return True, ""
    return False, (f"kill_rank refused on a '{backend}' job with NVLink multicast possible: set LK_NVLS=0 and "
                   "NCCL_NVLS_ENABLE=0, or inject raise_rank / delay_rank instead")


class FaultInjector:
    def __init__(self, rank: int, spec: Optional[str] = None):
        self.rank = rank
        self.faults = parse_faults(spec)
        if any(f.kind == "kill_rank" for f in self.faults):
            ok, why = kill_is_safe()
            if not ok:
                raise ValueError(why)

    def _mine(self, f: Fault, step: int) -> bool:
        return f.step == step and (f.rank < 0 or f.rank == self.rank)

    def at_step(self, step: int) -> None:
        """Host faults at the start of a step (between steps: nothing in flight)."""
        for f in self.faults:
            if not self._mine(f, step):
                continue
            if f.kind == "kill_rank":
                ok, why = kill_is_safe()
                if not ok:
                    raise RuntimeError(why)
                os._exit(17)
            elif f.kind == "delay_rank":
                time.sleep(f.arg)
            elif f.kind == "raise_rank":
                raise RuntimeError(f"injected failure on rank {self.rank} at step {step}")

    def on_grads(self, step: int, grads) -> None:
        """Gradient faults, applied after backward and before the optimizer."""
        for f in self.faults:
            if self._mine(f, step) and f.kind == "nan_grad":
                grads.fill_(float("nan"))
