"""Serving replicas: several independent engines (one per GPU or per tensor-
parallel group) behind one server, each driven by its own worker thread.

Routing policies
  round_robin       1, 2, ..., N, 1, ...
  least_loaded      the replica with the fewest unfinished requests
  prefix_affinity   requests whose first `affinity_tokens` tokens agree go to
                    the same replica, so a shared prompt prefix is prefilled
                    once and then served from that replica's prefix cache;
                    falls back to least_loaded when the preferred replica has
                    `slack` more unfinished requests than the least loaded one.

Reference: ModelReplicas (include/serving/serving_production.hpp:246-265,
round-robin over replica objects).
"""
from __future__ import annotations

import hashlib
import threading
from typing import List, Sequence

from .server import EngineWorker


class ReplicaPool:
    POLICIES = ("round_robin", "least_loaded", "prefix_affinity")

    def __init__(self, engines: Sequence, policy: str = "least_loaded", affinity_tokens: int = 64,
                 slack: int = 8):
        if not engines:
            raise ValueError("ReplicaPool needs at least one engine")
        if policy not in self.POLICIES:
            raise ValueError(f"policy must be one of {self.POLICIES}")
        self.engines = list(engines)
        self.workers = [EngineWorker(e) for e in self.engines]
        self.policy = policy
        self.affinity_tokens = affinity_tokens
        self.slack = slack
        self.outstanding: List[int] = [0] * len(self.engines)
        self.routed: List[int] = [0] * len(self.engines)
        self._rr = 0
        self._lock = threading.Lock()

    @property
    def cfg(self):
        return self.engines[0].cfg

    def _least(self) -> int:
        return min(range(len(self.outstanding)), key=lambda i: (self.outstanding[i], i))

    def pick(self, prompt: Sequence[int]) -> int:
        with self._lock:
            if self.policy == "round_robin":
                i = self._rr % len(self.workers)
                self._rr += 1
            elif self.policy == "least_loaded":
                i = self._least()
            else:
                key = ",".join(map(str, prompt[: self.affinity_tokens])).encode()
                i = int.from_bytes(hashlib.blake2b(key, digest_size=8).digest(), "little") % len(self.workers)
                j = self._least()
                if self.outstanding[i] > self.outstanding[j] + self.slack:
                    i = j
            self.outstanding[i] += 1
            self.routed[i] += 1
            return i

    def submit(self, prompt, params, on_token, priority: int = 0) -> int:
        """Route a request to a replica; returns a pool-wide request handle
        (replica index in the low bits), which abort() takes."""
        i = self.pick(prompt)

        def wrapped(r, t, _i=i):
            if r.finished:
                with self._lock:
                    self.outstanding[_i] -= 1
            on_token(r, t)
        try:
            rid = self.workers[i].submit(prompt, params, wrapped, priority)
        except Exception:
            with self._lock:
                self.outstanding[i] -= 1
            raise
        return rid * len(self.workers) + i

    def abort(self, handle: int, on_done=None) -> None:
        n = len(self.workers)
        i, rid = handle % n, handle // n

        def done(ok, _i=i):
            if ok:
                with self._lock:
                    self.outstanding[_i] -= 1
            if on_done is not None:
                on_done(ok)
        self.workers[i].abort(rid, done)

    def running(self) -> int:
        return sum(len(e.running) for e in self.engines)

    def waiting(self) -> int:
        return sum(len(e.waiting) for e in self.engines)

    def shutdown(self) -> None:
        for w in self.workers:
            w.shutdown()
