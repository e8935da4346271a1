"""Token data sources.

NativeTokens: the C++ loader (csrc/runtime/token_loader.cpp): worker threads
fill a ring of page-locked host slots ahead of the step, synthetic or from a
memmap'd token file, each slot one contiguous ids|targets pair that a single
host-to-device copy moves.  SyntheticTokens: uniform random ids in [0, vocab)
from a seeded torch generator per rank, with next-token targets.  MemmapTokens: a flat
uint16 / uint32 token file read through numpy.memmap, sharded across data-
parallel ranks by contiguous windows.  CurriculumScheduler: sequence-length
warm-up.  Each source keeps a cursor so a checkpoint can resume the stream.

Reference: DataLoader (include/data/dataloader.hpp:63-159, which returns
random tokens regardless of the file), StreamDataset and CurriculumScheduler
(:162-200), ShardedDataset / DistributedDataLoader (include/data/datasets.hpp).
"""
from __future__ import annotations

import collections
from typing import Optional, Tuple

import numpy as np
import torch


class NativeTokens:
    """Prefetching token loader backed by the native runtime.

    next() returns host (ids, targets) [B, S] int64 tensors that stay valid
    for the next depth-2 calls; next_device(device) returns device tensors
    after one asynchronous copy on the current stream (the slot goes back to
    the producers once that copy has completed).  path=None: synthetic ids
    uniform in [0, vocab); otherwise a flat uint16 / uint32 token file cut
    into windows of seq+1 tokens, shuffled per epoch, sharded by rank.
    state()/load_state() carry the batch cursor for checkpoint resume."""

    def __init__(self, vocab: int, batch: int, seq: int, seed: int = 0, rank: int = 0, world: int = 1, *,
                 path: Optional[str] = None, dtype: str = "uint16", depth: int = 6, threads: int = 4,
                 shuffle: bool = True, fixed: bool = False, pin: bool = True):
        from .. import _rt
        if depth < 3:
            raise ValueError("NativeTokens: depth must be >= 3")
        tb = {"uint16": 2, "uint32": 4}[dtype]
        self.vocab, self.batch, self.seq, self.depth = vocab, batch, seq, depth
        self._l = _rt.TokenLoader(path or "", tb, vocab, batch, seq, rank, world, seed, depth, threads,
                                  shuffle, fixed)
        self._views = [self._l.slot_tensor(s, batch, seq) for s in range(depth)]
        self._held = collections.deque()  # [slot, event or None]
        self._pinned = False
        if pin and torch.cuda.is_available():
            err = torch.cuda.cudart().cudaHostRegister(self._l.arena_ptr, self._l.arena_bytes, 0)
            self._pinned = int(err) == 0
        self._stage = {}

    @property
    def pinned(self) -> bool:
        return self._pinned

    @property
    def num_windows(self) -> int:
        return self._l.num_windows

    def _recycle(self, keep: int) -> None:
        while len(self._held) > keep:
            slot, ev = self._held.popleft()
            if ev is not None:
                ev.synchronize()
            self._l.release(slot)

    def _acquire(self, timeout_ms: int = 600_000) -> int:
        slot = self._l.acquire(timeout_ms)
        if slot < 0:
            raise TimeoutError(f"NativeTokens: no batch within {timeout_ms} ms")
        return slot

    def next(self) -> Tuple[torch.Tensor, torch.Tensor]:
        # copies the caller issued from the previous slot are ordered before this event
        if self._held and self._held[-1][1] is None and torch.cuda.is_available() and self._pinned:
            ev = torch.cuda.Event()
            ev.record()
            self._held[-1][1] = ev
        self._recycle(self.depth - 2)
        slot = self._acquire()
        self._held.append([slot, None])
        v = self._views[slot]
        return v[0], v[1]

    def next_device(self, device) -> Tuple[torch.Tensor, torch.Tensor]:
        device = torch.device(device)
        ring = self._stage.get(device)
        if ring is None:
            ring = self._stage[device] = [[torch.empty(2, self.batch, self.seq, dtype=torch.int64, device=device)
                                           for _ in range(2)], 0]
        self._recycle(self.depth - 2)
        slot = self._acquire()
        buf = ring[0][ring[1]]
        ring[1] ^= 1
        # same stream as the step that reads buf, so reuse two steps later is ordered
        buf.copy_(self._views[slot], non_blocking=self._pinned)
        ev = None
        if device.type == "cuda":
            ev = torch.cuda.Event()
            ev.record()
        self._held.append([slot, ev])
        return buf[0], buf[1]

    def bytes_per_batch(self) -> int:
        return 2 * self.batch * self.seq * 8

    def state(self) -> dict:
        return {"cursor": self._l.cursor()}

    def load_state(self, s: dict) -> None:
        self._recycle(0)
        self._l.seek(int(s.get("cursor", 0)))

    def close(self) -> None:
        if getattr(self, "_l", None) is None:
            return
        if torch.cuda.is_available() and self._held:
            torch.cuda.synchronize()
        self._recycle(0)
        if self._pinned:
            torch.cuda.cudart().cudaHostUnregister(self._l.arena_ptr)
            self._pinned = False
        self._views = []
        self._l = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class SyntheticTokens:
    def __init__(self, vocab: int, batch: int, seq: int, seed: int = 0, rank: int = 0, pin: bool = True,
                 fixed: bool = False):
        self.vocab, self.batch, self.seq = vocab, batch, seq
        self.seed, self.rank = seed, rank
        self.fixed = fixed  # the same batch every call
        self.cursor = 0
        self.pin = pin and torch.cuda.is_available()

    def next(self) -> Tuple[torch.Tensor, torch.Tensor]:
        g = torch.Generator().manual_seed(self.seed * 1_000_003 + self.rank * 7919 + self.cursor)
        x = torch.randint(0, self.vocab, (self.batch, self.seq + 1), generator=g)
        if not self.fixed:
            self.cursor += 1
        if self.pin:
            x = x.pin_memory()
        return x[:, :-1], x[:, 1:]

    def state(self) -> dict:
        return {"cursor": self.cursor}

    def load_state(self, s: dict) -> None:
        self.cursor = int(s.get("cursor", 0))


class MemmapTokens:
    def __init__(self, path: str, batch: int, seq: int, rank: int = 0, world: int = 1, dtype: str = "uint16"):
        self.data = np.memmap(path, dtype=np.dtype(dtype), mode="r")
        self.batch, self.seq, self.rank, self.world = batch, seq, rank, world
        self.cursor = 0
        n = len(self.data) // (seq + 1)
        self.windows = n // world  # windows owned by this rank

    def next(self) -> Tuple[torch.Tensor, torch.Tensor]:
        rows = []
        for _ in range(self.batch):
            w = self.rank + self.world * (self.cursor % max(1, self.windows))
            a = w * (self.seq + 1)
            rows.append(np.asarray(self.data[a:a + self.seq + 1], dtype=np.int64))
            self.cursor += 1
        x = torch.from_numpy(np.stack(rows))
        return x[:, :-1], x[:, 1:]

    def state(self) -> dict:
        return {"cursor": self.cursor}

    def load_state(self, s: dict) -> None:
        self.cursor = int(s.get("cursor", 0))


class CurriculumScheduler:
    """Sequence length grows linearly from `start` to `end` over `steps`,
    rounded down to a multiple of `multiple` (at least `multiple`, at most
    `end`).  The trainer keeps the first seq_len(step) tokens of each batch
    (the targets stay the next tokens), so the loader and its resume cursor
    are unchanged.

    Reference: CurriculumScheduler (include/data/dataloader.hpp:185-200)."""

    def __init__(self, start: int, end: int, steps: int, multiple: int = 128):
        self.start, self.end, self.steps, self.multiple = start, end, steps, multiple

    def seq_len(self, step: int) -> int:
        f = min(1.0, step / max(1, self.steps))
        s = self.start + f * (self.end - self.start)
        return min(self.end, max(self.multiple, int(s) // self.multiple * self.multiple))

    def slice(self, ids, targets, step: int):
        """The first seq_len(step) positions of a batch [B, S] (contiguous)."""
        n = self.seq_len(step)
        if n >= ids.shape[1]:
            return ids, targets
        return ids[:, :n].contiguous(), targets[:, :n].contiguous()
