"""Token data sources.

SyntheticTokens: uniform random ids in [0, vocab) from a seeded generator per
rank (the benchmarks' data), with next-token targets.  MemmapTokens: a flat
uint16 / uint32 token file read through numpy.memmap, sharded across data-
parallel ranks by contiguous windows.  CurriculumScheduler: sequence-length
warm-up.  Each source keeps a cursor so a checkpoint can resume the stream.

Reference: DataLoader (include/data/dataloader.hpp:63-159, which returns
random tokens regardless of the file), StreamDataset and CurriculumScheduler
(:162-200), ShardedDataset / DistributedDataLoader (include/data/datasets.hpp).
"""
from __future__ import annotations

from typing import Tuple

import numpy as np
import torch


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
    rounded to a multiple of `multiple`."""

    def __init__(self, start: int, end: int, steps: int, multiple: int = 128):
        self.start, self.end, self.steps, self.multiple = start, end, steps, multiple

    def seq_len(self, step: int) -> int:
        f = min(1.0, step / max(1, self.steps))
        s = self.start + f * (self.end - self.start)
        return max(self.multiple, int(s) // self.multiple * self.multiple)
