"""Paged KV-cache block bookkeeping with block-granular prefix caching.

Physical blocks hold `block_size` tokens of K and V for every layer.  Each
sequence owns a block table (logical block -> physical block).  A full prompt
block is identified by a hash chain over the token ids of all blocks up to and
including it, so two prompts with the same first k blocks share k physical
blocks (reference counted); a shared block is never written again (only full
blocks are shared, a sequence's partial tail block is always private), so no
copy-on-write is needed.  Unreferenced cached blocks stay reusable until the
allocator needs them back (least recently used first).

Reference: PagedKVCache (include/nn/kv_cache.hpp:103-219: one global page
table, no sharing) and PrefixCache (include/api/serving_production.hpp:136-169:
exact-string match over a vector, O(n)).
"""
from __future__ import annotations

from collections import OrderedDict, deque
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple


def block_hashes(tokens: Sequence[int], block_size: int, parent: int = 0) -> List[int]:
    """Chained hashes of every full block of `tokens`."""
    out = []
    h = parent
    for i in range(len(tokens) // block_size):
        h = hash((h, tuple(tokens[i * block_size:(i + 1) * block_size])))
        out.append(h)
    return out


@dataclass
class CacheStats:
    queries: int = 0       # prompt blocks looked up
    hits: int = 0          # prompt blocks found in the cache
    evictions: int = 0

    @property
    def hit_rate(self) -> float:
        return self.hits / self.queries if self.queries else 0.0


class BlockManager:
    def __init__(self, num_blocks: int, block_size: int, enable_prefix_caching: bool = True):
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.prefix = enable_prefix_caching
        self.free: deque = deque(range(num_blocks))
        self.ref = [0] * num_blocks
        self.hash_of: Dict[int, int] = {}          # block -> hash (cached full blocks)
        self.block_of: Dict[int, int] = {}         # hash -> block
        self.evictable: "OrderedDict[int, None]" = OrderedDict()  # cached blocks with ref 0 (LRU)
        self.stats = CacheStats()

    # ------------------------------------------------------------ capacity
    def num_free(self) -> int:
        return len(self.free) + len(self.evictable)

    def usage(self) -> float:
        return 1.0 - self.num_free() / self.num_blocks

    def _take(self) -> int:
        if self.free:
            b = self.free.popleft()
        elif self.evictable:
            b, _ = self.evictable.popitem(last=False)
            h = self.hash_of.pop(b)
            self.block_of.pop(h, None)
            self.stats.evictions += 1
        else:
            raise MemoryError("out of KV-cache blocks")
        self.ref[b] = 1
        return b

    def _release(self, b: int) -> None:
        self.ref[b] -= 1
        if self.ref[b] == 0:
            if b in self.hash_of:
                self.evictable[b] = None
            else:
                self.free.append(b)

    # ----------------------------------------------------------- sequences
    def blocks_needed(self, tokens: Sequence[int]) -> int:
        return (len(tokens) + self.block_size - 1) // self.block_size

    def allocate(self, tokens: Sequence[int]) -> Tuple[List[int], int]:
        """Block table for a new prompt and the number of leading tokens whose
        K/V are already cached (a multiple of block_size, < len(tokens))."""
        n_blocks = self.blocks_needed(tokens)
        table: List[int] = []
        cached = 0
        if self.prefix:
            hashes = block_hashes(tokens, self.block_size)
            # keep at least one token to compute: never reuse the block holding the last token
            usable = min(len(hashes), (len(tokens) - 1) // self.block_size)
            for h in hashes[:usable]:
                b = self.block_of.get(h)
                if b is None:
                    break
                if self.ref[b] == 0:
                    self.evictable.pop(b, None)
                self.ref[b] += 1
                table.append(b)
            self.stats.queries += usable
            self.stats.hits += len(table)
            cached = len(table) * self.block_size
        need = n_blocks - len(table)
        if need > self.num_free():
            for b in table:
                self._release(b)
            raise MemoryError("out of KV-cache blocks")
        for _ in range(need):
            table.append(self._take())
        return table, cached

    def register_full_blocks(self, tokens: Sequence[int], table: List[int], upto: int) -> None:
        """Publish the full blocks covering tokens[:upto] for prefix reuse."""
        if not self.prefix:
            return
        for i, h in enumerate(block_hashes(tokens[:upto], self.block_size)):
            b = table[i]
            if b in self.hash_of or h in self.block_of:
                continue
            self.hash_of[b] = h
            self.block_of[h] = b

    def append_slot(self, table: List[int], num_tokens: int) -> int:
        """Slot for token index `num_tokens` (0-based) of a sequence, growing the
        table by one block when the previous one is full."""
        bi, off = divmod(num_tokens, self.block_size)
        if bi == len(table):
            table.append(self._take())
        return table[bi] * self.block_size + off

    def free_seq(self, table: List[int]) -> None:
        for b in table:
            self._release(b)
        table.clear()

    def slots_for(self, table: List[int], start: int, end: int) -> List[int]:
        bs = self.block_size
        return [table[t // bs] * bs + t % bs for t in range(start, end)]
