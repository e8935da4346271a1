"""Gradient compression and hierarchical all-reduce for links slower than
NVSwitch (multi-node data parallelism, PCIe-only hosts).  Inside one NVSwitch
domain the fused peer-memory reductions (K10/K12) are faster than any
compressed exchange, so these are opt-in utilities, not the default path.

TopKCompressor   keeps the k = ratio * n largest-magnitude entries of a flat
                 gradient, int64 indices (the full index range), with error
                 feedback: what was not sent is added to the next step's
                 gradient, so the sum of all sent values tracks the sum of
                 all gradients.
compressed_all_reduce
                 every rank sends its (indices, values); each rank scatter-adds
                 all of them and divides by the world size.  Exact when
                 ratio = 1.
HierarchicalAllReduce
                 two-level all-reduce over `local_size` ranks per node:
                 reduce-scatter inside the node, all-reduce of each shard
                 across nodes (one rank per node per shard), all-gather inside
                 the node.  Inter-node traffic is 1/local_size of a flat ring.

Reference: GradientCompression (include/distributed/distributed_training.hpp:
17-47, top-k with int8 indices that wrap modulo 256) and HierarchicalAllReduce
(:267-287, communicators never initialised).
"""
from __future__ import annotations

from typing import List, Optional, Tuple

import torch
import torch.distributed as dist


class TopKCompressor:
    def __init__(self, ratio: float, error_feedback: bool = True):
        if not 0.0 < ratio <= 1.0:
            raise ValueError("ratio must be in (0, 1]")
        self.ratio = ratio
        self.error_feedback = error_feedback
        self.residual: Optional[torch.Tensor] = None

    def k_for(self, n: int) -> int:
        return max(1, min(n, int(round(self.ratio * n))))

    def compress(self, grad: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        g = grad.reshape(-1).float()
        if self.error_feedback:
            if self.residual is None or self.residual.numel() != g.numel():
                self.residual = torch.zeros_like(g)
            g = g + self.residual
        k = self.k_for(g.numel())
        idx = torch.topk(g.abs(), k, sorted=False).indices.to(torch.int64)
        vals = g.index_select(0, idx)
        if self.error_feedback:
            self.residual = g.index_fill(0, idx, 0.0)
        return idx, vals

    @staticmethod
    def decompress(idx: torch.Tensor, vals: torch.Tensor, n: int, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        out = torch.zeros(n, dtype=vals.dtype, device=vals.device) if out is None else out.zero_()
        out.index_add_(0, idx, vals)
        return out


def compressed_all_reduce(grad: torch.Tensor, comp: TopKCompressor, group=None, average: bool = True) -> torch.Tensor:
    """Mean (or sum) over ranks of the compressed gradients, written into grad."""
    world = dist.get_world_size(group)
    idx, vals = comp.compress(grad)
    k = idx.numel()
    all_idx = torch.empty(world * k, dtype=idx.dtype, device=idx.device)
    all_val = torch.empty(world * k, dtype=vals.dtype, device=vals.device)
    dist.all_gather_into_tensor(all_idx, idx, group=group)
    dist.all_gather_into_tensor(all_val, vals, group=group)
    dense = TopKCompressor.decompress(all_idx, all_val, grad.numel())
    if average:
        dense /= world
    grad.copy_(dense.view_as(grad).to(grad.dtype))
    return grad


class HierarchicalAllReduce:
    """Sum all-reduce over node-local then cross-node groups.  Ranks
    [n * local_size, (n + 1) * local_size) form node n.  Every rank must
    construct this object (group creation is collective)."""

    def __init__(self, local_size: int):
        world = dist.get_world_size()
        if local_size < 1 or world % local_size:
            raise ValueError(f"world {world} is not a multiple of local_size {local_size}")
        self.local_size = local_size
        self.nodes = world // local_size
        rank = dist.get_rank()
        self.node, self.local = divmod(rank, local_size)
        self.intra = None
        self.inter = None
        for n in range(self.nodes):
            g = dist.new_group(list(range(n * local_size, (n + 1) * local_size)))
            if n == self.node:
                self.intra = g
        for l in range(local_size):
            g = dist.new_group([n * local_size + l for n in range(self.nodes)])
            if l == self.local:
                self.inter = g

    def __call__(self, t: torch.Tensor) -> torch.Tensor:
        flat = t.reshape(-1)
        n = flat.numel()
        L = self.local_size
        pad = (-n) % L
        buf = torch.cat([flat, flat.new_zeros(pad)]) if pad else flat.clone()
        shard = buf.new_empty(buf.numel() // L)
        dist.reduce_scatter_tensor(shard, buf, group=self.intra)
        if self.nodes > 1:
            dist.all_reduce(shard, group=self.inter)
        dist.all_gather_into_tensor(buf, shard, group=self.intra)
        t.copy_(buf[:n].view_as(t))
        return t
