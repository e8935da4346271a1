"""Process groups, symmetric (peer-mapped) buffers and device-side signalling.

One process per GPU.  `torch.distributed` (NCCL) bootstraps the group and
carries the baseline path; the fused kernels of this package load and store
peer memory directly:

  * `SymBuffer`: a buffer allocated from symmetric memory (CUDA VMM, mapped
    into every peer) with a device table of the `world` peer base pointers;
  * `PeerComm`: flag slots for bounded-wait device barriers (epoch counters),
    the norm-exchange scratch and launch helpers for the collectives in
    csrc/comm.cu.

A kernel that waits for a peer gives up after a bounded time and records
LK_ERR_TIMEOUT_PEER in the status word (see _ext.check_status), so a missing
or dead rank surfaces as a Python error instead of a hung GPU.
"""
from __future__ import annotations

import datetime
import os
from typing import Dict, List, Optional

import torch
import torch.distributed as dist

from .._ext import C, status

# flag slots (csrc/lk_api.h LK_SIG_SLOTS = 16)
SLOT_STEP = 0       # step start: every rank finished its optimizer update
SLOT_GRAD = 1       # a layer's gradients are complete on every rank
SLOT_NORM = 2       # gradient-norm exchange
SLOT_AR_IN = 3      # all-reduce inputs ready
SLOT_AR_OUT = 4     # all-reduce outputs written
SLOT_GRAD_DONE = 5  # every rank has read a gradient slot (it may be overwritten)
SLOT_USER = 8


def init_distributed(backend: str = "nccl", timeout_s: int = 300) -> tuple:
    """Initialise the default process group from torchrun's environment.
    Returns (rank, world, local_rank)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if backend == "nccl":
        torch.cuda.set_device(local)
        if os.environ.get("LK_PIN_NUMA") == "1":  # CPU affinity = the GPU's NUMA node
            from ..utils.env import pin_to_gpu_numa
            pin_to_gpu_numa(local)
    if world > 1 and not dist.is_initialized():
        kw = dict(timeout=datetime.timedelta(seconds=timeout_s))
        if backend == "nccl":
            kw["device_id"] = torch.device("cuda", local)
        dist.init_process_group(backend, **kw)
    return rank, world, local


def _symm():
    import torch.distributed._symmetric_memory as symm_mem
    return symm_mem


class SymBuffer:
    """Symmetric buffer of `numel` elements plus its peer-pointer table."""

    def __init__(self, numel: int, dtype: torch.dtype, device, group=None):
        self.group = group or dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        sm = _symm()
        self.local = sm.empty(numel, dtype=dtype, device=device)
        self.local.zero_()
        self.handle = sm.rendezvous(self.local, self.group.group_name)
        ptrs = [int(p) for p in self.handle.buffer_ptrs]
        self.ptrs_host = ptrs
        self.ptrs = torch.tensor(ptrs, dtype=torch.int64, device=device)
        self.dtype = dtype
        self.numel = numel
        # NVLS multicast address of the buffer (0 when the switch/driver offers none)
        try:
            self.mc_ptr = int(self.handle.multicast_ptr) if self.world > 1 else 0
        except Exception:  # noqa: BLE001 - older builds expose no multicast
            self.mc_ptr = 0
        self._offset_tables: Dict[int, torch.Tensor] = {}

    def ptrs_at(self, off_elems: int) -> torch.Tensor:
        """Device table of every rank's address of element `off_elems`."""
        t = self._offset_tables.get(off_elems)
        if t is None:
            es = self.element_size()
            t = torch.tensor([p + es * off_elems for p in self.ptrs_host], dtype=torch.int64,
                             device=self.ptrs.device)
            self._offset_tables[off_elems] = t
        return t

    def element_size(self) -> int:
        return torch.empty((), dtype=self.dtype).element_size()


class PeerComm:
    """Device-side barrier / exchange helpers for one process group."""

    def __init__(self, device, group=None):
        self.device = torch.device(device)
        self.group = group or dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        nslots = C().SIG_SLOTS
        self.sig = SymBuffer(nslots * self.world, torch.int32, self.device, self.group)
        self.nbuf = SymBuffer(max(2, self.world) * 2, torch.float64, self.device, self.group)
        self.epochs: Dict[int, int] = {}
        # in-switch reductions (multimem) when NVLS is available and the group has 4+
        # ranks (at 2 the one-shot P2P kernels measured faster: 512 MB all-reduce
        # 0.84 vs 1.38 ms); LK_NVLS=1 / 0 forces the choice
        want = os.environ.get("LK_NVLS", "auto")
        self.nvls = self.sig.mc_ptr != 0 and (want == "1" or (want == "auto" and self.world >= 4))
        torch.cuda.synchronize(self.device)
        dist.barrier(self.group)

    def next_epoch(self, slot: int) -> int:
        e = self.epochs.get(slot, 0) + 1
        self.epochs[slot] = e
        return e

    def barrier_dev(self, slot: int) -> None:
        """Device barrier whose epoch lives on the device (replayable inside a
        CUDA graph).  A slot is used either with this or with barrier(), never both."""
        if not hasattr(self, "_dev_epochs"):
            self._dev_epochs = torch.zeros(C().SIG_SLOTS, dtype=torch.int32, device=self.device)
        C().signal_barrier_dev(self.sig.ptrs, self.rank, self.world, slot, self._dev_epochs[slot:slot + 1],
                               status(self.device))

    def barrier(self, slot: int) -> None:
        """Device barrier on the current stream (bounded wait per peer)."""
        C().signal_barrier(self.sig.ptrs, self.rank, self.world, slot, self.next_epoch(slot),
                           status(self.device))

    def allgather_copy(self, src: SymBuffer, src_off_elems: int, chunk_elems: int,
                       dst: torch.Tensor) -> None:
        es = src.element_size()
        C().allgather_copy(src.ptrs, src_off_elems * es, chunk_elems * es, dst, self.world)

    def reduce_scatter_sum(self, src: SymBuffer, src_off: int, n: int, dst: torch.Tensor,
                           accumulate: bool = False, partial: Optional[torch.Tensor] = None) -> None:
        """dst[:n] (+)= sum over ranks of src[src_off:src_off+n] (fp32).  The
        caller has made every rank's src ready (device barrier)."""
        if self.nvls and src.mc_ptr:
            C().reduce_scatter_sum_nvls(src.mc_ptr + 4 * src_off, n, dst, accumulate, partial)
        else:
            C().reduce_scatter_sum(src.ptrs, src_off, n, dst, self.world, accumulate, partial)

    def reduce_scatter_bf16(self, src: SymBuffer, src_off: int, n: int, dst: torch.Tensor,
                            accumulate: bool = False, partial: Optional[torch.Tensor] = None) -> None:
        """dst[:n] (fp32) (+)= sum over ranks of src[src_off:src_off+n] (bf16
        on the wire, fp32 sum).  The caller has made every rank's src ready."""
        if self.nvls and src.mc_ptr:
            C().reduce_scatter_bf16_nvls(src.mc_ptr + 2 * src_off, n, dst, accumulate, partial)
        else:
            C().reduce_scatter_bf16(src.ptrs, src_off, n, dst, self.world, accumulate, partial)

    def allreduce_sum_(self, buf: SymBuffer, n: int, partial: Optional[torch.Tensor] = None,
                       off: int = 0) -> None:
        """In-place sum over ranks of buf[off:off+n] (fp32), bracketed by barriers."""
        self.barrier(SLOT_AR_IN)
        if self.nvls and buf.mc_ptr:
            C().allreduce_sum_nvls(buf.mc_ptr + 4 * off, n, self.rank, self.world, partial, buf.local)
        else:
            C().allreduce_sum(buf.ptrs_at(off), n, self.rank, self.world, partial)
        self.barrier(SLOT_AR_OUT)

    def norm_exchange(self, partial: torch.Tensor, state: torch.Tensor, max_norm: float,
                      dynamic: bool, growth: float = 2.0, backoff: float = 0.5,
                      growth_interval: int = 2000, min_scale: float = 1.0) -> None:
        C().norm_exchange(partial, self.nbuf.ptrs, self.sig.ptrs, self.rank, self.world, SLOT_NORM,
                          self.next_epoch(SLOT_NORM), state, float(max_norm), bool(dynamic),
                          float(growth), float(backoff), int(growth_interval), float(min_scale),
                          status(self.device))
