"""Optimizer-state offload: fp32 master weights and both AdamW moments live in
page-locked host memory (12 bytes per parameter off the GPU) and stream
through the GPU in chunks for the fused AdamW kernel (K11).

Per step, after the device-side finaliser has decided clip / skip / loss
scale from the gradients (which stay on the GPU):
    copy stream    H2D  p32, m, v of chunk c+1        (double-buffered staging)
    compute stream AdamW on chunk c; the updated bf16 weights go straight
                   into the device parameter buffer
    copy stream    D2H  p32, m, v of chunk c back to the host
Events order the three so a staging buffer is refilled only after its
chunk's results have left the GPU.  The host arrays are never read by the CPU
during a step, so the next step can start as soon as the last D2H is queued.

Reference: UnifiedMemoryManager (include/core/unified_memory.hpp:19-165:
cudaMallocManaged + cudaMemAdvise/prefetch, never compiled).
"""
from __future__ import annotations

from typing import List, Optional, Tuple

import torch

from ..ops import optim as O
from .optimizer import DynamicLossScaler


class OffloadedAdamW:
    """Same interface as FusedAdamW (norm_partials / finalize / apply / step,
    state, scaler); `p32`, `m`, `v` are pinned host tensors."""

    def __init__(self, master_host: torch.Tensor, segments, device, *, lr: float = 3e-4, betas=(0.9, 0.95),
                 eps: float = 1e-8, weight_decay: float = 0.1, max_grad_norm: float = 1.0,
                 dynamic_loss_scale: bool = False, init_loss_scale: float = 65536.0,
                 growth_interval: int = 2000, chunk_elems: int = 64 << 20):
        dev = torch.device(device)
        self.device = dev
        n = master_host.numel()
        pin = torch.cuda.is_available()
        self.p32 = torch.empty(n, dtype=torch.float32, pin_memory=pin)
        self.p32.copy_(master_host.float())
        self.m = torch.zeros(n, dtype=torch.float32, pin_memory=pin)
        self.v = torch.zeros(n, dtype=torch.float32, pin_memory=pin)
        self.ema = None
        self.ema_decay = 0.0
        self.lr, self.betas, self.eps, self.wd = lr, betas, eps, weight_decay
        self.max_grad_norm = max_grad_norm
        self.state = O.new_state(dev, loss_scale=1.0, lr=lr)
        self.scaler = DynamicLossScaler(self.state, dynamic_loss_scale, init_loss_scale, growth_interval)
        nparts = max(1, min(1024, (n + 65535) // 65536))
        self.partial = torch.zeros(nparts, dtype=torch.float32, device=dev)
        # chunk boundaries on 64-element multiples; a chunk table per chunk,
        # positions relative to the chunk start
        c = max(64, chunk_elems // 64 * 64)
        self.ranges: List[Tuple[int, int]] = [(a, min(n, a + c)) for a in range(0, n, c)]
        segs = list(segments)
        self.tables = []
        for a, b in self.ranges:
            rel = []
            for s, ln, wd in segs:
                x, y = max(s, a), min(s + ln, b)
                if x < y:
                    rel.append((x - a, y - x, wd))
            self.tables.append(O.make_chunks(rel, device=dev))
        big = max((b - a) for a, b in self.ranges) if self.ranges else 0
        self.stage = [[torch.empty(big, dtype=torch.float32, device=dev) for _ in range(3)] for _ in range(2)]
        self.copy_stream = torch.cuda.Stream(dev) if dev.type == "cuda" else None

    def set_lr(self, lr: float) -> None:
        self.lr = lr
        self.state[O.ST_LR].fill_(lr)

    def norm_partials(self, grad: torch.Tensor) -> torch.Tensor:
        O.grad_norm_partials(grad, self.partial)
        return self.partial

    def finalize(self, partial: Optional[torch.Tensor] = None) -> None:
        s = self.scaler
        O.finalize(self.partial if partial is None else partial, self.state, self.max_grad_norm,
                   s.enabled, s.growth, s.backoff, s.growth_interval, s.min_scale)

    def apply(self, grad: torch.Tensor, p16: Optional[torch.Tensor], zero_grad: bool = True,
              p16_peers: Optional[torch.Tensor] = None) -> None:
        if p16_peers is not None:
            raise NotImplementedError("offloaded optimizer with the fused parameter all-gather")
        comp = torch.cuda.current_stream(self.device)
        cs = self.copy_stream
        host = (self.p32, self.m, self.v)
        loaded = [None, None]   # event: staging k holds chunk data (H2D done)
        drained = [None, None]  # event: staging k's results have been copied out

        def load(ci):
            k = ci % 2
            a, b = self.ranges[ci]
            with torch.cuda.stream(cs):
                if drained[k] is not None:
                    cs.wait_event(drained[k])
                for st, h in zip(self.stage[k], host):
                    st[:b - a].copy_(h[a:b], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(cs)
                loaded[k] = ev

        cs.wait_stream(comp)  # gradients and the finaliser's decisions are ready
        if self.ranges:
            load(0)
        for ci, (a, b) in enumerate(self.ranges):
            k = ci % 2
            if ci + 1 < len(self.ranges):
                load(ci + 1)
            comp.wait_event(loaded[k])
            p, m, v = (t[:b - a] for t in self.stage[k])
            O.adamw_(p, grad[a:b], m, v, self.tables[ci], self.state,
                     p16=None if p16 is None else p16[a:b], beta1=self.betas[0], beta2=self.betas[1],
                     eps=self.eps, wd=self.wd, zero_grad=zero_grad)
            done = torch.cuda.Event()
            done.record(comp)
            with torch.cuda.stream(cs):
                cs.wait_event(done)
                for st, h in zip(self.stage[k], host):
                    h[a:b].copy_(st[:b - a], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(cs)
                drained[k] = ev
        comp.wait_stream(cs)  # the host state is complete before anything reads it

    def step(self, grad: torch.Tensor, p16: Optional[torch.Tensor]) -> None:
        self.norm_partials(grad)
        self.finalize()
        self.apply(grad, p16)

    def grad_norm(self) -> float:
        return float(self.state[O.ST_GRAD_NORM])

    def step_count(self) -> int:
        return int(self.state[O.ST_STEP])

    def state_dict(self):
        return {"p32": self.p32, "m": self.m, "v": self.v, "state": self.state}

    def load_state_dict(self, sd) -> None:
        with torch.no_grad():
            self.p32.copy_(sd["p32"])
            self.m.copy_(sd["m"])
            self.v.copy_(sd["v"])
            self.state.copy_(sd["state"])
