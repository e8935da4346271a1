"""Device-resident AdamW over flat fp32 master weights (K11) with the step
finaliser: global-norm clipping, overflow skip and dynamic loss scaling, all
decided on the device (no host synchronisation per step).

`FusedAdamW` works on any contiguous range [lo, hi) of the flat parameter
layout, which is how ZeRO ranks own their shard; the single-GPU case is the
whole range.
"""
from __future__ import annotations

from typing import Optional

import torch

from ..ops import optim as O


class DynamicLossScaler:
    """Host view of the device-resident loss scaler (reference
    include/nn/loss_scaling.hpp:8-53: init 65536, x2 after `growth_interval`
    clean steps, /2 on overflow, floor 1)."""

    def __init__(self, state: torch.Tensor, enabled: bool, init_scale: float = 65536.0,
                 growth_interval: int = 2000, growth: float = 2.0, backoff: float = 0.5,
                 min_scale: float = 1.0):
        self.state = state
        self.enabled = enabled
        self.growth_interval = growth_interval
        self.growth = growth
        self.backoff = backoff
        self.min_scale = min_scale
        state[O.ST_LOSS_SCALE] = init_scale if enabled else 1.0

    def get_scale(self) -> float:
        return float(self.state[O.ST_LOSS_SCALE])

    def scale_tensor(self) -> torch.Tensor:
        return self.state[O.ST_LOSS_SCALE:O.ST_LOSS_SCALE + 1]

    def num_skipped(self) -> int:
        return int(self.state[O.ST_NUM_SKIPPED])

    def consecutive_skips(self) -> int:
        return int(self.state[O.ST_CONSEC_SKIPS])


class FusedAdamW:
    def __init__(self, master: torch.Tensor, segments, *, lr: float = 3e-4, betas=(0.9, 0.95),
                 eps: float = 1e-8, weight_decay: float = 0.1, max_grad_norm: float = 1.0,
                 dynamic_loss_scale: bool = False, init_loss_scale: float = 65536.0,
                 growth_interval: int = 2000, ema_decay: float = 0.0):
        """master: fp32 flat tensor (the owned range); segments: (start, len,
        decay) relative to master."""
        dev = master.device
        self.p32 = master
        self.m = torch.zeros_like(master)
        self.v = torch.zeros_like(master)
        self.ema = master.clone() if ema_decay > 0 else None
        self.ema_decay = ema_decay
        self.lr = lr
        self.betas = betas
        self.eps = eps
        self.wd = weight_decay
        self.max_grad_norm = max_grad_norm
        self.chunks = O.make_chunks(segments, device=dev)
        self.state = O.new_state(dev, loss_scale=1.0, lr=lr)
        self.scaler = DynamicLossScaler(self.state, dynamic_loss_scale, init_loss_scale, growth_interval)
        nparts = max(1, min(1024, (master.numel() + 65535) // 65536))
        self.partial = torch.zeros(nparts, dtype=torch.float32, device=dev)

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
        O.adamw_(self.p32, grad, self.m, self.v, self.chunks, self.state, p16=p16, ema=self.ema,
                 beta1=self.betas[0], beta2=self.betas[1], eps=self.eps, wd=self.wd,
                 ema_decay=self.ema_decay, zero_grad=zero_grad, p16_peers=p16_peers)

    def step(self, grad: torch.Tensor, p16: Optional[torch.Tensor]) -> None:
        """grad-norm partials -> finalize (clip/skip/scale) -> AdamW (+EMA),
        zeroing the gradient."""
        self.norm_partials(grad)
        self.finalize()
        self.apply(grad, p16)

    # --------------------------------------------------------------- stats
    def grad_norm(self) -> float:
        return float(self.state[O.ST_GRAD_NORM])

    def step_count(self) -> int:
        return int(self.state[O.ST_STEP])

    def state_dict(self):
        return {"p32": self.p32, "m": self.m, "v": self.v, "state": self.state,
                **({"ema": self.ema} if self.ema is not None else {})}

    def load_state_dict(self, sd) -> None:
        with torch.no_grad():
            self.p32.copy_(sd["p32"])
            self.m.copy_(sd["m"])
            self.v.copy_(sd["v"])
            self.state.copy_(sd["state"])
            if self.ema is not None and "ema" in sd:
                self.ema.copy_(sd["ema"])


class SWA:
    """Stochastic weight averaging from `start_step` (reference
    include/nn/training_enhancements.hpp:101-119): running mean of the fp32
    master weights, updated every `every` optimizer steps."""

    def __init__(self, master: torch.Tensor, start_step: int, every: int = 1):
        self.avg = torch.zeros_like(master)
        self.n = 0
        self.start = start_step
        self.every = every

    def update(self, master: torch.Tensor, step: int) -> None:
        if step < self.start or (step - self.start) % self.every:
            return
        self.n += 1
        self.avg.add_(master - self.avg, alpha=1.0 / self.n)
