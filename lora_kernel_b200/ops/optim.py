"""K11 fused AdamW, gradient-norm partials and the device-side step finaliser
(global-norm clip, overflow skip, dynamic loss scale, bias-correction step)."""
from __future__ import annotations

from typing import Optional

import torch

from .._ext import C, require_device

# indices of the fp32 optimizer state vector (csrc/lk_api.h LkOptState)
ST_LOSS_SCALE, ST_GROWTH, ST_STEP, ST_GRAD_MULT, ST_SKIP, ST_LR = 0, 1, 2, 3, 4, 5
ST_GRAD_NORM, ST_NUM_SKIPPED, ST_CONSEC_SKIPS, ST_CLIP_COEF, ST_SIZE = 6, 7, 8, 9, 16


def new_state(device, loss_scale: float = 1.0, lr: float = 0.0) -> torch.Tensor:
    s = torch.zeros(ST_SIZE, dtype=torch.float32, device=device)
    s[ST_LOSS_SCALE] = loss_scale
    s[ST_LR] = lr
    s[ST_GRAD_MULT] = 1.0 / loss_scale
    s[ST_CLIP_COEF] = 1.0
    return s


def make_chunks(segments, chunk: int = 16384, device=None) -> torch.Tensor:
    """segments: iterable of (start, length, weight_decay_on[, flat_delta]) ->
    int32 [n, 4].  flat_delta (a multiple of 64) maps a master element to its
    position in the full flat layout for the fused parameter all-gather."""
    rows = []
    for seg in segments:
        start, length, wd = seg[:3]
        delta = seg[3] if len(seg) > 3 else 0
        assert delta % 64 == 0
        for off in range(0, length, chunk):
            rows.append((start + off, min(chunk, length - off), 1 if wd else 0, delta // 64))
    t = torch.tensor(rows if rows else [(0, 0, 0, 0)], dtype=torch.int32)
    if not rows:
        t = t[:0]
    return t.to(device) if device is not None else t


def grad_norm_partials(grad: torch.Tensor, partial: torch.Tensor) -> None:
    require_device(grad)
    C().grad_norm_partials(grad, partial)


def finalize(partial: torch.Tensor, state: torch.Tensor, max_norm: float, dynamic: bool,
             growth: float = 2.0, backoff: float = 0.5, growth_interval: int = 2000,
             min_scale: float = 1.0) -> None:
    C().optimizer_finalize(partial, state, float(max_norm), bool(dynamic), float(growth),
                           float(backoff), int(growth_interval), float(min_scale))


def adamw_(p32: torch.Tensor, grad: torch.Tensor, m: torch.Tensor, v: torch.Tensor,
           chunks: torch.Tensor, state: torch.Tensor, *, p16: Optional[torch.Tensor] = None,
           ema: Optional[torch.Tensor] = None, beta1: float = 0.9, beta2: float = 0.95,
           eps: float = 1e-8, wd: float = 0.0, ema_decay: float = 0.0,
           zero_grad: bool = True, p16_peers: Optional[torch.Tensor] = None) -> None:
    """p16_peers: device int64 array of every rank's full bf16 parameter buffer;
    the updated values are stored into all of them (fused all-gather)."""
    require_device(p32)
    C().adamw(p32, grad, m, v, p16, ema, chunks, state, float(beta1), float(beta2), float(eps),
              float(wd), float(ema_decay), bool(zero_grad), p16_peers)
