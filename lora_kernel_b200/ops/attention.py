"""K3/K4: tcgen05 flash attention over the packed QKV activation.

qkv is [B*S, (Hq + 2*Hkv) * Dh] (query heads, then key heads, then value
heads); o is [B*S, Hq*Dh]; lse is [B, Hq, S] (natural log).  Causal, full and
sliding-window masks; GQA (Hq a multiple of Hkv); head_dim 64 or 128.
"""
from __future__ import annotations

import math
from typing import Optional

import torch

from .._ext import C, require_device, status

_scratch = {}


def _buf(key, numel, device):
    t = _scratch.get((key, device))
    if t is None or t.numel() < numel:
        t = torch.empty(numel, dtype=torch.float32, device=device)
        _scratch[(key, device)] = t
    return t[:numel]


def attention_fwd(qkv: torch.Tensor, B: int, S: int, Hq: int, Hkv: int, Dh: int, *,
                  causal: bool = True, window: int = 0, scale: Optional[float] = None,
                  out: Optional[torch.Tensor] = None, lse: Optional[torch.Tensor] = None,
                  kv: Optional[torch.Tensor] = None, q_off: int = 0):
    """Self-attention over packed qkv, or (kv given) queries qkv [B*S, Hq*Dh] at
    positions q_off.. against keys/values kv [B*Skv, 2*Hkv*Dh] at positions 0.."""
    require_device(qkv)
    scale = 1.0 / math.sqrt(Dh) if scale is None else scale
    if out is None:
        out = torch.empty(B * S, Hq * Dh, dtype=torch.bfloat16, device=qkv.device)
    if lse is None:
        lse = torch.empty(B, Hq, S, dtype=torch.float32, device=qkv.device)
    C().attention_fwd(qkv, out, lse, B, S, Hq, Hkv, Dh, bool(causal), int(window), float(scale),
                      status(qkv.device), kv, int(q_off))
    return out, lse


def attention_bwd(qkv: torch.Tensor, o: torch.Tensor, dout: torch.Tensor, lse: torch.Tensor,
                  B: int, S: int, Hq: int, Hkv: int, Dh: int, *, causal: bool = True,
                  window: int = 0, scale: Optional[float] = None,
                  dqkv: Optional[torch.Tensor] = None) -> torch.Tensor:
    require_device(qkv)
    scale = 1.0 / math.sqrt(Dh) if scale is None else scale
    if dqkv is None:
        dqkv = torch.empty(B * S, (Hq + 2 * Hkv) * Dh, dtype=torch.bfloat16, device=qkv.device)
    dq_acc = _buf("dq", B * S * Hq * Dh, qkv.device)
    dvec = _buf("dvec", 2 * ((B * Hq * S + 63) // 64 * 64), qkv.device)
    C().attention_bwd(qkv, o, dout, lse, dqkv, dq_acc, dvec, B, S, Hq, Hkv, Dh, bool(causal),
                      int(window), float(scale), status(qkv.device))
    return dqkv


def reference_attention(qkv: torch.Tensor, B: int, S: int, Hq: int, Hkv: int, Dh: int, *,
                        causal: bool = True, window: int = 0, scale: Optional[float] = None):
    """fp32 eager restatement (any device): returns (o [B*S, Hq*Dh], lse [B, Hq, S])."""
    scale = 1.0 / math.sqrt(Dh) if scale is None else scale
    x = qkv.float().reshape(B, S, Hq + 2 * Hkv, Dh)
    q = x[:, :, :Hq].permute(0, 2, 1, 3)
    k = x[:, :, Hq:Hq + Hkv].permute(0, 2, 1, 3).repeat_interleave(Hq // Hkv, dim=1)
    v = x[:, :, Hq + Hkv:].permute(0, 2, 1, 3).repeat_interleave(Hq // Hkv, dim=1)
    s = (q @ k.transpose(-1, -2)) * scale
    qi = torch.arange(S, device=qkv.device)[:, None]
    ki = torch.arange(S, device=qkv.device)[None, :]
    mask = torch.zeros(S, S, dtype=torch.bool, device=qkv.device)
    if causal:
        mask |= ki > qi
    if window > 0:
        mask |= ki <= qi - window
    s = s.masked_fill(mask, float("-inf"))
    lse = torch.logsumexp(s, -1)
    p = torch.softmax(s, -1)
    o = (p @ v).permute(0, 2, 1, 3).reshape(B * S, Hq * Dh)
    return o, lse
