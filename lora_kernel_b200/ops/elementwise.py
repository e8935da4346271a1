"""K6 RoPE, K7 SwiGLU and K8 embedding wrappers."""
from __future__ import annotations

import math
from typing import Optional

import torch

from .._ext import C, require_device, status

_tables = {}


def rope_table(max_pos: int, head_dim: int, base: float, device) -> torch.Tensor:
    """float32 [max_pos, head_dim/2, 2] of (cos, sin) computed in float64.
    theta_i = pos * base^(-2i/head_dim) for the interleaved pair (2i, 2i+1)."""
    key = (max_pos, head_dim, float(base), str(device))
    t = _tables.get(key)
    if t is None:
        inv = base ** (-torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim)
        ang = torch.arange(max_pos, dtype=torch.float64)[:, None] * inv[None, :]
        t = torch.stack([torch.cos(ang), torch.sin(ang)], dim=-1).to(torch.float32).contiguous()
        t = t.to(device)
        _tables[key] = t
    return t


def rope_(x: torch.Tensor, col0: int, nheads: int, head_dim: int, table: torch.Tensor, *,
          seq_len: int = 1 << 30, pos_offset: int = 0, positions: Optional[torch.Tensor] = None,
          inverse: bool = False) -> torch.Tensor:
    """Rotate `nheads` heads of width head_dim starting at column col0 of the
    row-major 2-D x [T, cols] in place.  Token t has position
    positions[t] or (t % seq_len) + pos_offset."""
    require_device(x)
    C().rope(x, int(col0), int(nheads), int(head_dim), table, positions, int(seq_len),
             int(pos_offset), bool(inverse))
    return x


def swiglu_fwd(gu: torch.Tensor, h: Optional[torch.Tensor] = None) -> torch.Tensor:
    require_device(gu)
    if h is None:
        h = torch.empty(*gu.shape[:-1], gu.shape[-1] // 2, dtype=gu.dtype, device=gu.device)
    C().swiglu_fwd(gu, h)
    return h


def swiglu_bwd(gu: torch.Tensor, dh: torch.Tensor, dgu: Optional[torch.Tensor] = None) -> torch.Tensor:
    require_device(gu)
    dgu = torch.empty_like(gu) if dgu is None else dgu
    C().swiglu_bwd(gu, dh, dgu)
    return dgu


def embedding_fwd(ids: torch.Tensor, W: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    require_device(W)
    ids = ids.reshape(-1)
    out = torch.empty(ids.numel(), W.shape[1], dtype=W.dtype, device=W.device) if out is None else out
    C().embedding_fwd(ids, W, out, status(W.device))
    return out


def embedding_bwd(ids: torch.Tensor, dy: torch.Tensor, dW: torch.Tensor) -> torch.Tensor:
    require_device(dW)
    C().embedding_bwd(ids.reshape(-1), dy, dW)
    return dW


def gelu_fwd(x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """GELU, tanh form (bf16)."""
    require_device(x)
    out = torch.empty_like(x) if out is None else out
    C().gelu_fwd(x, out)
    return out


def gelu_bwd(x: torch.Tensor, dy: torch.Tensor, dx: Optional[torch.Tensor] = None) -> torch.Tensor:
    require_device(x)
    dx = torch.empty_like(x) if dx is None else dx
    C().gelu_bwd(x, dy, dx)
    return dx


def dropout(x: torch.Tensor, p: float, seed: int, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Inverted dropout with the counter-hash mask of csrc/dropout.cu (out may
    be x: in place).  The same (seed, p) applied to a gradient is the exact
    backward."""
    require_device(x)
    out = torch.empty_like(x) if out is None else out
    C().dropout(x, out, float(p), int(seed) & 0x7FFFFFFFFFFFFFFF)
    return out


def dropout_mask_reference(n: int, p: float, seed: int) -> torch.Tensor:
    """The kernel's keep mask recomputed on the host (uint64 arithmetic)."""
    import numpy as np
    M = np.uint64(0xFFFFFFFFFFFFFFFF)
    with np.errstate(over="ignore"):
        i = np.arange(n, dtype=np.uint64)
        z = np.uint64(seed & 0x7FFFFFFFFFFFFFFF) ^ (i * np.uint64(0x9E3779B97F4A7C15))
        z = (z + np.uint64(0x9E3779B97F4A7C15)) & M
        z = ((z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)) & M
        z = ((z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)) & M
        z ^= z >> np.uint64(31)
        h = (z >> np.uint64(32)).astype(np.uint64)
    thresh = min(4294967295, int(float(np.float32(p)) * 4294967296.0))  # the kernel gets p as float
    return torch.from_numpy(h >= np.uint64(thresh))


def cast_f32_bf16(x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """bf16 copy of an fp32 tensor (round to nearest even), on the device."""
    require_device(x)
    out = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device) if out is None else out
    C().cast_f32_bf16(x, out)
    return out
