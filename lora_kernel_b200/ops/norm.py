"""K5: RMSNorm forward / backward wrappers (bf16 data, fp32 statistics)."""
from __future__ import annotations

from typing import Optional

import torch

from .._ext import C, require_device


def rmsnorm_fwd(x: torch.Tensor, gamma: torch.Tensor, eps: float, *,
                residual: Optional[torch.Tensor] = None, y: Optional[torch.Tensor] = None,
                h_out: Optional[torch.Tensor] = None, rstd: Optional[torch.Tensor] = None):
    """y = rmsnorm(x [+ residual]).  Returns (y, rstd, h) where h = x + residual
    (h is x itself when there is no residual)."""
    require_device(x)
    D = x.shape[-1]
    M = x.numel() // D
    y = torch.empty_like(x) if y is None else y
    rstd = torch.empty(M, dtype=torch.float32, device=x.device) if rstd is None else rstd
    if residual is not None and h_out is None:
        h_out = torch.empty_like(x)
    C().rmsnorm_fwd(x, residual, gamma, y, h_out if residual is not None else None, rstd, float(eps))
    return y, rstd, (h_out if residual is not None else x)


_partials = {}


def _partial(M: int, D: int, device) -> torch.Tensor:
    rows = C().rmsnorm_bwd_partial_rows(M)
    key = (device, D)
    buf = _partials.get(key)
    if buf is None or buf.shape[0] < rows:
        buf = torch.empty(rows, D, dtype=torch.float32, device=device)
        _partials[key] = buf
    return buf


def rmsnorm_bwd(dy: torch.Tensor, x: torch.Tensor, gamma: torch.Tensor, rstd: torch.Tensor,
                dgamma: torch.Tensor, *, dres: Optional[torch.Tensor] = None,
                dx: Optional[torch.Tensor] = None, accumulate: bool = True) -> torch.Tensor:
    """dx = d rmsnorm / dx (+ dres); dgamma (fp32) += / = sum over rows, or,
    for a bf16 dgamma, the sum stored (accumulate must then be False)."""
    require_device(x)
    D = x.shape[-1]
    dx = torch.empty_like(x) if dx is None else dx
    if dgamma.dtype == torch.bfloat16:
        accumulate = False
    C().rmsnorm_bwd(dy, x, gamma, rstd, dres, dx, dgamma, _partial(x.numel() // D, D, x.device),
                    bool(accumulate))
    return dx


def layernorm_fwd(x: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, eps: float = 1e-5):
    """LayerNorm with affine gamma / beta (bf16).  Returns (y, mean, rstd)."""
    require_device(x)
    D = x.shape[-1]
    M = x.numel() // D
    y = torch.empty_like(x)
    mean = torch.empty(M, dtype=torch.float32, device=x.device)
    rstd = torch.empty(M, dtype=torch.float32, device=x.device)
    C().layernorm_fwd(x, gamma, beta, y, mean, rstd, float(eps))
    return y, mean, rstd


def layernorm_bwd(dy: torch.Tensor, x: torch.Tensor, gamma: torch.Tensor, mean: torch.Tensor,
                  rstd: torch.Tensor, dgamma: torch.Tensor, dbeta: torch.Tensor) -> torch.Tensor:
    """dx; the parameter gradients are added into dgamma / dbeta (fp32)."""
    require_device(x)
    dx = torch.empty_like(x)
    C().layernorm_bwd(dy, x, gamma, mean, rstd, dx, dgamma, dbeta)
    return dx
