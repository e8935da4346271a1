"""K2: block-scaled fp8 GEMMs (1 x 128 activation / gradient scales, 128 x 128
weight scales) and their quantisers.

    w8 = Fp8Weight(w)                       # e4m3 W and W^T with shared block scales
    y  = linear_fp8(x, w8)                  # x quantised e4m3 on the fly: y = x W^T
    dx = linear_dgrad_fp8(dy, w8)           # dy quantised e5m2: dx = dy W

fp8 values travel as uint8 tensors holding the e4m3 / e5m2 bit patterns.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from .._ext import C, require_device, status

E4M3, E5M2 = 0, 1


def quantize_1x128(x: torch.Tensor, fmt: int = E4M3) -> Tuple[torch.Tensor, torch.Tensor]:
    """bf16 [M, K] -> (fp8 bits [M, K], fp32 scales [K/128, M])."""
    require_device(x)
    M, K = x.shape
    q = torch.empty(M, K, dtype=torch.uint8, device=x.device)
    s = torch.empty(K // 128, M, dtype=torch.float32, device=x.device)
    C().quant_1x128(x, fmt, q, s)
    return q, s


class Fp8Weight:
    """[N, K] weight as e4m3 with one scale per 128 x 128 block, plus the
    transposed copy [K, N] used by the data-gradient GEMM."""

    def __init__(self, w: torch.Tensor, transpose: bool = True):
        require_device(w)
        w = w.to(torch.bfloat16)
        self.N, self.K = w.shape
        dev = w.device
        self.q = torch.empty(self.N, self.K, dtype=torch.uint8, device=dev)
        self.qt = torch.empty(self.K, self.N, dtype=torch.uint8, device=dev) if transpose else None
        self.scale = torch.empty((self.N + 127) // 128, self.K // 128, dtype=torch.float32, device=dev)
        C().quant_128x128(w, self.q, self.qt, self.scale)

    @property
    def scale_t(self) -> torch.Tensor:
        """Block scales of W^T ([K/128, N/128])."""
        return self.scale.t().contiguous()

    def dequantize(self) -> torch.Tensor:
        v = self.q.view(torch.float8_e4m3fn).float()
        s = self.scale.repeat_interleave(128, 0)[:self.N].repeat_interleave(128, 1)
        return v * s


def gemm_fp8(a8: torch.Tensor, sa: torch.Tensor, b8: torch.Tensor, sb: torch.Tensor, *, a_fmt: int = E4M3,
             out: Optional[torch.Tensor] = None, residual: Optional[torch.Tensor] = None) -> torch.Tensor:
    M, N = a8.shape[0], b8.shape[0]
    if out is None:
        out = torch.empty(M, N, dtype=torch.bfloat16, device=a8.device)
    C().gemm_fp8(a8, sa, int(a_fmt), b8, sb, out, residual, status(a8.device))
    return out


def linear_fp8(x: torch.Tensor, w: Fp8Weight, out: Optional[torch.Tensor] = None,
               residual: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y = x W^T with x quantised to e4m3 (1 x 128 blocks)."""
    q, s = quantize_1x128(x, E4M3)
    return gemm_fp8(q, s, w.q, w.scale, out=out, residual=residual)


def linear_dgrad_fp8(dy: torch.Tensor, w: Fp8Weight, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """dx = dy W with dy quantised to e5m2 (1 x 128 blocks) against W^T (e4m3)."""
    assert w.qt is not None, "Fp8Weight was built without the transposed copy"
    q, s = quantize_1x128(dy, E5M2)
    return gemm_fp8(q, s, w.qt, w.scale_t, a_fmt=E5M2, out=out)


def dequantize_1x128(q: torch.Tensor, s: torch.Tensor, fmt: int = E4M3) -> torch.Tensor:
    v = q.view(torch.float8_e4m3fn if fmt == E4M3 else torch.float8_e5m2).float()
    return v * s.t().repeat_interleave(128, 1)
