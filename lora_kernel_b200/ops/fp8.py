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


# ------------------------------------------------------------------ MX form
# Hardware block scaling (tcgen05.mma.kind::mxf8f6f4.block_scale): power-of-two
# scales stored as UE8M0 bytes in 512-byte "SF tiles" (128 rows x 128 K columns
# each, 4 bytes per row = one per 32-wide K sub-block), applied inside the
# tensor core.  The 1 x 128 / 128 x 128 recipe is kept; only the scale is
# rounded up to a power of two.

def sf_tile_bytes(rows: int, K: int, row_multiple: int = 128) -> int:
    """Bytes of the SF tiles of an operand with `rows` rows padded to row_multiple."""
    return ((rows + row_multiple - 1) // row_multiple) * (row_multiple // 128) * (K // 128) * 512


def _sf_index(rows: int, K: int, device) -> torch.Tensor:
    """[rows, K/32] byte offsets of each (row, 32-wide block) exponent in the SF tiles."""
    r = torch.arange(rows, device=device).view(-1, 1)
    j = torch.arange(K // 32, device=device).view(1, -1)
    kb, sub = j // 4, j % 4
    return ((r // 128) * (K // 128) + kb) * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + sub


def sf_to_exponents(sf: torch.Tensor, rows: int, K: int) -> torch.Tensor:
    """SF tiles -> [rows, K/32] integer exponents (byte - 127)."""
    return sf.view(-1)[_sf_index(rows, K, sf.device)].to(torch.int32) - 127


def exponents_to_sf(e: torch.Tensor, row_multiple: int = 128) -> torch.Tensor:
    """[rows, K/32] exponents -> SF tiles (rows padded with exponent 0)."""
    rows, K = e.shape[0], e.shape[1] * 32
    sf = torch.full((sf_tile_bytes(rows, K, row_multiple),), 127, dtype=torch.uint8, device=e.device)
    sf[_sf_index(rows, K, e.device).reshape(-1)] = (e.reshape(-1) + 127).to(torch.uint8)
    return sf


def quantize_mx(x: torch.Tensor, fmt: int = E4M3, row_multiple: int = 128) -> Tuple[torch.Tensor, torch.Tensor]:
    """bf16 [M, K] -> (fp8 bits [M, K], SF tiles): one power-of-two scale per row
    and 128-wide K block."""
    require_device(x)
    M, K = x.shape
    q = torch.empty(M, K, dtype=torch.uint8, device=x.device)
    rows_pad = (M + row_multiple - 1) // row_multiple * row_multiple
    sf = torch.empty(sf_tile_bytes(M, K, row_multiple), dtype=torch.uint8, device=x.device)
    C().quant_mx_rows(x, fmt, q, sf, rows_pad)
    return q, sf


class MXWeight:
    """[N, K] weight as e4m3 with one power-of-two scale per 128 x 128 block (SF
    tiles padded to 256-row multiples, the B operand's tile height), plus the
    transposed copy [K, N] with its own SF tiles for the data-gradient GEMM."""

    def __init__(self, w: torch.Tensor, transpose: bool = True):
        require_device(w)
        w = w.to(torch.bfloat16)
        self.N, self.K = w.shape
        dev = w.device
        self.q = torch.empty(self.N, self.K, dtype=torch.uint8, device=dev)
        self.sf = torch.full((sf_tile_bytes(self.N, self.K, 256),), 127, dtype=torch.uint8, device=dev)
        self.scale = torch.empty((self.N + 127) // 128, self.K // 128, dtype=torch.float32, device=dev)
        self.qt = self.sft = None
        if transpose:
            self.qt = torch.empty(self.K, self.N, dtype=torch.uint8, device=dev)
            self.sft = torch.full((sf_tile_bytes(self.K, self.N, 256),), 127, dtype=torch.uint8, device=dev)
        C().quant_mx_128x128(w, self.q, self.sf, self.scale, self.qt, self.sft)

    def dequantize(self) -> torch.Tensor:
        v = self.q.view(torch.float8_e4m3fn).float()
        s = self.scale.repeat_interleave(128, 0)[:self.N].repeat_interleave(128, 1)
        return v * s


def gemm_mxf8(a8: torch.Tensor, sfa: torch.Tensor, b8: torch.Tensor, sfb: torch.Tensor, *, a_fmt: int = E4M3,
              b_fmt: int = E4M3, out: Optional[torch.Tensor] = None,
              residual: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out [M, N] (bf16) = block-scaled A8 . B8^T (+ residual)."""
    M, N = a8.shape[0], b8.shape[0]
    if out is None:
        out = torch.empty(M, N, dtype=torch.bfloat16, device=a8.device)
    C().gemm_mxf8(a8, sfa, int(a_fmt), b8, sfb, int(b_fmt), out, residual, status(a8.device), 0, 1,
                  None, None, 0, None, None, 0, 0)
    return out


def linear_mxf8(x: torch.Tensor, w: MXWeight, out: Optional[torch.Tensor] = None,
                residual: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y = x W^T with x quantised to e4m3 (1 x 128 blocks, power-of-two scales)."""
    q, sf = quantize_mx(x, E4M3)
    return gemm_mxf8(q, sf, w.q, w.sf, out=out, residual=residual)


def linear_dgrad_mxf8(dy: torch.Tensor, w: MXWeight, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """dx = dy W with dy quantised to e5m2 (1 x 128 blocks) against W^T (e4m3)."""
    assert w.qt is not None, "MXWeight was built without the transposed copy"
    q, sf = quantize_mx(dy, E5M2)
    return gemm_mxf8(q, sf, w.qt, w.sft, a_fmt=E5M2, out=out)


def dequantize_mx(q: torch.Tensor, sf: torch.Tensor, fmt: int = E4M3) -> torch.Tensor:
    """fp32 values of fp8 bits q [R, K] with SF tiles sf."""
    R, K = q.shape
    v = q.view(torch.float8_e4m3fn if fmt == E4M3 else torch.float8_e5m2).float()
    e = sf_to_exponents(sf, R, K).float()
    return v * torch.exp2(e).repeat_interleave(32, 1)
