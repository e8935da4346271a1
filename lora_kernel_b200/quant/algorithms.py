"""Quantisation algorithms and formats (offline / host side, plain PyTorch).

Formats (all round-to-nearest-even, saturating):
  int8  symmetric per tensor or per output channel            (DynamicQuantizer)
  int8  with calibrated abs-max                               (StaticQuantizer)
  int4  asymmetric per group of G input channels, two codes per byte
  fp8   e4m3 (max 448) / e5m2 (max 57344) with a per-tensor or per-row scale,
        or 1x128 block scales (the fp8 training format)
Algorithms:
  SmoothQuant   migrate activation outliers into the weights:
                s_j = max|X_j|^a / max|W_:,j|^(1-a);  X' = X / s, W' = W * s
  AWQ           activation-aware weight quantisation: per-input-channel scales
                s = mean|X_j|^a with a grid search over a that minimises the
                output error of the int4-quantised W * s on calibration data
  GPTQ          second-order (Hessian H = 2 X^T X) column-by-column int4/int8
                quantisation with error compensation through the Cholesky
                factor of H^-1, group-wise scales
  QAT           fake quantisation with a straight-through estimator
The device kernels (csrc/quant.cu) consume the int8 / fp8 / int4 codes these
produce; `pack_int4` / `unpack_int4` use the same nibble order (low nibble =
even column).

Reference: include/nn/quantization_production.hpp (DynamicQuantizer :14-47,
StaticQuantizer :52-82, QATWrapper :87-114, fp8 structs :119-175, INT4Quantizer
:190-221 which does not compile, GPTQ/AWQ stubs :226-266, SmoothQuant :271-288,
KVCacheQuantizer :293-316, MixedPrecisionConfig :321-347) and
include/nn/mixed_precision.hpp:73-196.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Callable, Dict, List, Optional, Tuple

import torch

FP8_MAX = {"e4m3": 448.0, "e5m2": 57344.0}
FP8_DTYPE = {"e4m3": torch.float8_e4m3fn, "e5m2": torch.float8_e5m2}


# ------------------------------------------------------------------ formats
def quantize_int8(w: torch.Tensor, per_channel: bool = True) -> Tuple[torch.Tensor, torch.Tensor]:
    wf = w.float()
    amax = wf.abs().amax(dim=1, keepdim=True) if per_channel else wf.abs().amax().reshape(1, 1)
    scale = torch.where(amax > 0, amax / 127.0, torch.ones_like(amax))
    q = torch.clamp(torch.round(wf / scale), -127, 127).to(torch.int8)
    return q, scale.squeeze(1) if per_channel else scale.reshape(())


def dequantize_int8(q: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    s = scale if scale.dim() == 0 else scale[:, None]
    return q.float() * s


def quantize_fp8(x: torch.Tensor, fmt: str = "e4m3", per_row: bool = False,
                 block: int = 0) -> Tuple[torch.Tensor, torch.Tensor]:
    """Scaled fp8: per tensor, per row, or 1 x `block` blocks along the last dim."""
    xf = x.float()
    mx = FP8_MAX[fmt]
    if block:
        R, K = xf.shape
        assert K % block == 0
        xb = xf.view(R, K // block, block)
        amax = xb.abs().amax(-1, keepdim=True)
        scale = torch.where(amax > 0, amax / mx, torch.ones_like(amax))
        q = (xb / scale).clamp(-mx, mx).to(FP8_DTYPE[fmt]).view(R, K)
        return q, scale.squeeze(-1)
    amax = xf.abs().amax(dim=-1, keepdim=True) if per_row else xf.abs().amax().reshape(1, 1)
    scale = torch.where(amax > 0, amax / mx, torch.ones_like(amax))
    q = (xf / scale).clamp(-mx, mx).to(FP8_DTYPE[fmt])
    return q, scale.squeeze(-1) if per_row else scale.reshape(())


def dequantize_fp8(q: torch.Tensor, scale: torch.Tensor, block: int = 0) -> torch.Tensor:
    if block:
        R, K = q.shape
        return (q.float().view(R, K // block, block) * scale[..., None]).view(R, K)
    s = scale if scale.dim() == 0 else scale[:, None]
    return q.float() * s


def quantize_int4_groupwise(w: torch.Tensor, group: int = 128,
                            symmetric: bool = False) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Returns (codes uint8 in [0, 15] [N, K], scale [N, K/G], zero [N, K/G])."""
    N, K = w.shape
    wg = w.float().view(N, K // group, group)
    if symmetric:
        amax = wg.abs().amax(-1)
        scale = torch.where(amax > 0, amax / 7.0, torch.ones_like(amax))
        zero = torch.full_like(scale, 8.0)
    else:
        lo = wg.amin(-1).clamp(max=0.0)
        hi = wg.amax(-1).clamp(min=0.0)
        scale = torch.where(hi > lo, (hi - lo) / 15.0, torch.ones_like(hi))
        zero = torch.round(-lo / scale)
    q = torch.clamp(torch.round(wg / scale[..., None] + zero[..., None]), 0, 15)
    return q.view(N, K).to(torch.uint8), scale, zero


def dequantize_int4_groupwise(q: torch.Tensor, scale: torch.Tensor, zero: torch.Tensor,
                              group: int = 128) -> torch.Tensor:
    N, K = q.shape
    return ((q.float().view(N, K // group, group) - zero[..., None]) * scale[..., None]).view(N, K)


def pack_int4(q: torch.Tensor) -> torch.Tensor:
    """[N, K] codes in [0, 15] -> [N, K/2] bytes, low nibble = even column."""
    q = q.to(torch.uint8)
    return (q[:, 0::2] | (q[:, 1::2] << 4)).contiguous()


def unpack_int4(p: torch.Tensor) -> torch.Tensor:
    out = torch.empty(p.shape[0], p.shape[1] * 2, dtype=torch.uint8, device=p.device)
    out[:, 0::2] = p & 15
    out[:, 1::2] = p >> 4
    return out


class DynamicQuantizer:
    """int8 with the scale taken from the tensor itself at quantisation time."""

    def __init__(self, per_channel: bool = True):
        self.per_channel = per_channel

    def quantize(self, w):
        return quantize_int8(w, self.per_channel)

    dequantize = staticmethod(dequantize_int8)


class StaticQuantizer:
    """int8 with an abs-max calibrated over observed batches."""

    def __init__(self):
        self.amax = 0.0

    def observe(self, x: torch.Tensor) -> None:
        self.amax = max(self.amax, float(x.abs().max()))

    @property
    def scale(self) -> float:
        return self.amax / 127.0 if self.amax > 0 else 1.0

    def quantize(self, x: torch.Tensor) -> torch.Tensor:
        return torch.clamp(torch.round(x.float() / self.scale), -127, 127).to(torch.int8)

    def dequantize(self, q: torch.Tensor) -> torch.Tensor:
        return q.float() * self.scale


# -------------------------------------------------------------- SmoothQuant
def smoothquant_scales(act_absmax: torch.Tensor, w: torch.Tensor, alpha: float = 0.5) -> torch.Tensor:
    """Per input channel: s_j = max|X_j|^alpha / max_i |W_ij|^(1-alpha)."""
    wmax = w.float().abs().amax(dim=0).clamp(min=1e-5)
    amax = act_absmax.float().clamp(min=1e-5)
    return (amax.pow(alpha) / wmax.pow(1.0 - alpha)).clamp(min=1e-5)


def apply_smoothquant(w: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """W' = W * s (columns); the preceding op must divide its output by s."""
    return w.float() * scales[None, :]


# ---------------------------------------------------------------------- AWQ
def awq_search(w: torch.Tensor, x: torch.Tensor, group: int = 128, grid: int = 20
               ) -> Tuple[torch.Tensor, float]:
    """Returns (per-input-channel scales, best alpha) minimising
    ||Q(W * s) (X / s)^T - W X^T|| with int4 group quantisation Q."""
    wf, xf = w.float(), x.float()
    ref = xf @ wf.t()
    xmean = xf.abs().mean(0).clamp(min=1e-6)
    best, best_s, best_a = float("inf"), torch.ones_like(xmean), 0.0
    for k in range(grid + 1):
        a = k / grid
        s = xmean.pow(a)
        s = s / (s.max() * s.min()).sqrt()
        q, sc, z = quantize_int4_groupwise(wf * s[None, :], group)
        wq = dequantize_int4_groupwise(q, sc, z, group) / s[None, :]
        err = float((xf @ wq.t() - ref).pow(2).mean())
        if err < best:
            best, best_s, best_a = err, s, a
    return best_s, best_a


# --------------------------------------------------------------------- GPTQ
def gptq_quantize(w: torch.Tensor, x: torch.Tensor, bits: int = 4, group: int = 128,
                  damp: float = 0.01, block: int = 128) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """GPTQ: quantise W [N, K] column by column, compensating each column's
    rounding error on the not-yet-quantised columns through H^-1 (Cholesky),
    H = 2 X^T X from calibration activations X [T, K].  Returns
    (codes [N, K], scales [N, K/group], zeros [N, K/group]) for asymmetric
    `bits`-bit groups (the int4 kernel format when bits == 4)."""
    W = w.double().clone()
    N, K = W.shape
    X = x.double()
    H = 2.0 * X.t() @ X
    dead = torch.diag(H) == 0
    H[dead, dead] = 1.0
    W[:, dead] = 0.0
    H += damp * torch.mean(torch.diag(H)) * torch.eye(K, dtype=H.dtype, device=H.device)
    Hinv = torch.linalg.cholesky(torch.cholesky_inverse(torch.linalg.cholesky(H)), upper=True)
    qmax = 2 ** bits - 1
    Q = torch.zeros_like(W)
    scales = torch.zeros(N, K // group, dtype=W.dtype, device=W.device)
    zeros = torch.zeros_like(scales)
    for b0 in range(0, K, block):
        b1 = min(b0 + block, K)
        W1 = W[:, b0:b1].clone()
        Q1 = torch.zeros_like(W1)
        Err1 = torch.zeros_like(W1)
        Hinv1 = Hinv[b0:b1, b0:b1]
        for i in range(b1 - b0):
            col = b0 + i
            if col % group == 0:
                g = W[:, col:col + group] if col + group <= b1 else torch.cat(
                    [W1[:, i:], W[:, b1:col + group]], dim=1)
                lo = g.amin(1).clamp(max=0.0)
                hi = g.amax(1).clamp(min=0.0)
                sc = torch.where(hi > lo, (hi - lo) / qmax, torch.ones_like(hi))
                scales[:, col // group] = sc
                zeros[:, col // group] = torch.round(-lo / sc)
            sc, z = scales[:, col // group], zeros[:, col // group]
            wcol = W1[:, i]
            q = torch.clamp(torch.round(wcol / sc + z), 0, qmax)
            Q1[:, i] = q
            deq = (q - z) * sc
            err = (wcol - deq) / Hinv1[i, i]
            W1[:, i:] -= err[:, None] * Hinv1[i, i:][None, :]
            Err1[:, i] = err
        Q[:, b0:b1] = Q1
        W[:, b1:] -= Err1 @ Hinv[b0:b1, b1:]
    return Q.to(torch.uint8), scales.float(), zeros.float()


# ---------------------------------------------------------------------- QAT
class _FakeQuant(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, scale, qmin, qmax):
        ctx.save_for_backward(x, scale)
        ctx.bounds = (qmin, qmax)
        return torch.clamp(torch.round(x / scale), qmin, qmax) * scale

    @staticmethod
    def backward(ctx, g):
        x, scale = ctx.saved_tensors
        qmin, qmax = ctx.bounds
        inside = ((x / scale) >= qmin) & ((x / scale) <= qmax)
        return g * inside, None, None, None  # straight-through inside the range


def fake_quant(x: torch.Tensor, bits: int = 8, per_channel: bool = False) -> torch.Tensor:
    qmax = 2 ** (bits - 1) - 1
    amax = x.detach().abs().amax(dim=1, keepdim=True) if per_channel else x.detach().abs().amax()
    scale = torch.where(amax > 0, amax / qmax, torch.ones_like(amax))
    return _FakeQuant.apply(x, scale, -qmax, qmax)


class QATLinear(torch.nn.Module):
    """Linear layer trained with fake-quantised weights (and optionally inputs)."""

    def __init__(self, inf: int, outf: int, w_bits: int = 8, a_bits: int = 0, bias: bool = False):
        super().__init__()
        self.linear = torch.nn.Linear(inf, outf, bias=bias)
        self.w_bits, self.a_bits = w_bits, a_bits

    def forward(self, x):
        if self.a_bits:
            x = fake_quant(x, self.a_bits)
        w = fake_quant(self.linear.weight, self.w_bits, per_channel=True)
        return torch.nn.functional.linear(x, w, self.linear.bias)


# --------------------------------------------------------- KV / mixed policy
def kv_quantize_reference(x: torch.Tensor, fmt: str = "fp8") -> Tuple[torch.Tensor, torch.Tensor]:
    """CPU restatement of the KV-append kernel: x [T, H, Dh] -> codes, scales [T, H]."""
    amax = x.float().abs().amax(-1, keepdim=True)
    qmax = 448.0 if fmt == "fp8" else 127.0
    scale = torch.where(amax > 0, amax / qmax, torch.ones_like(amax))
    if fmt == "fp8":
        q = (x.float() / scale).clamp(-qmax, qmax).to(torch.float8_e4m3fn)
    else:
        q = torch.clamp(torch.round(x.float() / scale), -127, 127).to(torch.int8)
    return q, scale.squeeze(-1)


@dataclass
class MixedPrecisionConfig:
    """Weight format by depth: the first and last `edge_layers` stay bf16, the
    middle uses `middle` (fp8 / int4) — embeddings and LM head stay bf16."""
    num_layers: int
    edge_layers: int = 2
    middle: str = "int4"

    def format_of(self, layer: int) -> str:
        if layer < self.edge_layers or layer >= self.num_layers - self.edge_layers:
            return "bf16"
        return self.middle
