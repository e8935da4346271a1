"""K1: tcgen05 GEMM wrappers.

`gemm(a, b)` computes a @ b.T for a [M, K] and b [N, K]; either operand may be a
transpose view (MN-major), which is how the three GEMMs of a linear layer run
without transpose copies:

    forward  y  = gemm(x, W)                 (both K-major)
    dgrad    dx = gemm(dy, W.t())            (B MN-major)
    wgrad    dW += gemm(dy.t(), x.t())       (both MN-major, fp32 accumulate)
"""
from __future__ import annotations

from typing import Optional

import torch

from .._ext import C, require_device, status

EPI = {"bf16": 0, "f32": 1, "f32_acc": 2, "bf16_resid": 3, "swiglu": 4, "swiglu_bwd": 6, "bf16_rope": 7}


_cap = {}

# optional per-problem tile widths measured by utils/autotune.py (LK_GEMM_TUNING)
_tuning = None
_tuning_loaded = False


def set_tuning(table) -> None:
    """Use `table` (utils.autotune.GemmTable, or a path to its JSON; None:
    the dispatcher's built-in rule) for every gemm call without an explicit bn."""
    global _tuning, _tuning_loaded
    if isinstance(table, str):
        from ..utils.autotune import GemmTable
        table = GemmTable.load(table)
    _tuning, _tuning_loaded = table, True


def tuned_bn(a: torch.Tensor, b: torch.Tensor, epi: str) -> int:
    """Tile width from the tuning table (0 = let the dispatcher choose)."""
    global _tuning_loaded
    if not _tuning_loaded:
        import os
        path = os.environ.get("LK_GEMM_TUNING", "")
        set_tuning(path or None)
    return _tuning.lookup(a, b, epi) if _tuning is not None else 0


def _check_device(t: torch.Tensor) -> None:
    idx = t.device.index
    if idx not in _cap:
        require_device(t)
        _cap[idx] = True


def gemm(a: torch.Tensor, b: torch.Tensor, out: Optional[torch.Tensor] = None, *,
         epi: str = "bf16", residual: Optional[torch.Tensor] = None,
         h_out: Optional[torch.Tensor] = None, alpha: float = 1.0, bn: int = 0,
         a2: Optional[torch.Tensor] = None, b2: Optional[torch.Tensor] = None,
         rope: Optional[tuple] = None) -> torch.Tensor:
    """out = alpha * (a @ b.T [+ a2 @ b2.T]) with the requested epilogue.
    swiglu_bwd: a @ b.T is dh, the gradient of silu(gate) * up; residual is the
    forward gate|up activation [M, 2N] and out receives its gradient [M, 2N].
    rope = (table, cols, head_dim, seq_len, pos_offset): the bf16 output's first
    `cols` columns are rotated (interleaved-pair RoPE, row m at position
    m % seq_len + pos_offset) in the epilogue (epi becomes "bf16_rope")."""
    _check_device(a)
    if bn == 0:
        bn = tuned_bn(a, b, epi)
    M, N = a.shape[0], b.shape[0]
    if out is None:
        dt = torch.float32 if epi in ("f32", "f32_acc") else torch.bfloat16
        cols = 2 * N if epi == "swiglu_bwd" else N  # gate|up gradients
        out = (torch.zeros if epi == "f32_acc" else torch.empty)(M, cols, dtype=dt, device=a.device)
    if rope is not None:
        table, cols, dh, seq, off = rope
        C().gemm(a, b, out, EPI["bf16_rope"], None, None, float(alpha), status(a.device), int(bn), a2, b2,
                 table, int(cols), int(dh), int(seq), int(off))
    else:
        C().gemm(a, b, out, EPI[epi], residual, h_out, float(alpha), status(a.device), int(bn), a2, b2,
                 None, 0, 0, 0, 0)
    return out


def linear(x: torch.Tensor, w: torch.Tensor, residual: Optional[torch.Tensor] = None,
           out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y = x @ w.T (+ residual) for x [T, K], w [N, K]."""
    return gemm(x, w, out, epi="bf16_resid" if residual is not None else "bf16", residual=residual)


def linear_swiglu(x: torch.Tensor, w_gu: torch.Tensor, gu_out: Optional[torch.Tensor] = None,
                  h_out: Optional[torch.Tensor] = None):
    """gate|up projection with the SwiGLU epilogue; w_gu rows are blocks of 128
    gate rows followed by 128 up rows.  Returns (gu [T, 2F], h [T, F])."""
    T, F2 = x.shape[0], w_gu.shape[0]
    if gu_out is None:
        gu_out = torch.empty(T, F2, dtype=torch.bfloat16, device=x.device)
    if h_out is None:
        h_out = torch.empty(T, F2 // 2, dtype=torch.bfloat16, device=x.device)
    gemm(x, w_gu, gu_out, epi="swiglu", h_out=h_out)
    return gu_out, h_out


def linear_dgrad(dy: torch.Tensor, w: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """dx = dy @ w for dy [T, N], w [N, K]."""
    return gemm(dy, w.t(), out)


def linear_wgrad(dy: torch.Tensor, x: torch.Tensor, grad: torch.Tensor) -> torch.Tensor:
    """grad (fp32 [N, K]) += dy.T @ x."""
    return gemm(dy.t(), x.t(), grad, epi="f32_acc")


def interleave_gate_up(w_gate: torch.Tensor, w_up: torch.Tensor) -> torch.Tensor:
    """[F, D] gate and up weights -> [2F, D] in blocks of 128 gate rows then 128 up rows."""
    F, D = w_gate.shape
    assert F % 128 == 0
    g = w_gate.reshape(F // 128, 128, D)
    u = w_up.reshape(F // 128, 128, D)
    return torch.stack([g, u], dim=1).reshape(2 * F, D)


def split_gate_up(w_gu: torch.Tensor):
    F2, D = w_gu.shape[0], w_gu.shape[1:]
    v = w_gu.reshape(F2 // 256, 2, 128, *D)
    return v[:, 0].reshape(F2 // 2, *D), v[:, 1].reshape(F2 // 2, *D)
