"""K13 paged decode attention, K15 KV append / gather, K19 sampling, K14
quantised-weight kernels: Python wrappers."""
from __future__ import annotations

import math
from typing import Optional

import torch

from .._ext import C, require_device, status

KV_DTYPES = {"bf16": 0, "fp8": 1, "int8": 2}
KV_TORCH = {"bf16": torch.bfloat16, "fp8": torch.float8_e4m3fn, "int8": torch.int8}
QFMT = {"int8": 0, "fp8": 1, "int4": 2}


def kv_append(qkv: torch.Tensor, Hq: int, Hkv: int, Dh: int, slots: torch.Tensor, k_cache, v_cache,
              k_scale=None, v_scale=None, kv_dtype: str = "bf16") -> None:
    require_device(qkv)
    C().kv_append(qkv, Hq, Hkv, Dh, slots, k_cache, v_cache, k_scale, v_scale, KV_DTYPES[kv_dtype],
                  status(qkv.device))


def kv_gather(k_cache, v_cache, k_scale, v_scale, slots: torch.Tensor, Hkv: int, Dh: int,
              kv_dtype: str = "bf16", out: Optional[torch.Tensor] = None) -> torch.Tensor:
    if out is None:
        out = torch.empty(slots.numel(), 2 * Hkv * Dh, dtype=torch.bfloat16, device=slots.device)
    C().kv_gather(k_cache, v_cache, k_scale, v_scale, slots, Hkv, Dh, out, KV_DTYPES[kv_dtype],
                  status(slots.device))
    return out


_parts = {}


def decode_attention(q: torch.Tensor, k_cache, v_cache, k_scale, v_scale, block_tables: torch.Tensor,
                     ctx_lens: torch.Tensor, block_size: int, Hq: int, Hkv: int, Dh: int, *,
                     kv_dtype: str = "bf16", max_ctx: int = 0, split_len: int = 512,
                     out: Optional[torch.Tensor] = None, scale: Optional[float] = None) -> torch.Tensor:
    """q [num_seqs, Hq*Dh] (post-RoPE) -> out [num_seqs, Hq*Dh]; ctx_lens include the new token."""
    require_device(q)
    n = q.shape[0]
    scale = 1.0 / math.sqrt(Dh) if scale is None else scale
    if out is None:
        out = torch.empty(n, Hq * Dh, dtype=torch.bfloat16, device=q.device)
    max_ctx = max_ctx or block_tables.shape[1] * block_size
    nsplit = max(1, (max_ctx + split_len - 1) // split_len)
    po = pm = None
    if nsplit > 1:
        key = (q.device, n, Hq, nsplit, Dh)
        bufs = _parts.get(key)
        if bufs is None:
            bufs = (torch.empty(n * Hq * nsplit * Dh, device=q.device),
                    torch.empty(n * Hq * nsplit * 2, device=q.device))
            _parts[key] = bufs
        po, pm = bufs
    C().decode_attention(q, k_cache, v_cache, k_scale, v_scale, block_tables, ctx_lens, block_size, Hq,
                         Hkv, Dh, float(scale), split_len, nsplit, po, pm, out, KV_DTYPES[kv_dtype],
                         status(q.device))
    return out


def sample(logits: torch.Tensor, temperature: Optional[torch.Tensor] = None, seed: int = 0, *,
           v0: int = 0, out_val: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Greedy (temperature 0 / None) or exact temperature sampling (Gumbel-max).
    v0: vocabulary id of column 0 (a vocabulary-parallel slice); out_val
    receives each row's winning (noised) score for the cross-rank pick."""
    require_device(logits)
    tok = torch.empty(logits.shape[0], dtype=torch.int64, device=logits.device)
    C().sample(logits, temperature, int(seed) & ((1 << 63) - 1), tok, out_val, int(v0))
    return tok


def sample_topp(logits: torch.Tensor, temperature: torch.Tensor, top_p: torch.Tensor, seed: int = 0,
                row_seeds: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Nucleus sampling on one GPU: each row draws from softmax(logits / T)
    restricted to its smallest top set of probability mass >= top_p (rows with
    T <= 0 are greedy, rows with top_p >= 1 sample from the whole vocabulary).
    row_seeds (int64 per row): each row's noise from its own seed instead of
    (seed, row), so a request's draws do not depend on its batch row."""
    require_device(logits)
    tok = torch.empty(logits.shape[0], dtype=torch.int64, device=logits.device)
    C().sample_topp(logits, temperature.float().contiguous(), top_p.float().contiguous(),
                    int(seed) & ((1 << 63) - 1), row_seeds, tok)
    return tok


class QuantizedWeight:
    """A [N, K] weight quantised on the device: int8 / fp8 per row, int4 per group."""

    def __init__(self, w: torch.Tensor, fmt: str = "int4", group: int = 128):
        require_device(w)
        w = w.to(torch.bfloat16).contiguous()
        N, K = w.shape
        self.fmt, self.group, self.N, self.K = fmt, group, N, K
        dev = w.device
        if fmt == "int4":
            self.q = torch.empty(N, K // 2, dtype=torch.uint8, device=dev)
            self.scale = torch.empty(N, K // group, dtype=torch.float32, device=dev)
            self.zero = torch.empty(N, K // group, dtype=torch.float32, device=dev)
        else:
            self.q = torch.empty(N, K, dtype=torch.int8 if fmt == "int8" else torch.uint8, device=dev)
            self.scale = torch.empty(N, dtype=torch.float32, device=dev)
            self.zero = None
        C().quantize(QFMT[fmt], w, group, self.q, self.scale, self.zero)

    @classmethod
    def from_parts(cls, fmt: str, group: int, N: int, K: int, q: torch.Tensor, scale: torch.Tensor,
                   zero: Optional[torch.Tensor] = None) -> "QuantizedWeight":
        """A weight quantised earlier (e.g. loaded from a checkpoint)."""
        self = cls.__new__(cls)
        self.fmt, self.group, self.N, self.K = fmt, group, N, K
        self.q, self.scale, self.zero = q, scale, zero
        return self

    def dequantize(self, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        if out is None:
            out = torch.empty(self.N, self.K, dtype=torch.bfloat16, device=self.q.device)
        C().dequantize(QFMT[self.fmt], self.q, self.scale, self.zero, self.N, self.K, self.group, out)
        return out

    def nbytes(self) -> int:
        n = self.q.numel() * self.q.element_size() + self.scale.numel() * 4
        return n + (self.zero.numel() * 4 if self.zero is not None else 0)

    def matmul_t(self, x: torch.Tensor, out: Optional[torch.Tensor] = None,
                 scratch: Optional[torch.Tensor] = None, residual: Optional[torch.Tensor] = None) -> torch.Tensor:
        """x [M, K] @ W^T (+ residual) -> [M, N].  Decode batches (M <= 256): the
        weight-streaming tcgen05 dequant GEMM (one pass over the packed weights
        for the whole batch, split-K partials summed in order); prefill: a
        dequantise-to-bf16 pass followed by the tcgen05 GEMM (the weight tile
        would otherwise be dequantised once per 128-row block of x)."""
        M = x.shape[0]
        if out is None:
            out = torch.empty(M, self.N, dtype=torch.bfloat16, device=x.device)
        if M <= 256 and self.K % 64 == 0 and self.N % 4 == 0 and (self.fmt != "int4" or self.group % 64 == 0):
            # split-K partials live in one fixed buffer per device (allocated once, so
            # CUDA graphs captured against it stay valid); the split count shrinks
            # to fit it
            splits = min(C().dq_gemm_splits(M, self.N, self.K), DQ_PARTIAL_FLOATS // (M * self.N))
            part = counters = None
            if splits > 1:
                part, counters = _dq_workspace(x.device)
            else:
                splits = 1
            C().dq_gemm(x, self.q, self.scale, self.zero, QFMT[self.fmt], self.N, self.K, self.group, out,
                        residual, part, splits, status(x.device), counters)
            return out
        from .gemm import gemm
        w = self.dequantize(scratch)
        return gemm(x, w, out, epi="bf16_resid" if residual is not None else "bf16", residual=residual)


DQ_PARTIAL_FLOATS = 16 << 20  # 64 MB of fp32 split-K partials per device
DQ_COUNTERS = 16384           # one per 128-row weight tile; the kernel leaves them zero
_dq_parts = {}


def _dq_workspace(device):
    """The split-K partial buffer and tile counters of `device`, allocated once
    (CUDA graphs captured against them stay valid; launches on one stream reuse
    them in order)."""
    ws = _dq_parts.get(device)
    if ws is None:
        ws = (torch.empty(DQ_PARTIAL_FLOATS, dtype=torch.float32, device=device),
              torch.zeros(DQ_COUNTERS, dtype=torch.int32, device=device))
        _dq_parts[device] = ws
    return ws
