"""Eager restatements of the reference's attention variants (any device).

The B200 kernels implement causal / full / sliding-window GQA attention (the
variants the Llama configurations use).  The rest of the reference's catalogue
is provided here as plain PyTorch for experimentation and as oracles:
MQA / GQA (K/V heads shared), sliding window, dilated, cross attention, ALiBi
and learned relative position biases, kernelised linear attention (elu+1
feature map), block-sparse attention (local band of blocks + strided "summary"
blocks, causal) and hybrid attention (some heads local, the others global).
Reference: include/nn/attention_variants.hpp:14-424 (whose MQA/GQA running
softmax is wrong and whose block-sparse / hybrid classes are stubs).
"""
from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn.functional as F


def _expand_kv(k, n_rep):
    return k.repeat_interleave(n_rep, dim=1) if n_rep > 1 else k


def attention(q, k, v, mask: Optional[torch.Tensor] = None, bias: Optional[torch.Tensor] = None):
    """q [B, Hq, Sq, D]; k, v [B, Hkv, Sk, D]; mask True = disallowed."""
    n_rep = q.shape[1] // k.shape[1]
    k, v = _expand_kv(k, n_rep), _expand_kv(v, n_rep)
    s = q.float() @ k.float().transpose(-1, -2) / math.sqrt(q.shape[-1])
    if bias is not None:
        s = s + bias
    if mask is not None:
        s = s.masked_fill(mask, float("-inf"))
    return torch.softmax(s, -1) @ v.float()


def causal_mask(Sq, Sk, device=None, offset: int = 0):
    qi = torch.arange(Sq, device=device)[:, None] + offset
    ki = torch.arange(Sk, device=device)[None, :]
    return ki > qi


def sliding_window_mask(S, window, device=None):
    qi = torch.arange(S, device=device)[:, None]
    ki = torch.arange(S, device=device)[None, :]
    return (ki > qi) | (ki <= qi - window)


def dilated_mask(S, dilation, device=None):
    qi = torch.arange(S, device=device)[:, None]
    ki = torch.arange(S, device=device)[None, :]
    return (ki > qi) | ((qi - ki) % dilation != 0)


def alibi_slopes(n_heads: int) -> torch.Tensor:
    start = 2 ** (-8.0 / n_heads)
    return torch.tensor([start ** (i + 1) for i in range(n_heads)])


def alibi_bias(n_heads, S, device=None):
    pos = torch.arange(S, device=device)
    rel = (pos[None, :] - pos[:, None]).float()  # key - query (<= 0 on the causal side)
    return alibi_slopes(n_heads).to(device)[:, None, None] * rel[None]


class RelativePositionBias(torch.nn.Module):
    def __init__(self, n_heads: int, max_distance: int = 128):
        super().__init__()
        self.max_distance = max_distance
        self.table = torch.nn.Parameter(torch.zeros(2 * max_distance + 1, n_heads))

    def forward(self, S):
        pos = torch.arange(S, device=self.table.device)
        rel = (pos[None, :] - pos[:, None]).clamp(-self.max_distance, self.max_distance) + self.max_distance
        return self.table[rel].permute(2, 0, 1)


def cross_attention(q, k, v):
    return attention(q, k, v)


def linear_attention(q, k, v, causal: bool = True, eps: float = 1e-6):
    fq, fk = F.elu(q.float()) + 1, F.elu(k.float()) + 1
    n_rep = q.shape[1] // k.shape[1]
    fk, v = _expand_kv(fk, n_rep), _expand_kv(v.float(), n_rep)
    if causal:
        kv = torch.einsum("bhsd,bhse->bhsde", fk, v).cumsum(2)
        z = fk.cumsum(2)
        num = torch.einsum("bhsd,bhsde->bhse", fq, kv)
        den = torch.einsum("bhsd,bhsd->bhs", fq, z)[..., None]
    else:
        kv = torch.einsum("bhsd,bhse->bhde", fk, v)
        num = fq @ kv
        den = (fq @ fk.sum(2, keepdim=True).transpose(-1, -2))
    return num / (den + eps)


def block_sparse_mask(S, block: int, local_blocks: int = 1, stride: int = 0, device=None):
    """Causal block-sparse pattern (True = disallowed): query block i sees key
    blocks i - local_blocks + 1 .. i, plus every block j with (j + 1) % stride
    == 0 (fixed "summary" columns; stride 0 = none)."""
    qb = torch.arange(S, device=device)[:, None] // block
    kb = torch.arange(S, device=device)[None, :] // block
    allowed = (kb <= qb) & (kb > qb - local_blocks)
    if stride > 0:
        allowed |= (kb <= qb) & ((kb + 1) % stride == 0)
    return ~allowed | causal_mask(S, S, device)


def hybrid_attention(q, k, v, local_heads: int, window: int):
    """The first `local_heads` query heads attend within a causal sliding
    window, the rest causally over the whole sequence."""
    S = q.shape[2]
    m = torch.stack([sliding_window_mask(S, window, q.device)] * local_heads +
                    [causal_mask(S, S, q.device)] * (q.shape[1] - local_heads))
    return attention(q, k, v, mask=m[None])

