"""Plain-PyTorch Llama trainer: the library baseline the B200 kernels are
measured against (cuBLAS via F.linear, SDPA attention, nn.RMSNorm, fused
torch.optim.AdamW, FSDP2 `fully_shard` + NCCL for more than one GPU).
Same math as the engine (interleaved RoPE, GQA, SwiGLU, final norm)."""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..config import TrainConfig, TransformerConfig


def _rope(x, cos, sin):
    x0, x1 = x[..., 0::2], x[..., 1::2]
    return torch.stack([x0 * cos - x1 * sin, x0 * sin + x1 * cos], dim=-1).flatten(-2)


class Block(nn.Module):
    def __init__(self, c: TransformerConfig):
        super().__init__()
        self.c = c
        self.n1 = nn.RMSNorm(c.hidden_dim, eps=c.norm_eps)
        self.qkv = nn.Linear(c.hidden_dim, c.qkv_dim, bias=False)
        self.o = nn.Linear(c.q_dim, c.hidden_dim, bias=False)
        self.n2 = nn.RMSNorm(c.hidden_dim, eps=c.norm_eps)
        self.gu = nn.Linear(c.hidden_dim, 2 * c.ff_dim, bias=False)
        self.down = nn.Linear(c.ff_dim, c.hidden_dim, bias=False)

    def forward(self, h, cos, sin):
        c = self.c
        B, S, _ = h.shape
        qkv = self.qkv(self.n1(h))
        q, k, v = qkv.split([c.q_dim, c.kv_dim, c.kv_dim], -1)
        q = _rope(q.view(B, S, c.num_heads, c.head_dim), cos, sin).transpose(1, 2)
        k = _rope(k.view(B, S, c.num_kv_heads, c.head_dim), cos, sin).transpose(1, 2)
        v = v.view(B, S, c.num_kv_heads, c.head_dim).transpose(1, 2)
        o = F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=True)
        h = h + self.o(o.transpose(1, 2).reshape(B, S, c.q_dim))
        g, u = self.gu(self.n2(h)).chunk(2, -1)
        return h + self.down(F.silu(g) * u)


class TorchLlama(nn.Module):
    def __init__(self, c: TransformerConfig):
        super().__init__()
        self.c = c
        self.embed = nn.Embedding(c.vocab_size, c.hidden_dim)
        self.blocks = nn.ModuleList([Block(c) for _ in range(c.num_layers)])
        self.norm = nn.RMSNorm(c.hidden_dim, eps=c.norm_eps)
        self.head = nn.Linear(c.hidden_dim, c.vocab_size, bias=False)
        for p in self.parameters():
            if p.dim() > 1:
                nn.init.normal_(p, 0.0, c.init_std)

    def forward(self, ids):
        c = self.c
        S = ids.shape[1]
        inv = c.rope_base ** (-torch.arange(0, c.head_dim, 2, device=ids.device, dtype=torch.float64) / c.head_dim)
        ang = torch.arange(S, device=ids.device, dtype=torch.float64)[:, None] * inv[None]
        cos = torch.cos(ang)[None, :, None].to(torch.bfloat16)
        sin = torch.sin(ang)[None, :, None].to(torch.bfloat16)
        h = self.embed(ids)
        for b in self.blocks:
            h = b(h, cos, sin)
        return self.head(self.norm(h))


class TorchBaselineTrainer:
    """The same training step on library code.

    precision "mixed" (default, the engine's numerics): fp32 master weights,
    bf16 compute (torch.autocast on one GPU; FSDP2 MixedPrecisionPolicy with
    bf16 parameters and fp32 gradient reduction on several), fused fp32 AdamW,
    global-norm clip.  "bf16": bf16 weights, moments and AdamW (no master
    copy), which does less optimizer work than the engine."""

    def __init__(self, cfg: TransformerConfig, tc: TrainConfig, device="cuda", world: int = 1,
                 precision: str = "mixed"):
        if precision not in ("mixed", "bf16"):
            raise ValueError(precision)
        torch.manual_seed(tc.seed)
        self.precision = precision
        dtype = torch.float32 if precision == "mixed" else torch.bfloat16
        m = TorchLlama(cfg).to(device=device, dtype=dtype)
        self.autocast = precision == "mixed" and world == 1
        if world > 1:
            from torch.distributed.fsdp import MixedPrecisionPolicy, fully_shard
            mp = (MixedPrecisionPolicy(param_dtype=torch.bfloat16, reduce_dtype=torch.float32)
                  if precision == "mixed" else MixedPrecisionPolicy())
            for b in m.blocks:
                fully_shard(b, mp_policy=mp)
            fully_shard(m, mp_policy=mp)
        self.m = m
        self.opt = torch.optim.AdamW(m.parameters(), lr=tc.lr, betas=(tc.beta1, tc.beta2), eps=tc.eps,
                                     weight_decay=tc.weight_decay, fused=True)
        self.tc = tc
        self.loss_acc = torch.zeros(2, device=device)

    def micro_step_async(self, ids, targets):
        from ..utils.profiler import ph
        with ph("fwd"):
            with torch.autocast("cuda", dtype=torch.bfloat16, enabled=self.autocast):
                logits = self.m(ids)
            loss = F.cross_entropy(logits.float().view(-1, logits.shape[-1]), targets.reshape(-1))
        with ph("bwd"):
            loss.backward()
        with ph("step.clip+adamw"):
            torch.nn.utils.clip_grad_norm_(self.m.parameters(), self.tc.max_grad_norm)
            self.opt.step()
            self.opt.zero_grad(set_to_none=True)
        self.loss_acc[0] += loss.detach() * ids.numel()
        self.loss_acc[1] += ids.numel()

    def train_step(self, ids, targets) -> float:
        self.loss_acc.zero_()
        self.micro_step_async(ids, targets)
        s, n = self.loss_acc.tolist()
        return s / n
