"""fp32/fp64 eager restatement of the Llama decoder: the correctness oracle.

Plain PyTorch ops only (no custom kernels), any device, gradients by autograd.
It reads the same internal parameter names as `FlatParams` (fp32 copies), so
the B200 engine's loss and every gradient can be compared tensor by tensor.

Math (the standard Llama decoder; the reference's deviations listed in its
transformer_blocks.cpp are deliberately not reproduced):
    RMSNorm(x) = x / sqrt(mean(x^2) + eps) * gamma
    RoPE: interleaved pairs (2i, 2i+1) per head, theta_i = pos * base^(-2i/Dh)
    attention: causal softmax(q k^T / sqrt(Dh)) v with GQA head sharing
    FFN: Wdown (silu(x Wgate^T) * (x Wup^T))
    loss: mean next-token cross-entropy (targets supplied by the caller)
"""
from __future__ import annotations

import math
from typing import Dict, Optional

import torch

from ..config import TransformerConfig


def rmsnorm(x: torch.Tensor, g: torch.Tensor, eps: float) -> torch.Tensor:
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * g


def rope(x: torch.Tensor, base: float, pos_offset: int = 0) -> torch.Tensor:
    """x [B, S, H, Dh] -> rotated (interleaved pairs)."""
    B, S, H, Dh = x.shape
    inv = base ** (-torch.arange(0, Dh, 2, dtype=torch.float64, device=x.device) / Dh)
    pos = torch.arange(pos_offset, pos_offset + S, dtype=torch.float64, device=x.device)
    ang = (pos[:, None] * inv[None, :]).to(x.dtype)
    c, s = torch.cos(ang)[None, :, None, :], torch.sin(ang)[None, :, None, :]
    xr = x.reshape(B, S, H, Dh // 2, 2)
    x0, x1 = xr[..., 0], xr[..., 1]
    return torch.stack([x0 * c - x1 * s, x0 * s + x1 * c], dim=-1).reshape(B, S, H, Dh)


def split_gate_up(wgu: torch.Tensor):
    F2, D = wgu.shape
    v = wgu.reshape(F2 // 256, 2, 128, D)
    return v[:, 0].reshape(F2 // 2, D), v[:, 1].reshape(F2 // 2, D)


def attention(q, k, v, causal=True, window=0):
    """q [B, S, Hq, Dh], k/v [B, S, Hkv, Dh] -> [B, S, Hq, Dh]."""
    B, S, Hq, Dh = q.shape
    rep = Hq // k.shape[2]
    qh = q.permute(0, 2, 1, 3)
    kh = k.permute(0, 2, 1, 3).repeat_interleave(rep, dim=1)
    vh = v.permute(0, 2, 1, 3).repeat_interleave(rep, dim=1)
    s = (qh @ kh.transpose(-1, -2)) / math.sqrt(Dh)
    qi = torch.arange(S, device=q.device)[:, None]
    ki = torch.arange(S, device=q.device)[None, :]
    mask = torch.zeros(S, S, dtype=torch.bool, device=q.device)
    if causal:
        mask |= ki > qi
    if window > 0:
        mask |= ki <= qi - window
    p = torch.softmax(s.masked_fill(mask, float("-inf")), dim=-1)
    return (p @ vh).permute(0, 2, 1, 3)


def forward(params: Dict[str, torch.Tensor], cfg: TransformerConfig, ids: torch.Tensor,
            window: int = 0, drop=None) -> torch.Tensor:
    """Logits [B, S, V] from fp32 parameters keyed by FlatParams names.
    drop(layer, site, x) -> x: optional dropout applied to the attention
    context (site 0, [B, S, q_dim]) and the SwiGLU hidden (site 1, [B, S, F])."""
    B, S = ids.shape
    H, KV, Dh = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim
    h = params["embed"][ids]
    for i in range(cfg.num_layers):
        p = f"layers.{i}."
        x = rmsnorm(h, params[p + "attn_norm"], cfg.norm_eps)
        qkv = x @ params[p + "wqkv"].t()
        q = qkv[..., :H * Dh].reshape(B, S, H, Dh)
        k = qkv[..., H * Dh:(H + KV) * Dh].reshape(B, S, KV, Dh)
        v = qkv[..., (H + KV) * Dh:].reshape(B, S, KV, Dh)
        q, k = rope(q, cfg.rope_base), rope(k, cfg.rope_base)
        o = attention(q, k, v, True, window).reshape(B, S, H * Dh)
        if drop is not None:
            o = drop(i, 0, o)
        h = h + o @ params[p + "wo"].t()
        x = rmsnorm(h, params[p + "ffn_norm"], cfg.norm_eps)
        wg, wu = split_gate_up(params[p + "wgu"])
        a = torch.nn.functional.silu(x @ wg.t()) * (x @ wu.t())
        if drop is not None:
            a = drop(i, 1, a)
        h = h + a @ params[p + "wdown"].t()
    x = rmsnorm(h, params["final_norm"], cfg.norm_eps)
    head = params["embed"] if cfg.tie_embeddings else params["lm_head"]
    return x @ head.t()


def loss_fn(params, cfg, ids, targets, label_smoothing: float = 0.0, drop=None) -> torch.Tensor:
    logits = forward(params, cfg, ids, drop=drop)
    if logits.dtype not in (torch.float32, torch.float64):
        logits = logits.float()
    return torch.nn.functional.cross_entropy(logits.reshape(-1, logits.shape[-1]),
                                             targets.reshape(-1), ignore_index=-100,
                                             label_smoothing=label_smoothing)


def loss_and_grads(params: Dict[str, torch.Tensor], cfg, ids, targets, dtype=torch.float32, drop=None):
    """(loss, {name: grad}) with autograd on copies of `params` in `dtype`."""
    leaf = {k: v.detach().to(dtype).clone().requires_grad_(True) for k, v in params.items()}
    loss = loss_fn(leaf, cfg, ids, targets, drop=drop)
    loss.backward()
    return loss.detach(), {k: v.grad for k, v in leaf.items()}


class OracleTrainer:
    """Reference training loop: AdamW (decoupled wd), global-norm clipping."""

    def __init__(self, params: Dict[str, torch.Tensor], cfg, lr=3e-4, wd=0.1, betas=(0.9, 0.95),
                 eps=1e-8, max_norm=1.0, decay: Optional[Dict[str, bool]] = None):
        self.cfg = cfg
        self.params = {k: v.detach().float().clone().requires_grad_(True) for k, v in params.items()}
        decay = decay or {k: v.dim() > 1 for k, v in self.params.items()}
        groups = [
            {"params": [v for k, v in self.params.items() if decay[k]], "weight_decay": wd},
            {"params": [v for k, v in self.params.items() if not decay[k]], "weight_decay": 0.0},
        ]
        self.opt = torch.optim.AdamW(groups, lr=lr, betas=betas, eps=eps)
        self.max_norm = max_norm

    def step(self, ids, targets) -> float:
        self.opt.zero_grad(set_to_none=True)
        loss = loss_fn(self.params, self.cfg, ids, targets)
        loss.backward()
        if self.max_norm > 0:
            torch.nn.utils.clip_grad_norm_(list(self.params.values()), self.max_norm)
        self.opt.step()
        return float(loss.detach())
