"""Offline model utilities: merging and pruning of state dicts.

Merging: linear interpolation, task arithmetic (base + lambda * sum of task
vectors) and TIES (trim each task vector to its top-k% magnitudes, elect a
per-parameter sign by total mass, average the values that agree with it).
Pruning: unstructured magnitude pruning and structured row (output-channel)
pruning by L2 norm.  Gradient noise for regularisation.
Reference: ModelMerging (include/nn/model_merging.hpp:7-35, TIES reduced to a
mean there), ModelPruning (include/nn/model_pruning.hpp:8-37), GradientNoise
(include/nn/training_enhancements.hpp:147-162).
"""
from __future__ import annotations

from typing import Dict, List, Optional, Sequence, Tuple

import torch

SD = Dict[str, torch.Tensor]


def linear_merge(models: Sequence[SD], weights: Sequence[float]) -> SD:
    tot = float(sum(weights))
    return {k: sum(w * m[k].float() for m, w in zip(models, weights)) / tot for k in models[0]}


def task_arithmetic(base: SD, finetuned: Sequence[SD], lam: float = 1.0) -> SD:
    return {k: base[k].float() + lam * sum(f[k].float() - base[k].float() for f in finetuned) for k in base}


def ties_merge(base: SD, finetuned: Sequence[SD], density: float = 0.2, lam: float = 1.0) -> SD:
    out = {}
    for k in base:
        b = base[k].float()
        taus = []
        for f in finetuned:
            t = f[k].float() - b
            n = t.numel()
            keep = max(1, int(round(density * n)))
            thr = t.abs().flatten().kthvalue(n - keep + 1).values if keep < n else t.abs().min() - 1
            taus.append(torch.where(t.abs() >= thr, t, torch.zeros_like(t)))
        T = torch.stack(taus)
        sign = torch.sign(T.sum(0))
        agree = (torch.sign(T) == sign) & (T != 0)
        cnt = agree.sum(0).clamp(min=1)
        out[k] = b + lam * (T * agree).sum(0) / cnt
    return out


def prune_magnitude(w: torch.Tensor, sparsity: float) -> torch.Tensor:
    n = w.numel()
    k = int(sparsity * n)
    if k <= 0:
        return w.clone()
    thr = w.abs().flatten().kthvalue(k).values
    return torch.where(w.abs() > thr, w, torch.zeros_like(w))


def prune_structured_rows(w: torch.Tensor, fraction: float) -> torch.Tensor:
    norms = w.float().norm(dim=1)
    k = int(fraction * w.shape[0])
    out = w.clone()
    if k > 0:
        out[norms.argsort()[:k]] = 0
    return out


def gradient_noise_(grads: torch.Tensor, step: int, eta: float = 0.01, gamma: float = 0.55,
                    generator=None, scale=None) -> torch.Tensor:
    """g += N(0, eta / (1 + step)^gamma) (Neelakantan et al. 2015).  `scale`
    (a number or a device tensor, e.g. the dynamic loss scale that the stored
    gradients still carry) multiplies the noise so it lands in the same units."""
    std = (eta / (1.0 + step) ** gamma) ** 0.5
    noise = torch.randn(grads.shape, generator=generator, device=grads.device, dtype=grads.dtype).mul_(std)
    if scale is not None:
        noise.mul_(scale)
    return grads.add_(noise)


def noise_seed(seed: int, step: int, rank: int = -1) -> int:
    """Generator seed of the gradient noise of one step: the same on every rank
    when the gradients are replicated (rank = -1), distinct per rank when each
    rank holds a different shard."""
    z = (seed * 0x9E3779B97F4A7C15 + step * 0xBF58476D1CE4E5B9 + (rank + 1) * 0x94D049BB133111EB)
    return z & ((1 << 63) - 1)


def fuse_conv_bn(conv_w: torch.Tensor, conv_b: Optional[torch.Tensor], bn_gamma: torch.Tensor,
                 bn_beta: torch.Tensor, bn_mean: torch.Tensor, bn_var: torch.Tensor,
                 eps: float = 1e-5) -> Tuple[torch.Tensor, torch.Tensor]:
    """Fold an inference-mode batch norm into the convolution (or linear layer)
    before it: y = gamma (conv(x) - mean) / sqrt(var + eps) + beta becomes a
    convolution with weight w * s (per output channel) and bias (b - mean) s +
    beta, s = gamma / sqrt(var + eps).  Output channels are dimension 0 of
    conv_w.  Returns (weight, bias) in conv_w's dtype, computed in fp32.

    Reference: BatchNormFusion::fuse_conv_bn
    (include/nn/training_enhancements.hpp:263-277), which uses eps = 1e-6."""
    s = bn_gamma.float() / torch.sqrt(bn_var.float() + eps)
    w = conv_w.float() * s.view(-1, *([1] * (conv_w.dim() - 1)))
    b0 = conv_b.float() if conv_b is not None else torch.zeros_like(s)
    b = (b0 - bn_mean.float()) * s + bn_beta.float()
    return w.to(conv_w.dtype), b.to(conv_w.dtype)
