"""Auxiliary training losses (autograd, over the model's logits / log-probs).

  distillation_loss   alpha * T^2 * KL(softmax(t/T) || softmax(s/T)) + (1-alpha) * CE
  ppo_loss            clipped surrogate: -mean(min(r A, clip(r, 1-eps, 1+eps) A)),
                      r = exp(logp_new - logp_old), optional KL penalty to a reference
  grpo_advantages     group-relative advantages: (R - mean_group) / (std_group + eps)
  grpo_loss           PPO-style clipped objective on group-relative advantages plus
                      beta * KL(new || ref) (k3 estimator)
  label_smoothing_ce  the fused CE kernel handles this on the B200 path; the eager
                      form is kept for tests and CPU use
Reference: KnowledgeDistillation (include/nn/distillation.hpp:7-45), PPOTrainer
(include/nn/ppo_training.hpp:9-39), GRPOTrainer (include/nn/grpo_training.hpp:9-39),
LabelSmoothing (include/nn/training_enhancements.hpp:167-192) - loss values only
there; here every loss is differentiable.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def distillation_loss(student_logits, teacher_logits, targets=None, temperature: float = 2.0,
                      alpha: float = 0.5):
    T = temperature
    s = F.log_softmax(student_logits.float() / T, -1)
    t = F.log_softmax(teacher_logits.float() / T, -1)
    kd = F.kl_div(s, t, log_target=True, reduction="batchmean") * T * T
    if targets is None:
        return kd
    ce = F.cross_entropy(student_logits.float().reshape(-1, student_logits.shape[-1]), targets.reshape(-1))
    return alpha * kd + (1.0 - alpha) * ce


def token_logprobs(logits, tokens):
    return torch.gather(F.log_softmax(logits.float(), -1), -1, tokens.unsqueeze(-1)).squeeze(-1)


def ppo_loss(logp_new, logp_old, advantages, clip_eps: float = 0.2, logp_ref=None, kl_coef: float = 0.0,
             mask=None):
    ratio = torch.exp(logp_new - logp_old)
    surr = torch.minimum(ratio * advantages, torch.clamp(ratio, 1 - clip_eps, 1 + clip_eps) * advantages)
    loss = -surr
    if logp_ref is not None and kl_coef:
        loss = loss + kl_coef * (logp_new - logp_ref)
    if mask is not None:
        return (loss * mask).sum() / mask.sum().clamp(min=1)
    return loss.mean()


def grpo_advantages(rewards: torch.Tensor, group_size: int, eps: float = 1e-6) -> torch.Tensor:
    r = rewards.float().view(-1, group_size)
    return ((r - r.mean(1, keepdim=True)) / (r.std(1, keepdim=True) + eps)).view(-1)


def grpo_loss(logp_new, logp_old, logp_ref, rewards, group_size: int, clip_eps: float = 0.2,
              beta: float = 0.04, mask=None):
    adv = grpo_advantages(rewards, group_size)
    while adv.dim() < logp_new.dim():
        adv = adv.unsqueeze(-1)
    ratio = torch.exp(logp_new - logp_old)
    surr = torch.minimum(ratio * adv, torch.clamp(ratio, 1 - clip_eps, 1 + clip_eps) * adv)
    kl = torch.exp(logp_ref - logp_new) - (logp_ref - logp_new) - 1.0
    loss = -(surr - beta * kl)
    if mask is not None:
        return (loss * mask).sum() / mask.sum().clamp(min=1)
    return loss.mean()


def label_smoothing_ce(logits, targets, eps: float = 0.1):
    return F.cross_entropy(logits.float().reshape(-1, logits.shape[-1]), targets.reshape(-1), label_smoothing=eps)
