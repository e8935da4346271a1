"""K9: fused softmax cross-entropy (loss and in-place bf16 gradient)."""
from __future__ import annotations

from typing import Optional

import torch

from .._ext import C, require_device


def cross_entropy_(logits: torch.Tensor, targets: torch.Tensor, loss_acc: torch.Tensor, *,
                   scale: Optional[torch.Tensor] = None, scale_mul: float = 1.0,
                   smoothing: float = 0.0, z_loss: float = 0.0, ignore_index: int = -100,
                   write_grad: bool = True, row_loss: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Accumulate (sum of losses, count) into loss_acc[0:2]; when write_grad,
    overwrite logits with d loss_sum / d logits * (*scale) * scale_mul."""
    require_device(logits)
    C().cross_entropy(logits, targets.reshape(-1), loss_acc, row_loss, scale, float(scale_mul),
                      float(smoothing), float(z_loss), int(ignore_index), bool(write_grad))
    return logits
