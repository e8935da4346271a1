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


def cross_entropy_chunk_stats(logits: torch.Tensor, targets: torch.Tensor, v0: int, v_total: int,
                              stats: torch.Tensor, dummy_acc: torch.Tensor, stat_ptrs: torch.Tensor) -> None:
    """Vocabulary chunk [v0, v0 + logits.shape[1]) of a row-wise cross-entropy:
    per-row {max, sum exp, sum z, z[target] if in the chunk} into stats [T, 4]."""
    require_device(logits)
    C().cross_entropy_vp(logits, targets.reshape(-1), dummy_acc, None, 1.0, 0.0, 0.0, -100, False, int(v0),
                         int(v_total), stats, stat_ptrs, 1)


def cross_entropy_chunk_grad(logits: torch.Tensor, targets: torch.Tensor, v0: int, v_total: int,
                             stats: torch.Tensor, stat_ptrs: torch.Tensor, loss_acc: torch.Tensor, *,
                             scale: Optional[torch.Tensor] = None, scale_mul: float = 1.0,
                             smoothing: float = 0.0, z_loss: float = 0.0, ignore_index: int = -100) -> None:
    """Combine every chunk's statistics (stat_ptrs: device table of the chunks'
    stats buffers) into the row loss, added to loss_acc, and overwrite this
    chunk's logits with its gradient slice (times *scale x scale_mul)."""
    require_device(logits)
    C().cross_entropy_vp(logits, targets.reshape(-1), loss_acc, scale, float(scale_mul), float(smoothing),
                         float(z_loss), int(ignore_index), True, int(v0), int(v_total), stats, stat_ptrs, 2)
