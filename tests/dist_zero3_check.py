"""Launched by tests/test_zero_multigpu.py under torchrun: ZeRO-3 on N GPUs
must match the single-GPU pipeline on the same global batch."""
import json
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from lora_kernel_b200._ext import check_status  # noqa: E402
from lora_kernel_b200.config import TrainConfig, TransformerConfig  # noqa: E402
from lora_kernel_b200.parallel.comm import init_distributed  # noqa: E402
from lora_kernel_b200.parallel.zero import Zero3Trainer  # noqa: E402


def main():
    mode = sys.argv[1]
    rank, world, local = init_distributed("nccl", timeout_s=120)
    cfg = TransformerConfig(hidden_dim=256, num_heads=4, num_kv_heads=2, head_dim=64, ff_dim=512,
                            vocab_size=512, num_layers=3, max_seq_len=256)
    tc = TrainConfig(lr=1e-3, weight_decay=0.1, dynamic_loss_scale=True, init_loss_scale=1024.0,
                     micro_batch=2, seq_len=128, seed=5)
    parts = mode.split("-")
    fused = "fused" in parts  # K17: the group gather inside the first consuming GEMM
    wire = "fp32" if "fp32" in parts else "bf16"  # gradients on the wire
    accum = 2 if "accum2" in parts else 1
    tc.grad_accum_steps = accum
    tr = Zero3Trainer(cfg, tc, device="cuda", comm=parts[0], fuse_gather=fused, grad_wire=wire)
    g = torch.Generator().manual_seed(0)
    batches = [torch.randint(0, cfg.vocab_size, (2 * world, 129), generator=g) for _ in range(3 * accum)]
    losses = []
    for b in batches:
        mine = b[2 * rank:2 * rank + 2].cuda()
        losses.append(tr.train_step(mine[:, :-1], mine[:, 1:]))
    torch.cuda.synchronize()
    check_status()
    full = tr.full_params().float().cpu()
    t = torch.tensor(losses, device="cuda")
    dist.all_reduce(t)
    if rank == 0:
        torch.save({"full": full, "losses": (t / world).tolist(),
                    "norm": float(tr.opt.state[6])}, os.environ["LK_OUT"])
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
