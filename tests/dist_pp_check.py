"""Launched by tests/test_pp_multigpu.py under torchrun: 1F1B pipeline
parallelism (one stage per rank) must match the single-GPU pipeline with the
same gradient accumulation."""
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from lora_kernel_b200._ext import check_status  # noqa: E402
from lora_kernel_b200.parallel.comm import init_distributed  # noqa: E402
from lora_kernel_b200.parallel.pp import PipelineTrainer  # noqa: E402

from test_pp_multigpu import CFG, TC, batches  # noqa: E402


def main():
    rank, world, local = init_distributed("nccl", timeout_s=120)
    tr = PipelineTrainer(CFG, TC, device="cuda")
    losses = []
    for step in batches():
        tr.loss_acc.zero_()
        for ids in step:
            d = ids.cuda()
            tr.micro_step_async(d[:, :-1].contiguous(), d[:, 1:].contiguous())
        s, n = tr.loss_acc.tolist()
        losses.append(s / n)
    torch.cuda.synchronize()
    check_status()
    full = tr.full_state_dict()
    if rank == 0:
        torch.save({"full": full, "losses": losses, "parts": [list(r) for r in tr.parts]}, os.environ["LK_OUT"])
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
