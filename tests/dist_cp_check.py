"""Launched by tests/test_cp_multigpu.py under torchrun: context parallelism
(Ulysses attention, sequence chunks per rank, data-parallel gradient sum)
must match the single-GPU pipeline on the same full micro-batches.
LK_CP_MODE selects Ulysses (default) or ring attention."""
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from lora_kernel_b200._ext import check_status  # noqa: E402
from lora_kernel_b200.parallel.comm import init_distributed  # noqa: E402
from lora_kernel_b200.parallel.cp import ContextParallelTrainer  # noqa: E402

from test_cp_multigpu import CFG, TC, batches  # noqa: E402


def main():
    rank, world, local = init_distributed("nccl", timeout_s=120)
    tr = ContextParallelTrainer(CFG, TC, zero_stage=0, device="cuda", mode=os.environ.get("LK_CP_MODE", "ulysses"))
    losses = [tr.train_step(b[:, :-1].cuda(), b[:, 1:].cuda()) for b in batches()]
    torch.cuda.synchronize()
    check_status()
    full = tr.full_params().float().cpu()
    ref = tr.full_params().clone()
    dist.broadcast(ref, 0)
    same = bool(torch.equal(ref, tr.full_params()))
    if rank == 0:
        torch.save({"full": full, "losses": losses, "same": same}, os.environ["LK_OUT"])
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
