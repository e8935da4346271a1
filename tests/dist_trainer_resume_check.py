"""Launched by tests/test_pp_multigpu.py / test_cp_multigpu.py under torchrun:
Trainer.fit under pipeline or context parallelism resumes from its checkpoint
with the same losses as an uninterrupted run."""
import json
import os
import sys

import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from lora_kernel_b200.config import get_preset  # noqa: E402
from lora_kernel_b200.parallel.comm import init_distributed  # noqa: E402
from lora_kernel_b200.train.trainer import Trainer  # noqa: E402


def _rc(kind, ck, steps):
    rc = get_preset("tiny")
    rc.train.total_steps = steps
    rc.train.log_every = 1
    rc.train.lr = 1e-3
    rc.train.grad_accum_steps = 2
    rc.train.checkpoint_dir = ck
    setattr(rc.parallel, kind, dist.get_world_size())
    return rc


def main():
    kind, root = sys.argv[1], sys.argv[2]
    rank, world, _ = init_distributed("nccl", timeout_s=120)
    os.environ["LORAK_HEARTBEAT"] = "0"
    full = Trainer(_rc(kind, "", 4)).fit()
    ck = os.path.join(root, "ck")
    Trainer(_rc(kind, ck, 2)).fit()
    resumed = Trainer(_rc(kind, ck, 4)).fit()
    if rank == 0:
        with open(os.environ["LK_OUT"], "w") as f:
            json.dump({"full": [h["loss"] for h in full], "resumed": [h["loss"] for h in resumed],
                       "steps": [h["step"] for h in resumed],
                       "saved": sorted(os.listdir(ck))}, f)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
