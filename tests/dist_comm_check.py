"""Launched by tests/test_comm_multigpu.py under torchrun: the peer-memory
collectives (one-shot P2P and NVLS multimem) against NCCL."""
import json
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from lora_kernel_b200._ext import check_status  # noqa: E402
from lora_kernel_b200.parallel import comm as CM  # noqa: E402


def main():
    rank, world, local = CM.init_distributed("nccl", timeout_s=120)
    dev = torch.device("cuda", local)
    pc = CM.PeerComm(dev)
    n = 1 << 20
    buf = CM.SymBuffer(n, torch.float32, dev)
    res = {"rank": rank, "nvls_available": bool(buf.mc_ptr)}
    g = torch.Generator(device=dev).manual_seed(rank)
    for use_nvls in ([False, True] if buf.mc_ptr else [False]):
        pc.nvls = use_nvls
        tag = "nvls" if use_nvls else "p2p"
        x = torch.randn(n, device=dev, generator=g)
        want = x.clone()
        dist.all_reduce(want)
        # all-reduce of a sub-range (offset 4096) with Σg² partials
        buf.local.copy_(x)
        part = torch.zeros(64, device=dev)
        off, m = 4096, n - 8192
        pc.allreduce_sum_(buf, m, part, off=off)
        torch.cuda.synchronize()
        got = buf.local[off:off + m]
        res[f"{tag}.ar_err"] = ((got - want[off:off + m]).norm() / want[off:off + m].norm()).item()
        res[f"{tag}.ar_untouched"] = bool(torch.equal(buf.local[:off], x[:off]))
        tot = part.sum().clone()
        dist.all_reduce(tot)
        res[f"{tag}.ar_sumsq_err"] = abs(tot.item() - want[off:off + m].pow(2).sum().item()) / want[off:off + m].pow(2).sum().item()
        # reduce-scatter of this rank's chunk
        buf.local.copy_(x)
        pc.barrier(CM.SLOT_GRAD)
        chunk = n // world
        dst = torch.zeros(chunk, device=dev)
        pc.reduce_scatter_sum(buf, rank * chunk, chunk, dst)
        pc.barrier(CM.SLOT_GRAD)
        torch.cuda.synchronize()
        w = want[rank * chunk:(rank + 1) * chunk]
        res[f"{tag}.rs_err"] = ((dst - w).norm() / w.norm()).item()
    check_status()
    with open(f"{os.environ['LK_OUT']}.{rank}", "w") as f:
        json.dump(res, f)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
