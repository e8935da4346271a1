"""Peer-memory collectives against NCCL: all-reduce (K12) and reduce-scatter
(K10 front half), each fused with the sum-of-squares partials of its result.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \\
        --master-port P -m lora_kernel_b200.utils.comm_bench [--sizes-mb 64,256,1024]

Device time with CUDA events, max over ranks, ranks aligned on the device before
each iteration.  Reported per size: time, bus bandwidth (all-reduce 2(N-1)/N x
bytes / t, reduce-scatter (N-1)/N x bytes / t) and the fraction of the roofline
= the bytes each GPU must move over NVLink at the measured 770 GB/s per direction.
One JSON line per (op, path, size) on rank 0.
"""
from __future__ import annotations

import argparse
import json

import torch
import torch.distributed as dist

from .tp_bench import NVLINK_GBS, _time


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--sizes-mb", default="64,256,1024")
    ap.add_argument("--iters", type=int, default=10)
    a = ap.parse_args(argv)
    from ..parallel import comm as CM
    rank, world, local = CM.init_distributed("nccl", timeout_s=300)
    dev = torch.device("cuda", local)
    pc = CM.PeerComm(dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    part = torch.zeros(1024, device=dev)
    for mb in (int(x) for x in a.sizes_mb.split(",")):
        n = (mb << 20) // 4
        buf = CM.SymBuffer(n, torch.float32, dev)
        buf.local.normal_()
        plain = torch.randn(n, device=dev)
        chunk = n // world
        dst = torch.empty(chunk, device=dev)
        results = []
        for path in (["nvls"] if buf.mc_ptr else []) + ["p2p", "nccl"]:
            if path == "nccl":
                t_ar = _time(lambda: dist.all_reduce(plain), a.iters, 3, flush)
                t_rs = _time(lambda: dist.reduce_scatter_tensor(dst, plain), a.iters, 3, flush)
            else:
                pc.nvls = path == "nvls"
                t_ar = _time(lambda: pc.allreduce_sum_(buf, n, part), a.iters, 3, flush)

                def rs():
                    pc.barrier(CM.SLOT_GRAD)
                    pc.reduce_scatter_sum(buf, rank * chunk, chunk, dst, partial=part)
                t_rs = _time(rs, a.iters, 3, flush)
            nbytes = n * 4
            for op, t, f in (("allreduce", t_ar, 2.0), ("reduce_scatter", t_rs, 1.0)):
                moved = f * (world - 1) / world * nbytes
                roof_ms = moved / (NVLINK_GBS * 1e9) * 1e3
                results.append({"op": op, "path": path, "mb": mb, "ms": round(t, 4),
                                "busbw_gbs": round(moved / t / 1e6, 1),
                                "frac_of_roofline": round(roof_ms / t, 3), "n_gpus": world})
        if rank == 0:
            for r in results:
                print(json.dumps(r), flush=True)
        del buf
        torch.cuda.synchronize()
        dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
