"""Headline benchmark: Llama-style 1.1B training throughput (tokens/s, whole job).

Workload (fixed): 22 layers, d_model 2048, 32 query / 4 KV heads (head_dim 64),
SwiGLU FFN 5632, vocab 32000, sequence 2048, micro-batch 4 per GPU, bf16
compute with fp32 master weights, AdamW + dynamic loss scaling + global-norm
clip 1.0, ZeRO-3 parameter / gradient / optimizer sharding across the GPUs,
uniform-random token ids, N(0, 0.02) random-init weights.  Weak scaling: the
per-GPU work is fixed as the GPU count grows.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl lk|reference|torch]
                    [--comm p2p|nccl] [--torch-precision mixed|bf16] [--no-phases]

Arms: `--impl lk` (default) is this framework: hand-written sm_100a kernels,
ZeRO-3 over peer memory (`--comm p2p`) or the same ZeRO-3 schedule with NCCL
collectives (`--comm nccl`); `--impl torch` is the same workload on library
code (cuBLAS, SDPA, fused AdamW, FSDP2 over NCCL); `--impl reference` reports
why the reference cannot run this workload.

For N > 1 launch one process per GPU:
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N \\
        --master-addr 127.0.0.1 --master-port P bench.py --gpus N

Timing: W untimed warm-up steps, then exactly K steps between a barrier +
torch.cuda.synchronize() on each side, timed with CUDA events on the training
stream; the reported time is the max over ranks.  Every step streams several
GB of weights and activations (far larger than the 126 MB L2), so no explicit
L2 flush is added.  SM clocks and throttle reasons are sampled with nvidia-smi
during the timed region.  A second, end-to-end pass times K more steps through
the public API: the native token loader fills page-locked host slots on its
worker threads, each step copies its ids and targets to the device in one
transfer, and the loss is read back to the host every step.  A third, short
pass (not part of either number) records CUDA events around every phase of
the step on each stream and reports the per-step device time of each phase,
max over ranks (`phases_ms`).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

METRIC = "train tokens/sec (max over ranks) at 1/2/4/8 B200; serve output tok/s + p50 TTFT"
MODEL_NAME = "Llama-style 1.1B (22 layers, d 2048, 32 heads/4 KV heads, ffn 5632, vocab 32000)"
PUBLISHED_VALUE = None  # the reference publishes no GPU number for this workload


class ClockSampler:
    """nvidia-smi sampling of SM clocks / throttle reasons in the background."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.rows = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return

        def reader():
            for line in self.proc.stdout:
                self.rows.append([x.strip() for x in line.split(",")])

        self.thread = threading.Thread(target=reader, daemon=True)
        self.thread.start()

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
                for nm, v in zip(names, r[5:9]):
                    if v.strip().lower() == "active":
                        reasons.add(nm)
            except (ValueError, IndexError):
                continue
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}; launch with torch.distributed.run")
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                             device_id=torch.device("cuda", local))
    return rank, world, local


def barrier(world):
    if world > 1:
        torch.distributed.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def build_trainer(impl: str, cfg, tc, rank: int, world: int, fuse_gather: bool = False, comm: str = "p2p",
                  torch_precision: str = "mixed", grad_wire: str = "bf16"):
    if impl == "lk":
        if world == 1:
            from lora_kernel_b200.train.pipeline import Transformer, TrainingPipeline
            model = Transformer(cfg, "cuda", seed=tc.seed)
            return TrainingPipeline(model, tc.lr, tc.weight_decay, tc.max_grad_norm, train_cfg=tc)
        from lora_kernel_b200.parallel.zero import Zero3Trainer
        return Zero3Trainer(cfg, tc, device="cuda", comm=comm, fuse_gather=fuse_gather, grad_wire=grad_wire)
    if impl == "torch":
        from lora_kernel_b200.models.torch_llama import TorchBaselineTrainer
        return TorchBaselineTrainer(cfg, tc, device="cuda", world=world, precision=torch_precision)
    raise ValueError(impl)


def measured_peaks():
    try:
        with open(os.path.join(HERE, "MEASURED_PEAKS.json")) as f:
            return json.load(f)
    except (OSError, ValueError):
        return {}


def launches():
    try:
        from lora_kernel_b200._ext import C
        return C().launch_count()
    except Exception:
        return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="lk", choices=["lk", "reference", "torch"])
    ap.add_argument("--preset", default="llama-1.1b-zero3",
                    help="workload: llama-1.1b-zero3 (the headline) or llama-8b-fsdp-dp8 (8B ZeRO-3, "
                         "accumulation 8, EMA); a timed step is one optimizer step")
    ap.add_argument("--micro-batch", type=int, default=0, help="0 = the preset's")
    ap.add_argument("--seq", type=int, default=0, help="0 = the preset's")
    ap.add_argument("--layers", type=int, default=0, help="override (testing only; invalid for the headline)")
    ap.add_argument("--fuse-gather", action="store_true",
                    help="ZeRO-3: gather each layer inside its first GEMM instead of prefetching it")
    ap.add_argument("--comm", default="p2p", choices=["p2p", "nccl"],
                    help="ZeRO-3 collectives: peer-memory kernels (p2p) or NCCL, same schedule")
    ap.add_argument("--grad-wire", default="bf16", choices=["bf16", "fp32"],
                    help="ZeRO-3: gradients reduce-scattered as bf16 every micro-batch (sharded fp32 "
                         "accumulation) or from a full fp32 buffer")
    ap.add_argument("--torch-precision", default="mixed", choices=["mixed", "bf16"],
                    help="--impl torch: fp32 master weights + bf16 compute (mixed), or bf16 weights")
    ap.add_argument("--no-phases", action="store_true", help="skip the per-phase timing pass")
    ap.add_argument("--phase-steps", type=int, default=3)
    args = ap.parse_args()

    if args.impl == "reference":
        print(json.dumps({
            "impl": "reference",
            "unavailable": ("the reference (sudish80/Lora-Kernel-) is a header-only C++ CPU engine with "
                            "no build system (no setup.py/pyproject.toml/CMakeLists.txt; pip reports "
                            "'not installable'), its CUDA/NCCL code is never compiled and does not "
                            "compile, so it cannot run Llama-1.1B ZeRO-3 training on B200")}))
        return

    from lora_kernel_b200.config import get_preset
    rc = get_preset(args.preset)
    cfg, tc = rc.model, rc.train
    tc.micro_batch = args.micro_batch or tc.micro_batch
    tc.seq_len = args.seq or tc.seq_len
    accum = max(1, tc.grad_accum_steps)
    model_name = MODEL_NAME if args.preset == "llama-1.1b-zero3" else (
        f"Llama-style {cfg.num_parameters() / 1e9:.1f}B ({cfg.num_layers} layers, d {cfg.hidden_dim}, "
        f"{cfg.num_heads} heads/{cfg.num_kv_heads} KV heads, ffn {cfg.ff_dim}, vocab {cfg.vocab_size})")
    if args.layers:
        cfg.num_layers = args.layers
    W = max(3, args.warmup)
    K = max(1, args.steps)

    rank, world, local = dist_setup(args.gpus)
    torch.manual_seed(tc.seed + rank)
    trainer = build_trainer(args.impl, cfg, tc, rank, world, fuse_gather=args.fuse_gather, comm=args.comm,
                            torch_precision=args.torch_precision, grad_wire=args.grad_wire)
    B, S, V = tc.micro_batch, tc.seq_len, cfg.vocab_size

    # synthetic data: uniform token ids from a seeded generator, next-token targets
    g = torch.Generator(device="cpu").manual_seed(tc.seed * 1000 + rank)
    n_batches = 4
    host_ids = [torch.randint(0, V, (B, S + 1), generator=g).pin_memory() for _ in range(n_batches)]
    dev_ids = [h.to("cuda") for h in host_ids]
    dev_batches = [(d[:, :-1].contiguous(), d[:, 1:].contiguous()) for d in dev_ids]

    # ---- warm-up (optimizer steps of `accum` micro-batches each)
    for i in range(W * accum):
        x, y = dev_batches[i % n_batches]
        trainer.micro_step_async(x, y)
    torch.cuda.synchronize()
    barrier(world)

    # ---- device-timed region
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    l0 = launches()
    barrier(world)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(K * accum):
        x, y = dev_batches[i % n_batches]
        trainer.micro_step_async(x, y)
    end.record()
    torch.cuda.synchronize()
    barrier(world)
    l1 = launches()
    clocks = sampler.stop()
    ms = start.elapsed_time(end) / K
    ms = max_over_ranks(ms, world)
    tokens_per_step = B * S * world * accum
    value = tokens_per_step / (ms / 1e3)

    # ---- end-to-end through the public API: the native loader fills page-locked
    # slots on host threads, one H2D copy per step moves ids|targets, the loss
    # is read back to the host every step
    from lora_kernel_b200.utils.data import NativeTokens
    loader = NativeTokens(V, B, S, seed=tc.seed, rank=rank, world=world, depth=6)
    h2d = 0
    d2h = 0
    losses = []
    loader.next_device("cuda")  # first fill outside the timed loop
    barrier(world)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(K):
        for _ in range(accum - 1):
            x, y = loader.next_device("cuda")
            h2d += loader.bytes_per_batch()
            trainer.micro_step_async(x, y)
        x, y = loader.next_device("cuda")
        h2d += loader.bytes_per_batch()
        loss = trainer.train_step(x, y)  # last micro-batch of the step; its loss read back
        d2h += 8
        losses.append(loss)
    torch.cuda.synchronize()
    e2e_s = (time.perf_counter() - t0) / K
    e2e_s = max_over_ranks(e2e_s, world)
    e2e_value = tokens_per_step / e2e_s

    # ---- per-phase device times (separate short pass; every rank takes part)
    phases = None
    if not args.no_phases:
        from lora_kernel_b200.utils.profiler import PhaseTimer, collecting
        timer = PhaseTimer()
        P = max(1, args.phase_steps)
        barrier(world)
        with collecting(timer):
            for i in range(P * accum):
                x, y = dev_batches[i % n_batches]
                trainer.micro_step_async(x, y)
        phases = timer.per_step_ms(P)

    n_launch = int(l1 - l0)
    peaks = measured_peaks()
    model_tflops = value / world * cfg.flops_per_token(S) / 1e12
    if args.impl == "lk":
        parallelism = f"zero3-dp{world}" + ("" if world == 1 else f" ({args.comm}, {args.grad_wire} grads)")
    else:
        parallelism = f"fsdp2-dp{world}" if world > 1 else "dp1"
    out = {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": K,
        "warmup": W,
        "ms_per_step": round(ms, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": (round(value / PUBLISHED_VALUE, 3) if PUBLISHED_VALUE else None),
        "dtype": "bf16",
        "data": "synthetic (uniform random token ids from the native loader, N(0,0.02) random-init weights)",
        "impl": args.impl,
        "config": {"model": model_name, "global_batch": B * world * accum, "micro_batch_per_gpu": B,
                   "seq_len": S, "parallelism": parallelism,
                   "layers": cfg.num_layers,
                   "optimizer": "AdamW+dynamic loss scale+global-norm clip 1.0"
                                + (f"+EMA {tc.ema_decay}" if tc.ema_decay else ""),
                   "grad_accum": accum,
                   "l2": "inputs larger than L2 (each step streams GBs of weights/activations)"},
        "clocks": clocks,
        "e2e": {"value": round(e2e_value, 1), "unit": "tokens/s", "h2d_bytes_per_step": h2d // K,
                "d2h_bytes_per_step": d2h // K},
        "gpu_launches": n_launch,
        "loss_last": round(losses[-1], 4) if losses else None,
        "mfu": round(model_tflops / 2250.0, 4),
        "model_tflops_per_gpu": round(model_tflops, 1),
    }
    if peaks.get("bf16_tflops_sustained"):
        out["frac_of_measured_sustained_bf16"] = round(model_tflops / peaks["bf16_tflops_sustained"], 4)
    if args.impl == "torch":
        out["torch_precision"] = args.torch_precision
    if hasattr(trainer, "grad_memory_bytes"):
        out["grad_wire"] = args.grad_wire
        out["grad_bytes_per_rank"] = int(trainer.grad_memory_bytes())
    if phases is not None:
        out["phases_ms"] = phases
        out["phases_note"] = ("separate pass of %d steps: CUDA events around each phase on the stream it runs "
                              "on, per-step mean, max over ranks; comm.* run on a side stream and overlap "
                              "compute, wait.* is the main stream waiting on them" % max(1, args.phase_steps))
    if rank == 0:
        print(json.dumps(out), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
