"""Launched by tests/test_tp_serve_multigpu.py under torchrun: tensor-parallel
serving (sharded weights and KV heads, fused all-reduce + RMSNorm over peer
memory, vocabulary-parallel sampling) must generate what the single-GPU
engine generates with the same weights."""
import json
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from lora_kernel_b200._ext import check_status  # noqa: E402
from lora_kernel_b200.config import ServeConfig, TransformerConfig  # noqa: E402
from lora_kernel_b200.parallel.comm import init_distributed  # noqa: E402
from lora_kernel_b200.serve.engine import LLMEngine, SamplingParams  # noqa: E402
from lora_kernel_b200.serve.tp_runner import RunnerProxy, build_tp_runner, worker_loop  # noqa: E402


def main():
    weights = sys.argv[1]
    rank, world, local = init_distributed("nccl", timeout_s=120)
    cfg = TransformerConfig(hidden_dim=256, num_heads=4, num_kv_heads=2, head_dim=64, ff_dim=512,
                            vocab_size=1024, num_layers=2, max_seq_len=512, init_std=0.05)
    sc = ServeConfig(max_num_seqs=8, max_num_batched_tokens=512, num_kv_blocks=128, max_model_len=512)
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (17, 40, 64, 5)]
    sp = SamplingParams(max_tokens=12, temperature=0.0)
    runner, ctrl = build_tp_runner(cfg, 7, weights=weights, kv_dtype="bf16", num_blocks=128,
                                   max_model_len=512, max_rows=512, max_batch=sc.max_num_seqs)
    if rank != 0:
        worker_loop(runner, ctrl)
    else:
        eng = LLMEngine(cfg, None, sc, kv_dtype="bf16", weights=weights, runner=RunnerProxy(runner, ctrl))
        got = eng.generate(prompts, sp)
        # sampled (temperature > 0) run: every rank must agree, so just check it completes
        got_t = eng.generate(prompts[:2], SamplingParams(max_tokens=6, temperature=0.8))
        eng.runner.stop()
        from lora_kernel_b200.models.params import FlatParams
        full = FlatParams(cfg, "cuda")
        full.init_(7, cfg.init_std)
        ref_eng = LLMEngine(cfg, full, sc, kv_dtype="bf16", weights=weights)
        want = ref_eng.generate(prompts, sp)
        same = sum(a == b for x, y in zip(got, want) for a, b in zip(x, y))
        total = sum(len(x) for x in want)
        first = all(x[0] == y[0] for x, y in zip(got, want))
        with open(os.environ["LK_OUT"], "w") as f:
            json.dump({"match": same / total, "first": first, "got": got, "want": want,
                       "sampled_len": [len(x) for x in got_t]}, f)
    torch.cuda.synchronize()
    check_status()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
