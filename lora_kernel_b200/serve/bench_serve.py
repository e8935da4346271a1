"""Serving benchmark: output tokens/s and time-to-first-token under Poisson load.

Workload (defaults): Llama-style 8B, INT4 group-128 weights, FP8 KV cache,
continuous batching up to 256 sequences, prompts of uniform [512, 2048]
random tokens of which 30% share a 1024-token prefix, 256 greedy output
tokens, Poisson arrivals at 20 requests/s.  Random-init weights and synthetic
token ids.

    python -m lora_kernel_b200.serve.bench_serve [--num-requests 200 --rate 20 ...]

Launched plainly it runs on one GPU.  Under torchrun with N processes it
serves with tensor parallelism N (serve.tp_runner): rank 0 runs the engine
and the clock, every rank runs its weight / KV-head shard.  Requests are
injected at their arrival times and the engine steps continuously.  Reported: output tok/s = generated tokens / (last completion -
first arrival), TTFT percentiles (arrival -> first token), inter-token latency,
request throughput and the prefix-cache hit rate.  One JSON line.
"""
from __future__ import annotations

import argparse
import json
import statistics
import time

import numpy as np
import torch


def _step_breakdown(log) -> dict:
    """Where a step's time goes: decode-only steps (time, batch) and steps with
    a prefill chunk (prefill time per token, decode part), host clock."""
    def med(x):
        return round(1e3 * statistics.median(x), 3) if x else None
    dec_only = [r for r in log if r[3] == 0 and r[4] > 0]
    mixed = [r for r in log if r[3] > 0]
    out = {"steps": len(log), "decode_only_steps": len(dec_only), "steps_with_prefill": len(mixed),
           "schedule_ms_p50": med([r[0] for r in log]),
           "decode_only_ms_p50": med([r[2] for r in dec_only]),
           "decode_only_batch_p50": statistics.median([r[4] for r in dec_only]) if dec_only else None,
           "prefill_ms_p50": med([r[1] for r in mixed]),
           "prefill_tokens_p50": statistics.median([r[3] for r in mixed]) if mixed else None,
           "prefill_us_per_token_p50": (round(1e6 * statistics.median([r[1] / r[3] for r in mixed]), 2)
                                        if mixed else None),
           "decode_in_mixed_ms_p50": med([r[2] for r in mixed if r[4] > 0])}
    busy = sum(r[0] + r[1] + r[2] for r in log)
    if busy > 0:
        out["share_schedule"] = round(sum(r[0] for r in log) / busy, 3)
        out["share_prefill"] = round(sum(r[1] for r in log) / busy, 3)
        out["share_decode"] = round(sum(r[2] for r in log) / busy, 3)
    return out


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--preset", default="llama-8b-serve-int4")
    ap.add_argument("--num-requests", type=int, default=200)
    ap.add_argument("--rate", type=float, default=20.0)
    ap.add_argument("--prompt-min", type=int, default=512)
    ap.add_argument("--prompt-max", type=int, default=2048)
    ap.add_argument("--shared-frac", type=float, default=0.3)
    ap.add_argument("--shared-len", type=int, default=1024)
    ap.add_argument("--output-len", type=int, default=256)
    ap.add_argument("--weights", default=None)
    ap.add_argument("--kv", default=None)
    ap.add_argument("--max-num-seqs", type=int, default=256)
    ap.add_argument("--max-batched-tokens", type=int, default=0,
                    help="token budget of a step (decode tokens + prefill chunk); 0 = the preset's")
    ap.add_argument("--layers", type=int, default=0, help="override (testing only)")
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args(argv)

    import os

    from ..config import get_preset
    from ..models.params import FlatParams
    from .engine import LLMEngine, SamplingParams

    rc = get_preset(a.preset)
    cfg = rc.model
    if a.layers:
        cfg.num_layers = a.layers
    sc = rc.serve
    sc.max_num_seqs = a.max_num_seqs
    if a.max_batched_tokens:
        sc.max_num_batched_tokens = a.max_batched_tokens
    sc.max_model_len = max(sc.max_model_len, a.prompt_max + a.output_len + 16)
    weights = a.weights or rc.quant.weights
    kv = a.kv or rc.quant.kv_cache
    tp = int(os.environ.get("WORLD_SIZE", "1"))
    proxy = None
    if tp > 1:
        from ..parallel.comm import init_distributed
        from .tp_runner import RunnerProxy, build_tp_runner, worker_loop
        rank, _, _ = init_distributed("nccl", timeout_s=600)
        runner, ctrl = build_tp_runner(cfg, a.seed, weights=weights, kv_dtype=kv,
                                       group_size=rc.quant.group_size, block_size=sc.block_size,
                                       max_model_len=sc.max_model_len,
                                       max_rows=max(sc.max_num_batched_tokens, sc.max_num_seqs),
                                       max_batch=sc.max_num_seqs)
        torch.cuda.synchronize()
        if rank != 0:
            worker_loop(runner, ctrl)
            torch.cuda.synchronize()
            torch.distributed.barrier()
            torch.distributed.destroy_process_group()
            return None
        proxy = RunnerProxy(runner, ctrl)
        eng = LLMEngine(cfg, None, sc, kv_dtype=kv, weights=weights, runner=proxy)
    else:
        params = FlatParams(cfg, "cuda")
        params.init_(a.seed, cfg.init_std)
        eng = LLMEngine(cfg, params, sc, kv_dtype=kv, weights=weights, group_size=rc.quant.group_size)
        del params
    torch.cuda.synchronize()

    rng = np.random.default_rng(a.seed)
    shared = rng.integers(0, cfg.vocab_size, a.shared_len).tolist()
    prompts = []
    for _ in range(a.num_requests):
        n = int(rng.integers(a.prompt_min, a.prompt_max + 1))
        if rng.random() < a.shared_frac and n > a.shared_len:
            p = shared + rng.integers(0, cfg.vocab_size, n - a.shared_len).tolist()
        else:
            p = rng.integers(0, cfg.vocab_size, n).tolist()
        prompts.append(p)
    gaps = rng.exponential(1.0 / a.rate, a.num_requests)
    arrivals = np.cumsum(gaps) - gaps[0]
    sp = SamplingParams(max_tokens=a.output_len, temperature=0.0)

    # warm-up: one short request through prefill and decode
    eng.generate([prompts[0][:64]], SamplingParams(max_tokens=4))
    torch.cuda.synchronize()
    eng.finished.clear()

    eng.step_log = []
    t0 = time.perf_counter()
    nxt = 0
    ids = []
    while nxt < a.num_requests or eng.has_work():
        now = time.perf_counter() - t0
        while nxt < a.num_requests and arrivals[nxt] <= now:
            ids.append(eng.add_request(prompts[nxt], sp, arrival=t0 + float(arrivals[nxt])))
            nxt += 1
        if eng.has_work():
            eng.step()
        elif nxt < a.num_requests:
            time.sleep(max(0.0, arrivals[nxt] - (time.perf_counter() - t0)))
    torch.cuda.synchronize()
    t_end = time.perf_counter()
    reqs = [eng.finished[i] for i in ids]
    out_tokens = sum(len(r.output) for r in reqs)
    last = max(r.token_times[-1] for r in reqs)
    span = last - t0
    ttft = sorted(r.first_token_time - r.arrival for r in reqs)
    itl = [b - a_ for r in reqs for a_, b in zip(r.token_times, r.token_times[1:])]
    res = {
        "metric": "serve output tok/s + p50 TTFT",
        "value": round(out_tokens / span, 1),
        "unit": "output tokens/s",
        "ttft_p50_ms": round(1e3 * statistics.median(ttft), 2),
        "ttft_p90_ms": round(1e3 * ttft[int(0.9 * (len(ttft) - 1))], 2),
        "itl_p50_ms": round(1e3 * statistics.median(itl), 2) if itl else None,
        "requests_per_s": round(len(reqs) / span, 2),
        "num_requests": a.num_requests, "rate": a.rate, "output_len": a.output_len,
        "prefix_cache_hit_rate": round(eng.blocks.stats.hit_rate, 3),
        "preemptions": eng.stats["preemptions"],
        "n_gpus": tp,
        "config": {"model": f"Llama-style 8B ({cfg.num_layers} layers)", "weights": weights, "kv_cache": kv,
                   "max_num_seqs": sc.max_num_seqs, "prompts": f"uniform [{a.prompt_min},{a.prompt_max}]",
                   "shared_prefix": f"{a.shared_frac:.0%} x {a.shared_len}", "parallelism": f"tp{tp}"},
        "data": "synthetic (random token ids, random-init weights)",
        "wall_s": round(t_end - t0, 2),
        "kv_blocks": eng.runner.num_blocks, "weight_gb": round(eng.runner.weight_bytes() / 1e9, 2),
        "max_batched_tokens": sc.max_num_batched_tokens,
        "step_breakdown": _step_breakdown(eng.step_log),
    }
    print(json.dumps(res), flush=True)
    if proxy is not None:
        proxy.stop()
        torch.cuda.synchronize()
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    return res


if __name__ == "__main__":
    main()
