"""Command line: `python -m lora_kernel_b200 {train,bench,serve,export,env}`.

  train  --preset NAME | --config FILE [--steps N] [--set section.key=value ...]
         [--tp N --pp N --cp N --cp-mode ulysses|ring --zero 0-3 --fp8]
         [--lr X --micro-batch B --seq-len S --grad-accum K --metrics-file F] [--device cpu]
         (launch with torch.distributed.run for more than one GPU)
  bench  [--gpus N --steps K --warmup W]   the headline training benchmark
         [--kernels]                       kernel micro-benchmarks instead
         [--serve ...]                     serving load generator
  serve  --preset NAME [--port P] [--weights int4|int8|fp8|none] [--kv fp8|int8|bf16]
         [--replicas N --replica-policy prefix_affinity|least_loaded|round_robin]
  export --out PATH [--format gguf|hf|onnx] [--dtype bf16|f16|f32] [--checkpoint model.safetensors]
  env    versions, GPU, NVLink, extension status

Mirrors the reference's train / bench / serve verbs (README.md:107-115,
main.cpp:18 always ran the train demo).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys


def _overrides(items):
    out = {}
    for it in items or []:
        k, _, v = it.partition("=")
        try:
            v = json.loads(v)
        except json.JSONDecodeError:
            pass
        out[k] = v
    return out


# train flags that are shorthands for dotted overrides (applied after --set)
TRAIN_FLAGS = {
    "tp": "parallel.tp", "pp": "parallel.pp", "cp": "parallel.cp", "cp_mode": "parallel.cp_mode",
    "zero": "parallel.zero_stage", "fp8": "parallel.fp8", "fp8_recipe": "parallel.fp8_recipe",
    "lr": "train.lr", "micro_batch": "train.micro_batch", "seq_len": "train.seq_len",
    "grad_accum": "train.grad_accum_steps", "metrics_file": "train.metrics_file",
    "init_from": "train.init_from", "init_format": "train.init_format",
    "lora_rank": "train.lora_rank", "lora_alpha": "train.lora_alpha",
}


def train_overrides(a) -> dict:
    """--set items, then the shorthand flags that were given."""
    out = _overrides(a.set)
    for flag, key in TRAIN_FLAGS.items():
        v = getattr(a, flag, None)
        if v is not None and v is not False:
            out[key] = v
    return out


def cmd_train(a):
    from .config import load_config
    rc = load_config(a.config, a.preset, train_overrides(a))
    if a.device == "cpu":
        # fp32 on the host CPU with the oracle model (no B200 kernels)
        from .train.cpu_demo import run_cpu
        every = max(1, rc.train.log_every)
        hist = run_cpu(rc, a.steps, log=lambda r: print(json.dumps(r)) if r["step"] % every == 0 else None)
        if hist:
            tps = sorted(r["tokens_per_s"] for r in hist[1:] or hist)
            print(json.dumps({"summary": "train-cpu", "steps": len(hist), "loss_first": hist[0]["loss"],
                              "loss_last": hist[-1]["loss"], "tokens_per_s_median": tps[len(tps) // 2]}))
        return
    from .parallel.comm import init_distributed
    from .train.trainer import Trainer
    if a.checkpoint_dir:
        rc.train.checkpoint_dir = a.checkpoint_dir
    init_distributed("nccl")
    tr = Trainer(rc)
    hist = tr.fit(a.steps)
    if tr.rank == 0 and hist:
        print(json.dumps(hist[-1]))


def cmd_bench(a, rest):
    here = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    if a.kernels:
        from .utils import kernel_bench
        sys.argv = ["kernel_bench"] + rest
        kernel_bench.main()
        return
    if a.serve:
        from .serve import bench_serve
        sys.argv = ["bench_serve"] + rest
        bench_serve.main()
        return
    cmd = [sys.executable, os.path.join(here, "bench.py")] + rest
    if a.gpus > 1:
        cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={a.gpus}",
               "--master-addr", "127.0.0.1", "--master-port", "29531", os.path.join(here, "bench.py"),
               "--gpus", str(a.gpus)] + rest
    raise SystemExit(subprocess.call(cmd))


def _tokenizer(a):
    if not getattr(a, "tokenizer", None):
        return None
    from .serve.tokenizer import HFTokenizer
    return HFTokenizer(a.tokenizer)


def cmd_serve(a):
    from .config import load_config
    from .models.params import FlatParams
    from .serve.engine import LLMEngine
    from .serve.server import serve
    rc = load_config(a.config, a.preset, _overrides(a.set))
    if a.checkpoint and a.checkpoint_format == "hf":  # the model shape comes with the checkpoint
        from .utils.export import config_from_hf
        rc.model = config_from_hf(a.checkpoint)
    cfg = rc.model
    kv, weights = a.kv or rc.quant.kv_cache, a.weights or rc.quant.weights

    def read_state_dict():
        if a.checkpoint_format == "hf":
            from .utils.export import import_hf
            return import_hf(a.checkpoint, cfg, dtype=torch.bfloat16)
        from .train.checkpoint import load_model_safetensors
        from .train.crypto import key_from_env
        return load_model_safetensors(a.checkpoint, key=key_from_env())

    import torch
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        # tensor-parallel serving under torchrun: rank 0 runs the HTTP server and
        # the scheduler, every rank its weight / KV-head shard
        import torch.distributed as dist
        from .parallel.comm import init_distributed
        from .serve.tp_runner import RunnerProxy, build_tp_runner, worker_loop
        if a.checkpoint and a.checkpoint_format not in ("safetensors", "hf"):
            raise NotImplementedError("tensor-parallel serving loads model.safetensors checkpoints; "
                                      "serve GPTQ / AWQ files on one GPU or as replicas")
        rank, world, _ = init_distributed("nccl", timeout_s=3600)
        sc = rc.serve
        tp_params = None
        if a.checkpoint or a.lora:  # every rank reads the weights and keeps its shard
            from .serve.tp_runner import tp_params_from_state_dict
            if a.checkpoint:
                sd = read_state_dict()
            else:
                seeded = FlatParams(cfg, "cpu", torch.float32)
                seeded.init_(rc.train.seed, cfg.init_std)
                sd = seeded.to_reference_state_dict()
            if a.lora:  # adapters folded in before sharding
                from .models.lora import load_lora_file, merge_lora_state_dict
                sd = merge_lora_state_dict(sd, load_lora_file(a.lora, cfg, "cpu"))
            dev = torch.device("cuda", torch.cuda.current_device())
            tp_params = tp_params_from_state_dict(cfg, sd, world, rank, dev)
            del sd
        runner, ctrl = build_tp_runner(cfg, rc.train.seed, params=tp_params, weights=weights, kv_dtype=kv,
                                       group_size=rc.quant.group_size, block_size=sc.block_size,
                                       max_model_len=sc.max_model_len,
                                       max_rows=max(sc.max_num_batched_tokens, sc.max_num_seqs),
                                       cuda_graphs=sc.cuda_graphs, max_batch=sc.max_num_seqs)
        if rank != 0:
            worker_loop(runner, ctrl)
            dist.destroy_process_group()
            return
        proxy = RunnerProxy(runner, ctrl)
        eng = LLMEngine(cfg, None, sc, kv_dtype=kv, weights=weights, runner=proxy)
        try:
            serve(eng, host=a.host or sc.host, port=a.port or sc.port,
                  api_keys=tuple(sc.api_keys), rate_limit_rps=sc.rate_limit_rps,
                  max_inflight_per_client=sc.max_inflight_per_client, tokenizer=_tokenizer(a))
        finally:
            proxy.stop()
            dist.destroy_process_group()
        return
    engines = []
    n_rep = max(1, a.replicas)
    if n_rep > torch.cuda.device_count():
        raise SystemExit(f"--replicas {n_rep} but {torch.cuda.device_count()} GPUs")
    for g in range(n_rep):  # one independent engine per GPU
        dev = f"cuda:{g}"
        torch.cuda.set_device(g)
        if a.checkpoint and a.checkpoint_format in ("gptq", "awq"):
            # a 4-bit GPTQ / AWQ checkpoint of a Hugging Face Llama model
            from .quant.gptq_awq import load_gptq_awq
            params = load_gptq_awq(a.checkpoint, cfg, a.checkpoint_format, device=dev)
            weights = "int4"
        else:
            params = FlatParams(cfg, dev)
        if a.checkpoint and a.checkpoint_format in ("safetensors", "hf"):
            sd = read_state_dict()
            params.load_reference_state_dict({k: v.to(dev) for k, v in sd.items()})
        elif not a.checkpoint:
            params.init_(rc.train.seed, cfg.init_std)
        if a.lora:  # fold trained LoRA adapters into the base weights before serving
            if a.checkpoint_format in ("gptq", "awq"):
                raise NotImplementedError("--lora with a 4-bit checkpoint (merge into bf16 weights instead)")
            from .models.lora import load_lora_file
            load_lora_file(a.lora, cfg, dev).merge_into(params)
        engines.append(LLMEngine(cfg, params, rc.serve, device=dev, kv_dtype=kv, weights=weights,
                                 group_size=rc.quant.group_size))
    serve(engines[0] if n_rep == 1 else engines, host=a.host or rc.serve.host, port=a.port or rc.serve.port,
          api_keys=tuple(rc.serve.api_keys), rate_limit_rps=rc.serve.rate_limit_rps,
          replica_policy=a.replica_policy, max_inflight_per_client=rc.serve.max_inflight_per_client,
          tokenizer=_tokenizer(a))


def cmd_export(a):
    """Write a model as GGUF or Hugging Face safetensors from a checkpoint
    (model.safetensors, reference names) or from the preset's seeded weights."""
    import torch
    from .config import load_config
    from .models.params import FlatParams
    from .utils.export import export_gguf, export_hf
    rc = load_config(a.config, a.preset, _overrides(a.set))
    cfg = rc.model
    if a.checkpoint:
        from .train.checkpoint import load_model_safetensors
        from .train.crypto import key_from_env
        sd = load_model_safetensors(a.checkpoint, key=key_from_env())
    else:
        p = FlatParams(cfg, "cpu", torch.float32)
        p.init_(rc.train.seed, cfg.init_std)
        sd = p.to_reference_state_dict()
    if a.lora:  # fold trained LoRA adapters into the exported weights
        from .models.lora import load_lora_file, merge_lora_state_dict
        sd = merge_lora_state_dict(sd, load_lora_file(a.lora, cfg, "cpu"))
    if a.format == "onnx":
        from .utils.onnx_export import export_onnx
        export_onnx(sd, cfg, a.out)
        print(json.dumps({"exported": a.out, "format": "onnx", "dtype": "f32"}))
        return
    if a.format == "gguf":
        export_gguf(sd, cfg, a.out, dtype=a.dtype)
    else:
        export_hf(sd, cfg, a.out, dtype={"f32": torch.float32, "f16": torch.float16,
                                         "bf16": torch.bfloat16}[a.dtype])
    print(json.dumps({"exported": a.out, "format": a.format, "dtype": a.dtype}))


def cmd_env(_):
    from .utils.env import env_report
    print(json.dumps(env_report(), indent=1))


def main(argv=None):
    ap = argparse.ArgumentParser(prog="lora_kernel_b200")
    sub = ap.add_subparsers(dest="cmd", required=True)
    t = sub.add_parser("train")
    t.add_argument("--preset", default="cpu-demo")
    t.add_argument("--config")
    t.add_argument("--steps", type=int)
    t.add_argument("--checkpoint-dir")
    t.add_argument("--set", nargs="*")
    for n in ("tp", "pp", "cp", "zero", "micro-batch", "seq-len", "grad-accum"):
        t.add_argument(f"--{n}", type=int)
    t.add_argument("--cp-mode", choices=["ulysses", "ring"])
    t.add_argument("--lr", type=float)
    t.add_argument("--metrics-file")
    t.add_argument("--init-from", help="pretrained weights: model.safetensors or a Hugging Face directory")
    t.add_argument("--init-format", choices=["safetensors", "hf"])
    t.add_argument("--lora-rank", type=int, help="train LoRA adapters of this rank on the frozen base (one GPU)")
    t.add_argument("--lora-alpha", type=float)
    t.add_argument("--device", choices=["cuda", "cpu"], default="cuda",
                   help="cpu: fp32 training on the host with the oracle model (no GPU needed)")
    t.add_argument("--fp8", action="store_true", help="block-scaled fp8 GEMMs (tensor parallel)")
    t.add_argument("--fp8-recipe", choices=["mx", "exact"],
                   help="mx (default): power-of-two scales applied by the tensor core, e5m2 data gradients; "
                        "exact: fp32 scales, forward projections only")
    b = sub.add_parser("bench")
    b.add_argument("--gpus", type=int, default=1)
    b.add_argument("--kernels", action="store_true")
    b.add_argument("--serve", action="store_true")
    s = sub.add_parser("serve")
    s.add_argument("--preset", default="llama-8b-serve-int4")
    s.add_argument("--config")
    s.add_argument("--host")
    s.add_argument("--port", type=int)
    s.add_argument("--weights")
    s.add_argument("--replicas", type=int, default=1, help="independent engines, one per GPU")
    s.add_argument("--replica-policy", default="prefix_affinity",
                   choices=["round_robin", "least_loaded", "prefix_affinity"])
    s.add_argument("--kv")
    s.add_argument("--checkpoint")
    s.add_argument("--tokenizer", help="a Hugging Face tokenizer.json (default: bytes as token ids)")
    s.add_argument("--lora", help="LoRA adapters (lora_step_N.safetensors from train --lora-rank) merged at load")
    s.add_argument("--checkpoint-format", choices=["safetensors", "hf", "gptq", "awq"], default="safetensors",
                   help="hf: a Hugging Face Llama directory (config.json + safetensors); "
                        "gptq / awq: a 4-bit checkpoint of a Hugging Face Llama model")
    s.add_argument("--set", nargs="*")
    x = sub.add_parser("export")
    x.add_argument("--preset", default="cpu-demo")
    x.add_argument("--config")
    x.add_argument("--checkpoint", help="model.safetensors of a checkpoint (default: seeded weights)")
    x.add_argument("--format", choices=["gguf", "hf", "onnx"], default="gguf")
    x.add_argument("--dtype", choices=["f32", "f16", "bf16"], default="bf16")
    x.add_argument("--out", required=True)
    x.add_argument("--lora", help="LoRA adapters (lora_step_N.safetensors) merged into the exported weights")
    x.add_argument("--set", nargs="*")
    sub.add_parser("env")
    a, rest = ap.parse_known_args(argv)
    if a.cmd == "train":
        cmd_train(a)
    elif a.cmd == "bench":
        cmd_bench(a, rest)
    elif a.cmd == "serve":
        cmd_serve(a)
    elif a.cmd == "export":
        cmd_export(a)
    else:
        cmd_env(a)


if __name__ == "__main__":
    main()
