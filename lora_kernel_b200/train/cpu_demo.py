"""fp32 training on the host CPU, for machines without a B200.

The reference's only command-line behaviour is a CPU training demo
(main.cpp:60-72); the `cpu-demo` preset is that kind of workload at a fixed
size: Llama-style 4 layers, d 256, 4 heads x 64, ffn 688, vocab 1024, seq 128,
batch 8, fp32, AdamW.  This
module runs that workload on the CPU with the framework's fp32 oracle model
(oracle/llama_ref.py: eager PyTorch, autograd) and torch's AdamW with global-norm
clipping, so `train --device cpu` works where there is no GPU.  It is not the
B200 path (that is train/pipeline.py and the sm_100a kernels) and it computes
the same standard Llama decoder: pre-norm RMSNorm, RoPE per head, GQA attention
with an output projection, SwiGLU with ff_dim, final norm.
"""
from __future__ import annotations

import time
from typing import Callable, List, Optional

import torch

from ..config import RunConfig


def run_cpu(rc: RunConfig, steps: Optional[int] = None, log: Optional[Callable[[dict], None]] = None,
            threads: int = 0) -> List[dict]:
    """Train rc.model on the CPU in fp32 for `steps` (default
    rc.train.total_steps) optimizer steps; returns one record per step
    (step, loss, lr, tokens_per_s) and calls `log` with each."""
    from ..models.params import FlatParams
    from ..oracle.llama_ref import OracleTrainer, loss_fn
    from .schedules import lr_at
    if threads:
        torch.set_num_threads(threads)
    cfg, tc = rc.model, rc.train
    total = steps if steps is not None else tc.total_steps
    params = FlatParams(cfg, "cpu", torch.float32)
    params.init_(tc.seed, cfg.init_std)
    if tc.init_from:  # fine-tune pretrained weights
        if tc.init_format == "hf":
            from ..utils.export import import_hf
            sd = import_hf(tc.init_from, cfg)
        else:
            from .checkpoint import load_model_safetensors
            from .crypto import key_from_env
            sd = load_model_safetensors(tc.init_from, key=key_from_env())
        params.load_reference_state_dict({k: v.float() for k, v in sd.items()})
    decay = {k: (v.dim() > 1) or tc.decay_norms for k, v in params.views.items()}
    tr = OracleTrainer(dict(params.views), cfg, lr=tc.lr, wd=tc.weight_decay, betas=(tc.beta1, tc.beta2),
                       eps=tc.eps, max_norm=tc.max_grad_norm, decay=decay)
    lora = None
    if tc.lora_rank > 0:
        # LoRA: the base stays frozen, only the adapters (the same tensors and file format as the
        # GPU path, models/lora.py) are trained; W_eff = W + (alpha / r) B A for every target
        from ..models.lora import LoRAAdapters, LoRAConfig
        lora = LoRAAdapters(cfg, LoRAConfig(rank=tc.lora_rank, alpha=tc.lora_alpha, init_seed=tc.seed,
                                            targets=tuple(t for t in tc.lora_targets.split(",") if t)),
                            "cpu", torch.float32)
        lora.flat.requires_grad_(True)
        # views taken after requires_grad so that gradients reach the flat buffer
        lv_ = {nm: lora.flat[o:o + sh[0] * sh[1]].view(sh) for nm, sh, o in lora.specs}
        for v in tr.params.values():
            v.requires_grad_(False)
        tr.opt = torch.optim.AdamW([lora.flat], lr=tc.lr, betas=(tc.beta1, tc.beta2), eps=tc.eps,
                                   weight_decay=tc.weight_decay)

    def weights():
        if lora is None:
            return tr.params
        s = lora.lc.scale
        return {k: (v + s * (lv_[k + ".B"] @ lv_[k + ".A"]) if k + ".A" in lv_ else v)
                for k, v in tr.params.items()}
    g = torch.Generator().manual_seed(tc.seed)
    B, S = tc.micro_batch, tc.seq_len
    fixed = torch.randint(0, cfg.vocab_size, (B, S + 1), generator=g) if tc.fixed_batch else None
    out: List[dict] = []
    for step in range(total):
        lr = lr_at(step, tc.lr, tc.schedule, tc.warmup_steps, total, tc.min_lr_ratio)
        for grp in tr.opt.param_groups:
            grp["lr"] = lr
        t0 = time.perf_counter()
        loss = 0.0
        tr.opt.zero_grad(set_to_none=True)
        for _ in range(tc.grad_accum_steps):
            ids = fixed if fixed is not None else torch.randint(0, cfg.vocab_size, (B, S + 1), generator=g)
            lv = loss_fn(weights(), cfg, ids[:, :-1], ids[:, 1:]) / tc.grad_accum_steps
            lv.backward()
            loss += float(lv.detach())
        if tr.max_norm > 0:
            trained = [lora.flat] if lora is not None else list(tr.params.values())
            torch.nn.utils.clip_grad_norm_(trained, tr.max_norm)
        tr.opt.step()
        dt = time.perf_counter() - t0
        rec = {"step": step + 1, "loss": loss, "lr": lr,
               "tokens_per_s": B * S * tc.grad_accum_steps / dt, "device": "cpu", "dtype": "float32"}
        out.append(rec)
        if log is not None:
            log(rec)
    if lora is not None and tc.checkpoint_dir:
        import os

        from ..models.lora import save_lora_file
        os.makedirs(tc.checkpoint_dir, exist_ok=True)
        save_lora_file(lora, os.path.join(tc.checkpoint_dir, f"lora_step_{total}.safetensors"), total)
    return out
