"""`Trainer.fit()`: the training loop around the B200 engine.

One process per GPU.  World size 1 runs the single-GPU TrainingPipeline; more
ranks run ZeRO-3 (`parallel.zero.Zero3Trainer`) over peer memory.  The loop:
learning-rate schedule -> micro-batches (device-resident gradient
accumulation) -> device-side optimizer step; every `log_every` steps one host
read of loss / grad-norm / loss scale; periodic and final checkpoints
(resumable, reshardable); SIGTERM / SIGINT finish the current step, write a
checkpoint and return; consecutive overflow steps beyond the limit abort;
heartbeats detect dead ranks between steps; LORAK_FAULT injects host faults.

Reference: ProductionTrainer::train (include/nn/production_trainer.hpp:153-187)
and the main demo loop (main.cpp:60-72).
"""
from __future__ import annotations

import json
import os
import signal
import time
from typing import Dict, List, Optional, Tuple

import torch
import torch.distributed as dist

from ..config import RunConfig, to_dict
from ..models.params import FlatParams, build_layout
from ..parallel.fault import FaultInjector, HeartbeatMonitor
from ..utils.data import NativeTokens
from ..utils.logging import get_logger, log_fields
from .checkpoint import Checkpointer, latest
from .schedules import lr_at

log = get_logger("lora_kernel.train")


def _layout_info(cfg, align: int) -> dict:
    specs, groups, total = build_layout(cfg, align)
    return {"total": total, "align": align,
            "specs": {s.name: [s.offset, s.numel] for s in specs}}


def remap_flat(src: torch.Tensor, src_layout: dict, dst_layout: dict) -> torch.Tensor:
    """Move a flat vector between two layouts of the same model (parameter by name)."""
    out = torch.zeros(dst_layout["total"], dtype=src.dtype)
    for name, (o, n) in src_layout["specs"].items():
        if name in dst_layout["specs"]:
            o2, n2 = dst_layout["specs"][name]
            assert n == n2, name
            out[o2:o2 + n] = src[o:o + n]
    return out


def parallel_plan(par, world: int) -> dict:
    """Which trainer a run config selects on `world` ranks, after checking the
    parallel section: tp / pp / cp each span the whole job and exclude one
    another; dp (when set) is the number of data-parallel ranks, so it must be
    1 under tp / pp / cp and 1 or `world` otherwise.  fused_collectives=False
    runs the same schedules on NCCL collectives (the library baseline)."""
    from ..parallel.cp import CP_MODES
    modes = [k for k in ("tp", "pp", "cp") if getattr(par, k) > 1]
    if len(modes) > 1:
        raise ValueError(f"parallel: {' and '.join(modes)} cannot be combined (each spans the whole job)")
    if par.cp_mode not in CP_MODES:
        raise ValueError(f"parallel.cp_mode must be one of {CP_MODES}, got {par.cp_mode!r}")
    if par.zero_stage not in (0, 1, 2, 3):
        raise ValueError(f"parallel.zero_stage must be 0..3, got {par.zero_stage}")
    if par.tp > 1 and not par.sequence_parallel:
        raise ValueError("parallel.sequence_parallel=False: the tensor-parallel model always keeps activations "
                         "sequence-sharded between its fused all-gather and reduce-scatter GEMMs")
    comm = "p2p" if par.fused_collectives else "nccl"
    if world == 1:
        return {"trainer": "single", "comm": comm}
    if modes:
        k = modes[0]
        if getattr(par, k) != world:
            name = {"tp": "tensor", "pp": "pipeline", "cp": "context"}[k]
            raise ValueError(f"{name} parallelism spans the whole job: {k}={getattr(par, k)} but {world} ranks")
        if par.dp not in (1,):
            raise ValueError(f"parallel.dp={par.dp} with {k}={world}: data parallelism is not combined with {k}")
        return {"trainer": k, "comm": comm}
    if par.dp not in (1, world):
        raise ValueError(f"parallel.dp={par.dp} but the job has {world} ranks (data parallelism spans the job)")
    return {"trainer": "zero3" if par.zero_stage == 3 else "dp", "comm": comm}


class Trainer:
    def __init__(self, rc: RunConfig, device: Optional[str] = None, data=None):
        self.rc = rc
        cfg, tc = rc.model, rc.train
        self.world = dist.get_world_size() if dist.is_initialized() else 1
        self.rank = dist.get_rank() if dist.is_initialized() else 0
        self.device = torch.device(device or f"cuda:{torch.cuda.current_device()}")
        self.lora = tc.lora_rank > 0
        if self.lora and self.world > 1:
            raise NotImplementedError("train.lora_rank: LoRA fine-tuning runs on one GPU")
        if self.world == 1:
            from .pipeline import LoRATrainingPipeline, Transformer, TrainingPipeline
            self.model = Transformer(cfg, self.device, seed=tc.seed)
            if self.lora:  # adapters on the frozen base weights (models/lora.py, fused into the GEMMs)
                from ..models.lora import LoRAConfig
                lc = LoRAConfig(rank=tc.lora_rank, alpha=tc.lora_alpha,
                                targets=tuple(t for t in tc.lora_targets.split(",") if t), init_seed=tc.seed)
                self.pipe = LoRATrainingPipeline(self.model, lc, tc.lr, tc.weight_decay, tc.max_grad_norm,
                                                 train_cfg=tc)
            else:
                self.pipe = TrainingPipeline(self.model, tc.lr, tc.weight_decay, tc.max_grad_norm, train_cfg=tc)
            self.align = 64
        par = rc.parallel
        plan = parallel_plan(par, self.world)
        comm = plan["comm"]
        self.tp = plan["trainer"] == "tp"
        self.pp = plan["trainer"] == "pp"
        self.cp = plan["trainer"] == "cp"
        if tc.swa_start >= 0 and self.world > 1:
            raise NotImplementedError("train.swa_start: SWA runs on one GPU (TrainingPipeline.init_swa)")
        if self.world == 1:
            pass
        elif self.cp:
            # every rank takes its part of each sequence of the same micro-batch
            from ..parallel.cp import ContextParallelTrainer
            self.pipe = ContextParallelTrainer(cfg, tc, zero_stage=min(par.zero_stage, 2), device=self.device,
                                               comm=comm, mode=par.cp_mode)
            self.align = self.pipe.dp.L.align
        elif self.pp:
            # pipeline stages over every rank; all ranks read the same micro-batches
            from ..parallel.pp import PipelineTrainer
            self.pipe = PipelineTrainer(cfg, tc, device=self.device)
            self.align = 64
        elif self.tp:
            # tensor (+ sequence) parallelism over every rank: they share one batch
            from ..parallel.tp import TPTrainer
            self.pipe = TPTrainer(cfg, tc, micro_batch=tc.micro_batch, seq_len=tc.seq_len, device=self.device,
                                  comm=comm, fp8=(par.fp8_recipe if par.fp8 else False), seed=tc.seed)
            self.align = 64
        elif plan["trainer"] == "dp":
            from ..parallel.dp import DataParallelTrainer
            self.pipe = DataParallelTrainer(cfg, tc, zero_stage=par.zero_stage, device=self.device, comm=comm)
            self.align = self.pipe.L.align
        else:
            from ..parallel.zero import Zero3Trainer
            self.pipe = Zero3Trainer(cfg, tc, device=self.device, comm=comm, fuse_gather=par.fuse_gather)
            self.align = self.pipe.L.align
        # tensor and pipeline parallelism: every rank reads the same batch
        shared = self.tp or self.pp or self.cp
        self.data = data or NativeTokens(cfg.vocab_size, tc.micro_batch, tc.seq_len, tc.seed,
                                         0 if shared else self.rank, 1 if shared else self.world,
                                         path=tc.data_path or None, dtype=tc.data_dtype,
                                         threads=tc.loader_threads, fixed=tc.fixed_batch)
        from .crypto import key_from_env
        self.ckpt_key = key_from_env()  # LORAK_CKPT_KEY: encrypt checkpoints (AES-256-GCM)
        self.ckpt = (Checkpointer(tc.checkpoint_dir, self.rank, self.world,
                                  barrier=(dist.barrier if self.world > 1 else None), key=self.ckpt_key)
                     if tc.checkpoint_dir else None)
        self.step = 0
        self._stop = False
        if tc.init_from:
            if tc.init_format == "hf":
                from ..utils.export import import_hf
                sd = import_hf(tc.init_from, cfg)
            else:
                from .checkpoint import load_model_safetensors
                from .crypto import key_from_env
                sd = load_model_safetensors(tc.init_from, key=key_from_env())
            if self.lora:  # the frozen base takes the pretrained weights
                self.model.load_state_dict(sd)
            else:
                self.init_weights(sd)
            del sd
        self.faults = FaultInjector(self.rank)
        self._noise_rank = self._grad_noise_rank(plan["trainer"], par.zero_stage) if tc.grad_noise_eta > 0 else None
        self.pipe.pre_optimizer = self._pre_optimizer
        self.hb = None
        if self.world > 1 and os.environ.get("LORAK_HEARTBEAT", "1") == "1":
            store = dist.distributed_c10d._get_default_store()
            self.hb = HeartbeatMonitor(store, self.rank, self.world,
                                       timeout_s=float(os.environ.get("LORAK_HEARTBEAT_TIMEOUT", "60")))
        self.history: List[dict] = []

    # ------------------------------------------------------------ signals
    def _install_signals(self):
        def handler(signum, frame):
            self._stop = True
            log_fields(log, "signal received; stopping after this step", signal=signum)
        try:
            signal.signal(signal.SIGTERM, handler)
            signal.signal(signal.SIGINT, handler)
        except ValueError:  # not the main thread
            pass

    # ------------------------------------------------------- checkpointing
    def _optim(self):
        o = self.pipe.opt
        t = {"p32": o.p32, "m": o.m, "v": o.v, "state": o.state}
        if o.ema is not None:
            t["ema"] = o.ema
        return t

    def _dp_full_optimizer(self) -> bool:
        """Data parallelism with ZeRO stage 0: every rank holds the whole optimizer state."""
        return getattr(self.pipe, "stage", 3) == 0

    def _ranges(self) -> List[Tuple[int, int]]:
        if self.world == 1 or self._dp_full_optimizer():
            return [(0, self.pipe.engine.params.numel)]
        L = self.pipe.L
        return [(L.owned(g)[0], L.owned(g)[0] + L.chunk[g]) for g in L.names]

    def save_checkpoint(self, async_save: bool = False) -> Optional[str]:
        if self.ckpt is None:
            return None
        cfg = self.rc.model
        if self.lora:  # the adapters alone: lora_step_<N>.safetensors (rank / alpha in the metadata)
            from ..models.lora import save_lora_file
            os.makedirs(self.rc.train.checkpoint_dir, exist_ok=True)
            path = os.path.join(self.rc.train.checkpoint_dir, f"lora_step_{self.step}.safetensors")
            save_lora_file(self.pipe.lora, path, self.step)
            return path
        state = {"step": self.step, "data": self.data.state(), "config": to_dict(self.rc),
                 "world": self.world, "time": time.time()}
        if hasattr(self.pipe, "checkpoint_parts"):  # pipeline / tensor parallel
            layout, ranges, tensors = self.pipe.checkpoint_parts()
            sd = self.pipe.reference_state_dict()  # collective: every rank takes part
            return self.ckpt.save(self.step, sd if self.rank == 0 else None, ranges, tensors, layout, state,
                                  async_save=async_save)
        if self.world == 1:
            model_state = self.pipe.engine.params.to_reference_state_dict()
        else:
            full = self.pipe.full_params()
            fp = FlatParams(cfg, self.device, torch.bfloat16, buffer=full, group_align=self.align)
            model_state = fp.to_reference_state_dict() if self.rank == 0 else None
        path = self.ckpt.save(self.step, model_state, self._ranges(), self._optim(),
                              _layout_info(cfg, self.align), state, async_save=async_save)
        return path

    def init_weights(self, sd: Dict[str, torch.Tensor]) -> None:
        """Start from pretrained weights (a reference-named state dict): the
        fp32 master, its bf16 copies and the EMA take them, the AdamW moments
        stay zero.  Single GPU and the data-parallel / ZeRO / context-parallel
        trainers; a later checkpoint resume overrides it."""
        if self.tp or self.pp:
            raise NotImplementedError("train.init_from with tensor / pipeline parallelism")
        from ..models.params import FlatParams
        cpu = FlatParams(self.rc.model, "cpu", torch.float32)
        cpu.load_reference_state_dict({k: v.float() for k, v in sd.items()})
        full = remap_flat(cpu.flat, _layout_info(self.rc.model, 64), _layout_info(self.rc.model, self.align))
        o = self.pipe.opt
        with torch.no_grad():
            dst = full if (self.world == 1 or self._dp_full_optimizer()) else self.pipe.L.extract_shard(full)
            o.p32.copy_(dst.to(self.device))
            if o.ema is not None:
                o.ema.copy_(o.p32)
            if self.world == 1:
                self.pipe.engine.params.flat.copy_(o.p32.to(torch.bfloat16))
            elif hasattr(self.pipe, "shard_p16"):
                self.pipe.shard_p16.copy_(o.p32.to(torch.bfloat16))
            else:  # data parallel: every rank holds the full bf16 parameters
                self.pipe.params.flat.copy_(full.to(self.device, torch.bfloat16))

    def load_checkpoint(self, path: str) -> None:
        with open(os.path.join(path, "index.json")) as f:
            index = json.load(f)
        flat = Checkpointer.load_flat(path, key=self.ckpt_key)
        if hasattr(self.pipe, "load_checkpoint_flat"):  # pipeline / tensor parallel
            self.pipe.load_checkpoint_flat(flat, index["layout"])
            self._restore_trainer_state(path)
            return
        mine = _layout_info(self.rc.model, self.align)
        o = self.pipe.opt
        with torch.no_grad():
            for name in ("p32", "m", "v", "ema"):
                if name not in flat or (name == "ema" and o.ema is None):
                    continue
                full = remap_flat(flat[name], index["layout"], mine)
                if name == "p32":
                    full_p32 = full
                if self.world == 1 or self._dp_full_optimizer():
                    dst_full = full
                else:
                    dst_full = self.pipe.L.extract_shard(full)
                getattr(o, name).copy_(dst_full.to(self.device))
            o.state.copy_(flat["state"].to(self.device))
            if self.world == 1:
                self.pipe.engine.params.flat.copy_(o.p32.to(torch.bfloat16))
            elif hasattr(self.pipe, "shard_p16"):
                self.pipe.shard_p16.copy_(o.p32.to(torch.bfloat16))
            else:  # data parallel: every rank holds the full bf16 parameters
                self.pipe.params.flat.copy_(full_p32.to(self.device, torch.bfloat16))
        self._restore_trainer_state(path)

    def _grad_noise_rank(self, trainer: str, zero_stage: int) -> int:
        """-1 when every rank's optimizer sees the same (replicated) gradients,
        so they must draw the same noise; the rank when each holds a shard."""
        if trainer == "tp":
            raise NotImplementedError("train.grad_noise_eta with tensor parallelism (replicated and sharded "
                                      "gradients share one buffer)")
        if trainer == "single" or (trainer in ("dp", "cp") and zero_stage == 0):
            return -1
        return self.rank

    def _pre_optimizer(self, grads: torch.Tensor) -> None:
        """Runs on the gradients the optimizer is about to use: host fault
        injection, then optional gradient noise (in the loss-scaled units the
        buffer holds)."""
        self.faults.on_grads(self.step, grads)
        tc = self.rc.train
        if self._noise_rank is not None:
            from ..utils.model_ops import gradient_noise_, noise_seed
            g = torch.Generator(device=grads.device).manual_seed(noise_seed(tc.seed, self.step, self._noise_rank))
            gradient_noise_(grads, self.step, tc.grad_noise_eta, tc.grad_noise_gamma, generator=g,
                            scale=self.pipe.opt.scaler.scale_tensor())

    def _restore_trainer_state(self, path: str) -> None:
        st = Checkpointer.trainer_state(path)
        self.step = int(st["step"])
        self.data.load_state(st.get("data", {}))
        log_fields(log, "resumed", path=path, step=self.step)

    # ---------------------------------------------------------------- loop
    def fit(self, steps: Optional[int] = None, resume: bool = True) -> List[dict]:
        tc = self.rc.train
        total = steps if steps is not None else tc.total_steps
        if resume and self.ckpt is not None:
            p = latest(tc.checkpoint_dir, verify=self.rank == 0)
            if self.world > 1:  # rank 0 checks the checksums; every rank resumes from its choice
                box = [p]
                dist.broadcast_object_list(box, src=0)
                p = box[0]
            if p:
                self.load_checkpoint(p)
        self._install_signals()
        curriculum = None
        if tc.curriculum_start_len > 0:
            if self.tp or self.pp:
                raise NotImplementedError("train.curriculum_start_len: the tensor / pipeline-parallel trainers "
                                          "keep one sequence length")
            from ..utils.data import CurriculumScheduler
            curriculum = CurriculumScheduler(tc.curriculum_start_len, tc.seq_len, max(1, tc.curriculum_steps),
                                             multiple=min(128, tc.curriculum_start_len))
        tok_per_step = tc.micro_batch * tc.seq_len * tc.grad_accum_steps * (1 if (self.tp or self.pp or self.cp)
                                                                             else self.world)
        from ..utils.metrics import TrainMetrics, mfu, train_flops_per_token
        flops_tok = train_flops_per_token(self.rc.model, tc.seq_len)
        metrics = TrainMetrics(tc.metrics_file if self.rank == 0 else "")
        from ..utils.metrics import DeviceMetrics
        dev_metrics = DeviceMetrics(self.device.index or 0) if self.device.type == "cuda" else None
        t_last, s_last = time.perf_counter(), self.step
        tokens_done = 0
        while self.step < total:
            if self.hb is not None:
                self.hb.set_step(self.step)
                self.hb.check()
            self.faults.at_step(self.step)
            self.pipe.set_learning_rate(lr_at(self.step, tc.lr, tc.schedule, tc.warmup_steps, total,
                                              tc.min_lr_ratio))
            self.pipe.loss_acc.zero_()
            for _ in range(tc.grad_accum_steps):
                if hasattr(self.data, "next_device"):
                    x, y = self.data.next_device(self.device)
                else:
                    x, y = self.data.next()
                    x = x.to(self.device, non_blocking=True)
                    y = y.to(self.device, non_blocking=True)
                if curriculum is not None:
                    x, y = curriculum.slice(x, y, self.step)
                    tokens_done += x.numel()
                self.pipe.micro_step_async(x, y)
            self.step += 1
            o = self.pipe.opt
            if self.step % tc.log_every == 0 or self.step == total:
                s, n = self.pipe.loss_acc.tolist()
                now = time.perf_counter()
                steps_done = self.step - s_last
                if curriculum is not None:  # tokens actually trained (x numel is per rank)
                    scale = tok_per_step / (tc.micro_batch * tc.seq_len * tc.grad_accum_steps)
                    tps, tokens_done = tokens_done * scale / (now - t_last), 0
                else:
                    tps = tok_per_step * steps_done / (now - t_last)
                rec = {"step": self.step, "loss": s / max(n, 1.0), "grad_norm": o.grad_norm(),
                       "loss_scale": o.scaler.get_scale(), "skipped": o.scaler.num_skipped(),
                       "lr": o.lr, "tokens_per_s": tps, "mfu": mfu(tps, flops_tok, self.world)}
                t_last, s_last = now, self.step
                self.history.append(rec)
                if dev_metrics is not None:
                    dm = dev_metrics.update()
                    rec["gpu_memory_peak_gb"] = round(dm.get("gpu_memory_peak_bytes", 0) / 2 ** 30, 3)
                if self.rank == 0:
                    log_fields(log, "train", **rec)
                    metrics.record(rec)
                if o.scaler.consecutive_skips() > tc.max_consecutive_skips:
                    raise FloatingPointError(f"{o.scaler.consecutive_skips()} consecutive overflow steps")
            if self.ckpt is not None and tc.checkpoint_every and self.step % tc.checkpoint_every == 0:
                self.save_checkpoint(async_save=True)
            if self._stop:
                break
        metrics.close()
        if self.ckpt is not None:
            self.save_checkpoint()
            self.ckpt.finish()
        if self.hb is not None:
            self.hb.stop()
        return self.history
