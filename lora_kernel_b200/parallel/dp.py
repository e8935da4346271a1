"""Data parallelism with ZeRO stage 0, 1 or 2 on peer memory.

Every rank holds the full bf16 parameters (in symmetric memory) and a full
fp32 gradient buffer (symmetric memory), and runs the whole model on its own
micro-batches.  What differs is where the gradients meet the optimizer:

  stage 0   each finished layer group is all-reduced in place (K12: one-shot
            peer all-reduce fused with the sum-of-squares partials of the
            result), overlapped with the rest of the backward on a side
            stream; every rank then runs AdamW over the full parameters.
  stage 1/2 each finished group is reduce-scattered (K10 front half: the owner
            sums its chunk over the peers in fixed rank order, fused with the
            Σg² partials) - stage 2 as soon as the group's gradients are
            complete (overlapped), stage 1 after the whole backward; the owner
            runs AdamW on its shard only (sharded moments and master weights)
            and the same kernel stores each updated bf16 value into EVERY
            rank's parameter buffer (the parameter all-gather fused into the
            optimizer; K10 back half).
In all stages the global gradient norm is exchanged through peer memory and
the step finaliser (clip / overflow skip / dynamic loss scale) runs on the
device.  `comm="nccl"` is the same schedule on NCCL all-reduce /
reduce-scatter / all-gather: the baseline.

Reference: ZeROOptimizer::step_zero1 / step_zero2
(include/distributed/zero_optimizer.hpp:34-77), DataParallelTrainer and
RingAllReduce (include/distributed/distributed_training.hpp:20-110,152-230).
"""
from __future__ import annotations

from typing import Dict, List, Optional

import torch
import torch.distributed as dist

from .._ext import C
from ..config import TrainConfig, TransformerConfig
from ..models.llama import LlamaModel
from ..models.params import FlatParams
from ..train.optimizer import FusedAdamW
from . import comm as CM
from .zero import NP, ShardLayout


class DataParallelTrainer:
    def __init__(self, cfg: TransformerConfig, tc: TrainConfig, zero_stage: int = 2, device="cuda",
                 group=None, comm: str = "p2p"):
        if zero_stage not in (0, 1, 2):
            raise ValueError("DataParallelTrainer runs ZeRO stage 0, 1 or 2 (stage 3: Zero3Trainer)")
        self.cfg, self.tc, self.stage = cfg, tc, zero_stage
        self.device = torch.device(device)
        self.group = group or dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        self.mode = comm
        L = self.L = ShardLayout(cfg, self.world, self.rank)
        bf, f32 = torch.bfloat16, torch.float32
        if comm == "p2p":
            self.pc = CM.PeerComm(self.device, self.group)
            self.p_sym = CM.SymBuffer(L.total, bf, self.device, self.group)
            self.g_sym = CM.SymBuffer(L.total, f32, self.device, self.group)
            pbuf, gbuf = self.p_sym.local, self.g_sym.local
        else:
            self.pc = None
            pbuf = torch.zeros(L.total, dtype=bf, device=self.device)
            gbuf = torch.zeros(L.total, dtype=f32, device=self.device)
        self.params = FlatParams(cfg, self.device, bf, buffer=pbuf, group_align=L.align)
        self.params.init_(tc.seed, cfg.init_std)
        self.grads = FlatParams(cfg, self.device, f32, buffer=gbuf, group_align=L.align)
        self.engine = LlamaModel(cfg, self.device, params=self.params, with_grads=False)
        self.engine.dropout_seed = tc.seed + 7919 * self.rank  # ranks see different data: decorrelate masks
        self.engine.recompute = tc.recompute_activations
        self.engine.grads = self.grads
        self.engine.hooks = self
        okw = dict(lr=tc.lr, betas=(tc.beta1, tc.beta2), eps=tc.eps, weight_decay=tc.weight_decay,
                   max_grad_norm=tc.max_grad_norm, dynamic_loss_scale=tc.dynamic_loss_scale,
                   init_loss_scale=tc.init_loss_scale, growth_interval=tc.loss_scale_growth_interval,
                   ema_decay=tc.ema_decay)
        if zero_stage == 0:
            self.opt = FusedAdamW(self.params.flat.float(), self.params.segments(tc.decay_norms), **okw)
        else:
            master = L.extract_shard(self.params.flat).float()
            segs = []
            for s_off, n, decay in L.shard_segments(tc.decay_norms):
                g = self._group_of_shard_offset(s_off)
                a0, _ = L.owned(g)
                segs.append((s_off, n, decay, a0 - L.shard_off[g]))
            self.opt = FusedAdamW(master, segs, **okw)
            self.shard_grads = torch.zeros(L.shard_numel, dtype=f32, device=self.device)
        self.partial = torch.zeros(len(L.names) * NP, dtype=f32, device=self.device)
        self.comm_stream = torch.cuda.Stream(self.device)
        self.accum_steps = max(1, tc.grad_accum_steps)
        self._micro = 0
        self._last = True
        self._opt_steps = 0
        self.loss_acc = torch.zeros(2, dtype=f32, device=self.device)
        torch.cuda.synchronize(self.device)
        dist.barrier(self.group)

    def _group_of_shard_offset(self, s_off: int) -> str:
        for g in self.L.names:
            o = self.L.shard_off[g]
            if o <= s_off < o + self.L.chunk[g]:
                return g
        raise KeyError(s_off)

    # ----------------------------------------------------------- collectives
    def _reduce_group(self, g: str) -> None:
        gi = self.L.names.index(g)
        part = self.partial[gi * NP:(gi + 1) * NP]
        s, e = self.L.groups[g]
        if self.stage == 0:
            if self.mode == "p2p":
                self.pc.allreduce_sum_(self.g_sym, e - s, part, off=s)
            else:
                dist.all_reduce(self.grads.flat[s:e], group=self.group)
                part.zero_()
                C().grad_norm_partials(self.grads.flat[s:e], part)
                part.div_(self.world)
            return
        a0, n = self.L.owned(g)
        o = self.L.shard_off[g]
        if self.mode == "p2p":
            self.pc.barrier(CM.SLOT_GRAD)
            self.pc.reduce_scatter_sum(self.g_sym, a0, n, self.shard_grads[o:o + n], accumulate=False,
                                       partial=part)
        else:
            dist.reduce_scatter_tensor(self.shard_grads[o:o + n], self.grads.flat[s:e], group=self.group)
            part.zero_()
            C().grad_norm_partials(self.shard_grads[o:o + n], part)

    def _on_comm(self, fn, *a):
        ev = torch.cuda.Event()
        ev.record()
        self.comm_stream.wait_event(ev)
        with torch.cuda.stream(self.comm_stream):
            fn(*a)

    # --------------------------------------------------------- engine hooks
    def pre_forward(self):
        if self.mode == "p2p" and self.stage > 0:
            self.pc.barrier(CM.SLOT_STEP)  # every owner's fused all-gather has landed

    def pre_layer_fwd(self, i):
        pass

    def pre_layer_bwd(self, i):
        pass

    def _overlap(self) -> bool:
        return self._last and self.stage in (0, 2)

    def post_head_bwd(self):
        if self._overlap():
            self._on_comm(self._reduce_group, "head")

    def post_layer_bwd(self, i):
        if self._overlap():
            self._on_comm(self._reduce_group, f"layers.{i}")

    def post_backward(self):
        if self._last:
            if self._overlap():
                self._on_comm(self._reduce_group, "embed")
            else:
                for g in reversed(self.L.names):
                    self._on_comm(self._reduce_group, g)
        ev = torch.cuda.Event()
        ev.record(self.comm_stream)
        torch.cuda.current_stream().wait_event(ev)

    # -------------------------------------------------------------- stepping
    def _optimizer_step(self):
        if getattr(self, "pre_optimizer", None) is not None:
            self.pre_optimizer(self.grads.flat if self.stage == 0 else self.shard_grads)
        o = self.opt
        s = o.scaler
        if self.mode == "p2p":
            self.pc.norm_exchange(self.partial, o.state, o.max_grad_norm, s.enabled, s.growth,
                                  s.backoff, s.growth_interval, s.min_scale)
        else:
            tot = self.partial.sum().reshape(1)
            dist.all_reduce(tot, group=self.group)
            o.finalize(tot)
        if self.stage == 0:
            o.apply(self.grads.flat, self.params.flat, zero_grad=False)
        elif self.mode == "p2p":
            o.apply(self.shard_grads, None, zero_grad=False, p16_peers=self.p_sym.ptrs)
        else:
            shard16 = torch.empty(self.L.shard_numel, dtype=torch.bfloat16, device=self.device)
            o.apply(self.shard_grads, shard16, zero_grad=False)
            parts = [torch.empty_like(shard16) for _ in range(self.world)]
            dist.all_gather(parts, shard16, group=self.group)
            self.params.flat.copy_(self.L.assemble(parts))
        self._opt_steps += 1

    def micro_step_async(self, ids: torch.Tensor, targets: torch.Tensor) -> None:
        first = self._micro % self.accum_steps == 0
        self._last = (self._micro + 1) % self.accum_steps == 0
        self.engine.forward_backward(ids, targets, loss_scale=self.opt.scaler.scale_tensor(),
                                     grad_scale=1.0 / (ids.numel() * self.accum_steps * self.world),
                                     label_smoothing=self.tc.label_smoothing, z_loss=self.tc.z_loss,
                                     loss_acc=self.loss_acc, overwrite_grads=first)
        self._micro += 1
        if self._last:
            self._optimizer_step()

    def train_step(self, ids, targets) -> float:
        self.loss_acc.zero_()
        self.micro_step_async(ids, targets)
        s, n = self.loss_acc.tolist()
        return s / max(n, 1.0)

    def current_step(self) -> int:
        return self._opt_steps

    def set_learning_rate(self, lr: float) -> None:
        self.opt.set_lr(lr)

    def full_params(self) -> torch.Tensor:
        return self.params.flat.clone()
