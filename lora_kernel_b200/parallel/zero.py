"""ZeRO-3 / FSDP data parallelism on peer memory.

Sharding: the flat parameter layout is grouped per layer ("embed",
"layers.{i}", "head") and every group is padded to a multiple of 64 x world
elements, so rank r owns the contiguous chunk r of every group.  A rank keeps
only its chunks of the bf16 parameters (in symmetric memory, readable by every
peer), of the fp32 master weights and of the AdamW moments.

Per micro-batch (one process per GPU, all on NVLink / NVSwitch):
  forward    before layer i runs, its group is gathered from all owners into a
             local slot (P2P copy kernel on a side stream, one layer ahead;
             two slots, so layer i+1's gather overlaps layer i's compute);
  backward   layers are re-gathered in reverse (the last two are still
             resident).  grad_wire="bf16" (default): each layer's weight
             gradients are written as bf16 into one of three rotating slots of
             symmetric memory (the LM head into its own), and as soon as a
             layer's backward is done its slot is reduce-scattered on the side
             stream: a device barrier, K10 - the owner loads every peer's bf16
             chunk, sums in fp32 in a fixed rank order and adds it into its
             fp32 gradient shard (every micro-batch, so per-rank gradient
             memory is the 1/N shard plus the slots), with the sum-of-squares
             partials on the last micro-batch - then a second barrier after
             which the slot may be overwritten.  The embedding gradient
             (scatter-add) stays in a local fp32 buffer reduced once per
             window.  grad_wire="fp32": weight gradients accumulate in a
             full-size fp32 buffer reduce-scattered on the last micro-batch;
  step       the partials are exchanged through peer memory and the step
             finaliser runs on the device (global-norm clip, overflow skip,
             dynamic loss scale), then AdamW updates the owned shard and
             writes its bf16 chunk back into symmetric memory; the next
             micro-batch starts with a device barrier so no rank gathers a
             chunk that is still being updated.

`comm="nccl"` runs the same schedule with NCCL all-gather / reduce-scatter /
all-reduce instead of the peer-memory kernels: the baseline the kernels are
measured against.

Reference behaviour: ZeROOptimizer::step_zero1/step_zero2
(include/distributed/zero_optimizer.hpp:34-77) and FSDP::all_gather_params /
reduce_scatter_grads (include/distributed/distributed_training.hpp:115-147,
whose collectives are commented out there).
"""
from __future__ import annotations

from typing import Dict, List, Optional, Tuple

import torch
import torch.distributed as dist

from .._ext import C, status
from ..config import TrainConfig, TransformerConfig
from ..ops.gemm import EPI
from ..models.llama import LlamaModel
from ..models.params import FlatParams, build_layout
from ..train.optimizer import FusedAdamW
from ..utils.profiler import ph
from . import comm as CM

NP = 1024
N_GRAD_SLOTS = 3  # rotating bf16 gradient slots: layer i+3 must be read by every rank before layer i writes  # sum-of-squares partial slots per group (one per reduction CTA: the grid is not capped below the SM count)


class ShardLayout:
    """Pure index arithmetic of the ZeRO-3 shard layout (no device needed)."""

    def __init__(self, cfg: TransformerConfig, world: int, rank: int):
        self.cfg, self.world, self.rank = cfg, world, rank
        self.align = 64 * world
        self.specs, self.groups, self.total = build_layout(cfg, self.align)
        self.names = list(self.groups)
        self.chunk: Dict[str, int] = {}
        self.shard_off: Dict[str, int] = {}
        off = 0
        for g, (s, e) in self.groups.items():
            assert (e - s) % world == 0
            self.chunk[g] = (e - s) // world
            self.shard_off[g] = off
            off += self.chunk[g]
        self.shard_numel = off

    def owned(self, g: str, rank: Optional[int] = None) -> Tuple[int, int]:
        """(flat start, length) of `rank`'s chunk of group g."""
        r = self.rank if rank is None else rank
        s, _ = self.groups[g]
        return s + r * self.chunk[g], self.chunk[g]

    def shard_segments(self, decay_norms: bool = False) -> List[Tuple[int, int, bool]]:
        """Parameter pieces inside this rank's shard: (shard offset, length, decay)."""
        segs = []
        for sp in self.specs:
            a0, n = self.owned(sp.group)
            lo, hi = max(sp.offset, a0), min(sp.offset + sp.numel, a0 + n)
            if lo < hi:
                segs.append((self.shard_off[sp.group] + lo - a0, hi - lo, sp.decay or decay_norms))
        return segs

    def extract_shard(self, full: torch.Tensor, rank: Optional[int] = None) -> torch.Tensor:
        parts = []
        for g in self.names:
            a0, n = self.owned(g, rank)
            parts.append(full[a0:a0 + n])
        return torch.cat(parts)

    def assemble(self, shards: List[torch.Tensor]) -> torch.Tensor:
        """Full flat tensor from every rank's shard (rank order)."""
        full = torch.zeros(self.total, dtype=shards[0].dtype, device=shards[0].device)
        for r, sh in enumerate(shards):
            for g in self.names:
                a0, n = self.owned(g, r)
                o = self.shard_off[g]
                full[a0:a0 + n] = sh[o:o + n]
        return full


class _SlotParams:
    """Parameter lookup for the engine: views into whichever local buffer holds
    a group's gathered weights."""

    def __init__(self, layout: ShardLayout):
        self.L = layout
        self.by_name = {s.name: s for s in layout.specs}
        self.cur: Dict[str, torch.Tensor] = {}
        self._views: Dict[Tuple[int, str], torch.Tensor] = {}
        self.override: Dict[str, torch.Tensor] = {}  # name -> tensor read elsewhere (peer memory)

    def bind(self, group: str, buf: torch.Tensor) -> None:
        self.cur[group] = buf

    def __getitem__(self, name: str) -> torch.Tensor:
        if name == "lm_head" and self.L.cfg.tie_embeddings:
            name = "embed"
        ov = self.override.get(name) if self.override else None
        if ov is not None:
            return ov
        sp = self.by_name[name]
        buf = self.cur[sp.group]
        key = (buf.data_ptr(), name)
        v = self._views.get(key)
        if v is None:
            gs = self.L.groups[sp.group][0]
            v = buf[sp.offset - gs:sp.offset - gs + sp.numel].view(sp.shape)
            self._views[key] = v
        return v


class Zero3Trainer:
    """fuse_gather (p2p only): instead of prefetching layer i+1's group on a
    side stream, gather each layer's group inside the first GEMM that needs
    it (K17: the QKV projection in the forward, the Wdown dgrad in the
    backward); the layer's first RMSNorm reads its weight straight from the
    owner's shard in peer memory."""

    def __init__(self, cfg: TransformerConfig, tc: TrainConfig, device="cuda", group=None,
                 comm: str = "p2p", fuse_gather: bool = False, grad_wire: str = "bf16"):
        self.cfg, self.tc = cfg, tc
        self.device = torch.device(device)
        self.group = group or dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        self.mode = comm
        self.fuse_gather = fuse_gather and comm == "p2p"
        if self.fuse_gather and cfg.stochastic_depth > 0:
            raise ValueError("stochastic depth skips layers whose gather the fused GEMM would do; "
                             "use the prefetching gather (fuse_gather=False)")
        if grad_wire not in ("bf16", "fp32"):
            raise ValueError(grad_wire)
        self.grad_wire = grad_wire
        L = self.L = ShardLayout(cfg, self.world, self.rank)
        bf, f32 = torch.bfloat16, torch.float32

        def glen(g):
            s, e = L.groups[g]
            return e - s
        nl = cfg.num_layers
        gmax = max(glen(f"layers.{i}") for i in range(nl))

        # deterministic full init on the device, keep only the owned chunks
        full = FlatParams(cfg, self.device, bf, group_align=L.align)
        full.init_(tc.seed, cfg.init_std)
        shard = L.extract_shard(full.flat)
        del full
        bf16_wire = grad_wire == "bf16"
        self.n_gslots = min(N_GRAD_SLOTS, nl)
        self.gslot_len = gmax
        if comm == "p2p":
            self.pc = CM.PeerComm(self.device, self.group)
            self.shard_sym = CM.SymBuffer(L.shard_numel, bf, self.device, self.group)
            self.shard_p16 = self.shard_sym.local
            if bf16_wire:
                self.gslot_sym = CM.SymBuffer(self.n_gslots * gmax, bf, self.device, self.group)
                self.ghead_sym = CM.SymBuffer(glen("head"), bf, self.device, self.group)
                self.gembed_sym = CM.SymBuffer(glen("embed"), f32, self.device, self.group)
                gslot_flat, ghead, gembed = self.gslot_sym.local, self.ghead_sym.local, self.gembed_sym.local
            else:
                self.grads_sym = CM.SymBuffer(L.total, f32, self.device, self.group)
                grads_flat = self.grads_sym.local
        else:
            self.pc = None
            self.shard_p16 = torch.empty(L.shard_numel, dtype=bf, device=self.device)
            if bf16_wire:
                gslot_flat = torch.zeros(self.n_gslots * gmax, dtype=bf, device=self.device)
                ghead = torch.zeros(glen("head"), dtype=bf, device=self.device)
                gembed = torch.zeros(glen("embed"), dtype=f32, device=self.device)
                self.rs_tmp = torch.empty(max(L.chunk.values()), dtype=bf, device=self.device)
            else:
                grads_flat = torch.zeros(L.total, dtype=f32, device=self.device)
        self.shard_p16.copy_(shard)
        del shard
        self.opt = FusedAdamW(self.shard_p16.float(), L.shard_segments(tc.decay_norms), lr=tc.lr,
                              betas=(tc.beta1, tc.beta2), eps=tc.eps, weight_decay=tc.weight_decay,
                              max_grad_norm=tc.max_grad_norm,
                              dynamic_loss_scale=tc.dynamic_loss_scale,
                              init_loss_scale=tc.init_loss_scale,
                              growth_interval=tc.loss_scale_growth_interval, ema_decay=tc.ema_decay)
        self.shard_grads = torch.zeros(L.shard_numel, dtype=f32, device=self.device)
        self.partial = torch.zeros(len(L.names) * NP, dtype=f32, device=self.device)

        # gathered-weight buffers: embed, head, and two rotating layer slots
        self.buf = {"embed": torch.empty(glen("embed"), dtype=bf, device=self.device),
                    "head": torch.empty(glen("head"), dtype=bf, device=self.device)}
        self.slots = [torch.empty(gmax, dtype=bf, device=self.device) for _ in range(min(2, nl))]
        self.slot_layer = [-1] * len(self.slots)
        self.params = _SlotParams(L)
        self.params.bind("embed", self.buf["embed"])
        self.params.bind("head", self.buf["head"])

        self.gb_count = torch.zeros((max(cfg.qkv_dim, cfg.hidden_dim, cfg.ff_dim_padded) + 127) // 128,
                                    dtype=torch.int32, device=self.device)
        self.engine = LlamaModel(cfg, self.device, params=self.params, with_grads=False)
        self.engine.dropout_seed = tc.seed + 7919 * self.rank  # ranks see different data: decorrelate masks
        self.engine.recompute = tc.recompute_activations
        if bf16_wire:
            # gradient views: layer groups in rotating bf16 slots, the head in its
            # own bf16 buffer, the embedding in a local fp32 buffer (scatter-add)
            self.gslots = [gslot_flat[k * gmax:(k + 1) * gmax] for k in range(self.n_gslots)]
            self.ghead = ghead
            self.gembed = gembed
            self.grad_views = _SlotParams(L)
            self.grad_views.bind("embed", self.gembed)
            self.grad_views.bind("head", self.ghead)
            self.engine.grads = self.grad_views
            self.slot_free: List[Optional[torch.cuda.Event]] = [None] * self.n_gslots
        else:
            self.engine.grads = FlatParams(cfg, self.device, f32, buffer=grads_flat, group_align=L.align)
        self.engine.hooks = self
        self.comm_stream = torch.cuda.Stream(self.device)
        self.gathered: Dict[int, torch.cuda.Event] = {}
        self.accum_steps = max(1, tc.grad_accum_steps)
        self._micro = 0
        self._first = True
        self._last = True
        self._opt_steps = 0
        self.loss_acc = torch.zeros(2, dtype=f32, device=self.device)
        torch.cuda.synchronize(self.device)
        dist.barrier(self.group)

    # ----------------------------------------------------------- collectives
    def _gather(self, g: str, dst: torch.Tensor) -> None:
        """On the current stream: dst <- group g gathered from every rank."""
        n = self.L.chunk[g]
        with ph("comm.all_gather"):
            if self.mode == "p2p":
                self.pc.allgather_copy(self.shard_sym, self.L.shard_off[g], n, dst)
            else:
                o = self.L.shard_off[g]
                dist.all_gather_into_tensor(dst[:n * self.world], self.shard_p16[o:o + n], group=self.group)

    def _reduce_scatter(self, g: str, gi: int) -> None:
        """On the current stream: my shard of group g <- sum over ranks of the
        fp32 gradients (the whole window's, reduced on its last micro-batch)."""
        s, e = self.L.groups[g]
        a0, n = self.L.owned(g)
        o = self.L.shard_off[g]
        part = self.partial[gi * NP:(gi + 1) * NP]
        if self.grad_wire == "bf16":  # only the embedding group is fp32, in its own buffer
            if self.mode == "p2p":
                with ph("comm.barrier"):
                    self.pc.barrier(CM.SLOT_GRAD)
                with ph("comm.reduce_scatter"):
                    self.pc.reduce_scatter_sum(self.gembed_sym, a0 - s, n, self.shard_grads[o:o + n],
                                               accumulate=False, partial=part)
            else:
                with ph("comm.reduce_scatter"):
                    dist.reduce_scatter_tensor(self.shard_grads[o:o + n], self.gembed, group=self.group)
                    part.zero_()
                    part[0] = self.shard_grads[o:o + n].float().pow(2).sum()
            return
        if self.mode == "p2p":
            with ph("comm.barrier"):
                self.pc.barrier(CM.SLOT_GRAD)
            with ph("comm.reduce_scatter"):
                self.pc.reduce_scatter_sum(self.grads_sym, a0, n, self.shard_grads[o:o + n],
                                           accumulate=False, partial=part)
        else:
            full = self.engine.grads.flat[s:e]
            with ph("comm.reduce_scatter"):
                dist.reduce_scatter_tensor(self.shard_grads[o:o + n], full, group=self.group)
                part.zero_()
                part[0] = self.shard_grads[o:o + n].float().pow(2).sum()

    def _reduce_scatter_bf16(self, g: str, gi: int, buf: torch.Tensor, sym_off: int) -> None:
        """On the current stream: my fp32 shard of group g (+)= sum over ranks of
        the group's bf16 gradients in `buf` (every micro-batch; partials on the
        last one)."""
        s, _ = self.L.groups[g]
        a0, n = self.L.owned(g)
        o = self.L.shard_off[g]
        part = self.partial[gi * NP:(gi + 1) * NP] if self._last else None
        first = self._first
        dst = self.shard_grads[o:o + n]
        if self.mode == "p2p":
            sym = self.ghead_sym if g == "head" else self.gslot_sym
            with ph("comm.barrier"):
                self.pc.barrier(CM.SLOT_GRAD)
            with ph("comm.reduce_scatter"):
                self.pc.reduce_scatter_bf16(sym, sym_off + (a0 - s), n, dst, accumulate=not first, partial=part)
            with ph("comm.barrier"):
                self.pc.barrier(CM.SLOT_GRAD_DONE)  # every rank has read this slot
        else:
            glen = self.L.groups[g][1] - s
            with ph("comm.reduce_scatter"):
                dist.reduce_scatter_tensor(self.rs_tmp[:n], buf[:glen], group=self.group)
                if first:
                    dst.copy_(self.rs_tmp[:n])
                else:
                    dst.add_(self.rs_tmp[:n])
                if part is not None:
                    part.zero_()
                    part[0] = dst.pow(2).sum()

    def _on_comm(self, fn, *a):
        ev = torch.cuda.Event()
        ev.record()
        self.comm_stream.wait_event(ev)
        with torch.cuda.stream(self.comm_stream):
            fn(*a)
        done = torch.cuda.Event()
        done.record(self.comm_stream)
        return done

    def _prefetch_layer(self, i: int) -> None:
        if i < 0 or i >= self.cfg.num_layers:
            return
        s = i % len(self.slots)
        if self.slot_layer[s] == i:
            return
        self.slot_layer[s] = i
        self.gathered[i] = self._on_comm(self._gather, f"layers.{i}", self.slots[s])

    def _use_layer(self, i: int) -> None:
        s = i % len(self.slots)
        assert self.slot_layer[s] == i
        ev = self.gathered.pop(i, None)
        if ev is not None:
            with ph("wait.all_gather"):
                torch.cuda.current_stream().wait_event(ev)
        self.params.bind(f"layers.{i}", self.slots[s])

    # --------------------------------------------------------- engine hooks
    def pre_forward(self):
        if self.mode == "p2p":
            with ph("comm.barrier"):
                self.pc.barrier(CM.SLOT_STEP)  # every rank's previous update is visible
        self.slot_layer = [-1] * len(self.slots)

        def initial():
            self._gather("embed", self.buf["embed"])
            self._gather("head", self.buf["head"])
        ev = self._on_comm(initial)
        if not self.fuse_gather:
            for i in range(min(len(self.slots), self.cfg.num_layers)):
                self._prefetch_layer(i)
        with ph("wait.all_gather"):
            torch.cuda.current_stream().wait_event(ev)

    # ------------------------------------------------ K17 fused gather
    def _peer_view(self, name: str) -> Optional[torch.Tensor]:
        """The owner's copy of a small tensor that lies inside one rank's chunk."""
        sp = self.params.by_name[name]
        g = sp.group
        gs, _ = self.L.groups[g]
        ch = self.L.chunk[g]
        o = sp.offset - gs
        owner = o // ch
        if (o + sp.numel - 1) // ch != owner:
            return None
        off = self.L.shard_off[g] + o - owner * ch
        return self.shard_sym.handle.get_buffer(owner, (sp.numel,), torch.bfloat16, off).view(sp.shape)

    def _arm_fused(self, i: int, target: str, transpose: bool) -> None:
        g = f"layers.{i}"
        s = i % len(self.slots)
        gs, ge = self.L.groups[g]
        slot = self.slots[s][:ge - gs]
        self.slot_layer[s] = i
        self.params.bind(g, self.slots[s])
        sp = self.params.by_name[f"{g}.{target}"]
        src = self.shard_sym.ptrs_at(self.L.shard_off[g])
        boff = sp.offset - gs
        chunk, rank = self.L.chunk[g], self.rank
        st = status(self.device)

        def fn(a, b, out):
            C().gemm_gather(a, b, out, EPI["bf16"], None, src, chunk, slot, boff, rank, self.gb_count, st, 0)
        self.engine.fused_gather = (i, target, fn)

    def pre_layer_fwd(self, i):
        if self.fuse_gather:
            name = f"layers.{i}.attn_norm"
            pv = self._peer_view(name)
            if pv is not None:
                self.params.override = {name: pv}
                self._arm_fused(i, "wqkv", False)
                return
            self.params.override = {}
            self._prefetch_layer(i)
            self._use_layer(i)
            return
        self._use_layer(i)
        self._prefetch_layer(i + 1)

    def post_head_bwd(self):
        if self.grad_wire == "bf16":
            # the head buffer is reused next micro-batch, after post_backward has
            # waited for every side-stream collective of this one
            self._on_comm(self._reduce_scatter_bf16, "head", self.L.names.index("head"), self.ghead, 0)
        elif self._last:
            self._on_comm(self._reduce_scatter, "head", self.L.names.index("head"))

    def _bind_grad_slot(self, i):
        k = i % self.n_gslots
        ev = self.slot_free[k]
        if ev is not None:  # every rank has finished reading the slot's previous layer
            with ph("wait.reduce_scatter"):
                torch.cuda.current_stream().wait_event(ev)
            self.slot_free[k] = None
        self.grad_views.bind(f"layers.{i}", self.gslots[k])

    def pre_layer_bwd(self, i):
        if self.grad_wire == "bf16":
            self._bind_grad_slot(i)
        if self.fuse_gather:
            self.params.override = {}
            if self.slot_layer[i % len(self.slots)] == i:
                self.params.bind(f"layers.{i}", self.slots[i % len(self.slots)])
            else:
                self._arm_fused(i, "wdown", True)
            return
        if self.slot_layer[i % len(self.slots)] != i:
            self._prefetch_layer(i)
        self._use_layer(i)
        self._prefetch_layer(i - 1)

    def post_layer_bwd(self, i):
        g = f"layers.{i}"
        if self.grad_wire == "bf16":
            k = i % self.n_gslots
            self.slot_free[k] = self._on_comm(self._reduce_scatter_bf16, g, self.L.names.index(g), self.gslots[k],
                                              k * self.gslot_len)
        elif self._last:
            self._on_comm(self._reduce_scatter, g, self.L.names.index(g))

    def post_backward(self):
        if self._last:
            self._on_comm(self._reduce_scatter, "embed", self.L.names.index("embed"))
        if self.grad_wire == "bf16":
            self.slot_free = [None] * self.n_gslots  # the wait below covers them
        ev = torch.cuda.Event()
        ev.record(self.comm_stream)
        with ph("wait.reduce_scatter"):
            torch.cuda.current_stream().wait_event(ev)

    # -------------------------------------------------------------- stepping
    def _optimizer_step(self):
        if getattr(self, "pre_optimizer", None) is not None:
            self.pre_optimizer(self.shard_grads)
        o = self.opt
        s = o.scaler
        with ph("step.grad_norm+finalize"):
            if self.mode == "p2p":
                self.pc.norm_exchange(self.partial, o.state, o.max_grad_norm, s.enabled, s.growth,
                                      s.backoff, s.growth_interval, s.min_scale)
            else:
                tot = self.partial.sum().reshape(1)
                dist.all_reduce(tot, group=self.group)
                o.finalize(tot)
        with ph("step.adamw"):
            o.apply(self.shard_grads, self.shard_p16, zero_grad=False)
        self._opt_steps += 1

    def micro_step_async(self, ids: torch.Tensor, targets: torch.Tensor) -> None:
        first = self._micro % self.accum_steps == 0
        self._first = first
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

    # --------------------------------------------------------------- utils
    @staticmethod
    def grad_memory_plan(L: "ShardLayout", grad_wire: str = "bf16") -> Dict[str, int]:
        """Bytes of gradient buffers one rank holds (no device needed)."""
        def glen(g):
            s, e = L.groups[g]
            return e - s
        if grad_wire == "fp32":
            return {"full_fp32": 4 * L.total, "shard_fp32": 4 * L.shard_numel}
        nl = L.cfg.num_layers
        gmax = max(glen(f"layers.{i}") for i in range(nl))
        return {"shard_fp32": 4 * L.shard_numel, "layer_slots_bf16": 2 * min(N_GRAD_SLOTS, nl) * gmax,
                "head_bf16": 2 * glen("head"), "embed_fp32": 4 * glen("embed")}

    def grad_memory_bytes(self) -> int:
        return sum(self.grad_memory_plan(self.L, self.grad_wire).values())

    def full_params(self) -> torch.Tensor:
        """Gather the full bf16 flat parameters on every rank (checkpointing/tests)."""
        parts = [torch.empty_like(self.shard_p16) for _ in range(self.world)]
        dist.all_gather(parts, self.shard_p16.contiguous(), group=self.group)
        return self.L.assemble(parts)
