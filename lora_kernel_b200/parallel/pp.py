"""Pipeline parallelism: contiguous layer stages, one per rank, run with the
1F1B schedule.

Stage s owns layers [l0, l1) (stage 0 also the embedding, the last stage the
final norm, LM head and cross-entropy).  Its parameters are a stage-local flat
buffer whose tensors keep their global names and per-tensor init seeds, so
stage weights equal the single-GPU model's and checkpoints use the usual
reference names.

Schedule (1F1B, P stages, M micro-batches): stage s runs w = min(P-s-1, M)
warm-up forwards, then alternates one forward and one backward, then drains
the w remaining backwards.  At most min(P-s, M) micro-batches are in flight on
stage s, which bounds its activation memory.  Activations go to stage s+1 and
their gradients come back as bf16 [tokens, D] tensors.  A forward send is
paired with the backward receive from the same neighbour, and a backward send
with the next forward receive.  Each pair is issued as one batched P2P group,
so neighbours cannot block on each other's ordering.  The schedule is plain
data (`schedule_1f1b`), and `simulate` checks on the CPU that the ranks' comm
sequences match up with no deadlock.

Optimizer: each stage runs the fused AdamW (K11) on its own flat range.  The
global gradient norm is one all-reduce of the stages' Σg², so clipping, the
overflow skip and the dynamic loss scale are decided identically everywhere.
The loss is computed on the last stage and broadcast.

Reference: MicroBatchScheduler (include/nn/training_enhancements.hpp:345-366,
all forwards then all backwards despite its 1F1B comment),
ModelParallelPlanner (include/distributed/distributed_training.hpp:91-110,
round-robin layer placement), P2PScheduler (:179-199, no send) and
PipelineInference (include/serving/serving_production.hpp:194-206, empty).
"""
from __future__ import annotations

import dataclasses
from typing import Callable, Dict, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from ..config import TrainConfig, TransformerConfig

# --------------------------------------------------------------------------
# partition and schedule (pure Python; CPU-testable)
# --------------------------------------------------------------------------


def head_cost_in_layers(cfg: TransformerConfig) -> float:
    """FLOPs of the LM head + cross-entropy relative to one decoder layer."""
    D, V, F = cfg.hidden_dim, cfg.vocab_size, cfg.ff_dim
    layer = D * (cfg.qkv_dim + cfg.q_dim) + 3 * D * F
    return V * D / max(1, layer)


def partition_layers(num_layers: int, stages: int, head_cost: float = 0.0) -> List[range]:
    """Contiguous layer ranges, one per stage, minimising the largest stage
    cost when the last stage also carries `head_cost` layer-equivalents."""
    if stages < 1 or num_layers < stages:
        raise ValueError(f"cannot split {num_layers} layers into {stages} stages")
    if stages == 1:
        return [range(num_layers)]
    best = None
    for n_last in range(1, num_layers - stages + 2):
        rest = num_layers - n_last
        per = -(-rest // (stages - 1))
        # smallest bottleneck first, then the last stage closest to the others
        key = (round(max(n_last + head_cost, per), 9), abs(per - (n_last + head_cost)))
        if best is None or key < best[0]:
            best = (key, n_last)
    n_last = best[1]
    rest = num_layers - n_last
    q, r = divmod(rest, stages - 1)
    sizes = [q + (1 if i < r else 0) for i in range(stages - 1)]
    # give the remainder to the middle stages first (stage 0 also embeds)
    sizes.reverse()
    sizes.append(n_last)
    out, a = [], 0
    for n in sizes:
        out.append(range(a, a + n))
        a += n
    return out


# One schedule step: ("F", mb) / ("B", mb) compute, or ("X", [comm ops]) where
# a comm op is (kind, direction, mb): kind "send"/"recv", direction "next"
# (towards the last stage) or "prev"; the payload is the activation when the
# op points forward (send next / recv prev) and its gradient otherwise.
Step = Tuple[str, object]


def schedule_1f1b(stages: int, stage: int, micro: int) -> List[Step]:
    first, last = stage == 0, stage == stages - 1
    warm = min(stages - stage - 1, micro)
    rest = micro - warm
    out: List[Step] = []

    def x(*ops):
        ops = [o for o in ops if o is not None]
        if ops:
            out.append(("X", ops))

    recv_fwd = (lambda mb: None if first else ("recv", "prev", mb))
    send_fwd = (lambda mb: None if last else ("send", "next", mb))
    recv_bwd = (lambda mb: None if last else ("recv", "next", mb))
    send_bwd = (lambda mb: None if first else ("send", "prev", mb))

    for mb in range(warm):
        x(recv_fwd(mb))
        out.append(("F", mb))
        x(send_fwd(mb))
    if rest > 0:
        x(recv_fwd(warm))
    for i in range(rest):
        f, b = warm + i, i
        out.append(("F", f))
        x(send_fwd(f), recv_bwd(b))
        out.append(("B", b))
        if i == rest - 1:
            x(send_bwd(b))
        else:
            x(send_bwd(b), recv_fwd(f + 1))
    for b in range(rest, micro):
        x(recv_bwd(b))
        out.append(("B", b))
        x(send_bwd(b))
    return out


def simulate(stages: int, micro: int) -> Dict[str, object]:
    """Run every stage's schedule against the others with batched-group
    semantics (a group completes once each of its ops has its counterpart
    posted by the neighbour).  Raises on deadlock or a payload mismatch;
    returns per-stage peak in-flight micro-batches and the tick count."""
    scheds = [schedule_1f1b(stages, s, micro) for s in range(stages)]
    pc = [0] * stages
    posted: Dict[Tuple[int, int, str, int], int] = {}  # (src, dst, payload, mb) -> count
    consumed: Dict[Tuple[int, int, str, int], int] = {}
    inflight = [0] * stages
    peak = [0] * stages
    done_f = [set() for _ in range(stages)]
    done_b = [set() for _ in range(stages)]
    ticks = 0
    pending: List[Optional[list]] = [None] * stages

    def key(s, op):
        kind, d, mb = op
        peer = s + 1 if d == "next" else s - 1
        payload = "act" if (kind == "send") == (d == "next") else "grad"
        return (s, peer, payload, mb) if kind == "send" else (peer, s, payload, mb)

    while any(pc[s] < len(scheds[s]) for s in range(stages)):
        progressed = False
        for s in range(stages):
            if pc[s] >= len(scheds[s]):
                continue
            kind, arg = scheds[s][pc[s]]
            if kind == "F":
                if s > 0 and arg not in done_f[s - 1]:
                    raise RuntimeError(f"stage {s} forwards mb {arg} before stage {s-1} did")
                done_f[s].add(arg)
                inflight[s] += 1
                peak[s] = max(peak[s], inflight[s])
                pc[s] += 1
                progressed = True
            elif kind == "B":
                if arg not in done_f[s] or (s < stages - 1 and arg not in done_b[s + 1]):
                    raise RuntimeError(f"stage {s} backward of mb {arg} out of order")
                done_b[s].add(arg)
                inflight[s] -= 1
                pc[s] += 1
                progressed = True
            else:
                if pending[s] is None:
                    pending[s] = arg
                    for op in arg:
                        if op[0] == "send":
                            k = key(s, op)
                            posted[k] = posted.get(k, 0) + 1
                    progressed = True
                ok = all(op[0] == "send" or posted.get(key(s, op), 0) > consumed.get(key(s, op), 0)
                         for op in pending[s])
                if ok:
                    for op in pending[s]:
                        if op[0] == "recv":
                            k = key(s, op)
                            consumed[k] = consumed.get(k, 0) + 1
                    pending[s] = None
                    pc[s] += 1
                    progressed = True
        ticks += 1
        if not progressed:
            raise RuntimeError(f"pipeline deadlock at ticks={ticks}: pcs={pc}")
    if posted != consumed:
        raise RuntimeError("unmatched pipeline messages")
    return {"peak_inflight": peak, "ticks": ticks}


def stage_global_ranges(local, global_layout: dict) -> List[Tuple[int, int, int]]:
    """(local offset, global offset, numel) of every tensor of a stage's flat
    parameters (FlatParams) in the full model's layout ({"specs": {name:
    [offset, numel]}}), in local order."""
    out = []
    for sp in local.specs:
        g_off, n = global_layout["specs"][sp.name]
        assert n == sp.numel, sp.name
        out.append((sp.offset, g_off, n))
    return out


def gather_stage(flat_local: torch.Tensor, ranges) -> torch.Tensor:
    """The stage's values concatenated in the order of `ranges` (padding dropped)."""
    return torch.cat([flat_local[lo:lo + n] for lo, _, n in ranges])


def scatter_stage(flat_global: torch.Tensor, ranges, flat_local: torch.Tensor) -> torch.Tensor:
    """Copy the stage's tensors out of a full-layout vector into its local flat."""
    for lo, go, n in ranges:
        flat_local[lo:lo + n].copy_(flat_global[go:go + n])
    return flat_local


# --------------------------------------------------------------------------
# executor
# --------------------------------------------------------------------------


class StageCompute:
    """What the executor needs from a stage (the GPU engine below, or a test double)."""

    def forward(self, mb: int) -> None: ...
    def backward(self, mb: int) -> None: ...
    def act_out(self, mb: int) -> torch.Tensor: ...   # sent to the next stage
    def act_in(self, mb: int) -> torch.Tensor: ...    # received from the previous stage
    def grad_out(self, mb: int) -> torch.Tensor: ...  # sent to the previous stage
    def grad_in(self, mb: int) -> torch.Tensor: ...   # received from the next stage


def run_schedule(sched: Sequence[Step], compute: StageCompute, prev_rank: Optional[int],
                 next_rank: Optional[int], group=None) -> None:
    for kind, arg in sched:
        if kind == "F":
            compute.forward(arg)
        elif kind == "B":
            compute.backward(arg)
        else:
            ops = []
            for op_kind, d, mb in arg:
                peer = next_rank if d == "next" else prev_rank
                if op_kind == "send":
                    t = compute.act_out(mb) if d == "next" else compute.grad_out(mb)
                    ops.append(dist.P2POp(dist.isend, t, peer, group))
                else:
                    t = compute.grad_in(mb) if d == "next" else compute.act_in(mb)
                    ops.append(dist.P2POp(dist.irecv, t, peer, group))
            for r in dist.batch_isend_irecv(ops):
                r.wait()


# --------------------------------------------------------------------------
# the GPU stage engine and trainer
# --------------------------------------------------------------------------


class PipelineStageEngine:
    """One pipeline stage of the Llama engine (layers `layers`, plus the
    embedding on the first stage and the head on the last), with one
    workspace per in-flight micro-batch."""

    def __init__(self, cfg: TransformerConfig, stage: int, stages: int, layers: range, device,
                 seed: int = 1234):
        from ..models.llama import LlamaModel
        from ..models.params import FlatParams
        if cfg.tie_embeddings and stages > 1:
            raise NotImplementedError("pipeline parallelism with tied embeddings (first and last stage "
                                      "would share one matrix)")
        self.cfg = cfg
        self.stage, self.stages = stage, stages
        self.first, self.last = stage == 0, stage == stages - 1
        self.layers = layers
        self.device = torch.device(device)
        params = FlatParams(cfg, self.device, layers=layers, embed=self.first, head=self.last)
        params.init_(seed, cfg.init_std)
        self.model = LlamaModel(cfg, self.device, params=params)
        self.params, self.grads = self.model.params, self.model.grads
        self.local_cfg = dataclasses.replace(cfg, num_layers=len(layers))
        self._ws: Dict[Tuple[int, int, int], list] = {}

    def workspaces(self, B: int, S: int, n: int) -> list:
        from ..models.llama import _Workspace
        key = (B, S, n)
        if key not in self._ws:
            m = self.model
            if S > m.rope.shape[0]:
                from ..ops import elementwise as E
                m.rope = E.rope_table(S, self.cfg.head_dim, self.cfg.rope_base, self.device)
            wss = [_Workspace(self.local_cfg, B, S, self.device, save=True, logits=(self.last and k == 0),
                              dropout=self.cfg.dropout > 0)
                   for k in range(n)]
            for w in wss[1:]:
                w.logits = wss[0].logits  # the last stage runs F and B of one micro-batch back to back
            self._ws = {key: wss}
        return self._ws[key]

    def forward(self, ws, ids: Optional[torch.Tensor]) -> None:
        from ..ops import elementwise as E
        m = self.model
        m._saving = True
        if self.first:
            E.embedding_fwd(ids.reshape(-1), self.params["embed"], out=ws.h[0])
        for j, i in enumerate(self.layers):
            m._layer_fwd(i, ws, ws.h[j], ws.h[j + 1], j)

    def head(self, ws, targets, loss_scale, grad_scale: float, acc, overwrite: bool, tc: TrainConfig) -> None:
        """Last stage: final norm, LM head, fused CE (loss + dlogits), the head's
        backward; leaves d(last layer output) in ws.dh."""
        from ..ops import gemm as G
        from ..ops import loss as L
        from ..ops import norm as N
        m, n, cfg = self.model, len(self.layers), self.cfg
        m._overwrite = overwrite
        N.rmsnorm_fwd(ws.h[n], self.params["final_norm"], cfg.norm_eps, y=ws.xf, rstd=ws.rstdf)
        G.linear(ws.xf, self.params["lm_head"], out=ws.logits)
        L.cross_entropy_(ws.logits, targets.reshape(-1), acc, scale=loss_scale, scale_mul=grad_scale,
                         smoothing=tc.label_smoothing, z_loss=tc.z_loss)
        G.linear_dgrad(ws.logits, self.params["lm_head"], out=ws.dx)
        m._wgrad(ws.logits, ws.xf, "lm_head")
        N.rmsnorm_bwd(ws.dx, ws.h[n], self.params["final_norm"], ws.rstdf, self.grads["final_norm"], dx=ws.dh,
                      accumulate=not overwrite)

    def backward(self, ws, ids: Optional[torch.Tensor], overwrite: bool) -> None:
        from ..ops import elementwise as E
        m = self.model
        m._overwrite = overwrite
        for j in reversed(range(len(self.layers))):
            m._layer_bwd(self.layers[j], ws, slot=j, hidx=j)
        if self.first:
            if overwrite:
                self.grads["embed"].zero_()
            E.embedding_bwd(ids.reshape(-1), ws.dh, self.grads["embed"])
        m._overwrite = False


class _EngineCompute(StageCompute):
    def __init__(self, eng: PipelineStageEngine, wss, batches, loss_scale, grad_scale, acc, tc, micro_base: int):
        self.eng, self.wss, self.batches = eng, wss, batches
        self.loss_scale, self.grad_scale, self.acc, self.tc = loss_scale, grad_scale, acc, tc
        self.n = len(eng.layers)
        self.micro_base = micro_base  # global micro-batch index of mb 0 (dropout seeds)

    def _ws(self, mb):
        return self.wss[mb % len(self.wss)]

    def forward(self, mb):
        ws = self._ws(mb)
        # the same dropout masks as the single-GPU engine's micro-step counter
        self.eng.model._drop_step = self.micro_base + mb
        self.eng.forward(ws, self.batches[mb][0] if self.eng.first else None)
        if self.eng.last:
            self.eng.head(ws, self.batches[mb][1], self.loss_scale, self.grad_scale, self.acc, mb == 0, self.tc)

    def backward(self, mb):
        self.eng.model._drop_step = self.micro_base + mb
        self.eng.backward(self._ws(mb), self.batches[mb][0] if self.eng.first else None, mb == 0)

    def act_out(self, mb):
        return self._ws(mb).h[self.n]

    def act_in(self, mb):
        return self._ws(mb).h[0]

    def grad_out(self, mb):
        return self._ws(mb).dh

    def grad_in(self, mb):
        return self._ws(mb).dh


class PipelineTrainer:
    """1F1B pipeline-parallel training over every rank of the job (one stage
    per rank).  `step(batches)` runs one optimizer step over M micro-batches;
    the Trainer interface (`micro_step_async`) collects grad_accum_steps
    micro-batches and steps on the last one."""

    def __init__(self, cfg: TransformerConfig, tc: TrainConfig, device=None, seed: Optional[int] = None,
                 group=None):
        from ..train.optimizer import FusedAdamW
        self.group = group
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.granks = [dist.get_global_rank(group, r) if group is not None else r for r in range(self.world)] \
            if dist.is_initialized() else [0]
        self.device = torch.device(device or f"cuda:{torch.cuda.current_device()}")
        self.cfg, self.tc = cfg, tc
        if self.world > 1:
            # a collective first, so the communicator exists before any P2P group
            dist.all_reduce(torch.zeros(1, device=self.device), group=group)
        self.parts = partition_layers(cfg.num_layers, self.world, head_cost_in_layers(cfg))
        self.engine = PipelineStageEngine(cfg, self.rank, self.world, self.parts[self.rank], self.device,
                                          tc.seed if seed is None else seed)
        eng = self.engine
        self.opt = FusedAdamW(eng.params.flat.float(), eng.params.segments(decay_norms=tc.decay_norms),
                              lr=tc.lr, betas=(tc.beta1, tc.beta2), eps=tc.eps, weight_decay=tc.weight_decay,
                              max_grad_norm=tc.max_grad_norm, dynamic_loss_scale=tc.dynamic_loss_scale,
                              init_loss_scale=tc.init_loss_scale, growth_interval=tc.loss_scale_growth_interval,
                              ema_decay=tc.ema_decay)
        self.loss_acc = torch.zeros(2, dtype=torch.float32, device=self.device)
        self._gsq = torch.zeros(1, dtype=torch.float32, device=self.device)
        self.accum_steps = max(1, tc.grad_accum_steps)
        self._pending: List[Tuple[torch.Tensor, torch.Tensor]] = []
        self._opt_steps = 0
        self._micro_done = 0
        self.pre_optimizer: Optional[Callable] = None

    @property
    def prev_rank(self):
        return self.granks[self.rank - 1] if self.rank > 0 else None

    @property
    def next_rank(self):
        return self.granks[self.rank + 1] if self.rank < self.world - 1 else None

    def set_learning_rate(self, lr: float) -> None:
        self.opt.set_lr(lr)

    def current_step(self) -> int:
        return self._opt_steps

    def step(self, batches: Sequence[Tuple[torch.Tensor, torch.Tensor]]) -> None:
        M = len(batches)
        B, S = batches[0][0].shape
        eng = self.engine
        wss = eng.workspaces(B, S, max(1, min(self.world - self.rank, M)))
        comp = _EngineCompute(eng, wss, batches, self.opt.scaler.scale_tensor(), 1.0 / (B * S * M),
                              self.loss_acc, self.tc, self._micro_done)
        self._micro_done += M
        run_schedule(schedule_1f1b(self.world, self.rank, M), comp, self.prev_rank, self.next_rank, self.group)
        g = eng.grads.flat
        if self.pre_optimizer is not None:
            self.pre_optimizer(g)
        part = self.opt.norm_partials(g)
        torch.sum(part, dim=0, keepdim=True, out=self._gsq)
        if self.world > 1:
            dist.all_reduce(self._gsq, group=self.group)
            # every rank reports the loss the last stage computed
            dist.broadcast(self.loss_acc, self.granks[-1], group=self.group)
        self.opt.finalize(self._gsq)
        self.opt.apply(g, eng.params.flat, zero_grad=False)
        self._opt_steps += 1

    def micro_step_async(self, ids: torch.Tensor, targets: torch.Tensor) -> None:
        self._pending.append((ids, targets))
        if len(self._pending) == self.accum_steps:
            batches, self._pending = self._pending, []
            self.step(batches)

    def train_step(self, ids: torch.Tensor, targets: torch.Tensor) -> float:
        self.loss_acc.zero_()
        self.micro_step_async(ids, targets)
        s, n = self.loss_acc.tolist()
        return s / max(n, 1.0)

    # ------------------------------------------------------------ checkpoints
    def global_layout(self) -> dict:
        from ..models.params import build_layout
        specs, _, total = build_layout(self.cfg, 64)
        return {"total": total, "align": 64, "specs": {s.name: [s.offset, s.numel] for s in specs}}

    def checkpoint_parts(self):
        """(full-model layout, this stage's ranges in it, optimizer tensors
        concatenated in range order) for Checkpointer.save."""
        lay = self.global_layout()
        rr = stage_global_ranges(self.engine.params, lay)
        o = self.opt
        tensors = {n: gather_stage(getattr(o, n), rr) for n in ("p32", "m", "v")}
        tensors["state"] = o.state
        return lay, [(g, g + n) for _, g, n in rr], tensors

    def load_checkpoint_flat(self, flat: Dict[str, torch.Tensor], saved_layout: dict) -> None:
        """Restore this stage from full-model optimizer vectors (any alignment)."""
        from ..train.trainer import remap_flat
        lay = self.global_layout()
        rr = stage_global_ranges(self.engine.params, lay)
        o = self.opt
        with torch.no_grad():
            for n in ("p32", "m", "v"):
                full = remap_flat(flat[n], saved_layout, lay)
                scatter_stage(full.to(self.device), rr, getattr(o, n))
            o.state.copy_(flat["state"].to(self.device))
            self.engine.params.flat.copy_(o.p32.to(torch.bfloat16))

    def reference_state_dict(self) -> Dict[str, torch.Tensor]:
        return self.full_state_dict()

    def full_state_dict(self) -> Dict[str, torch.Tensor]:
        """Every stage's tensors, reference names, gathered on all ranks (CPU)."""
        mine = {k: v.detach().float().cpu() for k, v in self.engine.params.to_reference_state_dict().items()}
        if self.world == 1:
            return mine
        parts: List[Optional[dict]] = [None] * self.world
        dist.all_gather_object(parts, mine, group=self.group)
        out: Dict[str, torch.Tensor] = {}
        for p in parts:
            out.update(p)
        return out
