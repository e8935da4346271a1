"""Context (sequence) parallelism, Ulysses style: every rank holds a contiguous
chunk of each sequence for all per-token work (norms, GEMMs, SwiGLU, CE) and
trades sequence sharding for head sharding around attention.

    forward   qkv [B*S/P, (H+2KV)*Dh] (this rank's tokens, RoPE at global
              positions) --all-to-all--> [B*S, (H/P + 2KV/P)*Dh] (all tokens,
              this rank's heads) -> causal flash attention (K3, unchanged) ->
              o [B*S, H/P*Dh] --all-to-all--> [B*S/P, H*Dh]
    backward  dO by the same exchange, K4 on the head shard, dQKV back.
The attention kernels see an ordinary full-length sequence with fewer heads,
so causal masking, GQA and sliding windows need nothing new; H and KV must be
divisible by P.  Weights are replicated and their gradients are summed over
the ranks exactly like data parallelism, so the trainer is the data-parallel
trainer (ZeRO 0/1/2 on peer memory) with the attention swapped and each rank
fed its sequence chunk.

The exchange runs as NCCL all-to-all with the layout permutes as device
copies; fusing it into the QKV GEMM epilogue (peer stores, as K18 does for
tensor parallelism) is left for later.

Reference: none (the survey lists context parallelism / ring attention /
Ulysses as absent from the reference).
"""
from __future__ import annotations

from typing import Callable, Dict, Optional, Tuple

import torch
import torch.distributed as dist

from ..config import TrainConfig, TransformerConfig


class UlyssesAttention:
    """Attention over a sequence sharded across `world` ranks.  attn_fwd /
    attn_bwd have the signatures of ops.attention.attention_fwd / _bwd
    (injectable so the exchange can be tested on CPU)."""

    def __init__(self, cfg: TransformerConfig, group=None, attn_fwd: Optional[Callable] = None,
                 attn_bwd: Optional[Callable] = None):
        self.cfg = cfg
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        H, KV, Dh = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim
        P = self.world
        if H % P or KV % P:
            raise ValueError(f"context parallelism over {P} ranks needs heads ({H}) and kv heads ({KV}) "
                             f"divisible by {P}")
        self.Hl, self.KVl = H // P, KV // P
        self.cols_l = (self.Hl + 2 * self.KVl) * Dh
        # qkv columns owned by each rank: its q heads, then its k heads, then its v heads
        idx = []
        for r in range(P):
            q = range(r * self.Hl * Dh, (r + 1) * self.Hl * Dh)
            k = range((H + r * self.KVl) * Dh, (H + (r + 1) * self.KVl) * Dh)
            v = range((H + KV + r * self.KVl) * Dh, (H + KV + (r + 1) * self.KVl) * Dh)
            idx.append(list(q) + list(k) + list(v))
        self._col_idx_cpu = torch.tensor(idx, dtype=torch.int64)
        self._col_idx: Dict[torch.device, torch.Tensor] = {}
        if attn_fwd is None or attn_bwd is None:
            from ..ops import attention as A
            attn_fwd = attn_fwd or A.attention_fwd
            attn_bwd = attn_bwd or A.attention_bwd
        self.attn_fwd, self.attn_bwd = attn_fwd, attn_bwd
        self.saved: Dict[Tuple[int, int], dict] = {}

    def pos_offset(self, s_local: int) -> int:
        return self.rank * s_local

    def _cols(self, dev) -> torch.Tensor:
        t = self._col_idx.get(dev)
        if t is None:
            t = self._col_idx[dev] = self._col_idx_cpu.to(dev)
        return t

    def _a2a(self, send: torch.Tensor) -> torch.Tensor:
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=self.group)
        return recv

    def _bufs(self, key, B, S, dev, dtype) -> dict:
        b = self.saved.get(key)
        if b is None or b["qkv"].shape[0] != B * S:
            H, Dh = self.Hl, self.cfg.head_dim
            b = {"qkv": torch.empty(B * S, self.cols_l, dtype=dtype, device=dev),
                 "o": torch.empty(B * S, H * Dh, dtype=dtype, device=dev),
                 "lse": torch.empty(B, H, S, dtype=torch.float32, device=dev),
                 "dqkv": torch.empty(B * S, self.cols_l, dtype=dtype, device=dev)}
            self.saved[key] = b
        return b

    def forward(self, qkv: torch.Tensor, B: int, s_local: int, out: torch.Tensor, key=(0, 0),
                window: int = 0) -> torch.Tensor:
        """qkv: this rank's [B*s_local, (H+2KV)*Dh] (RoPE applied); writes the
        attention output of this rank's tokens, all heads, into out."""
        P, Dh = self.world, self.cfg.head_dim
        T = B * s_local
        S = s_local * P
        cols = self._cols(qkv.device)
        send = qkv.index_select(1, cols.view(-1)).view(T, P, self.cols_l).transpose(0, 1).contiguous()
        recv = self._a2a(send)                                  # [P, T, cols_l]: chunk r of every sequence
        b = self._bufs(key, B, S, qkv.device, qkv.dtype)
        b["qkv"].view(B, P, s_local, self.cols_l).copy_(recv.view(P, B, s_local, self.cols_l).transpose(0, 1))
        self.attn_fwd(b["qkv"], B, S, self.Hl, self.KVl, Dh, causal=True, window=window, out=b["o"], lse=b["lse"])
        send_o = b["o"].view(B, P, s_local, self.Hl * Dh).transpose(0, 1).contiguous().view(P, T, self.Hl * Dh)
        recv_o = self._a2a(send_o)                              # [P, T, Hl*Dh]: head group r of my tokens
        out.view(T, P, self.Hl * Dh).copy_(recv_o.transpose(0, 1))
        return out

    def backward(self, dout: torch.Tensor, B: int, s_local: int, dqkv: torch.Tensor, key=(0, 0),
                 window: int = 0) -> torch.Tensor:
        """dout: gradient of this rank's attention output [B*s_local, H*Dh];
        writes dL/dqkv of this rank's tokens into dqkv."""
        P, Dh = self.world, self.cfg.head_dim
        T = B * s_local
        S = s_local * P
        b = self.saved[key]
        send = dout.view(T, P, self.Hl * Dh).transpose(0, 1).contiguous()
        recv = self._a2a(send)
        do_h = recv.view(P, B, s_local, self.Hl * Dh).transpose(0, 1).reshape(B * S, self.Hl * Dh)
        self.attn_bwd(b["qkv"], b["o"], do_h.contiguous(), b["lse"], B, S, self.Hl, self.KVl, Dh, causal=True,
                      window=window, dqkv=b["dqkv"])
        send_d = b["dqkv"].view(B, P, s_local, self.cols_l).transpose(0, 1).contiguous().view(P, T, self.cols_l)
        recv_d = self._a2a(send_d)                              # [P, T, cols_l]: rank r's head columns
        cols = self._cols(dqkv.device)
        dqkv.index_copy_(1, cols.view(-1), recv_d.transpose(0, 1).reshape(T, P * self.cols_l))
        return dqkv


def shard_sequence(x: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """This rank's contiguous chunk of every sequence of x [B, S]."""
    S = x.shape[1]
    if S % world:
        raise ValueError(f"sequence length {S} is not divisible by {world} context-parallel ranks")
    n = S // world
    return x[:, rank * n:(rank + 1) * n].contiguous()


class ContextParallelTrainer:
    """Data-parallel trainer (ZeRO stage 0/1/2, peer-memory collectives) whose
    ranks share each micro-batch by sequence chunks, with Ulysses attention."""

    def __init__(self, cfg: TransformerConfig, tc: TrainConfig, zero_stage: int = 0, device="cuda",
                 group=None, comm: str = "p2p"):
        from .dp import DataParallelTrainer
        self.dp = DataParallelTrainer(cfg, tc, zero_stage=zero_stage, device=device, group=group, comm=comm)
        self.rank, self.world = self.dp.rank, self.dp.world
        self.dp.engine.ctx = UlyssesAttention(cfg, self.dp.group)
        self.opt = self.dp.opt
        # [loss sum, token count] over the whole micro-batches (all ranks' chunks)
        self.loss_acc = torch.zeros(2, dtype=torch.float32, device=self.dp.device)

    def micro_step_async(self, ids: torch.Tensor, targets: torch.Tensor) -> None:
        """ids / targets: the FULL micro-batch [B, S] (the same on every rank)."""
        self.dp.loss_acc.zero_()
        self.dp.micro_step_async(shard_sequence(ids, self.rank, self.world),
                                 shard_sequence(targets, self.rank, self.world))
        dist.all_reduce(self.dp.loss_acc, group=self.dp.group)
        self.loss_acc += self.dp.loss_acc

    def train_step(self, ids, targets) -> float:
        """Mean token loss of the full micro-batch (every rank returns it)."""
        self.loss_acc.zero_()
        self.micro_step_async(ids, targets)
        s, n = self.loss_acc.tolist()
        return s / max(n, 1.0)

    def __getattr__(self, name):
        # everything else (optimizer, layout, parameters, checkpoint hooks) is the data-parallel trainer's
        if name == "dp":
            raise AttributeError(name)
        return getattr(self.dp, name)

    @property
    def pre_optimizer(self):
        return getattr(self.dp, "pre_optimizer", None)

    @pre_optimizer.setter
    def pre_optimizer(self, fn) -> None:
        self.dp.pre_optimizer = fn

    def set_learning_rate(self, lr: float) -> None:
        self.dp.set_learning_rate(lr)

    def current_step(self) -> int:
        return self.dp.current_step()

    def full_params(self) -> torch.Tensor:
        return self.dp.full_params()
