"""Context (sequence) parallelism: every rank holds a part of each sequence
for all per-token work (norms, GEMMs, SwiGLU, CE); attention is the only op
that mixes tokens, and two schemes cover it.

Ulysses (UlyssesAttention): each rank holds a contiguous chunk of each
sequence and trades sequence sharding for head sharding around attention.

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

Ring (RingAttention): no head divisibility limit (the 1.1B model's 4 KV heads
allow Ulysses on at most 4 ranks).  The sequence is cut into 2P chunks and
rank r holds chunks r and 2P-1-r ("zigzag"), so under the causal mask every
rank does the same attention work.  Key/value chunks travel around the ring
(P2P send/recv to the neighbours, the next block's transfer overlapping the
current block's kernels); each block is one launch of the unchanged K3/K4
kernels and the partial outputs are merged by their log-sum-exp:

    step 0         own K/V: causal attention over the rank's 2 chunks (in
                   position order, so the ordinary causal mask is exact)
    owner j < r    K/V chunk j precedes both query chunks: full attention
                   of both query chunks against it
    owner j > r    both K/V chunks of j lie between the query chunks: full
                   attention of query chunk 2P-1-r against them
The backward recomputes each block with the merged LSE and output, so the
block gradients are exact parts of the full gradient; dK/dV accumulators
(fp32) travel with their K/V and return to the owner after P hops.

Reference: none (the reference has no context parallelism, ring attention
or Ulysses).
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

    def rope_args(self, B: int, s_local: int, device) -> dict:
        """Keyword arguments of ops.elementwise.rope_ that give this rank's
        tokens their global positions."""
        return {"pos_offset": self.pos_offset(s_local)}

    def shard(self, x: torch.Tensor) -> torch.Tensor:
        """This rank's tokens of every sequence of x [B, S]."""
        return shard_sequence(x, self.rank, self.world)

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


class RingAttention:
    """Causal attention over a sequence split into 2P chunks, rank r holding
    chunks r and 2P-1-r (shard_zigzag), by ring exchange of K/V blocks.
    attn_fwd / attn_bwd have the signatures of ops.attention.attention_fwd /
    _bwd (injectable so the schedule can be tested on CPU)."""

    def __init__(self, cfg: TransformerConfig, group=None, attn_fwd: Optional[Callable] = None,
                 attn_bwd: Optional[Callable] = None):
        self.cfg = cfg
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        H, KV, Dh = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim
        self.qc, self.kvc = H * Dh, 2 * KV * Dh
        self.cols = self.qc + self.kvc
        P, r = self.world, self.rank
        glob = (lambda g: g) if group is None else (lambda g: dist.get_global_rank(group, g))
        self.next, self.prev = glob((r + 1) % P), glob((r - 1) % P)
        if attn_fwd is None or attn_bwd is None:
            from ..ops import attention as A
            attn_fwd = attn_fwd or A.attention_fwd
            attn_bwd = attn_bwd or A.attention_bwd
        self.attn_fwd, self.attn_bwd = attn_fwd, attn_bwd
        self.saved: Dict[Tuple[int, int], dict] = {}
        self._bufs: Dict[tuple, torch.Tensor] = {}
        self._pos: Dict[tuple, torch.Tensor] = {}

    # ------------------------------------------------------------ layout
    def chunk(self, s_local: int) -> int:
        if s_local % 2:
            raise ValueError(f"ring attention needs an even local sequence length, got {s_local}")
        return s_local // 2

    def positions(self, B: int, s_local: int, device) -> torch.Tensor:
        """int32 [B*s_local]: global position of each of this rank's tokens."""
        k = (B, s_local, str(device))
        t = self._pos.get(k)
        if t is None:
            c, P, r = self.chunk(s_local), self.world, self.rank
            one = torch.cat([torch.arange(r * c, (r + 1) * c),
                             torch.arange((2 * P - 1 - r) * c, (2 * P - r) * c)])
            t = self._pos[k] = one.repeat(B).to(torch.int32).to(device)
        return t

    def rope_args(self, B: int, s_local: int, device) -> dict:
        return {"positions": self.positions(B, s_local, device)}

    def shard(self, x: torch.Tensor) -> torch.Tensor:
        return shard_zigzag(x, self.rank, self.world)

    def _buf(self, name: str, shape, dtype, dev) -> torch.Tensor:
        k = (name, tuple(shape), dtype, str(dev))
        t = self._bufs.get(k)
        if t is None:
            t = self._bufs[k] = torch.empty(shape, dtype=dtype, device=dev)
        return t

    # ------------------------------------------------------------ exchange
    def _shift(self, send: torch.Tensor, recv: torch.Tensor):
        """Start sending `send` to the next rank and receiving the previous
        rank's into `recv`; returns the pending works."""
        if self.world == 1:
            recv.copy_(send)
            return []
        ops = [dist.P2POp(dist.isend, send, self.next, self.group),
               dist.P2POp(dist.irecv, recv, self.prev, self.group)]
        return dist.batch_isend_irecv(ops)

    @staticmethod
    def _wait(works) -> None:
        for w in works:
            w.wait()

    @staticmethod
    def _merge(o_acc: torch.Tensor, lse_acc: torch.Tensor, o_b: torch.Tensor, lse_b: torch.Tensor) -> None:
        """o_acc [B, c, H, Dh] fp32, lse_acc [B, H, c] fp32 (views, updated in
        place) <- the log-sum-exp weighted combination with block (o_b, lse_b)."""
        new = torch.logaddexp(lse_acc, lse_b)
        a = torch.exp(lse_acc - new).transpose(1, 2).unsqueeze(-1)
        b = torch.exp(lse_b - new).transpose(1, 2).unsqueeze(-1)
        o_acc.mul_(a).add_(o_b.float() * b)
        lse_acc.copy_(new)

    # ------------------------------------------------------------ forward
    def forward(self, qkv: torch.Tensor, B: int, s_local: int, out: torch.Tensor, key=(0, 0),
                window: int = 0) -> torch.Tensor:
        """qkv: this rank's [B*s_local, (H+2KV)*Dh] in zigzag order, RoPE
        applied at global positions; writes this rank's attention output."""
        if window:
            raise NotImplementedError("ring attention: sliding-window attention is not supported")
        P, r, c = self.world, self.rank, self.chunk(s_local)
        H, KV, Dh, qc = self.cfg.num_heads, self.cfg.num_kv_heads, self.cfg.head_dim, self.qc
        dev, dt = qkv.device, qkv.dtype
        x = qkv.view(B, 2, c, self.cols)
        o_acc = self._buf("o_acc", (B, 2, c, H, Dh), torch.float32, dev)
        prev = self.saved.get(key)
        lse = prev["lse"] if prev is not None and prev["lse"].shape == (B, H, 2, c) else \
            torch.empty(B, H, 2, c, dtype=torch.float32, device=dev)   # kept for the backward
        kvb = [self._buf("kv0", (B, 2, c, self.kvc), dt, dev), self._buf("kv1", (B, 2, c, self.kvc), dt, dev)]
        kvb[0].copy_(x[..., qc:])
        works = self._shift(kvb[0], kvb[1]) if P > 1 else []
        # step 0: own K/V, causal over the two local chunks (position order)
        o_blk = self._buf("o_blk", (B * 2 * c, qc), dt, dev)
        lse_blk = self._buf("lse_blk", (B * 2, H, c), torch.float32, dev)
        self.attn_fwd(qkv, B, 2 * c, H, KV, Dh, causal=True, out=o_blk, lse=lse.view(B, H, 2 * c))
        o_acc.copy_(o_blk.view(B, 2, c, H, Dh))
        pk = self._buf("pk", (B, 2, c, self.cols), dt, dev) if P > 1 else None
        for t in range(1, P):
            self._wait(works)
            cur = kvb[t % 2]
            works = self._shift(cur, kvb[(t + 1) % 2]) if t < P - 1 else []
            j = (r - t) % P
            # owners r-1 .. 0 come first, then P-1 .. r+1: the query half changes once
            if j < r:   # K/V chunk j, seen by both query chunks
                if t == 1:
                    pk[..., :qc].copy_(x[..., :qc])
                pk[..., qc:].copy_(cur[:, :1].expand(B, 2, c, self.kvc))
            else:       # both K/V chunks of j, seen by query chunk 2P-1-r
                if t == r + 1:
                    pk[..., :qc].copy_(x[:, 1:, :, :qc].expand(B, 2, c, qc))
                pk[..., qc:].copy_(cur)
            self.attn_fwd(pk.view(B * 2 * c, self.cols), B * 2, c, H, KV, Dh, causal=False, out=o_blk,
                          lse=lse_blk)
            ob = o_blk.view(B, 2, c, H, Dh)
            lb = lse_blk.view(B, 2, H, c)
            if j < r:
                for h in range(2):
                    self._merge(o_acc[:, h], lse[:, :, h], ob[:, h], lb[:, h])
            else:
                for h in range(2):
                    self._merge(o_acc[:, 1], lse[:, :, 1], ob[:, h], lb[:, h])
        self._wait(works)
        out.view(B, 2, c, H, Dh).copy_(o_acc)
        self.saved[key] = {"qkv": qkv, "o": out, "lse": lse}
        return out

    # ------------------------------------------------------------ backward
    def backward(self, dout: torch.Tensor, B: int, s_local: int, dqkv: torch.Tensor, key=(0, 0),
                 window: int = 0) -> torch.Tensor:
        """dout: gradient of this rank's attention output [B*s_local, H*Dh];
        writes dL/dqkv of this rank's tokens (zigzag order) into dqkv."""
        if window:
            raise NotImplementedError("ring attention: sliding-window attention is not supported")
        P, r, c = self.world, self.rank, self.chunk(s_local)
        H, KV, Dh, qc = self.cfg.num_heads, self.cfg.num_kv_heads, self.cfg.head_dim, self.qc
        st = self.saved[key]
        qkv, o, lse = st["qkv"], st["o"], st["lse"]
        dev, dt = qkv.device, qkv.dtype
        x = qkv.view(B, 2, c, self.cols)
        kvb = [self._buf("kv0", (B, 2, c, self.kvc), dt, dev), self._buf("kv1", (B, 2, c, self.kvc), dt, dev)]
        kvb[0].copy_(x[..., qc:])
        works = self._shift(kvb[0], kvb[1]) if P > 1 else []
        dkv = [self._buf("dkv0", (B, 2, c, self.kvc), torch.float32, dev),
               self._buf("dkv1", (B, 2, c, self.kvc), torch.float32, dev)]
        dq = self._buf("dq_acc", (B, 2, c, qc), torch.float32, dev)
        dblk = self._buf("dblk", (B * 2 * c, self.cols), dt, dev)
        # step 0: own K/V, causal
        self.attn_bwd(qkv, o, dout, lse.view(B, H, 2 * c), B, 2 * c, H, KV, Dh, causal=True, dqkv=dblk)
        d = dblk.view(B, 2, c, self.cols)
        dq.copy_(d[..., :qc])
        dkv[0].copy_(d[..., qc:])
        # accumulators move one hop per step, each transfer overlapping the next block
        dworks = self._shift(dkv[0], dkv[1]) if P > 1 else []
        if P > 1:
            # per-sequence operands of the two off-diagonal block shapes, built once
            lse_lo = lse.transpose(1, 2).contiguous()                            # [B, 2, H, c]
            ov, dov = o.view(B, 2, c, qc), dout.view(B, 2, c, qc)
            o_hi = ov[:, 1:].expand(B, 2, c, qc).contiguous()
            do_hi = dov[:, 1:].expand(B, 2, c, qc).contiguous()
            lse_hi = lse[:, :, 1].unsqueeze(1).expand(B, 2, H, c).contiguous()
            pk = self._buf("pk", (B, 2, c, self.cols), dt, dev)
            part = self._buf("dkv_part", (B, 2, c, self.kvc), torch.float32, dev)
        for t in range(1, P):
            self._wait(works)
            cur = kvb[t % 2]
            works = self._shift(cur, kvb[(t + 1) % 2]) if t < P - 1 else []
            j = (r - t) % P
            if j < r:
                if t == 1:
                    pk[..., :qc].copy_(x[..., :qc])
                pk[..., qc:].copy_(cur[:, :1].expand(B, 2, c, self.kvc))
                self.attn_bwd(pk.view(B * 2 * c, self.cols), o, dout, lse_lo, B * 2, c, H, KV, Dh,
                              causal=False, dqkv=dblk)
                d = dblk.view(B, 2, c, self.cols)
                dq.add_(d[..., :qc])
                part.zero_()
                part[:, 0].copy_(d[:, 0, :, qc:])
                part[:, 0].add_(d[:, 1, :, qc:])
            else:
                if t == r + 1:
                    pk[..., :qc].copy_(x[:, 1:, :, :qc].expand(B, 2, c, qc))
                pk[..., qc:].copy_(cur)
                self.attn_bwd(pk.view(B * 2 * c, self.cols), o_hi.view(-1, qc), do_hi.view(-1, qc),
                              lse_hi, B * 2, c, H, KV, Dh, causal=False, dqkv=dblk)
                d = dblk.view(B, 2, c, self.cols)
                dq[:, 1].add_(d[:, 0, :, :qc])
                dq[:, 1].add_(d[:, 1, :, :qc])
                part.copy_(d[..., qc:])
            # the accumulator of the K/V held now has arrived from the previous rank
            self._wait(dworks)
            dkv[t % 2].add_(part)
            dworks = self._shift(dkv[t % 2], dkv[(t + 1) % 2])
        self._wait(works)
        self._wait(dworks)  # after P hops every accumulator is home
        mine = dkv[P % 2] if P > 1 else dkv[0]
        out = dqkv.view(B, 2, c, self.cols)
        out[..., :qc].copy_(dq)
        out[..., qc:].copy_(mine)
        return dqkv


def shard_zigzag(x: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """This rank's chunks r and 2P-1-r (of 2P equal chunks) of every sequence
    of x [B, S], concatenated in that (position) order."""
    S = x.shape[1]
    if S % (2 * world):
        raise ValueError(f"sequence length {S} is not divisible by 2 x {world} ring-attention ranks")
    c = S // (2 * world)
    return torch.cat([x[:, rank * c:(rank + 1) * c], x[:, (2 * world - 1 - rank) * c:(2 * world - rank) * c]],
                     dim=1).contiguous()


def shard_sequence(x: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """This rank's contiguous chunk of every sequence of x [B, S]."""
    S = x.shape[1]
    if S % world:
        raise ValueError(f"sequence length {S} is not divisible by {world} context-parallel ranks")
    n = S // world
    return x[:, rank * n:(rank + 1) * n].contiguous()


CP_MODES = ("ulysses", "ring")


def make_context_attention(cfg: TransformerConfig, mode: str = "ulysses", group=None, attn_fwd=None,
                           attn_bwd=None):
    """The engine's context-parallel attention hook for `mode`."""
    if mode == "ulysses":
        return UlyssesAttention(cfg, group, attn_fwd, attn_bwd)
    if mode == "ring":
        return RingAttention(cfg, group, attn_fwd, attn_bwd)
    raise ValueError(f"unknown context-parallel mode {mode!r} (one of {CP_MODES})")


class ContextParallelTrainer:
    """Data-parallel trainer (ZeRO stage 0/1/2, peer-memory collectives) whose
    ranks share each micro-batch by sequence parts, with Ulysses (contiguous
    chunks) or ring (zigzag chunks) attention."""

    def __init__(self, cfg: TransformerConfig, tc: TrainConfig, zero_stage: int = 0, device="cuda",
                 group=None, comm: str = "p2p", mode: str = "ulysses"):
        from .dp import DataParallelTrainer
        self.dp = DataParallelTrainer(cfg, tc, zero_stage=zero_stage, device=device, group=group, comm=comm)
        self.rank, self.world = self.dp.rank, self.dp.world
        self.ctx = self.dp.engine.ctx = make_context_attention(cfg, mode, self.dp.group)
        self.opt = self.dp.opt
        # [loss sum, token count] over the whole micro-batches (all ranks' chunks)
        self.loss_acc = torch.zeros(2, dtype=torch.float32, device=self.dp.device)

    def micro_step_async(self, ids: torch.Tensor, targets: torch.Tensor) -> None:
        """ids / targets: the FULL micro-batch [B, S] (the same on every rank)."""
        self.dp.loss_acc.zero_()
        self.dp.micro_step_async(self.ctx.shard(ids), self.ctx.shard(targets))
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
        if name in ("dp", "ctx"):
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
