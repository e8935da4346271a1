"""Tensor-parallel serving: one process per GPU, Megatron column/row split.

Every rank holds its shard of the weights (query/KV heads, FFN blocks and
vocabulary rows, optionally int4/int8/fp8 quantised) and the KV cache of its
own KV heads.  Activations between the linears are replicated: after each
row-parallel linear (Wo, Wdown) every rank has a partial [rows, D]; one kernel
then sums the partials of all ranks - through the NVLS multicast address
(multimem.ld_reduce, reduced inside the NVSwitch) or by peer loads in fixed
rank order - and fuses the residual add and the next RMSNorm (csrc/tp.cu).
The LM head is vocabulary-parallel: each rank samples over its slice with the
Gumbel noise of the global token id (K19) and the best (score, id) across
ranks is the exact single-GPU sample.

Scheduling runs on rank 0 only (the LLMEngine with a `RunnerProxy`); each
runner call is broadcast over a CPU (gloo) group to the other ranks, whose
`worker_loop` executes the same call on their shard, so every rank launches
the same kernels in the same order.

Reference: the reference's serving stack (include/api/serving_production.hpp)
runs in one process without tensor parallelism; its TP layers
(include/distributed/tensor_parallel.hpp:14-104) are forward-only matmul
splits with an all-reduce.
"""
from __future__ import annotations

import dataclasses
from typing import Dict, List, Optional

import numpy as np
import torch
import torch.distributed as dist

from .._ext import C
from ..config import TransformerConfig
from ..ops import elementwise as E
from ..ops import norm as N
from ..ops import serving as SV
from ..parallel import comm as CM
from .model_runner import ModelRunner, PrefillItem

SLOT_SERVE = 6


class TPServeComm:
    """Two alternating symmetric partial buffers + the fused all-reduce/norm."""

    def __init__(self, hidden: int, max_rows: int, device, group=None):
        self.group = group or dist.group.WORLD
        self.tp = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        self.device = torch.device(device)
        self.D, self.max_rows = hidden, max_rows
        self.pc = CM.PeerComm(self.device, self.group)
        self.part = [CM.SymBuffer(max_rows * hidden, torch.bfloat16, self.device, self.group) for _ in range(2)]
        self.k = 0
        self.pc.barrier_dev(SLOT_SERVE)  # create the device epoch counter before any graph capture
        torch.cuda.synchronize(self.device)

    def partial(self, rows: int) -> torch.Tensor:
        if rows > self.max_rows:
            raise ValueError(f"{rows} rows exceed the TP partial buffers ({self.max_rows})")
        return self.part[self.k].local[:rows * self.D].view(rows, self.D)

    def allreduce_norm(self, rows: int, out: torch.Tensor, resid: torch.Tensor, gamma: torch.Tensor,
                       y: torch.Tensor, eps: float) -> None:
        """out = resid + sum over ranks of partial(rows); y = rmsnorm(out).  Flips
        to the other partial buffer (a buffer is rewritten only after the next
        barrier, by which time every rank has finished reading it)."""
        buf = self.part[self.k]
        self.pc.barrier_dev(SLOT_SERVE)
        view = buf.local[:rows * self.D].view(rows, self.D)
        if self.pc.nvls and buf.mc_ptr:
            C().rs_sum(view, self.tp, out, resid, gamma, y, None, float(eps), 2, None, buf.mc_ptr)
        else:
            C().rs_sum(view, self.tp, out, resid, gamma, y, None, float(eps), 1, buf.ptrs, 0)
        self.k ^= 1


class TPModelRunner(ModelRunner):
    """ModelRunner over this rank's shard (`params`: parallel.tp.TPParams)."""

    # each rank holds a vocabulary slice; the top-p threshold would need the whole row
    supports_top_p = False

    def __init__(self, cfg: TransformerConfig, params, comm: TPServeComm, device="cuda", **kw):
        tp = comm.tp
        if cfg.num_heads % tp or cfg.num_kv_heads % tp:
            raise ValueError(f"tp={tp} must divide the head counts")
        self.full_cfg = cfg
        self.comm = comm
        self.tp, self.rank = tp, comm.rank
        local = dataclasses.replace(cfg, num_heads=cfg.num_heads // tp, num_kv_heads=cfg.num_kv_heads // tp)
        super().__init__(local, params, device, **kw)
        # every rank must index the same KV blocks: agree on the smallest pool
        nb = torch.tensor([self.num_blocks], dtype=torch.int64, device=self.device)
        dist.all_reduce(nb, op=dist.ReduceOp.MIN, group=comm.group)
        self.num_blocks = int(nb.item())
        self.vocab_local = self.W["lm_head"].shape[0]
        self._xn: Optional[torch.Tensor] = None

    def _layer(self, i, h, pos, slots, attn):
        cfg, c = self.cfg, self.comm
        p = f"layers.{i}."
        xn = self._xn if self._xn is not None else N.rmsnorm_fwd(h, self.W[p + "attn_norm"], cfg.norm_eps)[0]
        qkv = self._linear(xn, p + "wqkv")
        E.rope_(qkv, 0, cfg.num_heads + cfg.num_kv_heads, cfg.head_dim, self.rope, positions=pos)
        ks = self.k_scale[i] if self.k_scale is not None else None
        vs = self.v_scale[i] if self.v_scale is not None else None
        SV.kv_append(qkv, cfg.num_heads, cfg.num_kv_heads, cfg.head_dim, slots, self.k_cache[i],
                     self.v_cache[i], ks, vs, self.kv_dtype)
        o = attn(i, qkv)
        M = h.shape[0]
        self._row_parallel(o, p + "wo", c.partial(M))
        h2, xn2 = torch.empty_like(h), torch.empty_like(h)
        c.allreduce_norm(M, h2, h, self.W[p + "ffn_norm"], xn2, cfg.norm_eps)
        w = self.W[p + "wgu"]
        if isinstance(w, SV.QuantizedWeight):
            a = E.swiglu_fwd(self._linear(xn2, p + "wgu"))
        else:
            from ..ops import gemm as G
            _, a = G.linear_swiglu(xn2, w)
        self._row_parallel(a, p + "wdown", c.partial(M))
        last = i == cfg.num_layers - 1
        g = self.W["final_norm"] if last else self.W[f"layers.{i + 1}.attn_norm"]
        h3, xn3 = torch.empty_like(h), torch.empty_like(h)
        c.allreduce_norm(M, h3, h2, g, xn3, cfg.norm_eps)
        self._xn = None if last else xn3
        return h3

    def _row_parallel(self, x: torch.Tensor, name: str, part: torch.Tensor) -> None:
        y = self._linear(x, name, out=part)
        if y.data_ptr() != part.data_ptr():
            part.copy_(y)

    def prefill(self, items: List[PrefillItem]):
        self._xn = None
        return super().prefill(items)

    def decode(self, tokens, positions, slots, block_tables):
        self._xn = None
        return super().decode(tokens, positions, slots, block_tables)

    def sample(self, logits: torch.Tensor, temps: Optional[List[float]], seed: int) -> torch.Tensor:
        n = logits.shape[0]
        t = None if temps is None else torch.tensor(temps, dtype=torch.float32, device=logits.device)
        val = torch.empty(n, dtype=torch.float32, device=logits.device)
        tok = SV.sample(logits, t, seed, v0=self.rank * self.vocab_local, out_val=val)
        mine = torch.stack([val.double(), tok.double()], 1)
        allp = torch.empty(self.tp, n, 2, dtype=torch.float64, device=logits.device)
        dist.all_gather_into_tensor(allp, mine, group=self.comm.group)
        return pick_global(allp)


def pick_global(allp: torch.Tensor) -> torch.Tensor:
    """allp [ranks, rows, (score, token id)] -> the token of the best score per row;
    ties go to the lowest rank, i.e. the lowest token id (slices are in rank order)."""
    best = allp[:, :, 0].argmax(0)  # argmax returns the first maximum
    return allp[best, torch.arange(allp.shape[1], device=allp.device), 1].long()


# Runner calls travel rank 0 -> workers on the CPU (gloo) group as a 2-int64
# header (op, payload length) and, for decode and sample, one flat int32 payload:
#   decode  [n, max_blocks, tokens(n), positions(n), slots(n), block table (n x max_blocks)]
#   sample  [seed low 32 bits, seed high 32 bits, has temperatures, temperatures as float32 bits (n)]
# Prefill items (rarer, ragged) still go as one pickled object.
OP_STOP, OP_DECODE, OP_SAMPLE, OP_PREFILL = 0, 1, 2, 3


def pack_decode(tokens, positions, slots, block_tables) -> np.ndarray:
    n = len(tokens)
    mb = max(len(t) for t in block_tables)
    pk = np.zeros(2 + 3 * n + n * mb, dtype=np.int32)
    pk[0], pk[1] = n, mb
    pk[2:2 + n] = tokens
    pk[2 + n:2 + 2 * n] = positions
    pk[2 + 2 * n:2 + 3 * n] = slots
    bt = pk[2 + 3 * n:].reshape(n, mb)
    for k, t in enumerate(block_tables):
        bt[k, :len(t)] = t
    return pk


def unpack_decode(pk: np.ndarray):
    n, mb = int(pk[0]), int(pk[1])
    return (pk[2:2 + n], pk[2 + n:2 + 2 * n], pk[2 + 2 * n:2 + 3 * n], pk[2 + 3 * n:].reshape(n, mb))


def pack_sample(temps, seed: int) -> np.ndarray:
    n = 0 if temps is None else len(temps)
    pk = np.zeros(3 + n, dtype=np.int32)
    s = int(seed) & 0xFFFFFFFFFFFFFFFF
    pk[0] = np.int64(s & 0xFFFFFFFF).astype(np.uint32).view(np.int32)
    pk[1] = np.int64(s >> 32).astype(np.uint32).view(np.int32)
    pk[2] = 0 if temps is None else 1
    if n:
        pk[3:] = np.asarray(temps, dtype=np.float32).view(np.int32)
    return pk


def unpack_sample(pk: np.ndarray):
    seed = int(pk[0].view(np.uint32)) | (int(pk[1].view(np.uint32)) << 32)
    temps = pk[3:].view(np.float32).tolist() if pk[2] else None
    return temps, seed


def _send(op: int, payload: Optional[np.ndarray], group) -> None:
    hdr = torch.tensor([op, 0 if payload is None else payload.size], dtype=torch.int64)
    dist.broadcast(hdr, src=0, group=group)
    if payload is not None and payload.size:
        dist.broadcast(torch.from_numpy(payload), src=0, group=group)


def _recv(group):
    hdr = torch.empty(2, dtype=torch.int64)
    dist.broadcast(hdr, src=0, group=group)
    op, n = int(hdr[0]), int(hdr[1])
    payload = None
    if n:
        buf = torch.empty(n, dtype=torch.int32)
        dist.broadcast(buf, src=0, group=group)
        payload = buf.numpy()
    return op, payload


class RunnerProxy:
    """Rank 0's stand-in for the runner: sends every call to the workers (CPU
    group) and runs it on its own shard from the same message."""

    supports_top_p = False

    def __init__(self, runner: TPModelRunner, ctrl_group):
        self.runner = runner
        self.ctrl = ctrl_group
        self.num_blocks = runner.num_blocks
        self.block_size = runner.block_size
        self._logits = None

    def prefill(self, items):
        _send(OP_PREFILL, None, self.ctrl)
        dist.broadcast_object_list([items], src=0, group=self.ctrl)
        seq_ids, self._logits = self.runner.prefill(items)
        return seq_ids, self._logits

    def decode(self, tokens, positions, slots, block_tables):
        pk = pack_decode(tokens, positions, slots, block_tables)
        _send(OP_DECODE, pk, self.ctrl)
        self._logits = self.runner.decode(*unpack_decode(pk))
        return self._logits

    def sample(self, logits, temps, seed):
        _send(OP_SAMPLE, pack_sample(temps, seed), self.ctrl)
        return self.runner.sample(logits, temps, seed)

    def weight_bytes(self) -> int:
        return self.runner.weight_bytes()

    def stop(self) -> None:
        _send(OP_STOP, None, self.ctrl)


def worker_loop(runner: TPModelRunner, ctrl_group) -> None:
    """Ranks > 0: execute rank 0's runner calls until it says stop."""
    logits = None
    while True:
        op, payload = _recv(ctrl_group)
        if op == OP_STOP:
            return
        if op == OP_PREFILL:
            obj = [None]
            dist.broadcast_object_list(obj, src=0, group=ctrl_group)
            _, logits = runner.prefill(obj[0])
        elif op == OP_DECODE:
            logits = runner.decode(*unpack_decode(payload))
        elif op == OP_SAMPLE:
            runner.sample(logits, *unpack_sample(payload))
        else:
            raise RuntimeError(f"unknown runner call {op}")


def tp_params_from_state_dict(cfg: TransformerConfig, sd: Dict[str, torch.Tensor], tp: int, rank: int,
                              device) -> "TPParams":
    """This rank's shard of a reference-named state dict (a checkpoint's
    model.safetensors): the full weights are laid out once on `device`, the
    rank's slices copied out, and the full copy dropped."""
    from ..models.params import FlatParams
    from ..parallel.tp import TPParams
    full = FlatParams(cfg, device)
    full.load_reference_state_dict({k: v.to(device) for k, v in sd.items()})
    params = TPParams(cfg, tp, rank, device)
    params.load_full(full)
    del full
    return params


def build_tp_runner(cfg: TransformerConfig, seed: int, *, weights: str = "none", kv_dtype: str = "fp8",
                    group_size: int = 128, block_size: int = 16, max_model_len: int = 4096,
                    max_rows: int = 8192, num_blocks: int = 0, device=None, params=None,
                    cuda_graphs: bool = True, max_batch: int = 256):
    """This rank's TPModelRunner (weights initialised as FlatParams(cfg).init_(seed)
    would, then sharded) plus the CPU control group."""
    from ..parallel.tp import TPParams
    dev = torch.device(device or torch.cuda.current_device())
    tp, rank = dist.get_world_size(), dist.get_rank()
    comm = TPServeComm(cfg.hidden_dim, max_rows, dev)
    if params is None:
        params = TPParams(cfg, tp, rank, dev)
        params.init_(seed, cfg.init_std)
    runner = TPModelRunner(cfg, params, comm, dev, kv_dtype=kv_dtype, weights=weights, group_size=group_size,
                           num_blocks=num_blocks, block_size=block_size, max_model_len=max_model_len)
    if cuda_graphs:
        runner.enable_graphs(max_batch)  # every rank captures the same buckets in the same order
    ctrl = dist.new_group(backend="gloo")
    return runner, ctrl
