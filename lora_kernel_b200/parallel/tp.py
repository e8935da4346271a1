"""Tensor parallelism (Megatron column/row-parallel linears with sequence
parallelism) on the fused collective GEMMs.

Layout (tp ranks, rank r):
  * the residual stream, norms and the embedding lookup are sequence-sharded:
    rank r owns token rows [r*R, (r+1)*R) of the flattened batch (R = T / tp);
  * column-parallel linears (Wqkv by heads, Wgate|up by FFN blocks, the LM head
    by vocabulary rows) consume the all-gathered normalised activations
    through K16 - the all-gather runs inside the GEMM: a copy warp per CTA pulls
    peers' rows over NVLink into the local A buffer, and the TMA producer starts
    on a 128-row block as soon as its counter says it has landed;
  * row-parallel linears (Wo, Wdown, and every dgrad of a column-parallel
    linear) run K18 - the GEMM epilogue stores each output row block straight
    into its owner's receive slot in peer memory; the owner then sums the slots
    in fixed rank order fused with the residual add and the next RMSNorm,
    writing the normalised rows into the symmetric staging buffer the next K16
    reads (csrc/tp.cu);
  * the LM head is vocabulary-parallel and the cross-entropy combines per-row
    statistics from every rank through peer memory (no logits all-gather);
  * replicated parameters (embedding, norms) get their gradients summed by the
    one-shot peer-memory all-reduce (K12) at the end of the accumulation window.

`comm="nccl"` runs the same schedule on NCCL all-gather / reduce-scatter with
plain GEMMs: the baseline the fused kernels are measured against.

Hazards: every buffer a peer reads (staging rows, receive slots, CE
statistics) is rewritten only after a device barrier that follows the peers'
last read of it; the schedule alternates two staging and two receive buffers
so that one barrier per hand-off suffices.

Reference: ColumnParallelLinear / RowParallelLinear / TensorParallelTransformer
(include/distributed/tensor_parallel.hpp:14-104) - a forward-only column/row
split with an all-gather / all-reduce around a plain matmul.
"""
from __future__ import annotations

import copy
import os
from collections import OrderedDict
from typing import Dict, List, Optional, Tuple

import torch
import torch.distributed as dist

from .._ext import C, check_status, status
from ..config import TransformerConfig
from ..models.params import ALIGN, ParamSpec, build_layout
from ..ops import attention as A
from ..ops import elementwise as E
from ..ops import gemm as G
from ..ops import norm as N
from ..ops.gemm import EPI
from . import comm as CM

SLOT_TP = 5


def _round(n: int) -> int:
    return (n + ALIGN - 1) // ALIGN * ALIGN


def check_tp_config(cfg: TransformerConfig, tp: int) -> None:
    if cfg.num_heads % tp or cfg.num_kv_heads % tp:
        raise ValueError(f"tp={tp} must divide the query and KV head counts")
    if cfg.ff_dim_padded % (128 * tp):
        raise ValueError(f"tp={tp}: padded FFN width {cfg.ff_dim_padded} must split into 128-row blocks")
    if cfg.vocab_size % (8 * tp):
        raise ValueError(f"tp={tp}: vocabulary {cfg.vocab_size} must split into multiples of 8")


# --------------------------------------------------------------------- layout
def build_tp_layout(cfg: TransformerConfig, tp: int) -> Tuple[List[ParamSpec], int, int]:
    """Local parameter layout of one TP rank.  Replicated tensors first (so
    their gradients are one contiguous range for the all-reduce), then the
    sharded ones.  Returns (specs, replicated numel, total numel)."""
    check_tp_config(cfg, tp)
    D, V = cfg.hidden_dim, cfg.vocab_size
    Fl = cfg.ff_dim_padded // tp
    ql, kvl = cfg.q_dim // tp, cfg.kv_dim // tp
    specs: List[ParamSpec] = []
    off = 0

    def add(name, shape, group, decay, init):
        nonlocal off
        s = ParamSpec(name, tuple(shape), off, group, decay, init)
        specs.append(s)
        off += _round(s.numel)

    add("embed", (V, D), "replicated", True, "normal")
    for i in range(cfg.num_layers):
        add(f"layers.{i}.attn_norm", (D,), "replicated", False, "ones")
        add(f"layers.{i}.ffn_norm", (D,), "replicated", False, "ones")
    add("final_norm", (D,), "replicated", False, "ones")
    n_rep = off
    for i in range(cfg.num_layers):
        p = f"layers.{i}."
        add(p + "wqkv", (ql + 2 * kvl, D), f"layers.{i}", True, "normal")
        add(p + "wo", (D, ql), f"layers.{i}", True, "normal")
        add(p + "wgu", (2 * Fl, D), f"layers.{i}", True, "normal")
        add(p + "wdown", (D, Fl), f"layers.{i}", True, "normal")
    if not cfg.tie_embeddings:
        add("lm_head", (V // tp, D), "head", True, "normal")
    return specs, n_rep, off


def shard_tensor(cfg: TransformerConfig, name: str, full: torch.Tensor, r: int, tp: int) -> torch.Tensor:
    """Rank r's piece of a full (engine-layout) tensor."""
    q, kv = cfg.q_dim, cfg.kv_dim
    ql, kvl = q // tp, kv // tp
    Fl = cfg.ff_dim_padded // tp
    if name.endswith("wqkv"):
        return torch.cat([full[r * ql:(r + 1) * ql], full[q + r * kvl:q + (r + 1) * kvl],
                          full[q + kv + r * kvl:q + kv + (r + 1) * kvl]])
    if name.endswith(".wo"):
        return full[:, r * ql:(r + 1) * ql]
    if name.endswith("wgu"):  # blocked gate|up layout: rank r owns a contiguous run of blocks
        return full[r * 2 * Fl:(r + 1) * 2 * Fl]
    if name.endswith("wdown"):
        return full[:, r * Fl:(r + 1) * Fl]
    if name == "lm_head":
        Vl = cfg.vocab_size // tp
        return full[r * Vl:(r + 1) * Vl]
    return full


def unshard_tensor(cfg: TransformerConfig, name: str, pieces: List[torch.Tensor]) -> torch.Tensor:
    """Inverse of shard_tensor over all ranks' pieces (rank order)."""
    tp = len(pieces)
    if name.endswith("wqkv"):
        ql, kvl = cfg.q_dim // tp, cfg.kv_dim // tp
        qs = [p[:ql] for p in pieces]
        ks = [p[ql:ql + kvl] for p in pieces]
        vs = [p[ql + kvl:] for p in pieces]
        return torch.cat(qs + ks + vs)
    if name.endswith(".wo") or name.endswith("wdown"):
        return torch.cat(pieces, dim=1)
    if name.endswith("wgu") or name == "lm_head":
        return torch.cat(pieces, dim=0)
    return pieces[0]


class TPParams:
    """Flat local parameter buffer of one TP rank with named views."""

    def __init__(self, cfg: TransformerConfig, tp: int, rank: int, device, dtype=torch.bfloat16,
                 buffer: Optional[torch.Tensor] = None):
        self.cfg, self.tp, self.rank = cfg, tp, rank
        self.specs, self.n_rep, self.numel = build_tp_layout(cfg, tp)
        self.by_name = {s.name: s for s in self.specs}
        self.flat = torch.zeros(self.numel, dtype=dtype, device=device) if buffer is None else buffer
        assert self.flat.numel() == self.numel
        self.views: Dict[str, torch.Tensor] = {
            s.name: self.flat[s.offset:s.offset + s.numel].view(s.shape) for s in self.specs}
        Vl = cfg.vocab_size // tp
        if cfg.tie_embeddings:  # the vocabulary-parallel head is this rank's rows of the embedding
            self.views["lm_head"] = self.views["embed"][rank * Vl:(rank + 1) * Vl]

    def __getitem__(self, name: str) -> torch.Tensor:
        return self.views[name]

    def like(self, dtype=torch.float32, buffer: Optional[torch.Tensor] = None) -> "TPParams":
        return TPParams(self.cfg, self.tp, self.rank, self.flat.device, dtype,
                        buffer if buffer is not None else torch.zeros(self.numel, dtype=dtype,
                                                                      device=self.flat.device))

    def segments(self, lo: int = 0, hi: Optional[int] = None):
        hi = self.numel if hi is None else hi
        out = []
        for s in self.specs:
            a, b = max(s.offset, lo), min(s.offset + s.numel, hi)
            if a < b:
                out.append((a - lo, b - a, s.decay))
        return out

    @torch.no_grad()
    def load_full(self, full) -> None:
        """Copy this rank's shards out of a full FlatParams (same cfg)."""
        for s in self.specs:
            self.views[s.name].copy_(shard_tensor(self.cfg, s.name, full[s.name], self.rank, self.tp))

    @torch.no_grad()
    def init_(self, seed: int, std: float) -> None:
        """The shards of exactly the weights FlatParams(cfg).init_(seed, std)
        produces (same per-tensor generators), one full tensor at a time."""
        from ..models.params import FlatParams
        full_specs, _, _ = build_layout(self.cfg)
        idx = {s.name: k for k, s in enumerate(full_specs)}
        cfg = self.cfg
        F, Fp = cfg.ff_dim, cfg.ff_dim_padded
        dev = self.flat.device
        for s in self.specs:
            fs = full_specs[idx[s.name]]
            if fs.init == "ones":
                self.views[s.name].fill_(1.0)
                continue
            g = torch.Generator(device=dev).manual_seed(seed * 1000003 + idx[s.name])
            t = torch.empty(fs.shape, dtype=torch.float32, device=dev)
            t.normal_(0.0, std, generator=g)
            if s.name.endswith("wgu") and Fp != F:
                blk = t.view(Fp // 128, 2, 128, -1)
                mask = (torch.arange(Fp, device=dev) >= F).view(Fp // 128, 128)
                blk[:, 0][mask] = 0.0
                blk[:, 1][mask] = 0.0
            if s.name.endswith("wdown") and Fp != F:
                t[:, F:] = 0.0
            self.views[s.name].copy_(shard_tensor(cfg, s.name, t, self.rank, self.tp).to(self.flat.dtype))
            del t


# ------------------------------------------------------------ communication
class TPComm:
    """Symmetric buffers and the fused-collective launch helpers of one TP group."""

    def __init__(self, cfg: TransformerConfig, max_tokens: int, device, group=None, comm: str = "p2p"):
        self.cfg = cfg
        self.device = torch.device(device)
        self.group = group or dist.group.WORLD
        self.tp = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        self.comm = comm
        if max_tokens % (128 * self.tp):
            raise ValueError(f"tokens per micro-batch ({max_tokens}) must be a multiple of 128 x tp")
        self.max_tokens = max_tokens
        D = cfg.hidden_dim
        R = max_tokens // self.tp
        self.pc = CM.PeerComm(self.device, self.group)
        self.stage = [CM.SymBuffer(R * D, torch.bfloat16, self.device, self.group) for _ in range(2)]
        self.recv = [CM.SymBuffer(max_tokens * D, torch.bfloat16, self.device, self.group) for _ in range(2)]
        self.stats = CM.SymBuffer(max_tokens * 4, torch.float32, self.device, self.group)
        # fp8 staging (created on first use): e4m3 rows [R, D] and their 1x128 scales [D/128, R]
        self.stage8: List = []
        self.sscale: List = []
        self.count = torch.zeros(max_tokens // 128, dtype=torch.int32, device=self.device)
        self._nccl_tmp: Dict[Tuple[int, int], torch.Tensor] = {}
        self._tmaps: Dict[Tuple[int, int, int], torch.Tensor] = {}
        torch.cuda.synchronize(self.device)
        dist.barrier(self.group)

    # ------------------------------------------------------------- views
    def stage_view(self, k: int, rows: int, cols: int) -> torch.Tensor:
        return self.stage[k].local[:rows * cols].view(rows, cols)

    def recv_view(self, k: int, rows: int, cols: int) -> torch.Tensor:
        return self.recv[k].local[:self.tp * rows * cols].view(self.tp * rows, cols)

    def barrier(self) -> None:
        if self.comm == "nccl":
            return  # NCCL collectives synchronise by themselves
        self.pc.barrier(SLOT_TP)

    # ------------------------------------------------ fp8 (K2) variants
    def _fp8_bufs(self) -> None:
        if not self.stage8:
            R, D = self.max_tokens // self.tp, self.cfg.hidden_dim
            self.stage8 = [CM.SymBuffer(R * D, torch.uint8, self.device, self.group) for _ in range(2)]
            self.sscale = [CM.SymBuffer((D // 128) * R, torch.float32, self.device, self.group) for _ in range(2)]
            torch.cuda.synchronize(self.device)
            dist.barrier(self.group)

    def publish_fp8(self, k: int, rows: torch.Tensor) -> None:
        """Quantise this rank's staging rows (bf16 [R, D]) into fp8 staging k."""
        self._fp8_bufs()
        R, D = rows.shape
        q = self.stage8[k].local[:R * D].view(R, D)
        sc = self.sscale[k].local[:(D // 128) * R].view(D // 128, R)
        C().quant_1x128(rows, 0, q, sc)

    def ag_gemm_fp8(self, k: int, dst8: torch.Tensor, dsts: torch.Tensor, w8, out: torch.Tensor) -> None:
        """dst8 / dsts <- all-gather of every rank's fp8 staging rows / scales; out = dst . W^T
        (block-scaled fp8), the gather fused into the GEMM."""
        T, K = dst8.shape
        R = T // self.tp
        C().gemm_fp8_comm(dst8, dsts, 0, w8.q, w8.scale, out, status(self.device), self.rank, self.tp,
                          self.stage8[k].ptrs, self.sscale[k].ptrs, R, self.count, None, 0, 0)

    def gemm_rs_fp8(self, k: int, a: torch.Tensor, w8) -> None:
        """a (bf16, quantised here to e4m3 1x128) . W^T as block-scaled fp8, the bf16 rows
        stored straight into their owner's receive buffer k (reduce-scatter epilogue)."""
        from ..ops.fp8 import quantize_1x128
        T = a.shape[0]
        R, Nc = T // self.tp, w8.N
        q, sc = quantize_1x128(a)
        C().gemm_fp8_comm(q, sc, 0, w8.q, w8.scale, None, status(self.device), self.rank, self.tp,
                          None, None, 0, None, self.recv[k].ptrs, R, Nc)

    # ------------------------------------- MX fp8 (hardware block scaling)
    def _mx_bufs(self) -> None:
        if not getattr(self, "stage_mx", None):
            from ..ops.fp8 import sf_tile_bytes
            R, D = self.max_tokens // self.tp, self.cfg.hidden_dim
            # gathered operands are [R, D] rows: normalised inputs (e4m3) and residual gradients (e5m2)
            self.stage_mx = [CM.SymBuffer(R * D, torch.uint8, self.device, self.group) for _ in range(2)]
            self.ssf_mx = [CM.SymBuffer(sf_tile_bytes(R, D), torch.uint8, self.device, self.group)
                           for _ in range(2)]
            torch.cuda.synchronize(self.device)
            dist.barrier(self.group)

    def publish_mx(self, k: int, rows: torch.Tensor, fmt: int = 0) -> None:
        """Quantise this rank's rows (bf16 [R, K]: e4m3 activations or e5m2 gradients,
        one power-of-two scale per 128 block) into MX staging k."""
        from ..ops.fp8 import sf_tile_bytes
        self._mx_bufs()
        R, K = rows.shape
        q = self.stage_mx[k].local[:R * K].view(R, K)
        sf = self.ssf_mx[k].local[:sf_tile_bytes(R, K)]
        C().quant_mx_rows(rows, fmt, q, sf, R)

    def ag_gemm_mx(self, k: int, dst8: torch.Tensor, dstsf: torch.Tensor, b8: torch.Tensor, bsf: torch.Tensor,
                   out: torch.Tensor, a_fmt: int = 0) -> None:
        """dst8 / dstsf <- all-gather of every rank's MX staging rows / SF tiles;
        out = dst . B^T (tcgen05 block-scaled), the gather fused into the GEMM."""
        T = dst8.shape[0]
        C().gemm_mxf8(dst8, dstsf, int(a_fmt), b8, bsf, 0, out, None, status(self.device), self.rank, self.tp,
                      self.stage_mx[k].ptrs, self.ssf_mx[k].ptrs, T // self.tp, self.count, None, 0, 0)

    def gemm_rs_mx(self, k: int, a: torch.Tensor, b8: torch.Tensor, bsf: torch.Tensor, a_fmt: int = 0) -> None:
        """a (bf16, quantised here) . B^T as a block-scaled fp8 GEMM whose epilogue
        stores the bf16 rows into their owner's receive buffer k."""
        from ..ops.fp8 import quantize_mx
        T, Nc = a.shape[0], b8.shape[0]
        q, sf = quantize_mx(a, a_fmt)
        C().gemm_mxf8(q, sf, int(a_fmt), b8, bsf, 0, None, None, status(self.device), self.rank, self.tp,
                      None, None, 0, None, self.recv[k].ptrs, T // self.tp, Nc)

    # --------------------------------------------------- K16 AG -> GEMM
    def ag_gemm(self, k: int, dst: torch.Tensor, w: torch.Tensor, out: torch.Tensor,
                epi: str = "bf16", h_out: Optional[torch.Tensor] = None) -> None:
        """dst <- all-gather of every rank's staging rows k; out = dst @ w^T.
        The caller has written its own rows into stage k and called barrier()."""
        T, K = dst.shape
        R = T // self.tp
        if self.comm == "nccl":
            dist.all_gather_into_tensor(dst, self.stage_view(k, R, K), group=self.group)
            G.gemm(dst, w, out, epi=epi, h_out=h_out)
            return
        C().gemm_ag(dst, w, out, EPI[epi], h_out, self.stage[k].ptrs, K, R, self.rank, self.count,
                    (self.rank * R) // 128, status(self.device), 0)

    # --------------------------------------------------- K18 GEMM -> RS
    def gemm_rs(self, k: int, a: torch.Tensor, w: torch.Tensor) -> None:
        """Partial a @ w^T; rows go to their owner's receive buffer k, slot = rank."""
        T, Nc = a.shape[0], w.shape[0]
        R = T // self.tp
        if self.comm == "nccl":
            full = self._tmp((T, Nc))
            G.gemm(a, w, full)
            dist.reduce_scatter_tensor(self.recv_view(k, R, Nc)[:R], full, group=self.group)
            return
        C().gemm_rs(a, w, self.recv[k].ptrs, R, self.rank, Nc, ((self.rank + 1) % self.tp) * R // 128,
                    status(self.device), 0, self._maps(k, R, Nc))

    def _maps(self, k: int, R: int, Nc: int):
        """Per-owner TMA store maps of receive buffer k viewed as [tp*R, Nc]
        (LK_TMA_STORE=0 selects the generic-store epilogue)."""
        if os.environ.get("LK_TMA_STORE", "1") == "0":
            return None
        key = (k, R, Nc)
        m = self._tmaps.get(key)
        if m is None:
            m = C().make_remote_maps(self.recv[k].ptrs_host, self.tp * R, Nc, Nc, self.device)
            self._tmaps[key] = m
        return m

    def rs_sum(self, k: int, out: torch.Tensor, resid: Optional[torch.Tensor] = None,
               gamma: Optional[torch.Tensor] = None, y: Optional[torch.Tensor] = None,
               rstd: Optional[torch.Tensor] = None, eps: float = 1e-5) -> None:
        """After gemm_rs(k): out = sum of the slots (+ resid); y = rmsnorm(out)."""
        R, Nc = out.shape
        self.barrier()
        world = 1 if self.comm == "nccl" else self.tp
        C().rs_sum(self.recv_view(k, R, Nc), world, out, resid, gamma, y, rstd, float(eps), 0, None, 0)

    def _tmp(self, shape) -> torch.Tensor:
        t = self._nccl_tmp.get(shape)
        if t is None:
            t = torch.empty(shape, dtype=torch.bfloat16, device=self.device)
            self._nccl_tmp[shape] = t
        return t

    # ------------------------------------------------ vocab-parallel CE
    def cross_entropy(self, logits: torch.Tensor, targets: torch.Tensor, loss_acc: torch.Tensor, *,
                      scale: Optional[torch.Tensor], scale_mul: float, smoothing: float = 0.0,
                      z_loss: float = 0.0, ignore_index: int = -100) -> None:
        T, Vl = logits.shape
        v0 = self.rank * Vl
        st = self.stats.local[:T * 4]
        args = (targets, loss_acc, scale, float(scale_mul), float(smoothing), float(z_loss),
                int(ignore_index), True, v0, Vl * self.tp)
        if self.comm == "nccl":
            C().cross_entropy_vp(logits, *args, st, self._self_ptr(), 1)
            allst = self._tmp_f32((self.tp * T * 4,))
            dist.all_gather_into_tensor(allst, st, group=self.group)
            ptrs = self._ptrs_of(allst, T * 4)
            C().cross_entropy_vp(logits, *args, st, ptrs, 2)
            return
        C().cross_entropy_vp(logits, *args, st, self.stats.ptrs, 1)
        self.barrier()
        C().cross_entropy_vp(logits, *args, st, self.stats.ptrs, 2)

    def _self_ptr(self) -> torch.Tensor:
        if not hasattr(self, "_selfp"):
            self._selfp = torch.tensor([self.stats.local.data_ptr()], dtype=torch.int64, device=self.device)
        return self._selfp

    def _tmp_f32(self, shape) -> torch.Tensor:
        key = ("f32",) + tuple(shape)
        t = self._nccl_tmp.get(key)
        if t is None:
            t = torch.empty(shape, dtype=torch.float32, device=self.device)
            self._nccl_tmp[key] = t
        return t

    def _ptrs_of(self, buf: torch.Tensor, stride: int) -> torch.Tensor:
        key = ("ptrs", buf.data_ptr(), stride)
        t = self._nccl_tmp.get(key)
        if t is None:
            base = buf.data_ptr()
            t = torch.tensor([base + 4 * stride * p for p in range(self.tp)], dtype=torch.int64,
                             device=self.device)
            self._nccl_tmp[key] = t
        return t


# ------------------------------------------------------------------- model
class _TPWorkspace:
    def __init__(self, cfg: TransformerConfig, tp: int, B: int, S: int, device, fp8=False):
        T = B * S
        R = T // tp
        D = cfg.hidden_dim
        L = cfg.num_layers
        ql, kvl = cfg.q_dim // tp, cfg.kv_dim // tp
        Fl = cfg.ff_dim_padded // tp
        Vl = cfg.vocab_size // tp
        bf = dict(dtype=torch.bfloat16, device=device)
        f32 = dict(dtype=torch.float32, device=device)
        self.B, self.S, self.T, self.R = B, S, T, R
        self.h = [torch.empty(R, D, **bf) for _ in range(L + 1)]      # residual stream (local rows)
        self.hmid = [torch.empty(R, D, **bf) for _ in range(L)]
        self.rstd1 = [torch.empty(R, **f32) for _ in range(L)]
        self.rstd2 = [torch.empty(R, **f32) for _ in range(L)]
        self.rstdf = torch.empty(R, **f32)
        if fp8 == "mx":
            # gathered normalised inputs as e4m3 + SF tiles (power-of-two 1x128
            # scales), gathered e5m2 gradients for the data-gradient GEMMs; bf16
            # copies of the inputs are rebuilt right before each weight gradient
            from ..ops.fp8 import sf_tile_bytes
            u8 = dict(dtype=torch.uint8, device=device)
            Fl = cfg.ff_dim_padded // tp
            self.xn1_8 = [torch.empty(T, D, **u8) for _ in range(L)]
            self.xn2_8 = [torch.empty(T, D, **u8) for _ in range(L)]
            self.xn1_s = [torch.empty(sf_tile_bytes(T, D), **u8) for _ in range(L)]
            self.xn2_s = [torch.empty(sf_tile_bytes(T, D), **u8) for _ in range(L)]
            self.xn_deq = torch.empty(T, D, **bf)
            self.dfull8 = torch.empty(T, D, **u8)
            self.dfull_s = torch.empty(sf_tile_bytes(T, D), **u8)
            self.xn1 = self.xn2 = None
        elif fp8:
            # gathered normalised inputs as e4m3 + 1x128 scales; bf16 copies are
            # rebuilt (dequantised) right before each weight-gradient GEMM
            u8 = dict(dtype=torch.uint8, device=device)
            self.xn1_8 = [torch.empty(T, D, **u8) for _ in range(L)]
            self.xn2_8 = [torch.empty(T, D, **u8) for _ in range(L)]
            self.xn1_s = [torch.empty(D // 128, T, **f32) for _ in range(L)]
            self.xn2_s = [torch.empty(D // 128, T, **f32) for _ in range(L)]
            self.xn_deq = torch.empty(T, D, **bf)
            self.xn1 = self.xn2 = None
        else:
            self.xn1 = [torch.empty(T, D, **bf) for _ in range(L)]    # gathered normalised inputs
            self.xn2 = [torch.empty(T, D, **bf) for _ in range(L)]
        self.xf = torch.empty(T, D, **bf)
        self.qkv = [torch.empty(T, ql + 2 * kvl, **bf) for _ in range(L)]
        self.o = [torch.empty(T, ql, **bf) for _ in range(L)]
        self.lse = [torch.empty(B, cfg.num_heads // tp, S, **f32) for _ in range(L)]
        self.gu = [torch.empty(T, 2 * Fl, **bf) for _ in range(L)]
        self.act = [torch.empty(T, Fl, **bf) for _ in range(L)]
        self.logits = torch.empty(T, Vl, **bf)
        self.loss_acc = torch.zeros(2, **f32)
        self.dfull = torch.empty(T, D, **bf)       # gathered residual gradient
        self.dx = torch.empty(R, D, **bf)
        self.dact = torch.empty(T, Fl, **bf)
        self.dgu = torch.empty(T, 2 * Fl, **bf)
        self.do = torch.empty(T, ql, **bf)
        self.dqkv = torch.empty(T, ql + 2 * kvl, **bf)


class TPLlamaModel:
    """Llama decoder sharded over a TP group (one process per GPU).

    forward_backward(ids, targets) takes the FULL micro-batch [B, S] on every
    rank (every rank reads its own token rows of it) and returns the loss
    accumulator [sum of token losses, count] - identical on every rank."""

    def __init__(self, cfg: TransformerConfig, comm: TPComm, params: Optional[TPParams] = None,
                 seed: int = 1234, grads: Optional[TPParams] = None, fp8=False):
        """fp8: the four projections of every layer run as block-scaled fp8 GEMMs
        (e4m3 activations in 1x128 blocks, e4m3 weights in 128x128 blocks) with the
        all-gather / reduce-scatter fused in (the gather moves fp8 rows + scales,
        half the bf16 bytes).
          "mx" (or True): power-of-two scales applied by the tensor core
            (tcgen05 block-scaled MMA); the backward data-gradient GEMMs run the
            same way on e5m2 gradients (gathered or reduce-scattered as fp8);
            weight gradients are bf16 GEMMs on the dequantised fp8 operands.
          "exact": fp32 scales, each 128-wide K block promoted on the CUDA cores;
            backward data-gradient GEMMs and weight gradients stay bf16, the
            latter on the dequantised forward inputs."""
        self.cfg = cfg
        if fp8 is True:
            fp8 = "mx"
        if fp8 not in (False, None, "mx", "exact"):
            raise ValueError(f"fp8 must be False, 'mx' or 'exact', got {fp8!r}")
        self.fp8 = fp8 or False
        self.mx = fp8 == "mx"
        if fp8 and comm.comm != "p2p":
            raise ValueError("the fp8 tensor-parallel path runs on the peer-memory kernels (comm='p2p')")
        self.comm = comm
        self.tp, self.rank = comm.tp, comm.rank
        self.device = comm.device
        check_tp_config(cfg, self.tp)
        if params is None:
            params = TPParams(cfg, self.tp, self.rank, self.device)
            params.init_(seed, cfg.init_std)
        self.params = params
        self.grads = grads if grads is not None else params.like(torch.float32)
        self.rope = E.rope_table(max(cfg.max_seq_len, 1), cfg.head_dim, cfg.rope_base, self.device)
        self._ws: Dict[Tuple[int, int], _TPWorkspace] = {}
        self._overwrite = False
        self._w8 = None         # fp8 weight copies (see _forward)
        self._w8_fresh = True

    def workspace(self, B: int, S: int) -> _TPWorkspace:
        ws = self._ws.get((B, S))
        if ws is None:
            if B * S > self.comm.max_tokens:
                raise ValueError(f"micro-batch of {B * S} tokens exceeds the TP buffers ({self.comm.max_tokens})")
            if S > self.rope.shape[0]:
                self.rope = E.rope_table(S, self.cfg.head_dim, self.cfg.rope_base, self.device)
            ws = _TPWorkspace(self.cfg, self.tp, B, S, self.device, fp8=self.fp8)
            self._ws[(B, S)] = ws
        return ws

    def _p(self, n):
        return self.params[n]

    def _g(self, n):
        return self.grads[n]

    def _wgrad(self, dy, x, name):
        G.gemm(dy.t(), x.t(), self._g(name), epi="f32" if self._overwrite else "f32_acc")

    # -------------------------------------------------------------- forward
    def _forward(self, ids: torch.Tensor, ws: _TPWorkspace) -> None:
        cfg, c = self.cfg, self.comm
        R, D, eps = ws.R, cfg.hidden_dim, cfg.norm_eps
        Hl, Hkvl = cfg.num_heads // self.tp, cfg.num_kv_heads // self.tp
        ids_local = ids.reshape(-1)[self.rank * R:(self.rank + 1) * R]
        E.embedding_fwd(ids_local, self._p("embed"), out=ws.h[0])
        N.rmsnorm_fwd(ws.h[0], self._p("layers.0.attn_norm"), eps, y=c.stage_view(0, R, D), rstd=ws.rstd1[0])
        # fp8 copies of the projection weights: made on the first micro-step of an
        # accumulation window (the weights only change between windows) and
        # reused by the window's later micro-steps
        if self.fp8 and (self._w8 is None or self._w8_fresh):
            from ..ops.fp8 import Fp8Weight, MXWeight
            make = (lambda w: MXWeight(w, transpose=True)) if self.mx else \
                (lambda w: Fp8Weight(w, transpose=False))
            self._w8 = {f"layers.{i}.{t}": make(self._p(f"layers.{i}.{t}"))
                        for i in range(cfg.num_layers) for t in ("wqkv", "wo", "wgu", "wdown")}
        for i in range(cfg.num_layers):
            p = f"layers.{i}."
            if self.mx:
                self._layer_fwd_mx(i, ws)
                continue
            if self.fp8:
                self._layer_fwd_fp8(i, ws)
                continue
            c.barrier()
            c.ag_gemm(0, ws.xn1[i], self._p(p + "wqkv"), ws.qkv[i])
            E.rope_(ws.qkv[i], 0, Hl + Hkvl, cfg.head_dim, self.rope, seq_len=ws.S)
            A.attention_fwd(ws.qkv[i], ws.B, ws.S, Hl, Hkvl, cfg.head_dim, causal=True,
                            out=ws.o[i], lse=ws.lse[i])
            c.gemm_rs(0, ws.o[i], self._p(p + "wo"))
            c.rs_sum(0, ws.hmid[i], resid=ws.h[i], gamma=self._p(p + "ffn_norm"),
                     y=c.stage_view(1, R, D), rstd=ws.rstd2[i], eps=eps)
            c.barrier()
            c.ag_gemm(1, ws.xn2[i], self._p(p + "wgu"), ws.gu[i], epi="swiglu", h_out=ws.act[i])
            c.gemm_rs(1, ws.act[i], self._p(p + "wdown"))
            last = i == cfg.num_layers - 1
            nxt = "final_norm" if last else f"layers.{i + 1}.attn_norm"
            c.rs_sum(1, ws.h[i + 1], resid=ws.hmid[i], gamma=self._p(nxt), y=c.stage_view(0, R, D),
                     rstd=ws.rstdf if last else ws.rstd1[i + 1], eps=eps)
        c.barrier()
        c.ag_gemm(0, ws.xf, self._p("lm_head"), ws.logits)

    def _layer_fwd_fp8(self, i: int, ws: _TPWorkspace) -> None:
        cfg, c = self.cfg, self.comm
        R, D, eps = ws.R, cfg.hidden_dim, cfg.norm_eps
        Hl, Hkvl = cfg.num_heads // self.tp, cfg.num_kv_heads // self.tp
        p = f"layers.{i}."
        c.publish_fp8(0, c.stage_view(0, R, D))
        c.barrier()
        c.ag_gemm_fp8(0, ws.xn1_8[i], ws.xn1_s[i], self._w8[p + "wqkv"], ws.qkv[i])
        E.rope_(ws.qkv[i], 0, Hl + Hkvl, cfg.head_dim, self.rope, seq_len=ws.S)
        A.attention_fwd(ws.qkv[i], ws.B, ws.S, Hl, Hkvl, cfg.head_dim, causal=True, out=ws.o[i], lse=ws.lse[i])
        c.gemm_rs_fp8(0, ws.o[i], self._w8[p + "wo"])
        c.rs_sum(0, ws.hmid[i], resid=ws.h[i], gamma=self._p(p + "ffn_norm"), y=c.stage_view(1, R, D),
                 rstd=ws.rstd2[i], eps=eps)
        c.publish_fp8(1, c.stage_view(1, R, D))
        c.barrier()
        c.ag_gemm_fp8(1, ws.xn2_8[i], ws.xn2_s[i], self._w8[p + "wgu"], ws.gu[i])
        E.swiglu_fwd(ws.gu[i], ws.act[i])
        c.gemm_rs_fp8(1, ws.act[i], self._w8[p + "wdown"])
        last = i == cfg.num_layers - 1
        nxt = "final_norm" if last else f"layers.{i + 1}.attn_norm"
        c.rs_sum(1, ws.h[i + 1], resid=ws.hmid[i], gamma=self._p(nxt), y=c.stage_view(0, R, D),
                 rstd=ws.rstdf if last else ws.rstd1[i + 1], eps=eps)

    def _layer_fwd_mx(self, i: int, ws: _TPWorkspace) -> None:
        cfg, c = self.cfg, self.comm
        R, D, eps = ws.R, cfg.hidden_dim, cfg.norm_eps
        Hl, Hkvl = cfg.num_heads // self.tp, cfg.num_kv_heads // self.tp
        p = f"layers.{i}."
        w = self._w8
        c.publish_mx(0, c.stage_view(0, R, D))
        c.barrier()
        c.ag_gemm_mx(0, ws.xn1_8[i], ws.xn1_s[i], w[p + "wqkv"].q, w[p + "wqkv"].sf, ws.qkv[i])
        E.rope_(ws.qkv[i], 0, Hl + Hkvl, cfg.head_dim, self.rope, seq_len=ws.S)
        A.attention_fwd(ws.qkv[i], ws.B, ws.S, Hl, Hkvl, cfg.head_dim, causal=True, out=ws.o[i], lse=ws.lse[i])
        c.gemm_rs_mx(0, ws.o[i], w[p + "wo"].q, w[p + "wo"].sf)
        c.rs_sum(0, ws.hmid[i], resid=ws.h[i], gamma=self._p(p + "ffn_norm"), y=c.stage_view(1, R, D),
                 rstd=ws.rstd2[i], eps=eps)
        c.publish_mx(1, c.stage_view(1, R, D))
        c.barrier()
        c.ag_gemm_mx(1, ws.xn2_8[i], ws.xn2_s[i], w[p + "wgu"].q, w[p + "wgu"].sf, ws.gu[i])
        E.swiglu_fwd(ws.gu[i], ws.act[i])
        c.gemm_rs_mx(1, ws.act[i], w[p + "wdown"].q, w[p + "wdown"].sf)
        last = i == cfg.num_layers - 1
        nxt = "final_norm" if last else f"layers.{i + 1}.attn_norm"
        c.rs_sum(1, ws.h[i + 1], resid=ws.hmid[i], gamma=self._p(nxt), y=c.stage_view(0, R, D),
                 rstd=ws.rstdf if last else ws.rstd1[i + 1], eps=eps)

    def _ag_dgrad(self, k: int, ws: _TPWorkspace, name: str, out: torch.Tensor) -> torch.Tensor:
        """out = gathered residual gradient . W (the column-parallel linear's data
        gradient, all-gather fused); returns the gathered gradient (bf16) for the
        weight gradient.  MX: the gradient travels as e5m2 and is dequantised after."""
        c = self.comm
        if not self.mx:
            c.barrier()
            c.ag_gemm(k, ws.dfull, self._p(name).t(), out)
            return ws.dfull
        w = self._w8[name]
        c.publish_mx(k, c.stage_view(k, ws.R, self.cfg.hidden_dim), fmt=1)
        c.barrier()
        c.ag_gemm_mx(k, ws.dfull8, ws.dfull_s, w.qt, w.sft, out, a_fmt=1)
        C().dequant_mx_rows(ws.dfull8, 1, ws.dfull_s, ws.dfull)
        return ws.dfull

    def _dgrad_rs(self, k: int, dy: torch.Tensor, name: str) -> None:
        """Partial dy . W of a row-parallel input gradient, reduce-scattered to the owners."""
        if self.mx:
            w = self._w8[name]
            self.comm.gemm_rs_mx(k, dy, w.qt, w.sft, a_fmt=1)
        else:
            self.comm.gemm_rs(k, dy, self._p(name).t())

    def _xn_bf16(self, ws: _TPWorkspace, which: int, i: int) -> torch.Tensor:
        """The gathered normalised input of layer i (1: attention, 2: FFN) as bf16."""
        if not self.fp8:
            return ws.xn1[i] if which == 1 else ws.xn2[i]
        q, sc = (ws.xn1_8[i], ws.xn1_s[i]) if which == 1 else (ws.xn2_8[i], ws.xn2_s[i])
        if self.mx:
            C().dequant_mx_rows(q, 0, sc, ws.xn_deq)
        else:
            C().dequant_1x128(q, 0, sc, ws.xn_deq)
        return ws.xn_deq

    # ----------------------------------------------------- forward+backward
    @torch.no_grad()
    def forward_backward(self, ids: torch.Tensor, targets: torch.Tensor, *,
                         loss_scale: Optional[torch.Tensor] = None, grad_scale: float = 1.0,
                         label_smoothing: float = 0.0, z_loss: float = 0.0,
                         loss_acc: Optional[torch.Tensor] = None,
                         overwrite_grads: bool = False) -> torch.Tensor:
        cfg, c = self.cfg, self.comm
        self._overwrite = overwrite_grads
        self._w8_fresh = overwrite_grads  # a new accumulation window: the weights may have changed
        B, S = ids.shape
        ws = self.workspace(B, S)
        R, D, L = ws.R, cfg.hidden_dim, cfg.num_layers
        Hl, Hkvl = cfg.num_heads // self.tp, cfg.num_kv_heads // self.tp
        acc = ws.loss_acc if loss_acc is None else loss_acc
        if loss_acc is None:
            acc.zero_()
        self._forward(ids, ws)
        c.cross_entropy(ws.logits, targets.reshape(-1), acc, scale=loss_scale, scale_mul=grad_scale,
                        smoothing=label_smoothing, z_loss=z_loss)
        dlog = ws.logits
        # LM head: dW (local vocab rows), dx partial -> owners
        self._wgrad(dlog, ws.xf, "lm_head")
        c.gemm_rs(1, dlog, self._p("lm_head").t())
        c.rs_sum(1, ws.dx)
        dh = c.stage_view(0, R, D)
        N.rmsnorm_bwd(ws.dx, ws.h[L], self._p("final_norm"), ws.rstdf, self._g("final_norm"), dx=dh,
                      accumulate=not overwrite_grads)
        k = 0
        for i in reversed(range(L)):
            p = f"layers.{i}."
            # ---- FFN: dact = dh_full Wdown (all-gather fused), dgu, dxn2 -> owners
            dfull = self._ag_dgrad(k, ws, p + "wdown", ws.dact)
            self._wgrad(dfull, ws.act[i], p + "wdown")
            E.swiglu_bwd(ws.gu[i], ws.dact, ws.dgu)
            self._wgrad(ws.dgu, self._xn_bf16(ws, 2, i), p + "wgu")
            self._dgrad_rs(0, ws.dgu, p + "wgu")
            c.rs_sum(0, ws.dx)
            dh_in, dh_out = c.stage_view(k, R, D), c.stage_view(1 - k, R, D)
            N.rmsnorm_bwd(ws.dx, ws.hmid[i], self._p(p + "ffn_norm"), ws.rstd2[i], self._g(p + "ffn_norm"),
                          dres=dh_in, dx=dh_out, accumulate=not overwrite_grads)
            k = 1 - k
            # ---- attention
            dfull = self._ag_dgrad(k, ws, p + "wo", ws.do)
            self._wgrad(dfull, ws.o[i], p + "wo")
            A.attention_bwd(ws.qkv[i], ws.o[i], ws.do, ws.lse[i], ws.B, ws.S, Hl, Hkvl, cfg.head_dim,
                            causal=True, dqkv=ws.dqkv)
            E.rope_(ws.dqkv, 0, Hl + Hkvl, cfg.head_dim, self.rope, seq_len=ws.S, inverse=True)
            self._wgrad(ws.dqkv, self._xn_bf16(ws, 1, i), p + "wqkv")
            self._dgrad_rs(1, ws.dqkv, p + "wqkv")
            c.rs_sum(1, ws.dx)
            dh_in, dh_out = c.stage_view(k, R, D), c.stage_view(1 - k, R, D)
            N.rmsnorm_bwd(ws.dx, ws.h[i], self._p(p + "attn_norm"), ws.rstd1[i], self._g(p + "attn_norm"),
                          dres=dh_in, dx=dh_out, accumulate=not overwrite_grads)
            k = 1 - k
        if overwrite_grads and not cfg.tie_embeddings:
            self._g("embed").zero_()
        ids_local = ids.reshape(-1)[self.rank * R:(self.rank + 1) * R]
        E.embedding_bwd(ids_local, c.stage_view(k, R, D), self._g("embed"))
        self._overwrite = False
        return acc

    @torch.no_grad()
    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        """Local vocabulary slice of the logits, [B*S, V/tp] (bf16)."""
        B, S = ids.shape
        ws = self.workspace(B, S)
        self._w8_fresh = True
        self._forward(ids, ws)
        return ws.logits


# ----------------------------------------------------------------- trainer
class TPTrainer:
    """AdamW training of a TPLlamaModel: gradient accumulation, replicated-grad
    all-reduce (K12, peer memory), the global-norm exchange and finaliser on the
    device, then AdamW over this rank's local parameters."""

    def __init__(self, cfg: TransformerConfig, tc, *, micro_batch: int, seq_len: int, device=None,
                 group=None, comm: str = "p2p", seed: int = 1234, fp8: bool = False):
        if cfg.dropout > 0:
            raise NotImplementedError("dropout in the tensor-parallel model (use data / pipeline parallelism)")
        from ..ops import optim as O
        from ..train.optimizer import FusedAdamW
        self.cfg, self.tc = cfg, tc
        self.device = torch.device(device or torch.cuda.current_device())
        self.comm = TPComm(cfg, micro_batch * seq_len, self.device, group, comm)
        self.tp, self.rank = self.comm.tp, self.comm.rank
        params = TPParams(cfg, self.tp, self.rank, self.device)
        params.init_(seed, cfg.init_std)
        # fp32 gradients in symmetric memory: the replicated prefix is summed in place over peers
        self.gbuf = CM.SymBuffer(params.numel, torch.float32, self.device, self.comm.group)
        grads = params.like(torch.float32, buffer=self.gbuf.local)
        self.model = TPLlamaModel(cfg, self.comm, params, grads=grads, fp8=fp8)
        self.params, self.grads = params, grads
        self.master = params.flat.float()
        self.opt = FusedAdamW(self.master, params.segments(), lr=tc.lr, betas=(tc.beta1, tc.beta2),
                              eps=tc.eps, weight_decay=tc.weight_decay, max_grad_norm=tc.max_grad_norm,
                              dynamic_loss_scale=tc.dynamic_loss_scale,
                              init_loss_scale=tc.init_loss_scale, ema_decay=tc.ema_decay)
        self.n_rep = params.n_rep
        self.partial = torch.zeros(2048, dtype=torch.float32, device=self.device)
        self._O = O
        self.micro = 0
        # the train.trainer.Trainer interface (same as the data-parallel trainers)
        self.loss_acc = torch.zeros(2, dtype=torch.float32, device=self.device)
        self.accum_steps = max(1, tc.grad_accum_steps)
        self.pre_optimizer = None
        self._opt_steps = 0

    def micro_step_async(self, ids: torch.Tensor, targets: torch.Tensor) -> None:
        """One micro-batch (the same [B, S] batch on every rank); the optimizer
        steps after grad_accum_steps of them.  Loss sums go to self.loss_acc."""
        self.micro_step(ids, targets, 1.0 / (ids.numel() * self.accum_steps), self.loss_acc)
        if self.micro == self.accum_steps:
            self.optimizer_step()

    def current_step(self) -> int:
        return self._opt_steps

    def set_learning_rate(self, lr: float) -> None:
        self.opt.set_lr(lr)

    def micro_step(self, ids: torch.Tensor, targets: torch.Tensor, grad_scale: float,
                   loss_acc: torch.Tensor) -> None:
        self.model.forward_backward(ids, targets, loss_scale=self.opt.scaler.scale_tensor(),
                                    grad_scale=grad_scale, loss_acc=loss_acc,
                                    label_smoothing=self.tc.label_smoothing, z_loss=self.tc.z_loss,
                                    overwrite_grads=self.micro == 0)
        self.micro += 1

    def optimizer_step(self) -> None:
        c = self.comm
        P = self.partial
        if self.pre_optimizer is not None:
            self.pre_optimizer(self.gbuf.local)
        if self.tp > 1:
            # replicated grads: one-shot peer all-reduce + their sum-of-squares partials
            if c.comm == "nccl":
                dist.all_reduce(self.gbuf.local[:self.n_rep], group=c.group)
                P[1024:].zero_()
                C().grad_norm_partials(self.gbuf.local[:self.n_rep], P[1024:])
                P[1024:].div_(self.tp)  # every rank holds the same replicated grads
            else:
                c.pc.allreduce_sum_(self.gbuf, self.n_rep, P[1024:])
        else:
            C().grad_norm_partials(self.gbuf.local[:self.n_rep], P[1024:])
        C().grad_norm_partials(self.gbuf.local[self.n_rep:], P[:1024])
        o = self.opt
        s = o.scaler
        if self.tp > 1 and c.comm != "nccl":
            c.pc.norm_exchange(P, o.state, o.max_grad_norm, s.enabled, s.growth, s.backoff,
                               s.growth_interval, s.min_scale)
        elif self.tp > 1:
            dist.all_reduce(P, group=c.group)
            o.finalize(P)
        else:
            o.finalize(P)
        o.apply(self.gbuf.local, self.params.flat)
        self.micro = 0
        self._opt_steps += 1

    def train_step(self, batches) -> torch.Tensor:
        """batches: list of (ids, targets) [B, S] micro-batches (full batch on
        every rank).  Returns the loss accumulator [sum, count]."""
        acc = torch.zeros(2, dtype=torch.float32, device=self.device)
        n_tok = sum(int(t.numel()) for _, t in batches)
        for ids, tg in batches:
            self.micro_step(ids, tg, 1.0 / n_tok, acc)
        self.optimizer_step()
        return acc

    def check(self) -> None:
        check_status(self.device)

    # ------------------------------------------------------------ checkpoints
    def checkpoint_parts(self):
        """Per-rank local shards laid end to end ({"kind": "tp"} layout): a
        checkpoint restores onto the same tensor-parallel degree."""
        n = self.master.numel()
        lay = {"kind": "tp", "tp": self.tp, "total": self.tp * n, "align": 0, "specs": {}}
        o = self.opt
        t = {"p32": o.p32, "m": o.m, "v": o.v, "state": o.state}
        return lay, [(self.rank * n, (self.rank + 1) * n)], t

    def load_checkpoint_flat(self, flat, saved_layout: dict) -> None:
        n = self.master.numel()
        if saved_layout.get("kind") != "tp" or saved_layout.get("tp") != self.tp or saved_layout["total"] != self.tp * n:
            raise ValueError("tensor-parallel checkpoints restore onto the same tensor-parallel degree and model")
        o = self.opt
        with torch.no_grad():
            for name in ("p32", "m", "v"):
                getattr(o, name).copy_(flat[name][self.rank * n:(self.rank + 1) * n].to(self.device))
            o.state.copy_(flat["state"].to(self.device))
            self.params.flat.copy_(o.p32.to(torch.bfloat16))

    def reference_state_dict(self) -> "OrderedDict[str, torch.Tensor]":
        """Reference-named full tensors ([in, out]), gathered on every rank (CPU)."""
        from ..models.params import FlatParams
        full = FlatParams(self.cfg, "cpu", torch.bfloat16)
        for name, t in self.full_state_dict().items():
            full.views[name].copy_(t.cpu())
        return full.to_reference_state_dict()

    def full_state_dict(self) -> "OrderedDict[str, torch.Tensor]":
        """Engine-layout full tensors (gathered over the TP group with NCCL)."""
        out: "OrderedDict[str, torch.Tensor]" = OrderedDict()
        for s in self.params.specs:
            v = self.params[s.name].contiguous()
            pieces = [torch.empty_like(v) for _ in range(self.tp)]
            dist.all_gather(pieces, v, group=self.comm.group)
            out[s.name] = unshard_tensor(self.cfg, s.name, pieces)
        return out
