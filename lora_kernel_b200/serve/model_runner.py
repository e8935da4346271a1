"""Inference forward passes over the paged KV cache.

One `ModelRunner` per GPU holds the (optionally quantised) weights and the KV
cache of every layer and runs two kinds of batches:

  prefill   chunks of prompts (several sequences, token rows concatenated):
            GEMMs over all rows at once; RoPE at each token's position; the
            chunk's K/V appended to the cache (K15); attention per sequence
            with the tcgen05 flash kernel against the sequence's cached
            K/V gathered back to bf16 (so prefix-cached blocks are reused);
  decode    one new token per running sequence: the same GEMMs with M = batch,
            K15 append, then K13 paged decode attention straight over the
            (fp8 / int8 / bf16) pages.

The LM head runs only on each sequence's last row; K19 samples the next token.
Weights can stay bf16 (tcgen05 GEMM, SwiGLU fused into the gate|up epilogue)
or be int8 / fp8 per row or int4 group-128 (K14: dequantising GEMV for
decode-sized batches, dequantise + tcgen05 GEMM for prefill-sized ones).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
from typing import Dict, List, Optional, Tuple

import torch

from ..config import TransformerConfig
from ..models.params import FlatParams
from ..ops import elementwise as E
from ..ops import gemm as G
from ..ops import norm as N
from ..ops import serving as SV
from ..ops.attention import attention_fwd


@dataclass
class PrefillItem:
    seq_id: int
    tokens: List[int]       # this chunk's token ids
    start: int              # position of the chunk's first token
    slots: List[int]        # KV slots of positions [0, start + len(tokens))
    want_logits: bool       # chunk ends the prompt: sample its next token
    all_logits: bool = False  # logits of every row of the chunk (speculative verification)


class ModelRunner:
    def __init__(self, cfg: TransformerConfig, params: FlatParams, device="cuda", *,
                 kv_dtype: str = "fp8", weights: str = "none", group_size: int = 128,
                 num_blocks: int = 0, block_size: int = 16, max_model_len: int = 4096,
                 mem_fraction: float = 0.85):
        self.cfg = cfg
        self.device = torch.device(device)
        self.kv_dtype = kv_dtype
        self.wq = weights
        self.block_size = block_size
        self.max_model_len = max_model_len
        self.W: Dict[str, object] = {}
        self._scratch: Optional[torch.Tensor] = None
        self._load_weights(params, weights, group_size)
        H, KV, Dh = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim
        per_token = 2 * cfg.num_layers * KV * Dh * (2 if kv_dtype == "bf16" else 1)
        per_token += 2 * cfg.num_layers * KV * 4 if kv_dtype != "bf16" else 0
        if num_blocks <= 0:
            free, _ = torch.cuda.mem_get_info(self.device)
            num_blocks = max(16, int(free * mem_fraction) // (per_token * block_size))
        self.num_blocks = num_blocks
        # one extra block at the end: the KV sink of padding rows in graph-captured decode
        slots = (num_blocks + 1) * block_size
        self.dummy_block = num_blocks
        dt = SV.KV_TORCH[kv_dtype]
        self.k_cache = torch.zeros(cfg.num_layers, slots, KV, Dh, dtype=dt, device=self.device)
        self.v_cache = torch.zeros_like(self.k_cache)
        if kv_dtype != "bf16":
            self.k_scale = torch.zeros(cfg.num_layers, slots, KV, dtype=torch.float32, device=self.device)
            self.v_scale = torch.zeros_like(self.k_scale)
        else:
            self.k_scale = self.v_scale = None
        self.rope = E.rope_table(max_model_len, Dh, cfg.rope_base, self.device)
        self.use_graphs = False
        self._graphs: Dict[int, Tuple] = {}
        self._pool = None

    # --------------------------------------------------------------- weights
    def _load_weights(self, params: FlatParams, fmt: str, group: int) -> None:
        cfg = self.cfg
        quant_names = ("wqkv", "wo", "wgu", "wdown")
        # with quantised weights, copy the few bf16 tensors kept as-is out of the
        # flat buffer so the caller can free the full-precision weights
        keep = (lambda t: t.clone()) if fmt != "none" else (lambda t: t)
        for i in range(cfg.num_layers):
            p = f"layers.{i}."
            for n in ("attn_norm", "ffn_norm"):
                self.W[p + n] = keep(params[p + n])
            for n in quant_names:
                w = params[p + n]
                if isinstance(w, SV.QuantizedWeight):  # already quantised (loaded checkpoint)
                    self.W[p + n] = w
                else:
                    self.W[p + n] = SV.QuantizedWeight(w, fmt, group) if fmt != "none" else w
        self.W["embed"] = keep(params["embed"])
        self.W["final_norm"] = keep(params["final_norm"])
        self.W["lm_head"] = self.W["embed"] if cfg.tie_embeddings else keep(params["lm_head"])

    def weight_bytes(self) -> int:
        n = 0
        for w in self.W.values():
            n += w.nbytes() if isinstance(w, SV.QuantizedWeight) else w.numel() * w.element_size()
        return n

    def _linear(self, x: torch.Tensor, name: str, residual: Optional[torch.Tensor] = None,
                out: Optional[torch.Tensor] = None) -> torch.Tensor:
        w = self.W[name]
        if isinstance(w, SV.QuantizedWeight):
            scratch = None
            if x.shape[0] > 256:  # prefill: dequantise once, then the bf16 GEMM
                need = w.N * w.K
                if self._scratch is None or self._scratch.numel() < need:
                    self._scratch = torch.empty(need, dtype=torch.bfloat16, device=self.device)
                scratch = self._scratch[:need].view(w.N, w.K)
            return w.matmul_t(x, out=out, scratch=scratch, residual=residual)
        return G.linear(x, w, residual=residual, out=out)

    def _ffn(self, x: torch.Tensor, p: str, residual: torch.Tensor) -> torch.Tensor:
        w = self.W[p + "wgu"]
        if isinstance(w, SV.QuantizedWeight):
            gu = self._linear(x, p + "wgu")
            a = E.swiglu_fwd(gu)
        else:
            _, a = G.linear_swiglu(x, w)
        return self._linear(a, p + "wdown", residual=residual)

    # --------------------------------------------------------------- layers
    def _layer(self, i: int, h: torch.Tensor, pos: torch.Tensor, slots: torch.Tensor, attn) -> torch.Tensor:
        cfg = self.cfg
        p = f"layers.{i}."
        xn, _, _ = N.rmsnorm_fwd(h, self.W[p + "attn_norm"], cfg.norm_eps)
        qkv = self._linear(xn, p + "wqkv")
        E.rope_(qkv, 0, cfg.num_heads + cfg.num_kv_heads, cfg.head_dim, self.rope, positions=pos)
        ks = self.k_scale[i] if self.k_scale is not None else None
        vs = self.v_scale[i] if self.v_scale is not None else None
        SV.kv_append(qkv, cfg.num_heads, cfg.num_kv_heads, cfg.head_dim, slots, self.k_cache[i],
                     self.v_cache[i], ks, vs, self.kv_dtype)
        o = attn(i, qkv)
        h2 = self._linear(o, p + "wo", residual=h)
        xn2, _, _ = N.rmsnorm_fwd(h2, self.W[p + "ffn_norm"], cfg.norm_eps)
        return self._ffn(xn2, p, h2)

    def _head(self, h_last: torch.Tensor) -> torch.Tensor:
        xf, _, _ = N.rmsnorm_fwd(h_last, self.W["final_norm"], self.cfg.norm_eps)
        return G.linear(xf, self.W["lm_head"])

    # nucleus (top-p) sampling and per-request seeds run on a single-GPU kernel
    # (the nucleus threshold needs the whole vocabulary row)
    supports_top_p = True

    def sample(self, logits: torch.Tensor, temps: Optional[List[float]], seed: int,
               top_ps: Optional[List[float]] = None, row_seeds: Optional[List[int]] = None) -> torch.Tensor:
        """Next token per row (K19): greedy when temps is None, else Gumbel-max;
        with top_ps, Gumbel-max over each row's top-p nucleus; with row_seeds,
        each row's noise from its own seed."""
        n, dev = logits.shape[0], logits.device
        t = None if temps is None else torch.tensor(temps, dtype=torch.float32, device=dev)
        if top_ps is not None or row_seeds is not None:
            if t is None:
                t = torch.zeros(n, dtype=torch.float32, device=dev)
            p = torch.ones(n, dtype=torch.float32, device=dev) if top_ps is None else \
                torch.tensor(top_ps, dtype=torch.float32, device=dev)
            rs = None if row_seeds is None else \
                torch.tensor([x & ((1 << 63) - 1) for x in row_seeds], dtype=torch.int64, device=dev)
            return SV.sample_topp(logits, t, p, seed, row_seeds=rs)
        return SV.sample(logits, t, seed)

    # -------------------------------------------------------------- prefill
    @torch.no_grad()
    def prefill(self, items: List[PrefillItem]) -> Tuple[List[int], torch.Tensor]:
        """Returns (seq ids that want a token, logits [n, vocab]) for items whose
        chunk ends the prompt: one row per such item (its last token), or one
        per chunk token for items with all_logits."""
        cfg = self.cfg
        dev = self.device
        ids, pos, slots, bounds = [], [], [], []
        r = 0
        for it in items:
            n = len(it.tokens)
            ids += it.tokens
            pos += list(range(it.start, it.start + n))
            slots += it.slots[it.start:it.start + n]
            bounds.append((r, r + n))
            r += n
        ids_t = torch.tensor(ids, dtype=torch.int64, device=dev)
        pos_t = torch.tensor(pos, dtype=torch.int32, device=dev)
        slots_t = torch.tensor(slots, dtype=torch.int32, device=dev)
        all_slots = [torch.tensor(it.slots[:it.start + len(it.tokens)], dtype=torch.int32, device=dev)
                     for it in items]
        H, KV, Dh = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim

        def attn(i, qkv):
            o = torch.empty(qkv.shape[0], H * Dh, dtype=torch.bfloat16, device=dev)
            ks = self.k_scale[i] if self.k_scale is not None else None
            vs = self.v_scale[i] if self.v_scale is not None else None
            for it, (a, b), sl in zip(items, bounds, all_slots):
                kv = SV.kv_gather(self.k_cache[i], self.v_cache[i], ks, vs, sl, KV, Dh, self.kv_dtype)
                attention_fwd(qkv[a:b, :H * Dh], 1, b - a, H, KV, Dh, causal=True, out=o[a:b],
                              kv=kv, q_off=it.start)
            return o

        h = E.embedding_fwd(ids_t, self.W["embed"])
        for i in range(cfg.num_layers):
            h = self._layer(i, h, pos_t, slots_t, attn)
        want = [k for k, it in enumerate(items) if it.want_logits]
        if not want:
            return [], torch.empty(0, cfg.vocab_size, device=dev)
        rows, ids_out = [], []
        for k in want:
            a, b = bounds[k]
            r0 = a if items[k].all_logits else b - 1
            rows += range(r0, b)
            ids_out += [items[k].seq_id] * (b - r0)
        rows_t = torch.tensor(rows, dtype=torch.int64, device=dev)
        logits = self._head(h.index_select(0, rows_t).contiguous())
        return ids_out, logits

    # --------------------------------------------------------------- decode
    GRAPH_BUCKETS = (1, 2, 4, 8, 16, 24, 32, 48, 64, 96, 128, 160, 192, 224, 256)

    def enable_graphs(self, max_batch: int = 256, capture: bool = True) -> None:
        """Replay decode steps from CUDA graphs captured per batch-size bucket
        (inputs padded to the bucket; padding rows write their K/V into a
        reserved block).  The launch sequence of a whole decode step - every
        layer's GEMMs, norms, RoPE, KV append and paged attention - becomes one
        graph launch, which is what bounds small-batch decode otherwise."""
        if self.use_graphs:
            return
        need = 0
        for w in self.W.values():
            if isinstance(w, SV.QuantizedWeight):
                need = max(need, w.N * w.K)
        if need and (self._scratch is None or self._scratch.numel() < need):
            self._scratch = torch.empty(need, dtype=torch.bfloat16, device=self.device)
        self._pool = torch.cuda.graph_pool_handle()
        self.use_graphs = True
        self.graph_max_batch = max_batch
        if capture:
            # capture every bucket now (largest first) so no request waits on a capture later
            mb = (self.max_model_len + self.block_size - 1) // self.block_size
            for b in sorted((x for x in self.GRAPH_BUCKETS if x <= max_batch), reverse=True):
                self._graphs[b] = self._capture(b, mb)

    def _decode_body(self, ids_t, pos_t, slots_t, bt, ctx, max_ctx: int) -> torch.Tensor:
        cfg = self.cfg
        H, KV, Dh = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim

        def attn(i, qkv):
            ks = self.k_scale[i] if self.k_scale is not None else None
            vs = self.v_scale[i] if self.v_scale is not None else None
            return SV.decode_attention(qkv[:, :H * Dh], self.k_cache[i], self.v_cache[i], ks, vs, bt, ctx,
                                       self.block_size, H, KV, Dh, kv_dtype=self.kv_dtype, max_ctx=max_ctx)

        h = E.embedding_fwd(ids_t, self.W["embed"])
        for i in range(cfg.num_layers):
            h = self._layer(i, h, pos_t, slots_t, attn)
        return self._head(h)

    @torch.no_grad()
    def decode(self, tokens: List[int], positions: List[int], slots: List[int],
               block_tables: List[List[int]]) -> torch.Tensor:
        """One token per sequence; returns logits [n, vocab].  The arguments may
        also be int32 numpy arrays (block_tables [n, max_blocks], zero padded)."""
        n = len(tokens)
        if self.use_graphs and n <= getattr(self, "graph_max_batch", self.GRAPH_BUCKETS[-1]):
            return self._decode_graph(tokens, positions, slots, block_tables)
        dev = self.device
        ids_t = torch.tensor(tokens, dtype=torch.int64, device=dev)
        pos_t = torch.tensor(positions, dtype=torch.int32, device=dev)
        slots_t = torch.tensor(slots, dtype=torch.int32, device=dev)
        if isinstance(block_tables, np.ndarray):
            bt = torch.from_numpy(np.ascontiguousarray(block_tables, dtype=np.int32))
        else:
            mb = max(len(t) for t in block_tables)
            bt = torch.zeros(n, mb, dtype=torch.int32)
            for k, t in enumerate(block_tables):
                bt[k, :len(t)] = torch.tensor(t, dtype=torch.int32)
        bt = bt.to(dev)
        ctx = torch.tensor([int(p) + 1 for p in positions], dtype=torch.int32, device=dev)
        return self._decode_body(ids_t, pos_t, slots_t, bt, ctx, int(max(positions)) + 1)

    def _decode_graph(self, tokens, positions, slots, block_tables) -> torch.Tensor:
        n = len(tokens)
        b = next(x for x in self.GRAPH_BUCKETS if x >= n)
        mb = (self.max_model_len + self.block_size - 1) // self.block_size
        st = self._graphs.get(b)
        if st is None:
            st = self._capture(b, mb)
            self._graphs[b] = st
        graph, host, dev_in, out, _ = st
        # host staging (pinned): ids | pos | slots | ctx | block table, padding rows -> reserved block
        hi = host.numpy()
        hi[:] = 0
        hi[0:n] = tokens
        hi[b:b + n] = positions
        hi[2 * b:2 * b + n] = slots
        hi[2 * b + n:3 * b] = self.dummy_block * self.block_size
        hi[3 * b:3 * b + n] = np.asarray(positions, dtype=np.int32) + 1
        hi[3 * b + n:4 * b] = 1
        btab = hi[4 * b:].reshape(b, mb)
        if isinstance(block_tables, np.ndarray):
            btab[:n, :block_tables.shape[1]] = block_tables
        else:
            for k, t in enumerate(block_tables):
                btab[k, :len(t)] = t
        btab[n:, 0] = self.dummy_block
        dev_in.copy_(host, non_blocking=True)
        graph.replay()
        return out[:n]

    def _capture(self, b: int, mb: int):
        dev = self.device
        host = torch.zeros(4 * b + b * mb, dtype=torch.int32, pin_memory=True)
        dev_in = torch.zeros_like(host, device=dev)
        ids_t = dev_in[0:b]
        pos_t = dev_in[b:2 * b]
        slots_t = dev_in[2 * b:3 * b]
        ctx = dev_in[3 * b:4 * b]
        bt = dev_in[4 * b:].view(b, mb)
        # a valid dummy batch for warm-up and capture: every row is padding
        host[2 * b:3 * b] = self.dummy_block * self.block_size
        host[3 * b:4 * b] = 1
        host[4 * b:].view(b, mb)[:, 0] = self.dummy_block
        dev_in.copy_(host)
        ids64 = torch.empty(b, dtype=torch.int64, device=dev)

        def body():
            ids64.copy_(ids_t)
            return self._decode_body(ids64, pos_t, slots_t, bt, ctx, self.max_model_len)

        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            for _ in range(2):
                body()
        torch.cuda.current_stream(dev).wait_stream(s)
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, pool=self._pool):
            out = body()
        torch.cuda.synchronize(dev)
        # every tensor the graph reads or writes outside its private pool must
        # stay alive as long as the graph: the input buffers and ids64
        return graph, host, dev_in, out, ids64
