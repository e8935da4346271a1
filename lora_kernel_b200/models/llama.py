"""Llama decoder on the sm_100a kernels: a hand-scheduled forward and backward.

Per layer (T = B*S tokens):
    xn1, rstd1   = rmsnorm(h)                                   K5
    qkv          = xn1 Wqkv^T ; RoPE(q, k) in place              K1, K6
    o, lse       = flash_attention(qkv)                          K3
    h_mid        = h + o Wo^T            (residual epilogue)     K1
    xn2, rstd2   = rmsnorm(h_mid)                                K5
    gu, a        = xn2 Wgu^T, a = silu(gate)*up (epilogue)       K1+K7
    h_next       = h_mid + a Wdown^T     (residual epilogue)     K1
then final rmsnorm, LM head GEMM and the fused cross-entropy (loss + in-place
bf16 dlogits, K9).  The backward runs the mirror image: dgrad GEMMs with MN-major
weights, weight-gradient GEMMs accumulating straight into the fp32 gradient
views, the fused SwiGLU/RMSNorm backward kernels (residual gradient added in
place), the flash-attention backward (K4), inverse RoPE and the embedding
scatter-add (K8).

The reference's Transformer::forward/backward (src/nn/transformer_blocks.cpp:
603-718) skips Wo, keeps two weight sets and never trains the embeddings; this
is the standard Llama computation instead (pre-norm, GQA, RoPE per head,
SwiGLU with ff_dim, final norm).

Workspace activations are allocated once per (batch, seq) shape and reused, so
steady-state steps allocate nothing.
"""
from __future__ import annotations

import os

import math
from typing import Dict, Optional, Tuple

import torch

from ..config import TransformerConfig
from ..ops import attention as A
from ..ops import elementwise as E
from ..ops import gemm as G
from ..ops import loss as L
from ..ops import norm as N
from ..utils.profiler import ph
from .params import FlatParams


class _Workspace:
    def __init__(self, cfg: TransformerConfig, B: int, S: int, device, save: bool, recompute: bool = False,
                 logits: bool = True, dropout: bool = False):
        T = B * S
        D, F, V = cfg.hidden_dim, cfg.ff_dim_padded, cfg.vocab_size
        # recompute: keep every layer's input h, one slot of per-layer intermediates
        nl = cfg.num_layers if (save and not recompute) else 1
        bf = dict(dtype=torch.bfloat16, device=device)
        f32 = dict(dtype=torch.float32, device=device)
        self.B, self.S, self.T = B, S, T
        self.h = [torch.empty(T, D, **bf) for _ in range(cfg.num_layers + 1)] if save else \
            [torch.empty(T, D, **bf) for _ in range(2)]
        self.xn1 = [torch.empty(T, D, **bf) for _ in range(nl)]
        self.rstd1 = [torch.empty(T, **f32) for _ in range(nl)]
        self.qkv = [torch.empty(T, cfg.qkv_dim, **bf) for _ in range(nl)]
        self.o = [torch.empty(T, cfg.q_dim, **bf) for _ in range(nl)]
        # dropped attention context (the attention backward needs the undropped o)
        self.od = [torch.empty(T, cfg.q_dim, **bf) for _ in range(nl)] if dropout else None
        self.lse = [torch.empty(B, cfg.num_heads, S, **f32) for _ in range(nl)]
        self.hmid = [torch.empty(T, D, **bf) for _ in range(nl)]
        self.xn2 = [torch.empty(T, D, **bf) for _ in range(nl)]
        self.rstd2 = [torch.empty(T, **f32) for _ in range(nl)]
        self.gu = [torch.empty(T, 2 * F, **bf) for _ in range(nl)]
        self.act = [torch.empty(T, F, **bf) for _ in range(nl)]
        self.xf = torch.empty(T, D, **bf)
        self.rstdf = torch.empty(T, **f32)
        self.logits = torch.empty(T, V, **bf) if logits else None
        self.loss_acc = torch.zeros(2, **f32)
        if save:
            self.dh = torch.empty(T, D, **bf)
            self.dx = torch.empty(T, D, **bf)
            self.dact = torch.empty(T, F, **bf)
            self.dgu = torch.empty(T, 2 * F, **bf)
            self.do = torch.empty(T, cfg.q_dim, **bf)
            self.dqkv = torch.empty(T, cfg.qkv_dim, **bf)


class LlamaModel:
    """The B200 Llama engine.  `params` (bf16) are the weights the kernels read;
    `grads` (fp32, same layout) receive the accumulated weight gradients."""

    def __init__(self, cfg: TransformerConfig, device="cuda", params: Optional[FlatParams] = None,
                 seed: int = 1234, with_grads: bool = True):
        self.cfg = cfg
        self.device = torch.device(device)
        if params is None:
            params = FlatParams(cfg, self.device)
            params.init_(seed, cfg.init_std)
        self.params = params
        self.grads = params.like(torch.float32) if with_grads else None
        self._ws: Dict[Tuple[int, int, bool], _Workspace] = {}
        self.rope = E.rope_table(max(cfg.max_seq_len, 1), cfg.head_dim, cfg.rope_base, self.device)
        self.attn_window = 0
        self.hooks = None  # optional: pre_forward / pre_layer_fwd(i) / pre_layer_bwd(i) /
        #                    post_layer_bwd(i) / post_head_bwd / post_backward (ZeRO-3)
        self._overwrite = False
        # optional (layer, target, fn): the next _lin / _lin_bwd of that linear runs
        # fn(a, b, out) instead of the plain GEMM (ZeRO-3 gather fused into it, K17)
        self.fused_gather = None
        # activation checkpointing: the forward keeps only each layer's input; the
        # backward re-runs a layer's forward (same kernels, same values) right
        # before its backward
        self.recompute = False
        self._saving = False
        self._sd_scale = 1.0  # stochastic depth: 1 / keep probability of the current layer
        self.fuse_swiglu_bwd = os.environ.get("LK_FUSE_SWIGLU_BWD", "0") == "1"
        self.fuse_rope = os.environ.get("LK_FUSE_ROPE", "0") == "1"
        self.lora = None        # optional LoRAAdapters (models/lora.py)
        self.train_base = True  # False: frozen base weights (no base weight gradients)
        self._u: Dict[Tuple[int, str], torch.Tensor] = {}
        # dropout (training only): counter-hash masks seeded by (seed, micro-step,
        # layer, site); the backward regenerates the same masks
        self.dropout_seed = seed
        self._drop_step = 0
        # optional context-parallel attention (parallel/cp.py): ids are this rank's
        # chunk of every sequence; RoPE uses global positions
        self.ctx = None

    # -------------------------------------------------------------- helpers
    def ce_chunk(self, T: int) -> int:
        """Vocabulary columns per LM-head chunk in training (0: whole vocabulary)."""
        c, V = self.cfg.ce_vocab_chunk, self.cfg.vocab_size
        if c < 0:
            return 0
        if c == 0:
            return 8192 if T * V * 2 > (1 << 30) and V > 8192 else 0
        c = max(8, c // 8 * 8)
        return c if c < V else 0

    def workspace(self, B: int, S: int, save: bool = True) -> _Workspace:
        key = (B, S, save, self.recompute and save)
        ws = self._ws.get(key)
        if ws is None:
            full = S * (self.ctx.world if self.ctx is not None else 1)
            if full > self.rope.shape[0]:
                self.rope = E.rope_table(full, self.cfg.head_dim, self.cfg.rope_base, self.device)
            ws = _Workspace(self.cfg, B, S, self.device, save, recompute=self.recompute and save,
                            dropout=save and self.cfg.dropout > 0,
                            logits=not (save and self.ce_chunk(B * S)))
            self._ws[key] = ws
        return ws

    def num_parameters(self) -> int:
        return self.cfg.num_parameters()

    def _p(self, name):
        return self.params[name]

    def _g(self, name):
        return self.grads[name]

    def _hook(self, name, *a):
        if self.hooks is not None:
            getattr(self.hooks, name)(*a)

    def _wgrad(self, dy, x, name, rows: Optional[Tuple[int, int]] = None, alpha: float = 1.0):
        """Weight gradient: stored on the first micro-step of a window, else
        accumulated; rows = (r0, n): only those rows of the weight (dy holds
        their output columns)."""
        if not self.train_base and not name.endswith("norm") and name != "embed":
            return
        g = self._g(name)
        if rows is not None:
            g = g[rows[0]:rows[0] + rows[1]]
        # a bf16 gradient view (ZeRO-3 slot, reduce-scattered every micro-batch)
        # is stored; an fp32 one is stored on the first micro-batch of a window
        # and accumulated afterwards
        epi = "bf16" if g.dtype == torch.bfloat16 else ("f32" if self._overwrite else "f32_acc")
        with ph("bwd.gemm_wgrad"):
            G.gemm(dy.t(), x.t(), g, epi=epi, alpha=alpha)

    # ------------------------------------------------------ linear + LoRA
    def _lora_u(self, i: int, t: str, x: torch.Tensor, save: bool):
        """s * x A^T for an adapted linear (None without an adapter)."""
        if self.lora is None or not self.lora.has(i, t):
            return None
        key = (i, t)
        u = self._u.get(key) if save else None
        if u is None or u.shape[0] != x.shape[0]:
            u = torch.empty(x.shape[0], self.lora.lc.rank, dtype=torch.bfloat16, device=x.device)
            if save:
                self._u[key] = u
        G.gemm(x, self.lora.A(i, t), u, alpha=self.lora.lc.scale)
        return u

    def _take_fused(self, i: int, t: str):
        fg = self.fused_gather
        if fg is not None and fg[0] == i and fg[1] == t:
            self.fused_gather = None
            return fg[2]
        return None

    def _lin(self, i: int, t: str, x, out, residual=None, save: bool = True, rope=None) -> bool:
        """out = x W^T (+ residual); rope: the (table, cols, head_dim, seq, offset)
        rotation done in the GEMM epilogue.  Returns whether rope was applied."""
        fn = self._take_fused(i, t) if residual is None else None
        if fn is not None:
            with ph(f"fwd.gemm_{t}+gather"):
                fn(x, self._p(f"layers.{i}.{t}"), out)
            return False
        u = self._lora_u(i, t, x, save)
        B = self.lora.B(i, t) if u is not None else None
        alpha = self._sd_scale if residual is not None else 1.0  # a residual branch's output projection
        with ph(f"fwd.gemm_{t}" + ("+rope" if rope is not None else "")):
            G.gemm(x, self._p(f"layers.{i}.{t}"), out, epi="bf16_resid" if residual is not None else "bf16",
                   residual=residual, a2=u, b2=B, alpha=alpha, rope=rope)
        return rope is not None

    def _lin_swiglu(self, i: int, x, gu_out, h_out, save: bool = True):
        u = self._lora_u(i, "wgu", x, save)
        B = self.lora.B(i, "wgu") if u is not None else None
        with ph("fwd.gemm_wgu+swiglu"):
            G.gemm(x, self._p(f"layers.{i}.wgu"), gu_out, epi="swiglu", h_out=h_out, a2=u, b2=B)

    def _lin_bwd(self, i: int, t: str, dy, x, dx_out):
        """dx = dy W (+ s (dy B) A); base and adapter weight gradients."""
        name = f"layers.{i}.{t}"
        if self.lora is not None and self.lora.has(i, t):
            lc = self.lora.lc
            v = torch.empty(dy.shape[0], lc.rank, dtype=torch.bfloat16, device=dy.device)
            G.gemm(dy, self.lora.B(i, t).t(), v, alpha=lc.scale)           # s * dy B
            G.gemm(dy, self._p(name).t(), dx_out, a2=v, b2=self.lora.A(i, t).t())
            acc = "f32" if self._overwrite else "f32_acc"
            G.gemm(v.t(), x.t(), self.lora.gA(i, t), epi=acc)               # dA = (s v)^T x
            G.gemm(dy.t(), self._u[(i, t)].t(), self.lora.gB(i, t), epi=acc)  # dB = dy^T (s u)
        else:
            fn = self._take_fused(i, t)
            alpha = self._sd_scale if t in ("wo", "wdown") else 1.0
            if fn is not None:
                with ph("bwd.gemm_dgrad+gather"):
                    fn(dy, self._p(name).t(), dx_out)
            else:
                with ph("bwd.gemm_dgrad"):
                    G.gemm(dy, self._p(name).t(), dx_out, alpha=alpha)
        self._wgrad(dy, x, name, alpha=alpha if self.lora is None or not self.lora.has(i, t) else 1.0)

    # -------------------------------------------------------------- dropout
    def _drop_seed(self, i: int, site: int) -> int:
        return ((self.dropout_seed * 1000003 + self._drop_step) * 4099 + i * 2 + site) & 0x7FFFFFFFFFFFFFFF

    def _dropping(self, ws: _Workspace) -> bool:
        return self.cfg.dropout > 0 and ws.od is not None

    # ----------------------------------------------------- stochastic depth
    def _layer_keep_prob(self, i: int) -> float:
        return 1.0 - (i + 1) / self.cfg.num_layers * self.cfg.stochastic_depth

    def _layer_dropped(self, i: int) -> bool:
        """Training only: is layer i skipped in this micro-step?  A counter hash
        of (seed, micro-step, layer), so the backward and the recomputation see
        the forward's decision.  (Huang et al. 2016's linear decay; the
        reference's StochasticDepth keeps layer l with p (1 - l / L), which
        drops the deepest layers almost always.)"""
        sd = self.cfg.stochastic_depth
        if sd <= 0 or not self._saving:
            return False
        h = (self._drop_seed(i, 7) * 0x9E3779B97F4A7C15 + 0xD1B54A32D192ED03) & 0xFFFFFFFFFFFFFFFF
        h ^= h >> 31
        h = (h * 0xBF58476D1CE4E5B9) & 0xFFFFFFFFFFFFFFFF
        h ^= h >> 29
        return (h >> 11) / float(1 << 53) >= self._layer_keep_prob(i)

    def _skip_layer_fwd(self, i: int, h_in: torch.Tensor, h_out: torch.Tensor) -> bool:
        self._sd_scale = 1.0
        if self.cfg.stochastic_depth <= 0 or not self._saving:
            return False
        if self._layer_dropped(i):
            if h_out.data_ptr() != h_in.data_ptr():
                h_out.copy_(h_in)  # identity layer
            return True
        self._sd_scale = 1.0 / self._layer_keep_prob(i)
        return False

    # -------------------------------------------------------------- forward
    def _layer_fwd(self, i: int, ws: _Workspace, h_in: torch.Tensor, h_out: torch.Tensor, slot: int):
        cfg = self.cfg
        p = f"layers.{i}."
        if self._skip_layer_fwd(i, h_in, h_out):
            return
        drop = self._dropping(ws)
        xn1, rstd1 = ws.xn1[slot], ws.rstd1[slot]
        with ph("fwd.rmsnorm"):
            N.rmsnorm_fwd(h_in, self._p(p + "attn_norm"), cfg.norm_eps, y=xn1, rstd=rstd1)
        qkv = ws.qkv[slot]
        nrot = cfg.num_heads + cfg.num_kv_heads
        # With fuse_rope, RoPE of q and k runs in the QKV GEMM's epilogue (whole-sequence
        # micro-batches).  Off by default: the row-per-thread epilogue's table reads
        # measured 2.62 ms per step against 2.12 ms for GEMM + separate RoPE (1.1B).
        rope = (self.rope, nrot * cfg.head_dim, cfg.head_dim, ws.S, 0) \
            if self.ctx is None and self.fuse_rope else None
        roped = self._lin(i, "wqkv", xn1, qkv, save=self._saving, rope=rope)
        if self.ctx is None:
            if not roped:
                with ph("fwd.rope"):
                    E.rope_(qkv, 0, nrot, cfg.head_dim, self.rope, seq_len=ws.S)
            with ph("fwd.attention"):
                A.attention_fwd(qkv, ws.B, ws.S, cfg.num_heads, cfg.num_kv_heads, cfg.head_dim,
                                causal=True, window=self.attn_window, out=ws.o[slot], lse=ws.lse[slot])
        else:
            E.rope_(qkv, 0, cfg.num_heads + cfg.num_kv_heads, cfg.head_dim, self.rope, seq_len=ws.S,
                    **self.ctx.rope_args(ws.B, ws.S, self.device))
            self.ctx.forward(qkv, ws.B, ws.S, ws.o[slot], key=(id(ws), slot), window=self.attn_window)
        o_in = ws.o[slot]
        if drop:  # attention-context dropout into its own buffer
            o_in = E.dropout(o_in, cfg.dropout, self._drop_seed(i, 0), out=ws.od[slot])
        hmid = ws.hmid[slot]
        self._lin(i, "wo", o_in, hmid, residual=h_in, save=self._saving)
        with ph("fwd.rmsnorm"):
            N.rmsnorm_fwd(hmid, self._p(p + "ffn_norm"), cfg.norm_eps, y=ws.xn2[slot], rstd=ws.rstd2[slot])
        self._lin_swiglu(i, ws.xn2[slot], ws.gu[slot], ws.act[slot], save=self._saving)
        if drop:  # FFN-hidden dropout in place (its backward reads gu, not act)
            E.dropout(ws.act[slot], cfg.dropout, self._drop_seed(i, 1), out=ws.act[slot])
        self._lin(i, "wdown", ws.act[slot], h_out, residual=hmid, save=self._saving)

    def _forward(self, ids: torch.Tensor, ws: _Workspace, save: bool) -> torch.Tensor:
        cfg = self.cfg
        self._saving = save
        self._hook("pre_forward")
        with ph("fwd.embedding"):
            E.embedding_fwd(ids.reshape(-1), self._p("embed"), out=ws.h[0])
        for i in range(cfg.num_layers):
            self._hook("pre_layer_fwd", i)
            if save:
                self._layer_fwd(i, ws, ws.h[i], ws.h[i + 1], 0 if self.recompute else i)
            else:
                self._layer_fwd(i, ws, ws.h[i % 2], ws.h[(i + 1) % 2], 0)
        h_last = ws.h[cfg.num_layers] if save else ws.h[cfg.num_layers % 2]
        with ph("fwd.rmsnorm"):
            N.rmsnorm_fwd(h_last, self._p("final_norm"), cfg.norm_eps, y=ws.xf, rstd=ws.rstdf)
        if ws.logits is not None:  # else: the vocabulary-chunked head runs in forward_backward
            with ph("fwd.gemm_lm_head"):
                G.linear(ws.xf, self._p("lm_head"), out=ws.logits)
        return ws.logits

    @torch.no_grad()
    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        """Logits [B, S, V] (bf16) of a full-sequence forward."""
        B, S = ids.shape
        ws = self.workspace(B, S, save=False)
        return self._forward(ids, ws, save=False).view(B, S, -1)

    # ----------------------------------------------------- forward+backward
    @torch.no_grad()
    def forward_backward(self, ids: torch.Tensor, targets: torch.Tensor, *,
                         loss_scale: Optional[torch.Tensor] = None, grad_scale: float = 1.0,
                         label_smoothing: float = 0.0, z_loss: float = 0.0,
                         loss_acc: Optional[torch.Tensor] = None,
                         overwrite_grads: bool = False) -> torch.Tensor:
        """One micro-batch: forward, fused CE, backward.  Gradients (scaled by
        *loss_scale x grad_scale) accumulate into self.grads.  Returns the
        device tensor [sum of token losses, token count] (accumulated into
        loss_acc when given).  overwrite_grads: store instead of accumulate
        (first micro-step of an accumulation window; no zeroing pass needed)."""
        cfg = self.cfg
        self._overwrite = overwrite_grads
        B, S = ids.shape
        ws = self.workspace(B, S, save=True)
        acc = ws.loss_acc if loss_acc is None else loss_acc
        if loss_acc is None:
            acc.zero_()
        self._forward(ids, ws, save=True)
        if ws.logits is None:
            self._lm_head_ce_chunked(ws, targets.reshape(-1), acc, loss_scale, grad_scale, label_smoothing, z_loss)
        else:
            # K9: loss + dlogits in place (scaled)
            with ph("fwd.cross_entropy"):
                L.cross_entropy_(ws.logits, targets.reshape(-1), acc, scale=loss_scale, scale_mul=grad_scale,
                                 smoothing=label_smoothing, z_loss=z_loss)
            dlogits = ws.logits
            # LM head
            with ph("bwd.gemm_dgrad"):
                G.linear_dgrad(dlogits, self._p("lm_head"), out=ws.dx)
            self._wgrad(dlogits, ws.xf, "lm_head")
        L_ = cfg.num_layers
        with ph("bwd.rmsnorm"):
            N.rmsnorm_bwd(ws.dx, ws.h[L_], self._p("final_norm"), ws.rstdf, self._g("final_norm"), dx=ws.dh,
                          accumulate=not overwrite_grads)
        self._hook("post_head_bwd")
        for i in reversed(range(L_)):
            self._hook("pre_layer_bwd", i)
            if self.recompute:
                # regenerate slot 0 (h[i+1] is rewritten with identical values; layer
                # i+1's backward, its only other reader, has already run)
                self._saving = True
                self._layer_fwd(i, ws, ws.h[i], ws.h[i + 1], 0)
            self._layer_bwd(i, ws)
            self._hook("post_layer_bwd", i)
        if self.train_base:
            with ph("bwd.embedding"):
                if overwrite_grads and not cfg.tie_embeddings:
                    self._g("embed").zero_()
                E.embedding_bwd(ids.reshape(-1), ws.dh, self._g("embed"))
        self._hook("post_backward")
        self._overwrite = False
        self._drop_step += 1
        return acc

    def _lm_head_ce_chunked(self, ws: _Workspace, targets: torch.Tensor, acc: torch.Tensor, loss_scale,
                            grad_scale: float, smoothing: float, z_loss: float) -> None:
        """LM head + cross-entropy without the [T, V] logits: pass 1 computes
        each vocabulary chunk's logits into one reusable buffer and keeps per-row
        statistics {max, sum exp, sum z, z[target]}; pass 2 recomputes each
        chunk, turns it into its gradient slice with the combined statistics,
        and feeds the dgrad GEMM (fp32 sum over chunks into dx) and the weight
        gradient of the chunk's rows.  One extra LM-head GEMM buys the memory
        of the logits (2.1 GB at 8192 tokens x 128256 words)."""
        cfg = self.cfg
        T, V, D = ws.T, cfg.vocab_size, cfg.hidden_dim
        chunk = self.ce_chunk(T)
        n = (V + chunk - 1) // chunk
        W = self._p("lm_head")
        # scratch: the logits chunk (bf16) and the fp32 input gradient, in the
        # SwiGLU-gradient buffer (unused until the layers' backward) when it fits
        need = T * chunk + 2 * T * D
        buf = ws.dgu.view(-1)
        if buf.numel() < need:
            if getattr(ws, "ce_scratch", None) is None or ws.ce_scratch.numel() < need:
                ws.ce_scratch = torch.empty(need, dtype=torch.bfloat16, device=self.device)
            buf = ws.ce_scratch
        dx32 = buf[T * chunk:T * chunk + 2 * T * D].view(torch.float32).view(T, D)
        if getattr(ws, "ce_stats", None) is None or ws.ce_stats.shape[0] != n:
            ws.ce_stats = torch.empty(n, T, 4, dtype=torch.float32, device=self.device)
            ws.ce_stat_ptrs = torch.tensor([ws.ce_stats[c].data_ptr() for c in range(n)], dtype=torch.int64,
                                           device=self.device)
            ws.ce_dummy = torch.zeros(2, dtype=torch.float32, device=self.device)

        def logits_chunk(c):
            v0 = c * chunk
            vc = min(chunk, V - v0)
            lg = buf[:T * vc].view(T, vc)
            with ph("fwd.gemm_lm_head"):
                G.linear(ws.xf, W[v0:v0 + vc], out=lg)
            return v0, vc, lg

        for c in range(n):
            v0, vc, lg = logits_chunk(c)
            with ph("fwd.cross_entropy"):
                L.cross_entropy_chunk_stats(lg, targets, v0, V, ws.ce_stats[c], ws.ce_dummy, ws.ce_stat_ptrs)
        for c in range(n):
            v0, vc, lg = logits_chunk(c)  # recomputed: nothing of size [T, V] is kept
            with ph("fwd.cross_entropy"):
                L.cross_entropy_chunk_grad(lg, targets, v0, V, ws.ce_stats[c], ws.ce_stat_ptrs,
                                           acc if c == 0 else ws.ce_dummy, scale=loss_scale, scale_mul=grad_scale,
                                           smoothing=smoothing, z_loss=z_loss)
            with ph("bwd.gemm_dgrad"):
                G.gemm(lg, W[v0:v0 + vc].t(), dx32, epi="f32" if c == 0 else "f32_acc")
            self._wgrad(lg, ws.xf, "lm_head", rows=(v0, vc))
        E.cast_f32_bf16(dx32, out=ws.dx)

    def _layer_bwd(self, i: int, ws: _Workspace, slot: Optional[int] = None, hidx: Optional[int] = None):
        """Backward of layer i with the running residual gradient in ws.dh.
        slot: workspace slot of its intermediates; hidx: index of its input in
        ws.h (both default to the whole-model positions)."""
        cfg = self.cfg
        p = f"layers.{i}."
        self._sd_scale = 1.0
        if cfg.stochastic_depth > 0:
            if self._layer_dropped(i):  # identity: dh passes through, the weights get no gradient
                for t in ("wqkv", "wo", "wgu", "wdown", "attn_norm", "ffn_norm"):
                    g = self._g(p + t)
                    if self._overwrite or g.dtype == torch.bfloat16:
                        g.zero_()
                return
            self._sd_scale = 1.0 / self._layer_keep_prob(i)
        s = slot if slot is not None else (0 if self.recompute else i)
        h_in = ws.h[i if hidx is None else hidx]
        dh = ws.dh
        drop = self._dropping(ws)
        # FFN.  With fuse_swiglu_bwd the down projection's data gradient carries the
        # SwiGLU backward in its epilogue (gate|up gradients straight from the
        # accumulator; not with dropout, a LoRA adapter or a fused parameter gather
        # in between).  Off by default: the row-per-thread epilogue's uncoalesced
        # gate|up traffic measured 0.46 ms per layer against 0.20 ms for the GEMM
        # plus the separate bandwidth-bound SwiGLU backward (1.1B step).
        fg = self.fused_gather
        if (self.fuse_swiglu_bwd and not drop and not (self.lora is not None and self.lora.has(i, "wdown"))
                and not (fg is not None and fg[0] == i and fg[1] == "wdown")):
            with ph("bwd.gemm_dgrad+swiglu"):
                G.gemm(dh, self._p(p + "wdown").t(), ws.dgu, epi="swiglu_bwd", residual=ws.gu[s],
                       alpha=self._sd_scale)
            self._wgrad(dh, ws.act[s], p + "wdown", alpha=self._sd_scale)
        else:
            self._lin_bwd(i, "wdown", dh, ws.act[s], ws.dact)
            if drop:
                E.dropout(ws.dact, cfg.dropout, self._drop_seed(i, 1), out=ws.dact)
            with ph("bwd.swiglu"):
                E.swiglu_bwd(ws.gu[s], ws.dact, ws.dgu)
        self._lin_bwd(i, "wgu", ws.dgu, ws.xn2[s], ws.dx)
        with ph("bwd.rmsnorm"):
            N.rmsnorm_bwd(ws.dx, ws.hmid[s], self._p(p + "ffn_norm"), ws.rstd2[s], self._g(p + "ffn_norm"),
                          dres=dh, dx=dh, accumulate=not self._overwrite)
        # attention
        self._lin_bwd(i, "wo", dh, ws.od[s] if drop else ws.o[s], ws.do)
        if drop:
            E.dropout(ws.do, cfg.dropout, self._drop_seed(i, 0), out=ws.do)
        if self.ctx is None:
            with ph("bwd.attention"):
                A.attention_bwd(ws.qkv[s], ws.o[s], ws.do, ws.lse[s], ws.B, ws.S, cfg.num_heads,
                                cfg.num_kv_heads, cfg.head_dim, causal=True, window=self.attn_window,
                                dqkv=ws.dqkv)
            off = {}
        else:
            self.ctx.backward(ws.do, ws.B, ws.S, ws.dqkv, key=(id(ws), s), window=self.attn_window)
            off = self.ctx.rope_args(ws.B, ws.S, self.device)
        with ph("bwd.rope"):
            E.rope_(ws.dqkv, 0, cfg.num_heads + cfg.num_kv_heads, cfg.head_dim, self.rope, seq_len=ws.S,
                    inverse=True, **off)
        self._lin_bwd(i, "wqkv", ws.dqkv, ws.xn1[s], ws.dx)
        with ph("bwd.rmsnorm"):
            N.rmsnorm_bwd(ws.dx, h_in, self._p(p + "attn_norm"), ws.rstd1[s], self._g(p + "attn_norm"),
                          dres=dh, dx=dh, accumulate=not self._overwrite)
