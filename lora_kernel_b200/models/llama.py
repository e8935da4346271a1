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

import math
from typing import Dict, Optional, Tuple

import torch

from ..config import TransformerConfig
from ..ops import attention as A
from ..ops import elementwise as E
from ..ops import gemm as G
from ..ops import loss as L
from ..ops import norm as N
from .params import FlatParams


class _Workspace:
    def __init__(self, cfg: TransformerConfig, B: int, S: int, device, save: bool):
        T = B * S
        D, F, V = cfg.hidden_dim, cfg.ff_dim_padded, cfg.vocab_size
        nl = cfg.num_layers if save else 1
        bf = dict(dtype=torch.bfloat16, device=device)
        f32 = dict(dtype=torch.float32, device=device)
        self.B, self.S, self.T = B, S, T
        self.h = [torch.empty(T, D, **bf) for _ in range(cfg.num_layers + 1)] if save else \
            [torch.empty(T, D, **bf) for _ in range(2)]
        self.xn1 = [torch.empty(T, D, **bf) for _ in range(nl)]
        self.rstd1 = [torch.empty(T, **f32) for _ in range(nl)]
        self.qkv = [torch.empty(T, cfg.qkv_dim, **bf) for _ in range(nl)]
        self.o = [torch.empty(T, cfg.q_dim, **bf) for _ in range(nl)]
        self.lse = [torch.empty(B, cfg.num_heads, S, **f32) for _ in range(nl)]
        self.hmid = [torch.empty(T, D, **bf) for _ in range(nl)]
        self.xn2 = [torch.empty(T, D, **bf) for _ in range(nl)]
        self.rstd2 = [torch.empty(T, **f32) for _ in range(nl)]
        self.gu = [torch.empty(T, 2 * F, **bf) for _ in range(nl)]
        self.act = [torch.empty(T, F, **bf) for _ in range(nl)]
        self.xf = torch.empty(T, D, **bf)
        self.rstdf = torch.empty(T, **f32)
        self.logits = torch.empty(T, V, **bf)
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

    # -------------------------------------------------------------- helpers
    def workspace(self, B: int, S: int, save: bool = True) -> _Workspace:
        key = (B, S, save)
        ws = self._ws.get(key)
        if ws is None:
            if S > self.rope.shape[0]:
                self.rope = E.rope_table(S, self.cfg.head_dim, self.cfg.rope_base, self.device)
            ws = _Workspace(self.cfg, B, S, self.device, save)
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

    def _wgrad(self, dy, x, name):
        """Weight gradient: stored on the first micro-step of a window, else accumulated."""
        G.gemm(dy.t(), x.t(), self._g(name), epi="f32" if self._overwrite else "f32_acc")

    # -------------------------------------------------------------- forward
    def _layer_fwd(self, i: int, ws: _Workspace, h_in: torch.Tensor, h_out: torch.Tensor, slot: int):
        cfg = self.cfg
        p = f"layers.{i}."
        xn1, rstd1 = ws.xn1[slot], ws.rstd1[slot]
        N.rmsnorm_fwd(h_in, self._p(p + "attn_norm"), cfg.norm_eps, y=xn1, rstd=rstd1)
        qkv = ws.qkv[slot]
        G.linear(xn1, self._p(p + "wqkv"), out=qkv)
        E.rope_(qkv, 0, cfg.num_heads + cfg.num_kv_heads, cfg.head_dim, self.rope, seq_len=ws.S)
        A.attention_fwd(qkv, ws.B, ws.S, cfg.num_heads, cfg.num_kv_heads, cfg.head_dim,
                        causal=True, window=self.attn_window, out=ws.o[slot], lse=ws.lse[slot])
        hmid = ws.hmid[slot]
        G.linear(ws.o[slot], self._p(p + "wo"), residual=h_in, out=hmid)
        N.rmsnorm_fwd(hmid, self._p(p + "ffn_norm"), cfg.norm_eps, y=ws.xn2[slot], rstd=ws.rstd2[slot])
        G.linear_swiglu(ws.xn2[slot], self._p(p + "wgu"), gu_out=ws.gu[slot], h_out=ws.act[slot])
        G.linear(ws.act[slot], self._p(p + "wdown"), residual=hmid, out=h_out)

    def _forward(self, ids: torch.Tensor, ws: _Workspace, save: bool) -> torch.Tensor:
        cfg = self.cfg
        self._hook("pre_forward")
        E.embedding_fwd(ids.reshape(-1), self._p("embed"), out=ws.h[0])
        for i in range(cfg.num_layers):
            self._hook("pre_layer_fwd", i)
            if save:
                self._layer_fwd(i, ws, ws.h[i], ws.h[i + 1], i)
            else:
                self._layer_fwd(i, ws, ws.h[i % 2], ws.h[(i + 1) % 2], 0)
        h_last = ws.h[cfg.num_layers] if save else ws.h[cfg.num_layers % 2]
        N.rmsnorm_fwd(h_last, self._p("final_norm"), cfg.norm_eps, y=ws.xf, rstd=ws.rstdf)
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
        # K9: loss + dlogits in place (scaled)
        L.cross_entropy_(ws.logits, targets.reshape(-1), acc, scale=loss_scale, scale_mul=grad_scale,
                         smoothing=label_smoothing, z_loss=z_loss)
        dlogits = ws.logits
        # LM head
        G.linear_dgrad(dlogits, self._p("lm_head"), out=ws.dx)
        self._wgrad(dlogits, ws.xf, "lm_head")
        L_ = cfg.num_layers
        N.rmsnorm_bwd(ws.dx, ws.h[L_], self._p("final_norm"), ws.rstdf, self._g("final_norm"), dx=ws.dh,
                      accumulate=not overwrite_grads)
        self._hook("post_head_bwd")
        for i in reversed(range(L_)):
            self._hook("pre_layer_bwd", i)
            self._layer_bwd(i, ws)
            self._hook("post_layer_bwd", i)
        if overwrite_grads and not cfg.tie_embeddings:
            self._g("embed").zero_()
        E.embedding_bwd(ids.reshape(-1), ws.dh, self._g("embed"))
        self._hook("post_backward")
        self._overwrite = False
        return acc

    def _layer_bwd(self, i: int, ws: _Workspace):
        cfg = self.cfg
        p = f"layers.{i}."
        dh = ws.dh
        # FFN
        G.linear_dgrad(dh, self._p(p + "wdown"), out=ws.dact)
        self._wgrad(dh, ws.act[i], p + "wdown")
        E.swiglu_bwd(ws.gu[i], ws.dact, ws.dgu)
        G.linear_dgrad(ws.dgu, self._p(p + "wgu"), out=ws.dx)
        self._wgrad(ws.dgu, ws.xn2[i], p + "wgu")
        N.rmsnorm_bwd(ws.dx, ws.hmid[i], self._p(p + "ffn_norm"), ws.rstd2[i], self._g(p + "ffn_norm"),
                      dres=dh, dx=dh, accumulate=not self._overwrite)
        # attention
        G.linear_dgrad(dh, self._p(p + "wo"), out=ws.do)
        self._wgrad(dh, ws.o[i], p + "wo")
        A.attention_bwd(ws.qkv[i], ws.o[i], ws.do, ws.lse[i], ws.B, ws.S, cfg.num_heads,
                        cfg.num_kv_heads, cfg.head_dim, causal=True, window=self.attn_window,
                        dqkv=ws.dqkv)
        E.rope_(ws.dqkv, 0, cfg.num_heads + cfg.num_kv_heads, cfg.head_dim, self.rope, seq_len=ws.S,
                inverse=True)
        G.linear_dgrad(ws.dqkv, self._p(p + "wqkv"), out=ws.dx)
        self._wgrad(ws.dqkv, ws.xn1[i], p + "wqkv")
        N.rmsnorm_bwd(ws.dx, ws.h[i], self._p(p + "attn_norm"), ws.rstd1[i], self._g(p + "attn_norm"),
                      dres=dh, dx=dh, accumulate=not self._overwrite)
