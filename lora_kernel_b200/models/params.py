"""Flat parameter storage for the Llama decoder.

All weights live in one bf16 buffer (and, for training, one fp32 master buffer,
one fp32 gradient buffer and the AdamW moments with the same layout); every
named parameter is a view.  This makes the optimizer one kernel over one
buffer, lets the weight-gradient GEMMs accumulate straight into the fp32
gradient views, and makes ZeRO sharding a slice of a flat range.

Layout: parameters are grouped per layer ("embed", "layers.{i}", "head") so a
ZeRO-3 rank can gather one layer at a time; every tensor starts on a 64-element
(128-byte) boundary so TMA descriptors over any view are aligned.

Internal orientation is [out, in] (y = x W^T); Wq/Wk/Wv are fused row-wise into
`wqkv` and Wgate/Wup are interleaved in blocks of 128 rows into `wgu` (the
gate|up GEMM's SwiGLU epilogue layout).  `to_reference_state_dict` converts to
the reference's checkpoint names and [in, out] orientation
(include/io/serialization.hpp:13-44).
"""
from __future__ import annotations

import math
from collections import OrderedDict
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import torch

from ..config import TransformerConfig

ALIGN = 64


@dataclass
class ParamSpec:
    name: str
    shape: Tuple[int, ...]
    offset: int
    group: str
    decay: bool
    init: str  # "normal" | "ones" | "zeros"
    gidx: int = -1  # index of this tensor in the full model's layout (seeds its init)

    @property
    def numel(self) -> int:
        n = 1
        for s in self.shape:
            n *= s
        return n


def _round(n: int) -> int:
    return (n + ALIGN - 1) // ALIGN * ALIGN


LAYER_TENSORS = 6  # attn_norm, wqkv, wo, ffn_norm, wgu, wdown


def build_layout(cfg: TransformerConfig, group_align: int = ALIGN, layers: Optional[range] = None,
                 embed: bool = True, head: bool = True
                 ) -> Tuple[List[ParamSpec], Dict[str, Tuple[int, int]], int]:
    """Returns (specs, group ranges {group: (start, end)}, total numel).  Every
    group is padded to a multiple of `group_align` elements (64 x world size for
    ZeRO sharding, so each rank owns an equal, aligned chunk of every group).

    layers / embed / head select a subset of the model (a pipeline stage):
    layer tensors keep their global names ("layers.{i}.*") and every spec
    records its index in the full layout, so a stage initialises exactly the
    weights the whole model would."""
    assert group_align % ALIGN == 0
    D, V, F = cfg.hidden_dim, cfg.vocab_size, cfg.ff_dim_padded
    layers = range(cfg.num_layers) if layers is None else layers
    specs: List[ParamSpec] = []
    groups: Dict[str, Tuple[int, int]] = OrderedDict()
    off = 0

    def add(name, shape, group, decay, init, gidx):
        nonlocal off
        s = ParamSpec(name, tuple(shape), off, group, decay, init, gidx)
        specs.append(s)
        off += _round(s.numel)

    def group(name, items, g0):
        nonlocal off
        start = off
        for k, it in enumerate(items):
            add(*it[:2], name, *it[2:], g0 + k)
        off = (off + group_align - 1) // group_align * group_align
        groups[name] = (start, off)

    if embed:
        group("embed", [("embed", (V, D), True, "normal")], 0)
    for i in layers:
        p = f"layers.{i}."
        group(f"layers.{i}", [
            (p + "attn_norm", (D,), False, "ones"),
            (p + "wqkv", (cfg.qkv_dim, D), True, "normal"),
            (p + "wo", (D, cfg.q_dim), True, "normal"),
            (p + "ffn_norm", (D,), False, "ones"),
            (p + "wgu", (2 * F, D), True, "normal"),
            (p + "wdown", (D, F), True, "normal"),
        ], 1 + LAYER_TENSORS * i)
    if head:
        items = [("final_norm", (D,), False, "ones")]
        if not cfg.tie_embeddings:
            items.append(("lm_head", (V, D), True, "normal"))
        group("head", items, 1 + LAYER_TENSORS * cfg.num_layers)
    return specs, groups, off


class FlatParams:
    """A flat buffer plus named views following `build_layout(cfg)`."""

    def __init__(self, cfg: TransformerConfig, device, dtype=torch.bfloat16,
                 buffer: Optional[torch.Tensor] = None, group_align: int = ALIGN,
                 layers: Optional[range] = None, embed: bool = True, head: bool = True):
        self.cfg = cfg
        self.group_align = group_align
        self.layer_ids = range(cfg.num_layers) if layers is None else layers
        self.has_embed, self.has_head = embed, head
        self.specs, self.groups, self.numel = build_layout(cfg, group_align, self.layer_ids, embed, head)
        self.by_name = {s.name: s for s in self.specs}
        if buffer is None:
            buffer = torch.zeros(self.numel, dtype=dtype, device=device)
        assert buffer.numel() == self.numel
        self.flat = buffer
        self.views: Dict[str, torch.Tensor] = {
            s.name: self.flat[s.offset:s.offset + s.numel].view(s.shape) for s in self.specs}

    def __getitem__(self, name: str) -> torch.Tensor:
        if name == "lm_head" and self.cfg.tie_embeddings:
            return self.views["embed"]
        return self.views[name]

    def like(self, dtype=torch.float32, device=None) -> "FlatParams":
        return FlatParams(self.cfg, device or self.flat.device, dtype,
                          torch.zeros(self.numel, dtype=dtype, device=device or self.flat.device),
                          self.group_align, self.layer_ids, self.has_embed, self.has_head)

    def group_of(self, name: str) -> str:
        return self.by_name[name].group

    def segments(self, decay_norms: bool = False, lo: int = 0, hi: Optional[int] = None):
        """(start, length, decay) of every parameter clipped to [lo, hi), relative to lo."""
        hi = self.numel if hi is None else hi
        out = []
        for s in self.specs:
            a, b = max(s.offset, lo), min(s.offset + s.numel, hi)
            if a < b:
                out.append((a - lo, b - a, s.decay or decay_norms))
        return out

    # ------------------------------------------------------------------ init
    def init_(self, seed: int, std: float) -> None:
        """Deterministic N(0, std) for matrices, ones for norms; the padded FFN
        rows/columns are zero so the padding is exact."""
        cfg = self.cfg
        F, Fp = cfg.ff_dim, cfg.ff_dim_padded
        dev = self.flat.device
        for s in self.specs:
            idx = s.gidx
            v = self.views[s.name]
            if s.init == "ones":
                v.fill_(1.0)
            elif s.init == "zeros":
                v.zero_()
            else:
                # one generator per tensor, seeded by (seed, tensor index): every
                # rank reproduces the same weights for any tensor independently
                g = torch.Generator(device=dev).manual_seed(seed * 1000003 + idx)
                t = torch.empty(s.shape, dtype=torch.float32, device=dev)
                t.normal_(0.0, std, generator=g)
                if s.name.endswith("wgu") and Fp != F:
                    blk = t.view(Fp // 128, 2, 128, -1)
                    mask = (torch.arange(Fp, device=dev) >= F).view(Fp // 128, 128)
                    blk[:, 0][mask] = 0.0
                    blk[:, 1][mask] = 0.0
                if s.name.endswith("wdown") and Fp != F:
                    t[:, F:] = 0.0
                v.copy_(t.to(v.dtype))

    # ------------------------------------------------------- checkpoint names
    def to_reference_state_dict(self) -> "OrderedDict[str, torch.Tensor]":
        """Reference tensor names, [in, out] orientation, unpadded FFN."""
        cfg = self.cfg
        q, kv, F = cfg.q_dim, cfg.kv_dim, cfg.ff_dim
        out: "OrderedDict[str, torch.Tensor]" = OrderedDict()
        if self.has_embed:
            out["token_embedding.weight"] = self.views["embed"]
        for i in self.layer_ids:
            p, r = f"layers.{i}.", f"blocks.{i}."
            wqkv = self.views[p + "wqkv"]
            out[r + "attn.Wq.weight"] = wqkv[:q].t()
            out[r + "attn.Wk.weight"] = wqkv[q:q + kv].t()
            out[r + "attn.Wv.weight"] = wqkv[q + kv:].t()
            out[r + "attn.Wo.weight"] = self.views[p + "wo"].t()
            wgu = self.views[p + "wgu"]
            Fp = wgu.shape[0] // 2
            blk = wgu.view(Fp // 128, 2, 128, -1)
            out[r + "ffn.Wgate.weight"] = blk[:, 0].reshape(Fp, -1)[:F].t()
            out[r + "ffn.Wup.weight"] = blk[:, 1].reshape(Fp, -1)[:F].t()
            out[r + "ffn.Wdown.weight"] = self.views[p + "wdown"][:, :F].t()
            out[r + "rms_norm_attn.weight"] = self.views[p + "attn_norm"]
            out[r + "rms_norm_ffn.weight"] = self.views[p + "ffn_norm"]
        if self.has_head:
            out["final_norm.weight"] = self.views["final_norm"]
            if not cfg.tie_embeddings:
                out["lm_head.weight"] = self.views["lm_head"].t()
        return out

    def load_reference_state_dict(self, sd: Dict[str, torch.Tensor]) -> None:
        cfg = self.cfg
        q, kv, F = cfg.q_dim, cfg.kv_dim, cfg.ff_dim
        with torch.no_grad():
            if self.has_embed:
                self.views["embed"].copy_(sd["token_embedding.weight"])
            for i in self.layer_ids:
                p, r = f"layers.{i}.", f"blocks.{i}."
                wqkv = self.views[p + "wqkv"]
                wqkv[:q].copy_(sd[r + "attn.Wq.weight"].t())
                wqkv[q:q + kv].copy_(sd[r + "attn.Wk.weight"].t())
                wqkv[q + kv:].copy_(sd[r + "attn.Wv.weight"].t())
                self.views[p + "wo"].copy_(sd[r + "attn.Wo.weight"].t())
                wgu = self.views[p + "wgu"]
                Fp = wgu.shape[0] // 2
                blk = wgu.view(Fp // 128, 2, 128, -1)
                g = torch.zeros(Fp, wgu.shape[1], dtype=wgu.dtype, device=wgu.device)
                u = torch.zeros_like(g)
                g[:F] = sd[r + "ffn.Wgate.weight"].t()
                u[:F] = sd[r + "ffn.Wup.weight"].t()
                blk[:, 0].copy_(g.view(Fp // 128, 128, -1))
                blk[:, 1].copy_(u.view(Fp // 128, 128, -1))
                wd = self.views[p + "wdown"]
                wd.zero_()
                wd[:, :F].copy_(sd[r + "ffn.Wdown.weight"].t())
                self.views[p + "attn_norm"].copy_(sd[r + "rms_norm_attn.weight"])
                self.views[p + "ffn_norm"].copy_(sd[r + "rms_norm_ffn.weight"])
            if self.has_head:
                self.views["final_norm"].copy_(sd["final_norm.weight"])
                if not cfg.tie_embeddings:
                    self.views["lm_head"].copy_(sd["lm_head.weight"].t())
