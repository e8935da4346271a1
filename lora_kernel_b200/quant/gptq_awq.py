"""Import of 4-bit GPTQ and AWQ checkpoints into the int4 format of this framework.

Both public formats store, per linear layer `name` of a Hugging Face Llama
model (weights [out N, in K]):

    GPTQ (AutoGPTQ)  name.qweight int32 [K/8, N]: eight 4-bit codes along K per
                     int32, code k % 8 at bits 4*(k % 8);
                     name.qzeros  int32 [K/G, N/8]: eight zero points along N per
                     int32, stored minus one;
                     name.scales  fp16 [K/G, N]; name.g_idx int32 [K] (group of
                     each input column; only k // G, i.e. no activation reordering,
                     is accepted)
    AWQ (AutoAWQ)    name.qweight int32 [K, N/8]: eight codes along N per int32 in
                     the order 0, 2, 4, 6, 1, 3, 5, 7 of the eight columns;
                     name.qzeros  int32 [K/G, N/8]: zero points, same packing;
                     name.scales  fp16 [K/G, N]

with w[n, k] = scale[g, n] * (code[k, n] - zero[g, n]), g = k // G.  Here a
weight becomes Int4Parts (codes [N, K], scales and zero points [N, K/G]), the
layout of the int4 dequantising kernels (K14) once two codes are packed per
byte (`pack_nibbles`).  `llama_parts_to_engine` then maps a Llama model's
projections to the engine's fused layout: q|k|v rows stacked (q and k rows
reordered from rotate-half to adjacent-pair RoPE), gate|up interleaved in
blocks of 128 rows.  `load_gptq_awq` reads a safetensors file and returns the
dict the serving ModelRunner takes as `params`.

Reference: QuantizedModelLoader::load_awq / load_gptq
(include/api/serving_production.hpp:231-241), stubs there.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, Optional

import torch

AWQ_ORDER = (0, 2, 4, 6, 1, 3, 5, 7)   # column of the group of eight held by nibble i


@dataclass
class Int4Parts:
    q: torch.Tensor        # uint8 codes 0..15, [N, K]
    scale: torch.Tensor    # fp32 [N, K/G]
    zero: torch.Tensor     # fp32 [N, K/G]
    group: int

    @property
    def shape(self):
        return tuple(self.q.shape)

    def dequantize(self) -> torch.Tensor:
        g = self.group
        s = self.scale.repeat_interleave(g, dim=1)
        z = self.zero.repeat_interleave(g, dim=1)
        return (self.q.float() - z) * s

    def rows(self, idx: torch.Tensor) -> "Int4Parts":
        return Int4Parts(self.q[idx], self.scale[idx], self.zero[idx], self.group)


def _nibbles(x: torch.Tensor) -> torch.Tensor:
    """int32 [..., M] -> uint8 [..., M, 8]: nibble i = bits 4i..4i+3."""
    x = x.to(torch.int64) & 0xFFFFFFFF
    sh = torch.arange(0, 32, 4, dtype=torch.int64)
    return ((x[..., None] >> sh) & 0xF).to(torch.uint8)


def unpack_gptq(qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor,
                g_idx: Optional[torch.Tensor] = None) -> Int4Parts:
    K8, N = qweight.shape
    K = K8 * 8
    G = K // scales.shape[0]
    if g_idx is not None and not torch.equal(g_idx.to(torch.int64).cpu(), torch.arange(K) // G):
        raise NotImplementedError("GPTQ with activation reordering (g_idx other than k // group)")
    codes = _nibbles(qweight).permute(0, 2, 1).reshape(K, N)          # [K, N]
    zeros = _nibbles(qzeros).reshape(qzeros.shape[0], -1)[:, :N].float() + 1.0   # stored minus one
    return Int4Parts(codes.t().contiguous(), scales.float().t().contiguous(), zeros.t().contiguous(), G)


def unpack_awq(qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor) -> Int4Parts:
    K, N8 = qweight.shape
    N = N8 * 8
    G = K // scales.shape[0]
    inv = torch.tensor([AWQ_ORDER.index(c) for c in range(8)])

    def cols(x):  # [R, N/8] int32 -> [R, N] codes in column order
        return _nibbles(x)[..., inv].reshape(x.shape[0], -1)
    codes = cols(qweight)
    zeros = cols(qzeros)[:, :N].float()
    return Int4Parts(codes.t().contiguous(), scales.float().t().contiguous(), zeros.t().contiguous(), G)


def pack_nibbles(q: torch.Tensor) -> torch.Tensor:
    """uint8 codes [N, K] -> [N, K/2], the low nibble holding the even column."""
    q = q.to(torch.uint8)
    return (q[:, 0::2] | (q[:, 1::2] << 4)).contiguous()


def _half_to_interleaved(heads: int, dh: int) -> torch.Tensor:
    """Row order that turns a rotate-half head layout into adjacent pairs:
    pair row 2i takes half-layout row i, row 2i+1 takes row dh/2 + i."""
    per = torch.stack([torch.arange(dh // 2), torch.arange(dh // 2) + dh // 2], dim=1).reshape(dh)
    return (torch.arange(heads)[:, None] * dh + per[None, :]).reshape(-1)


def _gate_up_rows(F: int) -> torch.Tensor:
    """Row order of the engine's gate|up weight (blocks of 128 gate rows, then
    128 up rows) over the stacked [gate; up] rows."""
    g = torch.arange(F).reshape(F // 128, 128)
    return torch.stack([g, g + F], dim=1).reshape(-1)


def _cat(parts) -> Int4Parts:
    return Int4Parts(torch.cat([p.q for p in parts]), torch.cat([p.scale for p in parts]),
                     torch.cat([p.zero for p in parts]), parts[0].group)


def llama_parts_to_engine(parts: Dict[str, Int4Parts], cfg) -> Dict[str, Int4Parts]:
    """Hugging Face Llama projection names -> the engine's fused weights."""
    H, KV, Dh, F = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim, cfg.ff_dim
    if F % 128 or cfg.ff_dim_padded != F:
        raise NotImplementedError(f"ff_dim {F} is padded in the engine; import needs a multiple of 128")
    out: Dict[str, Int4Parts] = {}
    for i in range(cfg.num_layers):
        p = f"model.layers.{i}."
        q = parts[p + "self_attn.q_proj"].rows(_half_to_interleaved(H, Dh))
        k = parts[p + "self_attn.k_proj"].rows(_half_to_interleaved(KV, Dh))
        out[f"layers.{i}.wqkv"] = _cat([q, k, parts[p + "self_attn.v_proj"]])
        out[f"layers.{i}.wo"] = parts[p + "self_attn.o_proj"]
        gu = _cat([parts[p + "mlp.gate_proj"], parts[p + "mlp.up_proj"]])
        out[f"layers.{i}.wgu"] = gu.rows(_gate_up_rows(F))
        out[f"layers.{i}.wdown"] = parts[p + "mlp.down_proj"]
    return out


_PLAIN = {"model.embed_tokens.weight": "embed", "model.norm.weight": "final_norm", "lm_head.weight": "lm_head"}


def load_gptq_awq(path: str, cfg, fmt: str = "gptq", device="cuda") -> Dict[str, object]:
    """A GPTQ or AWQ safetensors file of a Llama model -> serving params
    (int4 projections as QuantizedWeight, the rest bf16) under engine names."""
    from safetensors import safe_open

    from ..ops.serving import QuantizedWeight
    if fmt not in ("gptq", "awq"):
        raise ValueError(f"format must be gptq or awq, got {fmt!r}")
    parts: Dict[str, Int4Parts] = {}
    plain: Dict[str, torch.Tensor] = {}
    with safe_open(path, framework="pt") as f:
        names = set(f.keys())
        for name in sorted(n[:-len(".qweight")] for n in names if n.endswith(".qweight")):
            qw, qz, sc = (f.get_tensor(f"{name}.{k}") for k in ("qweight", "qzeros", "scales"))
            if fmt == "gptq":
                gi = f.get_tensor(f"{name}.g_idx") if f"{name}.g_idx" in names else None
                parts[name] = unpack_gptq(qw, qz, sc, gi)
            else:
                parts[name] = unpack_awq(qw, qz, sc)
        for n in names:
            if n in _PLAIN:
                plain[_PLAIN[n]] = f.get_tensor(n)
            elif n.endswith("input_layernorm.weight") or n.endswith("post_attention_layernorm.weight"):
                i = int(n.split(".")[2])
                key = "attn_norm" if "input_layernorm" in n else "ffn_norm"
                plain[f"layers.{i}.{key}"] = f.get_tensor(n)
    out: Dict[str, object] = {}
    for name, p in llama_parts_to_engine(parts, cfg).items():
        N, K = p.shape
        out[name] = QuantizedWeight.from_parts("int4", p.group, N, K, pack_nibbles(p.q).to(device),
                                               p.scale.to(device), p.zero.to(device))
    for name, t in plain.items():
        out[name] = t.to(device=device, dtype=torch.bfloat16)
    if "lm_head" not in out:
        out["lm_head"] = out["embed"]
    return out
