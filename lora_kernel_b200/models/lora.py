"""LoRA adapters for the Llama engine (K20).

For a frozen linear y = x W^T (W [out, in]) an adapter adds
    y += s * (x A^T) B^T,   A [r, in], B [out, r], s = alpha / r.
On the B200 path the update is fused into the base GEMM's main loop: the
kernel contracts the concatenated dimension [x | s*u] . [W | B]^T with
u = x A^T, i.e. a second K segment of width r accumulated into the same TMEM
tile (and under the same SwiGLU / residual epilogue).  Backward:
    v  = dy B                       [T, r]
    dx = dy W + (s v) A             (the same two-segment GEMM, dgrad form)
    dA = (s v)^T x,  dB = dy^T (s u)
Merging (W += s B A) and unmerging are one GEMM each with the residual
epilogue.

Initialisation follows the reference (include/nn/lora.hpp:69-76): A is normal
with std sqrt(2 / in), B is zero, so a fresh adapter leaves the model
unchanged.  The reference applies no alpha/r scaling (alpha = r reproduces
that) and never propagates dX; both are handled here.  For the fused gate|up
projection, B's rows follow the same blocked gate/up interleave as Wgu.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, Iterable, List, Optional, Tuple

import torch

from ..config import TransformerConfig

ALIGN = 64


@dataclass
class LoRAConfig:
    rank: int = 16
    alpha: float = 16.0
    targets: Tuple[str, ...] = ("wqkv", "wo", "wgu", "wdown")
    init_seed: int = 0

    @property
    def scale(self) -> float:
        return self.alpha / self.rank


def _shapes(cfg: TransformerConfig, target: str) -> Tuple[int, int]:
    """(out, in) of a target linear in the engine's internal layout."""
    D, F = cfg.hidden_dim, cfg.ff_dim_padded
    return {"wqkv": (cfg.qkv_dim, D), "wo": (D, cfg.q_dim), "wgu": (2 * F, D), "wdown": (D, F)}[target]


class LoRAAdapters:
    def __init__(self, cfg: TransformerConfig, lc: LoRAConfig, device="cuda", dtype=torch.bfloat16):
        if lc.rank % 8 != 0:
            raise ValueError("LoRA rank must be a multiple of 8 (16-byte rows for TMA)")
        self.cfg, self.lc = cfg, lc
        self.device = torch.device(device)
        self.specs: List[Tuple[str, Tuple[int, int], int]] = []
        off = 0
        for i in range(cfg.num_layers):
            for t in lc.targets:
                out, inn = _shapes(cfg, t)
                for nm, shape in ((f"layers.{i}.{t}.A", (lc.rank, inn)), (f"layers.{i}.{t}.B", (out, lc.rank))):
                    self.specs.append((nm, shape, off))
                    off += (shape[0] * shape[1] + ALIGN - 1) // ALIGN * ALIGN
        self.numel = off
        self.flat = torch.zeros(off, dtype=dtype, device=self.device)
        self.grads = torch.zeros(off, dtype=torch.float32, device=self.device)
        self.views: Dict[str, torch.Tensor] = {}
        self.gviews: Dict[str, torch.Tensor] = {}
        for nm, shape, o in self.specs:
            n = shape[0] * shape[1]
            self.views[nm] = self.flat[o:o + n].view(shape)
            self.gviews[nm] = self.grads[o:o + n].view(shape)
        self.reset_parameters()

    def reset_parameters(self) -> None:
        for k, (nm, shape, _) in enumerate(self.specs):
            v = self.views[nm]
            if nm.endswith(".A"):
                g = torch.Generator(device=self.device).manual_seed(self.lc.init_seed * 1000003 + k)
                t = torch.empty(shape, dtype=torch.float32, device=self.device)
                t.normal_(0.0, (2.0 / shape[1]) ** 0.5, generator=g)
                v.copy_(t)
            else:
                v.zero_()

    def has(self, layer: int, target: str) -> bool:
        return target in self.lc.targets

    def A(self, i: int, t: str) -> torch.Tensor:
        return self.views[f"layers.{i}.{t}.A"]

    def B(self, i: int, t: str) -> torch.Tensor:
        return self.views[f"layers.{i}.{t}.B"]

    def gA(self, i: int, t: str) -> torch.Tensor:
        return self.gviews[f"layers.{i}.{t}.A"]

    def gB(self, i: int, t: str) -> torch.Tensor:
        return self.gviews[f"layers.{i}.{t}.B"]

    def segments(self):
        return [(o, shape[0] * shape[1], False) for _, shape, o in self.specs]

    def num_parameters(self) -> int:
        return sum(s[0] * s[1] for _, s, _ in self.specs)

    def state_dict(self) -> Dict[str, torch.Tensor]:
        return dict(self.views)

    def load_state_dict(self, sd: Dict[str, torch.Tensor]) -> None:
        with torch.no_grad():
            for k, v in sd.items():
                self.views[k].copy_(v)

    # ---------------------------------------------------------------- merging
    @torch.no_grad()
    def merge_into(self, params, sign: float = 1.0) -> None:
        """W <- W + sign * s * B A for every adapted linear (one GEMM each, in
        place through the residual epilogue)."""
        from ..ops.gemm import gemm
        s = sign * self.lc.scale
        for i in range(self.cfg.num_layers):
            for t in self.lc.targets:
                W = params[f"layers.{i}.{t}"]
                # the residual epilogue takes K-major operands: A^T ([in, r], tiny) made contiguous
                gemm(self.B(i, t), self.A(i, t).t().contiguous(), W, epi="bf16_resid", residual=W, alpha=s)

    def unmerge_from(self, params) -> None:
        self.merge_into(params, sign=-1.0)


def save_lora_file(adapters: "LoRAAdapters", path: str, step: int = 0) -> None:
    """The adapter tensors (fp32) with rank / alpha / targets in the metadata."""
    from safetensors.torch import save_file
    lc = adapters.lc
    save_file({k: v.detach().float().contiguous().cpu() for k, v in adapters.state_dict().items()}, path,
              metadata={"rank": str(lc.rank), "alpha": str(lc.alpha), "targets": ",".join(lc.targets),
                        "step": str(step)})


def load_lora_file(path: str, cfg: TransformerConfig, device="cuda") -> "LoRAAdapters":
    """Adapters saved by the trainer (lora_step_N.safetensors: the adapter
    tensors with rank / alpha / targets in the metadata)."""
    from safetensors import safe_open
    with safe_open(path, framework="pt") as f:
        meta = f.metadata() or {}
        tensors = {k: f.get_tensor(k) for k in f.keys()}
    lc = LoRAConfig(rank=int(meta["rank"]), alpha=float(meta["alpha"]),
                    targets=tuple(t for t in meta.get("targets", "wqkv,wo,wgu,wdown").split(",") if t))
    ad = LoRAAdapters(cfg, lc, device)
    ad.load_state_dict({k: v.to(device) for k, v in tensors.items()})
    return ad


@torch.no_grad()
def merge_lora_state_dict(sd: Dict[str, torch.Tensor], adapters: "LoRAAdapters") -> Dict[str, torch.Tensor]:
    """A reference-named state dict with the adapters folded in (W + (alpha/r) B A,
    fp32 on the host): the weights the merged model serves or exports."""
    from .params import FlatParams
    p = FlatParams(adapters.cfg, "cpu", torch.float32)
    p.load_reference_state_dict({k: v.float().cpu() for k, v in sd.items()})
    s = adapters.lc.scale
    for i in range(adapters.cfg.num_layers):
        for t in adapters.lc.targets:
            w = p.views[f"layers.{i}.{t}"]
            w += s * (adapters.B(i, t).float().cpu() @ adapters.A(i, t).float().cpu())
    return p.to_reference_state_dict()

