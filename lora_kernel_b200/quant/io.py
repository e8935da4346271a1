"""Quantised-weight checkpoints (safetensors).

Layout, per quantised linear `name` (engine orientation [out, in]):
    {name}.qweight   int4: uint8 [N, K/2] (two nibbles per byte); int8: int8 [N, K]; fp8: uint8 e4m3 bits [N, K]
    {name}.scales    fp32 [N, K/group] (int4) or [N] (int8 / fp8)
    {name}.zeros     fp32 [N, K/group] (int4 only)
and every other tensor (embedding, norms, LM head) as bf16 under its own name.
The header metadata records each quantised tensor's format, group size and
shape ("{name}.quant" = "fmt,group,N,K").  `load_quantized` returns a dict the
serving ModelRunner accepts as `params` (quantised entries are used as they
are, the rest are copied).

Reference: QuantizedModelLoader::load_awq / load_gptq
(include/api/serving_production.hpp:231-241), a stub there; this loader reads what our own
quantiser writes, and quant/gptq_awq.py imports GPTQ / AWQ checkpoints.
"""
from __future__ import annotations

from typing import Dict, Union

import torch

from ..ops.serving import QuantizedWeight


def save_quantized(weights: Dict[str, Union[QuantizedWeight, torch.Tensor]], path: str) -> None:
    from safetensors.torch import save_file
    tensors: Dict[str, torch.Tensor] = {}
    meta: Dict[str, str] = {"format": "lora_kernel_b200-quantized"}
    seen = set()
    for name, w in weights.items():
        if isinstance(w, QuantizedWeight):
            tensors[f"{name}.qweight"] = w.q.contiguous().cpu()
            tensors[f"{name}.scales"] = w.scale.contiguous().cpu()
            if w.zero is not None:
                tensors[f"{name}.zeros"] = w.zero.contiguous().cpu()
            meta[f"{name}.quant"] = f"{w.fmt},{w.group},{w.N},{w.K}"
        else:
            if w.data_ptr() in seen:  # tied tensors are stored once
                continue
            seen.add(w.data_ptr())
            tensors[name] = w.detach().contiguous().cpu()
    save_file(tensors, path, metadata=meta)


def load_quantized(path: str, device="cuda") -> Dict[str, Union[QuantizedWeight, torch.Tensor]]:
    from safetensors import safe_open
    out: Dict[str, Union[QuantizedWeight, torch.Tensor]] = {}
    with safe_open(path, framework="pt") as f:
        meta = f.metadata() or {}
        names = set(f.keys())
        quant = {k[:-len(".quant")]: v for k, v in meta.items() if k.endswith(".quant")}
        for name, spec in quant.items():
            fmt, group, N, K = spec.split(",")
            q = f.get_tensor(f"{name}.qweight").to(device)
            s = f.get_tensor(f"{name}.scales").to(device)
            z = f.get_tensor(f"{name}.zeros").to(device) if f"{name}.zeros" in names else None
            out[name] = QuantizedWeight.from_parts(fmt, int(group), int(N), int(K), q, s, z)
            names -= {f"{name}.qweight", f"{name}.scales", f"{name}.zeros"}
        for name in names:
            out[name] = f.get_tensor(name).to(device)
    if "lm_head" not in out and "embed" in out:
        out["lm_head"] = out["embed"]
    return out
