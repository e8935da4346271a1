"""GEMM tile-width tuning for K1.

The tcgen05 GEMM runs 128 x 128 or 128 x 256 output tiles per CTA.  Without a
table the dispatcher takes 256 unless that leaves SMs idle (fewer 128 x 256
tiles than SMs) or N <= 128.  This module times both widths with CUDA events on
the GEMM problems of one training step of a model (forward, dgrad and wgrad of
every linear layer, in the operand layouts the engine uses) and records the
faster one per problem in a JSON table.  ops.gemm consults the table for every
call that does not pin a width when the environment variable LK_GEMM_TUNING
names it (or after ops.gemm.set_tuning), and falls back to the rule otherwise.

    python -m lora_kernel_b200.utils.autotune --preset llama-1.1b-zero3 --out gemm_tuning.json
    LK_GEMM_TUNING=gemm_tuning.json python bench.py

Reference: KernelAutotuner (include/training/training_enhancements.hpp:371-411)
records per-kernel timings and suggests configurations round-robin; here the
sweep is an offline measurement whose table is loaded at start-up.
"""
from __future__ import annotations

import argparse
import json
from dataclasses import dataclass
from typing import Callable, Dict, Iterable, List, Optional

CANDIDATES = (128, 256)
VERSION = 1


@dataclass(frozen=True)
class GemmProblem:
    """out[M, N] = a[M, K] @ b[N, K]^T; a_kmajor / b_kmajor: K is the
    contiguous dimension of that operand (False: a transpose view)."""
    name: str
    M: int
    N: int
    K: int
    epi: str = "bf16"
    a_kmajor: bool = True
    b_kmajor: bool = True

    @property
    def key(self) -> str:
        return problem_key(self.M, self.N, self.K, self.epi, self.a_kmajor, self.b_kmajor)

    @property
    def flops(self) -> float:
        return 2.0 * self.M * self.N * self.K


def problem_key(M: int, N: int, K: int, epi: str, a_kmajor: bool, b_kmajor: bool) -> str:
    return f"{M}x{N}x{K}:{epi}:{'k' if a_kmajor else 'm'}{'k' if b_kmajor else 'm'}"


def tensor_key(a, b, epi: str) -> str:
    """The table key of gemm(a, b, epi=epi) for 2-D tensors a [M, K], b [N, K]."""
    return problem_key(a.shape[0], b.shape[0], a.shape[1], epi, a.stride(1) == 1, b.stride(1) == 1)


class GemmTable:
    """Problem key -> tile width (plus the timings it was chosen from)."""

    def __init__(self, entries: Optional[Dict[str, dict]] = None, device: str = ""):
        self.entries: Dict[str, dict] = dict(entries or {})
        self.device = device

    def __len__(self) -> int:
        return len(self.entries)

    def bn(self, key: str) -> int:
        e = self.entries.get(key)
        return int(e["bn"]) if e else 0

    def lookup(self, a, b, epi: str) -> int:
        """Tuned width for this call, 0 (dispatcher's rule) when untuned."""
        return self.bn(tensor_key(a, b, epi)) if self.entries else 0

    def record(self, problem: GemmProblem, times_ms: Dict[int, float]) -> int:
        best = min(times_ms, key=times_ms.get)
        self.entries[problem.key] = {"bn": int(best), "name": problem.name,
                                     "ms": {str(k): round(v, 5) for k, v in sorted(times_ms.items())}}
        return best

    def to_json(self) -> dict:
        return {"version": VERSION, "device": self.device, "entries": self.entries}

    def save(self, path: str) -> None:
        with open(path, "w") as f:
            json.dump(self.to_json(), f, indent=1, sort_keys=True)

    @classmethod
    def from_json(cls, d: dict) -> "GemmTable":
        if d.get("version") != VERSION:
            raise ValueError(f"GEMM tuning table version {d.get('version')!r}, expected {VERSION}")
        for k, e in d["entries"].items():
            if int(e["bn"]) not in CANDIDATES:
                raise ValueError(f"GEMM tuning table: {k} has tile width {e['bn']} (allowed {CANDIDATES})")
        return cls(d["entries"], d.get("device", ""))

    @classmethod
    def load(cls, path: str) -> "GemmTable":
        with open(path) as f:
            return cls.from_json(json.load(f))


def step_problems(cfg, tokens: int) -> List[GemmProblem]:
    """The K1 GEMMs of one training step of the Llama engine on `tokens`
    tokens (forward, dgrad, wgrad of the four linear layers), deduplicated."""
    D, F = cfg.hidden_dim, cfg.ff_dim
    qkv = (cfg.num_heads + 2 * cfg.num_kv_heads) * cfg.head_dim
    att = cfg.num_heads * cfg.head_dim
    layers = [("wqkv", qkv, D, "bf16"), ("wo", D, att, "bf16_resid"), ("wgu", 2 * F, D, "swiglu"),
              ("wdown", D, F, "bf16_resid")]
    out: Dict[str, GemmProblem] = {}
    for name, n_out, k_in, epi in layers:
        for p in (GemmProblem(f"{name}.fwd", tokens, n_out, k_in, epi),
                  GemmProblem(f"{name}.dgrad", tokens, k_in, n_out, "bf16", True, False),
                  GemmProblem(f"{name}.wgrad", n_out, k_in, tokens, "f32", False, False),
                  GemmProblem(f"{name}.wgrad_acc", n_out, k_in, tokens, "f32_acc", False, False)):
            out.setdefault(p.key, p)
    return list(out.values())


def _device_measure(device: str = "cuda", iters: int = 10) -> Callable[[GemmProblem, int], float]:
    """measure(problem, bn) -> median ms of gemm(..., bn=bn) on the device,
    operands in the problem's layout, L2 flushed before each timed launch."""
    import torch

    from ..ops.gemm import gemm
    from .kernel_bench import time_fn

    cache: Dict[str, tuple] = {}

    def operands(p: GemmProblem):
        t = cache.get(p.key)
        if t is None:
            cache.clear()
            g = torch.Generator(device=device).manual_seed(0)
            a = torch.randn(p.M, p.K, generator=g, device=device).mul_(0.05).to(torch.bfloat16)
            b = torch.randn(p.N, p.K, generator=g, device=device).mul_(0.05).to(torch.bfloat16)
            if not p.a_kmajor:
                a = a.t().contiguous().t()
            if not p.b_kmajor:
                b = b.t().contiguous().t()
            kw = {}
            if p.epi in ("f32", "f32_acc"):
                out = torch.zeros(p.M, p.N, dtype=torch.float32, device=device)
            elif p.epi == "swiglu":
                out = torch.empty(p.M, p.N, dtype=torch.bfloat16, device=device)
                kw["h_out"] = torch.empty(p.M, p.N // 2, dtype=torch.bfloat16, device=device)
            else:
                out = torch.empty(p.M, p.N, dtype=torch.bfloat16, device=device)
                if p.epi == "bf16_resid":
                    kw["residual"] = torch.zeros(p.M, p.N, dtype=torch.bfloat16, device=device)
            t = cache[p.key] = (a, b, out, kw)
        return t

    def measure(p: GemmProblem, bn: int) -> float:
        a, b, out, kw = operands(p)
        return time_fn(lambda: gemm(a, b, out, epi=p.epi, bn=bn, **kw), iters=iters)

    return measure


def tune(problems: Iterable[GemmProblem], measure: Optional[Callable[[GemmProblem, int], float]] = None,
         candidates=CANDIDATES, table: Optional[GemmTable] = None, device: str = "",
         log: Optional[Callable[[str], None]] = None) -> GemmTable:
    """Time every candidate width on every problem; the fastest goes in the table."""
    measure = measure or _device_measure()
    table = table if table is not None else GemmTable(device=device)
    for p in problems:
        times = {bn: float(measure(p, bn)) for bn in candidates}
        best = table.record(p, times)
        if log:
            tf = p.flops / (times[best] * 1e-3) / 1e12
            log(json.dumps({"gemm": p.name, "key": p.key, "bn": best,
                            "ms": {str(k): round(v, 4) for k, v in times.items()}, "tflops": round(tf, 1)}))
    return table


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--preset", default="llama-1.1b-zero3")
    ap.add_argument("--tokens", type=int, default=0, help="GEMM rows (default micro_batch x seq_len)")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--out", default="gemm_tuning.json")
    a = ap.parse_args(argv)
    import torch

    from ..config import get_preset
    rc = get_preset(a.preset)
    tokens = a.tokens or rc.train.micro_batch * rc.train.seq_len
    table = tune(step_problems(rc.model, tokens), _device_measure(iters=a.iters),
                 device=torch.cuda.get_device_name(), log=print)
    table.save(a.out)
    print(json.dumps({"saved": a.out, "problems": len(table)}))


if __name__ == "__main__":
    main()
