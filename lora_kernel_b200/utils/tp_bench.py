"""Tensor-parallel benchmark: the fused collective GEMMs against the NCCL
baseline on one layer's shapes, and a whole TP training step.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \
        --master-port P -m lora_kernel_b200.utils.tp_bench [--ops] [--step] \
        [--preset llama-8b-tp8-fp8] [--layers L] [--micro-batch B] [--seq S] [--accum A]

`--ops` times, per op, the fused peer-memory path and the NCCL path (device
time with CUDA events, max over ranks, L2 flushed before every iteration):
    qkv   all-gather(x) -> x Wqkv_local^T          (K16)
    gu    all-gather(x) -> x Wgu_local^T + SwiGLU   (K16)
    wo    o Wo_local^T -> reduce-scatter + resid + RMSNorm   (K18)
    down  a Wdown_local^T -> reduce-scatter + resid + RMSNorm (K18)
and reports each against its roofline: the slower of FLOPs at the measured
cuBLAS bf16 peak and the bytes that must enter this GPU over NVLink
((N-1)/N of the gathered / reduced tensor) at the measured 770 GB/s per
direction.  `--step` runs TPTrainer steps (bf16) and prints whole-job tokens/s.
One JSON line per result on rank 0.
"""
from __future__ import annotations

import argparse
import json
import os
import time

import torch
import torch.distributed as dist

NVLINK_GBS = 770.0  # measured peer copy bandwidth per direction (GB/s)


def _peaks():
    here = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    try:
        with open(os.path.join(here, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["bf16_tflops"]), "measured"
    except (OSError, KeyError, ValueError):
        return 1590.0, "fallback"


def _max_over_ranks(x: float) -> float:
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


_ALIGN = {}


def _align() -> None:
    """Device-side rendezvous of all ranks on the current stream, so that a
    timed region starts at the same moment everywhere (host skew between
    ranks is not charged to the op)."""
    t = _ALIGN.get("t")
    if t is None:
        t = _ALIGN["t"] = torch.zeros(1, device="cuda")
    dist.all_reduce(t)


def _time(fn, iters: int, warmup: int, flush: torch.Tensor) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    tot = 0.0
    for _ in range(iters):
        flush.zero_()
        _align()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        tot += s.elapsed_time(e)
    return _max_over_ranks(tot / iters)


def bench_diag(cfg, B, S, iters, rank0):
    """Pieces of the fused ops timed separately (qkv / wo shapes)."""
    from .._ext import C, status
    from ..ops import gemm as G
    from ..parallel import tp as TP
    dev = torch.device("cuda", torch.cuda.current_device())
    W, r = dist.get_world_size(), dist.get_rank()
    T = B * S
    R, D = T // W, cfg.hidden_dim
    ql, kvl = cfg.q_dim // W, cfg.kv_dim // W
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    bf = dict(dtype=torch.bfloat16, device=dev)
    w = torch.randn(ql + 2 * kvl, D, device=dev).bfloat16() * 0.02
    wo = torch.randn(D, ql, device=dev).bfloat16() * 0.02
    xfull = torch.randn(T, D, device=dev).bfloat16()
    o = torch.randn(T, ql, device=dev).bfloat16()
    out = torch.empty(T, ql + 2 * kvl, **bf)
    full_o = torch.empty(T, D, **bf)
    c = TP.TPComm(cfg, T, dev, comm="p2p")
    c.stage_view(0, R, D).copy_(xfull[:R])
    res = {}
    res["gemm_qkv_local"] = _time(lambda: G.gemm(xfull, w, out), iters, 3, flush)
    res["barrier"] = _time(c.barrier, iters, 3, flush)
    res["ag_gemm_qkv"] = _time(lambda: c.ag_gemm(0, xfull, w, out), iters, 3, flush)
    res["allgather_copy_kernel"] = _time(
        lambda: c.pc.allgather_copy(c.stage[0], 0, R * D, xfull), iters, 3, flush)
    res["nccl_allgather"] = _time(
        lambda: dist.all_gather_into_tensor(xfull, c.stage_view(0, R, D)), iters, 3, flush)
    res["gemm_wo_local"] = _time(lambda: G.gemm(o, wo, full_o), iters, 3, flush)
    res["gemm_rs_wo"] = _time(lambda: c.gemm_rs(0, o, wo), iters, 3, flush)
    hout = torch.empty(R, D, **bf)
    res["rs_sum_plain"] = _time(lambda: C().rs_sum(c.recv_view(0, R, D), W, hout, None, None, None, None, 1e-5, 0, None, 0),
                                iters, 3, flush)
    res["nccl_reduce_scatter"] = _time(
        lambda: dist.reduce_scatter_tensor(hout, full_o), iters, 3, flush)
    if rank0:
        print(json.dumps({"diag": {k: round(v, 4) for k, v in res.items()}, "shape": f"T={T} D={D} tp={W}"}),
              flush=True)


def bench_ops(cfg, B, S, iters, warmup, rank0):
    from ..parallel import tp as TP
    dev = torch.device("cuda", torch.cuda.current_device())
    W, r = dist.get_world_size(), dist.get_rank()
    T = B * S
    R, D = T // W, cfg.hidden_dim
    ql, kvl, Fl = cfg.q_dim // W, cfg.kv_dim // W, cfg.ff_dim_padded // W
    peak, src = _peaks()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    g = torch.Generator(device=dev).manual_seed(r)
    bf = dict(dtype=torch.bfloat16, device=dev)

    def rnd(*shape, s=0.02):
        return (torch.randn(*shape, device=dev, generator=g) * s).to(torch.bfloat16)

    w = {"qkv": rnd(ql + 2 * kvl, D), "gu": rnd(2 * Fl, D), "wo": rnd(D, ql), "down": rnd(D, Fl)}
    a = {"wo": rnd(T, ql, s=1.0), "down": rnd(T, Fl, s=1.0)}
    gamma = torch.ones(D, **bf)
    resid = rnd(R, D, s=1.0)
    xfull = torch.empty(T, D, **bf)
    out = {"qkv": torch.empty(T, ql + 2 * kvl, **bf), "gu": torch.empty(T, 2 * Fl, **bf)}
    act = torch.empty(T, Fl, **bf)
    hout = torch.empty(R, D, **bf)
    rstd = torch.empty(R, dtype=torch.float32, device=dev)
    results = []
    for mode in ("p2p", "nccl"):
        c = TP.TPComm(cfg, T, dev, comm=mode)
        c.stage_view(0, R, D).copy_(rnd(R, D, s=1.0))

        def qkv():
            c.barrier()
            c.ag_gemm(0, xfull, w["qkv"], out["qkv"])

        def gu():
            c.barrier()
            c.ag_gemm(0, xfull, w["gu"], out["gu"], epi="swiglu", h_out=act)

        def wo():
            c.gemm_rs(0, a["wo"], w["wo"])
            c.rs_sum(0, hout, resid=resid, gamma=gamma, y=c.stage_view(1, R, D), rstd=rstd)

        def down():
            c.gemm_rs(1, a["down"], w["down"])
            c.rs_sum(1, hout, resid=resid, gamma=gamma, y=c.stage_view(1, R, D), rstd=rstd)

        for name, fn, N, K, nv in (("qkv", qkv, ql + 2 * kvl, D, T * D * 2),
                                   ("gu", gu, 2 * Fl, D, T * D * 2),
                                   ("wo", wo, D, ql, T * D * 2),
                                   ("down", down, D, Fl, T * D * 2)):
            ms = _time(fn, iters, warmup, flush)
            flops = 2.0 * T * N * K
            link = nv * (W - 1) / W
            roof_ms = max(flops / (peak * 1e12), link / (NVLINK_GBS * 1e9)) * 1e3
            results.append({"op": name, "comm": mode, "ms": round(ms, 4), "tflops": round(flops / ms / 1e9, 1),
                            "nvlink_gb": round(link / 1e9, 4), "roofline_ms": round(roof_ms, 4),
                            "frac_of_roofline": round(roof_ms / ms, 3), "peak_src": src,
                            "shape": f"T={T} N={N} K={K} tp={W}"})
        torch.cuda.synchronize()
        dist.barrier()
        del c
    if rank0:
        for x in results:
            print(json.dumps(x), flush=True)
    return results


def bench_ops_mx(cfg, B, S, iters, warmup, rank0):
    """The MX fp8 forms of the four fused ops as the MX TP step runs them
    (quantise own rows -> device barrier -> gathered block-scaled GEMM; quantise
    -> block-scaled GEMM storing into the owners' slots -> owner sum), forward
    (e4m3 x e4m3) and data gradient (e5m2 x e4m3, the gathered gradient
    dequantised for the weight gradient), against the bf16 fused ops."""
    from .._ext import C
    from ..ops import elementwise as E
    from ..ops.fp8 import MXWeight
    from ..parallel import tp as TP
    dev = torch.device("cuda", torch.cuda.current_device())
    W, r = dist.get_world_size(), dist.get_rank()
    T = B * S
    R, D = T // W, cfg.hidden_dim
    ql, kvl, Fl = cfg.q_dim // W, cfg.kv_dim // W, cfg.ff_dim_padded // W
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    g = torch.Generator(device=dev).manual_seed(r)
    bf = dict(dtype=torch.bfloat16, device=dev)

    def rnd(*shape, s=0.02):
        return (torch.randn(*shape, device=dev, generator=g) * s).to(torch.bfloat16)

    w = {"qkv": rnd(ql + 2 * kvl, D), "gu": rnd(2 * Fl, D), "wo": rnd(D, ql), "down": rnd(D, Fl)}
    w8 = {k: MXWeight(v, transpose=True) for k, v in w.items()}
    a = {"wo": rnd(T, ql, s=1.0), "down": rnd(T, Fl, s=1.0)}
    gamma = torch.ones(D, **bf)
    resid = rnd(R, D, s=1.0)
    out = {"qkv": torch.empty(T, ql + 2 * kvl, **bf), "gu": torch.empty(T, 2 * Fl, **bf)}
    act = torch.empty(T, Fl, **bf)
    hout = torch.empty(R, D, **bf)
    rstd = torch.empty(R, dtype=torch.float32, device=dev)
    x8 = torch.empty(T, D, dtype=torch.uint8, device=dev)
    from ..ops.fp8 import sf_tile_bytes
    xs = torch.empty(sf_tile_bytes(T, D), dtype=torch.uint8, device=dev)
    dfull = torch.empty(T, D, **bf)
    c = TP.TPComm(cfg, T, dev, comm="p2p")
    rows = rnd(R, D, s=1.0)
    c.stage_view(0, R, D).copy_(rows)
    c.stage_view(1, R, D).copy_(rows)

    def fwd_col(name, k):
        def f():
            c.publish_mx(k, c.stage_view(k, R, D))
            c.barrier()
            c.ag_gemm_mx(k, x8, xs, w8[name].q, w8[name].sf, out[name])
            if name == "gu":
                E.swiglu_fwd(out["gu"], act)
        return f

    def fwd_row(name, k):
        def f():
            c.gemm_rs_mx(k, a[name], w8[name].q, w8[name].sf)
            c.rs_sum(k, hout, resid=resid, gamma=gamma, y=c.stage_view(1 - k, R, D), rstd=rstd)
        return f

    dx = {"wo": torch.empty(T, ql, **bf), "down": torch.empty(T, Fl, **bf)}
    dy = {"qkv": rnd(T, ql + 2 * kvl, s=1.0), "gu": rnd(T, 2 * Fl, s=1.0)}

    def bwd_ag(name, k):
        # row-parallel layer: dX = gathered dY (e5m2) . W, dY dequantised for dW
        def f():
            c.publish_mx(k, c.stage_view(k, R, D), fmt=1)
            c.barrier()
            c.ag_gemm_mx(k, x8, xs, w8[name].qt, w8[name].sft, dx[name], a_fmt=1)
            C().dequant_mx_rows(x8, 1, xs, dfull)
        return f

    def bwd_rs(name, k):
        # column-parallel layer: partial dY . W reduce-scattered, summed by the owner
        def f():
            c.gemm_rs_mx(k, dy[name], w8[name].qt, w8[name].sft, a_fmt=1)
            c.rs_sum(k, hout, resid=resid, gamma=None, y=None, rstd=None)
        return f

    res = {}
    for name, fn in (("fwd.qkv", fwd_col("qkv", 0)), ("fwd.gu", fwd_col("gu", 1)),
                     ("fwd.wo", fwd_row("wo", 0)), ("fwd.down", fwd_row("down", 1)),
                     ("bwd.wo", bwd_ag("wo", 0)), ("bwd.down", bwd_ag("down", 1)),
                     ("bwd.qkv", bwd_rs("qkv", 0)), ("bwd.gu", bwd_rs("gu", 1))):
        res[name] = round(_time(fn, iters, warmup, flush), 4)
    torch.cuda.synchronize()
    dist.barrier()
    del c
    if rank0:
        print(json.dumps({"mx_ops_ms": res, "shape": f"T={T} D={D} tp={W}"}), flush=True)
    return res


def bench_step(cfg, tc, B, S, accum, steps, warmup, comm, rank0, fp8=False):
    from ..parallel.tp import TPTrainer
    tr = TPTrainer(cfg, tc, micro_batch=B, seq_len=S, comm=comm, seed=tc.seed, fp8=fp8)
    g = torch.Generator().manual_seed(0)
    tok = torch.randint(0, cfg.vocab_size, (accum, B, S + 1), generator=g).cuda()
    batches = [(tok[i, :, :-1].contiguous(), tok[i, :, 1:].contiguous()) for i in range(accum)]
    for _ in range(warmup):
        tr.train_step(batches)
    torch.cuda.synchronize()
    tr.check()
    dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        acc = tr.train_step(batches)
    e.record()
    torch.cuda.synchronize()
    ms = _max_over_ranks(s.elapsed_time(e) / steps)
    tr.check()
    loss = (acc[0] / acc[1]).item()
    tokens = accum * B * S  # the TP group shares one batch
    res = {"metric": "train tokens/sec", "value": round(tokens / ms * 1e3, 1), "unit": "tokens/s",
           "ms_per_step": round(ms, 2), "comm": comm + (f"+fp8-{tr.model.fp8}" if fp8 else ""),
           "n_gpus": dist.get_world_size(),
           "config": {"model": f"Llama-style {cfg.num_layers} layers d{cfg.hidden_dim}",
                      "global_batch": accum * B, "seq_len": S, "parallelism": f"tp{dist.get_world_size()}",
                      "micro_batch": B, "accum": accum},
           "dtype": ("fp8 projections: e4m3 forward, e5m2 data gradients, power-of-two 1x128 / 128x128 scales "
                     "applied by the tensor core (MX); bf16 weight gradients, attention and LM head"
                     if tr.model.mx else
                     "fp8 e4m3 forward projections (1x128 / 128x128 fp32 scales), bf16 rest") if fp8 else "bf16",
           "loss": round(loss, 4), "nvls": bool(tr.comm.pc.nvls)}
    if rank0:
        print(json.dumps(res), flush=True)
    del tr
    return res


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--preset", default="llama-8b-tp8-fp8")
    ap.add_argument("--layers", type=int, default=0)
    ap.add_argument("--micro-batch", type=int, default=2)
    ap.add_argument("--seq", type=int, default=4096)
    ap.add_argument("--accum", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--ops", action="store_true")
    ap.add_argument("--step", action="store_true")
    ap.add_argument("--comm", default="p2p,nccl")
    ap.add_argument("--diag", action="store_true")
    ap.add_argument("--fp8", default="", help="also run the block-scaled fp8 TP step (p2p): "
                    "comma list of recipes, mx (tensor-core scales) and/or exact (fp32 scales)")
    a = ap.parse_args(argv)
    from ..config import get_preset
    from ..parallel.comm import init_distributed
    rank, world, local = init_distributed("nccl", timeout_s=300)
    rc = get_preset(a.preset)
    cfg = rc.model
    if a.layers:
        cfg.num_layers = a.layers
    tc = rc.train
    tc.dynamic_loss_scale = False
    if a.diag:
        bench_diag(cfg, a.micro_batch, a.seq, a.iters, rank == 0)
    if a.ops:
        bench_ops(cfg, a.micro_batch, a.seq, a.iters, 3, rank == 0)
        if "mx" in a.fp8.split(","):
            bench_ops_mx(cfg, a.micro_batch, a.seq, a.iters, 3, rank == 0)
    if a.step:
        for comm in a.comm.split(","):
            bench_step(cfg, tc, a.micro_batch, a.seq, a.accum, a.steps, a.warmup, comm, rank == 0)
        for recipe in [r for r in a.fp8.split(",") if r]:
            bench_step(cfg, tc, a.micro_batch, a.seq, a.accum, a.steps, a.warmup, "p2p", rank == 0, fp8=recipe)
    torch.cuda.synchronize()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
