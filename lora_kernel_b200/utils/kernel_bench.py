"""Kernel micro-benchmarks: device-timed (CUDA events) throughput of the
sm_100a kernels next to the library equivalent (cuBLAS via torch.matmul),
reported against the measured peaks of this machine when they are available.

    python -m lora_kernel_b200.utils.kernel_bench [--only gemm,norm,...]

Each case runs warm-up iterations, then times `iters` launches between two
events with an L2 flush (a 256 MiB write, larger than the 126 MB L2) before
each timed launch, and prints one JSON line per case.
"""
from __future__ import annotations

import argparse
import json
import os

import torch

_flush = None


def _l2_flush():
    global _flush
    if _flush is None:
        _flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    _flush.zero_()


def time_fn(fn, iters: int = 10, warmup: int = 3, flush: bool = True) -> float:
    """Median milliseconds per call (CUDA events on the current stream)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        if flush:
            _l2_flush()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e))
    times.sort()
    return times[len(times) // 2]


def peaks():
    p = os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "src": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "src": "fallback"}


def bench_gemm(shapes, iters):
    from lora_kernel_b200.ops.gemm import gemm
    pk = peaks()
    for (M, N, K, layout) in shapes:
        a = torch.randn(M, K, device="cuda").to(torch.bfloat16)
        if layout == "tn":
            b = torch.randn(N, K, device="cuda").to(torch.bfloat16)
            A, B = a, b
        elif layout == "dgrad":
            b = torch.randn(K, N, device="cuda").to(torch.bfloat16)
            A, B = a, b.t()
        else:  # wgrad: A = X1^T (MN-major), B = X2^T
            a = torch.randn(K, M, device="cuda").to(torch.bfloat16)
            b = torch.randn(K, N, device="cuda").to(torch.bfloat16)
            A, B = a.t(), b.t()
        out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
        t_lk = time_fn(lambda: gemm(A, B, out), iters)
        t_cb = time_fn(lambda: torch.matmul(A, B.t(), out=out), iters)
        fl = 2.0 * M * N * K
        print(json.dumps({"kernel": "gemm_tc", "M": M, "N": N, "K": K, "layout": layout,
                          "ms": round(t_lk, 4), "tflops": round(fl / t_lk / 1e9, 1),
                          "cublas_ms": round(t_cb, 4), "cublas_tflops": round(fl / t_cb / 1e9, 1),
                          "frac_of_peak": round(fl / t_lk / 1e9 / pk["bf16_tflops"], 3),
                          "peak_src": pk["src"]}), flush=True)


def bench_fp8(shapes, iters):
    """K2 block-scaled fp8 GEMM (quantised operands prepared outside the timed
    region) against the bf16 tcgen05 GEMM and cuBLAS bf16 on the same shape."""
    from lora_kernel_b200.ops import fp8 as F
    from lora_kernel_b200.ops.gemm import gemm
    pk = peaks()
    for (M, N, K) in shapes:
        x = torch.randn(M, K, device="cuda").to(torch.bfloat16)
        w = (torch.randn(N, K, device="cuda") * 0.02).to(torch.bfloat16)
        w8 = F.Fp8Weight(w, transpose=False)
        q, s = F.quantize_1x128(x)
        out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
        t8 = time_fn(lambda: F.gemm_fp8(q, s, w8.q, w8.scale, out=out), iters)
        tq = time_fn(lambda: F.quantize_1x128(x), iters)
        tb = time_fn(lambda: gemm(x, w, out), iters)
        tc = time_fn(lambda: torch.matmul(x, w.t(), out=out), iters)
        fl = 2.0 * M * N * K
        print(json.dumps({"kernel": "gemm_fp8_blockscaled", "M": M, "N": N, "K": K,
                          "ms": round(t8, 4), "tflops": round(fl / t8 / 1e9, 1),
                          "act_quant_ms": round(tq, 4),
                          "bf16_tc_ms": round(tb, 4), "cublas_bf16_ms": round(tc, 4),
                          "speedup_vs_bf16_tc": round(tb / t8, 3),
                          "frac_of_bf16_peak": round(fl / t8 / 1e9 / pk["bf16_tflops"], 3),
                          "peak_src": pk["src"]}), flush=True)


def bench_mxf8(shapes, iters):
    """K2 in MX form (tcgen05 block-scaled fp8, power-of-two scales) against the
    bf16 tcgen05 GEMM and cuBLAS bf16 on the same shape; quantisation outside the
    timed region (timed on its own as act_quant_ms)."""
    from lora_kernel_b200.ops import fp8 as F
    from lora_kernel_b200.ops.gemm import gemm
    pk = peaks()
    for (M, N, K) in shapes:
        x = torch.randn(M, K, device="cuda").to(torch.bfloat16)
        w = (torch.randn(N, K, device="cuda") * 0.02).to(torch.bfloat16)
        w8 = F.MXWeight(w, transpose=False)
        q, sf = F.quantize_mx(x)
        out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
        t8 = time_fn(lambda: F.gemm_mxf8(q, sf, w8.q, w8.sf, out=out), iters)
        tq = time_fn(lambda: F.quantize_mx(x), iters)
        tb = time_fn(lambda: gemm(x, w, out), iters)
        tc = time_fn(lambda: torch.matmul(x, w.t(), out=out), iters)
        fl = 2.0 * M * N * K
        print(json.dumps({"kernel": "gemm_mxf8", "M": M, "N": N, "K": K,
                          "ms": round(t8, 4), "tflops": round(fl / t8 / 1e9, 1),
                          "act_quant_ms": round(tq, 4),
                          "bf16_tc_ms": round(tb, 4), "cublas_bf16_ms": round(tc, 4),
                          "speedup_vs_bf16_tc": round(tb / t8, 3),
                          "speedup_vs_cublas_bf16": round(tc / t8, 3),
                          "frac_of_bf16_peak": round(fl / t8 / 1e9 / pk["bf16_tflops"], 3),
                          "peak_src": pk["src"]}), flush=True)


def graph_time(calls, reps: int = 10) -> float:
    """Median device milliseconds per call when `calls` (closures) replay back to
    back from one CUDA graph: launch overhead is off the clock, as in the serving
    engine's captured decode step.  Callers rotate the operands across enough
    copies that one pass over them exceeds L2."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for c in calls:  # first use allocates workspaces outside the capture
            c()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for c in calls:
            c()
    g.replay()
    torch.cuda.synchronize()
    times = []
    for _ in range(reps):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        g.replay()
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e) / len(calls))
    times.sort()
    del g
    return times[len(times) // 2]


def bench_decode(iters):
    """Serving kernels of the Llama 8B shape (TP=8 shard and the whole model on one
    GPU): the int4 group-128 dequant GEMM (K14 decode) and the paged decode
    attention over an fp8 KV cache (K13), as fractions of the measured HBM copy
    bandwidth (bytes: the int4 weights + scales once; the KV pages each sequence
    reads).  Timed as CUDA-graph replays over rotating weight copies / KV block
    sets (about 400 MB per pass, so L2 holds none of it)."""
    from lora_kernel_b200.ops import serving as SV
    pk = peaks()
    from lora_kernel_b200._ext import C
    for (N, K, tag) in [(6144, 4096, "qkv_tp1"), (28672, 4096, "gate_up_tp1"),
                        (4096, 14336, "down_tp1"), (3584, 4096, "gate_up_tp8"), (4096, 1792, "down_tp8")]:
        w = (torch.randn(N, K, device="cuda") * 0.02).to(torch.bfloat16)
        q0 = SV.QuantizedWeight(w, "int4", 128)
        copies = max(2, min(48, -(-400 * 2 ** 20 // q0.nbytes())))
        qws = [q0] + [SV.QuantizedWeight.from_parts("int4", 128, N, K, q0.q.clone(), q0.scale.clone(),
                                                     q0.zero.clone()) for _ in range(copies - 1)]
        del w
        for M in (1, 8, 16, 64, 128, 256):
            x = torch.randn(M, K, device="cuda").to(torch.bfloat16)
            out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
            t = graph_time([(lambda qw=qw: qw.matmul_t(x, out=out)) for qw in qws], iters)
            by = q0.nbytes() + M * K * 2 + M * N * 2
            rec = {"kernel": "int4_dq_gemm", "shape": tag, "M": M, "N": N, "K": K, "ms": round(t, 4),
                   "splits": C().dq_gemm_splits(M, N, K), "gbs": round(by / t / 1e6, 1),
                   "frac_of_hbm": round(by / t / 1e6 / pk["hbm_gbs"], 3), "timing": "cuda graph"}
            if M <= 16:  # the CUDA-core GEMV it replaces
                tg = graph_time([(lambda qw=qw: C().dequant_gemv(SV.QFMT["int4"], x, qw.q, qw.scale, qw.zero, N, K,
                                                                 128, out)) for qw in qws], iters)
                rec["cuda_core_gemv_ms"] = round(tg, 4)
            print(json.dumps(rec), flush=True)
        del qws, q0
        torch.cuda.empty_cache()
    # paged decode attention: Llama 8B, 32 q / 8 kv heads (TP=8: 4 / 1), head_dim 128, fp8 pages of 16
    for (nseq, ctx, Hq, Hkv) in [(256, 2048, 4, 1), (64, 2048, 32, 8), (256, 1024, 32, 8)]:
        Dh, bs = 128, 16
        per = nseq * ((ctx + bs - 1) // bs)  # blocks one call reads
        pass_bytes = per * bs * Hkv * (2 * Dh + 8)
        sets = max(2, min(16, -(-400 * 2 ** 20 // pass_bytes)))
        nblk = sets * per
        kc = torch.randn(nblk * bs, Hkv, Dh, device="cuda").to(torch.float8_e4m3fn)
        vc = torch.randn(nblk * bs, Hkv, Dh, device="cuda").to(torch.float8_e4m3fn)
        ks = torch.full((nblk * bs, Hkv), 0.01, device="cuda")
        vs = torch.full((nblk * bs, Hkv), 0.01, device="cuda")
        perm = torch.randperm(nblk, device="cuda", dtype=torch.int32)
        bts = [perm[i * per:(i + 1) * per].view(nseq, -1).contiguous() for i in range(sets)]
        lens = torch.full((nseq,), ctx, dtype=torch.int32, device="cuda")
        q = torch.randn(nseq, Hq * Dh, device="cuda").to(torch.bfloat16)
        out = torch.empty_like(q)
        t = graph_time([(lambda bt=bt: SV.decode_attention(q, kc, vc, ks, vs, bt, lens, bs, Hq, Hkv, Dh,
                                                           kv_dtype="fp8", max_ctx=ctx, out=out)) for bt in bts],
                       iters)
        by = nseq * ctx * Hkv * (2 * Dh + 8) + 2 * q.numel() * 2
        print(json.dumps({"kernel": "decode_attention_fp8", "seqs": nseq, "ctx": ctx, "Hq": Hq, "Hkv": Hkv,
                          "Dh": Dh, "ms": round(t, 4), "gbs": round(by / t / 1e6, 1),
                          "frac_of_hbm": round(by / t / 1e6 / pk["hbm_gbs"], 3), "timing": "cuda graph"}),
              flush=True)
        del kc, vc, ks, vs
        torch.cuda.empty_cache()


def bench_norm(iters):
    from lora_kernel_b200.ops.norm import rmsnorm_bwd, rmsnorm_fwd
    pk = peaks()
    for (M, D) in [(8192, 2048), (16384, 4096)]:
        x = torch.randn(M, D, device="cuda").to(torch.bfloat16)
        g = torch.ones(D, device="cuda").to(torch.bfloat16)
        y = torch.empty_like(x)
        r = torch.empty(M, device="cuda")
        t = time_fn(lambda: rmsnorm_fwd(x, g, 1e-5, y=y, rstd=r), iters)
        by = 2 * M * D * 2
        print(json.dumps({"kernel": "rmsnorm_fwd", "M": M, "D": D, "ms": round(t, 4),
                          "gbs": round(by / t / 1e6, 1),
                          "frac_of_hbm": round(by / t / 1e6 / pk["hbm_gbs"], 3)}), flush=True)
        # backward with the residual gradient added in place (the engine's form):
        # reads dy, x, dres, writes dx
        dy = torch.randn_like(x)
        dh = torch.randn_like(x)
        dg = torch.zeros(D, device="cuda")
        t = time_fn(lambda: rmsnorm_bwd(dy, x, g, r, dg, dres=dh, dx=dh, accumulate=True), iters)
        by = 4 * M * D * 2
        print(json.dumps({"kernel": "rmsnorm_bwd", "M": M, "D": D, "ms": round(t, 4),
                          "gbs": round(by / t / 1e6, 1),
                          "frac_of_hbm": round(by / t / 1e6 / pk["hbm_gbs"], 3)}), flush=True)


def bench_attention(iters, B=4, S=2048, Hq=32, Hkv=4, Dh=64):
    from lora_kernel_b200.ops.attention import attention_bwd, attention_fwd
    qkv = torch.randn(B * S, (Hq + 2 * Hkv) * Dh, device="cuda").to(torch.bfloat16)
    o, lse = attention_fwd(qkv, B, S, Hq, Hkv, Dh)
    dout = torch.randn_like(o)
    dqkv = torch.empty_like(qkv)
    t_f = time_fn(lambda: attention_fwd(qkv, B, S, Hq, Hkv, Dh, out=o, lse=lse), iters)
    t_b = time_fn(lambda: attention_bwd(qkv, o, dout, lse, B, S, Hq, Hkv, Dh, dqkv=dqkv), iters)
    fl = 4.0 * B * Hq * Dh * S * S / 2  # causal
    q = qkv[:, :Hq * Dh].view(B, S, Hq, Dh).transpose(1, 2)
    k = qkv[:, Hq * Dh:(Hq + Hkv) * Dh].view(B, S, Hkv, Dh).transpose(1, 2)
    v = qkv[:, (Hq + Hkv) * Dh:].view(B, S, Hkv, Dh).transpose(1, 2)
    sdpa = torch.nn.functional.scaled_dot_product_attention
    t_ref = time_fn(lambda: sdpa(q, k, v, is_causal=True, enable_gqa=True), iters)
    qg, kg, vg = (x.detach().clone().requires_grad_(True) for x in (q, k, v))
    og = sdpa(qg, kg, vg, is_causal=True, enable_gqa=True)
    gref = torch.randn_like(og)
    t_refb = time_fn(lambda: torch.autograd.grad(og, (qg, kg, vg), gref, retain_graph=True), iters)
    print(json.dumps({"kernel": "attention", "B": B, "S": S, "Hq": Hq, "Hkv": Hkv, "Dh": Dh,
                      "fwd_ms": round(t_f, 4), "fwd_tflops": round(fl / t_f / 1e9, 1),
                      "bwd_ms": round(t_b, 4), "bwd_tflops": round(2.5 * fl / t_b / 1e9, 1),
                      "sdpa_fwd_ms": round(t_ref, 4), "sdpa_fwd_tflops": round(fl / t_ref / 1e9, 1),
                      "sdpa_bwd_ms": round(t_refb, 4), "sdpa_bwd_tflops": round(2.5 * fl / t_refb / 1e9, 1)}),
          flush=True)


def attention_once(B=4, S=2048, Hq=32, Hkv=4, Dh=64):
    """One attention forward + backward and nothing else (the case ncu captures)."""
    from lora_kernel_b200._ext import check_status
    from lora_kernel_b200.ops.attention import attention_bwd, attention_fwd
    qkv = torch.randn(B * S, (Hq + 2 * Hkv) * Dh, device="cuda").to(torch.bfloat16)
    o, lse = attention_fwd(qkv, B, S, Hq, Hkv, Dh)
    dout = torch.randn_like(o)
    attention_bwd(qkv, o, dout, lse, B, S, Hq, Hkv, Dh)
    torch.cuda.synchronize()
    check_status()
    print(json.dumps({"kernel": "attention_once", "B": B, "S": S, "Hq": Hq, "Hkv": Hkv, "Dh": Dh}), flush=True)


def decode_once():
    """One int4 dequant GEMM (Llama 8B qkv, 64 rows) and one paged fp8 decode
    attention (256 sequences x 2048 tokens, 4 q / 1 kv heads) and nothing else
    (the case ncu captures)."""
    from lora_kernel_b200._ext import check_status
    from lora_kernel_b200.ops import serving as SV
    N, K, M = 6144, 4096, 64
    qw = SV.QuantizedWeight((torch.randn(N, K, device="cuda") * 0.02).to(torch.bfloat16), "int4", 128)
    x = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    qw.matmul_t(x)
    nseq, ctx, Hq, Hkv, Dh, bs = 256, 2048, 4, 1, 128, 16
    nblk = nseq * ctx // bs
    kc = torch.randn(nblk * bs, Hkv, Dh, device="cuda").to(torch.float8_e4m3fn)
    vc = torch.randn(nblk * bs, Hkv, Dh, device="cuda").to(torch.float8_e4m3fn)
    ks = torch.full((nblk * bs, Hkv), 0.01, device="cuda")
    vs = torch.full((nblk * bs, Hkv), 0.01, device="cuda")
    bt = torch.randperm(nblk, device="cuda", dtype=torch.int32).view(nseq, -1)
    lens = torch.full((nseq,), ctx, dtype=torch.int32, device="cuda")
    q = torch.randn(nseq, Hq * Dh, device="cuda").to(torch.bfloat16)
    SV.decode_attention(q, kc, vc, ks, vs, bt, lens, bs, Hq, Hkv, Dh, kv_dtype="fp8", max_ctx=ctx)
    torch.cuda.synchronize()
    check_status()
    print(json.dumps({"kernel": "decode_once", "dq_gemm": [M, N, K], "decode": [nseq, ctx, Hq, Hkv, Dh]}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default="gemm,norm")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--small", action="store_true", help="one small GEMM (for profiling)")
    ap.add_argument("--pair", type=int, default=-1,
                    help="GEMMs on CTA pairs (cta_group::2, 256-row tiles): 1 on, 0 off, -1 the default")
    args = ap.parse_args()
    if args.pair >= 0:
        from lora_kernel_b200._ext import C
        C().gemm_set_pair(args.pair)
    which = set(args.only.split(","))
    if "gemm" in which:
        if args.small:
            shapes = [(8192, 8192, 8192, "tn")]
        else:
            shapes = [(8192, 8192, 8192, "tn"), (8192, 8192, 8192, "dgrad"),
                      (8192, 8192, 8192, "wgrad"),
                      (8192, 2560, 2048, "tn"), (8192, 11264, 2048, "tn"),
                      (8192, 2048, 5632, "tn"), (8192, 32000, 2048, "tn"),
                      (8192, 2048, 11264, "dgrad"), (11264, 2048, 8192, "wgrad")]
        bench_gemm(shapes, args.iters)
    if "fp8" in which:
        bench_fp8([(8192, 8192, 8192), (8192, 3584, 4096), (8192, 4096, 1792), (8192, 768, 4096)]
                  if not args.small else [(8192, 8192, 8192)], args.iters)
    if "mx" in which:
        bench_mxf8([(8192, 8192, 8192), (8192, 3584, 4096), (8192, 4096, 1792), (8192, 768, 4096),
                    (8192, 4096, 512)] if not args.small else [(4096, 4096, 4096)], args.iters)
    if "decode" in which:
        bench_decode(args.iters)
    if "norm" in which:
        bench_norm(args.iters)
    if "attn" in which:
        bench_attention(args.iters)  # Llama 1.1B: B 4, S 2048, 32 / 4 heads, head_dim 64
    if "attn_once" in which:
        attention_once()
    if "decode_once" in which:
        decode_once()
    if "attn8b_once" in which:
        attention_once(B=2, S=4096, Hq=32, Hkv=8, Dh=128)
    if "attn8b" in which:
        bench_attention(args.iters, B=2, S=4096, Hq=32, Hkv=8, Dh=128)  # Llama 8B shape


if __name__ == "__main__":
    main()
