"""Launched by tests/test_tp_multigpu.py under torchrun (one process per GPU).

  ops    K16 all-gather->GEMM, K18 GEMM->reduce-scatter + owner-side sum/norm and
         the vocabulary-parallel cross-entropy against plain PyTorch fp32
  model  TP forward/backward (fused peer-memory path and the NCCL baseline)
         against the single-GPU engine with the same weights
  train  a few TPTrainer steps: finite, decreasing loss; p2p and NCCL agree
Writes a JSON verdict per rank to $LK_OUT.<rank>."""
import json
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from lora_kernel_b200._ext import C, check_status, status  # noqa: E402
from lora_kernel_b200.config import TrainConfig, TransformerConfig  # noqa: E402
from lora_kernel_b200.parallel import tp as TP  # noqa: E402
from lora_kernel_b200.parallel.comm import init_distributed  # noqa: E402

CFG = dict(hidden_dim=256, num_heads=4, num_kv_heads=2, head_dim=64, ff_dim=512, vocab_size=1024,
           num_layers=2, max_seq_len=256)


def rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


def check_ops(rank, world, res):
    cfg = TransformerConfig(**CFG)
    dev = torch.device("cuda", torch.cuda.current_device())
    T = 256 * world
    R = T // world
    D = cfg.hidden_dim
    comm = TP.TPComm(cfg, T, dev)
    g = torch.Generator(device=dev).manual_seed(100 + rank)
    # ---- K16: every rank's rows -> gathered A -> GEMM (plain and SwiGLU epilogue)
    mine = torch.randn(R, D, device=dev, generator=g).bfloat16()
    comm.stage_view(0, R, D).copy_(mine)
    allrows = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(allrows, mine)
    full = torch.cat(allrows)
    gw = torch.Generator(device=dev).manual_seed(7)
    w = (torch.randn(384, D, device=dev, generator=gw) * 0.05).bfloat16()
    dst = torch.empty(T, D, dtype=torch.bfloat16, device=dev)
    out = torch.empty(T, 384, dtype=torch.bfloat16, device=dev)
    comm.barrier()
    comm.ag_gemm(0, dst, w, out)
    torch.cuda.synchronize()
    res["ag_gather_exact"] = bool(torch.equal(dst, full))
    res["ag_gemm_err"] = rel(out, full.float() @ w.float().t())
    # B MN-major (dgrad form)
    wt = (torch.randn(D, 256, device=dev, generator=gw) * 0.05).bfloat16()
    out2 = torch.empty(T, 256, dtype=torch.bfloat16, device=dev)
    comm.barrier()
    comm.ag_gemm(0, dst, wt.t(), out2)
    torch.cuda.synchronize()
    res["ag_gemm_mn_err"] = rel(out2, full.float() @ wt.float())
    # SwiGLU epilogue
    wgu = (torch.randn(512, D, device=dev, generator=gw) * 0.05).bfloat16()
    gu = torch.empty(T, 512, dtype=torch.bfloat16, device=dev)
    act = torch.empty(T, 256, dtype=torch.bfloat16, device=dev)
    comm.barrier()
    comm.ag_gemm(1 - 1, dst, wgu, gu, epi="swiglu", h_out=act)
    torch.cuda.synchronize()
    ref_gu = full.float() @ wgu.float().t()
    blk = ref_gu.view(T, 2, 2, 128)
    ref_act = (torch.nn.functional.silu(blk[:, :, 0]) * blk[:, :, 1]).reshape(T, 256)
    res["ag_swiglu_err"] = rel(act, ref_act)
    # ---- K18: partial rows -> owners; owner sum + residual + RMSNorm
    a = (torch.randn(T, 512, device=dev, generator=g) * 0.5).bfloat16()
    wo = (torch.randn(D, 512, device=dev, generator=gw) * 0.05).bfloat16()
    part = a.float() @ wo.float().t()                 # this rank's partial [T, D]
    tot = part.clone()
    dist.all_reduce(tot)
    resid = torch.randn(R, D, device=dev, generator=g).bfloat16()
    gamma = (1 + 0.1 * torch.randn(D, device=dev, generator=gw)).bfloat16()
    hout = torch.empty(R, D, dtype=torch.bfloat16, device=dev)
    y = comm.stage_view(1, R, D)
    rstd = torch.empty(R, dtype=torch.float32, device=dev)
    comm.gemm_rs(0, a, wo)
    comm.rs_sum(0, hout, resid=resid, gamma=gamma, y=y, rstd=rstd, eps=1e-5)
    torch.cuda.synchronize()
    want_h = tot[rank * R:(rank + 1) * R] + resid.float()
    res["rs_sum_err"] = rel(hout, want_h)
    hq = hout.float()
    want_y = hq * torch.rsqrt(hq.pow(2).mean(-1, keepdim=True) + 1e-5) * gamma.float()
    res["rs_norm_err"] = rel(y, want_y)
    # MN-major B into K18 (dgrad form), plain sum
    wb = (torch.randn(512, D, device=dev, generator=gw) * 0.05).bfloat16()
    comm.gemm_rs(1, a, wb.t())
    plain = torch.empty(R, D, dtype=torch.bfloat16, device=dev)
    comm.rs_sum(1, plain)
    tot2 = a.float() @ wb.float()
    dist.all_reduce(tot2)
    torch.cuda.synchronize()
    res["rs_mn_err"] = rel(plain, tot2[rank * R:(rank + 1) * R])
    # ---- vocabulary-parallel cross-entropy vs full-vocabulary fp32
    V = cfg.vocab_size
    Vl = V // world
    gl = torch.Generator(device=dev).manual_seed(3)
    logits_full = (torch.randn(T, V, device=dev, generator=gl) * 2).bfloat16()
    tgt = torch.randint(0, V, (T,), device=dev, generator=gl)
    tgt[5] = -100
    local = logits_full[:, rank * Vl:(rank + 1) * Vl].contiguous()
    acc = torch.zeros(2, device=dev)
    comm.cross_entropy(local, tgt, acc, scale=None, scale_mul=1.0 / T, smoothing=0.1)
    torch.cuda.synchronize()
    lf = logits_full.float().requires_grad_(True)
    loss = torch.nn.functional.cross_entropy(lf, tgt, ignore_index=-100, label_smoothing=0.1,
                                             reduction="sum")
    (loss / T).backward()
    res["ce_loss_err"] = abs(acc[0].item() - loss.item()) / abs(loss.item())
    res["ce_count"] = acc[1].item() == T - 1
    res["ce_grad_err"] = rel(local, lf.grad[:, rank * Vl:(rank + 1) * Vl])
    check_status()


def check_fp8(rank, world, res):
    """fp8 (K2) with the collectives fused: gather of e4m3 rows + scales, and the
    reduce-scatter epilogue, against unfused fp8 GEMMs + NCCL; then the TP model
    with fp8 projections against the bf16 TP model."""
    from lora_kernel_b200.ops import fp8 as F
    cfg = TransformerConfig(**CFG)
    dev = torch.device("cuda", torch.cuda.current_device())
    T = 256 * world
    R, D = T // world, cfg.hidden_dim
    comm = TP.TPComm(cfg, T, dev)
    g = torch.Generator(device=dev).manual_seed(200 + rank)
    mine = torch.randn(R, D, device=dev, generator=g).bfloat16()
    gw = torch.Generator(device=dev).manual_seed(9)
    w8 = F.Fp8Weight((torch.randn(384, D, device=dev, generator=gw) * 0.05).bfloat16(), transpose=False)
    comm.publish_fp8(0, mine)
    comm.barrier()
    dst8 = torch.empty(T, D, dtype=torch.uint8, device=dev)
    dsts = torch.empty(D // 128, T, dtype=torch.float32, device=dev)
    out = torch.empty(T, 384, dtype=torch.bfloat16, device=dev)
    comm.ag_gemm_fp8(0, dst8, dsts, w8, out)
    torch.cuda.synchronize()
    q, sc = F.quantize_1x128(mine)
    allq = [torch.empty_like(q) for _ in range(world)]
    alls = [torch.empty_like(sc) for _ in range(world)]
    dist.all_gather(allq, q)
    dist.all_gather(alls, sc)
    fq, fs = torch.cat(allq), torch.cat(alls, dim=1).contiguous()
    res["fp8_ag_rows_exact"] = bool(torch.equal(dst8, fq)) and bool(torch.equal(dsts, fs))
    ref = F.gemm_fp8(fq, fs, w8.q, w8.scale)
    res["fp8_ag_gemm_err"] = rel(out, ref)
    # reduce-scatter epilogue
    a = (torch.randn(T, 256, device=dev, generator=g)).bfloat16()
    wo8 = F.Fp8Weight((torch.randn(D, 256, device=dev, generator=gw) * 0.05).bfloat16(), transpose=False)
    comm.gemm_rs_fp8(0, a, wo8)
    hout = torch.empty(R, D, dtype=torch.bfloat16, device=dev)
    comm.rs_sum(0, hout)
    part = F.linear_fp8(a, wo8).float()
    dist.all_reduce(part)
    torch.cuda.synchronize()
    res["fp8_rs_err"] = rel(hout, part[rank * R:(rank + 1) * R])
    # model: fp8 projections vs bf16
    B, S = 2, 128
    gt = torch.Generator().manual_seed(11)
    tok = torch.randint(0, cfg.vocab_size, (B, S + 1), generator=gt).cuda()
    ids, tg = tok[:, :-1].contiguous(), tok[:, 1:].contiguous()
    outs = []
    for fp8 in (False, "exact", "mx"):
        c2 = TP.TPComm(cfg, B * S, dev)
        params = TP.TPParams(cfg, world, rank, dev)
        params.init_(5, cfg.init_std)
        m = TP.TPLlamaModel(cfg, c2, params, fp8=fp8)
        acc = m.forward_backward(ids, tg, grad_scale=1.0 / tg.numel(), overwrite_grads=True)
        torch.cuda.synchronize()
        outs.append((acc.clone(), m.grads.flat.clone()))
    check_status()
    res["fp8_model_loss_rel"] = abs(outs[1][0][0].item() - outs[0][0][0].item()) / outs[0][0][0].item()
    res["fp8_model_grad_rel"] = rel(outs[1][1], outs[0][1])
    res["mx_model_loss_rel"] = abs(outs[2][0][0].item() - outs[0][0][0].item()) / outs[0][0][0].item()
    res["mx_model_grad_rel"] = rel(outs[2][1], outs[0][1])


def check_mx(rank, world, res):
    """MX fp8 (tcgen05 block-scaled) with the collectives fused: the gather of e4m3
    rows + SF tiles, the gather of e5m2 gradient rows against W^T, and the
    reduce-scatter epilogue, against unfused MX GEMMs + NCCL."""
    from lora_kernel_b200.ops import fp8 as F
    cfg = TransformerConfig(**CFG)
    dev = torch.device("cuda", torch.cuda.current_device())
    T = 256 * world
    R, D = T // world, cfg.hidden_dim
    comm = TP.TPComm(cfg, T, dev)
    g = torch.Generator(device=dev).manual_seed(300 + rank)
    gw = torch.Generator(device=dev).manual_seed(19)
    mine = torch.randn(R, D, device=dev, generator=g).bfloat16()
    w = F.MXWeight((torch.randn(384, D, device=dev, generator=gw) * 0.05).bfloat16())
    comm.publish_mx(0, mine)
    comm.barrier()
    dst8 = torch.empty(T, D, dtype=torch.uint8, device=dev)
    dstsf = torch.empty(F.sf_tile_bytes(T, D), dtype=torch.uint8, device=dev)
    out = torch.empty(T, 384, dtype=torch.bfloat16, device=dev)
    comm.ag_gemm_mx(0, dst8, dstsf, w.q, w.sf, out)
    torch.cuda.synchronize()
    q, sf = F.quantize_mx(mine)
    allq = [torch.empty_like(q) for _ in range(world)]
    allsf = [torch.empty_like(sf) for _ in range(world)]
    dist.all_gather(allq, q)
    dist.all_gather(allsf, sf)
    fq, fsf = torch.cat(allq), torch.cat(allsf)
    res["mx_ag_rows_exact"] = bool(torch.equal(dst8, fq)) and bool(torch.equal(dstsf, fsf))
    res["mx_ag_gemm_err"] = rel(out, F.gemm_mxf8(fq, fsf, w.q, w.sf))
    # e5m2 rows gathered into the data-gradient GEMM against W^T
    w2 = F.MXWeight((torch.randn(D, 256, device=dev, generator=gw) * 0.05).bfloat16())
    dmine = (torch.randn(R, D, device=dev, generator=g) * 1e-3).bfloat16()
    comm.publish_mx(1, dmine, fmt=1)
    comm.barrier()
    out2 = torch.empty(T, 256, dtype=torch.bfloat16, device=dev)
    comm.ag_gemm_mx(1, dst8, dstsf, w2.qt, w2.sft, out2, a_fmt=1)
    torch.cuda.synchronize()
    alld = [torch.empty_like(dmine) for _ in range(world)]
    dist.all_gather(alld, dmine)
    dfull = torch.cat(alld).float()
    res["mx_ag_dgrad_err"] = rel(out2, dfull @ w2.dequantize())
    # reduce-scatter epilogue (e5m2 input against W^T, the row-parallel data gradient)
    a = (torch.randn(T, 256, device=dev, generator=g) * 1e-3).bfloat16()
    comm.gemm_rs_mx(0, a, w2.q, w2.sf, a_fmt=1)
    hout = torch.empty(R, D, dtype=torch.bfloat16, device=dev)
    comm.rs_sum(0, hout)
    qa, sfa = F.quantize_mx(a, F.E5M2)
    part = F.gemm_mxf8(qa, sfa, w2.q, w2.sf, a_fmt=F.E5M2).float()
    dist.all_reduce(part)
    torch.cuda.synchronize()
    res["mx_rs_err"] = rel(hout, part[rank * R:(rank + 1) * R])
    check_status()


def _single_gpu(cfg, ids, tg, seed):
    from lora_kernel_b200.models.llama import LlamaModel
    m = LlamaModel(cfg, "cuda", seed=seed)
    acc = m.forward_backward(ids, tg, grad_scale=1.0 / tg.numel(), overwrite_grads=True)
    torch.cuda.synchronize()
    return m, acc.clone()


def check_model(rank, world, res, mode):
    cfg = TransformerConfig(**CFG)
    dev = torch.device("cuda", torch.cuda.current_device())
    B, S = 2, 128
    g = torch.Generator().manual_seed(11)
    tok = torch.randint(0, cfg.vocab_size, (B, S + 1), generator=g).cuda()
    ids, tg = tok[:, :-1].contiguous(), tok[:, 1:].contiguous()
    ref, ref_acc = _single_gpu(cfg, ids, tg, seed=5)
    comm = TP.TPComm(cfg, B * S, dev, comm=mode)
    params = TP.TPParams(cfg, world, rank, dev)
    params.init_(5, cfg.init_std)
    # the shards of the single-GPU weights
    for s in params.specs:
        want = TP.shard_tensor(cfg, s.name, ref.params[s.name], rank, world)
        if not torch.equal(params[s.name], want):
            res[f"init_mismatch.{s.name}"] = True
    model = TP.TPLlamaModel(cfg, comm, params)
    acc = model.forward_backward(ids, tg, grad_scale=1.0 / tg.numel(), overwrite_grads=True)
    torch.cuda.synchronize()
    check_status()
    res[f"{mode}.loss_rel"] = abs(acc[0].item() - ref_acc[0].item()) / ref_acc[0].item()
    worst = 0.0
    for s in params.specs:
        got = model.grads[s.name].clone()
        if s.group == "replicated":
            dist.all_reduce(got)
        want = TP.shard_tensor(cfg, s.name, ref.grads[s.name], rank, world)
        e = rel(got, want)
        res[f"{mode}.grad.{s.name}"] = round(e, 5)
        worst = max(worst, e)
    res[f"{mode}.grad_worst"] = worst


def check_train(rank, world, res, mode):
    cfg = TransformerConfig(**CFG)
    tc = TrainConfig(lr=2e-3, weight_decay=0.1, dynamic_loss_scale=True, init_loss_scale=1024.0, seed=5)
    tr = TP.TPTrainer(cfg, tc, micro_batch=2, seq_len=128, comm=mode, seed=5)
    g = torch.Generator().manual_seed(1)
    tok = torch.randint(0, cfg.vocab_size, (2, 129), generator=g).cuda()
    batch = [(tok[:, :-1].contiguous(), tok[:, 1:].contiguous())]
    losses = []
    for _ in range(6):
        acc = tr.train_step(batch)
        losses.append((acc[0] / acc[1]).item())
    torch.cuda.synchronize()
    check_status()
    res[f"train.{mode}.losses"] = losses
    res[f"train.{mode}.norm"] = float(tr.opt.state[6])


def main():
    what = sys.argv[1]
    rank, world, local = init_distributed("nccl", timeout_s=120)
    res = {"rank": rank, "world": world}
    if what == "ops":
        check_ops(rank, world, res)
    elif what == "model":
        check_model(rank, world, res, "p2p")
        check_model(rank, world, res, "nccl")
    elif what == "fp8":
        check_fp8(rank, world, res)
        check_mx(rank, world, res)
    elif what == "train":
        check_train(rank, world, res, "p2p")
        check_train(rank, world, res, "nccl")
    with open(f"{os.environ['LK_OUT']}.{rank}", "w") as f:
        json.dump(res, f)
    torch.cuda.synchronize()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
