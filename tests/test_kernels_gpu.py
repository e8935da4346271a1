"""Numerics of the sm_100a kernels against plain fp32 PyTorch references."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

dev = "cuda"


def _bf(*shape, scale=1.0):
    return (torch.randn(*shape, device=dev) * scale).to(torch.bfloat16)


def _mn(rows, K):
    """[rows, K] logical operand stored MN-major with a pitch padded to 8."""
    ld = (rows + 7) // 8 * 8
    return _bf(K, ld)[:, :rows].t()


def _close(out, ref, rtol, atol):
    err = (out.float() - ref.float()).abs()
    tol = atol + rtol * ref.float().abs()
    bad = (err > tol).sum().item()
    assert bad == 0, f"{bad} mismatches, max err {err.max().item():.4g}"


def _status_ok():
    from lora_kernel_b200._ext import check_status
    check_status()


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 256), (300, 264, 200),
                                   (1024, 2560, 2048), (77, 128, 1000), (513, 1032, 96)])
@pytest.mark.parametrize("layout", ["tn", "dgrad", "wgrad", "mn_k"])
def test_gemm_layouts(M, N, K, layout):
    from lora_kernel_b200.ops.gemm import gemm
    torch.manual_seed(0)
    if layout == "tn":
        a, b = _bf(M, K), _bf(N, K)
    elif layout == "dgrad":
        a, b = _bf(M, K), _mn(N, K)
    elif layout == "wgrad":
        a, b = _mn(M, K), _mn(N, K)
    else:
        a, b = _mn(M, K), _bf(N, K)
    out = gemm(a, b)
    ref = a.float() @ b.float().t()
    _close(out, ref, 2e-2, 2e-2 * math.sqrt(K) * 0.1 + 1e-2)
    _status_ok()


@pytest.mark.parametrize("bn", [128, 256])
def test_gemm_epilogues(bn):
    from lora_kernel_b200.ops.gemm import gemm
    torch.manual_seed(1)
    M, N, K = 384, 512, 320
    a, b = _bf(M, K), _bf(N, K)
    ref = a.float() @ b.float().t()
    out = gemm(a, b, epi="f32", bn=bn)
    _close(out, ref, 1e-3, 1e-2)
    acc = torch.ones(M, N, device=dev)
    gemm(a, b, acc, epi="f32_acc", bn=bn, alpha=0.5)
    _close(acc, 1 + 0.5 * ref, 1e-3, 1e-2)
    r = _bf(M, N)
    out = gemm(a, b, epi="bf16_resid", residual=r, bn=bn)
    _close(out, ref + r.float(), 2e-2, 5e-2)
    # in-place residual (out aliases the residual)
    r2 = r.clone()
    gemm(a, b, r2, epi="bf16_resid", residual=r2, bn=bn)
    _close(r2, ref + r.float(), 2e-2, 5e-2)
    _status_ok()


def test_gemm_swiglu():
    from lora_kernel_b200.ops.gemm import interleave_gate_up, linear_swiglu
    torch.manual_seed(2)
    T, D, F = 260, 256, 384
    x = _bf(T, D)
    wg, wu = _bf(F, D, scale=0.1), _bf(F, D, scale=0.1)
    gu, h = linear_swiglu(x, interleave_gate_up(wg, wu))
    g = x.float() @ wg.float().t()
    u = x.float() @ wu.float().t()
    _close(h, torch.nn.functional.silu(g) * u, 3e-2, 3e-2)
    from lora_kernel_b200.ops.gemm import split_gate_up
    # gate|up blocks run along the activation's column dimension
    gg, uu = split_gate_up(gu.t().contiguous())
    _close(gg.t(), g, 2e-2, 2e-2)
    _close(uu.t(), u, 2e-2, 2e-2)


@pytest.mark.parametrize("D", [256, 2048, 4096])
@pytest.mark.parametrize("with_res", [False, True])
def test_rmsnorm(D, with_res):
    from lora_kernel_b200.ops.norm import rmsnorm_bwd, rmsnorm_fwd
    torch.manual_seed(3)
    M = 777
    x, g = _bf(M, D), (1 + 0.1 * torch.randn(D, device=dev)).to(torch.bfloat16)
    r = _bf(M, D) if with_res else None
    y, rstd, h = rmsnorm_fwd(x, g, 1e-5, residual=r)
    hf = (x.float() + r.float()) if with_res else x.float()
    hf = hf.to(torch.bfloat16).float()
    ref = hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + 1e-5) * g.float()
    _close(y, ref, 2e-2, 2e-2)
    _close(h, hf, 1e-2, 1e-2)
    # backward vs autograd on the fp32 restatement
    dy = _bf(M, D)
    dres = _bf(M, D)
    hv = h.float().requires_grad_(True)
    gv = g.float().requires_grad_(True)
    out = hv * torch.rsqrt(hv.pow(2).mean(-1, keepdim=True) + 1e-5) * gv
    out.backward(dy.float())
    dgamma = torch.zeros(D, device=dev)
    dx = rmsnorm_bwd(dy, h, g, rstd, dgamma, dres=dres)
    _close(dx, hv.grad + dres.float(), 3e-2, 3e-2)
    _close(dgamma, gv.grad, 1e-2, 1e-1)


def test_rope_roundtrip_and_values():
    from lora_kernel_b200.ops.elementwise import rope_, rope_table
    torch.manual_seed(4)
    B, S, H, Dh = 2, 64, 3, 64
    x = _bf(B * S, H * Dh + 64)
    tab = rope_table(S, Dh, 10000.0, dev)
    y = x.clone()
    rope_(y, 0, H, Dh, tab, seq_len=S)
    # reference: interleaved pairs
    xf = x.float()[:, :H * Dh].reshape(B, S, H, Dh // 2, 2)
    pos = torch.arange(S, device=dev, dtype=torch.float64)
    inv = 10000.0 ** (-torch.arange(0, Dh, 2, device=dev, dtype=torch.float64) / Dh)
    ang = (pos[:, None] * inv[None]).float()
    c, s = torch.cos(ang)[None, :, None], torch.sin(ang)[None, :, None]
    r0 = xf[..., 0] * c - xf[..., 1] * s
    r1 = xf[..., 0] * s + xf[..., 1] * c
    ref = torch.stack([r0, r1], -1).reshape(B * S, H * Dh)
    _close(y[:, :H * Dh], ref, 2e-2, 2e-2)
    assert torch.equal(y[:, H * Dh:], x[:, H * Dh:])
    rope_(y, 0, H, Dh, tab, seq_len=S, inverse=True)
    _close(y, x, 2e-2, 2e-2)


def test_swiglu_bwd():
    from lora_kernel_b200.ops.elementwise import swiglu_bwd, swiglu_fwd
    from lora_kernel_b200.ops.gemm import interleave_gate_up, split_gate_up
    torch.manual_seed(5)
    T, F = 100, 256
    g, u = _bf(T, F), _bf(T, F)
    gu = interleave_gate_up(g.t().contiguous(), u.t().contiguous()).t().contiguous()
    h = swiglu_fwd(gu)
    gv, uv = g.float().requires_grad_(True), u.float().requires_grad_(True)
    hv = torch.nn.functional.silu(gv) * uv
    _close(h, hv, 2e-2, 2e-2)
    dh = _bf(T, F)
    hv.backward(dh.float())
    dgu = swiglu_bwd(gu, dh)
    dg, du = split_gate_up(dgu.t().contiguous())
    _close(dg.t(), gv.grad, 3e-2, 3e-2)
    _close(du.t(), uv.grad, 3e-2, 3e-2)


def test_embedding():
    from lora_kernel_b200.ops.elementwise import embedding_bwd, embedding_fwd
    torch.manual_seed(6)
    V, D, T = 1000, 256, 555
    W = _bf(V, D)
    ids = torch.randint(0, V, (T,), device=dev)
    out = embedding_fwd(ids, W)
    assert torch.equal(out, W[ids])
    dy = _bf(T, D)
    dW = torch.zeros(V, D, device=dev)
    embedding_bwd(ids, dy, dW)
    ref = torch.zeros(V, D, device=dev).index_add_(0, ids, dy.float())
    _close(dW, ref, 1e-4, 1e-3)
    _status_ok()


@pytest.mark.parametrize("V", [1024, 32000])
@pytest.mark.parametrize("smooth,zl", [(0.0, 0.0), (0.1, 1e-4)])
def test_cross_entropy(V, smooth, zl):
    from lora_kernel_b200.ops.loss import cross_entropy_
    torch.manual_seed(7)
    T = 300
    logits = _bf(T, V, scale=2.0)
    tgt = torch.randint(0, V, (T,), device=dev)
    tgt[5] = -100
    zf = logits.float().requires_grad_(True)
    lse = torch.logsumexp(zf, -1)
    nll = torch.nn.functional.cross_entropy(zf, tgt, ignore_index=-100, reduction="none",
                                            label_smoothing=smooth)
    valid = (tgt != -100).float()
    loss = (nll + zl * lse ** 2 * valid).sum()
    loss.backward()
    acc = torch.zeros(2, device=dev)
    scale = torch.tensor([4.0], device=dev)
    g = logits.clone()
    cross_entropy_(g, tgt, acc, scale=scale, scale_mul=0.5, smoothing=smooth, z_loss=zl)
    assert abs(acc[0].item() - loss.item()) < 1e-3 * abs(loss.item()) + 1e-2
    assert acc[1].item() == T - 1
    _close(g, zf.grad * 2.0, 2e-2, 2e-3)


def test_adamw_and_finalize():
    from lora_kernel_b200.ops import optim
    torch.manual_seed(8)
    n = 10000 + 36
    p = torch.randn(n, device=dev)
    g = torch.randn(n, device=dev) * 3.0
    scale = 1024.0
    st = optim.new_state(dev, loss_scale=scale, lr=1e-2)
    chunks = optim.make_chunks([(0, 5000, True), (5000, n - 5000, False)], chunk=2048, device=dev)
    m, v = torch.zeros(n, device=dev), torch.zeros(n, device=dev)
    p16 = torch.empty(n, dtype=torch.bfloat16, device=dev)
    partial = torch.zeros(64, device=dev)
    gs = g * scale
    optim.grad_norm_partials(gs, partial)
    optim.finalize(partial, st, max_norm=1.0, dynamic=True)
    p_ref = p.clone().requires_grad_(True)
    opt = torch.optim.AdamW([{"params": [p_ref]}], lr=1e-2, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.0)
    norm = g.norm()
    gclip = g * (1.0 / (norm + 1e-6))
    p_ref.grad = gclip.clone()
    # decoupled wd only on the first segment
    with torch.no_grad():
        p_ref[:5000] *= (1 - 1e-2 * 0.1)
    opt.step()
    optim.adamw_(p, gs, m, v, chunks, st, p16=p16, beta1=0.9, beta2=0.95, eps=1e-8, wd=0.1)
    _close(p, p_ref.detach(), 1e-5, 1e-5)
    assert abs(st[optim.ST_GRAD_NORM].item() - norm.item()) < 1e-3 * norm.item()
    assert st[optim.ST_STEP].item() == 1 and st[optim.ST_SKIP].item() == 0
    assert torch.count_nonzero(gs) == 0  # zero_grad fused
    # overflow: step skipped, scale halved
    gs2 = torch.randn(n, device=dev)
    gs2[7] = float("inf")
    optim.grad_norm_partials(gs2, partial)
    optim.finalize(partial, st, max_norm=1.0, dynamic=True)
    before = p.clone()
    optim.adamw_(p, gs2, m, v, chunks, st, p16=p16)
    assert torch.equal(p, before)
    assert st[optim.ST_SKIP].item() == 1 and st[optim.ST_LOSS_SCALE].item() == scale / 2


def test_gelu_fwd_bwd_vs_fp32():
    from lora_kernel_b200.ops import elementwise as E
    torch.manual_seed(0)
    x = (torch.randn(300, 1024, device="cuda") * 3).bfloat16()
    dy = torch.randn_like(x)
    xf = x.float().requires_grad_(True)
    ref = torch.nn.functional.gelu(xf, approximate="tanh")
    ref.backward(dy.float())
    y = E.gelu_fwd(x)
    dx = E.gelu_bwd(x, dy)
    torch.cuda.synchronize()
    assert ((y.float() - ref).abs() <= 1e-2 * ref.abs() + 1e-2).all()
    assert ((dx.float() - xf.grad).norm() / xf.grad.norm()).item() < 1e-2


@pytest.mark.parametrize("D", [256, 1024, 4096])
def test_layernorm_fwd_bwd_vs_fp32(D):
    from lora_kernel_b200.ops import norm as N
    torch.manual_seed(1)
    M = 333
    x = (torch.randn(M, D, device="cuda") * 2 + 0.5).bfloat16()
    g = (1 + 0.2 * torch.randn(D, device="cuda")).bfloat16()
    b = (0.1 * torch.randn(D, device="cuda")).bfloat16()
    dy = torch.randn(M, D, device="cuda").bfloat16()
    xf, gf, bf = (t.float().requires_grad_(True) for t in (x, g, b))
    ref = torch.nn.functional.layer_norm(xf, (D,), gf, bf, 1e-5)
    ref.backward(dy.float())
    y, mean, rstd = N.layernorm_fwd(x, g, b, 1e-5)
    dgamma = torch.zeros(D, device="cuda")
    dbeta = torch.zeros(D, device="cuda")
    dx = N.layernorm_bwd(dy, x, g, mean, rstd, dgamma, dbeta)
    torch.cuda.synchronize()
    rel = lambda a, r: ((a.float() - r).norm() / r.norm()).item()  # noqa: E731
    assert rel(y, ref.detach()) < 1e-2
    assert rel(dx, xf.grad) < 2e-2
    assert rel(dgamma, gf.grad) < 1e-3 and rel(dbeta, bf.grad) < 1e-3


@pytest.mark.gpu
def test_peer_wait_gives_up_with_a_status_and_the_context_survives():
    """Failure detection on one GPU without a fault: a two-rank signal barrier
    whose second "peer" flag array is a local buffer that nothing writes.  The
    waiting thread gives up after the kernels' bound (2 s), records "timeout
    waiting for a peer GPU" (4) in the status word and returns; the same
    barrier with the flag set passes and the context keeps working."""
    import time as _time
    from lora_kernel_b200._ext import C, STATUS_NAMES
    mine = torch.zeros(2, dtype=torch.int32, device="cuda")     # rank 0's slots: [from 0, from 1]
    peer = torch.zeros(2, dtype=torch.int32, device="cuda")     # the absent rank 1's slots
    table = torch.tensor([mine.data_ptr(), peer.data_ptr()], dtype=torch.int64, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    t0 = _time.perf_counter()
    C().signal_barrier(table, 0, 2, 0, 1, status)
    torch.cuda.synchronize()
    waited = _time.perf_counter() - t0
    assert STATUS_NAMES[int(status.item())] == "timeout waiting for a peer GPU"
    assert 1.5 < waited < 30.0, waited
    assert int(peer[0].item()) == 1          # rank 0 still signalled the peer
    # the peer "arrives": epoch 2 is already in rank 0's slot from rank 1
    mine[1] = 2
    status.zero_()
    C().signal_barrier(table, 0, 2, 0, 2, status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    x = torch.arange(1024, device="cuda", dtype=torch.float32)
    assert float(x.sum().item()) == 1023 * 1024 / 2


@pytest.mark.parametrize("layout", ["tn", "dgrad", "wgrad", "nt"])
def test_gemm_cta_pair_matches_fp32(layout):
    """256 x 256 tiles computed by a CTA pair (tcgen05.mma.cta_group::2) with
    ragged M, N and K edges, every operand layout and epilogue."""
    from lora_kernel_b200._ext import C
    from lora_kernel_b200.ops.gemm import gemm
    torch.manual_seed(3)
    M, N, K = 2600, 2056, 320
    if layout == "tn":
        a, b = _bf(M, K), _bf(N, K)
    elif layout == "dgrad":
        a, b = _bf(M, K), _mn(N, K)
    elif layout == "wgrad":
        a, b = _mn(M, K), _mn(N, K)
    else:
        a, b = _mn(M, K), _bf(N, K)
    ref = a.float() @ b.float().t()
    C().gemm_set_pair(1)
    try:
        n0 = C().gemm_pair_count()
        out = gemm(a, b)
        _close(out, ref, 2e-2, 2e-2 * math.sqrt(K) * 0.1 + 1e-2)
        if layout != "nt":
            out = gemm(a, b, epi="f32")
            _close(out, ref, 1e-3, 1e-2)
            acc = torch.ones(M, N, device=dev)
            gemm(a, b, acc, epi="f32_acc", alpha=0.5)
            _close(acc, 1 + 0.5 * ref, 1e-3, 1e-2)
        if layout == "tn":
            r = _bf(M, N)
            r0 = r.float()
            gemm(a, b, r, epi="bf16_resid", residual=r)  # in place
            _close(r, ref + r0, 2e-2, 5e-2)
        assert C().gemm_pair_count() > n0, "the CTA-pair path did not run"
        _status_ok()
    finally:
        C().gemm_set_pair(1)


def test_gemm_cta_pair_fused_epilogues():
    from lora_kernel_b200._ext import C
    from lora_kernel_b200.ops.gemm import gemm, interleave_gate_up, linear_swiglu
    torch.manual_seed(4)
    T, D, F = 2600, 256, 1536
    x = _bf(T, D)
    wg, wu = _bf(F, D, scale=0.1), _bf(F, D, scale=0.1)
    w = _bf(2048, D)
    r = _bf(T, 2048)
    C().gemm_set_pair(1)
    try:
        n0 = C().gemm_pair_count()
        gu, h = linear_swiglu(x, interleave_gate_up(wg, wu))
        g = x.float() @ wg.float().t()
        u = x.float() @ wu.float().t()
        _close(h, torch.nn.functional.silu(g) * u, 3e-2, 3e-2)
        out = gemm(x, w, epi="bf16_resid", residual=r)
        _close(out, x.float() @ w.float().t() + r.float(), 2e-2, 5e-2)
        assert C().gemm_pair_count() >= n0 + 2
        _status_ok()
    finally:
        C().gemm_set_pair(1)


@pytest.mark.parametrize("M,F,D", [(256, 256, 256), (1000, 640, 384), (4096, 1536, 1024)])
def test_gemm_swiglu_bwd_epilogue(M, F, D):
    """The down projection's data gradient with the SwiGLU backward in its
    epilogue (gate|up in 128-column blocks) against fp32 PyTorch."""
    from lora_kernel_b200.ops import gemm as G
    g = torch.Generator(device="cuda").manual_seed(4)
    dy = torch.randn(M, D, device="cuda", generator=g).bfloat16()
    w = (torch.randn(D, F, device="cuda", generator=g) * 0.05).bfloat16()
    gu = torch.randn(M, 2 * F, device="cuda", generator=g).bfloat16()
    dgu = G.gemm(dy, w.t(), epi="swiglu_bwd", residual=gu, alpha=0.5)
    torch.cuda.synchronize()
    dh = 0.5 * (dy.float() @ w.float())
    blk = gu.float().view(M, F // 128, 2, 128)
    gate, up = blk[:, :, 0].reshape(M, F), blk[:, :, 1].reshape(M, F)
    s = torch.sigmoid(gate)
    dgate = dh * up * s * (1 + gate * (1 - s))
    dup = dh * gate * s
    ref = torch.stack([dgate.view(M, F // 128, 128), dup.view(M, F // 128, 128)], 2).view(M, 2 * F)
    err = (dgu.float() - ref).norm() / ref.norm()
    assert err < 1e-2, err


@pytest.mark.parametrize("S,Dh,Hq,Hkv", [(256, 64, 4, 2), (512, 128, 2, 1)])
def test_gemm_rope_epilogue(S, Dh, Hq, Hkv):
    """The QKV GEMM with RoPE in its epilogue against fp32 PyTorch: x W^T, then the
    interleaved-pair rotation of the q and k heads at position row % S; v untouched."""
    from lora_kernel_b200.ops import gemm as G
    from lora_kernel_b200.ops.elementwise import rope_table
    g = torch.Generator(device="cuda").manual_seed(6)
    B, D = 3, 256
    N = (Hq + 2 * Hkv) * Dh
    x = torch.randn(B * S, D, device="cuda", generator=g).bfloat16()
    w = (torch.randn(N, D, device="cuda", generator=g) * 0.05).bfloat16()
    tab = rope_table(S, Dh, 10000.0, "cuda")
    y = G.gemm(x, w, rope=(tab, (Hq + Hkv) * Dh, Dh, S, 0))
    torch.cuda.synchronize()
    ref = x.float() @ w.float().t()
    nrot = (Hq + Hkv) * Dh
    r = ref[:, :nrot].view(B * S, Hq + Hkv, Dh // 2, 2)
    pos = torch.arange(B * S, device="cuda") % S
    c, s = tab[pos, :, 0][:, None, :], tab[pos, :, 1][:, None, :]
    x0, x1 = r[..., 0], r[..., 1]
    rot = torch.stack([x0 * c - x1 * s, x0 * s + x1 * c], -1).view(B * S, nrot)
    ref = torch.cat([rot, ref[:, nrot:]], 1)
    err = (y.float() - ref).norm() / ref.norm()
    assert err < 1e-2, err
