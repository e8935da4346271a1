"""K2 in MX form (tcgen05 block-scaled fp8, UE8M0 scales in TMEM) against plain
PyTorch fp32 references.

The first group feeds hand-built scale tiles, one dimension of variation at a
time (unit scales, per-row of A, per-row of B, per 32-wide K sub-block), so a
mistake in any part of the scale layout shows up as its own failing case; the
second group runs the quantisers and the training-path wrappers."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm()).item()


def _rand_fp8(R, K, fmt, g):
    x = torch.randn(R, K, device="cuda", generator=g) * 4
    dt = torch.float8_e4m3fn if fmt == 0 else torch.float8_e5m2
    return x.to(dt).view(torch.uint8)


def _deq(q, e, fmt):
    dt = torch.float8_e4m3fn if fmt == 0 else torch.float8_e5m2
    return q.view(dt).float() * torch.exp2(e.float()).repeat_interleave(32, 1)


@pytest.mark.parametrize("case", ["unit", "rows_a", "rows_b", "sub_k", "random"])
@pytest.mark.parametrize("M,N,K", [(128, 256, 128), (384, 512, 512), (200, 264, 256)])
def test_mxf8_scale_layout(case, M, N, K):
    from lora_kernel_b200.ops import fp8 as F
    g = torch.Generator(device="cuda").manual_seed(3)
    a8, b8 = _rand_fp8(M, K, 0, g), _rand_fp8(N, K, 0, g)
    ea = torch.zeros(M, K // 32, dtype=torch.int32, device="cuda")
    eb = torch.zeros(N, K // 32, dtype=torch.int32, device="cuda")
    if case == "rows_a":
        ea += (torch.arange(M, device="cuda") % 7 - 3).view(-1, 1)
    elif case == "rows_b":
        eb += (torch.arange(N, device="cuda") % 5 - 2).view(-1, 1)
    elif case == "sub_k":
        ea += (torch.arange(K // 32, device="cuda") % 4).view(1, -1)
        eb -= (torch.arange(K // 32, device="cuda") % 3).view(1, -1)
    elif case == "random":
        ea = torch.randint(-4, 5, ea.shape, device="cuda", dtype=torch.int32, generator=g)
        eb = torch.randint(-4, 5, eb.shape, device="cuda", dtype=torch.int32, generator=g)
    sfa = F.exponents_to_sf(ea, 128)
    sfb = F.exponents_to_sf(eb, 256)
    y = F.gemm_mxf8(a8, sfa, b8, sfb)
    torch.cuda.synchronize()
    ref = _deq(a8, ea, 0) @ _deq(b8, eb, 0).t()
    assert _rel(y, ref) < 1e-2, case


def test_mxf8_quantisers_and_error_bound():
    from lora_kernel_b200.ops import fp8 as F
    g = torch.Generator(device="cuda").manual_seed(0)
    M, N, K = 1000, 1536, 2048
    x = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    x[:, :128] *= 300  # blocks of very different magnitude
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.05).bfloat16()
    q, sf = F.quantize_mx(x)
    # power-of-two scales: every block's amax lands in (fmax/2, fmax] of e4m3
    xd = F.dequantize_mx(q, sf)
    blk = x.float().abs().view(M, K // 128, 128).amax(-1)
    e = F.sf_to_exponents(sf, M, K)[:, ::4].float()
    scaled = blk / torch.exp2(e)
    assert bool(((scaled <= 448) & ((scaled > 224) | (blk == 0))).all())
    assert _rel(xd, x.float()) < 4e-2
    w8 = F.MXWeight(w)
    y = F.linear_mxf8(x, w8)
    torch.cuda.synchronize()
    ref = xd @ w8.dequantize().t()   # fp32 product of the quantised operands
    assert _rel(y, ref) < 1e-2
    assert _rel(y, x.float() @ w.float().t()) < 6e-2
    # the MX form stays within the error of the exact 1x128 fp32-scale form (K2)
    w8e = F.Fp8Weight(w)
    qe, se = F.quantize_1x128(x)
    ye = F.gemm_fp8(qe, se, w8e.q, w8e.scale)
    ref32 = x.float() @ w.float().t()
    assert _rel(y, ref32) < 1.5 * _rel(ye, ref32) + 1e-3


def test_mxf8_dgrad_e5m2_and_residual():
    from lora_kernel_b200.ops import fp8 as F
    g = torch.Generator(device="cuda").manual_seed(1)
    M, N, K = 512, 768, 1024
    dy = (torch.randn(M, N, device="cuda", generator=g) * 1e-3).bfloat16()
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.05).bfloat16()
    w8 = F.MXWeight(w)
    assert torch.equal(w8.q.t().contiguous(), w8.qt)
    dx = F.linear_dgrad_mxf8(dy, w8)
    torch.cuda.synchronize()
    assert _rel(dx, dy.float() @ w.float()) < 0.1
    x = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    r = torch.randn(M, N, device="cuda", generator=g).bfloat16()
    y = F.linear_mxf8(x, w8, residual=r)
    torch.cuda.synchronize()
    assert _rel(y, x.float() @ w.float().t() + r.float()) < 5e-2


def test_mxf8_many_tiles_persistent():
    """More tiles than SMs: the single accumulator is reused tile after tile."""
    from lora_kernel_b200.ops import fp8 as F
    g = torch.Generator(device="cuda").manual_seed(5)
    M, N, K = 4096, 4096, 1024
    a8, b8 = _rand_fp8(M, K, 0, g), _rand_fp8(N, K, 0, g)
    ea = torch.randint(-3, 4, (M, K // 32), device="cuda", dtype=torch.int32, generator=g)
    eb = torch.randint(-3, 4, (N, K // 32), device="cuda", dtype=torch.int32, generator=g)
    y = F.gemm_mxf8(a8, F.exponents_to_sf(ea, 128), b8, F.exponents_to_sf(eb, 256))
    torch.cuda.synchronize()
    ref = _deq(a8, ea, 0) @ _deq(b8, eb, 0).t()
    assert _rel(y, ref) < 1e-2
