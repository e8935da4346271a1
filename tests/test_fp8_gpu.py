"""K2 block-scaled fp8 GEMM against a plain PyTorch fp32 reference."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm()).item()


@pytest.mark.parametrize("M,N,K", [(256, 256, 512), (300, 384, 1024), (1024, 1536, 2048)])
def test_fp8_gemm_exact_vs_dequantised(M, N, K):
    from lora_kernel_b200.ops import fp8 as F
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.05).bfloat16()
    w8 = F.Fp8Weight(w)
    q, s = F.quantize_1x128(x)
    y = F.gemm_fp8(q, s, w8.q, w8.scale)
    torch.cuda.synchronize()
    ref = F.dequantize_1x128(q, s) @ w8.dequantize().t()   # fp32 product of the quantised operands
    assert _rel(y, ref) < 1e-2
    assert _rel(y, x.float() @ w.float().t()) < 6e-2       # quantisation error vs bf16 operands


def test_fp8_dgrad_e5m2_and_residual():
    from lora_kernel_b200.ops import fp8 as F
    g = torch.Generator(device="cuda").manual_seed(1)
    M, N, K = 512, 768, 1024
    dy = (torch.randn(M, N, device="cuda", generator=g) * 1e-3).bfloat16()
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.05).bfloat16()
    w8 = F.Fp8Weight(w)
    dx = F.linear_dgrad_fp8(dy, w8)
    torch.cuda.synchronize()
    assert _rel(dx, dy.float() @ w.float()) < 0.1
    # residual epilogue, e4m3 activations
    x = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    r = torch.randn(M, N, device="cuda", generator=g).bfloat16()
    y = F.linear_fp8(x, w8, residual=r)
    assert _rel(y, x.float() @ w.float().t() + r.float()) < 5e-2


def test_fp8_weight_transpose_consistent():
    from lora_kernel_b200.ops import fp8 as F
    w = (torch.randn(384, 256, device="cuda") * 0.05).bfloat16()
    w8 = F.Fp8Weight(w)
    assert torch.equal(w8.q.t().contiguous(), w8.qt)
