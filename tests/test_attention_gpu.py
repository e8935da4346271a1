"""tcgen05 flash attention forward/backward vs an fp32 autograd reference."""
import pytest
import torch

pytestmark = pytest.mark.gpu
dev = "cuda"


def _close(out, ref, rtol, atol, what=""):
    err = (out.float() - ref.float()).abs()
    tol = atol + rtol * ref.float().abs()
    bad = (err > tol).sum().item()
    assert bad == 0, f"{what}: {bad}/{err.numel()} mismatches, max err {err.max().item():.4g}"


def _rel_per_head(out, ref, heads, dh, tol, what=""):
    """Relative L2 error of every head's slice (and of every 64-row block of
    it): an error confined to a few low-magnitude heads or rows would pass a
    check scaled by the whole tensor's maximum, not this one."""
    o = out.float().reshape(out.shape[0], heads, dh)
    r = ref.float().reshape(ref.shape[0], heads, dh)
    for h in range(heads):
        num = (o[:, h] - r[:, h]).norm().item()
        den = r[:, h].norm().item()
        assert num <= tol * den + 1e-6, f"{what} head {h}: relative error {num / max(den, 1e-30):.3g}"
        for b0 in range(0, o.shape[0], 64):
            rb = r[b0:b0 + 64, h]
            dn = rb.norm().item()
            if dn > 1e-3 * den:
                nb = (o[b0:b0 + 64, h] - rb).norm().item()
                assert nb <= 3 * tol * dn, f"{what} head {h} rows {b0}+: relative error {nb / dn:.3g}"


CASES = [
    # B, S, Hq, Hkv, Dh, causal, window
    (1, 128, 1, 1, 64, True, 0),
    (2, 256, 4, 2, 64, True, 0),
    (1, 384, 8, 1, 64, False, 0),
    (2, 200, 4, 4, 64, True, 0),      # ragged sequence length
    (1, 512, 4, 2, 128, True, 0),
    (1, 256, 2, 1, 128, False, 0),
    (1, 512, 2, 1, 64, True, 200),    # sliding window
]


@pytest.mark.parametrize("B,S,Hq,Hkv,Dh,causal,window", CASES)
def test_attention_fwd_bwd(B, S, Hq, Hkv, Dh, causal, window):
    from lora_kernel_b200._ext import check_status
    from lora_kernel_b200.ops.attention import attention_bwd, attention_fwd, reference_attention
    torch.manual_seed(0)
    W = (Hq + 2 * Hkv) * Dh
    qkv = torch.randn(B * S, W, device=dev).to(torch.bfloat16)
    o, lse = attention_fwd(qkv, B, S, Hq, Hkv, Dh, causal=causal, window=window)
    check_status()
    ref_in = qkv.float().requires_grad_(True)
    o_ref, lse_ref = reference_attention(ref_in, B, S, Hq, Hkv, Dh, causal=causal, window=window)
    _close(o, o_ref, 2e-2, 2e-2, "o")
    _close(lse, lse_ref, 1e-3, 1e-3, "lse")
    dout = torch.randn(B * S, Hq * Dh, device=dev).to(torch.bfloat16)
    o_ref.backward(dout.float())
    dqkv = attention_bwd(qkv, o, dout, lse, B, S, Hq, Hkv, Dh, causal=causal, window=window)
    check_status()
    g = ref_in.grad
    scale_ref = g.abs().max().item()
    _close(dqkv[:, :Hq * Dh], g[:, :Hq * Dh], 5e-2, 2e-2 * scale_ref, "dq")
    _close(dqkv[:, Hq * Dh:(Hq + Hkv) * Dh], g[:, Hq * Dh:(Hq + Hkv) * Dh], 5e-2, 2e-2 * scale_ref, "dk")
    _close(dqkv[:, (Hq + Hkv) * Dh:], g[:, (Hq + Hkv) * Dh:], 5e-2, 2e-2 * scale_ref, "dv")
    _rel_per_head(o, o_ref.detach(), Hq, Dh, 1e-2, "o")
    _rel_per_head(dqkv[:, :Hq * Dh], g[:, :Hq * Dh], Hq, Dh, 3e-2, "dq")
    _rel_per_head(dqkv[:, Hq * Dh:(Hq + Hkv) * Dh], g[:, Hq * Dh:(Hq + Hkv) * Dh], Hkv, Dh, 3e-2, "dk")
    _rel_per_head(dqkv[:, (Hq + Hkv) * Dh:], g[:, (Hq + Hkv) * Dh:], Hkv, Dh, 3e-2, "dv")
