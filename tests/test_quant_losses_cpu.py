"""Quantisation algorithms, losses, model utilities, attention variants (CPU)."""
import math

import pytest
import torch

from lora_kernel_b200.quant import algorithms as Q


def test_int8_fp8_int4_roundtrips():
    torch.manual_seed(0)
    w = torch.randn(64, 256)
    q, s = Q.quantize_int8(w)
    assert (Q.dequantize_int8(q, s) - w).abs().max() <= s.max() * 0.5 + 1e-6
    for fmt in ("e4m3", "e5m2"):
        qf, sf = Q.quantize_fp8(w, fmt, per_row=True)
        rel = ((Q.dequantize_fp8(qf, sf) - w).abs() / (w.abs() + 1e-3)).median()
        assert rel < (0.04 if fmt == "e4m3" else 0.08)
    qb, sb = Q.quantize_fp8(w, "e4m3", block=128)
    assert sb.shape == (64, 2)
    assert (Q.dequantize_fp8(qb, sb, block=128) - w).abs().max() < 0.3
    c, sc, z = Q.quantize_int4_groupwise(w, 128)
    assert c.max() <= 15 and torch.equal(Q.unpack_int4(Q.pack_int4(c)), c)
    err = (Q.dequantize_int4_groupwise(c, sc, z, 128) - w).abs()
    assert torch.all(err <= sc.repeat_interleave(128, 1) * 0.5 + 1e-5)


def test_static_quantizer_and_kv_reference():
    sq = Q.StaticQuantizer()
    for _ in range(3):
        sq.observe(torch.randn(100) * 2)
    x = torch.randn(100)
    assert (sq.dequantize(sq.quantize(x)) - x).abs().max() <= sq.scale
    kv = torch.randn(10, 2, 64)
    codes, scale = Q.kv_quantize_reference(kv, "int8")
    assert codes.dtype == torch.int8 and scale.shape == (10, 2)


def test_smoothquant_preserves_output():
    torch.manual_seed(1)
    x = torch.randn(32, 128)
    x[:, 3] *= 50  # an outlier channel
    w = torch.randn(64, 128)
    s = Q.smoothquant_scales(x.abs().amax(0), w, 0.5)
    y = (x / s) @ Q.apply_smoothquant(w, s).t()
    assert torch.allclose(y, x @ w.t(), rtol=1e-4, atol=1e-3)
    assert (x / s).abs().amax(0)[3] < x.abs().amax(0)[3]


def _rtn_err(w, x, group=128):
    c, s, z = Q.quantize_int4_groupwise(w, group)
    return float((x @ Q.dequantize_int4_groupwise(c, s, z, group).t() - x @ w.t()).pow(2).mean())


def test_gptq_and_awq_beat_round_to_nearest():
    torch.manual_seed(2)
    K, N = 256, 64
    x = torch.randn(512, K) @ torch.randn(K, K) * 0.1  # correlated activations
    x[:, :8] *= 10
    w = torch.randn(N, K) * 0.05
    base = _rtn_err(w, x)
    c, s, z = Q.gptq_quantize(w, x, bits=4, group=128, block=128)
    err_g = float((x @ Q.dequantize_int4_groupwise(c.long(), s, z, 128).t() - x @ w.t()).pow(2).mean())
    assert err_g < base
    scales, a = Q.awq_search(w, x, group=128)
    c2, s2, z2 = Q.quantize_int4_groupwise(w * scales[None], 128)
    wq = Q.dequantize_int4_groupwise(c2, s2, z2, 128) / scales[None]
    err_a = float((x @ wq.t() - x @ w.t()).pow(2).mean())
    assert err_a <= base + 1e-12


def test_qat_straight_through():
    lin = Q.QATLinear(16, 8, w_bits=4, a_bits=8)
    x = torch.randn(4, 16, requires_grad=True)
    lin(x).sum().backward()
    assert x.grad is not None and lin.linear.weight.grad is not None
    assert torch.count_nonzero(lin.linear.weight.grad) > 0


def test_losses():
    from lora_kernel_b200.train import losses as L
    torch.manual_seed(3)
    s = torch.randn(4, 10, requires_grad=True)
    t = torch.randn(4, 10)
    kd = L.distillation_loss(s, s.detach(), temperature=2.0)
    assert abs(float(kd)) < 1e-6
    L.distillation_loss(s, t, torch.randint(0, 10, (4,)), 2.0, 0.5).backward()
    assert s.grad is not None
    lp_old = torch.randn(8)
    lp_new = (lp_old + 0.5).requires_grad_(True)
    adv = torch.ones(8)
    loss = L.ppo_loss(lp_new, lp_old, adv, clip_eps=0.2)
    assert abs(float(loss) + 1.2) < 1e-5  # ratio clipped at 1 + eps
    r = torch.tensor([1.0, 2.0, 3.0, 0.0, 0.0, 6.0])
    a = L.grpo_advantages(r, 3)
    assert torch.allclose(a.view(2, 3).mean(1), torch.zeros(2), atol=1e-6)
    g = L.grpo_loss(torch.zeros(6, requires_grad=True), torch.zeros(6), torch.zeros(6), r, 3)
    assert g.requires_grad


def test_merging_pruning():
    from lora_kernel_b200.utils import model_ops as M
    base = {"w": torch.zeros(100)}
    f1 = {"w": torch.linspace(-1, 1, 100)}
    f2 = {"w": torch.linspace(-1, 1, 100) * 2}
    assert torch.allclose(M.linear_merge([f1, f2], [1, 1])["w"], 1.5 * f1["w"])
    assert torch.allclose(M.task_arithmetic(base, [f1, f2], 0.5)["w"], 1.5 * f1["w"])
    t = M.ties_merge(base, [f1, f2], density=0.2)["w"]
    assert torch.count_nonzero(t) <= 40 and t[-1] > 0
    w = torch.randn(10, 10)
    p = M.prune_magnitude(w, 0.5)
    assert torch.count_nonzero(p) == 50
    r = M.prune_structured_rows(w, 0.3)
    assert int((r.abs().sum(1) == 0).sum()) == 3


def test_attention_variants():
    from lora_kernel_b200.oracle import attention_variants as A
    torch.manual_seed(4)
    q = torch.randn(1, 4, 16, 8)
    k = torch.randn(1, 2, 16, 8)
    v = torch.randn(1, 2, 16, 8)
    o = A.attention(q, k, v, mask=A.causal_mask(16, 16))
    ref = torch.nn.functional.scaled_dot_product_attention(q, k.repeat_interleave(2, 1), v.repeat_interleave(2, 1),
                                                           is_causal=True)
    assert torch.allclose(o, ref, atol=1e-5)
    assert A.sliding_window_mask(8, 2)[5].tolist() == [True] * 4 + [False, False] + [True] * 2
    assert A.dilated_mask(8, 2)[6, 4] == False and A.dilated_mask(8, 2)[6, 5] == True
    b = A.alibi_bias(4, 8)
    assert b.shape == (4, 8, 8) and float(b[0, 3, 3]) == 0.0
    assert A.RelativePositionBias(4)(8).shape == (4, 8, 8)
    lo = A.linear_attention(q, k, v, causal=True)
    assert lo.shape == (1, 4, 16, 8) and torch.isfinite(lo).all()
    # block-sparse: a band covering every block is plain causal attention
    assert torch.equal(A.block_sparse_mask(16, 4, local_blocks=4), A.causal_mask(16, 16))
    m = A.block_sparse_mask(16, 4, local_blocks=1, stride=2)
    assert not m[13, 12] and m[13, 8] and not m[13, 5] and m[13, 14] and m[2, 3]   # band, strided summary, causal
    # hybrid: local heads see the window, global heads everything before them
    hy = A.hybrid_attention(q, k, v, local_heads=2, window=3)
    loc = A.attention(q, k, v, mask=A.sliding_window_mask(16, 3))
    assert torch.allclose(hy[:, :2], loc[:, :2], atol=1e-6) and torch.allclose(hy[:, 2:], o[:, 2:], atol=1e-6)
    assert torch.allclose(A.hybrid_attention(q, k, v, 4, 16), o, atol=1e-6)


def test_quantized_checkpoint_roundtrip(tmp_path):
    """qweight / scales / zeros + bf16 tensors survive a safetensors round trip."""
    from lora_kernel_b200.ops.serving import QuantizedWeight
    from lora_kernel_b200.quant.io import load_quantized, save_quantized
    g = torch.Generator().manual_seed(0)
    w4 = QuantizedWeight.from_parts("int4", 128, 64, 256, torch.randint(0, 255, (64, 128), dtype=torch.uint8, generator=g),
                                    torch.rand(64, 2, generator=g), torch.rand(64, 2, generator=g))
    w8 = QuantizedWeight.from_parts("int8", 128, 32, 256, torch.randint(-127, 127, (32, 256), dtype=torch.int8, generator=g),
                                    torch.rand(32, generator=g))
    emb = torch.randn(10, 4, generator=g).bfloat16()
    path = str(tmp_path / "q.safetensors")
    save_quantized({"layers.0.wqkv": w4, "layers.0.wo": w8, "embed": emb, "lm_head": emb}, path)
    back = load_quantized(path, device="cpu")
    assert back["layers.0.wqkv"].fmt == "int4" and back["layers.0.wqkv"].N == 64 and back["layers.0.wqkv"].K == 256
    assert torch.equal(back["layers.0.wqkv"].q, w4.q) and torch.equal(back["layers.0.wqkv"].zero, w4.zero)
    assert back["layers.0.wo"].zero is None and torch.equal(back["layers.0.wo"].scale, w8.scale)
    assert torch.equal(back["embed"], emb) and back["lm_head"] is back["embed"]


def _pack_int32(nibbles):
    """[..., 8] codes 0..15 -> int32 words, nibble i at bits 4i (wrapping as int32)."""
    import numpy as np
    w = np.zeros(nibbles.shape[:-1], dtype=np.uint64)
    for i in range(8):
        w |= nibbles[..., i].astype(np.uint64) << np.uint64(4 * i)
    return torch.from_numpy(w.astype(np.uint32).view(np.int32))


def test_gptq_and_awq_unpacking():
    """Codes, zero points and scales packed the GPTQ way (codes along K,
    zeros minus one along N) and the AWQ way (codes along N in the order
    0,2,4,6,1,3,5,7) come back as [N, K] codes with per-group scales/zeros."""
    import numpy as np
    from lora_kernel_b200.quant.gptq_awq import AWQ_ORDER, pack_nibbles, unpack_awq, unpack_gptq
    rng = np.random.default_rng(0)
    K, N, G = 256, 64, 128
    codes = rng.integers(0, 16, (K, N))
    zeros = rng.integers(1, 16, (K // G, N))
    scales = torch.from_numpy(rng.random((K // G, N)).astype(np.float16))
    want = torch.from_numpy((codes - np.repeat(zeros, G, 0)).astype(np.float32)).t() * \
        scales.float().repeat_interleave(G, 0).t()
    # GPTQ
    qweight = _pack_int32(codes.reshape(K // 8, 8, N).transpose(0, 2, 1))
    qzeros = _pack_int32((zeros - 1).reshape(K // G, N // 8, 8))
    p = unpack_gptq(qweight, qzeros, scales, torch.arange(K, dtype=torch.int32) // G)
    assert torch.equal(p.q.long(), torch.from_numpy(codes).t()) and p.group == G
    assert torch.allclose(p.dequantize(), want)
    with pytest.raises(NotImplementedError):
        unpack_gptq(qweight, qzeros, scales, torch.randperm(K) // G)
    # AWQ
    order = list(AWQ_ORDER)
    qweight = _pack_int32(codes.reshape(K, N // 8, 8)[..., order])
    qzeros = _pack_int32(zeros.reshape(K // G, N // 8, 8)[..., order])
    a = unpack_awq(qweight, qzeros, scales)
    assert torch.equal(a.q.long(), torch.from_numpy(codes).t()) and torch.allclose(a.dequantize(), want)
    # two codes per byte, the even column in the low nibble (the int4 kernels' layout)
    pk = pack_nibbles(p.q)
    assert pk.shape == (N, K // 2) and int(pk[3, 5]) == int(p.q[3, 10]) | (int(p.q[3, 11]) << 4)


def test_llama_gptq_parts_map_to_the_engine_layout():
    from lora_kernel_b200.config import TransformerConfig
    from lora_kernel_b200.ops.gemm import split_gate_up
    from lora_kernel_b200.quant.gptq_awq import Int4Parts, llama_parts_to_engine
    from lora_kernel_b200.utils.export import _interleaved_to_half
    cfg = TransformerConfig(hidden_dim=128, num_heads=4, num_kv_heads=2, head_dim=32, ff_dim=256,
                            vocab_size=64, num_layers=1)
    g = torch.Generator().manual_seed(1)

    def rand(n, k):
        return Int4Parts(torch.randint(0, 16, (n, k), generator=g, dtype=torch.uint8),
                         torch.rand(n, k // 128, generator=g), torch.randint(0, 16, (n, k // 128), generator=g).float(),
                         128)
    p = "model.layers.0."
    parts = {p + "self_attn.q_proj": rand(128, 128), p + "self_attn.k_proj": rand(64, 128),
             p + "self_attn.v_proj": rand(64, 128), p + "self_attn.o_proj": rand(128, 128),
             p + "mlp.gate_proj": rand(256, 128), p + "mlp.up_proj": rand(256, 128),
             p + "mlp.down_proj": rand(128, 256)}
    e = llama_parts_to_engine(parts, cfg)
    qkv = e["layers.0.wqkv"].dequantize()
    assert torch.equal(_interleaved_to_half(qkv[:128], 4, 32), parts[p + "self_attn.q_proj"].dequantize())
    assert torch.equal(_interleaved_to_half(qkv[128:192], 2, 32), parts[p + "self_attn.k_proj"].dequantize())
    assert torch.equal(qkv[192:], parts[p + "self_attn.v_proj"].dequantize())
    gate, up = split_gate_up(e["layers.0.wgu"].dequantize())
    assert torch.equal(gate, parts[p + "mlp.gate_proj"].dequantize())
    assert torch.equal(up, parts[p + "mlp.up_proj"].dequantize())
    assert e["layers.0.wdown"] is parts[p + "mlp.down_proj"]


def test_lora_file_round_trip(tmp_path):
    from lora_kernel_b200.config import TransformerConfig
    from lora_kernel_b200.models.lora import LoRAAdapters, LoRAConfig, load_lora_file, save_lora_file
    cfg = TransformerConfig(hidden_dim=128, num_heads=4, num_kv_heads=2, head_dim=32, ff_dim=256,
                            vocab_size=64, num_layers=2)
    ad = LoRAAdapters(cfg, LoRAConfig(rank=8, alpha=4.0, targets=("wqkv", "wdown"), init_seed=3), "cpu",
                      torch.float32)
    g = torch.Generator().manual_seed(0)
    for v in ad.state_dict().values():
        v.copy_(torch.randn(v.shape, generator=g))
    path = str(tmp_path / "lora_step_7.safetensors")
    save_lora_file(ad, path, 7)
    back = load_lora_file(path, cfg, "cpu")
    assert (back.lc.rank, back.lc.alpha, back.lc.targets) == (8, 4.0, ("wqkv", "wdown"))
    for k, v in ad.state_dict().items():
        torch.testing.assert_close(back.state_dict()[k].float(), v.float(), rtol=1e-2, atol=1e-2)


def test_lora_merge_into_state_dict_matches_the_adapted_forward():
    """Folding the adapters into the weights gives the logits of the base model
    run with W + (alpha/r) B A."""
    from lora_kernel_b200.config import TransformerConfig
    from lora_kernel_b200.models.lora import LoRAAdapters, LoRAConfig, merge_lora_state_dict
    from lora_kernel_b200.models.params import FlatParams
    from lora_kernel_b200.oracle import llama_ref
    cfg = TransformerConfig(hidden_dim=128, num_heads=4, num_kv_heads=2, head_dim=32, ff_dim=256,
                            vocab_size=64, num_layers=1)
    base = FlatParams(cfg, "cpu", torch.float32)
    base.init_(2, 0.05)
    ad = LoRAAdapters(cfg, LoRAConfig(rank=8, alpha=16.0, targets=("wqkv", "wgu")), "cpu", torch.float32)
    g = torch.Generator().manual_seed(1)
    for v in ad.state_dict().values():
        v.copy_(torch.randn(v.shape, generator=g) * 0.05)
    merged = FlatParams(cfg, "cpu", torch.float32)
    merged.load_reference_state_dict(merge_lora_state_dict(base.to_reference_state_dict(), ad))
    want = {k: v.clone() for k, v in base.views.items()}
    for t in ("wqkv", "wgu"):
        want[f"layers.0.{t}"] += 2.0 * ad.B(0, t) @ ad.A(0, t)
    ids = torch.randint(0, 64, (2, 9), generator=g)
    torch.testing.assert_close(llama_ref.forward(dict(merged.views), cfg, ids), llama_ref.forward(want, cfg, ids),
                               rtol=1e-5, atol=1e-5)


def test_conv_bn_fusion_matches_conv_then_batch_norm():
    from lora_kernel_b200.utils.model_ops import fuse_conv_bn
    torch.manual_seed(0)
    conv = torch.nn.Conv2d(6, 8, 3, padding=1)
    bn = torch.nn.BatchNorm2d(8, eps=1e-5).eval()
    bn.running_mean.uniform_(-1, 1)
    bn.running_var.uniform_(0.5, 2.0)
    bn.weight.data.uniform_(0.5, 1.5)
    bn.bias.data.uniform_(-0.5, 0.5)
    x = torch.randn(2, 6, 9, 9)
    with torch.no_grad():
        want = bn(conv(x))
        w, b = fuse_conv_bn(conv.weight, conv.bias, bn.weight, bn.bias, bn.running_mean, bn.running_var, 1e-5)
        got = torch.nn.functional.conv2d(x, w, b, padding=1)
    assert torch.allclose(got, want, atol=1e-5, rtol=1e-5)
    # a linear layer without bias folds the same way
    lin = torch.nn.Linear(5, 4, bias=False)
    bn1 = torch.nn.BatchNorm1d(4).eval()
    bn1.running_mean.uniform_(-1, 1)
    w, b = fuse_conv_bn(lin.weight, None, bn1.weight, bn1.bias, bn1.running_mean, bn1.running_var)
    z = torch.randn(3, 5)
    with torch.no_grad():
        assert torch.allclose(torch.nn.functional.linear(z, w, b), bn1(lin(z)), atol=1e-5)


def test_mx_scale_tiles_round_trip_cpu():
    """The SF-tile layout helpers: exponents -> tiles -> exponents is exact, and a
    row's four 32-wide blocks of one 128 block sit in one 4-byte word."""
    import torch
    from lora_kernel_b200.ops import fp8 as F
    g = torch.Generator().manual_seed(0)
    for rows, K, mult in [(128, 128, 128), (200, 512, 128), (300, 256, 256)]:
        e = torch.randint(-20, 21, (rows, K // 32), generator=g, dtype=torch.int32)
        sf = F.exponents_to_sf(e, mult)
        assert sf.numel() == F.sf_tile_bytes(rows, K, mult)
        assert torch.equal(F.sf_to_exponents(sf, rows, K), e)
    idx = F._sf_index(256, 256, "cpu")
    assert idx[37, 5].item() == ((0 * 2 + 1) * 512 + 5 * 16 + 1 * 4 + 1)
    assert idx[200, 0].item() == ((1 * 2 + 0) * 512 + 8 * 16 + 2 * 4 + 0)
