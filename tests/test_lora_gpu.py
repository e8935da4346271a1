"""LoRA adapters: fused two-segment GEMM, engine gradients vs autograd, merge."""
import pytest
import torch

pytestmark = pytest.mark.gpu
dev = "cuda"


def _close(out, ref, rtol, atol, what=""):
    err = (out.float() - ref.float()).abs()
    bad = (err > atol + rtol * ref.float().abs()).sum().item()
    assert bad == 0, f"{what}: {bad} mismatches, max err {err.max().item():.4g}"


def test_two_segment_gemm():
    from lora_kernel_b200.ops.gemm import gemm
    torch.manual_seed(0)
    M, N, K, r = 300, 384, 512, 16
    x = torch.randn(M, K, device=dev).to(torch.bfloat16)
    W = torch.randn(N, K, device=dev).to(torch.bfloat16)
    u = torch.randn(M, r, device=dev).to(torch.bfloat16)
    B = torch.randn(N, r, device=dev).to(torch.bfloat16)
    out = gemm(x, W, a2=u, b2=B)
    ref = x.float() @ W.float().t() + u.float() @ B.float().t()
    _close(out, ref, 2e-2, 0.5, "fwd")
    # dgrad form: both segments with an MN-major B
    A = torch.randn(r, K, device=dev).to(torch.bfloat16)
    dy = torch.randn(M, N, device=dev).to(torch.bfloat16)
    v = torch.randn(M, r, device=dev).to(torch.bfloat16)
    dx = gemm(dy, W.t(), a2=v, b2=A.t())
    _close(dx, dy.float() @ W.float() + v.float() @ A.float(), 2e-2, 0.5, "dgrad")


def test_lora_engine_grads_match_autograd():
    from lora_kernel_b200.config import TransformerConfig
    from lora_kernel_b200.models.llama import LlamaModel
    from lora_kernel_b200.models.lora import LoRAAdapters, LoRAConfig
    from lora_kernel_b200.oracle import llama_ref
    torch.manual_seed(1)
    cfg = TransformerConfig(hidden_dim=256, num_heads=4, num_kv_heads=2, head_dim=64, ff_dim=384,
                            vocab_size=512, num_layers=2, max_seq_len=256)
    eng = LlamaModel(cfg, dev, seed=2)
    lc = LoRAConfig(rank=16, alpha=32.0)
    ad = LoRAAdapters(cfg, lc, dev)
    with torch.no_grad():  # non-zero B so both adapter gradients are exercised
        for nm, v in ad.views.items():
            if nm.endswith(".B"):
                v.copy_(torch.randn_like(v, dtype=torch.float32) * 0.02)
    eng.lora, eng.train_base = ad, False
    ids = torch.randint(0, cfg.vocab_size, (2, 128), device=dev)
    tgt = torch.randint(0, cfg.vocab_size, (2, 128), device=dev)
    acc = eng.forward_backward(ids, tgt, grad_scale=1.0 / ids.numel(), overwrite_grads=True)
    loss = (acc[0] / acc[1]).item()
    # autograd reference: merged weights W + s B A with A, B as leaves
    base = {k: v.float() for k, v in eng.params.views.items()}
    leaves = {k: v.float().clone().requires_grad_(True) for k, v in ad.views.items()}
    merged = dict(base)
    for i in range(cfg.num_layers):
        for t in lc.targets:
            merged[f"layers.{i}.{t}"] = base[f"layers.{i}.{t}"] + lc.scale * (
                leaves[f"layers.{i}.{t}.B"] @ leaves[f"layers.{i}.{t}.A"])
    ref = llama_ref.loss_fn(merged, cfg, ids, tgt)
    ref.backward()
    assert abs(loss - ref.item()) < 2e-2 * abs(ref.item())
    for k, v in leaves.items():
        err = ((ad.gviews[k] - v.grad).norm() / (v.grad.norm() + 1e-12)).item()
        assert err < 8e-2, (k, err)


def test_lora_finetune_and_merge():
    from lora_kernel_b200.config import TransformerConfig
    from lora_kernel_b200.models.lora import LoRAConfig
    from lora_kernel_b200.train.pipeline import LoRATrainingPipeline, Transformer
    cfg = TransformerConfig(hidden_dim=256, num_heads=4, num_kv_heads=2, head_dim=64, ff_dim=384,
                            vocab_size=512, num_layers=2, max_seq_len=256)
    model = Transformer(cfg, dev, seed=3)
    base_before = model.engine.params.flat.clone()
    pipe = LoRATrainingPipeline(model, LoRAConfig(rank=16, alpha=16.0), lr=5e-3)
    ids = torch.randint(0, cfg.vocab_size, (4, 129), device=dev)
    losses = [pipe.train_step(ids[:, :-1], ids[:, 1:]) for _ in range(25)]
    assert losses[-1] < losses[0] - 0.5, losses
    assert torch.equal(model.engine.params.flat, base_before)  # base frozen
    logits_adapter = model.forward(ids[:, :-1]).float()
    pipe.merge()
    logits_merged = model.forward(ids[:, :-1]).float()
    rel = (logits_adapter - logits_merged).norm() / logits_adapter.norm()
    assert rel < 2e-2, rel
