"""Optimizer-state offload: the streamed AdamW over pinned host state gives
bit-identical results to the device-resident optimizer."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_offloaded_adamw_matches_resident():
    from lora_kernel_b200.train.offload import OffloadedAdamW
    from lora_kernel_b200.train.optimizer import FusedAdamW
    torch.manual_seed(0)
    n = 50_000
    segs = [(0, 30_000, True), (30_016, 19_984, False)]
    master = torch.randn(n)
    kw = dict(lr=1e-2, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1, max_grad_norm=1.0,
              dynamic_loss_scale=True, init_loss_scale=1024.0)
    ref = FusedAdamW(master.cuda(), segs, **kw)
    off = OffloadedAdamW(master, segs, "cuda", chunk_elems=4096, **kw)  # 13 chunks, both buffers
    p16a = master.cuda().bfloat16()
    p16b = p16a.clone()
    for step in range(4):
        g = torch.randn(n, device="cuda") * 1024.0
        if step == 2:
            g[123] = float("inf")  # overflow: both skip and halve the scale
        ref.step(g.clone(), p16a)
        off.step(g.clone(), p16b)
    torch.cuda.synchronize()
    assert torch.equal(ref.p32.cpu(), off.p32)
    assert torch.equal(ref.m.cpu(), off.m) and torch.equal(ref.v.cpu(), off.v)
    assert torch.equal(p16a, p16b)
    assert torch.equal(ref.state, off.state)
    assert off.p32.is_pinned()


def test_pipeline_with_offloaded_optimizer():
    from lora_kernel_b200.config import TrainConfig, TransformerConfig
    from lora_kernel_b200.train.pipeline import Transformer, TrainingPipeline
    cfg = TransformerConfig(hidden_dim=256, num_heads=4, num_kv_heads=2, head_dim=64, ff_dim=512,
                            vocab_size=512, num_layers=2, max_seq_len=128)
    ids = torch.randint(0, 512, (2, 129), generator=torch.Generator().manual_seed(1)).cuda()
    losses = []
    for offload in (False, True):
        tc = TrainConfig(offload_optimizer=offload, seed=4)
        pipe = TrainingPipeline(Transformer(cfg, "cuda", seed=4), 1e-3, 0.1, 1.0, train_cfg=tc)
        losses.append([pipe.train_step(ids[:, :-1], ids[:, 1:]) for _ in range(3)])
    # the loss sum is accumulated with fp32 atomics, so runs agree to rounding only
    for a, b in zip(*losses):
        assert abs(a - b) < 1e-4 * abs(a), losses
