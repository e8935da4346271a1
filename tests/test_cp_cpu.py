"""Context parallelism (Ulysses) on CPU: the sequence<->head all-to-all
exchange around attention on gloo ranks reproduces full-sequence attention
and its input gradients, with injected CPU attention functions."""
import random

import pytest
import torch

from lora_kernel_b200.config import TransformerConfig
from lora_kernel_b200.oracle import llama_ref

CFG = TransformerConfig(hidden_dim=128, num_heads=8, num_kv_heads=4, head_dim=16, ff_dim=128,
                        vocab_size=64, num_layers=1, max_seq_len=64)
B, S = 2, 12


def _split(qkv, Bq, Sq, Hq, Hkv, Dh):
    q = qkv[:, :Hq * Dh].reshape(Bq, Sq, Hq, Dh)
    k = qkv[:, Hq * Dh:(Hq + Hkv) * Dh].reshape(Bq, Sq, Hkv, Dh)
    v = qkv[:, (Hq + Hkv) * Dh:].reshape(Bq, Sq, Hkv, Dh)
    return q, k, v


def attn_fwd(qkv, Bq, Sq, Hq, Hkv, Dh, causal=True, window=0, out=None, lse=None):
    q, k, v = _split(qkv, Bq, Sq, Hq, Hkv, Dh)
    out.copy_(llama_ref.attention(q, k, v, causal, window).reshape(Bq * Sq, Hq * Dh))
    return out, lse


def attn_bwd(qkv, o, dout, lse, Bq, Sq, Hq, Hkv, Dh, causal=True, window=0, dqkv=None):
    x = qkv.detach().clone().requires_grad_(True)
    q, k, v = _split(x, Bq, Sq, Hq, Hkv, Dh)
    llama_ref.attention(q, k, v, causal, window).reshape(Bq * Sq, Hq * Dh).backward(dout)
    dqkv.copy_(x.grad)
    return dqkv


def _worker(rank, world, port, q):
    import datetime
    import torch.distributed as dist
    from lora_kernel_b200.parallel.cp import UlyssesAttention, shard_sequence
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        g = torch.Generator().manual_seed(0)
        cols = (CFG.num_heads + 2 * CFG.num_kv_heads) * CFG.head_dim
        qkv = torch.randn(B, S, cols, generator=g)
        dout = torch.randn(B, S, CFG.num_heads * CFG.head_dim, generator=g)
        sl = S // world
        mine = qkv[:, rank * sl:(rank + 1) * sl].reshape(B * sl, cols).contiguous()
        ctx = UlyssesAttention(CFG, None, attn_fwd, attn_bwd)
        out = torch.empty(B * sl, CFG.num_heads * CFG.head_dim)
        ctx.forward(mine, B, sl, out)
        dq = torch.empty(B * sl, cols)
        ctx.backward(dout[:, rank * sl:(rank + 1) * sl].reshape(B * sl, -1).contiguous(), B, sl, dq)
        assert torch.equal(shard_sequence(torch.arange(2 * S).view(2, S), rank, world)[0],
                           torch.arange(rank * sl, (rank + 1) * sl))
        q.put((rank, out.tolist(), dq.tolist()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_ulysses_exchange_matches_full_attention(world):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = random.randint(20000, 40000)
    ps = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(world))
    for p in ps:
        p.join(timeout=60)
    g = torch.Generator().manual_seed(0)
    H, KV, Dh = CFG.num_heads, CFG.num_kv_heads, CFG.head_dim
    cols = (H + 2 * KV) * Dh
    qkv = torch.randn(B, S, cols, generator=g)
    dout = torch.randn(B, S, H * Dh, generator=g)
    full_o = torch.empty(B * S, H * Dh)
    attn_fwd(qkv.reshape(B * S, cols), B, S, H, KV, Dh, out=full_o)
    full_dq = torch.empty(B * S, cols)
    attn_bwd(qkv.reshape(B * S, cols), None, dout.reshape(B * S, -1), None, B, S, H, KV, Dh, dqkv=full_dq)
    sl = S // world
    for rank, out, dq in res:
        want_o = full_o.view(B, S, -1)[:, rank * sl:(rank + 1) * sl].reshape(B * sl, -1)
        want_d = full_dq.view(B, S, -1)[:, rank * sl:(rank + 1) * sl].reshape(B * sl, -1)
        torch.testing.assert_close(torch.tensor(out), want_o, rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(torch.tensor(dq), want_d, rtol=1e-5, atol=1e-5)


def test_head_divisibility_is_checked():
    import torch.distributed as dist
    from lora_kernel_b200.parallel import cp
    cfg = TransformerConfig(hidden_dim=64, num_heads=4, num_kv_heads=1, head_dim=16, ff_dim=128, vocab_size=64)
    orig = (dist.get_world_size, dist.get_rank)
    dist.get_world_size, dist.get_rank = (lambda g=None: 2), (lambda g=None: 0)
    try:
        with pytest.raises(ValueError, match="divisible"):
            cp.UlyssesAttention(cfg, None, attn_fwd, attn_bwd)
    finally:
        dist.get_world_size, dist.get_rank = orig
