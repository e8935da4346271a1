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


# ---------------------------------------------------------------- ring attention
def ring_fwd(qkv, Bq, Sq, Hq, Hkv, Dh, causal=True, window=0, out=None, lse=None):
    from lora_kernel_b200.ops.attention import reference_attention
    o, l = reference_attention(qkv, Bq, Sq, Hq, Hkv, Dh, causal=causal, window=window)
    out.copy_(o)
    lse.copy_(l.reshape(lse.shape))
    return out, lse


def ring_bwd(qkv, o, dout, lse, Bq, Sq, Hq, Hkv, Dh, causal=True, window=0, dqkv=None):
    """Block backward from the given (merged) LSE and output, as the K4 kernel
    computes it: P = exp(s - lse), D = rowsum(dO * O)."""
    import math
    q, k, v = _split(qkv.float(), Bq, Sq, Hq, Hkv, Dh)
    g = Hq // Hkv
    q, k, v = (t.permute(0, 2, 1, 3) for t in (q, k, v))              # [B, H, S, Dh]
    k, v = k.repeat_interleave(g, 1), v.repeat_interleave(g, 1)
    do = dout.float().reshape(Bq, Sq, Hq, Dh).permute(0, 2, 1, 3)
    of = o.float().reshape(Bq, Sq, Hq, Dh).permute(0, 2, 1, 3)
    sc = 1.0 / math.sqrt(Dh)
    s = (q @ k.transpose(-1, -2)) * sc
    if causal:
        s = s.masked_fill(torch.ones(Sq, Sq, dtype=torch.bool).triu(1), float("-inf"))
    p = torch.exp(s - lse.reshape(Bq, Hq, Sq, 1))
    dv = p.transpose(-1, -2) @ do
    dp = do @ v.transpose(-1, -2)
    ds = p * (dp - (do * of).sum(-1, keepdim=True))
    dq = ds @ k * sc
    dk = ds.transpose(-1, -2) @ q * sc
    dk = dk.reshape(Bq, Hkv, g, Sq, Dh).sum(2)
    dv = dv.reshape(Bq, Hkv, g, Sq, Dh).sum(2)
    cat = torch.cat([t.permute(0, 2, 1, 3).reshape(Bq * Sq, -1) for t in (dq, dk, dv)], dim=1)
    dqkv.copy_(cat)
    return dqkv


RB, RS = 2, 16


def _ring_worker(rank, world, port, q):
    import datetime
    import torch.distributed as dist
    from lora_kernel_b200.parallel.cp import RingAttention, shard_zigzag
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        g = torch.Generator().manual_seed(1)
        cols = (CFG.num_heads + 2 * CFG.num_kv_heads) * CFG.head_dim
        qkv = torch.randn(RB, RS, cols, generator=g)
        dout = torch.randn(RB, RS, CFG.num_heads * CFG.head_dim, generator=g)
        sl = RS // world
        mine = shard_zigzag(qkv, rank, world).reshape(RB * sl, cols)
        ctx = RingAttention(CFG, None, ring_fwd, ring_bwd)
        pos = ctx.positions(RB, sl, "cpu")
        want_pos = shard_zigzag(torch.arange(RS).repeat(RB, 1), rank, world).reshape(-1)
        assert torch.equal(pos.long(), want_pos), (pos, want_pos)
        out = torch.empty(RB * sl, CFG.num_heads * CFG.head_dim)
        dq = torch.empty(RB * sl, cols)
        for _ in range(2):  # buffers are reused across calls
            ctx.forward(mine, RB, sl, out)
            ctx.backward(shard_zigzag(dout, rank, world).reshape(RB * sl, -1), RB, sl, dq)
        q.put((rank, out.tolist(), dq.tolist()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [1, 2, 4])
def test_ring_attention_matches_full_attention(world):
    """Zigzag ring attention on gloo ranks: outputs and dQKV of every rank's
    tokens equal full-sequence causal attention (GQA: 8 q heads, 4 kv heads,
    more ranks than Ulysses would allow per kv head at 8)."""
    import torch.multiprocessing as mp
    from lora_kernel_b200.parallel.cp import shard_zigzag
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = random.randint(20000, 40000)
    ps = [ctx.Process(target=_ring_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(world))
    for p in ps:
        p.join(timeout=60)
    g = torch.Generator().manual_seed(1)
    H, KV, Dh = CFG.num_heads, CFG.num_kv_heads, CFG.head_dim
    cols = (H + 2 * KV) * Dh
    qkv = torch.randn(RB, RS, cols, generator=g)
    dout = torch.randn(RB, RS, H * Dh, generator=g)
    full_o = torch.empty(RB * RS, H * Dh)
    attn_fwd(qkv.reshape(RB * RS, cols), RB, RS, H, KV, Dh, out=full_o)
    full_dq = torch.empty(RB * RS, cols)
    attn_bwd(qkv.reshape(RB * RS, cols), None, dout.reshape(RB * RS, -1), None, RB, RS, H, KV, Dh, dqkv=full_dq)
    sl = RS // world
    for rank, out, dq in res:
        want_o = shard_zigzag(full_o.view(RB, RS, -1), rank, world).reshape(RB * sl, -1)
        want_d = shard_zigzag(full_dq.view(RB, RS, -1), rank, world).reshape(RB * sl, -1)
        torch.testing.assert_close(torch.tensor(out), want_o, rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(torch.tensor(dq), want_d, rtol=1e-4, atol=1e-5)


def test_zigzag_shards_cover_the_sequence_once():
    from lora_kernel_b200.parallel.cp import shard_zigzag
    x = torch.arange(3 * 24).view(3, 24)
    parts = [shard_zigzag(x, r, 3) for r in range(3)]
    assert sorted(torch.cat(parts, 1)[0].tolist()) == list(range(24))
    # every rank's causal work (sum over its query positions of visible keys) is equal
    work = [int((shard_zigzag(torch.arange(24)[None], r, 3)[0] + 1).sum()) for r in range(3)]
    assert len(set(work)) == 1
    with pytest.raises(ValueError, match="divisible"):
        shard_zigzag(torch.zeros(1, 20), 0, 3)


def test_ring_mode_is_selectable():
    import torch.distributed as dist
    from lora_kernel_b200.parallel import cp
    cfg = TransformerConfig(hidden_dim=64, num_heads=4, num_kv_heads=1, head_dim=16, ff_dim=128, vocab_size=64)
    orig = (dist.get_world_size, dist.get_rank)
    dist.get_world_size, dist.get_rank = (lambda g=None: 2), (lambda g=None: 1)
    try:
        ring = cp.make_context_attention(cfg, "ring", None, attn_fwd, attn_bwd)   # 1 kv head over 2 ranks
        assert isinstance(ring, cp.RingAttention)
        assert ring.rope_args(1, 4, "cpu")["positions"].tolist() == [2, 3, 4, 5]
        with pytest.raises(ValueError, match="unknown"):
            cp.make_context_attention(cfg, "tree", None, attn_fwd, attn_bwd)
    finally:
        dist.get_world_size, dist.get_rank = orig
