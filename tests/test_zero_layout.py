"""ZeRO-3 shard layout (CPU): chunking, round trips, optimizer segments."""
import pytest
import torch

from lora_kernel_b200.config import TransformerConfig
from lora_kernel_b200.parallel.zero import ShardLayout


def _cfg(tie=False):
    return TransformerConfig(hidden_dim=256, num_heads=4, num_kv_heads=2, head_dim=64, ff_dim=688,
                             vocab_size=1000, num_layers=3, tie_embeddings=tie)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
@pytest.mark.parametrize("tie", [False, True])
def test_shard_roundtrip_and_segments(world, tie):
    cfg = _cfg(tie)
    layouts = [ShardLayout(cfg, world, r) for r in range(world)]
    L0 = layouts[0]
    full = torch.arange(L0.total, dtype=torch.float64)
    shards = [L.extract_shard(full) for L in layouts]
    assert all(s.numel() == L0.shard_numel for s in shards)
    assert torch.equal(L0.assemble(shards), full)
    # every parameter element is covered by exactly one rank's optimizer segments
    cover = torch.zeros(L0.total, dtype=torch.int32)
    for r, L in enumerate(layouts):
        for g in L.names:
            a0, n = L.owned(g)
            o = L.shard_off[g]
            for (so, ln, _) in L.shard_segments():
                lo, hi = max(so, o), min(so + ln, o + n)
                if lo < hi:
                    cover[a0 + lo - o:a0 + hi - o] += 1
    for sp in L0.specs:
        assert torch.all(cover[sp.offset:sp.offset + sp.numel] == 1), sp.name
    assert int(cover.sum()) == sum(sp.numel for sp in L0.specs)
    # groups are aligned for equal, 64-element aligned chunks
    for g, (s, e) in L0.groups.items():
        assert (e - s) % (64 * world) == 0 and s % 64 == 0


def _gloo_worker(rank, world, port, q):
    import os
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = _cfg()
        L = ShardLayout(cfg, world, rank)
        torch.manual_seed(0)
        full_params = torch.randn(L.total)
        shard = L.extract_shard(full_params)
        # all-gather of one group through the layout = the group's full slice
        g = "layers.1"
        s, e = L.groups[g]
        o, n = L.shard_off[g], L.chunk[g]
        out = torch.empty(n * world)
        dist.all_gather_into_tensor(out, shard[o:o + n].contiguous())
        ok_gather = torch.equal(out, full_params[s:e])
        # reduce-scatter of per-rank gradients through the layout
        grads = torch.full((L.total,), float(rank + 1))
        mine = torch.empty(n)
        dist.reduce_scatter_tensor(mine, grads[s:e].contiguous())
        ok_rs = torch.allclose(mine, torch.full((n,), world * (world + 1) / 2.0))
        q.put((rank, ok_gather, ok_rs))
    finally:
        dist.destroy_process_group()


def test_layout_collectives_gloo():
    import random
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    world, port = 2, random.randint(20000, 40000)
    ps = [ctx.Process(target=_gloo_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in ps:
        p.join(timeout=60)
    assert all(ok_g and ok_r for _, ok_g, ok_r in res), res


def test_tp_layout_shard_roundtrip():
    """Every rank's TP shard of the seeded weights reassembles the full tensors."""
    from lora_kernel_b200.models.params import FlatParams
    from lora_kernel_b200.parallel import tp as TP
    cfg = TransformerConfig(hidden_dim=256, num_heads=4, num_kv_heads=2, head_dim=64, ff_dim=512,
                            vocab_size=1024, num_layers=2, max_seq_len=256)
    full = FlatParams(cfg, "cpu", torch.float32)
    full.init_(5, 0.02)
    for tp in (1, 2):
        shards = [TP.TPParams(cfg, tp, r, "cpu", torch.float32) for r in range(tp)]
        for s in shards:
            s.init_(5, 0.02)
        for sp in shards[0].specs:
            rec = TP.unshard_tensor(cfg, sp.name, [s[sp.name] for s in shards])
            assert torch.equal(rec, full[sp.name]), sp.name
        # replicated tensors come first and are contiguous
        assert all(s.group == "replicated" for s in shards[0].specs if s.offset < shards[0].n_rep)


def test_tp_config_checks():
    from lora_kernel_b200.parallel import tp as TP
    cfg = TransformerConfig(hidden_dim=256, num_heads=4, num_kv_heads=2, head_dim=64, ff_dim=512,
                            vocab_size=1024, num_layers=2)
    TP.check_tp_config(cfg, 2)
    with pytest.raises(ValueError):
        TP.check_tp_config(cfg, 4)  # 2 KV heads cannot split 4 ways


def test_dp_shard_to_flat_deltas():
    """The sharded AdamW writes master element o of a rank's shard to flat element
    o + delta of its chunk: every owned parameter piece maps back onto itself."""
    from lora_kernel_b200.ops.optim import make_chunks
    cfg = TransformerConfig(hidden_dim=256, num_heads=4, num_kv_heads=2, head_dim=64, ff_dim=512,
                            vocab_size=512, num_layers=3)
    for world in (2, 4):
        for rank in range(world):
            L = ShardLayout(cfg, world, rank)
            flat = torch.arange(L.total, dtype=torch.float64)
            shard = L.extract_shard(flat)
            segs = []
            for s_off, n, decay in L.shard_segments():
                g = next(g for g in L.names if L.shard_off[g] <= s_off < L.shard_off[g] + L.chunk[g])
                a0, _ = L.owned(g)
                segs.append((s_off, n, decay, a0 - L.shard_off[g]))
            ch = make_chunks(segs, chunk=97)
            for start, length, _, d64 in ch.tolist():
                assert torch.equal(shard[start:start + length], flat[start + 64 * d64:start + 64 * d64 + length])


def test_vocab_parallel_pick_matches_global_argmax():
    from lora_kernel_b200.serve.tp_runner import pick_global
    g = torch.Generator().manual_seed(0)
    V, ranks, rows = 64, 4, 5
    scores = torch.randn(rows, V, generator=g).to(torch.bfloat16).float()
    scores[2, 10] = scores[2, 40] = scores[2].max() + 1  # a tie across slices
    Vl = V // ranks
    allp = torch.empty(ranks, rows, 2, dtype=torch.float64)
    for r in range(ranks):
        sl = scores[:, r * Vl:(r + 1) * Vl]
        v, i = sl.max(1)  # first maximum inside the slice
        allp[r, :, 0] = v.double()
        allp[r, :, 1] = (i + r * Vl).double()
    assert pick_global(allp).tolist() == scores.argmax(1).tolist()
    assert pick_global(allp)[2].item() == 10


@pytest.mark.parametrize("preset", ["llama-1.1b-zero3", "llama-8b-fsdp-dp8"])
def test_zero3_gradient_memory_is_a_shard_plus_slots(preset):
    """With bf16 gradients on the wire a rank holds its fp32 gradient shard,
    three bf16 layer slots, the bf16 head and the fp32 embedding gradient -
    a fraction of the full fp32 gradient buffer of the fp32 wire."""
    from lora_kernel_b200.config import get_preset
    from lora_kernel_b200.parallel.zero import ShardLayout, Zero3Trainer
    cfg = get_preset(preset).model
    L = ShardLayout(cfg, 8, 0)
    full = sum(Zero3Trainer.grad_memory_plan(L, "fp32").values()) - 4 * L.shard_numel
    plan = Zero3Trainer.grad_memory_plan(L, "bf16")
    assert plan["shard_fp32"] == 4 * L.shard_numel
    assert sum(plan.values()) < 0.35 * full, (plan, full)
