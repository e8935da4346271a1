"""Top-k gradient compression with error feedback and the hierarchical
all-reduce, on gloo ranks (CPU)."""
import random

import pytest
import torch

from lora_kernel_b200.parallel.compression import TopKCompressor


def test_topk_indices_cover_large_tensors_and_error_feedback():
    n = 100_000  # indices far beyond 256 (the reference's int8 indices wrap)
    g = torch.zeros(n)
    g[[5, 70_000, 99_999]] = torch.tensor([3.0, -4.0, 2.0])
    c = TopKCompressor(3 / n)
    idx, vals = c.compress(g)
    assert sorted(idx.tolist()) == [5, 70_000, 99_999]
    assert torch.equal(TopKCompressor.decompress(idx, vals, n), g)
    # error feedback: the sum of everything sent converges to the sum of the gradients
    torch.manual_seed(0)
    c = TopKCompressor(0.05)
    sent = torch.zeros(2000)
    total = torch.zeros(2000)
    for _ in range(200):
        x = torch.randn(2000)
        total += x
        i, v = c.compress(x)
        sent += TopKCompressor.decompress(i, v, 2000)
    assert torch.allclose(sent + c.residual, total, atol=1e-3)
    assert (total - sent).abs().max() < 10.0


def _worker(rank, world, port, q):
    import datetime
    import torch.distributed as dist
    from lora_kernel_b200.parallel.compression import HierarchicalAllReduce, TopKCompressor, compressed_all_reduce
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        g = torch.Generator().manual_seed(rank)
        x = torch.randn(1001, generator=g)
        exact = x.clone()
        dist.all_reduce(exact)
        h = HierarchicalAllReduce(2)
        y = x.clone().view(7, 143)
        h(y)
        full = x.clone()
        compressed_all_reduce(full, TopKCompressor(1.0), average=False)
        part = x.clone()
        compressed_all_reduce(part, TopKCompressor(0.1), average=True)
        q.put((rank, (y.reshape(-1) - exact).abs().max().item(), (full - exact).abs().max().item(),
               int((part != 0).sum())))
    finally:
        dist.destroy_process_group()


def test_hierarchical_and_compressed_all_reduce_on_gloo():
    import torch.multiprocessing as mp
    world = 4
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = random.randint(20000, 40000)
    ps = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in ps:
        p.join(timeout=60)
    for rank, h_err, c_err, nnz in res:
        assert h_err < 1e-5 and c_err < 1e-5, (rank, h_err, c_err)
        assert 0 < nnz <= world * 100  # at most k = 100 entries from each rank
    with pytest.raises(ValueError):
        TopKCompressor(0.0)
