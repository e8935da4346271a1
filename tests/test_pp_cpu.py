"""Pipeline parallelism on CPU: layer partition, the 1F1B schedule (deadlock
freedom and in-flight bound by simulation), and the executor over real gloo
ranks with autograd stages, checked against the unpipelined computation."""
import random

import pytest
import torch

from lora_kernel_b200.config import TransformerConfig
from lora_kernel_b200.parallel.pp import (StageCompute, head_cost_in_layers, partition_layers,
                                          run_schedule, schedule_1f1b, simulate)


def test_partition_covers_layers_and_balances_head():
    for L, P in [(22, 2), (22, 4), (32, 8), (8, 8), (5, 3)]:
        parts = partition_layers(L, P, 0.0)
        assert [i for r in parts for i in r] == list(range(L))
        assert all(len(r) >= 1 for r in parts)
        assert max(len(r) for r in parts) - min(len(r) for r in parts) <= 1
    # a heavy head moves layers off the last stage
    parts = partition_layers(22, 4, 3.0)
    assert len(parts[-1]) < len(parts[0])
    with pytest.raises(ValueError):
        partition_layers(3, 4)
    cfg = TransformerConfig(hidden_dim=4096, num_heads=32, num_kv_heads=8, head_dim=128, ff_dim=14336,
                            vocab_size=128256, num_layers=32)
    assert 1.5 < head_cost_in_layers(cfg) < 3.0


@pytest.mark.parametrize("P", [1, 2, 3, 4, 8])
@pytest.mark.parametrize("M", [1, 2, 3, 5, 8, 16])
def test_1f1b_schedule_is_deadlock_free_and_bounded(P, M):
    r = simulate(P, M)
    for s in range(P):
        sched = schedule_1f1b(P, s, M)
        assert [a for k, a in sched if k == "F"] == list(range(M))
        assert [a for k, a in sched if k == "B"] == list(range(M))
        assert r["peak_inflight"][s] <= min(P - s, M)


def test_schedule_comm_pairs_with_neighbours():
    # forward sends are batched with the matching backward receive
    s = schedule_1f1b(4, 1, 8)
    groups = [a for k, a in s if k == "X" and len(a) == 2]
    assert groups and all({op[1] for op in g} in ({"next"}, {"prev"}) for g in groups)


# ------------------------------------------------------------ gloo ranks
L_TOTAL, D, M, B = 6, 16, 4, 3


def _full_model(seed=0):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(D, D, generator=g) / D ** 0.5 for _ in range(L_TOTAL)]


def _inputs(seed=1):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(B, D, generator=g) for _ in range(M)]


class _AutogradStage(StageCompute):
    def __init__(self, ws, first, last, xs):
        self.ws = [w.clone().requires_grad_(True) for w in ws]
        self.first, self.last, self.xs = first, last, xs
        self.inp = {mb: torch.zeros(B, D) for mb in range(M)}
        self.gin = {mb: torch.zeros(B, D) for mb in range(M)}
        self.out, self.xin, self.loss = {}, {}, 0.0

    def forward(self, mb):
        x = (self.xs[mb] if self.first else self.inp[mb]).clone().requires_grad_(True)
        y = x
        for w in self.ws:
            y = torch.tanh(y @ w)
        self.xin[mb], self.out[mb] = x, y

    def backward(self, mb):
        y = self.out.pop(mb)
        if self.last:
            loss = (y ** 2).sum()
            self.loss += float(loss)
            loss.backward()
        else:
            y.backward(self.gin[mb])

    def act_out(self, mb):
        return self.out[mb].detach().contiguous()

    def act_in(self, mb):
        return self.inp[mb]

    def grad_out(self, mb):
        return self.xin[mb].grad.contiguous()

    def grad_in(self, mb):
        return self.gin[mb]


def _pp_worker(rank, world, port, q):
    import datetime
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        parts = partition_layers(L_TOTAL, world)
        full = _full_model()
        st = _AutogradStage([full[i] for i in parts[rank]], rank == 0, rank == world - 1, _inputs())
        run_schedule(schedule_1f1b(world, rank, M), st, rank - 1 if rank else None,
                     rank + 1 if rank < world - 1 else None)
        # plain lists: a tensor put on an mp queue lives in the child's shared
        # memory, which disappears when the child exits
        grads = {i: w.grad.tolist() for i, w in zip(parts[rank], st.ws)}
        out = [None] * world
        dist.all_gather_object(out, (grads, st.loss))
        if rank == 0:
            q.put(out)
    finally:
        dist.destroy_process_group()


def test_pipeline_executor_matches_unpipelined_on_gloo_ranks():
    import torch.multiprocessing as mp
    world = 3
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = random.randint(20000, 40000)
    ps = [ctx.Process(target=_pp_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    out = q.get(timeout=120)
    for p in ps:
        p.join(timeout=60)
    # reference: all micro-batches through the whole chain, gradients summed
    ws = [w.clone().requires_grad_(True) for w in _full_model()]
    tot = 0.0
    for x in _inputs():
        y = x
        for w in ws:
            y = torch.tanh(y @ w)
        loss = (y ** 2).sum()
        tot += float(loss)
        loss.backward()
    got = {}
    for grads, _ in out:
        got.update(grads)
    assert sorted(got) == list(range(L_TOTAL))
    for i in range(L_TOTAL):
        torch.testing.assert_close(torch.tensor(got[i]), ws[i].grad, rtol=1e-5, atol=1e-6)
    assert abs(out[-1][1] - tot) < 1e-4 * abs(tot)


def test_stage_params_reproduce_full_model_init():
    from lora_kernel_b200.models.params import FlatParams
    cfg = TransformerConfig(hidden_dim=128, num_heads=2, head_dim=64, ff_dim=200, vocab_size=300, num_layers=5)
    full = FlatParams(cfg, "cpu", torch.float32)
    full.init_(7, 0.02)
    ref = full.to_reference_state_dict()
    seen = {}
    for s, r in enumerate(partition_layers(5, 3)):
        p = FlatParams(cfg, "cpu", torch.float32, layers=r, embed=(s == 0), head=(s == 2))
        p.init_(7, 0.02)
        sd = p.to_reference_state_dict()
        assert not set(sd) & set(seen)
        seen.update(sd)
        assert p.like().numel == p.numel and p.like().layer_ids == r
    assert sorted(seen) == sorted(ref)
    for k in ref:
        assert torch.equal(seen[k], ref[k]), k


def test_stage_checkpoint_mapping_roundtrip():
    from lora_kernel_b200.models.params import FlatParams, build_layout
    from lora_kernel_b200.parallel.pp import gather_stage, scatter_stage, stage_global_ranges
    cfg = TransformerConfig(hidden_dim=128, num_heads=2, head_dim=64, ff_dim=200, vocab_size=300, num_layers=5)
    specs, _, total = build_layout(cfg, 64)
    lay = {"total": total, "specs": {s.name: [s.offset, s.numel] for s in specs}}
    full = FlatParams(cfg, "cpu", torch.float32)
    full.flat.copy_(torch.randn(full.numel))
    rebuilt = torch.zeros(total)
    for s, r in enumerate(partition_layers(5, 3)):
        st = FlatParams(cfg, "cpu", torch.float32, layers=r, embed=(s == 0), head=(s == 2))
        rr = stage_global_ranges(st, lay)
        scatter_stage(full.flat, rr, st.flat)
        for sp in st.specs:
            assert torch.equal(st.views[sp.name], full.views[sp.name])
        packed = gather_stage(st.flat, rr)
        o = 0
        for _, g, n in rr:  # what Checkpointer.load_flat reassembles from the saved ranges
            rebuilt[g:g + n] = packed[o:o + n]
            o += n
    mask = torch.zeros(total, dtype=torch.bool)
    for o, n in lay["specs"].values():
        mask[o:o + n] = True
    assert torch.equal(rebuilt[mask], full.flat[mask])
