"""Failure detection (gloo / TCPStore ranks on CPU) and checkpoint logic."""
import json
import os
import random
import time

import pytest
import torch

from lora_kernel_b200.config import TransformerConfig
from lora_kernel_b200.parallel.fault import FaultInjector, HeartbeatMonitor, RankFailure, parse_faults


def test_parse_faults():
    f = parse_faults("kill_rank:3@step:7, delay_rank:1@step:2:0.5,nan_grad@step:4")
    assert [(x.kind, x.rank, x.step, x.arg) for x in f] == [
        ("kill_rank", 3, 7, 0.0), ("delay_rank", 1, 2, 0.5), ("nan_grad", -1, 4, 0.0)]
    fi = FaultInjector(0, "raise_rank:0@step:2,nan_grad@step:1")
    fi.at_step(1)
    g = torch.zeros(4)
    fi.on_grads(1, g)
    assert torch.isnan(g).all()
    with pytest.raises(RuntimeError):
        fi.at_step(2)


def test_kill_rank_is_refused_when_nvlink_multicast_is_possible(monkeypatch):
    """Killing a rank is allowed on CPU / gloo jobs; on an NCCL job only with
    multicast off in this library and in NCCL."""
    import torch.distributed as dist
    from lora_kernel_b200.parallel import fault
    FaultInjector(0, "kill_rank:1@step:3")  # no process group: allowed
    monkeypatch.setattr(dist, "is_initialized", lambda: True)
    monkeypatch.setattr(dist, "get_backend", lambda *a: "nccl")
    monkeypatch.delenv("LK_NVLS", raising=False)
    monkeypatch.delenv("NCCL_NVLS_ENABLE", raising=False)
    with pytest.raises(ValueError, match="LK_NVLS=0"):
        FaultInjector(0, "kill_rank:1@step:3")
    FaultInjector(0, "raise_rank:1@step:3")  # other faults stay available
    monkeypatch.setenv("LK_NVLS", "0")
    with pytest.raises(ValueError):
        FaultInjector(0, "kill_rank:1@step:3")
    monkeypatch.setenv("NCCL_NVLS_ENABLE", "0")
    assert fault.kill_is_safe()[0]
    FaultInjector(0, "kill_rank:1@step:3")
    monkeypatch.setattr(dist, "get_backend", lambda *a: "gloo")
    monkeypatch.delenv("LK_NVLS")
    assert fault.kill_is_safe()[0]


def _hb_worker(rank, world, port, q):
    from torch.distributed import TCPStore
    store = TCPStore("127.0.0.1", port, world, is_master=(rank == 0), timeout=__import__("datetime").timedelta(seconds=30))
    hb = HeartbeatMonitor(store, rank, world, interval_s=0.1, timeout_s=1.0)
    time.sleep(0.5)
    if rank == 1:
        os._exit(0)  # the rank dies without warning (store stays up on rank 0)
    hb.check()  # everyone alive so far
    deadline = time.time() + 10
    found = None
    while time.time() < deadline:
        try:
            hb.check()
        except RankFailure as e:
            found = e.ranks
            break
        time.sleep(0.1)
    q.put(found)


def test_heartbeat_detects_dead_rank():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = random.randint(20000, 40000)
    ps = [ctx.Process(target=_hb_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    found = q.get(timeout=60)
    for p in ps:
        p.join(timeout=30)
    assert found == [1]


def test_checkpoint_roundtrip_and_reshard(tmp_path):
    from lora_kernel_b200.parallel.zero import ShardLayout
    from lora_kernel_b200.train.checkpoint import Checkpointer, latest
    from lora_kernel_b200.train.trainer import _layout_info, remap_flat
    cfg = TransformerConfig(hidden_dim=128, num_heads=2, head_dim=64, ff_dim=256, vocab_size=300, num_layers=2)
    # a "2-rank" ZeRO checkpoint written rank by rank
    world = 2
    L0 = ShardLayout(cfg, world, 0)
    lay = _layout_info(cfg, L0.align)
    full = torch.randn(L0.total)
    for r in range(world):
        L = ShardLayout(cfg, world, r)
        ck = Checkpointer(str(tmp_path), r, world)
        shard = L.extract_shard(full)
        ranges = [(L.owned(g)[0], L.owned(g)[0] + L.chunk[g]) for g in L.names]
        if r == world - 1:
            ck.save(5, None, ranges, {"p32": shard, "m": shard * 2, "v": shard * 3, "state": torch.arange(16.)},
                    lay, {"step": 5})
        else:  # the non-final rank only writes its file (rank 0 publishes)
            import threading
            os.makedirs(os.path.join(tmp_path, "step_5.tmp"), exist_ok=True)
            from safetensors.torch import save_file
            save_file({"p32": shard, "m": shard * 2, "v": shard * 3, "state": torch.arange(16.)},
                      os.path.join(tmp_path, "step_5.tmp", f"optim-rank{r}-of-{world}.safetensors"),
                      metadata={"ranges": json.dumps(ranges)})
    # rank 1 (non-zero) does not publish; publish as rank 0 would
    ck0 = Checkpointer(str(tmp_path), 0, world)
    ck0._pending = (str(tmp_path / "step_5.tmp"), str(tmp_path / "step_5"), 5, lay, {"step": 5})
    ck0.finish()
    p = latest(str(tmp_path))
    assert p.endswith("step_5") and Checkpointer.verify(p)
    flat = Checkpointer.load_flat(p)
    # padding between groups is not covered by any shard; parameters must match exactly
    one = _layout_info(cfg, 64)
    a = remap_flat(flat["p32"], lay, one)
    b = remap_flat(full, lay, one)
    assert torch.equal(a, b)
    assert torch.equal(remap_flat(flat["m"], lay, one), 2 * b)
    assert Checkpointer.trainer_state(p)["step"] == 5


def test_model_safetensors_reference_names(tmp_path):
    from lora_kernel_b200.models.params import FlatParams
    from lora_kernel_b200.train.checkpoint import load_model_safetensors, save_model_safetensors
    cfg = TransformerConfig(hidden_dim=128, num_heads=2, head_dim=64, ff_dim=200, vocab_size=300, num_layers=2)
    p = FlatParams(cfg, "cpu", torch.float32)
    p.init_(0, 0.02)
    path = str(tmp_path / "model.safetensors")
    save_model_safetensors(p.to_reference_state_dict(), path)
    sd = load_model_safetensors(path)
    assert "blocks.1.ffn.Wdown.weight" in sd and sd["token_embedding.weight"].shape == (300, 128)
    q = FlatParams(cfg, "cpu", torch.float32)
    q.load_reference_state_dict(sd)
    assert torch.equal(q.flat, p.flat)


def test_resume_passes_over_a_corrupted_checkpoint(tmp_path):
    """A flipped byte or a truncated shard fails the crc32 index check;
    latest(verify=True) then returns the newest checkpoint that passes."""
    import shutil
    from lora_kernel_b200.train.checkpoint import Checkpointer, complete_steps, latest
    from lora_kernel_b200.train.trainer import _layout_info
    cfg = TransformerConfig(hidden_dim=128, num_heads=2, head_dim=64, ff_dim=256, vocab_size=300, num_layers=1)
    lay = _layout_info(cfg, 64)
    ck = Checkpointer(str(tmp_path), 0, 1)
    state = {"p32": torch.randn(lay["total"]), "m": torch.zeros(lay["total"]), "v": torch.zeros(lay["total"]),
             "state": torch.arange(16.)}
    ck.save(3, None, [(0, lay["total"])], state, lay, {"step": 3})
    ck.finish()
    for step in (5, 7):
        shutil.copytree(tmp_path / "step_3", tmp_path / f"step_{step}")
    assert [os.path.basename(p) for p in complete_steps(str(tmp_path))] == ["step_7", "step_5", "step_3"]
    shard = next(f for f in os.listdir(tmp_path / "step_7") if f.startswith("optim"))
    with open(tmp_path / "step_7" / shard, "r+b") as f:   # flip one byte in the middle
        f.seek(os.path.getsize(tmp_path / "step_7" / shard) // 2)
        b = f.read(1)
        f.seek(-1, 1)
        f.write(bytes([b[0] ^ 0x40]))
    with open(tmp_path / "step_5" / shard, "r+b") as f:   # truncate
        f.truncate(100)
    assert latest(str(tmp_path)).endswith("step_7")
    assert not Checkpointer.verify(str(tmp_path / "step_7"))
    assert latest(str(tmp_path), verify=True).endswith("step_3")
    os.remove(tmp_path / "step_3" / shard)                 # a missing file fails too
    assert latest(str(tmp_path), verify=True) is None
