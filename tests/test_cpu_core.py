"""CPU tests: configs, schedules, parameter layout, checkpoint names, oracle."""
import json
import math
import subprocess
import sys

import pytest
import torch

from lora_kernel_b200.config import TransformerConfig, get_preset, load_config


def test_presets_and_param_counts():
    c = get_preset("llama-1.1b-zero3").model
    assert 1.09e9 < c.num_parameters() < 1.11e9
    c8 = get_preset("llama-8b-tp8-fp8").model
    assert 8.0e9 < c8.num_parameters() < 8.1e9
    demo = get_preset("cpu-demo")
    assert demo.model.hidden_dim == 256 and demo.model.ff_dim == 688
    assert demo.model.ff_dim_padded == 768
    assert demo.train.micro_batch == 8 and demo.train.seq_len == 128


def test_load_config_overrides(tmp_path):
    p = tmp_path / "c.yaml"
    p.write_text("model:\n  num_layers: 3\ntrain:\n  lr: 0.001\n")
    cfg = load_config(str(p), preset="tiny", overrides={"parallel.zero_stage": 2})
    assert cfg.model.num_layers == 3 and cfg.train.lr == 0.001 and cfg.parallel.zero_stage == 2
    with pytest.raises(KeyError):
        load_config(None, preset="tiny", overrides={"train.nope": 1})


def test_lr_schedules():
    from lora_kernel_b200.train.schedules import lr_at
    assert lr_at(0, 1.0, "constant") == 1.0
    assert lr_at(0, 1.0, "cosine", warmup_steps=10, total_steps=100) == pytest.approx(0.1)
    assert lr_at(10, 1.0, "cosine", warmup_steps=10, total_steps=100) == pytest.approx(1.0)
    assert lr_at(100, 1.0, "cosine", warmup_steps=10, total_steps=100, min_lr_ratio=0.1) == pytest.approx(0.1)
    assert lr_at(55, 1.0, "linear", warmup_steps=10, total_steps=100) == pytest.approx(0.5)
    assert lr_at(50, 1.0, "polynomial", total_steps=100, power=2.0) == pytest.approx(0.25)
    assert lr_at(25, 1.0, "cosine_restarts", total_steps=100, num_cycles=2) == pytest.approx(0.5, abs=1e-6)


def test_flat_layout_alignment_and_names():
    from lora_kernel_b200.models.params import FlatParams
    cfg = TransformerConfig(hidden_dim=256, num_heads=4, num_kv_heads=2, head_dim=64, ff_dim=688,
                            vocab_size=1024, num_layers=2)
    p = FlatParams(cfg, "cpu", torch.float32)
    for s in p.specs:
        assert s.offset % 64 == 0
    p.init_(0, 0.02)
    sd = p.to_reference_state_dict()
    assert sd["blocks.0.attn.Wq.weight"].shape == (256, 256)
    assert sd["blocks.0.attn.Wk.weight"].shape == (256, 128)
    assert sd["blocks.1.ffn.Wgate.weight"].shape == (256, 688)
    assert sd["blocks.1.ffn.Wdown.weight"].shape == (688, 256)
    assert sd["lm_head.weight"].shape == (256, 1024)
    # padding rows are exactly zero
    wgu = p["layers.0.wgu"].view(6, 2, 128, 256)
    assert torch.count_nonzero(wgu[5, :, 688 - 640:]) == 0
    q = FlatParams(cfg, "cpu", torch.float32)
    q.load_reference_state_dict({k: v.clone() for k, v in sd.items()})
    assert torch.equal(q.flat, p.flat)
    tot = sum(v.numel() for v in sd.values())
    assert tot == cfg.num_parameters()


def test_oracle_gradcheck_float64():
    from lora_kernel_b200.models.params import FlatParams
    from lora_kernel_b200.oracle import llama_ref
    cfg = TransformerConfig(hidden_dim=32, num_heads=2, num_kv_heads=1, head_dim=16, ff_dim=128,
                            vocab_size=16, num_layers=1)
    p = FlatParams(cfg, "cpu", torch.float64)
    p.init_(1, 0.2)
    ids = torch.randint(0, 16, (1, 6))
    tgt = torch.randint(0, 16, (1, 6))
    w = p["layers.0.wo"].detach().clone().requires_grad_(True)

    def f(wo):
        d = {k: v for k, v in p.views.items()}
        d["layers.0.wo"] = wo
        return llama_ref.loss_fn(d, cfg, ids, tgt)

    assert torch.autograd.gradcheck(f, (w,), eps=1e-6, atol=1e-5)


def test_oracle_rope_is_rotation():
    from lora_kernel_b200.oracle.llama_ref import rope
    x = torch.randn(1, 5, 2, 8, dtype=torch.float64)
    y = rope(x, 10000.0)
    assert torch.allclose(x.norm(dim=-1), y.norm(dim=-1))
    assert torch.allclose(x[:, 0], y[:, 0])


def test_oracle_training_decreases_loss():
    from lora_kernel_b200.models.params import FlatParams
    from lora_kernel_b200.oracle.llama_ref import OracleTrainer
    cfg = TransformerConfig(hidden_dim=64, num_heads=2, head_dim=32, ff_dim=128, vocab_size=64,
                            num_layers=1)
    p = FlatParams(cfg, "cpu", torch.float32)
    p.init_(0, 0.02)
    tr = OracleTrainer(dict(p.views), cfg, lr=1e-2)
    ids = torch.randint(0, 64, (2, 17))
    l0 = tr.step(ids[:, :-1], ids[:, 1:])
    for _ in range(20):
        l = tr.step(ids[:, :-1], ids[:, 1:])
    assert l < l0 - 0.5


def test_bench_reference_arm_reports_unavailable():
    out = subprocess.run([sys.executable, "bench.py", "--impl", "reference"], capture_output=True,
                         text=True, check=True)
    d = json.loads(out.stdout.strip().splitlines()[-1])
    assert d["impl"] == "reference" and "unavailable" in d


def test_numa_cpulist_from_fake_sysfs(tmp_path):
    """The GPU's NUMA node CPUs are read from sysfs (a fake tree here)."""
    from lora_kernel_b200.utils.env import gpu_numa_cpus, parse_cpulist
    assert parse_cpulist("0-3,8,10-11\n") == {0, 1, 2, 3, 8, 10, 11}
    dev = tmp_path / "bus" / "pci" / "devices" / "0000:1b:00.0"
    dev.mkdir(parents=True)
    (dev / "numa_node").write_text("1\n")
    node = tmp_path / "devices" / "system" / "node" / "node1"
    node.mkdir(parents=True)
    (node / "cpulist").write_text("32-35,96\n")
    assert gpu_numa_cpus("00000000:1B:00.0", str(tmp_path)) == {32, 33, 34, 35, 96}
    (dev / "numa_node").write_text("-1\n")
    assert gpu_numa_cpus("0000:1b:00.0", str(tmp_path)) == set()


def test_train_cli_shorthand_flags():
    """`train --tp 8 --zero 3 ...` become the dotted overrides of the run config."""
    import argparse
    from lora_kernel_b200 import cli
    from lora_kernel_b200.config import load_config
    seen = {}
    orig = cli.cmd_train
    cli.cmd_train = lambda a: seen.update(a=a)
    try:
        cli.main(["train", "--preset", "llama-1.1b-zero3", "--cp", "8", "--cp-mode", "ring", "--zero", "2",
                  "--lr", "1e-4", "--seq-len", "4096", "--fp8", "--set", "train.seed=7"])
    finally:
        cli.cmd_train = orig
    ov = cli.train_overrides(seen["a"])
    assert ov == {"train.seed": 7, "parallel.cp": 8, "parallel.cp_mode": "ring", "parallel.zero_stage": 2,
                  "train.lr": 1e-4, "train.seq_len": 4096, "parallel.fp8": True}
    rc = load_config(None, "llama-1.1b-zero3", ov)
    assert (rc.parallel.cp, rc.parallel.cp_mode, rc.parallel.zero_stage) == (8, "ring", 2)
    assert rc.train.seq_len == 4096 and rc.train.seed == 7
    ov2 = cli.train_overrides(argparse.Namespace(set=None, tp=None, zero=0, fp8=False))
    assert ov2 == {"parallel.zero_stage": 0}


def test_swa_running_mean():
    """SWA from start_step every `every` steps equals the plain mean of the
    snapshots it took."""
    import torch
    from lora_kernel_b200.train.optimizer import SWA
    g = torch.Generator().manual_seed(0)
    snaps = [torch.randn(1000, generator=g, dtype=torch.float64) for _ in range(12)]
    swa = SWA(torch.zeros(1000, dtype=torch.float64), start_step=3, every=2)
    for step, w in enumerate(snaps):
        swa.update(w, step)
    took = [snaps[s] for s in range(3, 12, 2)]
    assert swa.n == len(took) == 5
    torch.testing.assert_close(swa.avg, torch.stack(took).mean(0), rtol=1e-12, atol=1e-12)


def test_parallel_plan_validates_and_selects():
    from lora_kernel_b200.config import ParallelConfig
    from lora_kernel_b200.train.trainer import parallel_plan
    P = ParallelConfig
    assert parallel_plan(P(), 1) == {"trainer": "single", "comm": "p2p"}
    assert parallel_plan(P(zero_stage=3, fused_collectives=False), 8) == {"trainer": "zero3", "comm": "nccl"}
    assert parallel_plan(P(dp=8, zero_stage=2), 8)["trainer"] == "dp"
    assert parallel_plan(P(tp=8, fp8=True), 8)["trainer"] == "tp"
    assert parallel_plan(P(cp=4, cp_mode="ring"), 4)["trainer"] == "cp"
    for bad, msg in [(P(tp=2, pp=2), "cannot be combined"), (P(tp=4), "spans the whole job"),
                     (P(dp=4), "data parallelism spans"), (P(cp=8, dp=8), "not combined"),
                     (P(cp=8, cp_mode="tree"), "cp_mode"), (P(zero_stage=4), "zero_stage"),
                     (P(tp=8, sequence_parallel=False), "sequence-sharded")]:
        with pytest.raises(ValueError, match=msg):
            parallel_plan(bad, 8)


def test_cpu_training_path_runs_and_learns():
    """`train --device cpu`: fp32 oracle model + AdamW on the host, on a fixed batch."""
    from lora_kernel_b200.config import get_preset
    from lora_kernel_b200.train.cpu_demo import run_cpu
    rc = get_preset("cpu-demo")
    rc.model.num_layers, rc.train.micro_batch, rc.train.seq_len, rc.train.lr = 1, 2, 32, 3e-3
    seen = []
    hist = run_cpu(rc, steps=8, log=seen.append)
    assert len(hist) == len(seen) == 8 and hist[-1]["step"] == 8
    assert abs(hist[0]["loss"] - math.log(rc.model.vocab_size)) < 0.2
    assert hist[-1]["loss"] < hist[0]["loss"] - 0.3
    assert all(r["tokens_per_s"] > 0 and r["dtype"] == "float32" for r in hist)


def test_curriculum_sequence_length_and_slice():
    import torch
    from lora_kernel_b200.utils.data import CurriculumScheduler
    c = CurriculumScheduler(256, 2048, 100, multiple=128)
    lens = [c.seq_len(s) for s in (0, 25, 50, 99, 100, 500)]
    assert lens == [256, 640, 1152, 1920, 2048, 2048]
    assert all(x % 128 == 0 for x in lens) and lens == sorted(lens)
    ids = torch.arange(2 * 2048).view(2, 2048)
    x, y = c.slice(ids, ids + 1, 0)
    assert x.shape == (2, 256) and x.is_contiguous() and torch.equal(y, x + 1)
    x, y = c.slice(ids, ids + 1, 1000)
    assert x.data_ptr() == ids.data_ptr()


def test_gradient_noise_units_and_seeding():
    """Noise variance eta / (1 + t)^gamma, multiplied by the loss scale the
    stored gradients carry; replicated gradients draw the same noise on every
    rank, shards draw their own; tensor parallelism refuses."""
    from types import SimpleNamespace
    import torch
    from lora_kernel_b200.train.trainer import Trainer
    from lora_kernel_b200.utils.model_ops import gradient_noise_, noise_seed
    g = torch.zeros(200_000)
    gen = torch.Generator().manual_seed(noise_seed(1, 9))
    gradient_noise_(g, 9, eta=0.3, gamma=0.55, generator=gen, scale=torch.tensor([1024.0]))
    want = 1024.0 * (0.3 / 10 ** 0.55) ** 0.5
    assert abs(g.std().item() / want - 1) < 0.02
    assert noise_seed(1, 9) == noise_seed(1, 9) != noise_seed(1, 10)
    assert noise_seed(1, 9, 0) != noise_seed(1, 9, 1) != noise_seed(1, 9)
    fake = SimpleNamespace(rank=3)
    assert Trainer._grad_noise_rank(fake, "single", 0) == -1
    assert Trainer._grad_noise_rank(fake, "dp", 0) == -1 and Trainer._grad_noise_rank(fake, "cp", 0) == -1
    assert Trainer._grad_noise_rank(fake, "dp", 2) == 3 and Trainer._grad_noise_rank(fake, "zero3", 3) == 3
    assert Trainer._grad_noise_rank(fake, "pp", 0) == 3
    with pytest.raises(NotImplementedError):
        Trainer._grad_noise_rank(fake, "tp", 0)


def test_perf_regression_check(tmp_path):
    from lora_kernel_b200.utils.perf_check import compare, last_json, main
    ref = last_json("profiles/bench_llama1b_2gpu_lk.json")
    assert ref["n_gpus"] == 2 and ref["value"] > 0
    new = dict(ref, value=ref["value"] * 0.97)
    assert compare(new, ref)["status"] == "ok"
    assert compare(dict(ref, value=ref["value"] * 0.9), ref)["status"] == "regression"
    assert compare(dict(ref, n_gpus=4), ref)["status"] == "not_comparable"
    hot = dict(ref, clocks={"reasons": ["sw_power_cap", "hw_thermal_slowdown"]})
    assert compare(hot, ref)["status"] == "not_comparable"
    p = tmp_path / "new.json"
    p.write_text("noise\n" + json.dumps(dict(ref, value=ref["value"] * 0.5)) + "\n")
    assert main([str(p), "profiles/bench_llama1b_2gpu_lk.json"]) == 1


def test_cpu_training_starts_from_pretrained_weights(tmp_path):
    """train.init_from (reference safetensors and a Hugging Face directory):
    the first step's loss is the loss of the loaded weights, not of a fresh init."""
    import torch
    from lora_kernel_b200.config import get_preset
    from lora_kernel_b200.models.params import FlatParams
    from lora_kernel_b200.oracle.llama_ref import loss_fn
    from lora_kernel_b200.train.checkpoint import save_model_safetensors
    from lora_kernel_b200.train.cpu_demo import run_cpu
    from lora_kernel_b200.utils.export import export_hf
    rc = get_preset("cpu-demo")
    rc.model.num_layers, rc.train.micro_batch, rc.train.seq_len = 1, 2, 32
    cfg, tc = rc.model, rc.train
    src = FlatParams(cfg, "cpu", torch.float32)
    src.init_(99, 0.2)                                   # far from the default init
    g = torch.Generator().manual_seed(tc.seed)
    ids = torch.randint(0, cfg.vocab_size, (tc.micro_batch, tc.seq_len + 1), generator=g)
    want = float(loss_fn(dict(src.views), cfg, ids[:, :-1], ids[:, 1:]))
    save_model_safetensors(src.to_reference_state_dict(), str(tmp_path / "model.safetensors"))
    export_hf(src.to_reference_state_dict(), cfg, str(tmp_path / "hf"), dtype=torch.float32)
    for path, fmt in ((str(tmp_path / "model.safetensors"), "safetensors"), (str(tmp_path / "hf"), "hf")):
        tc.init_from, tc.init_format = path, fmt
        first = run_cpu(rc, steps=1)[0]["loss"]
        assert abs(first - want) < 1e-4, (fmt, first, want)


def test_cpu_lora_trains_adapters_only(tmp_path):
    """`train --device cpu --lora-rank 8`: the loss falls with the base frozen,
    and the adapters are written in the GPU path's file format."""
    from lora_kernel_b200.config import get_preset
    from lora_kernel_b200.models.lora import load_lora_file
    from lora_kernel_b200.train.cpu_demo import run_cpu
    rc = get_preset("cpu-demo")
    rc.model.num_layers, rc.train.micro_batch, rc.train.seq_len = 1, 2, 32
    rc.train.lr, rc.train.lora_rank, rc.train.lora_alpha = 1e-2, 8, 16.0
    rc.train.checkpoint_dir = str(tmp_path)
    hist = run_cpu(rc, steps=12)
    assert hist[-1]["loss"] < hist[0]["loss"] - 0.2
    ad = load_lora_file(str(tmp_path / "lora_step_12.safetensors"), rc.model, "cpu")
    b = ad.state_dict()["layers.0.wqkv.B"]
    assert ad.lc.rank == 8 and float(b.abs().sum()) > 0      # B starts at zero and was trained


def test_vocab_chunk_policy():
    """Chunk the LM head only when the whole logits would be large."""
    from lora_kernel_b200.models.llama import LlamaModel
    from lora_kernel_b200.config import get_preset
    big = get_preset("llama-8b-fsdp-dp8").model
    small = get_preset("llama-1.1b-zero3").model
    # the 1.1B logits at 8192 tokens (0.5 GB) stay whole; the 8B ones (2.1 GB) are chunked
    assert LlamaModel.ce_chunk(type("M", (), {"cfg": small})(), 8192) == 0
    assert LlamaModel.ce_chunk(type("M", (), {"cfg": big})(), 8192) == 8192
