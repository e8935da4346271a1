"""Pipeline parallelism (1F1B, one stage per GPU) on 2 GPUs against the
single-GPU pipeline on the same micro-batches."""
import os
import random
import subprocess
import sys

import pytest
import torch

from lora_kernel_b200.config import TrainConfig, TransformerConfig

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

HERE = os.path.dirname(os.path.abspath(__file__))
CFG = TransformerConfig(hidden_dim=256, num_heads=4, num_kv_heads=2, head_dim=64, ff_dim=512,
                        vocab_size=512, num_layers=4, max_seq_len=256)
TC = TrainConfig(lr=1e-3, weight_decay=0.1, dynamic_loss_scale=True, init_loss_scale=1024.0,
                 micro_batch=2, seq_len=128, seed=5, grad_accum_steps=4)


def batches():
    g = torch.Generator().manual_seed(0)
    return [[torch.randint(0, CFG.vocab_size, (2, 129), generator=g) for _ in range(4)] for _ in range(2)]


def _single_gpu():
    from lora_kernel_b200.train.pipeline import Transformer, TrainingPipeline
    model = Transformer(CFG, "cuda", seed=TC.seed)
    pipe = TrainingPipeline(model, TC.lr, TC.weight_decay, TC.max_grad_norm, train_cfg=TC)
    losses = []
    for step in batches():
        pipe.loss_acc.zero_()
        for ids in step:
            d = ids.cuda()
            pipe.micro_step_async(d[:, :-1].contiguous(), d[:, 1:].contiguous())
        s, n = pipe.loss_acc.tolist()
        losses.append(s / n)
    sd = {k: v.float().cpu() for k, v in model.engine.params.to_reference_state_dict().items()}
    return sd, losses


def test_pipeline_matches_single_gpu(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    out = str(tmp_path / "pp.pt")
    env = dict(os.environ, LK_OUT=out, NCCL_NVLS_ENABLE="0", PYTHONPATH=HERE)
    port = random.randint(20000, 40000)
    cmd = ["timeout", "-k", "10", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port", str(port),
           os.path.join(HERE, "dist_pp_check.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    res = torch.load(out)
    assert res["parts"] == [[0, 1], [2, 3]]
    ref, ref_losses = _single_gpu()
    for a, b in zip(res["losses"], ref_losses):
        assert abs(a - b) < 1e-2 * abs(b), (res["losses"], ref_losses)
    assert sorted(res["full"]) == sorted(ref)
    for k, want in ref.items():
        got = res["full"][k]
        err = ((got - want).norm() / (want.norm() + 1e-12)).item()
        assert err < 2e-2, (k, err)


def test_trainer_resume_pp(tmp_path):
    """Trainer.fit with parallel.pp=2: 2 steps + checkpoint + resume to 4
    gives the losses of 4 uninterrupted steps."""
    import json
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    out = str(tmp_path / "resume.json")
    env = dict(os.environ, LK_OUT=out, NCCL_NVLS_ENABLE="0", LK_NVLS="0", LORAK_HEARTBEAT="0")
    port = random.randint(20000, 40000)
    cmd = ["timeout", "-k", "10", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port", str(port),
           os.path.join(HERE, "dist_trainer_resume_check.py"), "pp", str(tmp_path)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    res = json.load(open(out))
    assert res["steps"] == [3, 4] and "step_2" in res["saved"] and "step_4" in res["saved"]
    for a, b in zip(res["full"][2:], res["resumed"]):
        assert abs(a - b) < 1e-3 * abs(a), res
