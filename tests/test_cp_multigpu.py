"""Context parallelism (Ulysses and ring attention) on 2 GPUs against the
single-GPU pipeline."""
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
                        vocab_size=512, num_layers=2, max_seq_len=512)
TC = TrainConfig(lr=1e-3, weight_decay=0.1, dynamic_loss_scale=True, init_loss_scale=1024.0,
                 micro_batch=2, seq_len=256, seed=5)


def batches():
    g = torch.Generator().manual_seed(0)
    return [torch.randint(0, CFG.vocab_size, (2, 257), generator=g) for _ in range(3)]


@pytest.mark.parametrize("mode", ["ulysses", "ring"])
def test_context_parallel_matches_single_gpu(tmp_path, mode):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from lora_kernel_b200.parallel.zero import ShardLayout
    from lora_kernel_b200.train.pipeline import Transformer, TrainingPipeline
    out = str(tmp_path / "cp.pt")
    env = dict(os.environ, LK_OUT=out, NCCL_NVLS_ENABLE="0", LK_NVLS="0", PYTHONPATH=HERE, LK_CP_MODE=mode)
    port = random.randint(20000, 40000)
    cmd = ["timeout", "-k", "10", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port", str(port),
           os.path.join(HERE, "dist_cp_check.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    res = torch.load(out)
    assert res["same"], "ranks disagree on the parameters"
    model = Transformer(CFG, "cuda", seed=TC.seed)
    pipe = TrainingPipeline(model, TC.lr, TC.weight_decay, TC.max_grad_norm, train_cfg=TC)
    ref_losses = [pipe.train_step(b[:, :-1], b[:, 1:]) for b in batches()]
    for a, b in zip(res["losses"], ref_losses):
        assert abs(a - b) < 2e-2 * abs(b), (res["losses"], ref_losses)
    L = ShardLayout(CFG, 2, 0)
    for sp in L.specs:
        got = res["full"][sp.offset:sp.offset + sp.numel].view(sp.shape)
        want = model.engine.params.views[sp.name].float().cpu()
        err = ((got - want).norm() / (want.norm() + 1e-12)).item()
        assert err < 2e-2, (sp.name, err)


def test_trainer_resume_cp(tmp_path):
    """Trainer.fit with parallel.cp=2: 2 steps + checkpoint + resume to 4
    gives the losses of 4 uninterrupted steps."""
    import json
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    out = str(tmp_path / "resume.json")
    env = dict(os.environ, LK_OUT=out, NCCL_NVLS_ENABLE="0", LK_NVLS="0", LORAK_HEARTBEAT="0")
    port = random.randint(20000, 40000)
    cmd = ["timeout", "-k", "10", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port", str(port),
           os.path.join(HERE, "dist_trainer_resume_check.py"), "cp", str(tmp_path)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    res = json.load(open(out))
    assert res["steps"] == [3, 4] and "step_2" in res["saved"] and "step_4" in res["saved"]
    for a, b in zip(res["full"][2:], res["resumed"]):
        assert abs(a - b) < 1e-3 * abs(a), res
