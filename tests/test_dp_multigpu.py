"""Data parallelism (ZeRO stage 0/1/2) on 2 GPUs: the fused peer-memory path
(K12 all-reduce, K10 reduce-scatter + AdamW with the parameter all-gather
fused into the update) and the NCCL baseline, against 1 GPU."""
import os
import random
import subprocess
import sys

import pytest
import torch

from test_zero_multigpu import _single_gpu_reference

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.parametrize("stage,mode", [(0, "p2p"), (1, "p2p"), (2, "p2p"), (2, "nccl"), (0, "nccl"),
                                        (0, "p2p-nonvls"), (2, "p2p-nonvls")])
def test_dp_matches_single_gpu(stage, mode, tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    out = str(tmp_path / "dp.pt")
    env = dict(os.environ, LK_OUT=out, NCCL_NVLS_ENABLE="0")
    if mode.endswith("-nonvls"):  # the one-shot P2P kernels instead of multimem
        env["LK_NVLS"] = "0"
        mode = mode.split("-")[0]
    elif mode == "p2p":  # exercise the multimem kernels even on 2 ranks
        env["LK_NVLS"] = "1"
    port = random.randint(20000, 40000)
    cmd = ["timeout", "-k", "10", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr", "127.0.0.1", "--master-port", str(port),
           os.path.join(HERE, "dist_dp_check.py"), str(stage), mode]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    res = torch.load(out)
    assert res["same"], "ranks disagree on the parameters"
    ref_params, ref_losses, L, _ = _single_gpu_reference(world)
    for a, b in zip(res["losses"], ref_losses):
        assert abs(a - b) < 2e-2 * abs(b), (res["losses"], ref_losses)
    full = res["full"]
    for sp in L.specs:
        got = full[sp.offset:sp.offset + sp.numel].view(sp.shape)
        want = ref_params[sp.name]
        err = ((got - want).norm() / (want.norm() + 1e-12)).item()
        assert err < 2e-2, (sp.name, err)
