"""Tensor-parallel serving on 2 GPUs against the single-GPU engine."""
import json
import os
import random
import subprocess
import sys

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.parametrize("weights", ["none", "int4"])
def test_tp_serving_matches_single_gpu(weights, tmp_path):
    world = 2
    if torch.cuda.device_count() < world:
        pytest.skip("needs 2 GPUs")
    out = str(tmp_path / "s.json")
    env = dict(os.environ, LK_OUT=out, NCCL_NVLS_ENABLE="0")
    port = random.randint(20000, 40000)
    cmd = ["timeout", "-k", "10", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr", "127.0.0.1", "--master-port", str(port),
           os.path.join(HERE, "dist_tp_serve_check.py"), weights]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    res = json.load(open(out))
    assert res["first"], res
    assert res["match"] >= 0.85, res
    assert res["sampled_len"] == [6, 6], res
