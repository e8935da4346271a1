"""Peer-memory collectives on 2 GPUs: one-shot P2P and NVLS (multimem)
all-reduce / reduce-scatter with fused sum-of-squares partials vs NCCL."""
import json
import os
import random
import subprocess
import sys

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

HERE = os.path.dirname(os.path.abspath(__file__))


def test_peer_collectives(tmp_path):
    world = 2
    if torch.cuda.device_count() < world:
        pytest.skip("needs 2 GPUs")
    out = str(tmp_path / "c")
    env = dict(os.environ, LK_OUT=out)
    port = random.randint(20000, 40000)
    cmd = ["timeout", "-k", "10", "180", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr", "127.0.0.1", "--master-port", str(port),
           os.path.join(HERE, "dist_comm_check.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=240)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    for k in range(world):
        res = json.load(open(f"{out}.{k}"))
        tags = ["p2p"] + (["nvls"] if res["nvls_available"] else [])
        for t in tags:
            assert res[f"{t}.ar_err"] < 1e-6, res
            assert res[f"{t}.ar_untouched"], res
            assert res[f"{t}.ar_sumsq_err"] < 1e-4, res
            assert res[f"{t}.rs_err"] < 1e-6, res
