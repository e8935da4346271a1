"""Trainer.fit on one GPU: resume equivalence, overflow skip, CPU-demo config."""
import os

import pytest
import torch

pytestmark = pytest.mark.gpu


def _rc(tmp, steps, **kw):
    from lora_kernel_b200.config import get_preset
    rc = get_preset("tiny")
    rc.train.total_steps = steps
    rc.train.log_every = 1
    rc.train.checkpoint_dir = str(tmp) if tmp else ""
    rc.train.lr = 1e-3
    for k, v in kw.items():
        setattr(rc.train, k, v)
    return rc


def test_resume_matches_uninterrupted(tmp_path):
    from lora_kernel_b200.train.trainer import Trainer
    full = Trainer(_rc(None, 6)).fit()
    ck = tmp_path / "ck"
    Trainer(_rc(ck, 3)).fit()
    assert os.path.isdir(ck / "step_3")
    resumed = Trainer(_rc(ck, 6)).fit()
    assert [h["step"] for h in resumed] == [4, 5, 6]
    for a, b in zip(full[3:], resumed):
        assert abs(a["loss"] - b["loss"]) < 1e-3 * abs(a["loss"]), (a, b)


def test_nan_grad_step_is_skipped(monkeypatch):
    from lora_kernel_b200.train.trainer import Trainer
    monkeypatch.setenv("LORAK_FAULT", "nan_grad@step:2")
    tr = Trainer(_rc(None, 5, dynamic_loss_scale=True, init_loss_scale=1024.0))
    hist = tr.fit()
    assert hist[2]["skipped"] == 1 and hist[2]["loss_scale"] == 512.0
    assert hist[-1]["skipped"] == 1
    assert all(h["loss"] == h["loss"] for h in hist)


def test_cpu_demo_config_trains():
    from lora_kernel_b200.config import get_preset
    from lora_kernel_b200.train.trainer import Trainer
    rc = get_preset("cpu-demo")
    rc.train.total_steps = 30
    rc.train.log_every = 1
    rc.train.lr = 3e-3
    hist = Trainer(rc).fit()
    assert hist[-1]["loss"] < hist[0]["loss"] - 0.5
