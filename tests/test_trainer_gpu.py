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


def test_trainer_starts_from_pretrained_weights(tmp_path):
    """train.init_from on one GPU: the bf16 parameters and the fp32 master take
    the saved (reference-named) weights, and training continues from them."""
    from lora_kernel_b200.models.params import FlatParams
    from lora_kernel_b200.train.checkpoint import save_model_safetensors
    from lora_kernel_b200.train.trainer import Trainer
    rc = _rc(None, 2)
    src = FlatParams(rc.model, "cpu", torch.float32)
    src.init_(99, 0.2)                                   # far from the default init
    ref = src.to_reference_state_dict()
    path = str(tmp_path / "model.safetensors")
    save_model_safetensors(ref, path)
    rc.train.init_from, rc.train.init_format = path, "safetensors"
    tr = Trainer(rc)
    got = tr.model.state_dict()
    for k, v in ref.items():
        g = got[k].float().cpu()
        assert torch.allclose(g, v, rtol=1e-2, atol=1e-3), k
    fresh = Trainer(_rc(None, 2)).fit()
    hist = tr.fit()
    assert all(h["loss"] == h["loss"] for h in hist)
    assert abs(hist[0]["loss"] - fresh[0]["loss"]) > 1e-3   # not the default init's loss


def test_trainer_lora_trains_adapters_only(tmp_path):
    """train.lora_rank on one GPU: the base weights stay frozen, the adapters
    change and are written as lora_step_N.safetensors."""
    from lora_kernel_b200.models.lora import load_lora_file
    from lora_kernel_b200.train.trainer import Trainer
    rc = _rc(tmp_path, 4, lora_rank=8, lora_alpha=16.0, lr=1e-2)
    tr = Trainer(rc)
    base = {k: v.float().cpu().clone() for k, v in tr.model.state_dict().items()}
    hist = tr.fit()
    assert len(hist) == 4 and all(h["loss"] == h["loss"] for h in hist)
    after = tr.model.state_dict()
    for k, v in base.items():
        assert torch.equal(after[k].float().cpu(), v), k
    ad = load_lora_file(str(tmp_path / "lora_step_4.safetensors"), rc.model, "cpu")
    b = ad.state_dict()["layers.0.wqkv.B"]
    assert ad.lc.rank == 8 and float(b.abs().sum()) > 0      # B starts at zero and was trained
