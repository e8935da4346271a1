"""GEMM tile-width tuning table (utils/autotune.py) on CPU: the sweep keeps
the faster width per problem, the JSON round-trips, and ops.gemm resolves a
call's width from the table by shape, epilogue and operand layout."""
import json

import pytest
import torch

from lora_kernel_b200.config import get_preset
from lora_kernel_b200.ops import gemm as G
from lora_kernel_b200.utils import autotune as AT


def test_step_problems_cover_the_engine_gemms():
    cfg = get_preset("llama-1.1b-zero3").model
    probs = AT.step_problems(cfg, 8192)
    names = {p.name for p in probs}
    for layer in ("wqkv", "wo", "wgu", "wdown"):
        assert {f"{layer}.fwd", f"{layer}.dgrad", f"{layer}.wgrad"} <= names
    fwd = {p.name: p for p in probs}["wqkv.fwd"]
    assert (fwd.M, fwd.N, fwd.K) == (8192, (32 + 8) * 64, 2048)
    wg = {p.name: p for p in probs}["wdown.wgrad"]
    assert (wg.M, wg.N, wg.K, wg.a_kmajor, wg.b_kmajor) == (2048, 5632, 8192, False, False)
    assert len({p.key for p in probs}) == len(probs)


def test_tune_picks_the_faster_width_and_round_trips(tmp_path):
    probs = [AT.GemmProblem("small", 256, 384, 512), AT.GemmProblem("big", 8192, 11264, 2048, "swiglu")]
    fake = {("small", 128): 0.010, ("small", 256): 0.020, ("big", 128): 0.90, ("big", 256): 0.70}
    seen = []
    table = AT.tune(probs, lambda p, bn: fake[(p.name, bn)], device="fake", log=seen.append)
    assert table.bn(probs[0].key) == 128 and table.bn(probs[1].key) == 256
    assert len(seen) == 2 and json.loads(seen[1])["bn"] == 256
    path = str(tmp_path / "t.json")
    table.save(path)
    back = AT.GemmTable.load(path)
    assert back.entries == table.entries and back.device == "fake"
    bad = table.to_json()
    bad["entries"][probs[0].key]["bn"] = 192
    with pytest.raises(ValueError, match="tile width"):
        AT.GemmTable.from_json(bad)


def test_gemm_resolves_width_from_the_table(tmp_path, monkeypatch):
    a = torch.empty(256, 512, dtype=torch.bfloat16)
    w = torch.empty(384, 512, dtype=torch.bfloat16)
    table = AT.GemmTable()
    table.record(AT.GemmProblem("fwd", 256, 384, 512), {128: 1.0, 256: 2.0})
    table.record(AT.GemmProblem("dgrad", 256, 512, 384, "bf16", True, False), {128: 2.0, 256: 1.0})
    path = str(tmp_path / "t.json")
    table.save(path)
    try:
        G.set_tuning(path)
        assert G.tuned_bn(a, w, "bf16") == 128
        assert G.tuned_bn(a, w, "bf16_resid") == 0          # other epilogue: untuned
        dy = torch.empty(256, 384, dtype=torch.bfloat16)
        assert G.tuned_bn(dy, w.t(), "bf16") == 256          # transpose view of the weight
        assert G.tuned_bn(dy, w.t().contiguous(), "bf16") == 0
        # the environment variable is read on first use
        G._tuning_loaded = False
        monkeypatch.setenv("LK_GEMM_TUNING", path)
        assert G.tuned_bn(a, w, "bf16") == 128
        G.set_tuning(None)
        assert G.tuned_bn(a, w, "bf16") == 0
    finally:
        G.set_tuning(None)
        G._tuning_loaded = False


@pytest.mark.gpu
def test_tuned_widths_give_the_default_result():
    """On the device: a two-problem sweep, then the GEMMs run through the
    loaded table match the untuned dispatch and the fp32 reference, and both
    tile widths match the reference."""
    from lora_kernel_b200._ext import check_status
    probs = [AT.GemmProblem("fwd", 512, 768, 1024), AT.GemmProblem("dgrad", 512, 1024, 768, "bf16", True, False)]
    table = AT.tune(probs, AT._device_measure(iters=3), device="cuda")
    assert all(table.bn(p.key) in AT.CANDIDATES for p in probs)
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(512, 1024, generator=g, device="cuda").to(torch.bfloat16)
    w = torch.randn(768, 1024, generator=g, device="cuda").to(torch.bfloat16)
    dy = torch.randn(512, 768, generator=g, device="cuda").to(torch.bfloat16)
    try:
        G.set_tuning(None)
        y0, dx0 = G.gemm(x, w), G.gemm(dy, w.t())
        G.set_tuning(table)
        y1, dx1 = G.gemm(x, w), G.gemm(dy, w.t())
        for bn in AT.CANDIDATES:  # both widths agree with the reference
            yb = G.gemm(x, w, bn=bn)
            torch.testing.assert_close(yb.float(), x.float() @ w.float().t(), rtol=2e-2, atol=2e-2)
        torch.cuda.synchronize()
        check_status()
    finally:
        G.set_tuning(None)
        G._tuning_loaded = False
    torch.testing.assert_close(y1.float(), x.float() @ w.float().t(), rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(dx1.float(), dy.float() @ w.float(), rtol=2e-2, atol=2e-1)
    torch.testing.assert_close(y1.float(), y0.float(), rtol=1e-2, atol=1e-2)
    torch.testing.assert_close(dx1.float(), dx0.float(), rtol=1e-2, atol=1e-1)
