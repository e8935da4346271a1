"""Speculative decoding with real serving runners on the GPU: the greedy
output equals the target runner's own greedy decode, and a target that
drafts for itself has every proposal accepted."""
import pytest
import torch

pytestmark = pytest.mark.gpu
dev = "cuda"


def _runner(layers, seed, std=0.08):
    from lora_kernel_b200.config import TransformerConfig
    from lora_kernel_b200.models.params import FlatParams
    from lora_kernel_b200.serve.model_runner import ModelRunner
    cfg = TransformerConfig(hidden_dim=256, num_heads=4, num_kv_heads=2, head_dim=64, ff_dim=512,
                            vocab_size=512, num_layers=layers, max_seq_len=512)
    params = FlatParams(cfg, dev)
    params.init_(seed, std)
    return ModelRunner(cfg, params, dev, kv_dtype="bf16", num_blocks=64, block_size=16, max_model_len=512)


@pytest.mark.parametrize("k", [2, 4])
def test_speculative_greedy_matches_target_greedy(k):
    from lora_kernel_b200.serve.speculative import RunnerScorer, SpeculativeDecoder, greedy_reference
    target, draft = _runner(2, 3), _runner(1, 9)
    torch.manual_seed(0)
    prompt = torch.randint(0, 512, (37,)).tolist()
    ref = greedy_reference(RunnerScorer(target), prompt, 48)
    sd = SpeculativeDecoder(RunnerScorer(target), RunnerScorer(draft), k=k)
    out = sd.generate(prompt, 48)
    torch.cuda.synchronize()
    assert out == ref
    assert sd.stats.target_forwards < 48 or sd.stats.acceptance_rate == 0.0


def test_self_draft_accepts_all():
    from lora_kernel_b200.serve.speculative import RunnerScorer, SpeculativeDecoder
    target = _runner(2, 3)
    twin = _runner(2, 3)
    sd = SpeculativeDecoder(RunnerScorer(target), RunnerScorer(twin), k=4)
    sd.generate(list(range(20)), 40)
    assert sd.stats.acceptance_rate > 0.95
