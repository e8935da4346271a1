"""Tensor-parallel serving from a checkpoint, host side: every rank's shard
taken from a reference-named state dict reassembles into the full weights."""
import torch

from lora_kernel_b200.config import TransformerConfig
from lora_kernel_b200.models.params import FlatParams


def test_tp_shards_from_state_dict_reassemble():
    from lora_kernel_b200.parallel.tp import unshard_tensor
    from lora_kernel_b200.serve.tp_runner import tp_params_from_state_dict
    cfg = TransformerConfig(hidden_dim=128, num_heads=4, num_kv_heads=2, head_dim=32, ff_dim=256,
                            vocab_size=96, num_layers=2)
    full = FlatParams(cfg, "cpu", torch.float32)
    full.init_(7, 0.05)
    sd = full.to_reference_state_dict()
    tp = 2
    shards = [tp_params_from_state_dict(cfg, sd, tp, r, "cpu") for r in range(tp)]
    for s in shards[0].specs:
        got = unshard_tensor(cfg, s.name, [sh[s.name].float() for sh in shards])
        torch.testing.assert_close(got, full.views[s.name].float(), rtol=0, atol=1e-2)
