"""Model export on CPU: GGUF round trip and a Hugging Face LlamaForCausalLM
that reproduces the fp32 oracle's logits."""
import pytest
import torch

from lora_kernel_b200.config import TransformerConfig
from lora_kernel_b200.models.params import FlatParams
from lora_kernel_b200.oracle import llama_ref
from lora_kernel_b200.utils.export import export_gguf, export_hf, read_gguf

CFG = TransformerConfig(hidden_dim=128, num_heads=4, num_kv_heads=2, head_dim=32, ff_dim=200,
                        vocab_size=300, num_layers=2, max_seq_len=64)


def _params():
    p = FlatParams(CFG, "cpu", torch.float32)
    p.init_(3, 0.05)
    return p


@pytest.mark.parametrize("dtype", ["f32", "bf16", "f16"])
def test_gguf_roundtrip(tmp_path, dtype):
    p = _params()
    sd = p.to_reference_state_dict()
    path = str(tmp_path / "m.gguf")
    export_gguf(sd, CFG, path, dtype=dtype)
    meta, t = read_gguf(path)
    assert meta["general.architecture"] == "llama" and meta["llama.block_count"] == 2
    assert meta["llama.attention.head_count_kv"] == 2 and meta["llama.feed_forward_length"] == 200
    assert len(meta["tokenizer.ggml.tokens"]) == 300
    assert t["token_embd.weight"].shape == (300, 128)
    assert t["blk.1.attn_k.weight"].shape == (64, 128)  # [out, in]
    assert t["blk.0.ffn_down.weight"].shape == (128, 200)
    tol = {"f32": 0.0, "bf16": 1e-2, "f16": 1e-3}[dtype]
    want = sd["blocks.1.attn.Wq.weight"].t()
    got = t["blk.1.attn_q.weight"].float()
    assert ((got - want).abs().max() <= tol * want.abs().max() + 1e-12)
    assert t["output_norm.weight"].dtype == torch.float32


def test_hf_export_matches_oracle(tmp_path):
    from transformers import LlamaForCausalLM
    p = _params()
    export_hf(p.to_reference_state_dict(), CFG, str(tmp_path), dtype=torch.float32)
    hf = LlamaForCausalLM.from_pretrained(str(tmp_path), torch_dtype=torch.float32).eval()
    ids = torch.randint(0, CFG.vocab_size, (2, 17), generator=torch.Generator().manual_seed(0))
    want = llama_ref.forward({k: v for k, v in p.views.items()}, CFG, ids)
    with torch.no_grad():
        got = hf(ids).logits
    assert torch.allclose(got, want, atol=1e-4, rtol=1e-4), (got - want).abs().max()


@pytest.mark.parametrize("tie", [False, True])
def test_onnx_export_reproduces_the_oracle(tmp_path, tie):
    """The ONNX file parses back (IR 8, opset 17, standard operators only) and,
    evaluated by the operator definitions with numpy, gives the fp32 oracle's
    logits for two sequence lengths (symbolic sequence axis)."""
    import dataclasses
    from lora_kernel_b200.utils.onnx_export import export_onnx, load_onnx, run_onnx
    cfg = dataclasses.replace(CFG, tie_embeddings=tie)
    p = FlatParams(cfg, "cpu", torch.float32)
    p.init_(3, 0.05)
    path = str(tmp_path / "m.onnx")
    export_onnx(p.to_reference_state_dict(), cfg, path)
    m = load_onnx(path)
    assert m["opset"] == 17 and m["inputs"] == ["input_ids"] and m["outputs"] == ["logits"]
    ops = {n[0] for n in m["nodes"]}
    assert ops <= {"Gather", "Shape", "Slice", "Concat", "Unsqueeze", "Reshape", "Transpose", "MatMul", "Add",
                   "Sub", "Mul", "Div", "Sqrt", "Sigmoid", "ReduceMean", "Softmax"}
    for S in (17, 40):
        ids = torch.randint(0, cfg.vocab_size, (2, S), generator=torch.Generator().manual_seed(S))
        want = llama_ref.forward({k: v for k, v in p.views.items()}, cfg, ids)
        got = run_onnx(m, {"input_ids": ids.numpy().astype("int64")})["logits"]
        assert got.shape == (2, S, cfg.vocab_size)
        assert torch.allclose(torch.from_numpy(got), want, atol=1e-4, rtol=1e-4), \
            (torch.from_numpy(got) - want).abs().max()


def test_hf_import_inverts_export(tmp_path):
    from lora_kernel_b200.utils.export import config_from_hf, import_hf
    p = _params()
    sd = p.to_reference_state_dict()
    export_hf(sd, CFG, str(tmp_path), dtype=torch.float32)
    cfg = config_from_hf(str(tmp_path))
    for k in ("hidden_dim", "num_heads", "num_kv_heads", "head_dim", "ff_dim", "vocab_size", "num_layers",
              "norm_eps", "rope_base", "tie_embeddings"):
        assert getattr(cfg, k) == getattr(CFG, k), k
    back = import_hf(str(tmp_path), cfg)
    assert set(back) == set(sd)
    for k, v in sd.items():
        assert torch.equal(back[k], v.float()), k
