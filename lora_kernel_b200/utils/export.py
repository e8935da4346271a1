"""Model export: GGUF (llama.cpp) and Hugging Face Llama safetensors.

Both start from the reference-named state dict (`FlatParams.
to_reference_state_dict()`: [in, out] matrices, unpadded FFN).

GGUF v3: header (magic "GGUF", version 3, tensor and metadata counts),
metadata key/values (llama.* hyper-parameters, a byte-level vocabulary),
tensor infos (name, dims innermost-first, ggml type, offset) and the tensor
data, every tensor aligned to `general.alignment` (32).  Matrices are written
as [out, in] row-major (ggml dims [in, out]); the RoPE pairs of this framework
are adjacent dimensions (2i, 2i+1), which is llama.cpp's native "llama" rope,
so q/k need no permutation.  `read_gguf` parses a file back for validation.

Hugging Face: `model.safetensors` + `config.json` for LlamaForCausalLM.  HF
rotates dimension i with i + Dh/2, so every head's q/k rows are reordered
(even dimensions first, then odd) to keep the same function.

ONNX export is in utils/onnx_export.py.  TensorRT and OpenVINO engines are
built from an ONNX file by those toolchains, which are not part of this
framework's runtime.

Reference: ExportSuite::export_gguf / export_onnx / export_trt / export_ov
(include/io/export_suite.hpp:7-13, print-only stubs).
"""
from __future__ import annotations

import json
import os
import struct
from typing import Dict, List, Tuple

import numpy as np
import torch

from ..config import TransformerConfig

# ggml tensor types and GGUF metadata value types
GGML_F32, GGML_F16, GGML_BF16 = 0, 1, 30
_T_U32, _T_I32, _T_F32, _T_BOOL, _T_STR, _T_ARR, _T_U64 = 4, 5, 6, 7, 8, 9, 10
FILE_TYPE = {"f32": 0, "f16": 1, "bf16": 32}
ALIGN = 32


def _gguf_names(cfg: TransformerConfig) -> List[Tuple[str, str]]:
    """(reference name, gguf name) in file order."""
    out = [("token_embedding.weight", "token_embd.weight")]
    for i in range(cfg.num_layers):
        r, g = f"blocks.{i}.", f"blk.{i}."
        out += [(r + "rms_norm_attn.weight", g + "attn_norm.weight"),
                (r + "attn.Wq.weight", g + "attn_q.weight"),
                (r + "attn.Wk.weight", g + "attn_k.weight"),
                (r + "attn.Wv.weight", g + "attn_v.weight"),
                (r + "attn.Wo.weight", g + "attn_output.weight"),
                (r + "rms_norm_ffn.weight", g + "ffn_norm.weight"),
                (r + "ffn.Wgate.weight", g + "ffn_gate.weight"),
                (r + "ffn.Wup.weight", g + "ffn_up.weight"),
                (r + "ffn.Wdown.weight", g + "ffn_down.weight")]
    out.append(("final_norm.weight", "output_norm.weight"))
    if not cfg.tie_embeddings:
        out.append(("lm_head.weight", "output.weight"))
    return out


class _W:
    def __init__(self, f):
        self.f = f

    def u32(self, v):
        self.f.write(struct.pack("<I", v))

    def u64(self, v):
        self.f.write(struct.pack("<Q", v))

    def s(self, text: str):
        b = text.encode("utf-8")
        self.u64(len(b))
        self.f.write(b)

    def kv(self, key: str, typ: int, val):
        self.s(key)
        self.u32(typ)
        self.val(typ, val)

    def val(self, typ, v):
        if typ == _T_U32:
            self.u32(v)
        elif typ == _T_I32:
            self.f.write(struct.pack("<i", v))
        elif typ == _T_F32:
            self.f.write(struct.pack("<f", v))
        elif typ == _T_BOOL:
            self.f.write(struct.pack("<?", v))
        elif typ == _T_STR:
            self.s(v)
        elif typ == _T_U64:
            self.u64(v)
        elif typ == _T_ARR:
            et, items = v
            self.u32(et)
            self.u64(len(items))
            for it in items:
                self.val(et, it)
        else:
            raise ValueError(typ)


def _tensor_bytes(t: torch.Tensor, dtype: str) -> Tuple[bytes, int]:
    t = t.detach().contiguous().cpu()
    if dtype == "f32":
        return t.float().numpy().tobytes(), GGML_F32
    if dtype == "f16":
        return t.half().numpy().tobytes(), GGML_F16
    return t.bfloat16().view(torch.int16).numpy().tobytes(), GGML_BF16


def export_gguf(sd: Dict[str, torch.Tensor], cfg: TransformerConfig, path: str, dtype: str = "bf16",
                name: str = "lora-kernel-b200-llama") -> None:
    """sd: reference-named state dict ([in, out] matrices).  Norm weights are
    always f32 (llama.cpp expects that)."""
    if dtype not in FILE_TYPE:
        raise ValueError(f"dtype must be one of {sorted(FILE_TYPE)}")
    names = _gguf_names(cfg)
    blobs = []
    for ref, gname in names:
        t = sd[ref]
        if t.dim() == 2:
            if ref != "token_embedding.weight":  # the embedding is already [vocab, D]
                t = t.t()  # [in, out] -> [out, in] row-major == ggml dims [in, out]
            data, typ = _tensor_bytes(t, dtype)
            dims = [t.shape[1], t.shape[0]]
        else:
            data, typ = _tensor_bytes(t, "f32")
            dims = [t.shape[0]]
        blobs.append((gname, dims, typ, data))
    V = cfg.vocab_size
    tokens = [f"<0x{i:02X}>" if i < 256 else f"<unused_{i}>" for i in range(V)]
    meta = [
        ("general.architecture", _T_STR, "llama"),
        ("general.name", _T_STR, name),
        ("general.alignment", _T_U32, ALIGN),
        ("general.file_type", _T_U32, FILE_TYPE[dtype]),
        ("llama.vocab_size", _T_U32, V),
        ("llama.context_length", _T_U32, cfg.max_seq_len),
        ("llama.embedding_length", _T_U32, cfg.hidden_dim),
        ("llama.block_count", _T_U32, cfg.num_layers),
        ("llama.feed_forward_length", _T_U32, cfg.ff_dim),
        ("llama.attention.head_count", _T_U32, cfg.num_heads),
        ("llama.attention.head_count_kv", _T_U32, cfg.num_kv_heads),
        ("llama.rope.dimension_count", _T_U32, cfg.head_dim),
        ("llama.rope.freq_base", _T_F32, float(cfg.rope_base)),
        ("llama.attention.layer_norm_rms_epsilon", _T_F32, float(cfg.norm_eps)),
        ("tokenizer.ggml.model", _T_STR, "llama"),
        ("tokenizer.ggml.tokens", _T_ARR, (_T_STR, tokens)),
        ("tokenizer.ggml.scores", _T_ARR, (_T_F32, [0.0] * V)),
        ("tokenizer.ggml.token_type", _T_ARR, (_T_I32, [6 if i < 256 else 5 for i in range(V)])),
    ]
    tmp = path + ".part"
    with open(tmp, "wb") as f:
        w = _W(f)
        f.write(b"GGUF")
        w.u32(3)
        w.u64(len(blobs))
        w.u64(len(meta))
        for k, t, v in meta:
            w.kv(k, t, v)
        off = 0
        offsets = []
        for gname, dims, typ, data in blobs:
            w.s(gname)
            w.u32(len(dims))
            for d in dims:
                w.u64(d)
            w.u32(typ)
            w.u64(off)
            offsets.append(off)
            off += (len(data) + ALIGN - 1) // ALIGN * ALIGN
        f.write(b"\0" * ((-f.tell()) % ALIGN))
        for (_, _, _, data), o in zip(blobs, offsets):
            f.write(data)
            f.write(b"\0" * ((-len(data)) % ALIGN))
    os.replace(tmp, path)


def read_gguf(path: str):
    """(metadata dict, {name: tensor}) of a GGUF file written by export_gguf
    (types f32 / f16 / bf16)."""
    with open(path, "rb") as f:
        buf = f.read()
    pos = 0

    def take(fmt):
        nonlocal pos
        v = struct.unpack_from(fmt, buf, pos)
        pos += struct.calcsize(fmt)
        return v[0]

    def s():
        nonlocal pos
        n = take("<Q")
        v = buf[pos:pos + n].decode("utf-8")
        pos += n
        return v

    def val(t):
        if t == _T_U32:
            return take("<I")
        if t == _T_I32:
            return take("<i")
        if t == _T_F32:
            return take("<f")
        if t == _T_BOOL:
            return take("<?")
        if t == _T_STR:
            return s()
        if t == _T_U64:
            return take("<Q")
        if t == _T_ARR:
            et, n = take("<I"), take("<Q")
            return [val(et) for _ in range(n)]
        raise ValueError(f"unsupported metadata type {t}")

    if buf[:4] != b"GGUF":
        raise ValueError("not a GGUF file")
    pos = 4
    if take("<I") != 3:
        raise ValueError("unsupported GGUF version")
    nt, nkv = take("<Q"), take("<Q")
    meta = {}
    for _ in range(nkv):
        k = s()
        meta[k] = val(take("<I"))
    infos = []
    for _ in range(nt):
        name = s()
        nd = take("<I")
        dims = [take("<Q") for _ in range(nd)]
        infos.append((name, dims, take("<I"), take("<Q")))
    align = meta.get("general.alignment", ALIGN)
    base = (pos + align - 1) // align * align
    out = {}
    for name, dims, typ, off in infos:
        n = int(np.prod(dims))
        shape = list(reversed(dims))
        a = base + off
        if typ == GGML_F32:
            t = torch.from_numpy(np.frombuffer(buf, np.float32, n, a).copy())
        elif typ == GGML_F16:
            t = torch.from_numpy(np.frombuffer(buf, np.float16, n, a).copy())
        elif typ == GGML_BF16:
            t = torch.from_numpy(np.frombuffer(buf, np.int16, n, a).copy()).view(torch.bfloat16)
        else:
            raise ValueError(f"unsupported tensor type {typ}")
        out[name] = t.view(shape)
    return meta, out


# ------------------------------------------------------------- Hugging Face
def _interleaved_to_half(w_out_in: torch.Tensor, heads: int, dh: int) -> torch.Tensor:
    """Reorder each head's rows from adjacent-pair RoPE to rotate-half order."""
    w = w_out_in.reshape(heads, dh // 2, 2, -1)
    return torch.cat([w[:, :, 0], w[:, :, 1]], dim=1).reshape(heads * dh, -1)


def export_hf(sd: Dict[str, torch.Tensor], cfg: TransformerConfig, out_dir: str,
              dtype: torch.dtype = torch.bfloat16) -> None:
    from safetensors.torch import save_file
    os.makedirs(out_dir, exist_ok=True)
    H, KV, Dh = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim
    t = {}
    cv = (lambda x: x.detach().to(dtype).contiguous().cpu())
    t["model.embed_tokens.weight"] = cv(sd["token_embedding.weight"])
    for i in range(cfg.num_layers):
        r, p = f"blocks.{i}.", f"model.layers.{i}."
        t[p + "self_attn.q_proj.weight"] = cv(_interleaved_to_half(sd[r + "attn.Wq.weight"].t(), H, Dh))
        t[p + "self_attn.k_proj.weight"] = cv(_interleaved_to_half(sd[r + "attn.Wk.weight"].t(), KV, Dh))
        t[p + "self_attn.v_proj.weight"] = cv(sd[r + "attn.Wv.weight"].t())
        t[p + "self_attn.o_proj.weight"] = cv(sd[r + "attn.Wo.weight"].t())
        t[p + "mlp.gate_proj.weight"] = cv(sd[r + "ffn.Wgate.weight"].t())
        t[p + "mlp.up_proj.weight"] = cv(sd[r + "ffn.Wup.weight"].t())
        t[p + "mlp.down_proj.weight"] = cv(sd[r + "ffn.Wdown.weight"].t())
        t[p + "input_layernorm.weight"] = cv(sd[r + "rms_norm_attn.weight"])
        t[p + "post_attention_layernorm.weight"] = cv(sd[r + "rms_norm_ffn.weight"])
    t["model.norm.weight"] = cv(sd["final_norm.weight"])
    if not cfg.tie_embeddings:
        t["lm_head.weight"] = cv(sd["lm_head.weight"].t())
    save_file(t, os.path.join(out_dir, "model.safetensors"), metadata={"format": "pt"})
    conf = {
        "architectures": ["LlamaForCausalLM"], "model_type": "llama",
        "hidden_size": cfg.hidden_dim, "intermediate_size": cfg.ff_dim,
        "num_hidden_layers": cfg.num_layers, "num_attention_heads": H, "num_key_value_heads": KV,
        "head_dim": Dh, "vocab_size": cfg.vocab_size, "max_position_embeddings": cfg.max_seq_len,
        "rms_norm_eps": cfg.norm_eps, "rope_theta": float(cfg.rope_base),
        "tie_word_embeddings": bool(cfg.tie_embeddings), "hidden_act": "silu",
        "attention_bias": False, "mlp_bias": False,
        "torch_dtype": str(dtype).replace("torch.", ""),
    }
    with open(os.path.join(out_dir, "config.json"), "w") as f:
        json.dump(conf, f, indent=1)


def _half_to_interleaved_rows(w_out_in: torch.Tensor, heads: int, dh: int) -> torch.Tensor:
    """Inverse of _interleaved_to_half: rotate-half rows back to adjacent pairs."""
    w = w_out_in.reshape(heads, 2, dh // 2, -1)
    return torch.stack([w[:, 0], w[:, 1]], dim=2).reshape(heads * dh, -1)


def config_from_hf(path: str) -> TransformerConfig:
    """TransformerConfig from a Hugging Face LlamaForCausalLM config.json (or its directory)."""
    if os.path.isdir(path):
        path = os.path.join(path, "config.json")
    with open(path) as f:
        c = json.load(f)
    H = c["num_attention_heads"]
    return TransformerConfig(hidden_dim=c["hidden_size"], num_heads=H,
                             num_kv_heads=c.get("num_key_value_heads", H),
                             head_dim=c.get("head_dim") or c["hidden_size"] // H, ff_dim=c["intermediate_size"],
                             vocab_size=c["vocab_size"], num_layers=c["num_hidden_layers"],
                             max_seq_len=c.get("max_position_embeddings", 4096),
                             norm_eps=c.get("rms_norm_eps", 1e-5), rope_base=float(c.get("rope_theta", 10000.0)),
                             tie_embeddings=bool(c.get("tie_word_embeddings", False)))


def import_hf(path: str, cfg: TransformerConfig, dtype: torch.dtype = torch.float32) -> Dict[str, torch.Tensor]:
    """Reference-named state dict ([in, out] matrices, adjacent-pair RoPE rows)
    from a Hugging Face Llama checkpoint: a directory with model.safetensors or
    sharded model-*.safetensors (with or without the index file), or one file."""
    from safetensors import safe_open
    files = [path]
    if os.path.isdir(path):
        files = sorted(os.path.join(path, f) for f in os.listdir(path) if f.endswith(".safetensors"))
    t: Dict[str, torch.Tensor] = {}
    for fn in files:
        with safe_open(fn, framework="pt") as f:
            for k in f.keys():
                t[k] = f.get_tensor(k)
    H, KV, Dh = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim
    cv = (lambda x: x.to(dtype).contiguous())
    sd = {"token_embedding.weight": cv(t["model.embed_tokens.weight"])}
    for i in range(cfg.num_layers):
        r, p = f"blocks.{i}.", f"model.layers.{i}."
        sd[r + "attn.Wq.weight"] = cv(_half_to_interleaved_rows(t[p + "self_attn.q_proj.weight"], H, Dh).t())
        sd[r + "attn.Wk.weight"] = cv(_half_to_interleaved_rows(t[p + "self_attn.k_proj.weight"], KV, Dh).t())
        sd[r + "attn.Wv.weight"] = cv(t[p + "self_attn.v_proj.weight"].t())
        sd[r + "attn.Wo.weight"] = cv(t[p + "self_attn.o_proj.weight"].t())
        sd[r + "ffn.Wgate.weight"] = cv(t[p + "mlp.gate_proj.weight"].t())
        sd[r + "ffn.Wup.weight"] = cv(t[p + "mlp.up_proj.weight"].t())
        sd[r + "ffn.Wdown.weight"] = cv(t[p + "mlp.down_proj.weight"].t())
        sd[r + "rms_norm_attn.weight"] = cv(t[p + "input_layernorm.weight"])
        sd[r + "rms_norm_ffn.weight"] = cv(t[p + "post_attention_layernorm.weight"])
    sd["final_norm.weight"] = cv(t["model.norm.weight"])
    if not cfg.tie_embeddings:
        sd["lm_head.weight"] = cv(t["lm_head.weight"].t())
    return sd

