"""Encrypted checkpoints (AES-256-GCM, chunked, authenticated) on CPU."""
import json
import os

import pytest
import torch

from lora_kernel_b200.train import crypto


def test_encrypt_roundtrip_multi_chunk_and_tamper(tmp_path):
    key = os.urandom(32)
    src = tmp_path / "a.bin"
    data = os.urandom(1000_003)
    src.write_bytes(data)
    enc = str(tmp_path / "a.enc")
    crypto.encrypt_file(str(src), enc, key, chunk=65536)
    assert crypto.is_encrypted(enc) and not crypto.is_encrypted(str(src))
    assert crypto.decrypt_bytes(enc, key) == data
    with pytest.raises(crypto.DecryptionError):
        crypto.decrypt_bytes(enc, os.urandom(32))
    raw = bytearray(open(enc, "rb").read())
    raw[500_000] ^= 1
    open(enc, "wb").write(raw)
    with pytest.raises(crypto.DecryptionError, match="authentication"):
        crypto.decrypt_bytes(enc, key)
    open(enc, "wb").write(raw[:-10])
    with pytest.raises(crypto.DecryptionError, match="length"):
        crypto.decrypt_bytes(enc, key)


def test_key_parsing_and_derivation():
    k = os.urandom(32)
    assert crypto.parse_key(k.hex()) == k
    import base64
    assert crypto.parse_key(base64.b64encode(k).decode()) == k
    with pytest.raises(ValueError):
        crypto.parse_key("abcd")
    a = crypto.derive_key("pass", b"salt" * 4)
    assert len(a) == 32 and a == crypto.derive_key("pass", b"salt" * 4) != crypto.derive_key("pass2", b"salt" * 4)


def test_encrypted_checkpoint_roundtrip(tmp_path):
    from lora_kernel_b200.train.checkpoint import Checkpointer, load_model_safetensors
    key = os.urandom(32)
    ck = Checkpointer(str(tmp_path), key=key)
    p32 = torch.randn(1000)
    model = {"token_embedding.weight": torch.randn(10, 4)}
    path = ck.save(3, model, [(0, 1000)], {"p32": p32, "m": p32 * 2, "v": p32 * 3, "state": torch.arange(16.)},
                   {"total": 1000}, {"step": 3})
    idx = json.load(open(os.path.join(path, "index.json")))
    assert idx["encrypted"] and Checkpointer.verify(path)
    for f in idx["files"]:
        assert crypto.is_encrypted(os.path.join(path, f))
    flat = Checkpointer.load_flat(path, key=key)
    assert torch.equal(flat["p32"], p32) and torch.equal(flat["v"], p32 * 3)
    assert torch.equal(load_model_safetensors(os.path.join(path, "model.safetensors"), key=key)
                       ["token_embedding.weight"], model["token_embedding.weight"])
    with pytest.raises(ValueError, match="encrypted"):
        Checkpointer.load_flat(path)
