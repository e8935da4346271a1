"""Authenticated encryption of checkpoint files (AES-256-GCM).

File layout
  header   magic "LKENC1\\0\\0" | 12-byte random nonce base | u32 chunk size |
           u64 plaintext length                                   (32 bytes)
  chunks   AES-256-GCM(chunk i) with nonce = nonce base XOR i (last 8 bytes),
           associated data = header || u64 i; each chunk carries its 16-byte
           tag, so truncation, reordering and bit flips are all detected.
Chunks (64 MiB) are encrypted and decrypted on a thread pool; a file is never
held twice in memory beyond one chunk per thread.

Keys are 32 bytes: from hex / base64 text (LORAK_CKPT_KEY), a key file, or
derived from a passphrase with scrypt (n=2^15, r=8, p=1) and a stored salt.

Reference: AES256CTR / EncryptedCheckpointStorage
(include/crypto/crypto_engine.hpp:14-132), unauthenticated CTR with a fresh
random key per instance, so a checkpoint cannot be decrypted by a new process.
"""
from __future__ import annotations

import base64
import binascii
import os
import struct
from concurrent.futures import ThreadPoolExecutor
from typing import Optional

from cryptography.hazmat.primitives.ciphers.aead import AESGCM
from cryptography.hazmat.primitives.kdf.scrypt import Scrypt

MAGIC = b"LKENC1\x00\x00"
HEADER = struct.Struct("<8s12sIQ")
CHUNK = 64 << 20
TAG = 16


class DecryptionError(ValueError):
    pass


def parse_key(text: str) -> bytes:
    """32-byte key from 64 hex characters or base64."""
    t = text.strip()
    try:
        k = binascii.unhexlify(t) if len(t) == 64 else base64.b64decode(t, validate=True)
    except (binascii.Error, ValueError) as e:
        raise ValueError("key must be 32 bytes as hex or base64") from e
    if len(k) != 32:
        raise ValueError("key must be 32 bytes")
    return k


def derive_key(passphrase: str, salt: bytes) -> bytes:
    return Scrypt(salt=salt, length=32, n=1 << 15, r=8, p=1).derive(passphrase.encode())


def key_from_env(var: str = "LORAK_CKPT_KEY") -> Optional[bytes]:
    v = os.environ.get(var)
    return parse_key(v) if v else None


def _nonce(base: bytes, i: int) -> bytes:
    tail = struct.unpack("<Q", base[4:])[0] ^ i
    return base[:4] + struct.pack("<Q", tail)


def encrypt_file(src: str, dst: str, key: bytes, chunk: int = CHUNK, threads: int = 8) -> None:
    aes = AESGCM(key)
    n = os.path.getsize(src)
    header = HEADER.pack(MAGIC, os.urandom(12), chunk, n)
    nchunks = (n + chunk - 1) // chunk
    tmp = dst + ".part"

    def enc(i):
        with open(src, "rb") as f:
            f.seek(i * chunk)
            data = f.read(chunk)
        return aes.encrypt(_nonce(header[8:20], i), data, header + struct.pack("<Q", i))

    with open(tmp, "wb") as out, ThreadPoolExecutor(max(1, threads)) as ex:
        out.write(header)
        for ct in ex.map(enc, range(nchunks)):
            out.write(ct)
    os.replace(tmp, dst)


def _read_header(f):
    raw = f.read(HEADER.size)
    if len(raw) != HEADER.size:
        raise DecryptionError("file too short for an encrypted checkpoint")
    magic, nonce, chunk, n = HEADER.unpack(raw)
    if magic != MAGIC:
        raise DecryptionError("not an encrypted checkpoint file")
    return raw, nonce, chunk, n


def decrypt_bytes(path: str, key: bytes, threads: int = 8) -> bytes:
    aes = AESGCM(key)
    with open(path, "rb") as f:
        header, nonce, chunk, n = _read_header(f)
        body_off = HEADER.size
    nchunks = (n + chunk - 1) // chunk
    size = os.path.getsize(path)
    if size != body_off + n + nchunks * TAG:
        raise DecryptionError("encrypted file has the wrong length (truncated or extended)")
    out = bytearray(n)

    def dec(i):
        ln = min(chunk, n - i * chunk)
        with open(path, "rb") as f:
            f.seek(body_off + i * (chunk + TAG))
            ct = f.read(ln + TAG)
        try:
            pt = aes.decrypt(_nonce(nonce, i), ct, header + struct.pack("<Q", i))
        except Exception as e:  # InvalidTag
            raise DecryptionError(f"chunk {i} failed authentication (wrong key or tampered file)") from e
        out[i * chunk:i * chunk + ln] = pt

    with ThreadPoolExecutor(max(1, threads)) as ex:
        list(ex.map(dec, range(nchunks)))
    return bytes(out)


def decrypt_file(src: str, dst: str, key: bytes) -> None:
    data = decrypt_bytes(src, key)
    with open(dst + ".part", "wb") as f:
        f.write(data)
    os.replace(dst + ".part", dst)


def is_encrypted(path: str) -> bool:
    with open(path, "rb") as f:
        return f.read(8) == MAGIC
