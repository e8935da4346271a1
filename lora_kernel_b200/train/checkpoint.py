"""Checkpoints: weights in the reference's tensor names, optimizer state,
trainer state; sharded ZeRO checkpoints that reshard on load.

Layout of `<dir>/step_<N>/`:
  model.safetensors                 full weights, reference names / [in, out]
                                    orientation (include/io/serialization.hpp:13-44)
  optim-rank{r}-of-{W}.safetensors  flat fp32 master / m / v (/ ema) of rank r's
                                    range of the flat layout, plus the device
                                    state vector (loss scale, step, ...)
  index.json                        world size, flat layout (groups, chunks),
                                    per-file crc32
  trainer.json                      step, micro-step, config, data cursor, rng
A checkpoint is written to `step_<N>.tmp/` and renamed when complete, so a
crash never leaves a half-written `step_<N>/`; `latest()` ignores `.tmp`.

Resharding: every optimizer file stores its ranges of the flat layout, so a
load at a different world size concatenates them into full flat vectors and
slices out the new owner's chunks.

Reference: DistributedCheckpointer (include/distributed/checkpointing.hpp:
10-72: raw per-rank float shards and a YAML-ish .meta), ProductionTrainer's
header-only checkpoint (include/nn/production_trainer.hpp:35-84) and
SafetensorsWriter (include/tensor/safetensors.hpp:11-83).
"""
from __future__ import annotations

import json
import os
import shutil
import logging
import threading
from typing import Dict, List, Optional, Tuple

import torch
from safetensors.torch import load_file, save_file

log = logging.getLogger(__name__)


def _crc(path: str) -> int:
    """CRC-32 of a file (zlib's polynomial), chunks checksummed in parallel by
    the native runtime."""
    from .. import _rt
    c = 0
    buf = bytearray(1 << 28)
    mv = memoryview(buf)
    with open(path, "rb") as f:
        while True:
            n = f.readinto(buf)
            if not n:
                return c
            c = _rt.crc32(mv[:n], c)


def complete_steps(root: str) -> List[str]:
    """Published checkpoints under root (index written, not `.tmp`), newest first."""
    if not os.path.isdir(root):
        return []
    steps = []
    for d in os.listdir(root):
        if d.startswith("step_") and not d.endswith(".tmp") and os.path.exists(os.path.join(root, d, "index.json")):
            try:
                steps.append((int(d[5:]), d))
            except ValueError:
                pass
    return [os.path.join(root, d) for _, d in sorted(steps, reverse=True)]


def latest(root: str, verify: bool = False) -> Optional[str]:
    """Newest published checkpoint; with verify, the newest whose files all
    match their crc32 in the index (a corrupted or truncated checkpoint is
    passed over for the one before it)."""
    for p in complete_steps(root):
        if not verify:
            return p
        try:
            if Checkpointer.verify(p):
                return p
        except (OSError, ValueError, KeyError):
            pass
        log.warning("checkpoint %s fails its crc32 check; trying the one before it", p)
    return None


def save_model_safetensors(state: Dict[str, torch.Tensor], path: str, dtype=None) -> None:
    """Write reference-named weights (contiguous CPU copies)."""
    out = {k: (v.to(dtype) if dtype is not None else v).detach().contiguous().cpu() for k, v in state.items()}
    save_file(out, path, metadata={"format": "lora_kernel_b200"})


def _read_safetensors(path: str, key: Optional[bytes] = None) -> Tuple[Dict[str, torch.Tensor], dict]:
    """(tensors, metadata) of a safetensors file, decrypting it first when it
    is an encrypted checkpoint file (train/crypto.py)."""
    from safetensors.torch import load as load_bytes
    from .crypto import decrypt_bytes, is_encrypted
    if is_encrypted(path):
        if key is None:
            raise ValueError(f"{path} is encrypted; set LORAK_CKPT_KEY or pass the key")
        data = decrypt_bytes(path, key)
    else:
        with open(path, "rb") as f:
            data = f.read()
    hlen = int.from_bytes(data[:8], "little")
    meta = json.loads(data[8:8 + hlen]).get("__metadata__", {}) or {}
    return load_bytes(data), meta


def load_model_safetensors(path: str, key: Optional[bytes] = None) -> Dict[str, torch.Tensor]:
    from .crypto import is_encrypted
    if is_encrypted(path):
        return _read_safetensors(path, key)[0]
    return load_file(path)


class Checkpointer:
    def __init__(self, root: str, rank: int = 0, world: int = 1, barrier=None, key: Optional[bytes] = None):
        """key: 32-byte AES-256-GCM key; every file of the checkpoint is then
        encrypted and authenticated (train/crypto.py)."""
        self.root = root
        self.rank, self.world = rank, world
        self.key = key
        self.barrier = barrier or (lambda: None)
        self._thread: Optional[threading.Thread] = None
        self._pending = None

    # ---------------------------------------------------------------- save
    def save(self, step: int, model_state: Optional[Dict[str, torch.Tensor]],
             optim_ranges: List[Tuple[int, int]], optim_tensors: Dict[str, torch.Tensor],
             layout: dict, trainer_state: dict, async_save: bool = False) -> str:
        """optim_ranges: this rank's [start, end) ranges of the flat layout, in
        the order its flat optimizer tensors concatenate them.  With
        async_save the files are written by a background thread from a host
        snapshot; the checkpoint becomes visible (index + rename) at the next
        save() or finish()."""
        self.finish()
        final = os.path.join(self.root, f"step_{step}")
        tmp = final + ".tmp"
        if self.rank == 0:
            os.makedirs(tmp, exist_ok=True)
        self.barrier()
        # snapshot to host memory now; training may continue on the device
        snap = {k: v.detach().to("cpu", non_blocking=True).contiguous() for k, v in optim_tensors.items()}
        msnap = ({k: v.detach().contiguous().to("cpu", non_blocking=True) for k, v in model_state.items()}
                 if model_state is not None else None)
        if torch.cuda.is_available():
            torch.cuda.synchronize()

        def write():
            name = f"optim-rank{self.rank}-of-{self.world}.safetensors"
            paths = [os.path.join(tmp, name)]
            save_file(snap, paths[0], metadata={"ranges": json.dumps(optim_ranges)})
            if msnap is not None:
                paths.append(os.path.join(tmp, "model.safetensors"))
                save_file(msnap, paths[1], metadata={"format": "lora_kernel_b200"})
            if self.key is not None:
                from .crypto import encrypt_file
                for p in paths:
                    encrypt_file(p, p, self.key)

        self._pending = (tmp, final, step, layout, trainer_state)
        if async_save:
            self._thread = threading.Thread(target=write, daemon=True)
            self._thread.start()
        else:
            write()
            self.finish()
        return final

    def finish(self) -> None:
        """Complete a pending save: join the writer, then publish atomically."""
        pending = getattr(self, "_pending", None)
        if pending is None:
            return
        self.wait()
        self.barrier()
        tmp, final, step, layout, trainer_state = pending
        if self.rank == 0:
            files = sorted(f for f in os.listdir(tmp) if f.endswith(".safetensors"))
            index = {"world": self.world, "step": step, "layout": layout, "encrypted": self.key is not None,
                     "files": {f: {"crc32": _crc(os.path.join(tmp, f))} for f in files}}
            with open(os.path.join(tmp, "trainer.json"), "w") as f:
                json.dump(trainer_state, f, indent=1, default=str)
            with open(os.path.join(tmp, "index.json"), "w") as f:
                json.dump(index, f, indent=1)
            if os.path.exists(final):
                shutil.rmtree(final)
            os.replace(tmp, final)
        self.barrier()
        self._pending = None

    def wait(self) -> None:
        if self._thread is not None:
            self._thread.join()
            self._thread = None

    # ---------------------------------------------------------------- load
    @staticmethod
    def verify(path: str) -> bool:
        with open(os.path.join(path, "index.json")) as f:
            index = json.load(f)
        return all(_crc(os.path.join(path, n)) == m["crc32"] for n, m in index["files"].items())

    @staticmethod
    def load_flat(path: str, names=("p32", "m", "v"), total: Optional[int] = None,
                  key: Optional[bytes] = None) -> Dict[str, torch.Tensor]:
        """Full flat optimizer vectors reassembled from every rank's file."""
        with open(os.path.join(path, "index.json")) as f:
            index = json.load(f)
        total = total or int(index["layout"]["total"])
        out: Dict[str, torch.Tensor] = {}
        for fname in sorted(index["files"]):
            if not fname.startswith("optim-rank"):
                continue
            tensors, meta = _read_safetensors(os.path.join(path, fname), key)
            ranges = json.loads(meta["ranges"])
            for n, t in tensors.items():
                if n == "state":
                    out.setdefault("state", t)
                    continue
                full = out.setdefault(n, torch.zeros(total, dtype=t.dtype))
                o = 0
                for s, e in ranges:
                    full[s:e] = t[o:o + e - s]
                    o += e - s
        return out

    @staticmethod
    def trainer_state(path: str) -> dict:
        with open(os.path.join(path, "trainer.json")) as f:
            return json.load(f)
