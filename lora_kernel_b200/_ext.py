"""Loader for the in-tree sm_100a extension `lora_kernel_b200._C`.

There is no fallback: every op of the B200 path calls into this extension and
raises if it is missing or if the device is not an sm_100 GPU.  The per-device
int32 status word is where kernels record bounded-wait timeouts and bad
indices instead of trapping.

LK_DEBUG_BOUNDS=1 loads the bounds-checked build `lora_kernel_b200._C_debug`
instead (same sources compiled with -DLK_BOUNDS_CHECK): data-dependent indices
(KV block-table entries, cache slots) are verified on the device, a bad one is
recorded in the status word and the access is skipped.
"""
from __future__ import annotations

import os
import threading

import torch

_C = None
_lock = threading.Lock()
_status = {}

STATUS_NAMES = {
    0: "ok",
    1: "timeout waiting for a TMA stage",
    2: "timeout waiting for a free stage",
    3: "timeout waiting for the accumulator",
    4: "timeout waiting for a peer GPU",
    5: "index out of range",
    6: "timeout draining copies on abort",
}


class KernelStatusError(RuntimeError):
    pass


def C():
    """Return the compiled extension module, importing it on first use."""
    global _C
    if _C is None:
        with _lock:
            if _C is None:
                debug = os.environ.get("LK_DEBUG_BOUNDS", "0") == "1"
                try:
                    if debug:
                        from lora_kernel_b200 import _C_debug as mod  # noqa: F401
                    else:
                        from lora_kernel_b200 import _C as mod  # noqa: F401
                except ImportError as e:  # pragma: no cover - depends on the build
                    raise RuntimeError(
                        "lora_kernel_b200 CUDA extension%s is not built; run "
                        "`python setup.py build_ext --inplace` in the repository root"
                        % (" (bounds-checked _C_debug)" if debug else "")) from e
                _C = mod
    return _C


def available() -> bool:
    try:
        C()
        return True
    except RuntimeError:
        return False


def require_device(t: torch.Tensor) -> None:
    if not t.is_cuda:
        raise RuntimeError("lora_kernel_b200 ops run on CUDA tensors only")
    major, _ = torch.cuda.get_device_capability(t.device)
    if major != 10:
        raise RuntimeError("lora_kernel_b200 kernels are built for sm_100a (B200) only")


def status(device) -> torch.Tensor:
    """Per-device int32 status word shared by all kernels."""
    device = torch.device(device)
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _status.get(idx)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _status[idx] = t
    return t


def check_status(device=None, reset: bool = True) -> None:
    """Raise KernelStatusError if any kernel recorded a failure (synchronises)."""
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    t = status(device)
    code = int(t.item())
    if code != 0:
        if reset:
            t.zero_()
        raise KernelStatusError(f"kernel status {code}: {STATUS_NAMES.get(code, 'unknown')}")
