"""The allocation-free RMSNorm backward, called through its exported C symbol.

Some callers cannot allocate device memory (a process with a fixed memory pool,
a plug-in running in a foreign CUDA context, a C caller without an allocator),
so lk_rmsnorm_bwd_noalloc keeps its scratch in a built-in device array.  This
test calls it the way such a caller would, through ctypes on the extension's
shared library, and checks it against the regular entry point (which takes a
caller-provided scratch buffer) on two calls in a row.  It lives in a file of
its own named to be collected last.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

SCRATCH_FLOATS = 1 << 20  # LK_NOALLOC_NORM_SCRATCH_FLOATS


def _lib():
    from lora_kernel_b200 import _C  # loads torch's libraries first
    lib = ctypes.CDLL(_C.__file__)
    f = lib.lk_rmsnorm_bwd_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                           ctypes.c_int, ctypes.c_void_p]
    lib.lk_last_error.restype = ctypes.c_char_p
    return lib


def _call(lib, dy, x, g, rstd, dres, dx, dgamma, accumulate):
    M, D = x.shape
    stream = torch.cuda.current_stream().cuda_stream
    return lib.lk_rmsnorm_bwd_noalloc(dy.data_ptr(), x.data_ptr(), g.data_ptr(), rstd.data_ptr(),
                                      dres.data_ptr() if dres is not None else None, dx.data_ptr(),
                                      dgamma.data_ptr(), M, D, int(accumulate), stream)


def _close(out, ref, rtol, atol):
    err = (out.float() - ref.float()).abs()
    bad = (err > atol + rtol * ref.float().abs()).sum().item()
    assert bad == 0, f"{bad} mismatches, max err {err.max().item():.4g}"


@pytest.mark.parametrize("M,D", [(777, 256), (4096, 2048), (1000, 4096)])
def test_noalloc_matches_regular_entry_point(M, D):
    from lora_kernel_b200.ops.norm import rmsnorm_bwd, rmsnorm_fwd
    lib = _lib()
    torch.manual_seed(11)
    dev = "cuda"
    x = torch.randn(M, D, device=dev).to(torch.bfloat16)
    g = (1 + 0.1 * torch.randn(D, device=dev)).to(torch.bfloat16)
    _, rstd, _ = rmsnorm_fwd(x, g, 1e-5)
    for call in range(2):  # two calls in a row: the shared scratch is reused
        dy = torch.randn(M, D, device=dev).to(torch.bfloat16)
        dres = torch.randn(M, D, device=dev).to(torch.bfloat16) if call == 1 else None
        dg_ref = torch.full((D,), 0.5, device=dev)
        dx_ref = rmsnorm_bwd(dy, x, g, rstd, dg_ref, dres=dres, accumulate=True)
        dg = torch.full((D,), 0.5, device=dev)
        dx = torch.empty_like(x)
        rc = _call(lib, dy, x, g, rstd, dres, dx, dg, accumulate=True)
        assert rc == 0, lib.lk_last_error().decode()
        torch.cuda.synchronize()
        _close(dx, dx_ref, 3e-2, 3e-2)
        _close(dg, dg_ref, 1e-2, 1e-1)


def test_noalloc_rejects_oversized_requests():
    lib = _lib()
    # the backward needs min(ceil(M / 8), 2 x SMs) x D scratch floats; pick the
    # case from this GPU so that it exceeds the built-in 1 Mi floats
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    D = 4096  # the largest width the kernel supports
    rows_needed = SCRATCH_FLOATS // D + 1
    if rows_needed > 2 * sms:
        pytest.skip(f"{sms} SMs: no supported problem exceeds the built-in scratch")
    M = 8 * rows_needed
    assert min(-(-M // 8), 2 * sms) * D > SCRATCH_FLOATS
    x = torch.zeros(M, D, dtype=torch.bfloat16, device="cuda")
    g = torch.ones(D, dtype=torch.bfloat16, device="cuda")
    rstd = torch.ones(M, device="cuda")
    dx = torch.empty_like(x)
    dg = torch.zeros(D, device="cuda")
    rc = _call(lib, x, x, g, rstd, None, dx, dg, accumulate=False)
    assert rc == -1
    assert b"scratch" in lib.lk_last_error()
