"""Native host runtime (lora_kernel_b200._rt): work-stealing pool, host arena,
parallel CRC-32 and the prefetching token loader.  CPU only."""
import os
import zlib

import numpy as np
import pytest
import torch

from lora_kernel_b200 import _rt
from lora_kernel_b200.utils.data import NativeTokens


@pytest.mark.parametrize("threads", [1, 3, 8])
def test_pool_tasks_parallel_for_and_errors(threads):
    r = _rt.pool_selftest(threads, 500, 100_003)
    assert r["count"] == 500 * 4
    assert r["sum"] == 100_003 * 100_002 // 2
    assert r["raised"]
    assert r["executed"] >= 2000


@pytest.mark.parametrize("n", [0, 1, 7, 8, 4096 + 3, (8 << 20) * 2 + 12345])
def test_crc32_matches_zlib(n):
    rng = np.random.default_rng(n)
    b = rng.integers(0, 256, n, dtype=np.uint8).tobytes()
    assert _rt.crc32(b) == zlib.crc32(b)
    half = n // 3
    assert _rt.crc32(b[half:], zlib.crc32(b[:half])) == zlib.crc32(b)
    assert _rt.crc32_combine(zlib.crc32(b[:half]), zlib.crc32(b[half:]), n - half) == zlib.crc32(b)


def test_crc32_of_tensor_pointer():
    t = torch.randn(3_000_001)
    ref = zlib.crc32(t.numpy().tobytes())
    assert _rt.crc32_ptr(t.data_ptr(), t.numel() * 4) == ref


def test_parallel_copy():
    src = torch.randint(0, 255, (9 << 20,), dtype=torch.uint8)
    dst = torch.zeros_like(src)
    _rt.parallel_copy(dst.data_ptr(), src.data_ptr(), src.numel())
    assert torch.equal(src, dst)


def test_host_arena_bump_and_reset():
    a = _rt.HostArena(3 << 20)
    assert a.capacity == 4 << 20 and a.base % 4096 == 0
    p1 = a.allocate(1000)
    p2 = a.allocate(10, 1024)
    assert p1 == a.base and p2 % 1024 == 0 and p2 >= p1 + 1000
    assert a.allocate(a.capacity) == 0  # exhausted: null, not an exception
    assert a.allocations == 2
    a.reset()
    assert a.used == 0 and a.allocate(64) == a.base and a.peak >= 1010


def _take(loader, k):
    out = []
    for _ in range(k):
        x, y = loader.next()
        out.append((x.clone(), y.clone()))
    return out


def test_synthetic_loader_is_deterministic_and_shifted():
    a = _take(NativeTokens(777, 3, 64, seed=5, depth=3, threads=1, pin=False), 6)
    b = _take(NativeTokens(777, 3, 64, seed=5, depth=8, threads=6, pin=False), 6)
    for (x1, y1), (x2, y2) in zip(a, b):
        assert torch.equal(x1, x2) and torch.equal(y1, y2)
        assert torch.equal(x1[:, 1:], y1[:, :-1])
        assert int(x1.min()) >= 0 and int(x1.max()) < 777
    assert not torch.equal(a[0][0], a[1][0])
    # ranks read different samples
    r1 = _take(NativeTokens(777, 3, 64, seed=5, rank=1, world=2, pin=False), 1)
    assert not torch.equal(r1[0][0], a[0][0])
    # fixed: batch 0 every call
    f = _take(NativeTokens(777, 3, 64, seed=5, fixed=True, pin=False), 3)
    assert torch.equal(f[0][0], f[2][0]) and torch.equal(f[0][0], a[0][0])


def test_synthetic_token_histogram_is_uniform():
    l = NativeTokens(16, 8, 1024, seed=1, pin=False)
    x, _ = l.next()
    counts = torch.bincount(x.reshape(-1), minlength=16).double()
    e = x.numel() / 16
    chi2 = (((counts - e) ** 2) / e).sum().item()
    assert chi2 < 60  # 15 dof; p ~ 1e-7


def _write_tokens(path, n, dtype=np.uint16):
    data = (np.arange(n) * 7 % 50000).astype(dtype)
    data.tofile(path)
    return data


def test_file_loader_sequential_windows_and_sharding(tmp_path):
    p = str(tmp_path / "tok.bin")
    data = _write_tokens(p, 10_000)
    B, S, W = 2, 100, 2
    for rank in range(W):
        l = NativeTokens(50000, B, S, path=p, rank=rank, world=W, shuffle=False, pin=False)
        assert l.num_windows == (10_000 - 1) // S
        for b in range(3):
            x, y = l.next()
            for r in range(B):
                w = (b * W + rank) * B + r
                win = torch.from_numpy(data[w * S: w * S + S + 1].astype(np.int64))
                assert torch.equal(x[r], win[:-1]) and torch.equal(y[r], win[1:])


def test_file_loader_shuffle_is_a_permutation_per_epoch(tmp_path):
    p = str(tmp_path / "tok32.bin")
    _write_tokens(p, 5 * 37 + 1, np.uint32)
    l = NativeTokens(50000, 1, 5, path=p, dtype="uint32", seed=9, pin=False)
    n = l.num_windows
    assert n == 37
    e0 = [l._l.window_of(i) for i in range(n)]
    e1 = [l._l.window_of(n + i) for i in range(n)]
    assert sorted(e0) == list(range(n)) and sorted(e1) == list(range(n))
    assert e0 != list(range(n)) and e0 != e1


def test_file_loader_rejects_ids_beyond_vocab(tmp_path):
    p = str(tmp_path / "tok.bin")
    _write_tokens(p, 1000)
    l = NativeTokens(100, 2, 10, path=p, shuffle=False, pin=False)
    with pytest.raises(RuntimeError, match="not below vocab"):
        l.next()


def test_loader_resume_from_cursor():
    l = NativeTokens(1000, 2, 32, seed=2, pin=False)
    first = _take(l, 8)
    st = {"cursor": 5}
    l2 = NativeTokens(1000, 2, 32, seed=2, pin=False)
    _take(l2, 2)
    l2.load_state(st)
    again = _take(l2, 3)
    for (x1, _), (x2, _) in zip(first[5:8], again):
        assert torch.equal(x1, x2)
    assert l2.state()["cursor"] == 8


def test_loader_missing_file():
    with pytest.raises(RuntimeError, match="cannot open"):
        NativeTokens(10, 1, 4, path=os.path.join("/nonexistent", "x.bin"), pin=False)
