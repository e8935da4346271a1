"""The native host runtime (thread pool, host arena, token loader, CRC-32)
under AddressSanitizer + UndefinedBehaviorSanitizer and ThreadSanitizer: the
stand-alone self-test csrc/runtime/test/runtime_selftest.cpp must pass its
checks with no sanitizer report."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_runtime_is_sanitizer_clean(tmp_path):
    script = os.path.join(ROOT, "csrc", "runtime", "test", "sanitize.sh")
    r = subprocess.run(["bash", script, str(tmp_path)], capture_output=True, text=True, timeout=600)
    if r.returncode == 2 and "no C++ compiler" in r.stderr:
        pytest.skip(r.stderr.strip())
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-4000:]
    assert r.stdout.count("runtime selftest ok") == 2
    assert "sanitizers clean" in r.stdout
