#!/usr/bin/env bash
# CPU CI: build the extension for sm_100a (cross-compiled), then the tests that need no GPU
# (fp32 oracle, layouts, gloo multi-process paths, serving contract).  GPU suites: pytest -m gpu on a B200.
set -euo pipefail
cd "$(dirname "$0")"
python -c "import __graft_entry__ as g; g.build()"
python -m pytest tests/ -x -q -m "not gpu"
# native host runtime under ASan+UBSan and TSan (also run by tests/test_runtime_sanitizers.py)
csrc/runtime/test/sanitize.sh
