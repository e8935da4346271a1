#!/usr/bin/env bash
# Build the native host runtime's self-test twice -- under AddressSanitizer +
# UndefinedBehaviorSanitizer, and under ThreadSanitizer -- and run both.  Any
# sanitizer report fails the run (halt_on_error / exitcode), as does a failed
# check.  Usage: csrc/runtime/test/sanitize.sh [build-dir]   (default build/sanitize)
set -euo pipefail
here="$(cd "$(dirname "$0")" && pwd)"
rt="$(dirname "$here")"
out="${1:-$(cd "$rt/../.." && pwd)/build/sanitize}"
mkdir -p "$out"
# the first compiler that can link both sanitizer runtimes (a wrapper toolchain may lack them)
probe="$out/probe.cpp"
echo 'int main() { return 0; }' > "$probe"
CXX_SAN=""
for cand in "${CXX:-}" g++ /usr/bin/g++ clang++; do
  [ -n "$cand" ] && command -v "$cand" > /dev/null || continue
  if "$cand" -fsanitize=address,undefined "$probe" -o "$out/probe_asan" 2> /dev/null &&
     "$cand" -fsanitize=thread "$probe" -o "$out/probe_tsan" 2> /dev/null; then
    CXX_SAN="$cand"
    break
  fi
done
[ -n "$CXX_SAN" ] || { echo "no C++ compiler here links -fsanitize=address,undefined and thread" >&2; exit 2; }
CXX="$CXX_SAN"
srcs=("$here/runtime_selftest.cpp" "$rt/thread_pool.cpp" "$rt/host_arena.cpp" "$rt/token_loader.cpp" "$rt/crc32.cpp")
common=(-std=c++17 -O1 -g -fno-omit-frame-pointer -pthread -I"$rt")

"$CXX" "${common[@]}" -fsanitize=address,undefined -fno-sanitize-recover=undefined "${srcs[@]}" -o "$out/selftest_asan"
ASAN_OPTIONS=detect_leaks=1:halt_on_error=1:abort_on_error=0 UBSAN_OPTIONS=print_stacktrace=1:halt_on_error=1 \
  "$out/selftest_asan"

"$CXX" "${common[@]}" -fsanitize=thread "${srcs[@]}" -o "$out/selftest_tsan"
TSAN_OPTIONS=halt_on_error=1:exitcode=66 "$out/selftest_tsan"
echo "sanitizers clean: asan+ubsan, tsan"
