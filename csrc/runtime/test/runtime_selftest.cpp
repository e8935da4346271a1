// Stand-alone self-test of the native host runtime (no torch, no CUDA), built
// under AddressSanitizer + UndefinedBehaviorSanitizer and, separately,
// ThreadSanitizer by csrc/runtime/test/sanitize.sh.  It drives every class the
// way the Python side does (and harder: many more tasks, seeks while filling,
// exceptions inside parallel_for, arena exhaustion) so that the sanitizers see
// the concurrent paths.  Exit code 0 and the line "runtime selftest ok" mean
// every check passed and no sanitizer report was raised.
//
// Reference: none (the reference has no sanitizer configuration); this keeps
// the native host code ASan / UBSan / TSan clean in CI.
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <numeric>
#include <stdexcept>
#include <string>
#include <vector>

#include "../crc32.h"
#include "../host_arena.h"
#include "../thread_pool.h"
#include "../token_loader.h"

namespace {

int g_failures = 0;

#define CHECK(cond)                                                        \
  do {                                                                     \
    if (!(cond)) {                                                         \
      std::fprintf(stderr, "%s:%d: check failed: %s\n", __FILE__, __LINE__, #cond); \
      ++g_failures;                                                        \
    }                                                                      \
  } while (0)

// bitwise CRC-32 (reflected 0xEDB88320), the definition the fast path must match
uint32_t crc_bitwise(const uint8_t* p, size_t n) {
  uint32_t c = 0xFFFFFFFFu;
  for (size_t i = 0; i < n; ++i) {
    c ^= p[i];
    for (int k = 0; k < 8; ++k) c = (c >> 1) ^ (0xEDB88320u & (0u - (c & 1u)));
  }
  return c ^ 0xFFFFFFFFu;
}

void test_pool() {
  lkrt::WorkStealingPool pool(4);
  // many small submitted tasks, some of which submit more work
  std::atomic<int64_t> sum{0};
  for (int i = 0; i < 2000; ++i) {
    pool.submit([&pool, &sum, i] {
      sum += i;
      if (i % 10 == 0) pool.submit([&sum] { sum += 1; });
    });
  }
  pool.wait_idle();
  CHECK(sum.load() == 1999LL * 2000 / 2 + 200);
  // parallel_for covers the range exactly once
  std::vector<int> hits(100000, 0);
  pool.parallel_for((int64_t)hits.size(), 97, [&](int64_t b, int64_t e) {
    for (int64_t i = b; i < e; ++i) hits[i] += 1;
  });
  CHECK(std::all_of(hits.begin(), hits.end(), [](int h) { return h == 1; }));
  // the first exception of a grain reaches the caller after every grain ran
  std::atomic<int> ran{0};
  bool caught = false;
  try {
    pool.parallel_for(64, 1, [&](int64_t b, int64_t) {
      ++ran;
      if (b == 17) throw std::runtime_error("grain 17");
    });
  } catch (const std::runtime_error& e) {
    caught = std::string(e.what()) == "grain 17";
  }
  CHECK(caught);
  CHECK(ran.load() == 64);
  // a throwing submitted task is counted, not fatal
  const uint64_t before = pool.task_errors();
  pool.submit([] { throw std::runtime_error("dropped"); });
  pool.wait_idle();
  CHECK(pool.task_errors() == before + 1);
  // nested parallel_for from inside a task does not deadlock
  std::atomic<int64_t> nested{0};
  pool.parallel_for(8, 1, [&](int64_t, int64_t) {
    pool.parallel_for(100, 7, [&](int64_t b, int64_t e) { nested += e - b; });
  });
  CHECK(nested.load() == 800);
}

void test_arena() {
  lkrt::HostArena arena(1 << 20);
  void* a = arena.allocate(100);
  void* b = arena.allocate(1000, 4096);
  CHECK(a != nullptr && b != nullptr);
  CHECK(reinterpret_cast<uintptr_t>(a) % 256 == 0);
  CHECK(reinterpret_cast<uintptr_t>(b) % 4096 == 0);
  std::memset(a, 1, 100);
  std::memset(b, 2, 1000);
  CHECK(arena.allocate(2 << 20) == nullptr);  // exhaustion is a null, not an overrun
  CHECK(arena.allocations() == 2);
  const size_t peak = arena.peak();
  arena.reset();
  CHECK(arena.used() == 0 && arena.peak() == peak);
  // concurrent allocations never overlap
  lkrt::WorkStealingPool pool(4);
  std::vector<uint8_t*> ptrs(512, nullptr);
  pool.parallel_for(512, 1, [&](int64_t b, int64_t e) {
    for (int64_t i = b; i < e; ++i) {
      ptrs[i] = static_cast<uint8_t*>(arena.allocate(1024));
      if (ptrs[i]) std::memset(ptrs[i], (int)(i & 0xFF), 1024);
    }
  });
  for (int i = 0; i < 512; ++i) {
    CHECK(ptrs[i] != nullptr);
    if (ptrs[i]) CHECK(ptrs[i][0] == (uint8_t)(i & 0xFF) && ptrs[i][1023] == (uint8_t)(i & 0xFF));
  }
}

void test_crc() {
  std::vector<uint8_t> buf(3 * 1000 * 1000 + 17);
  uint32_t x = 12345;
  for (auto& v : buf) {
    x = x * 1664525u + 1013904223u;
    v = (uint8_t)(x >> 24);
  }
  const uint32_t want = crc_bitwise(buf.data(), buf.size());
  CHECK(lkrt::crc32_update(0, buf.data(), buf.size()) == want);
  lkrt::WorkStealingPool pool(3);
  CHECK(lkrt::crc32_parallel(buf.data(), buf.size(), pool, 4096) == want);
  CHECK(lkrt::crc32_parallel(buf.data(), buf.size(), pool, 1 << 20) == want);
  const size_t cut = 777777;
  const uint32_t a = lkrt::crc32_update(0, buf.data(), cut);
  const uint32_t b = lkrt::crc32_update(0, buf.data() + cut, buf.size() - cut);
  CHECK(lkrt::crc32_combine(a, b, buf.size() - cut) == want);
  const char* s = "123456789";
  CHECK(lkrt::crc32_update(0, s, 9) == 0xCBF43926u);  // the standard check value
}

std::string write_tokens(int n, int bytes) {
  char path[] = "/tmp/lkrt_selftest_XXXXXX";
  const int fd = mkstemp(path);
  if (fd < 0) throw std::runtime_error("mkstemp failed");
  std::vector<uint8_t> data((size_t)n * bytes);
  for (int i = 0; i < n; ++i) {
    const uint32_t v = (uint32_t)(i % 1000);
    std::memcpy(&data[(size_t)i * bytes], &v, bytes);
  }
  const ssize_t w = ::write(fd, data.data(), data.size());
  ::close(fd);
  if (w != (ssize_t)data.size()) throw std::runtime_error("short write");
  return path;
}

void test_loader_synthetic() {
  lkrt::TokenLoaderConfig c;
  c.vocab = 5000;
  c.batch = 3;
  c.seq = 64;
  c.seed = 7;
  c.depth = 3;
  c.threads = 3;
  lkrt::TokenLoader ld(c);
  const int n = c.batch * c.seq;
  std::vector<int64_t> batch5;
  for (int step = 0; step < 30; ++step) {
    const int s = ld.acquire(10000);
    CHECK(s >= 0);
    if (s < 0) return;
    CHECK(ld.slot_batch(s) == step);
    const int64_t* ids = ld.ids(s);
    const int64_t* tg = ld.targets(s);
    for (int i = 0; i < n; ++i) {
      CHECK(ids[i] >= 0 && ids[i] < c.vocab);
      if (i % c.seq != c.seq - 1) CHECK(tg[i] == ids[i + 1]);
    }
    if (step == 5) batch5.assign(ids, ids + n);
    ld.release(s);
  }
  // resume at batch 5 while the workers are filling ahead: the same tokens again
  ld.seek(5);
  for (int step = 5; step < 12; ++step) {
    const int s = ld.acquire(10000);
    CHECK(s >= 0);
    if (s < 0) return;
    CHECK(ld.slot_batch(s) == step);
    if (step == 5) CHECK(std::equal(batch5.begin(), batch5.end(), ld.ids(s)));
    ld.release(s);
  }
  CHECK(ld.cursor() == 12);
}

void test_loader_file() {
  for (int bytes : {2, 4}) {
    const std::string path = write_tokens(20000, bytes);
    for (int rank = 0; rank < 2; ++rank) {
      lkrt::TokenLoaderConfig c;
      c.path = path;
      c.token_bytes = bytes;
      c.vocab = 1000;
      c.batch = 2;
      c.seq = 32;
      c.rank = rank;
      c.world = 2;
      c.seed = 3;
      c.depth = 2;
      c.threads = 2;
      c.shuffle = true;
      lkrt::TokenLoader ld(c);
      // the shuffled window order is a permutation of the windows
      std::vector<int> seen(ld.num_windows(), 0);
      for (int64_t sidx = 0; sidx < ld.num_windows(); ++sidx) {
        const int64_t w = ld.window_of(sidx);
        CHECK(w >= 0 && w < ld.num_windows());
        if (w >= 0 && w < ld.num_windows()) seen[w] += 1;
      }
      CHECK(std::all_of(seen.begin(), seen.end(), [](int v) { return v == 1; }));
      for (int step = 0; step < 25; ++step) {
        const int s = ld.acquire(10000);
        CHECK(s >= 0);
        if (s < 0) break;
        const int64_t* ids = ld.ids(s);
        const int64_t* tg = ld.targets(s);
        for (int i = 0; i < c.batch * c.seq; ++i) {
          // the file holds i % 1000, so every target is the next id mod 1000
          CHECK(tg[i] == (ids[i] + 1) % 1000);
        }
        ld.release(s);
      }
    }
    ::unlink(path.c_str());
  }
  // an id outside the vocabulary is reported, not read past
  const std::string path = write_tokens(5000, 2);
  lkrt::TokenLoaderConfig c;
  c.path = path;
  c.vocab = 10;
  c.batch = 1;
  c.seq = 16;
  c.depth = 2;
  c.threads = 1;
  bool threw = false;
  try {
    lkrt::TokenLoader ld(c);
    const int s = ld.acquire(10000);
    if (s >= 0) ld.release(s);
  } catch (const std::exception&) {
    threw = true;
  }
  CHECK(threw);
  ::unlink(path.c_str());
}

}  // namespace

int main() {
  test_pool();
  test_arena();
  test_crc();
  test_loader_synthetic();
  test_loader_file();
  if (g_failures) {
    std::fprintf(stderr, "runtime selftest: %d check(s) failed\n", g_failures);
    return 1;
  }
  std::printf("runtime selftest ok\n");
  return 0;
}
