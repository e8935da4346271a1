#include "token_loader.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <chrono>
#include <cstring>
#include <stdexcept>

namespace lkrt {

namespace {

// splitmix64 finaliser (Steele, Lea & Flood, "Fast splittable pseudorandom
// number generators", 2014): a bijective 64-bit mixer.
inline uint64_t mix64(uint64_t z) {
  z += 0x9e3779b97f4a7c15ull;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

inline uint64_t hash3(uint64_t a, uint64_t b, uint64_t c) { return mix64(mix64(mix64(a) ^ b) ^ c); }

// uniform in [0, n) from 32 random bits (Lemire's multiply-shift reduction)
inline uint64_t below(uint64_t x, uint64_t n) { return ((x >> 32) * n) >> 32; }

}  // namespace

TokenLoader::TokenLoader(const TokenLoaderConfig& cfg) : cfg_(cfg) {
  if (cfg_.batch <= 0 || cfg_.seq <= 0) throw std::invalid_argument("TokenLoader: batch and seq must be positive");
  if (cfg_.world <= 0 || cfg_.rank < 0 || cfg_.rank >= cfg_.world) throw std::invalid_argument("TokenLoader: bad rank/world");
  if (cfg_.depth < 1) throw std::invalid_argument("TokenLoader: depth must be >= 1");
  if (cfg_.vocab <= 0 || cfg_.vocab > (int64_t)UINT32_MAX) throw std::invalid_argument("TokenLoader: vocab out of range");

  if (!cfg_.path.empty()) {
    if (cfg_.token_bytes != 2 && cfg_.token_bytes != 4) throw std::invalid_argument("TokenLoader: token_bytes must be 2 or 4");
    const int fd = open(cfg_.path.c_str(), O_RDONLY);
    if (fd < 0) throw std::runtime_error("TokenLoader: cannot open " + cfg_.path);
    struct stat st;
    if (fstat(fd, &st) != 0) {
      close(fd);
      throw std::runtime_error("TokenLoader: cannot stat " + cfg_.path);
    }
    map_bytes_ = (size_t)st.st_size;
    ntok_ = (int64_t)(map_bytes_ / cfg_.token_bytes);
    if (ntok_ < cfg_.seq + 1) {
      close(fd);
      throw std::runtime_error("TokenLoader: " + cfg_.path + " holds fewer than seq+1 tokens");
    }
    void* p = mmap(nullptr, map_bytes_, PROT_READ, MAP_SHARED, fd, 0);
    close(fd);
    if (p == MAP_FAILED) throw std::runtime_error("TokenLoader: mmap failed for " + cfg_.path);
    madvise(p, map_bytes_, cfg_.shuffle ? MADV_RANDOM : MADV_SEQUENTIAL);
    map_ = (const uint8_t*)p;
    nwin_ = (ntok_ - 1) / cfg_.seq;
    int bits = 2;
    while ((int64_t(1) << bits) < nwin_) ++bits;
    if (bits & 1) ++bits;
    half_bits_ = bits / 2;
  }

  const size_t n = (size_t)cfg_.batch * cfg_.seq;
  slot_bytes_ = 2 * n * sizeof(int64_t);
  const size_t stride = (slot_bytes_ + 255) / 256 * 256;
  arena_.reset(new HostArena(stride * cfg_.depth));
  for (int s = 0; s < cfg_.depth; ++s) slots_.push_back((int64_t*)arena_->allocate(slot_bytes_));
  pool_.reset(new WorkStealingPool(cfg_.threads));
  state_.assign(cfg_.depth, FREE);
  batch_of_.assign(cfg_.depth, -1);
  thread_ = std::thread([this] { coordinator(); });
}

TokenLoader::~TokenLoader() {
  {
    std::lock_guard<std::mutex> g(m_);
    stop_ = true;
  }
  cv_.notify_all();
  thread_.join();
  pool_.reset();
  if (map_) munmap((void*)map_, map_bytes_);
}

int64_t* TokenLoader::ids(int slot) const { return slots_.at(slot); }
int64_t* TokenLoader::targets(int slot) const { return slots_.at(slot) + (size_t)cfg_.batch * cfg_.seq; }

int64_t TokenLoader::slot_batch(int slot) const {
  std::lock_guard<std::mutex> g(m_);
  return batch_of_.at(slot);
}

int64_t TokenLoader::cursor() const {
  std::lock_guard<std::mutex> g(m_);
  return consume_next_;
}

int64_t TokenLoader::window_of(int64_t sample) const {
  if (nwin_ <= 0) return -1;
  const int64_t epoch = sample / nwin_;
  uint64_t x = (uint64_t)(sample % nwin_);
  if (!cfg_.shuffle || nwin_ == 1) return (int64_t)x;
  const uint64_t mask = (uint64_t(1) << half_bits_) - 1;
  // balanced Feistel network on 2*half_bits bits (a bijection for any round
  // function), cycle-walked until the value lands inside [0, windows)
  do {
    uint64_t L = x >> half_bits_, R = x & mask;
    for (int round = 0; round < 4; ++round) {
      const uint64_t F = hash3(cfg_.seed ^ 0x5bd1e995ull, (uint64_t)epoch * 4 + round, R) & mask;
      const uint64_t nl = R;
      R = L ^ F;
      L = nl;
    }
    x = (L << half_bits_) | R;
  } while (x >= (uint64_t)nwin_);
  return (int64_t)x;
}

void TokenLoader::fill_row(int64_t sample, int64_t* ids, int64_t* tgt) const {
  const int S = cfg_.seq;
  if (!map_) {
    uint64_t prev = below(hash3(cfg_.seed, (uint64_t)sample, 0), (uint64_t)cfg_.vocab);
    for (int t = 0; t < S; ++t) {
      const uint64_t nxt = below(hash3(cfg_.seed, (uint64_t)sample, (uint64_t)t + 1), (uint64_t)cfg_.vocab);
      ids[t] = (int64_t)prev;
      tgt[t] = (int64_t)nxt;
      prev = nxt;
    }
    return;
  }
  const int64_t start = window_of(sample) * S;
  auto tok = [&](int64_t i) -> int64_t {
    if (cfg_.token_bytes == 2) {
      uint16_t v;
      std::memcpy(&v, map_ + (size_t)i * 2, 2);
      return v;
    }
    uint32_t v;
    std::memcpy(&v, map_ + (size_t)i * 4, 4);
    return v;
  };
  int64_t prev = tok(start);
  for (int t = 0; t < S; ++t) {
    const int64_t nxt = tok(start + t + 1);
    if (prev >= cfg_.vocab || nxt >= cfg_.vocab)
      throw std::runtime_error("TokenLoader: token id " + std::to_string(prev >= cfg_.vocab ? prev : nxt) +
                               " at position " + std::to_string(start + t) + " is not below vocab " +
                               std::to_string(cfg_.vocab));
    ids[t] = prev;
    tgt[t] = nxt;
    prev = nxt;
  }
}

void TokenLoader::fill(int slot, int64_t batch) {
  const int64_t b = cfg_.fixed ? 0 : batch;
  int64_t* ids = this->ids(slot);
  int64_t* tgt = this->targets(slot);
  const int S = cfg_.seq;
  const int64_t first = (b * cfg_.world + cfg_.rank) * cfg_.batch;
  pool_->parallel_for(cfg_.batch, 1, [&](int64_t r0, int64_t r1) {
    for (int64_t r = r0; r < r1; ++r) fill_row(first + r, ids + r * S, tgt + r * S);
  });
}

void TokenLoader::coordinator() {
  std::unique_lock<std::mutex> lk(m_);
  for (;;) {
    cv_.wait(lk, [&] {
      return stop_ || (error_.empty() && produce_next_ < consume_next_ + cfg_.depth &&
                       state_[produce_next_ % cfg_.depth] == FREE);
    });
    if (stop_) return;
    const int64_t b = produce_next_++;
    const int s = (int)(b % cfg_.depth);
    state_[s] = FILLING;
    batch_of_[s] = b;
    const uint64_t gen = generation_;
    lk.unlock();
    std::string err;
    try {
      fill(s, b);
    } catch (const std::exception& e) {
      err = e.what();
    }
    lk.lock();
    if (gen != generation_) {
      state_[s] = FREE;  // a seek happened while filling: drop the batch
    } else if (!err.empty()) {
      state_[s] = FREE;
      error_ = err;
    } else {
      state_[s] = READY;
    }
    cv_.notify_all();
  }
}

int TokenLoader::acquire(int64_t timeout_ms) {
  std::unique_lock<std::mutex> lk(m_);
  const int64_t want = consume_next_;
  const int s = (int)(want % cfg_.depth);
  auto ready = [&] { return !error_.empty() || (state_[s] == READY && batch_of_[s] == want); };
  if (timeout_ms < 0) {
    cv_.wait(lk, ready);
  } else if (!cv_.wait_for(lk, std::chrono::milliseconds(timeout_ms), ready)) {
    return -1;
  }
  if (!error_.empty()) throw std::runtime_error(error_);
  state_[s] = HELD;
  ++consume_next_;
  cv_.notify_all();
  return s;
}

void TokenLoader::release(int slot) {
  std::lock_guard<std::mutex> g(m_);
  if (slot < 0 || slot >= cfg_.depth || state_[slot] != HELD)
    throw std::invalid_argument("TokenLoader: release of a slot that is not held");
  state_[slot] = FREE;
  cv_.notify_all();
}

void TokenLoader::seek(int64_t cursor) {
  if (cursor < 0) throw std::invalid_argument("TokenLoader: negative cursor");
  std::lock_guard<std::mutex> g(m_);
  ++generation_;
  for (int s = 0; s < cfg_.depth; ++s)
    if (state_[s] == READY) state_[s] = FREE;
  consume_next_ = produce_next_ = cursor;
  error_.clear();
  cv_.notify_all();
}

}  // namespace lkrt
