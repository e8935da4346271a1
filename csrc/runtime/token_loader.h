// Token batch loader: worker threads fill a ring of host slots ahead of the
// trainer, each slot holding one micro-batch as two contiguous int64 arrays
// (ids[B*S] followed by targets[B*S]) so a single host-to-device copy moves a
// step's input and the kernels read both arrays in place.
//
// Sources
//   synthetic  uniform ids in [0, vocab) from a counter-based hash of
//              (seed, sample, position): the same sample has the same tokens
//              whatever thread fills it and whatever the prefetch depth.
//   file       a flat uint16 / uint32 token file, mmap'd read-only, cut into
//              windows of S+1 tokens at stride S (neighbouring windows share
//              one token so every position is a target once).  With shuffle,
//              each epoch visits the windows in the order of a seeded Feistel
//              permutation (O(1) memory, cycle-walked onto [0, windows)).
// Data-parallel sharding: batch b of rank r holds global samples
// (b * world + r) * B + [0, B), so the ranks of one step read disjoint windows
// and an epoch covers every window once across them.
// The consumer's cursor (batches handed out) is the resume state: seek(c)
// restarts the stream at batch c.
//
// Reference: DataLoader with worker threads and a bounded SampleQueue
// (include/data/dataloader.hpp:26-159; its samples are random tokens whatever
// the file), ShardedDataset / DistributedDataLoader (include/data/datasets.hpp:7-43).
#pragma once

#include <condition_variable>
#include <cstdint>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "host_arena.h"
#include "thread_pool.h"

namespace lkrt {

struct TokenLoaderConfig {
  std::string path;     // empty: synthetic
  int token_bytes = 2;  // file element size: 2 (uint16) or 4 (uint32)
  int64_t vocab = 0;    // synthetic range; file ids must be below it
  int batch = 1;
  int seq = 1;
  int rank = 0;
  int world = 1;
  uint64_t seed = 0;
  int depth = 4;        // slots in the ring
  int threads = 4;      // fill workers
  bool shuffle = true;  // file source: permute windows per epoch
  bool fixed = false;   // every batch is batch 0
};

class TokenLoader {
 public:
  explicit TokenLoader(const TokenLoaderConfig& cfg);
  ~TokenLoader();

  // Slot of the next batch in order; blocks up to timeout_ms (<0: forever).
  // Returns -1 on timeout; throws if filling failed (e.g. an id >= vocab).
  int acquire(int64_t timeout_ms);
  void release(int slot);
  void seek(int64_t cursor);

  int64_t* ids(int slot) const;
  int64_t* targets(int slot) const;
  int64_t slot_batch(int slot) const;
  size_t slot_bytes() const { return slot_bytes_; }
  int depth() const { return cfg_.depth; }
  int64_t cursor() const;
  int64_t num_windows() const { return nwin_; }
  void* arena_base() const { return arena_->base(); }
  size_t arena_bytes() const { return arena_->capacity(); }
  const WorkStealingPool& pool() const { return *pool_; }

  // Global sample index -> the window it reads (file source); exposed for tests.
  int64_t window_of(int64_t sample) const;

 private:
  enum State : int { FREE = 0, FILLING, READY, HELD };
  void coordinator();
  void fill(int slot, int64_t batch);
  void fill_row(int64_t sample, int64_t* ids, int64_t* tgt) const;

  TokenLoaderConfig cfg_;
  std::unique_ptr<HostArena> arena_;
  std::unique_ptr<WorkStealingPool> pool_;
  std::vector<int64_t*> slots_;
  size_t slot_bytes_ = 0;

  const uint8_t* map_ = nullptr;
  size_t map_bytes_ = 0;
  int64_t ntok_ = 0;
  int64_t nwin_ = 0;
  int half_bits_ = 1;

  mutable std::mutex m_;
  std::condition_variable cv_;
  std::vector<int> state_;
  std::vector<int64_t> batch_of_;
  int64_t consume_next_ = 0;
  int64_t produce_next_ = 0;
  uint64_t generation_ = 0;
  std::string error_;
  bool stop_ = false;
  std::thread thread_;
};

}  // namespace lkrt
