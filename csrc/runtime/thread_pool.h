// Work-stealing thread pool for the host runtime (data loading, checkpoint
// packing, checksums).
//
// Every worker owns a deque: it pushes and pops its own tasks at the back
// (LIFO, cache-warm) and, when empty, steals from the front of another
// worker's deque (FIFO, the oldest and usually largest piece of work).
// Tasks submitted from outside the pool are spread round-robin over the
// deques.  parallel_for splits a range into grains that the caller and the
// workers claim from one atomic counter, so a blocked caller does useful work
// instead of waiting; the first exception thrown by a grain is rethrown in
// the caller once every grain has finished.
//
// Reference: WorkStealingScheduler (include/core/scheduler.hpp:7-33), which
// keeps per-worker vectors but has no threads and no locking.
#pragma once

#include <atomic>
#include <condition_variable>
#include <cstdint>
#include <deque>
#include <exception>
#include <functional>
#include <memory>
#include <mutex>
#include <thread>
#include <vector>

namespace lkrt {

class WorkStealingPool {
 public:
  using Task = std::function<void()>;

  explicit WorkStealingPool(int n_threads);
  ~WorkStealingPool();
  WorkStealingPool(const WorkStealingPool&) = delete;
  WorkStealingPool& operator=(const WorkStealingPool&) = delete;

  // Queue one task (any thread).  Exceptions escaping a submitted task are
  // counted and dropped; use parallel_for for work whose errors matter.
  void submit(Task fn);

  // fn(begin, end) over [0, n) in grains of `grain`; returns when all grains
  // are done, rethrowing the first exception.  The caller takes part.
  void parallel_for(int64_t n, int64_t grain, const std::function<void(int64_t, int64_t)>& fn);

  // Block until no task is queued or running.
  void wait_idle();

  int size() const { return (int)workers_.size(); }
  uint64_t steals() const { return steals_.load(std::memory_order_relaxed); }
  uint64_t executed() const { return executed_.load(std::memory_order_relaxed); }
  uint64_t task_errors() const { return errors_.load(std::memory_order_relaxed); }

 private:
  struct Queue {
    std::mutex m;
    std::deque<Task> q;
  };
  void worker_loop(int id);
  bool try_pop_local(int id, Task& out);
  bool try_steal(int thief, Task& out);
  void run(Task& t);

  std::vector<std::unique_ptr<Queue>> queues_;
  std::vector<std::thread> workers_;
  std::mutex sleep_m_;
  std::condition_variable sleep_cv_;
  std::condition_variable idle_cv_;
  std::atomic<int64_t> queued_{0};
  std::atomic<int64_t> running_{0};
  std::atomic<uint64_t> rr_{0};
  std::atomic<uint64_t> steals_{0};
  std::atomic<uint64_t> executed_{0};
  std::atomic<uint64_t> errors_{0};
  std::atomic<bool> stop_{false};
};

}  // namespace lkrt
