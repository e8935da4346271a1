#include "thread_pool.h"

#include <algorithm>

namespace lkrt {

namespace {
thread_local const WorkStealingPool* tl_pool = nullptr;
thread_local int tl_worker = -1;
}  // namespace

WorkStealingPool::WorkStealingPool(int n_threads) {
  n_threads = std::max(1, n_threads);
  for (int i = 0; i < n_threads; ++i) queues_.emplace_back(new Queue);
  workers_.reserve(n_threads);
  for (int i = 0; i < n_threads; ++i) workers_.emplace_back([this, i] { worker_loop(i); });
}

WorkStealingPool::~WorkStealingPool() {
  {
    std::lock_guard<std::mutex> g(sleep_m_);
    stop_.store(true);
  }
  sleep_cv_.notify_all();
  for (auto& t : workers_) t.join();
}

void WorkStealingPool::submit(Task fn) {
  int q;
  if (tl_pool == this && tl_worker >= 0) {
    q = tl_worker;  // own deque: LIFO for locality
  } else {
    q = (int)(rr_.fetch_add(1, std::memory_order_relaxed) % queues_.size());
  }
  {
    std::lock_guard<std::mutex> g(queues_[q]->m);
    queues_[q]->q.push_back(std::move(fn));
  }
  queued_.fetch_add(1, std::memory_order_release);
  {
    // pairs with the predicate check under sleep_m_ in worker_loop, so a
    // worker about to sleep cannot miss this task
    std::lock_guard<std::mutex> g(sleep_m_);
  }
  sleep_cv_.notify_one();
}

bool WorkStealingPool::try_pop_local(int id, Task& out) {
  Queue& q = *queues_[id];
  std::lock_guard<std::mutex> g(q.m);
  if (q.q.empty()) return false;
  out = std::move(q.q.back());
  q.q.pop_back();
  return true;
}

bool WorkStealingPool::try_steal(int thief, Task& out) {
  const int n = (int)queues_.size();
  for (int k = 1; k < n; ++k) {
    Queue& q = *queues_[(thief + k) % n];
    std::lock_guard<std::mutex> g(q.m);
    if (q.q.empty()) continue;
    out = std::move(q.q.front());
    q.q.pop_front();
    steals_.fetch_add(1, std::memory_order_relaxed);
    return true;
  }
  return false;
}

void WorkStealingPool::run(Task& t) {
  try {
    t();
  } catch (...) {
    errors_.fetch_add(1, std::memory_order_relaxed);
  }
  executed_.fetch_add(1, std::memory_order_relaxed);
}

void WorkStealingPool::worker_loop(int id) {
  tl_pool = this;
  tl_worker = id;
  for (;;) {
    Task t;
    // running_ is raised before queued_ drops so wait_idle never sees both at zero
    // while a task is between the deque and its execution
    running_.fetch_add(1, std::memory_order_acq_rel);
    if (try_pop_local(id, t) || try_steal(id, t)) {
      queued_.fetch_sub(1, std::memory_order_acq_rel);
      run(t);
      t = nullptr;
      if (running_.fetch_sub(1, std::memory_order_acq_rel) == 1 && queued_.load() == 0) {
        std::lock_guard<std::mutex> g(sleep_m_);
        idle_cv_.notify_all();
      }
      continue;
    }
    if (running_.fetch_sub(1, std::memory_order_acq_rel) == 1 && queued_.load() == 0) {
      std::lock_guard<std::mutex> g(sleep_m_);
      idle_cv_.notify_all();
    }
    std::unique_lock<std::mutex> lk(sleep_m_);
    sleep_cv_.wait(lk, [&] { return stop_.load() || queued_.load(std::memory_order_acquire) > 0; });
    if (stop_.load() && queued_.load() == 0) return;
  }
}

void WorkStealingPool::wait_idle() {
  std::unique_lock<std::mutex> lk(sleep_m_);
  idle_cv_.wait(lk, [&] { return queued_.load() == 0 && running_.load() == 0; });
}

void WorkStealingPool::parallel_for(int64_t n, int64_t grain, const std::function<void(int64_t, int64_t)>& fn) {
  if (n <= 0) return;
  grain = std::max<int64_t>(1, grain);
  const int64_t chunks = (n + grain - 1) / grain;
  struct Shared {
    std::atomic<int64_t> next{0};
    std::atomic<int64_t> done{0};
    std::mutex m;
    std::condition_variable cv;
    std::exception_ptr err;
    std::atomic<bool> failed{false};
  };
  auto sh = std::make_shared<Shared>();
  auto body = [sh, n, grain, chunks, &fn]() {
    for (;;) {
      const int64_t c = sh->next.fetch_add(1, std::memory_order_relaxed);
      if (c >= chunks) return;
      if (!sh->failed.load(std::memory_order_relaxed)) {
        try {
          fn(c * grain, std::min(n, (c + 1) * grain));
        } catch (...) {
          std::lock_guard<std::mutex> g(sh->m);
          if (!sh->err) sh->err = std::current_exception();
          sh->failed.store(true);
        }
      }
      if (sh->done.fetch_add(1, std::memory_order_acq_rel) + 1 == chunks) {
        std::lock_guard<std::mutex> g(sh->m);
        sh->cv.notify_all();
      }
    }
  };
  // helpers never outlive this call: they only touch fn while a grain is
  // unclaimed, and the caller returns after every grain is done
  const int64_t helpers = std::min<int64_t>(chunks - 1, (int64_t)workers_.size());
  for (int64_t i = 0; i < helpers; ++i) submit(body);
  body();
  {
    std::unique_lock<std::mutex> lk(sh->m);
    sh->cv.wait(lk, [&] { return sh->done.load() == chunks; });
  }
  if (sh->err) std::rethrow_exception(sh->err);
}

}  // namespace lkrt
