// Python bindings of the host runtime (module lora_kernel_b200._rt).
// Blocking calls release the GIL so loader threads and the training loop run
// side by side.
#include <torch/extension.h>

#include <atomic>
#include <cstring>
#include <stdexcept>

#include "crc32.h"
#include "host_arena.h"
#include "thread_pool.h"
#include "token_loader.h"

namespace py = pybind11;
using namespace lkrt;

namespace {

WorkStealingPool& default_pool() {
  static WorkStealingPool pool((int)std::max(1u, std::min(16u, std::thread::hardware_concurrency())));
  return pool;
}

// Exercises the pool the way its users do: tasks that spawn tasks (stealing),
// a parallel_for reduction, and an exception thrown by one grain.
py::dict pool_selftest(int threads, int64_t tasks, int64_t n) {
  WorkStealingPool pool(threads);
  std::atomic<int64_t> count{0};
  {
    py::gil_scoped_release nogil;
    for (int64_t i = 0; i < tasks; ++i) {
      pool.submit([&pool, &count] {
        count.fetch_add(1);
        for (int c = 0; c < 3; ++c) pool.submit([&count] { count.fetch_add(1); });
      });
    }
    pool.wait_idle();
  }
  std::atomic<int64_t> sum{0};
  {
    py::gil_scoped_release nogil;
    pool.parallel_for(n, 7, [&](int64_t a, int64_t b) {
      int64_t s = 0;
      for (int64_t i = a; i < b; ++i) s += i;
      sum.fetch_add(s);
    });
  }
  bool raised = false;
  try {
    py::gil_scoped_release nogil;
    pool.parallel_for(n, 5, [&](int64_t a, int64_t b) {
      if (a <= n / 2 && n / 2 < b) throw std::runtime_error("grain failure");
    });
  } catch (const std::runtime_error&) {
    raised = true;
  }
  py::dict d;
  d["count"] = count.load();
  d["sum"] = sum.load();
  d["raised"] = raised;
  d["steals"] = pool.steals();
  d["executed"] = pool.executed();
  return d;
}

uint32_t crc32_ptr(int64_t ptr, int64_t nbytes, uint32_t crc) {
  if (nbytes < 0) throw std::invalid_argument("crc32: negative size");
  py::gil_scoped_release nogil;
  const uint32_t c = crc32_parallel((const void*)ptr, (size_t)nbytes, default_pool());
  return crc == 0 ? c : crc32_combine(crc, c, (uint64_t)nbytes);
}

uint32_t crc32_buffer(py::buffer b, uint32_t crc) {
  py::buffer_info info = b.request();
  const int64_t nbytes = info.size * info.itemsize;
  return crc32_ptr((int64_t)info.ptr, nbytes, crc);
}

void parallel_copy(int64_t dst, int64_t src, int64_t nbytes) {
  if (nbytes <= 0) return;
  py::gil_scoped_release nogil;
  const int64_t grain = 4 << 20;
  default_pool().parallel_for((nbytes + grain - 1) / grain, 1, [&](int64_t c0, int64_t c1) {
    for (int64_t c = c0; c < c1; ++c) {
      const int64_t off = c * grain;
      std::memcpy((char*)dst + off, (const char*)src + off, (size_t)std::min(grain, nbytes - off));
    }
  });
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "lora_kernel_b200 host runtime: work-stealing pool, host arena, token loader, CRC-32";

  m.def("pool_selftest", &pool_selftest, py::arg("threads"), py::arg("tasks"), py::arg("n"));
  m.def("crc32_ptr", &crc32_ptr, py::arg("ptr"), py::arg("nbytes"), py::arg("crc") = 0u);
  m.def("crc32", &crc32_buffer, py::arg("buffer"), py::arg("crc") = 0u);
  m.def("crc32_combine", &crc32_combine);
  m.def("parallel_copy", &parallel_copy, py::arg("dst"), py::arg("src"), py::arg("nbytes"));
  m.def("default_pool_size", [] { return default_pool().size(); });

  py::class_<HostArena>(m, "HostArena")
      .def(py::init<size_t>())
      .def("allocate", [](HostArena& a, size_t n, size_t align) { return (int64_t)a.allocate(n, align); },
           py::arg("nbytes"), py::arg("align") = 256)
      .def("reset", &HostArena::reset)
      .def_property_readonly("base", [](const HostArena& a) { return (int64_t)a.base(); })
      .def_property_readonly("capacity", &HostArena::capacity)
      .def_property_readonly("used", &HostArena::used)
      .def_property_readonly("peak", &HostArena::peak)
      .def_property_readonly("allocations", &HostArena::allocations);

  py::class_<TokenLoader>(m, "TokenLoader")
      .def(py::init([](const std::string& path, int token_bytes, int64_t vocab, int batch, int seq, int rank,
                       int world, uint64_t seed, int depth, int threads, bool shuffle, bool fixed) {
             TokenLoaderConfig c;
             c.path = path;
             c.token_bytes = token_bytes;
             c.vocab = vocab;
             c.batch = batch;
             c.seq = seq;
             c.rank = rank;
             c.world = world;
             c.seed = seed;
             c.depth = depth;
             c.threads = threads;
             c.shuffle = shuffle;
             c.fixed = fixed;
             return new TokenLoader(c);
           }),
           py::arg("path"), py::arg("token_bytes"), py::arg("vocab"), py::arg("batch"), py::arg("seq"),
           py::arg("rank") = 0, py::arg("world") = 1, py::arg("seed") = 0, py::arg("depth") = 4,
           py::arg("threads") = 4, py::arg("shuffle") = true, py::arg("fixed") = false)
      .def("acquire",
           [](TokenLoader& l, int64_t timeout_ms) {
             py::gil_scoped_release nogil;
             return l.acquire(timeout_ms);
           },
           py::arg("timeout_ms") = -1)
      .def("release", &TokenLoader::release)
      .def("seek", &TokenLoader::seek)
      .def("cursor", &TokenLoader::cursor)
      .def("slot_batch", &TokenLoader::slot_batch)
      .def("window_of", &TokenLoader::window_of)
      .def("slot_ptr", [](const TokenLoader& l, int s) { return (int64_t)l.ids(s); })
      .def("slot_tensor",
           [](const TokenLoader& l, int s, int64_t batch, int64_t seq) {
             // [2, B, S] int64 view over the slot (ids, targets); no ownership
             return torch::from_blob(l.ids(s), {2, batch, seq}, torch::dtype(torch::kInt64));
           })
      .def_property_readonly("slot_bytes", &TokenLoader::slot_bytes)
      .def_property_readonly("depth", &TokenLoader::depth)
      .def_property_readonly("num_windows", &TokenLoader::num_windows)
      .def_property_readonly("arena_ptr", [](const TokenLoader& l) { return (int64_t)l.arena_base(); })
      .def_property_readonly("arena_bytes", &TokenLoader::arena_bytes)
      .def_property_readonly("steals", [](const TokenLoader& l) { return l.pool().steals(); });
}
