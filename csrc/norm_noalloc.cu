// Allocation-free RMSNorm backward (declared and documented in lk_noalloc.h).
// This entry point has no counterpart in the reference.
//
// The dgamma partials that lk_rmsnorm_bwd normally writes to a caller-provided
// fp32 buffer go to `g_norm_scratch`, a file-scope device array, so a caller
// that cannot allocate device memory can still run the backward pass.
#include <mutex>

#include "host_util.h"
#include "lk_noalloc.h"

namespace {

static __device__ __align__(256) float g_norm_scratch[LK_NOALLOC_NORM_SCRATCH_FLOATS];

constexpr int kMaxDevices = 64;
float* g_scratch_ptr[kMaxDevices] = {nullptr};
std::mutex g_setup_mutex;

// Device address of g_norm_scratch on the current device.  In host code the
// symbol name is only a host-side stand-in, so the address must come from
// cudaGetSymbolAddress, looked up once per device with that device current.
int scratch_for_current_device(float** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return lk::fail("rmsnorm_bwd_noalloc: no usable current device");
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_norm_scratch);
    if (e != cudaSuccess || p == nullptr) {
      lk::last_error() = std::string("rmsnorm_bwd_noalloc: cudaGetSymbolAddress failed: ") +
                         cudaGetErrorString(e);
      return -1;
    }
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_ptr[dev];
  return 0;
}

}  // namespace

extern "C" int lk_rmsnorm_bwd_noalloc(const void* dy, const void* x, const void* gamma,
                                      const float* rstd, const void* dres, void* dx,
                                      float* dgamma, int M, int D, int accumulate,
                                      cudaStream_t stream) {
  LK_REQUIRE(M > 0 && D > 0, "rmsnorm_bwd_noalloc: empty problem");
  const int rows = lk_rmsnorm_bwd_partial_rows(M);
  if ((long long)rows * D > LK_NOALLOC_NORM_SCRATCH_FLOATS) {
    char buf[200];
    snprintf(buf, sizeof(buf),
             "rmsnorm_bwd_noalloc: needs %lld scratch floats (%d partial rows x D=%d) but the "
             "built-in scratch holds %d; use lk_rmsnorm_bwd with your own buffer",
             (long long)rows * D, rows, D, LK_NOALLOC_NORM_SCRATCH_FLOATS);
    lk::last_error() = buf;
    return -1;
  }
  float* scratch = nullptr;
  if (scratch_for_current_device(&scratch)) return -1;
  LkNormBwdDesc d{};
  d.dy = dy;
  d.x = x;
  d.gamma = gamma;
  d.rstd = rstd;
  d.dres = dres;
  d.dx = dx;
  d.dgamma = dgamma;
  d.partial = scratch;  // every row the kernel reads back is written by this call
  d.partial_rows = rows;
  d.M = M;
  d.D = D;
  d.accumulate = accumulate;
  return lk_rmsnorm_bwd(&d, stream);
}
