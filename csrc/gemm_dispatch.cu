// K1 GEMM entry point: picks the tile width and the operand-major variant.
// Instantiations are spread over gemm_bf16.cu / gemm_f32.cu / gemm_fused.cu so
// they compile in parallel.
#include <atomic>
#include <cstdlib>

#include "gemm_kernel.cuh"

extern "C" const char* lk_last_error(void) { return lk::last_error().c_str(); }

extern "C" unsigned long long lk_launch_count(void) { return lk::launch_counter().load(); }

extern "C" int lk_gemm(const LkGemmDesc* g, cudaStream_t stream) {
  using namespace lk;
  LK_REQUIRE(g != nullptr, "lk_gemm: null descriptor");
  LK_REQUIRE(g->M > 0 && g->N > 0 && g->K > 0, "lk_gemm: empty problem");
  LK_REQUIRE(g->N % 8 == 0, "lk_gemm: N must be a multiple of 8");
  LK_REQUIRE(g->a_ld % 8 == 0 && g->b_ld % 8 == 0, "lk_gemm: operand pitch must be a multiple of 8");
  LK_REQUIRE(g->ldd % 4 == 0, "lk_gemm: output pitch must be 16-byte aligned");
  if (g->comm_mode != 0) return gemm_dispatch_comm(*g, stream);
  switch (g->epi) {
    case LK_EPI_BF16:
      return gemm_dispatch_bf16(*g, stream);
    case LK_EPI_F32:
    case LK_EPI_F32_ACC:
      return gemm_dispatch_f32(*g, stream);
    case LK_EPI_BF16_RESID:
    case LK_EPI_SWIGLU:
    case LK_EPI_SWIGLU_BWD:
    case LK_EPI_BF16_ROPE:
      return gemm_dispatch_fused(*g, stream);
    default:
      return fail("lk_gemm: unknown epilogue");
  }
}

namespace lk {
std::atomic<unsigned long long>& gemm_pair_count();
}

extern "C" void lk_gemm_set_pair(int mode) { lk::gemm_pair_mode() = mode; }

extern "C" unsigned long long lk_gemm_pair_count(void) { return lk::gemm_pair_count().load(); }

namespace lk {
int& gemm_pair_mode() {
  static int mode = [] {
    const char* e = getenv("LK_GEMM_PAIR");
    return e ? atoi(e) : 1;
  }();
  return mode;
}

// CTA-pair (256-row) tiles for plain GEMMs with at least two 256-row tiles
// per SM pair's worth of work; 128-row tiles otherwise.
std::atomic<unsigned long long>& gemm_pair_count() {
  static std::atomic<unsigned long long> n{0};
  return n;
}

bool use_pair(const LkGemmDesc& g) {
  if (gemm_pair_mode() == 0 || g.comm_mode != 0 || g.bn == 128) return false;
  if (g.M < 256 || g.N < 256) return false;
  const int64_t tiles = (int64_t)cdiv(g.M, 256) * cdiv(g.N, 256);
  if (tiles < num_sms() / 2) return false;
  ++gemm_pair_count();
  return true;
}

int choose_bn(const LkGemmDesc& g) {
  if (g.bn == 128 || g.bn == 256) return g.bn;
  const int64_t tiles256 = (int64_t)cdiv(g.M, 128) * cdiv(g.N, 256);
  return (g.N <= 128 || tiles256 < num_sms()) ? 128 : 256;
}
}  // namespace lk
