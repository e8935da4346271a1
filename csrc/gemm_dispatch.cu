// K1 GEMM entry point: picks the tile width and the operand-major variant.
// Instantiations are spread over gemm_bf16.cu / gemm_f32.cu / gemm_fused.cu so
// they compile in parallel.
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
      return gemm_dispatch_fused(*g, stream);
    default:
      return fail("lk_gemm: unknown epilogue");
  }
}

namespace lk {
int choose_bn(const LkGemmDesc& g) {
  if (g.bn == 128 || g.bn == 256) return g.bn;
  const int64_t tiles256 = (int64_t)cdiv(g.M, 128) * cdiv(g.N, 256);
  return (g.N <= 128 || tiles256 < num_sms()) ? 128 : 256;
}
}  // namespace lk
