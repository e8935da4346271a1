// K1 GEMM instantiations: bf16 output, all operand-major combinations.
#include "gemm_kernel.cuh"

namespace lk {
int choose_bn(const LkGemmDesc& g);

template <int BN>
static int bf16_major(const LkGemmDesc& g, cudaStream_t s) {
  if (!g.a_mn && !g.b_mn) return launch_gemm<BN, false, false, EPI_BF16>(g, s);
  if (!g.a_mn && g.b_mn) return launch_gemm<BN, false, true, EPI_BF16>(g, s);
  if (g.a_mn && g.b_mn) return launch_gemm<BN, true, true, EPI_BF16>(g, s);
  return launch_gemm<BN, true, false, EPI_BF16>(g, s);
}

static int bf16_pair(const LkGemmDesc& g, cudaStream_t s) {
  if (!g.a_mn && !g.b_mn) return launch_gemm<256, false, false, EPI_BF16, 0, 2>(g, s);
  if (!g.a_mn && g.b_mn) return launch_gemm<256, false, true, EPI_BF16, 0, 2>(g, s);
  if (g.a_mn && g.b_mn) return launch_gemm<256, true, true, EPI_BF16, 0, 2>(g, s);
  return launch_gemm<256, true, false, EPI_BF16, 0, 2>(g, s);
}

int gemm_dispatch_bf16(const LkGemmDesc& g, cudaStream_t s) {
  if (use_pair(g)) return bf16_pair(g, s);
  return choose_bn(g) == 128 ? bf16_major<128>(g, s) : bf16_major<256>(g, s);
}
}  // namespace lk
