// K1 GEMM instantiations: fp32 output (plain store or accumulate, the latter
// used by weight-gradient GEMMs writing straight into the fp32 grad buffer).
#include "gemm_kernel.cuh"

namespace lk {
int choose_bn(const LkGemmDesc& g);

template <int BN, int EPI>
static int f32_major(const LkGemmDesc& g, cudaStream_t s) {
  if (!g.a_mn && !g.b_mn) return launch_gemm<BN, false, false, EPI>(g, s);
  if (g.a_mn && g.b_mn) return launch_gemm<BN, true, true, EPI>(g, s);
  if (!g.a_mn && g.b_mn) return launch_gemm<BN, false, true, EPI>(g, s);
  return fail("lk_gemm: fp32 epilogue does not support MN-major A with K-major B");
}

template <int EPI>
static int f32_pair(const LkGemmDesc& g, cudaStream_t s) {
  if (!g.a_mn && !g.b_mn) return launch_gemm<256, false, false, EPI, 0, 2>(g, s);
  if (g.a_mn && g.b_mn) return launch_gemm<256, true, true, EPI, 0, 2>(g, s);
  if (!g.a_mn && g.b_mn) return launch_gemm<256, false, true, EPI, 0, 2>(g, s);
  return fail("lk_gemm: fp32 epilogue does not support MN-major A with K-major B");
}

int gemm_dispatch_f32(const LkGemmDesc& g, cudaStream_t s) {
  if (use_pair(g)) return g.epi == LK_EPI_F32 ? f32_pair<EPI_F32>(g, s) : f32_pair<EPI_F32_ACC>(g, s);
  const int bn = choose_bn(g);
  if (g.epi == LK_EPI_F32)
    return bn == 128 ? f32_major<128, EPI_F32>(g, s) : f32_major<256, EPI_F32>(g, s);
  return bn == 128 ? f32_major<128, EPI_F32_ACC>(g, s) : f32_major<256, EPI_F32_ACC>(g, s);
}
}  // namespace lk
