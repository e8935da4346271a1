// K1 GEMM instantiations with fused epilogues used by the transformer block:
// residual add (attention output / down projection) and SwiGLU (gate|up).
#include "gemm_kernel.cuh"

namespace lk {
int choose_bn(const LkGemmDesc& g);

int gemm_dispatch_fused(const LkGemmDesc& g, cudaStream_t s) {
  if (g.epi == LK_EPI_SWIGLU_BWD) {
    // the down projection's data gradient: A = dy (K-major), B = W_down^T (MN-major view)
    LK_REQUIRE(!g.a_mn && g.b_mn && g.N % 128 == 0 && g.r != nullptr && g.ldr % 8 == 0 && g.ldd % 8 == 0,
               "lk_gemm: swiglu_bwd needs K-major A, MN-major B, N % 128 == 0 and the gate|up input r");
    if (use_pair(g)) return launch_gemm<256, false, true, EPI_SWIGLU_BWD, 0, 2>(g, s);
    return choose_bn(g) == 128 ? launch_gemm<128, false, true, EPI_SWIGLU_BWD>(g, s)
                               : launch_gemm<256, false, true, EPI_SWIGLU_BWD>(g, s);
  }
  LK_REQUIRE(!g.a_mn && !g.b_mn, "lk_gemm: fused epilogues need K-major operands");
  if (g.epi == LK_EPI_BF16_ROPE) {
    LK_REQUIRE(g.rope_table != nullptr && g.rope_dh % 8 == 0 && g.rope_dh > 0 && g.rope_cols % g.rope_dh == 0 &&
                   g.rope_seq > 0,
               "lk_gemm: rope epilogue needs the table, head_dim % 8 == 0, whole heads and seq > 0");
    if (use_pair(g)) return launch_gemm<256, false, false, EPI_BF16_ROPE, 0, 2>(g, s);
    return choose_bn(g) == 128 ? launch_gemm<128, false, false, EPI_BF16_ROPE>(g, s)
                               : launch_gemm<256, false, false, EPI_BF16_ROPE>(g, s);
  }
  if (g.epi == LK_EPI_SWIGLU) {
    LK_REQUIRE(g.N % 256 == 0 && g.h != nullptr, "lk_gemm: swiglu needs N % 256 == 0 and h");
    if (use_pair(g)) return launch_gemm<256, false, false, EPI_SWIGLU, 0, 2>(g, s);
    return launch_gemm<256, false, false, EPI_SWIGLU>(g, s);
  }
  LK_REQUIRE(g.r != nullptr && g.ldr % 8 == 0, "lk_gemm: residual epilogue needs r");
  if (use_pair(g)) return launch_gemm<256, false, false, EPI_BF16_RESID, 0, 2>(g, s);
  return choose_bn(g) == 128 ? launch_gemm<128, false, false, EPI_BF16_RESID>(g, s)
                             : launch_gemm<256, false, false, EPI_BF16_RESID>(g, s);
}
}  // namespace lk
