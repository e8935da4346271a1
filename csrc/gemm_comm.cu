// K1 GEMM instantiations with fused collectives:
//   K18  GEMM -> reduce-scatter: the epilogue stores each output tile into the
//        owner rank's receive slot in peer memory (the owner sums the slots);
//   K16  all-gather -> GEMM: a copy warp per CTA pulls peers' rows of A into
//        local memory on first use; the TMA producer waits (bounded) on per-chunk
//        counters before loading a remote row block.  Cooperative launch.
// Both rotate the M-tile order by rank so peers do not all hit the same owner.
#include "gemm_kernel.cuh"

namespace lk {
int choose_bn(const LkGemmDesc& g);

int gemm_dispatch_comm(const LkGemmDesc& g, cudaStream_t s) {
  LK_REQUIRE(!g.a_mn, "fused-collective GEMM: A must be K-major");
  const int bn = choose_bn(g);
  if (g.comm_mode == 1) {
    LK_REQUIRE(g.epi == LK_EPI_REMOTE && g.rptrs && g.rs_rows > 0, "gemm_rs: needs rptrs / rs_rows");
    if (!g.b_mn) return bn == 128 ? launch_gemm<128, false, false, EPI_REMOTE>(g, s)
                                  : launch_gemm<256, false, false, EPI_REMOTE>(g, s);
    return bn == 128 ? launch_gemm<128, false, true, EPI_REMOTE>(g, s)
                     : launch_gemm<256, false, true, EPI_REMOTE>(g, s);
  }
  if (g.comm_mode == 2) {
    LK_REQUIRE(g.ag_src && g.ag_count && g.ag_rows % 128 == 0 && g.ag_world >= 1 &&
                   (int64_t)g.ag_rows * g.ag_world == g.M && (g.a_cols * 2) % 16 == 0,
               "gemm_ag: M must be world * ag_rows with ag_rows % 128 == 0");
    if (g.epi == LK_EPI_SWIGLU) {
      LK_REQUIRE(!g.b_mn && g.N % 256 == 0 && g.h, "gemm_ag swiglu: K-major B, N % 256");
      return launch_gemm<256, false, false, EPI_SWIGLU, 1>(g, s);
    }
    LK_REQUIRE(g.epi == LK_EPI_BF16, "gemm_ag: bf16 or swiglu epilogue");
    if (!g.b_mn) return bn == 128 ? launch_gemm<128, false, false, EPI_BF16, 1>(g, s)
                                  : launch_gemm<256, false, false, EPI_BF16, 1>(g, s);
    return bn == 128 ? launch_gemm<128, false, true, EPI_BF16, 1>(g, s)
                     : launch_gemm<256, false, true, EPI_BF16, 1>(g, s);
  }
  if (g.comm_mode == 3) {
    LK_REQUIRE(g.gb_src && g.gb_count && g.gb_dst && g.gb_chunk > 0 && g.ag_world >= 1 &&
                   g.gb_chunk * g.ag_world == g.gb_len && g.gb_chunk % 8 == 0,
               "gemm_gather: group must be world equal chunks of 8-element multiples");
    LK_REQUIRE(g.b == (const void*)((const uint8_t*)g.gb_dst + 2 * g.gb_boff), "gemm_gather: B must lie in gb_dst");
    LK_REQUIRE(g.epi == LK_EPI_BF16 || g.epi == LK_EPI_SWIGLU, "gemm_gather: bf16 or swiglu epilogue");
    if (g.epi == LK_EPI_SWIGLU) {
      LK_REQUIRE(!g.b_mn && g.N % 256 == 0 && g.h, "gemm_gather swiglu: K-major B, N % 256");
      return launch_gemm<256, false, false, EPI_SWIGLU, 2>(g, s);
    }
    if (!g.b_mn) return bn == 128 ? launch_gemm<128, false, false, EPI_BF16, 2>(g, s)
                                  : launch_gemm<256, false, false, EPI_BF16, 2>(g, s);
    return bn == 128 ? launch_gemm<128, false, true, EPI_BF16, 2>(g, s)
                     : launch_gemm<256, false, true, EPI_BF16, 2>(g, s);
  }
  return fail("gemm: unknown comm_mode");
}
}  // namespace lk

extern "C" int lk_make_remote_maps(void* const* host_ptrs, int world, int64_t rows, int64_t cols, int64_t ld,
                                   void* out) {
  CUtensorMap* m = reinterpret_cast<CUtensorMap*>(out);
  for (int p = 0; p < world; ++p)
    if (!lk::make_tmap_2d(m + p, host_ptrs[p], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, rows, cols, ld, 32, 64))
      return -1;
  return 0;
}
