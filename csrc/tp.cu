// Tensor-parallel (Megatron sequence-parallel) helpers around the fused
// collective GEMMs (K16 all-gather -> GEMM, K18 GEMM -> reduce-scatter):
//
//   rs_sum: the owner's half of K18.  The GEMM epilogue of every rank stores
//   its bf16 partial of the owner's rows into slot (rank) of the owner's
//   receive buffer [world * rows, cols]; after a device barrier the owner sums
//   the slots in fixed rank order (fp32, so every run is bit-identical), adds
//   the residual stream and - optionally - applies the next RMSNorm, writing
//   the normalised rows straight into the symmetric staging buffer that the
//   next K16 all-gather reads from.  One warp per row, the row held in
//   registers (cols = 256 * VPT).
//
// Reference: the reference's TP layers (include/distributed/
// tensor_parallel.hpp:14-104) all-gather / all-reduce around an unfused
// matmul; this is the sequence-parallel form with the reduction fused into the
// GEMM epilogue and the norm fused into the reduction.
#include "common.cuh"
#include "host_util.h"
#include "lk_api.h"

namespace lk {

// Sum of 8 bf16 over every rank, reduced inside the NVSwitch (fp32 accumulation).
__device__ __forceinline__ uint4 mm_ld_reduce_bf16x8(const void* mc) {
  uint4 r;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(mc)
               : "memory");
  return r;
}

__device__ __forceinline__ void acc_bf16x8(float* v, uint4 a) {
  const uint32_t aw[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 f = unpack_bf16x2(aw[e]);
    v[2 * e] += f.x;
    v[2 * e + 1] += f.y;
  }
}

// SRC 0: the owner's receive slots (K18); 1: every rank's own partial, read
// from peer memory in fixed rank order (all-reduce, every rank sums every
// row); 2: the same through the multicast address (NVLS ld_reduce).
template <int VPT, bool NORM, int SRC>
__global__ void __launch_bounds__(256) rs_sum_norm_kernel(LkRsSumDesc d) {
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  const __nv_bfloat16* recv = reinterpret_cast<const __nv_bfloat16*>(d.recv);
  for (int row = blockIdx.x * warps + (threadIdx.x >> 5); row < d.rows; row += gridDim.x * warps) {
    float v[VPT][8];
#pragma unroll
    for (int i = 0; i < VPT; ++i)
#pragma unroll
      for (int e = 0; e < 8; ++e) v[i][e] = 0.f;
    if constexpr (SRC == 2) {
      const __nv_bfloat16* mc = reinterpret_cast<const __nv_bfloat16*>(d.mc) + (int64_t)row * d.ld_recv;
#pragma unroll
      for (int i = 0; i < VPT; ++i) acc_bf16x8(v[i], mm_ld_reduce_bf16x8(mc + 8 * (i * 32 + lane)));
    } else {
      for (int s = 0; s < d.world; ++s) {
        const __nv_bfloat16* base =
            SRC == 1 ? reinterpret_cast<const __nv_bfloat16*>(d.peers[s]) + (int64_t)row * d.ld_recv
                     : recv + ((int64_t)s * d.rows + row) * d.ld_recv;
        const uint4* src = reinterpret_cast<const uint4*>(base);
#pragma unroll
        for (int i = 0; i < VPT; ++i) acc_bf16x8(v[i], src[i * 32 + lane]);
      }
    }
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int c = i * 32 + lane;
      if (d.resid) {
        const uint4 b = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(d.resid) +
                                                       (int64_t)row * d.ld_resid)[c];
        const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = unpack_bf16x2(bw[e]);
          v[i][2 * e] += f.x;
          v[i][2 * e + 1] += f.y;
        }
      }
      uint32_t hw[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        hw[e] = pack_bf16x2(v[i][2 * e], v[i][2 * e + 1]);
        const float2 hr = unpack_bf16x2(hw[e]);  // normalise the rounded sum (as stored)
        v[i][2 * e] = hr.x;
        v[i][2 * e + 1] = hr.y;
        ss += hr.x * hr.x + hr.y * hr.y;
      }
      reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(d.out) + (int64_t)row * d.ld_out)[c] =
          make_uint4(hw[0], hw[1], hw[2], hw[3]);
    }
    if constexpr (NORM) {
      ss = warp_sum(ss);
      const float rstd = rsqrtf(ss / (float)d.cols + d.eps);
      if (lane == 0 && d.rstd) d.rstd[row] = rstd;
      const uint4* g = reinterpret_cast<const uint4*>(d.gamma);
      uint4* y = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(d.y) + (int64_t)row * d.ld_y);
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const int c = i * 32 + lane;
        const uint4 gv = g[c];
        const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
        uint32_t o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 gf = unpack_bf16x2(gw[e]);
          o[e] = pack_bf16x2(v[i][2 * e] * rstd * gf.x, v[i][2 * e + 1] * rstd * gf.y);
        }
        y[c] = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
  }
}

// Plain slot sum for any width (cols % 8 == 0): out = sum_s recv[s] (+ resid).
__global__ void __launch_bounds__(256) rs_sum_kernel(LkRsSumDesc d) {
  const int vpr = d.cols / 8;
  const int64_t n = (int64_t)d.rows * vpr;
  const __nv_bfloat16* recv = reinterpret_cast<const __nv_bfloat16*>(d.recv);
  for (int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; u < n; u += (int64_t)gridDim.x * blockDim.x) {
    const int row = (int)(u / vpr), c = (int)(u % vpr);
    float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int s = 0; s < d.world; ++s) {
      const uint4 a = reinterpret_cast<const uint4*>(recv + ((int64_t)s * d.rows + row) * d.ld_recv)[c];
      const uint32_t aw[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = unpack_bf16x2(aw[e]);
        v[2 * e] += f.x;
        v[2 * e + 1] += f.y;
      }
    }
    if (d.resid) {
      const uint4 b = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(d.resid) +
                                                     (int64_t)row * d.ld_resid)[c];
      const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = unpack_bf16x2(bw[e]);
        v[2 * e] += f.x;
        v[2 * e + 1] += f.y;
      }
    }
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) o[e] = pack_bf16x2(v[2 * e], v[2 * e + 1]);
    reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(d.out) + (int64_t)row * d.ld_out)[c] =
        make_uint4(o[0], o[1], o[2], o[3]);
  }
}

}  // namespace lk

using namespace lk;

extern "C" int lk_rs_sum(const LkRsSumDesc* d, cudaStream_t s) {
  LK_REQUIRE(d->cols % 8 == 0 && d->ld_recv % 8 == 0 && d->ld_out % 8 == 0, "rs_sum: 16-byte rows");
  LK_REQUIRE(!d->resid || d->ld_resid % 8 == 0, "rs_sum: residual pitch");
  if (d->rows == 0) return 0;
  if (!d->gamma) {
    const int64_t n = (int64_t)d->rows * (d->cols / 8);
    const int grid = (int)std::min<int64_t>((n + 255) / 256, 8 * num_sms());
    rs_sum_kernel<<<grid, 256, 0, s>>>(*d);
    return check_launch("rs_sum");
  }
  LK_REQUIRE(d->y && d->cols % 256 == 0 && d->ld_y % 8 == 0, "rs_sum+norm: cols % 256 and y needed");
  LK_REQUIRE(d->src_mode == 0 || (d->src_mode == 1 && d->peers) || (d->src_mode == 2 && d->mc),
             "rs_sum+norm: source pointers missing");
  const int grid = (int)std::min<int64_t>((d->rows + 7) / 8, 4 * num_sms());
  switch (d->cols / 256) {
#define LK_RS_CASE(V)                                                                    \
  case V:                                                                                \
    if (d->src_mode == 0) rs_sum_norm_kernel<V, true, 0><<<grid, 256, 0, s>>>(*d);       \
    else if (d->src_mode == 1) rs_sum_norm_kernel<V, true, 1><<<grid, 256, 0, s>>>(*d);  \
    else rs_sum_norm_kernel<V, true, 2><<<grid, 256, 0, s>>>(*d);                        \
    break;
    LK_RS_CASE(1)
    LK_RS_CASE(2)
    LK_RS_CASE(3)
    LK_RS_CASE(4)
    LK_RS_CASE(8)
    LK_RS_CASE(12)
    LK_RS_CASE(16)
#undef LK_RS_CASE
    default:
      return fail("rs_sum+norm: cols must be 256 x {1,2,3,4,8,12,16}");
  }
  return check_launch("rs_sum_norm");
}
