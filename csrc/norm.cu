// K5: RMSNorm forward / backward (bf16 activations, fp32 statistics).
//
// Forward   y = x * rstd * gamma,  rstd = 1/sqrt(mean(x^2) + eps)
//           with an optional fused residual add: h = x + r, y = norm(h).
// Backward  dx = rstd * (dy*gamma - xhat * mean(dy*gamma*xhat)) (+ dres)
//           dgamma = sum_rows dy * xhat (fp32, accumulated into the grad).
// The reference's rmsnorm_backward (include/core/tensor.hpp:402-414) applies
// gamma after the projection, which is exact only for gamma == 1; this kernel
// uses the exact form above.  Forward parity: tensor.hpp:394-400, block use in
// src/nn/transformer_blocks.cpp:417-421,507-511.
//
// One warp per row; each lane owns VPT 16-byte vectors (8 bf16 each) of the row,
// so a row is read once and kept in registers (D = 256 * VPT).
#include "common.cuh"
#include "host_util.h"
#include "lk_api.h"

namespace lk {

template <int VPT>
__global__ void __launch_bounds__(256) rmsnorm_fwd_kernel(
    const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ res,
    const __nv_bfloat16* __restrict__ gamma, __nv_bfloat16* __restrict__ y,
    __nv_bfloat16* __restrict__ h_out, float* __restrict__ rstd_out, int M, int D, float eps) {
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  for (int row = blockIdx.x * warps + (threadIdx.x >> 5); row < M; row += gridDim.x * warps) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + (int64_t)row * D);
    float v[VPT][8];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int c = i * 32 + lane;
      uint4 a = xr[c];
      const uint32_t aw[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float2 f = unpack_bf16x2(aw[e]);
        v[i][2 * e] = f.x;
        v[i][2 * e + 1] = f.y;
      }
      if (res) {
        uint4 b = reinterpret_cast<const uint4*>(res + (int64_t)row * D)[c];
        const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
        uint32_t hw[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float2 f = unpack_bf16x2(bw[e]);
          v[i][2 * e] += f.x;
          v[i][2 * e + 1] += f.y;
          hw[e] = pack_bf16x2(v[i][2 * e], v[i][2 * e + 1]);
          // normalise the rounded sum so forward and backward see the same h
          float2 hr = unpack_bf16x2(hw[e]);
          v[i][2 * e] = hr.x;
          v[i][2 * e + 1] = hr.y;
        }
        reinterpret_cast<uint4*>(h_out + (int64_t)row * D)[c] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += v[i][e] * v[i][e];
    }
    ss = warp_sum(ss);
    const float rstd = rsqrtf(ss / (float)D + eps);
    if (lane == 0 && rstd_out) rstd_out[row] = rstd;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int c = i * 32 + lane;
      uint4 g = reinterpret_cast<const uint4*>(gamma)[c];
      const uint32_t gw[4] = {g.x, g.y, g.z, g.w};
      uint32_t o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float2 gf = unpack_bf16x2(gw[e]);
        o[e] = pack_bf16x2(v[i][2 * e] * rstd * gf.x, v[i][2 * e + 1] * rstd * gf.y);
      }
      reinterpret_cast<uint4*>(y + (int64_t)row * D)[c] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

// Backward: one warp per row, 4 warps per block, grid-stride over rows.  Rows
// up to 2048 wide (VPT <= 8) come into registers with one pass of loads (every
// load of the row in flight at once); wider rows read x and dy again in the
// second pass (L1 hits).  dres is fetched into L2 during the first pass and the
// warp's next row while the current one is processed, so the loads that wait are
// L2 hits.  dgamma partial sums accumulate per warp in shared memory (float4
// read-modify-write); at the end each block writes one partial row to
// partial[blockIdx.x, :] (fp32 scratch, gridDim.x x D), summed by colsum_kernel.
constexpr int NORM_BWD_WARPS = 4;

template <int VPT>
__global__ void __launch_bounds__(32 * NORM_BWD_WARPS) rmsnorm_bwd_kernel(
    const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
    const __nv_bfloat16* __restrict__ gamma, const float* __restrict__ rstd,
    const __nv_bfloat16* dres, __nv_bfloat16* dx, float* __restrict__ partial, int M, int D) {
  constexpr bool HOLD = VPT <= 8;
  constexpr int NH = HOLD ? VPT : 1;  // row registers
  extern __shared__ float red[];      // [warps][D]
  const int w = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  float* my = red + (int64_t)w * D;
  for (int c = lane; c < D; c += 32) my[c] = 0.f;
  __syncwarp();
  const uint4* gr = reinterpret_cast<const uint4*>(gamma);
  for (int row = blockIdx.x * NORM_BWD_WARPS + w; row < M; row += gridDim.x * NORM_BWD_WARPS) {
    const float rs = rstd[row];
    const uint4* xr = reinterpret_cast<const uint4*>(x + (int64_t)row * D);
    const uint4* yr = reinterpret_cast<const uint4*>(dy + (int64_t)row * D);
    const uint4* rr = dres ? reinterpret_cast<const uint4*>(dres + (int64_t)row * D) : nullptr;
    uint4 xa[NH], ya[NH];
    if constexpr (HOLD) {
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        xa[i] = xr[i * 32 + lane];
        ya[i] = yr[i * 32 + lane];
      }
    }
    {
      // the warp's next row into L2 (one prefetch per 128-byte line)
      const int nrow = row + gridDim.x * NORM_BWD_WARPS;
      if (nrow < M) {
        const int64_t o = (int64_t)nrow * D;
        for (int c = lane * 8; c < VPT * 32; c += 256) {
          asm volatile("prefetch.global.L2 [%0];" ::"l"(reinterpret_cast<const uint4*>(x + o) + c));
          asm volatile("prefetch.global.L2 [%0];" ::"l"(reinterpret_cast<const uint4*>(dy + o) + c));
          if (dres) asm volatile("prefetch.global.L2 [%0];" ::"l"(reinterpret_cast<const uint4*>(dres + o) + c));
        }
      }
    }
    float dot = 0.f;
#pragma unroll(HOLD ? VPT : 4)
    for (int i = 0; i < VPT; ++i) {
      const int c = i * 32 + lane;
      uint4 a, b;
      if constexpr (HOLD) {
        a = xa[i];
        b = ya[i];
      } else {
        a = xr[c];
        b = yr[c];
      }
      if (rr && (lane & 7) == 0) asm volatile("prefetch.global.L2 [%0];" ::"l"(rr + c));
      const uint4 g = gr[c];
      const uint32_t aw[4] = {a.x, a.y, a.z, a.w};
      const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
      const uint32_t gw[4] = {g.x, g.y, g.z, g.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 xf = unpack_bf16x2(aw[e]), yf = unpack_bf16x2(bw[e]), gf = unpack_bf16x2(gw[e]);
        dot += yf.x * gf.x * xf.x + yf.y * gf.y * xf.y;
      }
    }
    dot = warp_sum(dot) * rs / (float)D;  // mean(dy*gamma*xhat)
    uint4* dxr = reinterpret_cast<uint4*>(dx + (int64_t)row * D);
#pragma unroll(HOLD ? VPT : 4)
    for (int i = 0; i < VPT; ++i) {
      const int c = i * 32 + lane;
      uint4 a, b;
      if constexpr (HOLD) {
        a = xa[i];
        b = ya[i];
      } else {
        a = xr[c];
        b = yr[c];
      }
      const uint4 r = rr ? rr[c] : make_uint4(0u, 0u, 0u, 0u);
      const uint4 g = gr[c];
      const uint32_t aw[4] = {a.x, a.y, a.z, a.w};
      const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
      const uint32_t gw[4] = {g.x, g.y, g.z, g.w};
      const uint32_t rw[4] = {r.x, r.y, r.z, r.w};
      float4* a4 = reinterpret_cast<float4*>(my + c * 8);
      const float4 a0 = a4[0], a1 = a4[1];
      float accv[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      uint32_t o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 xf = unpack_bf16x2(aw[e]), yf = unpack_bf16x2(bw[e]), gf = unpack_bf16x2(gw[e]);
        const float2 rf = unpack_bf16x2(rw[e]);
        const float xh0 = xf.x * rs, xh1 = xf.y * rs;
        accv[2 * e] += yf.x * xh0;
        accv[2 * e + 1] += yf.y * xh1;
        o[e] = pack_bf16x2(rs * (yf.x * gf.x - xh0 * dot) + rf.x,
                           rs * (yf.y * gf.y - xh1 * dot) + rf.y);
      }
      a4[0] = make_float4(accv[0], accv[1], accv[2], accv[3]);
      a4[1] = make_float4(accv[4], accv[5], accv[6], accv[7]);
      dxr[c] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
  __syncthreads();
  for (int col = threadIdx.x; col < D; col += blockDim.x) {
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < NORM_BWD_WARPS; ++k) s += red[k * D + col];
    partial[(int64_t)blockIdx.x * D + col] = s;
  }
}

// dgamma[c] (+)= sum_b partial[b, c]; bf16_out: dgamma is bf16 and stored.
// One block per 32 columns: the 8 warps split the partial rows (coalesced
// 128-byte loads, independent adds in flight), then combine in shared memory.
__global__ void __launch_bounds__(256) colsum_kernel(const float* __restrict__ partial, int nrows, int D,
                                                     float* __restrict__ out, int accumulate, int bf16_out) {
  __shared__ float red[8][33];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int col = blockIdx.x * 32 + lane;
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
  if (col < D) {
    int r = w;
    for (; r + 24 < nrows; r += 32) {
      s0 += partial[(int64_t)r * D + col];
      s1 += partial[(int64_t)(r + 8) * D + col];
      s2 += partial[(int64_t)(r + 16) * D + col];
      s3 += partial[(int64_t)(r + 24) * D + col];
    }
    for (; r < nrows; r += 8) s0 += partial[(int64_t)r * D + col];
  }
  red[w][lane] = (s0 + s1) + (s2 + s3);
  __syncthreads();
  if (w == 0 && col < D) {
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) s += red[k][lane];
    if (bf16_out)
      reinterpret_cast<__nv_bfloat16*>(out)[col] = __float2bfloat16_rn(s);
    else
      out[col] = accumulate ? out[col] + s : s;
  }
}

template <int VPT>
static void fwd_launch(const LkNormFwdDesc& d, cudaStream_t s) {
  const int rows_per_block = 8;
  int grid = cdiv(d.M, rows_per_block);
  rmsnorm_fwd_kernel<VPT><<<grid, 256, 0, s>>>(
      (const __nv_bfloat16*)d.x, (const __nv_bfloat16*)d.res, (const __nv_bfloat16*)d.gamma,
      (__nv_bfloat16*)d.y, (__nv_bfloat16*)d.h_out, d.rstd, d.M, d.D, d.eps);
}

template <int VPT>
static void bwd_launch(const LkNormBwdDesc& d, int grid, cudaStream_t s) {
  const int smem = NORM_BWD_WARPS * d.D * (int)sizeof(float);
  auto k = rmsnorm_bwd_kernel<VPT>;
  if (smem > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  k<<<grid, 32 * NORM_BWD_WARPS, smem, s>>>(
      (const __nv_bfloat16*)d.dy, (const __nv_bfloat16*)d.x, (const __nv_bfloat16*)d.gamma, d.rstd,
      (const __nv_bfloat16*)d.dres, (__nv_bfloat16*)d.dx, d.partial, d.M, d.D);
}

int norm_bwd_grid(int M) {
  const int g = cdiv(M, 8);
  const int cap = 2 * num_sms();
  return g < cap ? g : cap;
}

}  // namespace lk

using namespace lk;

extern "C" int lk_rmsnorm_fwd(const LkNormFwdDesc* d, cudaStream_t s) {
  LK_REQUIRE(d->D % 256 == 0 && d->D <= 4096, "rmsnorm: D must be a multiple of 256, <= 4096");
  LK_REQUIRE(!d->res || d->h_out, "rmsnorm: residual input needs h_out");
  switch (d->D / 256) {
    case 1: fwd_launch<1>(*d, s); break;
    case 2: fwd_launch<2>(*d, s); break;
    case 3: fwd_launch<3>(*d, s); break;
    case 4: fwd_launch<4>(*d, s); break;
    case 8: fwd_launch<8>(*d, s); break;
    case 12: fwd_launch<12>(*d, s); break;
    case 16: fwd_launch<16>(*d, s); break;
    default: return fail("rmsnorm: unsupported D (256 x {1,2,3,4,8,12,16})");
  }
  return check_launch("rmsnorm_fwd");
}

extern "C" int lk_rmsnorm_bwd_partial_rows(int M) { return norm_bwd_grid(M); }

extern "C" int lk_rmsnorm_bwd(const LkNormBwdDesc* d, cudaStream_t s) {
  LK_REQUIRE(d->D % 256 == 0 && d->D <= 4096, "rmsnorm_bwd: D must be a multiple of 256, <= 4096");
  const int grid = norm_bwd_grid(d->M);
  LK_REQUIRE(d->partial_rows >= grid, "rmsnorm_bwd: partial scratch too small");
  switch (d->D / 256) {
    case 1: bwd_launch<1>(*d, grid, s); break;
    case 2: bwd_launch<2>(*d, grid, s); break;
    case 3: bwd_launch<3>(*d, grid, s); break;
    case 4: bwd_launch<4>(*d, grid, s); break;
    case 8: bwd_launch<8>(*d, grid, s); break;
    case 12: bwd_launch<12>(*d, grid, s); break;
    case 16: bwd_launch<16>(*d, grid, s); break;
    default: return fail("rmsnorm_bwd: unsupported D");
  }
  if (check_launch("rmsnorm_bwd")) return -1;
  LK_REQUIRE(!d->dgamma_bf16 || !d->accumulate, "rmsnorm_bwd: a bf16 dgamma is stored, not accumulated");
  colsum_kernel<<<cdiv(d->D, 32), 256, 0, s>>>(d->partial, grid, d->D, d->dgamma, d->accumulate,
                                               d->dgamma_bf16);
  return check_launch("rmsnorm_dgamma");
}
