// Ops outside the Llama path that the reference also provides:
//
//   GELU (tanh form, Hendrycks & Gimpel):
//     gelu(x)  = 0.5 x (1 + tanh(u)),  u = sqrt(2/pi) (x + 0.044715 x^3)
//     gelu'(x) = 0.5 (1 + tanh(u)) + 0.5 x (1 - tanh(u)^2) sqrt(2/pi) (1 + 3 * 0.044715 x^2)
//   LayerNorm with affine gamma / beta:
//     y = (x - mean) * rstd * gamma + beta,   rstd = 1 / sqrt(var + eps)
//     dx = rstd * (g - mean(g) - xhat * mean(g * xhat)),  g = dy * gamma
//     dgamma = sum_rows dy * xhat,  dbeta = sum_rows dy
// bf16 tensors, fp32 arithmetic; LayerNorm is one warp per row with the row in
// registers (D = 256 * VPT), its parameter gradients reduced per block in shared
// memory and added to the fp32 outputs with one atomic per column per block.
//
// Reference: gelu_forward / gelu_backward (include/core/tensor.hpp:416-438),
// FusedKernels::fused_layernorm (include/nn/fused_kernels.hpp:10-18) and the
// guarded CUDA layernorm_kernel (include/hw/cuda_kernels.hpp:108-151).
#include "common.cuh"
#include "host_util.h"
#include "lk_api.h"

namespace lk {
namespace {

constexpr float kGeluC = 0.7978845608028654f;  // sqrt(2 / pi)
constexpr float kGeluA = 0.044715f;

__global__ void gelu_fwd_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ y, int64_t n8) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
    const uint4 v = reinterpret_cast<const uint4*>(x)[i];
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = unpack_bf16x2(w[e]);
      const float a = 0.5f * f.x * (1.f + tanhf(kGeluC * (f.x + kGeluA * f.x * f.x * f.x)));
      const float b = 0.5f * f.y * (1.f + tanhf(kGeluC * (f.y + kGeluA * f.y * f.y * f.y)));
      o[e] = pack_bf16x2(a, b);
    }
    reinterpret_cast<uint4*>(y)[i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

__device__ __forceinline__ float gelu_grad(float x) {
  const float t = tanhf(kGeluC * (x + kGeluA * x * x * x));
  return 0.5f * (1.f + t) + 0.5f * x * (1.f - t * t) * kGeluC * (1.f + 3.f * kGeluA * x * x);
}

__global__ void gelu_bwd_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ dy,
                                __nv_bfloat16* __restrict__ dx, int64_t n8) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
    const uint4 v = reinterpret_cast<const uint4*>(x)[i];
    const uint4 g = reinterpret_cast<const uint4*>(dy)[i];
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    const uint32_t gw[4] = {g.x, g.y, g.z, g.w};
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = unpack_bf16x2(w[e]);
      const float2 d = unpack_bf16x2(gw[e]);
      o[e] = pack_bf16x2(d.x * gelu_grad(f.x), d.y * gelu_grad(f.y));
    }
    reinterpret_cast<uint4*>(dx)[i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

template <int VPT>
__global__ void __launch_bounds__(256) layernorm_fwd_kernel(const __nv_bfloat16* __restrict__ x,
                                                            const __nv_bfloat16* __restrict__ gamma,
                                                            const __nv_bfloat16* __restrict__ beta,
                                                            __nv_bfloat16* __restrict__ y, float* __restrict__ mean_out,
                                                            float* __restrict__ rstd_out, int M, int D, float eps) {
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  for (int row = blockIdx.x * warps + (threadIdx.x >> 5); row < M; row += gridDim.x * warps) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + (int64_t)row * D);
    float v[VPT][8];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const uint4 a = xr[i * 32 + lane];
      const uint32_t aw[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = unpack_bf16x2(aw[e]);
        v[i][2 * e] = f.x;
        v[i][2 * e + 1] = f.y;
        s += f.x + f.y;
      }
    }
    const float mean = warp_sum(s) / (float)D;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i)
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float d = v[i][e] - mean;
        q += d * d;
      }
    const float rstd = rsqrtf(warp_sum(q) / (float)D + eps);
    if (lane == 0) {
      mean_out[row] = mean;
      rstd_out[row] = rstd;
    }
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int c = i * 32 + lane;
      const uint4 g = reinterpret_cast<const uint4*>(gamma)[c];
      const uint4 bb = reinterpret_cast<const uint4*>(beta)[c];
      const uint32_t gw[4] = {g.x, g.y, g.z, g.w}, bw[4] = {bb.x, bb.y, bb.z, bb.w};
      uint32_t o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 gf = unpack_bf16x2(gw[e]), bf = unpack_bf16x2(bw[e]);
        o[e] = pack_bf16x2((v[i][2 * e] - mean) * rstd * gf.x + bf.x, (v[i][2 * e + 1] - mean) * rstd * gf.y + bf.y);
      }
      reinterpret_cast<uint4*>(y + (int64_t)row * D)[c] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

template <int VPT>
__global__ void __launch_bounds__(256) layernorm_bwd_kernel(const __nv_bfloat16* __restrict__ dy,
                                                            const __nv_bfloat16* __restrict__ x,
                                                            const __nv_bfloat16* __restrict__ gamma,
                                                            const float* __restrict__ mean_in,
                                                            const float* __restrict__ rstd_in,
                                                            __nv_bfloat16* __restrict__ dx, float* __restrict__ dgamma,
                                                            float* __restrict__ dbeta, int M, int D) {
  extern __shared__ float red[];  // [2][D]: dgamma, dbeta partials of this block
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  for (int c = threadIdx.x; c < 2 * D; c += blockDim.x) red[c] = 0.f;
  __syncthreads();
  for (int row = blockIdx.x * warps + (threadIdx.x >> 5); row < M; row += gridDim.x * warps) {
    const float mean = mean_in[row], rstd = rstd_in[row];
    const uint4* xr = reinterpret_cast<const uint4*>(x + (int64_t)row * D);
    const uint4* yr = reinterpret_cast<const uint4*>(dy + (int64_t)row * D);
    float xh[VPT][8], gg[VPT][8];
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int c = i * 32 + lane;
      const uint4 a = xr[c], b = yr[c], g = reinterpret_cast<const uint4*>(gamma)[c];
      const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, bw[4] = {b.x, b.y, b.z, b.w}, gw[4] = {g.x, g.y, g.z, g.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 xf = unpack_bf16x2(aw[e]), df = unpack_bf16x2(bw[e]), gf = unpack_bf16x2(gw[e]);
        xh[i][2 * e] = (xf.x - mean) * rstd;
        xh[i][2 * e + 1] = (xf.y - mean) * rstd;
        gg[i][2 * e] = df.x * gf.x;
        gg[i][2 * e + 1] = df.y * gf.y;
        s1 += gg[i][2 * e] + gg[i][2 * e + 1];
        s2 += gg[i][2 * e] * xh[i][2 * e] + gg[i][2 * e + 1] * xh[i][2 * e + 1];
        // parameter gradients of this row
        const int col = c * 8 + 2 * e;
        atomicAdd(&red[col], df.x * xh[i][2 * e]);
        atomicAdd(&red[col + 1], df.y * xh[i][2 * e + 1]);
        atomicAdd(&red[D + col], df.x);
        atomicAdd(&red[D + col + 1], df.y);
      }
    }
    const float m1 = warp_sum(s1) / (float)D, m2 = warp_sum(s2) / (float)D;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int c = i * 32 + lane;
      uint32_t o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e)
        o[e] = pack_bf16x2(rstd * (gg[i][2 * e] - m1 - xh[i][2 * e] * m2),
                           rstd * (gg[i][2 * e + 1] - m1 - xh[i][2 * e + 1] * m2));
      reinterpret_cast<uint4*>(dx + (int64_t)row * D)[c] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    atomicAdd(dgamma + c, red[c]);
    atomicAdd(dbeta + c, red[D + c]);
  }
}

}  // namespace
}  // namespace lk

using namespace lk;

extern "C" int lk_gelu_fwd(const void* x, void* y, int64_t n, cudaStream_t s) {
  LK_REQUIRE(n % 8 == 0, "gelu: element count must be a multiple of 8");
  if (n == 0) return 0;
  const int grid = (int)std::min<int64_t>((n / 8 + 255) / 256, 8 * num_sms());
  gelu_fwd_kernel<<<grid, 256, 0, s>>>((const __nv_bfloat16*)x, (__nv_bfloat16*)y, n / 8);
  return check_launch("gelu_fwd");
}

extern "C" int lk_gelu_bwd(const void* x, const void* dy, void* dx, int64_t n, cudaStream_t s) {
  LK_REQUIRE(n % 8 == 0, "gelu: element count must be a multiple of 8");
  if (n == 0) return 0;
  const int grid = (int)std::min<int64_t>((n / 8 + 255) / 256, 8 * num_sms());
  gelu_bwd_kernel<<<grid, 256, 0, s>>>((const __nv_bfloat16*)x, (const __nv_bfloat16*)dy, (__nv_bfloat16*)dx,
                                       n / 8);
  return check_launch("gelu_bwd");
}

extern "C" int lk_layernorm_fwd(const void* x, const void* gamma, const void* beta, void* y, float* mean,
                                float* rstd, int M, int D, float eps, cudaStream_t s) {
  if (M == 0) return 0;
  const int grid = (int)std::min<int64_t>((M + 7) / 8, 4 * num_sms());
  switch (D / 256 * (D % 256 == 0)) {
#define LK_LN_CASE(V)                                                                                        \
  case V:                                                                                                  \
    layernorm_fwd_kernel<V><<<grid, 256, 0, s>>>((const __nv_bfloat16*)x, (const __nv_bfloat16*)gamma,    \
                                                 (const __nv_bfloat16*)beta, (__nv_bfloat16*)y, mean, rstd, \
                                                 M, D, eps);                                                \
    break;
    LK_LN_CASE(1) LK_LN_CASE(2) LK_LN_CASE(4) LK_LN_CASE(8) LK_LN_CASE(16)
#undef LK_LN_CASE
    default:
      return fail("layernorm: D must be 256 x {1, 2, 4, 8, 16}");
  }
  return check_launch("layernorm_fwd");
}

extern "C" int lk_layernorm_bwd(const void* dy, const void* x, const void* gamma, const float* mean,
                                const float* rstd, void* dx, float* dgamma, float* dbeta, int M, int D,
                                cudaStream_t s) {
  if (M == 0) return 0;
  const int grid = (int)std::min<int64_t>((M + 7) / 8, 2 * num_sms());
  const size_t smem = 2 * (size_t)D * sizeof(float);
  switch (D / 256 * (D % 256 == 0)) {
#define LK_LN_CASE(V)                                                                                      \
  case V:                                                                                                \
    if (smem > 48 * 1024)                                                                                \
      cudaFuncSetAttribute(layernorm_bwd_kernel<V>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
    layernorm_bwd_kernel<V><<<grid, 256, smem, s>>>((const __nv_bfloat16*)dy, (const __nv_bfloat16*)x,    \
                                                    (const __nv_bfloat16*)gamma, mean, rstd,               \
                                                    (__nv_bfloat16*)dx, dgamma, dbeta, M, D);              \
    break;
    LK_LN_CASE(1) LK_LN_CASE(2) LK_LN_CASE(4) LK_LN_CASE(8) LK_LN_CASE(16)
#undef LK_LN_CASE
    default:
      return fail("layernorm: D must be 256 x {1, 2, 4, 8, 16}");
  }
  return check_launch("layernorm_bwd");
}
