// K14: weight quantisation and dequantising matrix products.
//
// Formats (rows = output features N, columns = input features K):
//   int8   symmetric per row:        w = q * s[n],            q in [-127, 127]
//   fp8    e4m3 per row:              w = fp8(q) * s[n],       |q| <= 448
//   int4   asymmetric per group of G: w = (q - z[n,g]) * s[n,g], q in [0, 15],
//          two values per byte (low nibble = even column)
//
// Kernels: row/group quantisers (round-to-nearest-even, saturating), a
// dequantising GEMV for decode-sized batches (M <= 16 rows of activations;
// reads every weight once, memory-bound by design) and a dequantise-to-bf16
// kernel that feeds the tcgen05 GEMM for prefill-sized batches.
//
// Replaces the reference's DynamicQuantizer / INT4Quantizer (which does not
// compile: undefined int4_t) / fp8 structs (truncating) and
// QuantizedInferenceKernels::matmul_int4_int8 (include/nn/quantization_production.hpp:
// 14-221, include/api/serving_production.hpp:211-226).
#include "common.cuh"
#include "host_util.h"
#include "lk_api.h"

namespace lk {

// One warp per row: amax -> scale -> codes.
template <int FMT>  // 0 int8, 1 fp8
__global__ void quant_rowwise_kernel(const __nv_bfloat16* __restrict__ w, int N, int K, void* __restrict__ q,
                                     float* __restrict__ scale) {
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= N) return;
  const __nv_bfloat16* src = w + (int64_t)row * K;
  float amax = 0.f;
  for (int k = lane; k < K; k += 32) amax = fmaxf(amax, fabsf(__bfloat162float(src[k])));
  amax = warp_max(amax);
  const float qmax = FMT == 0 ? 127.f : 448.f;
  const float s = amax > 0.f ? amax / qmax : 1.f;
  const float inv = 1.f / s;
  for (int k = lane; k < K; k += 32) {
    const float x = __bfloat162float(src[k]) * inv;
    if (FMT == 0) {
      reinterpret_cast<int8_t*>(q)[(int64_t)row * K + k] = (int8_t)fminf(fmaxf(rintf(x), -127.f), 127.f);
    } else {
      reinterpret_cast<__nv_fp8_e4m3*>(q)[(int64_t)row * K + k] = __nv_fp8_e4m3(x);
    }
  }
  if (lane == 0) scale[row] = s;
}

// One thread per (row, group): min/max -> scale, zero -> packed codes.
__global__ void quant_int4_kernel(const __nv_bfloat16* __restrict__ w, int N, int K, int G,
                                  uint8_t* __restrict__ q, float* __restrict__ scale, float* __restrict__ zero) {
  const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int ng = K / G;
  if (idx >= (int64_t)N * ng) return;
  const int row = (int)(idx / ng), g = (int)(idx % ng);
  const __nv_bfloat16* src = w + (int64_t)row * K + g * G;
  float lo = INFINITY, hi = -INFINITY;
  for (int k = 0; k < G; ++k) {
    const float x = __bfloat162float(src[k]);
    lo = fminf(lo, x);
    hi = fmaxf(hi, x);
  }
  lo = fminf(lo, 0.f);
  hi = fmaxf(hi, 0.f);
  const float s = hi > lo ? (hi - lo) / 15.f : 1.f;
  const float z = rintf(-lo / s);
  scale[idx] = s;
  zero[idx] = z;
  uint8_t* dst = q + (int64_t)row * (K / 2) + g * (G / 2);
  for (int k = 0; k < G; k += 2) {
    const float a = fminf(fmaxf(rintf(__bfloat162float(src[k]) / s + z), 0.f), 15.f);
    const float b = fminf(fmaxf(rintf(__bfloat162float(src[k + 1]) / s + z), 0.f), 15.f);
    dst[k / 2] = (uint8_t)((int)a | ((int)b << 4));
  }
}

// Decode 8 consecutive weights of row n starting at column k (k % 8 == 0).
template <int FMT>
__device__ __forceinline__ void load_w8(const void* q, const float* scale, const float* zero, int K, int G,
                                        int n, int k, float (&w)[8]) {
  if constexpr (FMT == 0) {
    const uint2 v = *reinterpret_cast<const uint2*>(reinterpret_cast<const int8_t*>(q) + (int64_t)n * K + k);
    const int8_t* b = reinterpret_cast<const int8_t*>(&v);
    const float s = scale[n];
#pragma unroll
    for (int i = 0; i < 8; ++i) w[i] = (float)b[i] * s;
  } else if constexpr (FMT == 1) {
    const uint2 v = *reinterpret_cast<const uint2*>(reinterpret_cast<const uint8_t*>(q) + (int64_t)n * K + k);
    const __nv_fp8_e4m3* b = reinterpret_cast<const __nv_fp8_e4m3*>(&v);
    const float s = scale[n];
#pragma unroll
    for (int i = 0; i < 8; ++i) w[i] = float(b[i]) * s;
  } else {
    const uint32_t v = *reinterpret_cast<const uint32_t*>(reinterpret_cast<const uint8_t*>(q) + (int64_t)n * (K / 2) + k / 2);
    const int64_t gi = (int64_t)n * (K / G) + k / G;
    const float s = scale[gi], z = zero[gi];
#pragma unroll
    for (int i = 0; i < 8; ++i) w[i] = ((float)((v >> (4 * i)) & 15u) - z) * s;
  }
}

// y[m, n] = sum_k x[m, k] w[n, k] for m < M (<= MM).  One warp per output n.
template <int FMT, int MM>
__global__ void __launch_bounds__(256) dequant_gemv_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, int M,
                                                           const void* __restrict__ q, const float* __restrict__ scale,
                                                           const float* __restrict__ zero, int N, int K, int G,
                                                           __nv_bfloat16* __restrict__ y, int64_t ldy) {
  const int n = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (n >= N) return;
  float acc[MM];
#pragma unroll
  for (int m = 0; m < MM; ++m) acc[m] = 0.f;
  for (int k = lane * 8; k < K; k += 256) {
    float w[8];
    load_w8<FMT>(q, scale, zero, K, G, n, k, w);
#pragma unroll
    for (int m = 0; m < MM; ++m) {
      if (m >= M) break;
      const uint4 xv = __ldg(reinterpret_cast<const uint4*>(x + (int64_t)m * ldx + k));
      const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = unpack_bf16x2(xw[e]);
        acc[m] += f.x * w[2 * e] + f.y * w[2 * e + 1];
      }
    }
  }
#pragma unroll
  for (int m = 0; m < MM; ++m) {
    if (m >= M) break;
    const float s = warp_sum(acc[m]);
    if (lane == 0) y[(int64_t)m * ldy + n] = __float2bfloat16(s);
  }
}

template <int FMT>
__global__ void dequant_kernel(const void* __restrict__ q, const float* __restrict__ scale,
                               const float* __restrict__ zero, int N, int K, int G, __nv_bfloat16* __restrict__ w) {
  const int64_t total = (int64_t)N * K / 8;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int n = (int)(idx / (K / 8));
    const int k = (int)(idx % (K / 8)) * 8;
    float v[8];
    load_w8<FMT>(q, scale, zero, K, G, n, k, v);
    *reinterpret_cast<uint4*>(w + (int64_t)n * K + k) =
        make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
  }
}

}  // namespace lk

using namespace lk;

extern "C" int lk_quantize(int fmt, const void* w, int N, int K, int group, void* q, float* scale, float* zero,
                           cudaStream_t s) {
  LK_REQUIRE(K % 8 == 0, "quantize: K must be a multiple of 8");
  if (fmt == LK_Q_INT8) {
    quant_rowwise_kernel<0><<<cdiv((int64_t)N * 32, 256), 256, 0, s>>>((const __nv_bfloat16*)w, N, K, q, scale);
  } else if (fmt == LK_Q_FP8) {
    quant_rowwise_kernel<1><<<cdiv((int64_t)N * 32, 256), 256, 0, s>>>((const __nv_bfloat16*)w, N, K, q, scale);
  } else if (fmt == LK_Q_INT4) {
    LK_REQUIRE(group % 8 == 0 && K % group == 0 && zero, "quantize: int4 needs K % group == 0, group % 8 == 0");
    quant_int4_kernel<<<cdiv((int64_t)N * (K / group), 256), 256, 0, s>>>((const __nv_bfloat16*)w, N, K, group,
                                                                          (uint8_t*)q, scale, zero);
  } else {
    return fail("quantize: unknown format");
  }
  return check_launch("quantize");
}

extern "C" int lk_dequant_gemv(int fmt, const void* x, int64_t ldx, int M, const void* q, const float* scale,
                               const float* zero, int N, int K, int group, void* y, int64_t ldy, cudaStream_t s) {
  LK_REQUIRE(M >= 1 && M <= 16, "dequant_gemv: 1 <= M <= 16");
  LK_REQUIRE(K % 256 == 0 || K % 8 == 0, "dequant_gemv: K % 8");
  LK_REQUIRE(ldx % 8 == 0, "dequant_gemv: x pitch % 8");
  const int grid = cdiv((int64_t)N * 32, 256);
#define LK_GV(F, MM)                                                                                     \
  dequant_gemv_kernel<F, MM><<<grid, 256, 0, s>>>((const __nv_bfloat16*)x, ldx, M, q, scale, zero, N, K, \
                                                  group, (__nv_bfloat16*)y, ldy)
#define LK_GV_M(F)           \
  if (M <= 1) LK_GV(F, 1);   \
  else if (M <= 4) LK_GV(F, 4); \
  else if (M <= 8) LK_GV(F, 8); \
  else LK_GV(F, 16);
  if (fmt == LK_Q_INT8) {
    LK_GV_M(0)
  } else if (fmt == LK_Q_FP8) {
    LK_GV_M(1)
  } else if (fmt == LK_Q_INT4) {
    LK_GV_M(2)
  } else {
    return fail("dequant_gemv: unknown format");
  }
#undef LK_GV_M
#undef LK_GV
  return check_launch("dequant_gemv");
}

extern "C" int lk_dequantize(int fmt, const void* q, const float* scale, const float* zero, int N, int K, int group,
                             void* w, cudaStream_t s) {
  const int64_t work = (int64_t)N * K / 8;
  int grid = (int)std::min<int64_t>((work + 255) / 256, (int64_t)num_sms() * 16);
  if (fmt == LK_Q_INT8)
    dequant_kernel<0><<<grid, 256, 0, s>>>(q, scale, zero, N, K, group, (__nv_bfloat16*)w);
  else if (fmt == LK_Q_FP8)
    dequant_kernel<1><<<grid, 256, 0, s>>>(q, scale, zero, N, K, group, (__nv_bfloat16*)w);
  else if (fmt == LK_Q_INT4)
    dequant_kernel<2><<<grid, 256, 0, s>>>(q, scale, zero, N, K, group, (__nv_bfloat16*)w);
  else
    return fail("dequantize: unknown format");
  return check_launch("dequantize");
}
